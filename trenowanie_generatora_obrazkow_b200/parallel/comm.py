"""Peer-memory communication between the GPUs of one node (NVLink / NVSwitch).

``PeerBuffers`` allocates device buffers with cudaMalloc on every rank, exports CUDA IPC handles, exchanges them
through the process group (any backend: only the small handles travel) and maps every peer's buffers, so a kernel
on one GPU can load from and store to its peers' memory directly. ``PeerAllReduce`` is the data-parallel gradient
average on top of it (csrc/comm.cu: one fused cast + reduce-scatter + all-gather launch with bf16 on the wire, the
reference's DDP bf16-compress semantics). Flag waits inside the kernels are bounded; a peer that does not arrive
turns into an error code that ``check_errors`` raises on the host.
"""
import torch
import torch.distributed as dist

from ..ops._ext import err_buf, ext


class PeerBuffers:
    """Named buffers of the same size on every rank, each mapped on every rank: ``ptrs[name][peer]``."""

    def __init__(self, sizes, group=None, device=None):
        self.group = group
        single = not dist.is_initialized()  # one process: the buffers are only this GPU's
        self.rank = 0 if single else dist.get_rank(group)
        self.world = 1 if single else dist.get_world_size(group)
        self.group_ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.world))
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.local, self.ptrs, self._opened = {}, {}, []
        handles = {}
        for name, nbytes in sizes.items():
            ptr, h = ext().symm_alloc(int(nbytes), self.device.index)
            self.local[name] = ptr
            handles[name] = h
        gathered = [handles]
        if not single:
            gathered = [None] * self.world
            dist.all_gather_object(gathered, handles, group=group)
        for name in sizes:
            row = []
            for peer in range(self.world):
                if peer == self.rank:
                    row.append(self.local[name])
                else:
                    p = ext().ipc_open(gathered[peer][name], self.device.index)
                    self._opened.append(p)
                    row.append(p)
            self.ptrs[name] = row

    def close(self):
        torch.cuda.synchronize(self.device)
        multi = dist.is_initialized() and self.world > 1
        if multi:
            dist.barrier(group=self.group)  # nobody may still access a peer's memory
        for p in self._opened:
            ext().ipc_close(p, self.device.index)
        if multi:
            dist.barrier(group=self.group)
        for p in self.local.values():
            ext().symm_free(p, self.device.index)
        self._opened, self.local, self.ptrs = [], {}, {}


class PeerAllReduce:
    """In-place average of fp32 buffers of up to ``max_elems`` elements over the group (bf16 transport)."""

    def __init__(self, max_elems, group=None, device=None, blocks=32, timeout_s=30.0):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.blocks = blocks
        self.timeout_ns = int(timeout_s * 1e9)
        self.slice_max = self._slice(max_elems)
        nbytes = self.world * self.slice_max * 2
        self.buf = PeerBuffers({"staging": nbytes, "result": nbytes, "flags": (1 + self.world) * blocks * 4},
                               group, device)
        self.epoch = 0
        self.max_elems = max_elems

    def _slice(self, n):
        return (-(-n // self.world) + 7) // 8 * 8

    def __call__(self, buf):
        assert buf.dtype == torch.float32 and buf.is_contiguous() and buf.numel() <= self.max_elems
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        p = self.buf.ptrs
        ext().allreduce_bf16(buf, p["staging"], p["result"], p["flags"], self.rank, self.world,
                             self._slice(buf.numel()), self.epoch, 1.0 / self.world, self.blocks, self.timeout_ns,
                             err_buf(buf.device))
        return buf

    def close(self):
        self.buf.close()
