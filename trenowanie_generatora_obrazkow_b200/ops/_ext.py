"""Loader of the in-tree sm_100a extension and the device error word shared by its kernels.

CUDA tensors always go to the compiled kernels: if the extension is missing on a GPU machine the call raises
instead of falling back to PyTorch. CPU tensors use the fp32 PyTorch oracles next to each op (tests only).
"""
import torch

_C = None
_ERR = {}


def ext():
    """The compiled module ``trenowanie_generatora_obrazkow_b200._C`` (built by ``python setup.py build_ext
    --inplace`` or ``__graft_entry__.build()``)."""
    global _C
    if _C is None:
        try:
            from .. import _C as mod
        except ImportError as e:  # fail loudly: no silent eager fallback for CUDA tensors
            raise ImportError("trenowanie_generatora_obrazkow_b200._C is not built; run "
                              "`python setup.py build_ext --inplace` in the repository root") from e
        _C = mod
    return _C


def err_buf(device) -> torch.Tensor:
    """One int32 error word per device. Kernels with bounded waits write a non-zero code on time-out."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _ERR.get(idx)
    if buf is None:
        buf = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR[idx] = buf
    return buf


ERROR_NAMES = {1: "mbarrier wait timed out (TMA producer)", 2: "mbarrier wait timed out (MMA issuer)",
               3: "mbarrier wait timed out (epilogue)", 4: "peer flag wait timed out", 5: "bad kernel arguments"}


def check_errors(device=None, reset=True):
    """Raise if any kernel on `device` recorded an error code (synchronises with the device)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    buf = err_buf(device)
    code = int(buf[0].item())
    if code:
        if reset:
            buf.zero_()
        raise RuntimeError(f"sm_100a kernel error {code}: {ERROR_NAMES.get(code, 'unknown')}")
