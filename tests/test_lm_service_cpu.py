"""LM / VAE service ranks and the pipeline's distributed LM states over Gloo on CPU: states served remotely equal
local ones (null rows and pads zero), VAE encodes and text jobs round-trip, micro-batch states gather to stage 0 in
order, and the LM layer split across two stages equals the whole LM."""
import os
import socket
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trenowanie_generatora_obrazkow_b200.models.frozen_lm import LM_NULL, LM_PAD


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gpt():
    from trenowanie_generatora_obrazkow_b200.models.slayer import GPT, GPTConfig
    torch.manual_seed(5)
    g = GPT(GPTConfig(vocab=200, n_layer=3, n_embd=32, n_head=2, block=64)).float().eval()
    with torch.no_grad():
        for blk in g.blocks[1:]:
            blk.vr_lambda.fill_(0.5)
    return g


def _ids(seed, n=40, L=11):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 200, (n, L), generator=g)
    lens = torch.randint(1, L + 1, (n,), generator=g)
    ids[torch.arange(L)[None] >= lens[:, None]] = LM_PAD
    ids[3, 0] = LM_NULL
    ids[3, 1:] = LM_PAD
    return ids


def _vae(u8):
    return torch.nn.functional.avg_pool2d(u8.float(), 4)


def _local_states(gpt, ids):
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import SlayerFrozenLM
    return SlayerFrozenLM(None, skip_last=0, model=gpt, dtype=torch.float32, packed=True).states(ids)


def _worker(rank, world, port, d):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctl = dist.new_group(backend="gloo")
    text = dist.new_group(backend="gloo")
    from trenowanie_generatora_obrazkow_b200.models.frozen_lm import SlayerFrozenLM
    from trenowanie_generatora_obrazkow_b200.parallel.lm_service import (LMClient, LMService, TextLookahead,
                                                                         encode_remote, gather_to_stage,
                                                                         lm_split_forward)
    gpt = _gpt()
    lm = SlayerFrozenLM(None, skip_last=0, model=gpt, dtype=torch.float32, packed=True)
    if rank == 2:
        svc = LMService(lm.states, 32, "cpu", ctl, clients=[0, 1], vae=_vae, text_group=text,
                        text_fn=lambda job: dict(n_texts=torch.tensor([len(job["texts"])])), log=lambda *a: None)
        svc.serve()
    else:
        res = {}
        client = LMClient(2, 32, "cpu", ctl)
        if rank == 0:
            u8 = torch.randint(0, 255, (2, 3, 16, 16), dtype=torch.uint8)
            hv = client.request_vae(u8, (2, 3, 4, 4))
            res["vae"] = (LMClient.vae_collect(hv), _vae(u8))
        h = client.request(_ids(rank))
        res["lm"] = client.collect(h)
        if rank == 1:
            la = TextLookahead(lambda s: dict(ids=_ids(100 + s), texts=["a"] * (s + 1), step=s),
                               lambda job: encode_remote(job, 2, ctl, text), 0, 3, 1, 2)
            res["text"] = [la.take(s) for s in range(3)]
            la.close()
        client.stop()
        # pipeline of two stages (ranks 0, 1): micro-batch states, then the LM layer split
        s, pp = rank, 2
        mine = {k: torch.full((2, 3), float(k)) for k in range(4) if k % pp == s}
        res["gather"] = gather_to_stage(mine, 4, s, pp, 0, 0)
        chunks = [_ids(7, n=6), _ids(8, n=5)]
        lo, hi = (0, 2) if s == 0 else (2, 3)
        res["split"] = lm_split_forward(lambda x: gpt.run_slice(x, lo, hi).float(), chunks, s, pp, 0, "cpu", 32,
                                        carry_width=64)
        torch.save(res, os.path.join(d, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_lm_service_and_stage_helpers():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(3, _port(), d), nprocs=3, join=True)
        r0, r1 = (torch.load(os.path.join(d, f"r{r}.pt")) for r in (0, 1))
    gpt = _gpt()
    for rank, res in ((0, r0), (1, r1)):
        ids = _ids(rank)
        want = _local_states(gpt, ids)
        got = res["lm"].float()
        assert got.shape == want.shape
        assert torch.allclose(got, want.to(torch.bfloat16).float(), atol=1e-2)
        assert got[3].abs().max() == 0 and got[ids.eq(LM_PAD)].abs().max() == 0
    got, want = r0["vae"]
    assert torch.allclose(got, want)
    for s, job in enumerate(r1["text"]):
        assert int(job["n_texts"]) == s + 1 and job["step"] == s
        assert torch.allclose(job["lm"].float(), _local_states(gpt, _ids(100 + s)).to(torch.bfloat16).float(),
                              atol=1e-2)
    assert [int(t[0, 0]) for t in r0["gather"]] == [0, 1, 2, 3] and r1["gather"] is None
    assert r1["split"] is None
    for c, out in zip([_ids(7, n=6), _ids(8, n=5)], r0["split"]):
        real = c[:, 0].ne(LM_NULL)
        want = gpt.hidden(c.masked_fill(c.eq(LM_PAD) | c.eq(LM_NULL), 0), 3)
        tok = c.ne(LM_PAD) & real[:, None]  # real tokens (the split LM runs the trimmed, padded rows)
        assert torch.allclose(out[tok].float(), want[tok], rtol=3e-2, atol=6e-2)  # bf16 carry between stages
        assert out[~real].abs().max() == 0
