"""The allocation-free adanorm backward entry point (C symbol ``tgo_adanorm_bwd_noalloc``), called through ctypes
like a caller that cannot allocate device memory would call it, against the regular entry point.

Collected last on purpose (file name), so that a run stopping at the first failure has run everything else.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

c_p, c_ll, c_i = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int


def _entry():
    from trenowanie_generatora_obrazkow_b200.ops._ext import ext
    lib = ctypes.CDLL(ext().__file__)
    f = lib.tgo_adanorm_bwd_noalloc
    f.restype = c_i
    f.argtypes = [c_p, c_p, c_p, c_p, c_p, c_p, c_ll, c_p, c_p, c_ll, c_p, c_p, c_p, c_p, c_p, c_p, c_i, c_i, c_i,
                  c_p]
    lib.tgo_noalloc_scratch_floats.restype = c_ll
    lib.tgo_noalloc_error_string.restype = ctypes.c_char_p
    return lib, f


def _ptr(t):
    return None if t is None else t.data_ptr()


def _inputs(seed, B, T, D):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    mod = (0.3 * r(B, 6, D)).bfloat16()
    return dict(dh=r(B * T, D).bfloat16(), dxe=r(B * T, D).bfloat16(), xn=r(B * T, D).bfloat16(),
                rstd=(1 + 0.1 * r(B * T)).abs(), w=1 + 0.1 * r(D), scale=mod[:, 1], gate=mod[:, 2],
                y=r(B * T, D).bfloat16())


def _regular(x, T):
    from trenowanie_generatora_obrazkow_b200.ops._ext import ext
    dw = torch.zeros_like(x["w"])
    dx, dy, dshift, dscale, dgate = ext().adanorm_bwd(x["dh"], x["dxe"], x["xn"], x["rstd"], x["w"], dw,
                                                      x["scale"], x["y"], x["gate"], T)
    return dict(dx=dx, dy=dy, dshift=dshift, dscale=dscale, dgate=dgate, dw=dw)


def _noalloc(f, x, B, T, D):
    out = dict(dx=torch.empty_like(x["dh"]), dy=torch.empty_like(x["dh"]),
               dshift=torch.empty(B, D, device="cuda"), dscale=torch.empty(B, D, device="cuda"),
               dgate=torch.empty(B, D, device="cuda"), dw=torch.zeros_like(x["w"]))
    rc = f(_ptr(x["dh"]), _ptr(x["dxe"]), _ptr(x["xn"]), _ptr(x["rstd"]), _ptr(x["w"]), _ptr(x["scale"]),
           x["scale"].stride(0), _ptr(x["y"]), _ptr(x["gate"]), x["gate"].stride(0), _ptr(out["dx"]),
           _ptr(out["dy"]), _ptr(out["dshift"]), _ptr(out["dscale"]), _ptr(out["dgate"]), _ptr(out["dw"]), B * T, D,
           T, torch.cuda.current_stream().cuda_stream)
    return rc, out


def test_noalloc_matches_regular_entry_point_twice():
    lib, f = _entry()
    B, T, D = 4, 256, 2048
    for call, seed in enumerate((11, 12)):  # two calls in a row share (and reuse) the scratch array
        x = _inputs(seed, B, T, D)
        rc, got = _noalloc(f, x, B, T, D)
        assert rc == 0, lib.tgo_noalloc_error_string(rc)
        want = _regular(x, T)
        torch.cuda.synchronize()
        for k in want:
            torch.testing.assert_close(got[k].float(), want[k].float(), rtol=1e-3, atol=1e-4,
                                       msg=lambda m: f"call {call}, {k}: {m}")


def test_noalloc_rejects_oversized_problem():
    lib, f = _entry()
    cap = lib.tgo_noalloc_scratch_floats()
    D = 4096
    B = cap // (4 * D) + 1  # one chunk per sample no longer fits
    x = torch.zeros(B, D, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(D, device="cuda")
    rstd = torch.ones(B, device="cuda")
    dw = torch.zeros(D, device="cuda")
    rc = f(_ptr(x), None, _ptr(x), _ptr(rstd), _ptr(w), None, 0, None, None, 0, _ptr(x), None, None, None, None,
           _ptr(dw), B, D, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert b"too large" in lib.tgo_noalloc_error_string(rc)
