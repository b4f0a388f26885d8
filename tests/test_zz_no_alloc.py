"""The allocation-free adanorm backward entry point (C symbol ``tgo_adanorm_bwd_noalloc``, declared in
``csrc/noalloc.h``), called through ctypes the way a caller that may not allocate device memory while it runs (a
plugin inside a host framework that owns all device memory, or code that cannot take cudaMalloc's implicit
synchronisation) would call it, and compared with the regular, allocating entry point.

Collected last on purpose (file name), so that a run stopping at the first failure has run everything else.
"""
import ctypes

import pytest
import torch

c_p, c_ll, c_i = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int

# status codes of noalloc.h
OK, BAD_ARGS, TOO_LARGE = 0, 1, 2


def _entry():
    from trenowanie_generatora_obrazkow_b200.ops._ext import ext
    lib = ctypes.CDLL(ext().__file__)
    f = lib.tgo_adanorm_bwd_noalloc
    f.restype = c_i
    f.argtypes = [c_p, c_p, c_p, c_p, c_p, c_p, c_ll, c_p, c_p, c_ll, c_p, c_p, c_p, c_p, c_p, c_p, c_i, c_i, c_i,
                  c_p]
    lib.tgo_noalloc_scratch_floats.restype = c_ll
    lib.tgo_noalloc_error_string.restype = ctypes.c_char_p
    lib.tgo_noalloc_adanorm_rows.restype = c_i
    lib.tgo_noalloc_adanorm_rows.argtypes = [c_i, c_i, c_i]
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


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,D,rows", [(4, 256, 2048, 32),
                                        # partials at 32 rows (6.3 Mi floats) exceed the 4 Mi-float array: the
                                        # entry point widens the row chunk to 64, unlike the regular entry point
                                        (3, 4096, 4096, 64)])
def test_noalloc_matches_regular_entry_point_twice(B, T, D, rows):
    lib, f = _entry()
    assert lib.tgo_noalloc_adanorm_rows(B * T, D, T) == rows
    for call, seed in enumerate((11, 12)):  # two calls in a row share (and reuse) the scratch array
        x = _inputs(seed, B, T, D)
        rc, got = _noalloc(f, x, B, T, D)
        assert rc == OK, lib.tgo_noalloc_error_string(rc)
        want = _regular(x, T)
        torch.cuda.synchronize()
        for k in want:
            torch.testing.assert_close(got[k].float(), want[k].float(), rtol=1e-3, atol=1e-4,
                                       msg=lambda m: f"call {call}, {k}: {m}")
        del x, got, want


@pytest.mark.gpu
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
    assert rc == TOO_LARGE
    assert b"too large" in lib.tgo_noalloc_error_string(rc)
    assert lib.tgo_noalloc_adanorm_rows(B, D, 1) == -1


@pytest.mark.skipif(torch.cuda.is_available(), reason="host-side checks; run where no kernel can be reached")
def test_noalloc_rejects_bad_arguments_on_the_host():
    """Misaligned pointers / strides and too many samples are rejected before anything is launched. The buffers
    are host memory, and no CUDA device is present, so even a missed check could not touch a GPU."""
    pytest.importorskip("trenowanie_generatora_obrazkow_b200._C")
    lib, f = _entry()
    D, T, B = 256, 4, 2
    buf = (ctypes.c_uint8 * (1 << 16))()
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    a = lambda off: base + off  # 256-aligned host addresses inside the buffer
    args = dict(dh=a(0), dxe=None, xn=a(4096), rstd=a(8192), w=a(8448), scale=a(9472), mod_bs=6 * D, y=a(12288),
                gate=a(9472 + 2 * D), gate_bs=6 * D, dx=a(16384), dy=a(20480), dshift=a(24576), dscale=a(26624),
                dgate=a(28672), dw=a(30720), M=B * T, D=D, T=T, stream=None)

    def call(**kw):
        v = dict(args, **kw)
        return f(v["dh"], v["dxe"], v["xn"], v["rstd"], v["w"], v["scale"], v["mod_bs"], v["y"], v["gate"],
                 v["gate_bs"], v["dx"], v["dy"], v["dshift"], v["dscale"], v["dgate"], v["dw"], v["M"], v["D"],
                 v["T"], v["stream"])

    for bad in (dict(dh=a(2)), dict(xn=a(8)), dict(dx=a(4)), dict(dy=a(6)), dict(y=a(12288 + 2)),
                dict(scale=a(9472 + 2)), dict(gate=a(9472 + 8)), dict(mod_bs=6 * D + 4), dict(gate_bs=-8),
                dict(rstd=a(8192 + 2)), dict(w=a(8448 + 1)), dict(dw=a(30720 + 2)), dict(dh=None),
                dict(D=260), dict(M=B * T + 1)):
        assert call(**bad) == BAD_ARGS, bad
    assert b"aligned" in lib.tgo_noalloc_error_string(BAD_ARGS)
    assert call(M=65536, T=1, D=8) == TOO_LARGE  # 65536 samples: more than one grid row each
    assert lib.tgo_noalloc_adanorm_rows(65536, 8, 1) == -1
    assert lib.tgo_noalloc_adanorm_rows(4 * 256, 2048, 256) == 32
    assert lib.tgo_noalloc_adanorm_rows(3 * 4096, 4096, 4096) == 64
