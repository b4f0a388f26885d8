"""tcgen05 GEMM numerics vs an fp32 PyTorch reference (forward / dgrad / wgrad layouts, batched, odd shapes)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, a_mn, b_mn):
    A = a.float().mT if a_mn else a.float()
    B = b.float() if b_mn else b.float().mT
    return A @ B


def _rel(x, y):
    return ((x.float() - y.float()).norm() / y.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (200, 136, 72), (1000, 384, 520), (64, 8, 8),
                                   (4096, 2048, 2048), (8192, 6144, 2048), (8192, 2048, 520)])
def test_gemm_layouts(a_mn, b_mn, M, N, K):
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors
    torch.manual_seed(0)
    a = torch.randn(*((K, M) if a_mn else (M, K)), device="cuda").bfloat16()
    b = torch.randn(*((K, N) if b_mn else (N, K)), device="cuda").bfloat16()
    c = gemm(a, b, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    check_errors()
    assert _rel(c, _ref(a, b, a_mn, b_mn)) < 1e-2


def test_gemm_fp32_accumulate_and_beta():
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm
    torch.manual_seed(1)
    a = torch.randn(384, 256, device="cuda").bfloat16()
    b = torch.randn(384, 320, device="cuda").bfloat16()
    out = torch.randn(256, 320, device="cuda")
    ref = out + _ref(a, b, True, True)
    gemm(a, b, out=out, a_mn=True, b_mn=True, accumulate=True)
    assert _rel(out, ref) < 1e-3
    x = torch.randn(3, 128, 256, device="cuda").bfloat16()
    d = torch.randn(3, 128, 128, device="cuda").bfloat16()
    c = gemm(x, x, d=d, alpha=0.5, beta=-2.0)
    ref = 0.5 * (x.float() @ x.float().mT) - 2.0 * d.float()
    assert _rel(c, ref) < 1e-2


def test_gemm_batched_strided():
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm
    torch.manual_seed(2)
    base = torch.randn(4, 192, 512, device="cuda").bfloat16()
    a = base[:, :, :256]  # row stride 512
    b = torch.randn(4, 256, 192, device="cuda").bfloat16()
    c = gemm(a, b, b_mn=True)
    assert _rel(c, a.float() @ b.float()) < 1e-2


@pytest.mark.parametrize("M,N,K,batch", [(4000, 2312, 512, 1), (1024, 2048, 256, 3), (200, 136, 72, 1),
                                         (192, 264, 128, 2), (296, 88, 64, 1)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True)])
def test_gemm_tma_epilogue(M, N, K, batch, a_mn, b_mn):
    """GEMM whose epilogue writes C by TMA stores (clipped at ragged M / N edges, batched C) and fp32 TMA
    reduce-adds, against the per-row store epilogue (bitwise) and the fp32 oracle; the first two shapes run the
    2-CTA kernel, the others the 1-CTA kernel (128- and 256-column tiles)."""
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors, ext
    torch.manual_seed(3)
    lead = (batch,) if batch > 1 else ()
    a = torch.randn(*lead, *((K, M) if a_mn else (M, K)), device="cuda").bfloat16()
    b = torch.randn(*lead, *((K, N) if b_mn else (N, K)), device="cuda").bfloat16()
    c_tma = gemm(a, b, a_mn=a_mn, b_mn=b_mn)
    acc_tma = torch.randn(*lead, M, N, device="cuda")
    acc_rows = acc_tma.clone()
    gemm(a, b, out=acc_tma, a_mn=a_mn, b_mn=b_mn, alpha=0.5, accumulate=True)
    ext().set_gemm_tma_epilogue(False)
    try:
        c_rows = gemm(a, b, a_mn=a_mn, b_mn=b_mn)
        gemm(a, b, out=acc_rows, a_mn=a_mn, b_mn=b_mn, alpha=0.5, accumulate=True)
    finally:
        ext().set_gemm_tma_epilogue(True)
    torch.cuda.synchronize()
    check_errors()
    A = a.float().mT if a_mn else a.float()
    B = b.float() if b_mn else b.float().mT
    ref = A @ B
    assert torch.equal(c_tma, c_rows)
    assert _rel(c_tma, ref) < 1e-2
    assert _rel(acc_tma, acc_rows) < 1e-6


@pytest.mark.parametrize("b_mn", [False, True])
def test_gemm_grouped_device_schedule(b_mn):
    """Grouped GEMM with the tile schedule built on the device: uneven, empty and sub-tile groups, routing-weight row
    scale, against fp32 per-group products."""
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm_grouped
    torch.manual_seed(0)
    counts = [300, 0, 5, 128, 257, 0]
    K, N = 512, 384
    M = sum(counts)
    off = torch.tensor([0] + counts).cumsum(0).to(torch.int32)
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(len(counts), K, N, device="cuda").bfloat16() if b_mn else \
        torch.randn(len(counts), N, K, device="cuda").bfloat16()
    rs = torch.rand(M, device="cuda")
    out = gemm_grouped(a, b, off.cuda(), b_mn=b_mn, row_scale=rs)
    ref = gemm_grouped(a.cpu().float(), b.cpu().float(), off, b_mn=b_mn, row_scale=rs.cpu())
    err = ((out.float().cpu() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err


def test_fused_moe_inference_gpu():
    from trenowanie_generatora_obrazkow_b200.models.moe_infer import FusedMoE
    torch.manual_seed(2)
    E, H, I = 16, 256, 384
    router = torch.randn(E, H) * 0.1
    gu, dn = torch.randn(E, 2 * I, H) * H ** -0.5, torch.randn(E, H, I) * I ** -0.5
    x = torch.randn(500, H)
    ref = FusedMoE(router, gu, dn, 4)(x)  # CPU path (fp32 grouped products)
    got = FusedMoE(router, gu, dn, 4).to("cuda")(x.cuda().bfloat16())
    err = ((got.float().cpu() - ref).norm() / ref.norm()).item()
    assert err < 3e-2, err  # bf16 inputs and weights against the fp32 products


@pytest.mark.parametrize("batch,M,K,with_d", [(8, 2048, 2048, False), (8, 2048, 2048, True), (40, 1000, 512, True),
                                              (16, 1024, 2048, False), (2, 256, 128, True)])
def test_gemm_syrk_matches_full_product(batch, M, K, with_d):
    """Symmetric mode: lower-triangle tiles plus mirrored stores equal the full alpha A A^T + beta D (D symmetric);
    the last case is too small for the 2-CTA kernel and takes the full-product fallback."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors, err_buf, ext
    torch.manual_seed(2)
    a = (torch.randn(batch, M, K, device="cuda") / K ** 0.5).bfloat16()
    d = None
    if with_d:
        s = torch.randn(batch, M, M, device="cuda")
        d = (s + s.mT).bfloat16()
    c = torch.full((batch, M, M), float("nan"), device="cuda").bfloat16()  # every element must be written
    ext().gemm_syrk(a, c, d, 0.75, -0.5 if with_d else 0.0, err_buf(a.device))
    torch.cuda.synchronize()
    check_errors()
    ref = 0.75 * a.float() @ a.float().mT
    if with_d:
        ref = ref - 0.5 * d.float()
    assert not torch.isnan(c.float()).any()
    assert _rel(c, ref) < 1e-2
    assert torch.equal(c, c.mT)  # exactly symmetric: the upper half is the mirrored lower half


def test_newton_schulz_syrk_matches_reference():
    from trenowanie_generatora_obrazkow_b200.optim.newton_schulz import zeropower, zeropower_reference
    torch.manual_seed(3)
    g = torch.randn(12, 1024, 2560, device="cuda")
    x = zeropower(g)
    ref = zeropower_reference(g.float())
    assert _rel(x, ref) < 3e-2


def test_gemm_production_wgrad_accumulate():
    """The qkv weight gradient of the 1.24B model at 32 x 1024 tokens: dW (6144 x 2048) += dY^T X over K = 32768,
    fp32 accumulate into an existing gradient (many tiles per persistent CTA, TMA reduce-add epilogue)."""
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm
    torch.manual_seed(9)
    dy = (torch.randn(32768, 6144, device="cuda") * 0.05).bfloat16()
    x = (torch.randn(32768, 2048, device="cuda") * 0.05).bfloat16()
    out = torch.randn(6144, 2048, device="cuda")
    ref = out + _ref(dy, x, True, True)
    gemm(dy, x, out=out, a_mn=True, b_mn=True, accumulate=True)
    torch.cuda.synchronize()
    assert _rel(out, ref) < 1e-3


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 32768), (2048, 5504, 32768), (4096, 1024, 4096), (2000, 1000, 20000),
                                   (6144, 2048, 2048)])
def test_gemm_wgrad_split_k(M, N, K):
    """Weight-gradient layout, fp32 accumulate: with split-K (partial tiles reduce-added) and without, against fp32."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import check_errors, ext
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm
    torch.manual_seed(10)
    dy = (torch.randn(K, M, device="cuda") * 0.05).bfloat16()
    x = (torch.randn(K, N, device="cuda") * 0.05).bfloat16()
    base = torch.randn(M, N, device="cuda")
    ref = base + _ref(dy, x, True, True)
    outs = []
    for split in (True, False):
        ext().set_gemm_splitk(split)
        try:
            out = base.clone()
            gemm(dy, x, out=out, a_mn=True, b_mn=True, accumulate=True)
            torch.cuda.synchronize()
            check_errors()
        finally:
            ext().set_gemm_splitk(True)
        outs.append(out)
        assert _rel(out, ref) < 1e-3
    assert _rel(outs[0], outs[1]) < 1e-4  # different fp32 summation order over K


@pytest.mark.parametrize("M,N,K", [(300, 520, 256), (1024, 768, 2048), (64, 256, 4096)])
def test_gemm_i8_matches_integer_reference(M, N, K):
    """tcgen05 kind::i8 GEMM: the int32 products are exact, so C equals the scaled integer product up to the bf16
    rounding of the output (partial tiles at every edge in the first shape)."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import err_buf, ext
    torch.manual_seed(0)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
    sa = torch.rand(M, device="cuda") * 1e-3 + 1e-4
    sb = torch.rand(N, device="cuda") * 1e-3 + 1e-4
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    err = err_buf(a.device)
    ext().gemm_i8(a, b, c, sa, sb, err)
    ref = (a.double() @ b.double().T) * sa.double()[:, None] * sb.double()[None, :]
    assert err.sum().item() == 0
    torch.testing.assert_close(c.double(), ref, rtol=8e-3, atol=1e-6)


def test_quantize_rows_i8_and_w8a8_linear():
    from trenowanie_generatora_obrazkow_b200.models.quant import W8A8Linear
    from trenowanie_generatora_obrazkow_b200.ops._ext import ext
    torch.manual_seed(1)
    x = torch.randn(200, 1024, device="cuda").bfloat16()
    q, s = ext().quantize_rows_i8(x)
    want_s = x.float().abs().amax(1).clamp_min(1e-12) / 127
    torch.testing.assert_close(s, want_s, rtol=1e-6, atol=0)
    want_q = torch.round(x.float() / want_s[:, None]).clamp(-127, 127)
    assert (q.float() - want_q).abs().max().item() <= 1 and (q.float() != want_q).float().mean().item() < 1e-3
    lin = torch.nn.Linear(1024, 384).cuda()
    qlin = W8A8Linear(lin).cuda()
    y = qlin(x)
    ref = lin(x.float())
    assert y.dtype == torch.bfloat16 and ((y.float() - ref).norm() / ref.norm()).item() < 2e-2


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
def test_gemm_tail_split_is_exact(a_mn, b_mn):
    """The 2-CTA kernel's tail split (an A/B switch, off by default; the last wave's 34 tiles of 8192 x 2048 as 68
    half-width units) gives bitwise the products of whole tiles: each output element sums the same K-products in
    the same order."""
    from trenowanie_generatora_obrazkow_b200.ops._ext import ext
    from trenowanie_generatora_obrazkow_b200.ops.gemm import gemm
    torch.manual_seed(3)
    M, N, K = 8192, 2048, 1024
    a = torch.randn(*((K, M) if a_mn else (M, K)), device="cuda").bfloat16()
    b = torch.randn(*((K, N) if b_mn else (N, K)), device="cuda").bfloat16()
    try:
        ext().set_gemm_tail_split(False)
        whole = gemm(a, b, a_mn=a_mn, b_mn=b_mn)
        ext().set_gemm_tail_split(True)
        split = gemm(a, b, a_mn=a_mn, b_mn=b_mn)
    finally:
        ext().set_gemm_tail_split(False)
    assert torch.equal(whole, split)
    assert _rel(split, _ref(a, b, a_mn, b_mn)) < 1e-2
