"""tcgen05 GEMM entry point (``siglip2_gemm``) against torch fp32 math on the
same bf16/f16 inputs, for every fused epilogue and the ragged shapes of the
tower (N=4304, K=4304, M not a multiple of 128)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from siglip2_b200 import _lib as L  # noqa: E402
from siglip2_b200 import ops  # noqa: E402


@pytest.fixture(params=[1, 2], ids=["1sm", "2sm"], autouse=True)
def gemm_variant(request):
    """Every GEMM test runs on both kernels: one SM per 128-row tile and
    CTA pairs (tcgen05 cta_group::2) per 256-row tile."""
    lib = L.load()
    old = lib.siglip2_get_gemm_variant()
    L.check(lib.siglip2_set_gemm_variant(request.param))
    yield request.param
    L.check(lib.siglip2_set_gemm_variant(old))


def _gelu(x):
    return F.gelu(x, approximate="tanh")


def _close(out, ref, tol=1.5e-2):
    out = out.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    cos = F.cosine_similarity(out.flatten(), ref.flatten(), dim=0).item()
    assert err / scale < tol and cos > 0.9999, (err, scale, cos)


SHAPES = [(300, 1152, 1152), (1000, 4304, 1152), (777, 1152, 4304), (128, 256, 64), (4097, 3840, 1152),
          (64, 768, 768), (1, 2304, 768)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("epi", [L.EPI_BIAS, L.EPI_BIAS_RES, L.EPI_BIAS_GELU])
def test_gemm_bias_epilogues(dtype, M, N, K, epi):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).to(dtype)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    res = torch.randn(M, N, device="cuda", generator=g).to(dtype) if epi == L.EPI_BIAS_RES else None
    out = ops.gemm(a, w, epi, bias=bias, res=res)
    ref = a.float() @ w.float().T + bias
    if epi == L.EPI_BIAS_RES:
        ref = ref + res.float()
    if epi == L.EPI_BIAS_GELU:
        ref = _gelu(ref)
    torch.cuda.synchronize()
    _close(out, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(300, 3840, 1152), (1000, 4304, 1152), (513, 2304, 768), (200, 1536, 1536)])
@pytest.mark.parametrize("gelu", [False, True])
def test_gemm_layernorm_folded(dtype, M, N, K, gelu):
    g = torch.Generator(device="cuda").manual_seed(N + K)
    # residual-stream-like rows: non-zero mean, varied scale
    x = (torch.randn(M, K, device="cuda", generator=g) * (1 + 3 * torch.rand(M, 1, device="cuda", generator=g))
         + torch.randn(M, 1, device="cuda", generator=g) * 2).to(dtype)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.03
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    gamma = 1 + 0.2 * torch.randn(K, device="cuda", generator=g)
    beta = 0.1 * torch.randn(K, device="cuda", generator=g)
    wg, c1, c2 = ops.fold_layernorm(w, b, gamma, beta, dtype)
    out = ops.gemm(x, wg, L.EPI_LN_GELU if gelu else L.EPI_LN, c1=c1, c2=c2, eps=1e-6)
    ref = F.layer_norm(x.float(), (K,), gamma, beta, 1e-6) @ w.T + b
    if gelu:
        ref = _gelu(ref)
    torch.cuda.synchronize()
    _close(out, ref, tol=2e-2)


def test_gemm_inplace_residual():
    a = torch.randn(333, 1152, device="cuda").bfloat16()
    w = (torch.randn(1152, 1152, device="cuda") * 0.03).bfloat16()
    bias = torch.randn(1152, device="cuda") * 0.1
    x = torch.randn(333, 1152, device="cuda").bfloat16()
    ref = a.float() @ w.float().T + bias + x.float()
    ops.gemm(a, w, L.EPI_BIAS_RES, bias=bias, res=x, out=x)
    torch.cuda.synchronize()
    _close(x, ref)


def test_gemm_rejects_bad_args():
    a = torch.randn(16, 100, device="cuda").bfloat16()  # K=100 is not a multiple of 8
    w = torch.randn(64, 100, device="cuda").bfloat16()
    with pytest.raises(L.Siglip2Error):
        ops.gemm(a, w, L.EPI_BIAS, bias=torch.zeros(64, device="cuda"))
    L.check(L.load().siglip2_check_device(1))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(777, 1152, 4304), (300, 1152, 1152), (4097, 768, 3072)])
def test_gemm_residual_accumulates_row_sums(dtype, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).to(dtype)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    res = torch.randn(M, N, device="cuda", generator=g).to(dtype)
    acc = torch.full((M, ops.rowsum_slots(dtype, N), 2), float("nan"), device="cuda")  # every slot is written
    out = ops.gemm_rowsums(a, w, L.EPI_BIAS_RES_ROWSUMS, bias=bias, res=res, rs_acc=acc)
    torch.cuda.synchronize()
    _close(out, a.float() @ w.float().T + bias + res.float())
    o = out.float()  # statistics of exactly the stored (rounded) values, per column block
    ref = ops.rowsums_reference(out)
    assert torch.allclose(acc, ref, rtol=1e-4, atol=1e-3)
    mean, var = ops.slot_stats_merge(acc, N)
    assert torch.allclose(mean, o.mean(1), rtol=1e-4, atol=1e-5)
    assert torch.allclose(var, o.var(1, unbiased=False), rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(300, 3840, 1152), (1000, 4304, 1152), (513, 2304, 768)])
@pytest.mark.parametrize("gelu", [False, True])
def test_gemm_layernorm_from_row_sums(dtype, M, N, K, gelu):
    g = torch.Generator(device="cuda").manual_seed(N + K + 1)
    x = (torch.randn(M, K, device="cuda", generator=g) * (1 + 3 * torch.rand(M, 1, device="cuda", generator=g))
         + torch.randn(M, 1, device="cuda", generator=g) * 2).to(dtype)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.03
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    gamma = 1 + 0.2 * torch.randn(K, device="cuda", generator=g)
    beta = 0.1 * torch.randn(K, device="cuda", generator=g)
    wg, c1, c2 = ops.fold_layernorm(w, b, gamma, beta, dtype)
    xf = x.float()
    rs = ops.rowsums_reference(x)
    out = ops.gemm_rowsums(x, wg, L.EPI_LN_ROWSUMS_GELU if gelu else L.EPI_LN_ROWSUMS, c1=c1, c2=c2, eps=1e-6,
                           rs_in=rs)
    ref = F.layer_norm(xf, (K,), gamma, beta, 1e-6) @ w.T + b
    if gelu:
        ref = _gelu(ref)
    torch.cuda.synchronize()
    _close(out, ref, tol=2e-2)


@pytest.mark.parametrize("N,K", [(1152, 1152), (4304, 1152), (1152, 4304), (3840, 1152)])
@pytest.mark.parametrize("epi", ["bias", "bias_gelu", "lnrs", "lnrs_gelu", "bias_res_rs_inplace"])
def test_gemm_many_tiles_per_cta(N, K, epi):
    """M large enough that every CTA (pair) walks several tiles, so the
    accumulator, staging-buffer and barrier phases wrap; checked element by
    element against fp32 math on the same bf16 inputs."""
    M = 9001
    g = torch.Generator(device="cuda").manual_seed(N * 3 + K)
    x = (torch.randn(M, K, device="cuda", generator=g) * 2 + 0.5).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    xf, wf = x.float(), w.float()
    if epi in ("bias", "bias_gelu"):
        out = ops.gemm(x, w, L.EPI_BIAS if epi == "bias" else L.EPI_BIAS_GELU, bias=bias)
        ref = xf @ wf.T + bias
        if epi == "bias_gelu":
            ref = _gelu(ref)
    elif epi in ("lnrs", "lnrs_gelu"):
        rs = ops.rowsums_reference(x)
        c1 = torch.randn(N, device="cuda", generator=g) * 0.1
        c2 = torch.randn(N, device="cuda", generator=g) * 0.1
        out = ops.gemm_rowsums(x, w, L.EPI_LN_ROWSUMS_GELU if epi == "lnrs_gelu" else L.EPI_LN_ROWSUMS, c1=c1, c2=c2,
                               eps=1e-6, rs_in=rs)
        mu, var = ops.slot_stats_merge(rs, K)
        mu, rstd = mu[:, None], torch.rsqrt(var[:, None] + 1e-6)
        ref = rstd * (xf @ wf.T - mu * c1) + c2
        if epi == "lnrs_gelu":
            ref = _gelu(ref)
    else:  # out-projection / fc2 as the forward runs them: residual updated in place, row sums out
        res = torch.randn(M, N, device="cuda", generator=g).bfloat16()
        ref = xf @ wf.T + bias + res.float()
        acc = torch.full((M, ops.rowsum_slots(torch.bfloat16, N), 2), float("nan"), device="cuda")
        out = ops.gemm_rowsums(x, w, L.EPI_BIAS_RES_ROWSUMS, bias=bias, res=res, rs_acc=acc, out=res)
    torch.cuda.synchronize()
    o = out.float()
    bad = (o - ref).abs() > 1e-2 * ref.abs() + 2e-3 * ref.abs().max()
    assert not bad.any(), (bad.nonzero()[:8].tolist(), bad.sum().item())
    if epi == "bias_res_rs_inplace":
        assert torch.allclose(acc, ops.rowsums_reference(out), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("source", ["gemm", "rowsums"])
def test_layernorm_fold_large_row_mean(dtype, source):
    """Residual rows whose mean (50..200) is large against their spread
    (std 1), D = 1152: the slot statistics are shifted sums, so the variance
    does not cancel.  The statistics come from the GEMM that writes the rows
    (bias + residual epilogue) or from siglip2_rowsums; the LayerNorm-folded
    GEMMs are checked (a) with an identity weight, which exposes the
    statistics directly, and (b) with random weights and GELU, against
    F.layer_norm in fp32 on the same rounded rows."""
    M, D, N = 3000, 1152, 1536
    g = torch.Generator(device="cuda").manual_seed(4242)
    mean = 50 + 150 * torch.rand(M, 1, device="cuda", generator=g)
    res = (torch.randn(M, D, device="cuda", generator=g) + mean).to(dtype)
    if source == "gemm":
        a = torch.randn(M, 256, device="cuda", generator=g).to(dtype)
        w0 = (torch.randn(D, 256, device="cuda", generator=g) * 0.02).to(dtype)
        rs = torch.full((M, ops.rowsum_slots(dtype, D), 2), float("nan"), device="cuda")
        x = ops.gemm_rowsums(a, w0, L.EPI_BIAS_RES_ROWSUMS, bias=torch.zeros(D, device="cuda"), res=res, rs_acc=rs)
    else:
        x = res
        rs = ops.rowsums(x)
    xf = x.float()
    mu, var = ops.slot_stats_merge(rs, D)
    assert torch.allclose(mu, xf.mean(1), rtol=1e-6, atol=1e-4)
    assert torch.allclose(var, xf.var(1, unbiased=False), rtol=1e-4, atol=1e-5)
    # (a) identity weight: out = (x - mu) * rstd
    eye = torch.eye(D, device="cuda")
    wg, c1, c2 = ops.fold_layernorm(eye, None, torch.ones(D, device="cuda"), torch.zeros(D, device="cuda"), dtype)
    out = ops.gemm_rowsums(x, wg, L.EPI_LN_ROWSUMS, c1=c1, c2=c2, eps=1e-6, rs_in=rs).float()
    ref = F.layer_norm(xf, (D,), eps=1e-6)
    ulp = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -10
    err = (out - ref).abs() - (ulp * ref.abs() + 2e-3)
    assert err.max().item() <= 0, (out - ref).abs().max().item()
    # (b) random weights, affine LayerNorm, GELU epilogue
    w = torch.randn(N, D, device="cuda", generator=g) * 0.03
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    gamma = 1 + 0.2 * torch.randn(D, device="cuda", generator=g)
    beta = 0.1 * torch.randn(D, device="cuda", generator=g)
    wg, c1, c2 = ops.fold_layernorm(w, b, gamma, beta, dtype)
    for gelu in (False, True):
        out = ops.gemm_rowsums(x, wg, L.EPI_LN_ROWSUMS_GELU if gelu else L.EPI_LN_ROWSUMS, c1=c1, c2=c2, eps=1e-6,
                               rs_in=rs)
        ref = F.layer_norm(xf, (D,), gamma, beta, 1e-6) @ w.T + b
        if gelu:
            ref = _gelu(ref)
        torch.cuda.synchronize()
        _close(out, ref, tol=1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N_out,K_in", [(1001, 1152, 4304), (4097, 4304, 1152), (39178, 3456, 1152),
                                          (130, 768, 768), (7, 1152, 1152)])
def test_gemm_transposed_operands_dgrad_wgrad(dtype, M, N_out, K_in):
    """siglip2_gemm_t: dgrad dA = dY W (W read as the MN-major B operand) and
    wgrad dW = dY^T A (both read MN-major) against fp32 torch on the same
    inputs; token counts not multiples of the tile."""
    g = torch.Generator(device="cuda").manual_seed(M + N_out)
    dy = (torch.randn(M, N_out, device="cuda", generator=g) * 0.1).to(dtype)
    w = (torch.randn(N_out, K_in, device="cuda", generator=g) * 0.03).to(dtype)
    a = torch.randn(M, K_in, device="cuda", generator=g).to(dtype)
    da = ops.gemm_t(dy, w, False, True)
    dw = ops.gemm_t(dy, a, True, True)
    torch.cuda.synchronize()
    assert da.shape == (M, K_in) and dw.shape == (N_out, K_in)
    _close(da, dy.float() @ w.float())
    _close(dw, dy.float().T @ a.float())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(1000, 4304, 1152), (257, 3072, 768)])
def test_gemm_gelu_gradient_epilogue(dtype, M, N, K):
    """SIGLIP2_EPI_BIAS_GELU_GRAD: the pre-activation recomputed and the
    incoming gradient multiplied by GELU-tanh' in the epilogue."""
    g = torch.Generator(device="cuda").manual_seed(N + K)
    a = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).to(dtype)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    up = torch.randn(M, N, device="cuda", generator=g).to(dtype)
    out = ops.gemm(a, w, L.EPI_BIAS_GELU_GRAD, bias=bias, res=up)
    z = (a.float() @ w.float().T + bias).requires_grad_(True)
    _gelu(z).backward(up.float())
    torch.cuda.synchronize()
    _close(out, z.grad, tol=2e-2)


def test_gemm_transposed_rejects_bad_args():
    a = torch.zeros(64, 100, dtype=torch.bfloat16, device="cuda")  # pitch 100: not a multiple of 8
    w = torch.zeros(64, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(L.Siglip2Error):
        ops.gemm_t(a, w, True, True)
    with pytest.raises(L.Siglip2Error):  # tensor-core only
        ops.gemm_t(torch.zeros(64, 64, device="cuda"), torch.zeros(64, 128, device="cuda"), False, True)
    L.check(L.load().siglip2_check_device(1))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tokens,N_out,K_in", [(16384, 4304, 1152), (16384, 1152, 1152), (39178, 1152, 4304),
                                               (4097, 1152, 1152), (9000, 768, 768)])
def test_gemm_splitk_weight_gradient(dtype, tokens, N_out, K_in):
    """siglip2_gemm_t_ws: the weight gradient dW = dY^T A with K (= tokens)
    split over an fp32 workspace when the [N_out, K_in] output has few tiles,
    the slices summed in order (+ bias): against fp32 torch, against the
    unsplit siglip2_gemm_t, and bit-identical across two calls."""
    lib = L.load()
    nbytes = lib.siglip2_gemm_t_workspace_size(L.EPI_BIAS, 1, 1, N_out, K_in, tokens)
    assert nbytes > 0, "these shapes leave SMs idle without a split"
    g = torch.Generator(device="cuda").manual_seed(tokens + N_out)
    dy = (torch.randn(tokens, N_out, device="cuda", generator=g) * 0.1).to(dtype)
    a = torch.randn(tokens, K_in, device="cuda", generator=g).to(dtype)
    bias = torch.randn(K_in, device="cuda", generator=g)
    dw = ops.gemm_t_splitk(dy, a, True)
    dw2 = ops.gemm_t_splitk(dy, a, True)
    dwb = ops.gemm_t_splitk(dy, a, True, bias=bias)
    plain = ops.gemm_t(dy, a, True, True)
    torch.cuda.synchronize()
    ref = dy.float().T @ a.float()
    _close(dw, ref)
    _close(dwb, ref + bias)
    assert torch.equal(dw, dw2)
    # the same fp32 sums in another order, one rounding to 8 significant bits
    # (bf16): at most a couple of ulps of the largest magnitude apart
    assert (dw.float() - plain.float()).abs().max().item() <= 2 ** -6 * ref.abs().max().item()
