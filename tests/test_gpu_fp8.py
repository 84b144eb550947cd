"""8-bit (e4m3) GEMM operands: the per-row quantiser (``siglip2_quantize_e4m3``)
bit for bit against torch's float8_e4m3fn conversion of the same scaled
values, and the tcgen05 kind::f8f6f4 GEMM (``siglip2_gemm_e4m3``) against
torch fp32 math on the dequantised operands, for the bias epilogues and the
tower's projection shapes (N=4304, K=4304, M not a multiple of 256)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from siglip2_b200 import _lib as L  # noqa: E402
from siglip2_b200 import ops  # noqa: E402


def _torch_quantize(x):
    """The quantiser's definition in torch: scale = amax / 448, codes =
    e4m3(x * (448 / amax)) rounded to nearest even (zero row: zeros)."""
    xf = x.float()
    amax = xf.abs().amax(1)
    c448 = torch.full_like(amax, 448.0)
    # tensor / tensor: correctly rounded divisions (a tensor / python-float
    # division may multiply by the rounded reciprocal instead)
    inv = torch.where(amax > 0, c448 / amax, torch.zeros_like(amax))
    return (xf * inv[:, None]).to(torch.float8_e4m3fn), amax / c448


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(1, 8), (257, 1152), (1000, 4304), (64, 768)])
def test_quantize_e4m3_bitexact(dtype, rows, cols):
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = torch.randn(rows, cols, device="cuda", generator=g)
    # rows spanning magnitudes, an all-zero row, a row with one outlier
    x = x * torch.logspace(-3, 3, rows, device="cuda")[:, None]
    if rows > 2:
        x[1] = 0
        x[2, cols // 2] = 1e4
    x = x.to(dtype)
    q, s = ops.quantize_e4m3(x)
    rq, rs = _torch_quantize(x)
    torch.cuda.synchronize()
    assert torch.equal(s, rs)
    assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8))


def _dequant(q, s):
    return q.float() * s[:, None]


SHAPES = [(300, 1152, 1152), (1000, 4304, 1152), (777, 1152, 4304), (4097, 3456, 1152), (64, 768, 768),
          (1, 2304, 768), (39178, 1152, 1152)]


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("epi", [L.EPI_BIAS, L.EPI_BIAS_RES, L.EPI_BIAS_GELU])
def test_gemm_e4m3_epilogues(out_dtype, M, N, K, epi):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    res = torch.randn(M, N, device="cuda", generator=g).to(out_dtype) if epi == L.EPI_BIAS_RES else None
    qa, sa = ops.quantize_e4m3(a)
    qw, sw = ops.quantize_e4m3(w)
    out = ops.gemm_e4m3(qa, sa, qw, sw, epi, bias, res=res, out_dtype=out_dtype)
    ref = _dequant(qa, sa) @ _dequant(qw, sw).T + bias
    if epi == L.EPI_BIAS_RES:
        ref = ref + res.float()
    if epi == L.EPI_BIAS_GELU:
        ref = F.gelu(ref, approximate="tanh")
    torch.cuda.synchronize()
    o = out.float()
    scale = ref.abs().max().item() + 1e-6
    err = (o - ref).abs().max().item()
    cos = F.cosine_similarity(o.flatten(), ref.flatten(), dim=0).item()
    # same products, fp32 accumulation in another order, one rounding to the output type
    assert err / scale < 1e-2 and cos > 0.99999, (err, scale, cos)
    # and against the bf16 operands before quantisation: e4m3 keeps 3 mantissa bits
    full = a.float() @ w.float().T + bias
    if epi == L.EPI_BIAS_RES:
        full = full + res.float()
    if epi == L.EPI_BIAS_GELU:
        full = F.gelu(full, approximate="tanh")
    assert F.cosine_similarity(o.flatten(), full.flatten(), dim=0).item() > 0.998


def test_gemm_e4m3_rejects_bad_arguments():
    lib = L.load()
    a = torch.zeros(64, 40, dtype=torch.float8_e4m3fn, device="cuda")
    s = torch.ones(64, device="cuda")
    out = torch.empty(64, 64, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # K = 40 is not a multiple of 16
    rc = lib.siglip2_gemm_e4m3(L.DTYPE_BF16, L.EPI_BIAS, a.data_ptr(), 40, s.data_ptr(), a.data_ptr(), 40,
                               s.data_ptr(), out.data_ptr(), 64, 64, 64, 40, s.data_ptr(), None, 0, stream)
    assert rc != 0 and b"multiples of 16" in lib.siglip2_last_error()
    # LayerNorm epilogues are not built for 8-bit operands
    b = torch.zeros(64, 64, dtype=torch.float8_e4m3fn, device="cuda")
    rc = lib.siglip2_gemm_e4m3(L.DTYPE_BF16, L.EPI_LN, b.data_ptr(), 64, s.data_ptr(), b.data_ptr(), 64,
                               s.data_ptr(), out.data_ptr(), 64, 64, 64, 64, s.data_ptr(), None, 0, stream)
    assert rc != 0
