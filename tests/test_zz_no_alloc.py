"""The allocation-free head-pooling entry point (``siglip2_head_pool_noalloc``)
against the regular one (``siglip2_head_pool``, caller-provided scratch),
through the C ABI, on two calls in a row.

It exists for callers that cannot allocate device memory when they call in
(fixed-arena serving processes, C/FFI hosts without a caching allocator): its
score scratch is a fixed array inside the library, shared by every call.
Both entry points run the same kernel on the same inputs, so their results
must agree bit for bit.  A caller whose ``n_tokens`` understates
``cu_seqlens[B]`` must get an error status and no write outside the array.
This file sorts last so that a run stopping at the first failure has already
run every other test."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from siglip2_b200 import _lib as L  # noqa: E402

CAPACITY = 1 << 20  # floats in the library's fixed score array
ERR_SHAPE = -3


def _inputs(lens, D, H, dtype, seed, max_patches=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    N = sum(lens)
    rows = len(lens) * max_patches if max_patches else N
    x = torch.randn(rows, D, device="cuda", generator=g).to(dtype)
    u = torch.randn(H, D, device="cuda", generator=g) * 0.05
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    return x, u, cu, N


def _call(x, u, cu, n_tokens, H, D, dtype_code, with_scratch, max_patches=0, pooled=None):
    lib = L.load()
    B = cu.numel() - 1
    if pooled is None:
        pooled = torch.full((B, H, D), float("nan"), dtype=x.dtype, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if with_scratch:
        scores = torch.empty(n_tokens * H, dtype=torch.float32, device="cuda")
        rc = lib.siglip2_head_pool(dtype_code, x.data_ptr(), D, H, cu.data_ptr(), B, max_patches, u.data_ptr(),
                                   scores.data_ptr(), pooled.data_ptr(), stream)
    else:
        rc = lib.siglip2_head_pool_noalloc(dtype_code, x.data_ptr(), D, H, cu.data_ptr(), B, max_patches, n_tokens,
                                           u.data_ptr(), pooled.data_ptr(), stream)
    L.check(rc)
    return pooled


CASES = [(torch.bfloat16, L.DTYPE_BF16), (torch.float16, L.DTYPE_F16), (torch.float32, L.DTYPE_F32)]


@pytest.mark.parametrize("dtype,code", CASES, ids=["bf16", "f16", "f32"])
@pytest.mark.parametrize("padded", [False, True], ids=["packed", "padded"])
def test_noalloc_matches_regular_entry_point_twice(dtype, code, padded):
    D, H = 1152, 16
    L.check(L.load().siglip2_check_device(1))
    # two different calls in a row: the second reuses the shared fixed scratch
    for seed, lens in ((1, [300, 17, 1024, 1, 96]), (2, [640, 5, 222])):
        P = 1024 if padded else 0
        x, u, cu, N = _inputs(lens, D, H, dtype, seed, P)
        ref = _call(x, u, cu, N, H, D, code, True, P)
        got = _call(x, u, cu, N, H, D, code, False, P)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (got.float() - ref.float()).abs().max().item()
        assert not torch.isnan(got.float()).any()
    L.check(L.load().siglip2_check_device(1))


def test_noalloc_rejects_oversize():
    lib = L.load()
    D, H = 1152, 16
    x, u, cu, N = _inputs([64], D, H, torch.bfloat16, 3)
    pooled = torch.empty((1, H, D), dtype=torch.bfloat16, device="cuda")
    too_many = CAPACITY // H + 1
    rc = lib.siglip2_head_pool_noalloc(L.DTYPE_BF16, x.data_ptr(), D, H, cu.data_ptr(), 1, 0, too_many, u.data_ptr(),
                                       pooled.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == ERR_SHAPE
    assert b"fixed scratch" in lib.siglip2_last_error()


@pytest.mark.parametrize("lens,n_tokens", [([300, 200, 64], 400), ([65000, 1000], 65000)],
                         ids=["below_cu_B", "past_capacity"])
def test_noalloc_understated_n_tokens_is_reported(lens, n_tokens):
    """``n_tokens`` below ``cu_seqlens[B]``: the images whose score rows reach
    past it are skipped on the device and ``siglip2_check_device`` reports
    SIGLIP2_ERR_SHAPE; the images inside it are still pooled exactly.  In the
    second case ``cu_seqlens[B] * heads`` exceeds the fixed array, so without
    the device-side bound the kernel would write past it."""
    lib = L.load()
    D, H = 1152, 16
    assert n_tokens * H <= CAPACITY
    L.check(lib.siglip2_check_device(1))
    x, u, cu, N = _inputs(lens, D, H, torch.bfloat16, 5)
    ref = _call(x, u, cu, N, H, D, L.DTYPE_BF16, True)
    got = _call(x, u, cu, n_tokens, H, D, L.DTYPE_BF16, False)
    rc = lib.siglip2_check_device(1)
    assert rc == ERR_SHAPE, rc
    assert b"outside the buffer" in lib.siglip2_last_error()
    starts = [0] + torch.tensor(lens).cumsum(0).tolist()
    for b in range(len(lens)):
        if starts[b + 1] <= n_tokens:
            assert torch.equal(got[b], ref[b])
        else:
            assert torch.isnan(got[b].float()).all()  # skipped: left as it was
    L.check(lib.siglip2_check_device(1))  # the flag cleared; the context is usable
    again = _call(x[:n_tokens], u, cu[:2].clone(), lens[0], H, D, L.DTYPE_BF16, False)
    torch.cuda.synchronize()
    assert torch.equal(again[0], ref[0])
    L.check(lib.siglip2_check_device(1))
