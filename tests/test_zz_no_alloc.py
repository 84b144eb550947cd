"""The allocation-free head-pooling entry point (``siglip2_head_pool_noalloc``)
against the regular one (``siglip2_head_pool``, caller-provided scratch),
through the C ABI, on two calls in a row.

It exists for callers that cannot allocate device memory when they call in
(fixed-arena serving processes, C/FFI hosts without a caching allocator): its
score scratch is a fixed array inside the library, shared by every call.
This file sorts last so that a run stopping at the first failure has already
run every other test."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from siglip2_b200 import _lib as L  # noqa: E402


def _inputs(lens, D, H, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    N = sum(lens)
    x = torch.randn(N, D, device="cuda", generator=g).to(dtype)
    u = torch.randn(H, D, device="cuda", generator=g) * 0.05
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    return x, u, cu, N


def _call(x, u, cu, N, H, D, dtype_code, with_scratch):
    lib = L.load()
    B = cu.numel() - 1
    pooled = torch.empty((B, H, D), dtype=x.dtype, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if with_scratch:
        scores = torch.empty(N * H, dtype=torch.float32, device="cuda")
        rc = lib.siglip2_head_pool(dtype_code, x.data_ptr(), D, H, cu.data_ptr(), B, 0, u.data_ptr(),
                                   scores.data_ptr(), pooled.data_ptr(), stream)
    else:
        rc = lib.siglip2_head_pool_noalloc(dtype_code, x.data_ptr(), D, H, cu.data_ptr(), B, 0, N, u.data_ptr(),
                                           pooled.data_ptr(), stream)
    L.check(rc)
    return pooled


@pytest.mark.parametrize("dtype,code,tol", [(torch.bfloat16, L.DTYPE_BF16, 2e-2), (torch.float32, L.DTYPE_F32, 1e-4)])
def test_noalloc_matches_regular_entry_point_twice(dtype, code, tol):
    D, H = 1152, 16
    # two different calls in a row: the second reuses the shared fixed scratch
    for seed, lens in ((1, [300, 17, 1024, 1, 96]), (2, [640, 5, 222])):
        x, u, cu, N = _inputs(lens, D, H, dtype, seed)
        ref = _call(x, u, cu, N, H, D, code, True)
        got = _call(x, u, cu, N, H, D, code, False)
        torch.cuda.synchronize()
        assert (got.float() - ref.float()).abs().max().item() <= tol
    L.check(L.load().siglip2_check_device(1))


def test_noalloc_rejects_oversize():
    lib = L.load()
    D, H = 1152, 16
    x, u, cu, N = _inputs([64], D, H, torch.bfloat16, 3)
    pooled = torch.empty((1, H, D), dtype=torch.bfloat16, device="cuda")
    too_many = (1 << 20) // H + 1
    rc = lib.siglip2_head_pool_noalloc(L.DTYPE_BF16, x.data_ptr(), D, H, cu.data_ptr(), 1, 0, too_many, u.data_ptr(),
                                       pooled.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -3  # SIGLIP2_ERR_SHAPE
    assert b"fixed scratch" in lib.siglip2_last_error()
