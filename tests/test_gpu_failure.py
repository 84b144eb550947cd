"""Failure detection without a GPU fault: a kernel whose wait can never be
satisfied gives up after its (short) limit, the host reads an error status,
and the context keeps working (a GEMM right after is correct)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from siglip2_b200 import _lib as L  # noqa: E402
from siglip2_b200 import ops  # noqa: E402


def test_bounded_wait_times_out_into_an_error_status():
    lib = L.load()
    L.check(lib.siglip2_check_device(1))  # clean slate
    L.check(lib.siglip2_selftest_wait_timeout(50_000_000, torch.cuda.current_stream().cuda_stream))  # 50 ms
    rc = lib.siglip2_check_device(1)
    assert rc == -5  # SIGLIP2_ERR_TIMEOUT
    assert b"site 901" in lib.siglip2_last_error()
    assert lib.siglip2_check_device(0) == 0  # flag was reset
    a = torch.randn(256, 512, device="cuda").bfloat16()
    w = torch.randn(256, 512, device="cuda").bfloat16()
    out = ops.gemm(a, w, L.EPI_BIAS, bias=torch.zeros(256, device="cuda"))
    torch.cuda.synchronize()
    assert (out.float() - a.float() @ w.float().T).abs().max().item() < 0.5
