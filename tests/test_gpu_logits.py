"""Image-text logits after the tower against the formula of transformers'
``Siglip2Model.forward`` (``models/siglip2/modeling_siglip2.py:964-974``):
fp32 within 1e-4; bf16 / fp16 no less accurate than the same formula run at
that dtype (error against fp32 within one output ulp at the logits' size of
the same-dtype formula's own error)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from siglip2_b200.logits import image_text_logits, l2_normalize  # noqa: E402


def _hf_formula(img, txt, logit_scale, logit_bias):
    img = img / img.norm(p=2, dim=-1, keepdim=True)
    txt = txt / txt.norm(p=2, dim=-1, keepdim=True)
    per_text = torch.matmul(txt, img.t())
    ls = torch.tensor([logit_scale], dtype=img.dtype, device=img.device)
    lb = torch.tensor([logit_bias], dtype=img.dtype, device=img.device)
    per_text = per_text * ls.exp() + lb
    return per_text.t(), per_text


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,T,D", [(37, 53, 1152), (64, 64, 768), (5, 300, 1536), (1, 1, 1024)])
def test_logits_match_the_formula(dtype, B, T, D):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T)
    img = torch.randn(B, D, device="cuda", generator=g).to(dtype)
    txt = torch.randn(T, D, device="cuda", generator=g).to(dtype)
    ls, lb = math.log(10.0), -10.0  # SigLIP's initial logit scale and bias
    per_image, per_text = image_text_logits(img, txt, ls, lb)
    assert per_image.shape == (B, T) and per_text.shape == (T, B) and per_text.dtype == dtype
    ref_i32, ref_t32 = _hf_formula(img.float(), txt.float(), ls, lb)
    err = (per_text.float() - ref_t32).abs().max().item()
    assert torch.equal(per_image, per_text.t())
    if dtype == torch.float32:
        assert err < 1e-4, err
        return
    _, ref_tdt = _hf_formula(img, txt, ls, lb)
    err_ref = (ref_tdt.float() - ref_t32).abs().max().item()
    ulp = 2.0 ** (math.floor(math.log2(max(ref_t32.abs().max().item(), 1e-3))) - (7 if dtype == torch.bfloat16 else 10))
    print(f"\n[parity] logits {dtype} {B}x{T}x{D}: err {err:.4f}, same-dtype formula {err_ref:.4f}")
    assert err <= err_ref + ulp, (err, err_ref, ulp)


def test_zero_rows_and_normalisation():
    x = torch.randn(10, 768, device="cuda", dtype=torch.bfloat16)
    x[3] = 0
    y = l2_normalize(x, 2.0, rows_out=16)
    n = y.float().norm(dim=1)
    assert torch.allclose(n[[0, 1, 2, 4, 5, 6, 7, 8, 9]], torch.full((9,), 2.0, device="cuda"), rtol=1e-2)
    assert n[3].item() == 0 and not y[10:].any()
    per_image, _ = image_text_logits(x, x[:4], 0.0, -3.0)
    assert torch.all(per_image[3].float() == -3.0)
