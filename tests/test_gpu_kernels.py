"""Varlen attention, LayerNorm and position-embedding kernels against torch
fp32 math on the same inputs (GPU)."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from oracle import siglip2_oracle as O  # noqa: E402
from siglip2_b200 import _lib as L  # noqa: E402
from siglip2_b200 import ops  # noqa: E402


@pytest.fixture(params=[1, 2], ids=["single_tile", "tile_pairs"])
def fmha_variant(request):
    """Attention tests run on both kernels: one 128-row query tile per CTA
    (two CTAs per SM) and two query tiles per CTA sharing each K/V tile."""
    lib = L.load()
    old = lib.siglip2_get_fmha_variant()
    L.check(lib.siglip2_set_fmha_variant(request.param))
    yield request.param
    L.check(lib.siglip2_set_fmha_variant(old))


def _cu(lens):
    return torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")


def _pack_qkv(q, k, v):
    """q | k | v columns, as the fused QKV projection writes them."""
    return torch.cat([q, k, v], 1).contiguous()


def _ref_attn(q, k, v, lens, H, hd):
    out = torch.empty_like(q, dtype=torch.float32)
    s = 0
    for L in lens:
        sl = slice(s, s + L)
        qh = q[sl].float().view(L, H, hd).transpose(0, 1)
        kh = k[sl].float().view(L, H, hd).transpose(0, 1)
        vh = v[sl].float().view(L, H, hd).transpose(0, 1)
        p = torch.softmax(qh @ kh.transpose(1, 2) / math.sqrt(hd), -1)
        out[sl] = (p @ vh).transpose(0, 1).reshape(L, H * hd)
        s += L
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,hd", [(16, 72), (12, 64), (16, 96), (2, 72)])
@pytest.mark.parametrize("lens", [[1, 7, 129, 300, 1024, 128, 256, 65], [576], [900, 3, 1000],
                                  # an image's last key tile ends on / just past 16-key chunks, and its last
                                  # query tile ends on / just past 32-row warps
                                  [16, 17, 31, 32, 33, 48, 95, 97, 112, 113, 160, 161, 191, 192, 193, 224, 225]])
def test_fmha_varlen(dtype, H, hd, lens, fmha_variant):
    g = torch.Generator(device="cuda").manual_seed(sum(lens) + hd)
    N = sum(lens)
    q, k, v = (torch.randn(N, H * hd, device="cuda", generator=g).to(dtype) for _ in range(3))
    qkv = _pack_qkv(q, k, v)
    cu = _cu(lens)
    tiles = ops.attention_tiles(lens).cuda()
    out = ops.fmha_varlen(qkv, cu, tiles, H, hd)
    ref = _ref_attn(q, k, v, lens, H, hd)
    torch.cuda.synchronize()
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err
    cos = F.cosine_similarity(out.float().flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.9999


@pytest.mark.parametrize("H,hd", [(16, 72), (12, 64), (16, 96)])
def test_fmha_many_items_per_cta(H, hd, fmha_variant):
    """The persistent attention kernel walks many (query tile, head) items
    per CTA (about 13 here), across image sizes from 1 to 1024 tokens, so Q
    buffers, K/V ring stages and the TMEM O hand-off all wrap many times."""
    g = torch.Generator().manual_seed(hd)
    lens = [int(x) for x in torch.randint(1, 1025, (52,), generator=g)] + [1, 2, 3, 96, 97, 128, 129, 1024]
    N = sum(lens)
    gd = torch.Generator(device="cuda").manual_seed(hd + 1)
    q, k, v = (torch.randn(N, H * hd, device="cuda", generator=gd).bfloat16() for _ in range(3))
    qkv = _pack_qkv(q, k, v)
    tiles = ops.attention_tiles(lens).cuda()
    assert tiles.shape[0] * H > 8 * 296
    out = ops.fmha_varlen(qkv, _cu(lens), tiles, H, hd)
    ref = _ref_attn(q, k, v, lens, H, hd)
    torch.cuda.synchronize()
    err = (out.float() - ref).abs()
    assert err.max().item() < 2e-2, err.max().item()
    # every row of every image was written (no item skipped)
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [768, 1152, 1536, 1024])
def test_layernorm_packed_and_padded(dtype, D):
    lens = [5, 300, 17, 256]
    N, P = sum(lens), 320
    x = (torch.randn(N, D, device="cuda") * 3 + 1).to(dtype)
    gamma = 1 + 0.1 * torch.randn(D, device="cuda")
    beta = 0.1 * torch.randn(D, device="cuda")
    ref = F.layer_norm(x.float(), (D,), gamma, beta, 1e-6)
    y = ops.layernorm(x, gamma, beta, 1e-6)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (y.float() - ref).abs().max().item() < tol
    yp = ops.layernorm(x, gamma, beta, 1e-6, cu_seqlens=_cu(lens), batch=len(lens), max_patches=P)
    s = 0
    for b, L in enumerate(lens):
        assert (yp[b, :L].float() - ref[s:s + L]).abs().max().item() < tol
        assert not yp[b, L:].any()
        s += L


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_posemb_matches_interpolate(dtype):
    D = 1152
    table = torch.randn(256, D, device="cuda") * 0.02
    grids = [(18, 18), (24, 31), (11, 37), (8, 128), (1, 1), (3, 5), (16, 16), (40, 25)]
    lens = [h * w for h, w in grids]
    N = sum(lens)
    cu = _cu(lens)
    hw = torch.tensor(grids, dtype=torch.int32, device="cuda").flatten()
    tok = ops.token_image(cu, N)
    out = ops.posemb(table, hw, cu, tok, N, dtype)
    grid = table.view(16, 16, D).permute(2, 0, 1)[None]
    refs = [F.interpolate(grid, size=(h, w), mode="bilinear", align_corners=False, antialias=True)[0]
            .reshape(D, h * w).T for h, w in grids]
    ref = torch.cat(refs, 0)
    torch.cuda.synchronize()
    tol = 1e-6 if dtype == torch.float32 else 2e-3
    assert (out.float() - ref).abs().max().item() < tol
    assert (tok.cpu().numpy() == np.repeat(np.arange(len(lens)), lens)).all()


def _ref_pool(x, u, lens):
    out, s = [], 0
    for L_ in lens:
        xs = x[s:s + L_].float()
        p = torch.softmax((xs @ u.T) * math.log(2.0), dim=0)  # u is in base-2 units
        out.append(p.T @ xs)
        s += L_
    return torch.stack(out)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D,H", [(1152, 16), (768, 12), (1536, 16)])
def test_head_pool(dtype, D, H):
    lens = [1, 37, 300, 1024, 128]
    N = sum(lens)
    g = torch.Generator(device="cuda").manual_seed(D + H)
    x = torch.randn(N, D, device="cuda", generator=g).to(dtype)
    u = torch.randn(H, D, device="cuda", generator=g) * 0.05
    pooled = ops.head_pool(x, u, _cu(lens), N)
    ref = _ref_pool(x, u, lens)
    torch.cuda.synchronize()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert (pooled.float() - ref).abs().max().item() < tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [1152, 768])
def test_patch_embed_fused_position_resize(dtype, D):
    g = torch.Generator(device="cuda").manual_seed(D)
    grids = [(18, 18), (24, 31), (11, 37), (8, 128), (1, 1), (3, 5), (16, 16), (40, 25)]
    lens = [h * w for h, w in grids]
    N = sum(lens)
    cu = _cu(lens)
    hw = torch.tensor(grids, dtype=torch.int32, device="cuda").flatten()
    tok = ops.token_image(cu, N)
    patches = (torch.rand(N, 768, device="cuda", generator=g) * 2 - 1).to(dtype)
    w = (torch.randn(D, 768, device="cuda", generator=g) * 0.02).to(dtype)
    bias = torch.randn(D, device="cuda", generator=g) * 0.02
    table = torch.randn(256, D, device="cuda", generator=g) * 0.02
    rs = torch.full((N, ops.rowsum_slots(dtype, D), 2), float("nan"), device="cuda")  # every slot is written
    out = ops.patch_embed(patches, w, bias, table, hw, cu, tok, rs)
    grid = table.view(16, 16, D).permute(2, 0, 1)[None]
    pos = torch.cat([F.interpolate(grid, size=(h, w_), mode="bilinear", align_corners=False, antialias=True)[0]
                     .reshape(D, h * w_).T for h, w_ in grids], 0)
    ref = patches.float() @ w.float().T + bias + pos
    torch.cuda.synchronize()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert (out.float() - ref).abs().max().item() < tol
    o = out.float()
    mean, var = ops.slot_stats_merge(rs, D)
    assert torch.allclose(mean, o.mean(1), rtol=1e-4, atol=1e-5)
    assert torch.allclose(var, o.var(1, unbiased=False), rtol=1e-3, atol=1e-6)
    assert torch.allclose(rs, ops.rowsums_reference(out), rtol=1e-3, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,D", [(3000, 1152), (257, 768), (1, 1536), (2049, 1024)])
def test_layernorm_backward_matches_autograd(dtype, rows, D):
    """siglip2_layernorm_backward against torch autograd of F.layer_norm in
    fp32 on the same (rounded) inputs: dx, dgamma, dbeta."""
    g = torch.Generator(device="cuda").manual_seed(rows + D)
    x = (torch.randn(rows, D, device="cuda", generator=g) * 2 + 0.5).to(dtype)
    dy = torch.randn(rows, D, device="cuda", generator=g).to(dtype)
    gamma = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
    beta = 0.1 * torch.randn(D, device="cuda", generator=g)
    dx, dg, db = ops.layernorm_backward(x, dy, gamma, 1e-6, chunk_rows=512)
    xr = x.float().requires_grad_(True)
    gr, br = gamma.clone().requires_grad_(True), beta.clone().requires_grad_(True)
    F.layer_norm(xr, (D,), gr, br, 1e-6).backward(dy.float())
    torch.cuda.synchronize()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    scale = xr.grad.abs().max().item()
    assert (dx.float() - xr.grad).abs().max().item() <= tol * scale
    assert torch.allclose(dg, gr.grad, rtol=1e-3, atol=1e-3 * max(1.0, rows ** 0.5))
    assert torch.allclose(db, br.grad, rtol=1e-3, atol=1e-3 * max(1.0, rows ** 0.5))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(16384, 4304), (1, 8), (1000, 1152), (257, 3456)])
def test_colsum_bias_gradient(dtype, rows, cols):
    """siglip2_colsum_partial (+ the in-order chunk sum): fp32 column sums
    against torch's fp32 sum of the same values, identical on a second call."""
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = torch.randn(rows, cols, device="cuda", generator=g).to(dtype)
    s1 = ops.colsum(x)
    s2 = ops.colsum(x)
    ref = x.double().sum(0)
    torch.cuda.synchronize()
    assert s1.dtype == torch.float32 and torch.equal(s1, s2)
    assert (s1.double() - ref).abs().max().item() < 1e-5 * rows ** 0.5 * x.float().abs().max().item() + 1e-6
