"""Submodule parity on the GPU: the reference's submodule classes and call
signatures (``model.py`` and ``optimized_siglip2/model_optimized.py``, as
``run_tests.py`` calls them) running on the library's kernels, against the
reference's op sequence replayed in torch in fp32 (on the same rounded
weights) and at the same dtype.  Bars: fp32 1e-4 max-abs; bf16/fp16 cosine
>= 0.999 and max-abs error against fp32 within 3e-2 of the same-dtype
reference's own.  Also: the ``...Improved`` classes (fused ``qkv_proj``,
``BlockMask``) give bit-identical results to the base classes, the
registered ops pass ``torch.library.opcheck``, and ``torch.compile`` traces
them."""
import pytest
import torch
import torch.nn.functional as F
from torch.nn.attention.flex_attention import create_block_mask

pytestmark = pytest.mark.gpu

import siglip2_b200 as S  # noqa: E402
from oracle import torch_ref as TR  # noqa: E402
from siglip2_b200 import _lib as L  # noqa: E402
from siglip2_b200 import ops  # noqa: E402
from siglip2_b200 import workloads as W  # noqa: E402

O = torch.ops.siglip2_b200
BF16, F16, F32 = torch.bfloat16, torch.float16, torch.float32


def _cfg(preset, layers=1):
    return W.preset_config(preset, config_cls=S.Siglip2VisionConfig, num_hidden_layers=layers)


def _sd(cfg, seed=5):
    return W.init_state_dict(cfg, seed=seed, with_head=False, random_affine=True)


def _sub(sd, pre):
    return {k[len(pre):]: v for k, v in sd.items() if k.startswith(pre)}


def _fuse_qkv(sd):
    """``model.py`` q/k/v keys -> the fused ``qkv_proj`` of ``model_optimized.py:215``."""
    out = dict(sd)
    for k in [k for k in sd if k.endswith("q_proj.weight")]:
        p = k[:-len("q_proj.weight")]
        for t in ("weight", "bias"):
            out[p + f"qkv_proj.{t}"] = torch.cat([out.pop(p + f"{n}_proj.{t}") for n in "qkv"], 0)
    return out


def _load(module, sd, dtype):
    module.load_state_dict(sd)
    return module.to("cuda", dtype).eval()


def _check(ours, ref_dt, ref32, dtype, what):
    """fp32: max-abs < 1e-4 against the fp32 reference.  bf16 / fp16: cosine
    > 0.999 against the same-dtype reference, and our max-abs error against
    fp32 at most the same-dtype reference's own plus 3e-2 (accuracy compared
    like for like); the literal max-abs against the same-dtype run is printed,
    not asserted (the full-depth bar is reported in tests/test_gpu_depth.py)."""
    ours, ref_dt, ref32 = (t.detach().float().cpu().reshape(-1, t.shape[-1]) for t in (ours, ref_dt, ref32))
    err = (ours - ref32).abs().max().item()
    if dtype == F32:
        assert err < 1e-4, (what, err)
        return
    cos = F.cosine_similarity(ours.flatten(), ref_dt.flatten(), dim=0).item()
    err_ref = (ref_dt - ref32).abs().max().item()
    lit = (ours - ref_dt).abs().max().item()
    print(f"\n[parity] {what}: cos={cos:.6f} err={err:.4f} ref_err={err_ref:.4f} max-abs vs same dtype={lit:.4f}")
    assert cos > 0.999 and err <= err_ref + 3e-2, (what, cos, err, err_ref, lit)


def _rand(shape, dtype, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to("cuda", dtype)


LENS = [300, 1, 129, 64, 700, 17]


@pytest.mark.parametrize("preset,dtype", [("so400m", BF16), ("l16", F16), ("b16", F32)])
def test_mlp(preset, dtype):
    cfg, pre = _cfg(preset), "encoder.layers.0.mlp."
    sd = _sd(cfg)
    sdq = {k: v.to(dtype).float() for k, v in sd.items()}
    m = _load(S.Siglip2MLP(cfg), _sub(sd, pre), dtype)
    x = _rand((2, 333, cfg.hidden_size), dtype)
    out = m(x)
    assert out.shape == x.shape and out.dtype == dtype
    x2 = x.reshape(-1, cfg.hidden_size)
    _check(out, TR.mlp(sdq, pre, x2, dtype), TR.mlp(sdq, pre, x2.float(), F32), dtype, f"mlp {preset}")
    mi = _load(S.MLPImproved(cfg), _sub(sd, pre), dtype)
    assert torch.equal(mi(x), out)


@pytest.mark.parametrize("dtype", [BF16, F32])
def test_layernorm_modules(dtype):
    D = 1152
    g = torch.Generator().manual_seed(3)
    w, b = 1 + 0.1 * torch.randn(D, generator=g), 0.1 * torch.randn(D, generator=g)
    ln = _load(S.LayerNorm(D, eps=1e-6), {"weight": w, "bias": b}, dtype)
    lni = _load(S.LayerNormImproved(D, eps=1e-6), {"weight": w, "bias": b}, dtype)
    x = _rand((3, 77, D), dtype, seed=1, scale=2.0) + 0.5
    wq, bq = w.to(dtype).float().cuda(), b.to(dtype).float().cuda()
    tol = dict(rtol=0, atol=1e-4) if dtype == F32 else dict(rtol=1e-2, atol=2e-2)
    y = ln(x)
    assert y.dtype == dtype
    assert torch.allclose(y.float(), F.layer_norm(x.float(), (D,), wq, bq, 1e-6), **tol)
    assert torch.equal(lni(x), y)
    # optimized_siglip2/model_optimized.py:286-288: residual add, prenorm returns the sum
    r = _rand((3, 77, D), dtype, seed=2)
    s32 = x.float() + r.float()
    y2, res2 = lni(x, residual=r, prenorm=True)
    assert torch.allclose(y2.float(), F.layer_norm(s32, (D,), wq, bq, 1e-6), **tol)
    assert res2.dtype == dtype and torch.equal(res2, s32.to(dtype))
    y3, res3 = lni(x, residual=r, prenorm=True, residual_in_fp32=True)
    assert res3.dtype == F32 and torch.equal(res3, s32) and torch.equal(y3, y2)
    y4 = lni(x, out_dtype=F32)
    assert y4.dtype == F32
    out, rout = torch.empty_like(x), torch.empty_like(x)
    y5, r5 = lni(x, residual=r, prenorm=True, out=out, residual_out=rout)
    assert y5.data_ptr() == out.data_ptr() and r5.data_ptr() == rout.data_ptr() and torch.equal(y5, y2)


@pytest.mark.parametrize("preset,dtype", [("so400m", BF16), ("b16", F32)])
def test_embeddings(preset, dtype):
    cfg = _cfg(preset)
    sd = _sd(cfg)
    sdq = {k: v.to(dtype).float() for k, v in sd.items()}
    emb = _load(S.Siglip2SequenceEmbeddings(cfg), _sub(sd, "embeddings."), dtype)
    grids = [(18, 18), (24, 31), (11, 37), (8, 128), (1, 1), (5, 33)]
    g = torch.tensor(grids)
    lens = [h * w for h, w in grids]
    pv, _ = W.make_pixels(g, max(lens), cfg.num_channels * cfg.patch_size ** 2)
    packed = W.pack_rows(pv, g)
    out = emb((packed.to("cuda", dtype), g.prod(-1), g.cuda()))
    assert out.shape == (sum(lens), cfg.hidden_size)
    _check(out, TR.embeddings(sdq, cfg, packed, grids, dtype),
           TR.embeddings(sdq, cfg, packed.to(dtype).float(), grids, F32), dtype, f"embeddings {preset}")
    ei = _load(S.Siglip2SequenceEmbeddingsImproved(cfg), _sub(sd, "embeddings."), dtype)
    assert torch.equal(ei((packed.to("cuda", dtype), g.prod(-1), g)), out)
    with pytest.raises(ValueError):
        emb((packed.to("cuda", dtype), g.prod(-1) + 1, g))


def _doc_block_mask(ids, n):
    def doc(b, h, q, kv):
        return ids[q] == ids[kv]
    return create_block_mask(doc, 1, 1, n, n, device="cuda")


@pytest.mark.parametrize("preset,dtype", [("so400m", BF16), ("b16", F16), ("g16", BF16), ("b16", F32)])
def test_attention(preset, dtype):
    cfg, pre = _cfg(preset), "encoder.layers.0.self_attn."
    sd = _sd(cfg)
    sdq = {k: v.to(dtype).float() for k, v in sd.items()}
    attn = _load(S.Siglip2Attention(cfg), _sub(sd, pre), dtype)
    N = sum(LENS)
    x = _rand((1, N, cfg.hidden_size), dtype)
    ids = S.create_document_ids(torch.tensor(LENS), "cuda")
    out, weights = attn(x, document_ids=ids)
    assert weights is None and out.shape == x.shape
    _check(out, TR.attention(sdq, cfg, pre, x[0], LENS, dtype), TR.attention(sdq, cfg, pre, x[0].float(), LENS, F32),
           dtype, f"attention {preset}")
    # optimized form: fused qkv_proj and a BlockMask of the same documents
    ai = _load(S.Siglip2AttentionImproved(cfg), _sub(_fuse_qkv(sd), pre), dtype)
    out2, _ = ai(x, block_mask=_doc_block_mask(ids, N))
    assert torch.equal(out2, out)


def test_attention_batch_without_mask_attends_within_each_entry():
    cfg, pre = _cfg("b16"), "encoder.layers.0.self_attn."
    sd = _sd(cfg)
    sdq = {k: v.to(BF16).float() for k, v in sd.items()}
    attn = _load(S.Siglip2Attention(cfg), _sub(sd, pre), BF16)
    x = _rand((3, 200, cfg.hidden_size), BF16, seed=4)
    out, _ = attn(x)
    for b in range(3):
        _check(out[b], TR.attention(sdq, cfg, pre, x[b], [200], BF16),
               TR.attention(sdq, cfg, pre, x[b].float(), [200], F32), BF16, f"batch entry {b}")


@pytest.mark.parametrize("preset,dtype", [("so400m", BF16), ("l16", F16), ("b16", F32)])
def test_encoder_layer(preset, dtype):
    cfg, pre = _cfg(preset), "encoder.layers.0."
    sd = _sd(cfg)
    sdq = {k: v.to(dtype).float() for k, v in sd.items()}
    layer = _load(S.Siglip2EncoderLayer(cfg), _sub(sd, pre), dtype)
    N = sum(LENS)
    x = _rand((1, N, cfg.hidden_size), dtype)
    ids = S.create_document_ids(torch.tensor(LENS), "cuda")
    ref_dt = TR.encoder_layer(sdq, cfg, pre, x[0], LENS, dtype)
    ref32 = TR.encoder_layer(sdq, cfg, pre, x[0].float(), LENS, F32)
    li = _load(S.Siglip2EncoderLayerImproved(cfg), _sub(_fuse_qkv(sd), pre), dtype)
    with torch.no_grad():  # inference: LayerNorms folded into the GEMMs, row sums carried
        out = layer(x, ids)
        assert out.shape == x.shape
        _check(out, ref_dt, ref32, dtype, f"encoder layer {preset}")
        assert torch.equal(li(x, _doc_block_mask(ids, N)), out)
    out_g = layer(x, ids)  # autograd recording: the unfused layer
    _check(out_g, ref_dt, ref32, dtype, f"encoder layer {preset} (unfused)")
    assert torch.equal(li(x, _doc_block_mask(ids, N)), out_g)


@pytest.mark.parametrize("preset", ["b16", "so400m"])
def test_submodules_compose_to_the_tower(preset):
    """embeddings -> encoder -> post_layernorm (``model.py:260-292``) through
    the submodule forwards equals the tower's single library call up to the
    LayerNorm statistics of the first layer (summed by a separate kernel
    here, by the patch-embedding epilogue in the tower)."""
    cfg = _cfg(preset, layers=2)
    cfg.vision_use_head = False
    sd = _sd(cfg, seed=9)
    tower = _load(S.Siglip2SequenceVisionTransformer(cfg), sd, BF16)
    grids = [(18, 18), (24, 31), (11, 37), (32, 32), (8, 128), (5, 7)]
    g = torch.tensor(grids)
    lens = [h * w for h, w in grids]
    pv, _ = W.make_pixels(g, max(lens), cfg.num_channels * cfg.patch_size ** 2, seed=9)
    packed = W.pack_rows(pv, g).to("cuda", BF16)
    with torch.no_grad():
        ref = tower((packed, g))
    sizes = g.prod(-1)
    with torch.no_grad():
        x = tower.embeddings((packed, sizes, g))
        ids = S.create_document_ids(sizes, "cuda")
        y = tower.encoder(x[None], ids)
        ours = tower.post_layernorm(y)[0]
    s = 0
    for n in lens:
        c = F.cosine_similarity(ours[s:s + n].float().flatten(), ref[s:s + n].float().flatten(), dim=0).item()
        assert c > 0.9999, c
        s += n
    assert (ours.float() - ref.float()).abs().max().item() < 0.1
    enc = _load(S.Siglip2EncoderImproved(cfg), _sub(_fuse_qkv(sd), "encoder."), BF16)
    with torch.no_grad():
        assert torch.equal(enc(x[None], ids), y)


def test_vision_tower_op_matches_the_module():
    cfg = _cfg("b16", layers=2)
    sd = W.init_state_dict(cfg, seed=2, with_head=True, random_affine=True)
    m = _load(S.Siglip2SequenceVisionTransformer(cfg), sd, BF16)
    grids = [(12, 20), (16, 16), (30, 8), (3, 3)]
    g = torch.tensor(grids)
    pv, mask = W.make_pixels(g, 256, cfg.num_channels * cfg.patch_size ** 2, seed=2)
    pv = pv.to("cuda", BF16)
    with torch.no_grad():
        res = m(pv, mask.cuda(), g.cuda())
    pk = m.packed_weights()
    last, pooled = O.vision_tower(pv, g.to(torch.int32), 256, True, pk.tensors, pk.dims, pk.eps)
    assert torch.equal(last, res.last_hidden_state) and torch.equal(pooled, res.pooler_output)
    packed = W.pack_rows(pv.cpu(), g).to("cuda", BF16)
    last2, empty = O.vision_tower(packed, g.to(torch.int32), 0, False, pk.tensors, pk.dims, pk.eps)
    assert empty.shape == (0, cfg.hidden_size)
    with torch.no_grad():
        assert torch.equal(last2, m((packed, g)))


def test_registered_ops_pass_opcheck():
    """Fake (shape) implementations agree with the CUDA kernels and the
    schemas hold (``torch.library.opcheck``)."""
    tests = ("test_schema", "test_faketensor")
    a = _rand((200, 256), BF16)
    w = _rand((384, 256), BF16, seed=1, scale=0.05)
    bias = _rand((384,), F32, seed=2)
    torch.library.opcheck(O.gemm, (a, w, L.EPI_BIAS_GELU, bias, None, None, None, 0.0), test_utils=tests)
    torch.library.opcheck(O.rowsums, (a,), test_utils=tests)
    w2 = _rand((256, 384), BF16, seed=3, scale=0.05)
    h = O.gemm(a, w, L.EPI_BIAS, bias, None, None, None, 0.0)
    torch.library.opcheck(O.gemm_rowsums, (h, w2, L.EPI_BIAS_RES_ROWSUMS, bias[:256].contiguous(), a, None, None,
                                           0.0, None, True), test_utils=tests)
    gam, bet = _rand((256,), F32, seed=4), _rand((256,), F32, seed=5)
    torch.library.opcheck(O.layernorm, (a, gam, bet, 1e-6), test_utils=tests)
    sq = S.Sequences([120, 80], "cuda")
    qkv = _rand((200, 3 * 4 * 64), BF16, seed=6)
    torch.library.opcheck(O.fmha_varlen, (qkv, sq.cu_seqlens, sq.tiles, 4, 64, sq.lengths), test_utils=tests)
    torch.library.opcheck(O.token_image, (sq.cu_seqlens, 200), test_utils=tests)
    _, rs = O.gemm_rowsums(h, w2, L.EPI_BIAS_RES_ROWSUMS, bias[:256].contiguous(), a, None, None, 0.0, None, True)
    assert rs.shape == (200, ops.rowsum_slots(BF16, 256), 2)
    assert torch.allclose(rs, ops.rowsums_reference(O.gemm(h, w2, L.EPI_BIAS_RES, bias[:256].contiguous(), a, None,
                                                           None, 0.0)), rtol=1e-4, atol=1e-2)
    assert torch.allclose(O.rowsums(a), ops.rowsums_reference(a), rtol=1e-4, atol=1e-3)


def test_torch_compile_traces_the_submodules():
    cfg = _cfg("b16")
    sd = _sd(cfg)
    layer = _load(S.Siglip2EncoderLayer(cfg), _sub(sd, "encoder.layers.0."), BF16)
    mlp = _load(S.Siglip2MLP(cfg), _sub(sd, "encoder.layers.0.mlp."), BF16)
    x = _rand((1, 333, cfg.hidden_size), BF16)
    ids = S.create_document_ids(torch.tensor([200, 133]), "cuda")
    torch._dynamo.reset()
    assert torch.equal(torch.compile(mlp, backend="aot_eager")(x), mlp(x))
    assert torch.equal(torch.compile(layer, backend="aot_eager")(x, ids), layer(x, ids))


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_mlp_and_layernorm_backward(dtype):
    """The stop-gap backward (``run_tests.py:74-82`` back-propagates through
    MLPImproved and LayerNormImproved): gradients of the input and of every
    parameter against torch autograd on the same weights in fp32."""
    cfg, pre = _cfg("b16"), "encoder.layers.0.mlp."
    sd = _sd(cfg)
    mlp = _load(S.MLPImproved(cfg), _sub(sd, pre), dtype)
    ln = _load(S.LayerNormImproved(cfg.hidden_size, eps=1e-6), {"weight": 1 + 0.1 * torch.randn(cfg.hidden_size),
                                                                 "bias": 0.1 * torch.randn(cfg.hidden_size)}, dtype)
    x = _rand((3, 67, cfg.hidden_size), dtype).requires_grad_(True)
    r = _rand((3, 67, cfg.hidden_size), dtype, seed=7)
    g = torch.Generator().manual_seed(8)
    up = torch.randn(3, 67, cfg.hidden_size, generator=g).to("cuda", dtype)
    h, res = ln(x, residual=r, prenorm=True, residual_in_fp32=True)
    out = mlp(h)
    (out.float() * up.float()).sum().backward()
    # torch reference in fp32 on the same (rounded) parameters
    xr = x.detach().float().requires_grad_(True)
    params = {n: p.detach().float().requires_grad_(True) for n, p in
              [("ln.w", ln.weight), ("ln.b", ln.bias), ("fc1.w", mlp.fc1.weight), ("fc1.b", mlp.fc1.bias),
               ("fc2.w", mlp.fc2.weight), ("fc2.b", mlp.fc2.bias)]}
    hr = F.layer_norm(xr + r.float(), (cfg.hidden_size,), params["ln.w"], params["ln.b"], 1e-6)
    hr = F.gelu(F.linear(hr, params["fc1.w"], params["fc1.b"]), approximate="tanh")
    outr = F.linear(hr, params["fc2.w"], params["fc2.b"])
    (outr * up.float()).sum().backward()
    got = {"x": x.grad, "ln.w": ln.weight.grad, "ln.b": ln.bias.grad, "fc1.w": mlp.fc1.weight.grad,
           "fc1.b": mlp.fc1.bias.grad, "fc2.w": mlp.fc2.weight.grad, "fc2.b": mlp.fc2.bias.grad}
    want = {"x": xr.grad, **{k: v.grad for k, v in params.items()}}
    for k in got:
        a, b = got[k].float().flatten(), want[k].flatten()
        cos = F.cosine_similarity(a, b, dim=0).item()
        rel = ((a - b).norm() / b.norm()).item()
        print(f"\n[grad] {dtype} {k}: cos {cos:.6f} rel {rel:.2e}")
        assert cos > (0.99999 if dtype == F32 else 0.999) and rel < (1e-4 if dtype == F32 else 4e-2), (k, cos, rel)
    assert res.dtype == F32


def _grad_check(got, want, dtype, what):
    for k in got:
        a, b = got[k].float().flatten(), want[k].float().flatten()
        if k == "self_attn.k_proj.bias":
            # the key bias shifts every score of a query row equally: softmax
            # ignores it, its gradient is zero up to rounding on both sides
            scale = max(got["self_attn.v_proj.bias"].float().norm().item(), 1e-30)
            assert a.norm().item() < 1e-2 * scale and b.norm().item() < 1e-2 * scale, (k, a.norm(), b.norm())
            continue
        cos = F.cosine_similarity(a, b, dim=0).item()
        rel = ((a - b).norm() / b.norm()).item()
        print(f"\n[grad] {what} {dtype} {k}: cos {cos:.6f} rel {rel:.2e}")
        assert cos > (0.99999 if dtype == F32 else 0.999) and rel < (1e-3 if dtype == F32 else 5e-2), (k, cos, rel)


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_encoder_layer_and_embeddings_backward(dtype):
    """Encoder layer (document ids, and the BlockMask form) and embeddings
    back-propagate: gradients of the input and every parameter against torch
    autograd in fp32 on the same weights (``model.py:68-120, 144-223``)."""
    cfg, pre = _cfg("b16"), "encoder.layers.0."
    sd = _sd(cfg, seed=6)
    lens = [200, 1, 129, 64]
    N, D, H = sum(lens), cfg.hidden_size, cfg.num_attention_heads
    hd = D // H
    ids = S.create_document_ids(torch.tensor(lens), "cuda")
    g = torch.Generator().manual_seed(9)
    up = torch.randn(1, N, D, generator=g).to("cuda")
    for layer in (_load(S.Siglip2EncoderLayer(cfg), _sub(sd, pre), dtype),
                  _load(S.Siglip2EncoderLayerImproved(cfg), _sub(_fuse_qkv(sd), pre), dtype)):
        x = _rand((1, N, D), dtype, seed=10).requires_grad_(True)
        improved = isinstance(layer, S.Siglip2EncoderLayerImproved)
        out = layer(x, _doc_block_mask(ids, N)) if improved else layer(x, ids)
        (out.float() * up).sum().backward()
        params = {n: p.detach().float().requires_grad_(True) for n, p in layer.named_parameters()}
        xr = x.detach().float().requires_grad_(True)
        P = params
        h = F.layer_norm(xr[0], (D,), P["layer_norm1.weight"], P["layer_norm1.bias"], cfg.layer_norm_eps)
        if improved:
            qkv = F.linear(h, P["self_attn.qkv_proj.weight"], P["self_attn.qkv_proj.bias"])
        else:
            qkv = torch.cat([F.linear(h, P[f"self_attn.{n}_proj.weight"], P[f"self_attn.{n}_proj.bias"])
                             for n in "qkv"], 1)
        q, k, v = qkv.view(N, 3, H, hd).unbind(1)
        outs, s0 = [], 0
        for n in lens:
            sl = slice(s0, s0 + n)
            o = F.scaled_dot_product_attention(*(t[sl].transpose(0, 1)[None] for t in (q, k, v)), scale=hd ** -0.5)
            outs.append(o[0].transpose(0, 1).reshape(n, D))
            s0 += n
        r = xr[0] + F.linear(torch.cat(outs, 0), P["self_attn.out_proj.weight"], P["self_attn.out_proj.bias"])
        h = F.layer_norm(r, (D,), P["layer_norm2.weight"], P["layer_norm2.bias"], cfg.layer_norm_eps)
        h = F.gelu(F.linear(h, P["mlp.fc1.weight"], P["mlp.fc1.bias"]), approximate="tanh")
        ref = r + F.linear(h, P["mlp.fc2.weight"], P["mlp.fc2.bias"])
        (ref[None] * up).sum().backward()
        got = {"x": x.grad, **{n: p.grad for n, p in layer.named_parameters()}}
        want = {"x": xr.grad, **{n: p.grad for n, p in params.items()}}
        _grad_check(got, want, dtype, "layer (improved)" if improved else "layer")
    # embeddings: patch Linear + resized position grid
    emb = _load(S.Siglip2SequenceEmbeddings(cfg), _sub(sd, "embeddings."), dtype)
    grids = [(18, 18), (11, 37), (5, 3), (20, 12)]
    gt = torch.tensor(grids)
    n_tok = sum(a * b for a, b in grids)
    pv = _rand((n_tok, 768), dtype, seed=11).requires_grad_(True)
    out = emb((pv, gt.prod(-1), gt))
    up2 = torch.randn(n_tok, D, generator=g).to("cuda")
    (out.float() * up2).sum().backward()
    P = {n: p.detach().float().requires_grad_(True) for n, p in emb.named_parameters()}
    pr = pv.detach().float().requires_grad_(True)
    G = int(cfg.num_patches ** 0.5)
    table = P["position_embedding.weight"].reshape(G, G, D).permute(2, 0, 1)[None]
    pos = torch.cat([F.interpolate(table, size=hw, mode="bilinear", align_corners=False, antialias=True)
                     .reshape(D, -1).t() for hw in grids], 0)
    ref = F.linear(pr, P["patch_embedding.weight"], P["patch_embedding.bias"]) + pos
    (ref * up2).sum().backward()
    _grad_check({"x": pv.grad, **{n: p.grad for n, p in emb.named_parameters()}},
                {"x": pr.grad, **{n: p.grad for n, p in P.items()}}, dtype, "embeddings")


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_map_head_module(dtype):
    """The attention-pooling head's own forward (transformers
    ``modeling_siglip2.py:684-713``) on padded rows against the torch replay
    of it on each image's valid rows; padded rows (random here) are ignored."""
    cfg = _cfg("b16")
    sd = W.init_state_dict(cfg, seed=12, with_head=True, random_affine=True)
    sdq = {k: v.to(dtype).float() for k, v in sd.items()}
    head = _load(S.Siglip2MultiheadAttentionPoolingHead(cfg), _sub(sd, "head."), dtype)
    lens, P, D = [200, 37, 256, 1], 256, cfg.hidden_size
    x = _rand((len(lens), P, D), dtype, seed=13)
    mask = (torch.arange(P)[None] < torch.tensor(lens)[:, None]).to(torch.int64)
    with torch.no_grad():
        out = head(x, mask.cuda())
        full = head(x[:, :100])  # no mask: every row valid
    assert out.shape == (len(lens), D)
    # autograd recording: the differentiable steps give the same pooled rows
    # and gradients reach every parameter and the input
    xg = x.clone().requires_grad_(True)
    out_ag = head(xg, mask.cuda())
    c = F.cosine_similarity(out_ag.detach().float(), out.float(), dim=1).min().item()
    assert c > 0.9999, c
    out_ag.float().square().sum().backward()
    assert xg.grad is not None and xg.grad[0, lens[0]:].abs().max().item() == 0  # padded rows get nothing
    for n, p_ in head.named_parameters():
        assert p_.grad is not None and torch.isfinite(p_.grad).all(), n
    packed = torch.cat([x[b, :n] for b, n in enumerate(lens)], 0)
    grids = [(n, 1) for n in lens]
    _check(out, TR.map_head(sdq, cfg, packed, grids, dtype), TR.map_head(sdq, cfg, packed.float(), grids, F32),
           dtype, "MAP head")
    ref_full = TR.map_head(sdq, cfg, x[:, :100].reshape(-1, D).float(), [(100, 1)] * len(lens), F32)
    _check(full, TR.map_head(sdq, cfg, x[:, :100].reshape(-1, D), [(100, 1)] * len(lens), dtype), ref_full, dtype,
           "MAP head, no mask")
    bad = mask.clone()
    bad[0, 0] = 0
    with pytest.raises(NotImplementedError), torch.no_grad():
        head(x, bad)
