"""Host-side logic of the module API (no GPU): document ids, the sequences a
document mask or BlockMask describes, the flat packed-weight order, the
fake (shape) implementations of the registered ops, and the submodules'
parameter names and argument checks."""
import pytest
import torch
from torch.nn.attention.flex_attention import create_block_mask

import siglip2_b200 as S
from siglip2_b200 import _lib as L
from siglip2_b200 import model as M
from siglip2_b200 import workloads as W

O = torch.ops.siglip2_b200


def test_create_document_ids_known_answer():
    # model.py:12-36: ids per token, then unique pad ids counting up from N
    ids = S.create_document_ids(torch.tensor([3, 2, 4]))
    assert ids.numel() == 128
    assert ids[:9].tolist() == [0, 0, 0, 1, 1, 2, 2, 2, 2]
    assert ids[9:].tolist() == list(range(9, 128))
    full = S.create_document_ids(torch.tensor([100, 28]))
    assert full.numel() == 128 and full[-1].item() == 1


def test_sequences_from_document_ids():
    ids = S.create_document_ids(torch.tensor([5, 1, 130]))
    sq = M.Sequences.from_document_ids(ids, 136, 2, "cpu")
    assert sq.lengths == [5, 1, 130] * 2
    assert sq.cu_seqlens.tolist() == [0, 5, 6, 136, 141, 142, 272]
    assert sq.n_tokens == 272
    # tiles: every 128-row query tile of every sequence, longest first
    assert sorted(map(tuple, sq.tiles.tolist())) == sorted([(0, 0), (1, 0), (2, 0), (2, 1), (3, 0), (4, 0), (5, 0),
                                                            (5, 1)])
    assert sq.tiles[0].tolist()[0] in (2, 5)
    with pytest.raises(NotImplementedError):
        M.Sequences.from_document_ids(torch.tensor([0, 1, 0]), 3, 1, "cpu")
    with pytest.raises(ValueError):
        M.Sequences.from_document_ids(torch.tensor([0, 0]), 3, 1, "cpu")


def _doc_mask(ids):
    def doc(b, h, q, kv):
        return ids[q] == ids[kv]
    return doc


@pytest.mark.parametrize("sizes", [[3, 2], [1], [130, 7, 1, 64], [1, 1, 1]])
def test_sequences_from_block_mask(sizes):
    ids = S.create_document_ids(torch.tensor(sizes))
    n = sum(sizes)
    bm = create_block_mask(_doc_mask(ids), 1, 1, n, n, device="cpu")
    assert M.Sequences.from_block_mask(bm, n, 1, "cpu").lengths == sizes
    assert M.Sequences.from_block_mask(bm, n, 3, "cpu").lengths == sizes * 3


@pytest.mark.parametrize("mask", [
    lambda b, h, q, kv: q >= kv,                       # causal
    lambda b, h, q, kv: (q - kv).abs() <= 2,            # sliding window
    lambda b, h, q, kv: (q % 2) == (kv % 2),            # strided documents
])
def test_block_mask_other_than_documents_is_refused(mask):
    bm = create_block_mask(mask, 1, 1, 20, 20, device="cpu")
    with pytest.raises(NotImplementedError):
        M.Sequences.from_block_mask(bm, 20, 1, "cpu")


def test_block_mask_length_must_match():
    ids = S.create_document_ids(torch.tensor([4, 4]))
    bm = create_block_mask(_doc_mask(ids), 1, 1, 8, 8, device="cpu")
    with pytest.raises(ValueError):
        M.Sequences.from_block_mask(bm, 9, 1, "cpu")


def test_weight_structs_follow_the_flat_order():
    dims = [64, 128, 2, 2, 32, 48, 4, L.DTYPE_BF16, 1]
    n = 2 * len(M.LAYER_FIELDS) + len(M.TOWER_FIELDS) + len(M.HEAD_FIELDS)
    ts = [torch.empty(8) for _ in range(n)]
    cfg, w, layers = M.weight_structs(dims, 1e-6, ts)
    assert (cfg.hidden, cfg.layers, cfg.head_dim, cfg.dtype, cfg.has_head) == (64, 2, 32, L.DTYPE_BF16, 1)
    assert abs(cfg.eps - 1e-6) < 1e-12
    nl = len(M.LAYER_FIELDS)
    for i in range(2):
        for j, f in enumerate(M.LAYER_FIELDS):
            assert getattr(w.layers[i], f) == ts[i * nl + j].data_ptr()
    for j, f in enumerate(M.TOWER_FIELDS):
        assert getattr(w, f) == ts[2 * nl + j].data_ptr()
    for j, f in enumerate(M.HEAD_FIELDS):
        assert getattr(w, f) == ts[2 * nl + len(M.TOWER_FIELDS) + j].data_ptr()
    with pytest.raises(ValueError):
        M.weight_structs(dims, 1e-6, ts[:-1])
    dims[-1] = 0
    cfg, w, _ = M.weight_structs(dims, 1e-6, ts[:2 * nl + len(M.TOWER_FIELDS)])
    assert not w.head_u


def _meta(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, device="meta", dtype=dtype)


def test_fake_shapes_of_the_registered_ops():
    a, w = _meta(300, 1152), _meta(4304, 1152)
    assert O.gemm(a, w, L.EPI_BIAS_GELU, None, None, None, None, 0.0).shape == (300, 4304)
    out, rs = O.gemm_rowsums(a, w, L.EPI_LN_ROWSUMS, None, None, None, None, 1e-6, _meta(300, 9, 2), False)
    assert out.shape == (300, 4304) and rs.numel() == 0
    out, rs = O.gemm_rowsums(_meta(300, 4304), _meta(1152, 4304), L.EPI_BIAS_RES_ROWSUMS, None, a, None, None,
                             0.0, None, True)
    assert out.shape == (300, 1152) and rs.shape == (300, 9, 2) and rs.dtype == torch.float32
    assert O.rowsums(_meta(7, 4304)).shape == (7, 34, 2)
    assert O.rowsums(_meta(7, 768, dtype=torch.float32)).shape == (7, 6, 2)
    cu, tiles = _meta(3, dtype=torch.int32), _meta(4, 2, dtype=torch.int32)
    assert O.fmha_varlen(_meta(300, 3456), cu, tiles, 16, 72, [100, 200]).shape == (300, 1152)
    assert O.layernorm(a, _meta(1152, dtype=torch.float32), _meta(1152, dtype=torch.float32), 1e-6).shape == a.shape
    tok = O.token_image(cu, 300)
    assert tok.shape == (300,) and tok.dtype == torch.int32
    pe = O.patch_embed(_meta(300, 768), _meta(1152, 768), _meta(1152, dtype=torch.float32),
                       _meta(256, 1152, dtype=torch.float32), _meta(4, dtype=torch.int32), cu, tok, [10, 10, 10, 20])
    assert pe.shape == (300, 1152)


def test_fake_shapes_of_the_training_ops():
    """The ops a train step adds: transposed-operand GEMMs, the attention with
    its log-sum-exp and backward, the dropout mask and the LayerNorm backward."""
    dy, x = _meta(300, 4304), _meta(300, 1152)
    assert O.gemm_t(dy, _meta(4304, 1152), False, True, L.EPI_BIAS, None, None).shape == (300, 1152)
    assert O.gemm_t(dy, x, True, True, L.EPI_BIAS, None, None).shape == (4304, 1152)
    cu, tiles = _meta(3, dtype=torch.int32), _meta(4, 2, dtype=torch.int32)
    qkv = _meta(300, 3456)
    out, lse = O.fmha_varlen_train(qkv, cu, tiles, 16, 72, 0.1, 7)
    assert out.shape == (300, 1152) and lse.shape == (300, 16) and lse.dtype == torch.float32
    dqkv = O.fmha_varlen_backward(qkv, out, _meta(300, 1152), lse, cu, tiles, 16, 72, 0.1, 7)
    assert dqkv.shape == qkv.shape and dqkv.dtype == qkv.dtype
    assert O.dropout(x, 0.1, 3).shape == x.shape
    dx, dw, db = O.layernorm_backward(x, _meta(300, 1152), _meta(1152, dtype=torch.float32), 1e-6)
    assert dx.shape == x.shape and dw.shape == db.shape == (1152,) and dw.dtype == torch.float32


@pytest.mark.parametrize("max_patches,pooled", [(0, False), (0, True), (256, True)])
def test_fake_shapes_of_the_tower_op(max_patches, pooled):
    dims = [768, 3072, 1, 12, 64, 768, 16, L.DTYPE_BF16, 1]
    n = len(M.LAYER_FIELDS) + len(M.TOWER_FIELDS) + len(M.HEAD_FIELDS)
    ws = [_meta(8) for _ in range(n)]
    hw = torch.tensor([[10, 10], [8, 16]], dtype=torch.int32)
    patches = _meta(228, 768) if max_patches == 0 else _meta(2, max_patches, 768)
    last, pool = O.vision_tower(patches, hw, max_patches, pooled, ws, dims, 1e-6)
    assert last.shape == ((228, 768) if max_patches == 0 else (2, max_patches, 768))
    assert pool.shape == ((2, 768) if pooled else (0, 768))
    assert last.dtype == torch.bfloat16


def test_improved_submodules_have_the_reference_parameter_names():
    cfg = W.preset_config("b16", config_cls=S.Siglip2VisionConfig, num_hidden_layers=2)
    layer = S.Siglip2EncoderLayerImproved(cfg)
    assert set(layer.state_dict()) == {
        "self_attn.qkv_proj.weight", "self_attn.qkv_proj.bias", "self_attn.out_proj.weight",
        "self_attn.out_proj.bias", "layer_norm1.weight", "layer_norm1.bias", "mlp.fc1.weight", "mlp.fc1.bias",
        "mlp.fc2.weight", "mlp.fc2.bias", "layer_norm2.weight", "layer_norm2.bias"}
    assert layer.self_attn.qkv_proj.weight.shape == (3 * cfg.hidden_size, cfg.hidden_size)
    base = S.Siglip2EncoderLayer(cfg)
    assert {k for k in base.state_dict() if "proj" in k} == {
        f"self_attn.{n}_proj.{t}" for n in ("q", "k", "v", "out") for t in ("weight", "bias")}
    enc = S.Siglip2EncoderImproved(cfg)
    assert len(enc.layers) == 2 and isinstance(enc.layers[0], S.Siglip2EncoderLayerImproved)
    emb = S.Siglip2SequenceEmbeddingsImproved(cfg)
    assert set(emb.state_dict()) == {"patch_embedding.weight", "patch_embedding.bias", "position_embedding.weight"}
    mlp = S.MLPImproved(cfg)
    assert set(mlp.state_dict()) == {"fc1.weight", "fc1.bias", "fc2.weight", "fc2.bias"}


def test_layernorm_improved_init_and_refusals():
    ln = S.LayerNormImproved(16, eps=1e-6)
    assert torch.equal(ln.weight, torch.ones(16)) and ln.bias.shape == (16,)
    assert torch.equal(S.LayerNormImproved(16, 1e-6, bias=False, init_fn="zeros").weight, torch.zeros(16))
    with pytest.raises(ValueError):
        S.LayerNormImproved(16, 1e-6, init_fn="normal")
    x = torch.randn(4, 16)
    for kw in ({"dropout_p": 0.1}, {"x1": x}, {"rowscale": torch.ones(4)}, {"zero_centered_weight": True},
               {"return_dropout_mask": True}):
        with pytest.raises(NotImplementedError):
            ln(x, **kw)


def test_modules_refuse_cpu_parameters():
    cfg = W.preset_config("b16", config_cls=S.Siglip2VisionConfig, num_hidden_layers=1)
    with pytest.raises(RuntimeError, match="CUDA"):
        S.Siglip2MLP(cfg)(torch.randn(4, cfg.hidden_size))


def test_train_mode_dropout_arguments():
    """Attention-output dropout is active in train() mode only (as
    ``model.py:166-169``); each call draws its mask seed from torch's CPU
    generator, so ``torch.manual_seed`` reproduces it."""
    from siglip2_b200.model import _dropout_args
    cfg = W.preset_config("b16", config_cls=S.Siglip2VisionConfig, num_hidden_layers=1)
    cfg.attention_dropout = 0.1
    attn = S.Siglip2Attention(cfg)
    assert _dropout_args(attn.eval(), attn.dropout) == (0.0, 0)
    attn.train()
    torch.manual_seed(5)
    p, s1 = _dropout_args(attn, attn.dropout)
    _, s2 = _dropout_args(attn, attn.dropout)
    torch.manual_seed(5)
    _, s3 = _dropout_args(attn, attn.dropout)
    assert p == pytest.approx(0.1) and s1 == s3 and s1 != s2 and 0 <= s1 < 2 ** 63
    assert _dropout_args(attn, 0.0) == (0.0, 0)
