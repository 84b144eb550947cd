"""The C ABI library loads and exports every function the header declares
(no compute calls: these run without a GPU), and host-side validation
paths that need no device."""
import ctypes
import os
import re

import numpy as np

from siglip2_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "siglip2_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(siglip2_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.SIGNATURES), set(names) ^ set(L.SIGNATURES)


def test_version_and_errors_without_gpu():
    lib = L.load()
    assert lib.siglip2_version() >= 100
    assert lib.siglip2_padded_head_dim(72) == 80
    assert lib.siglip2_padded_head_dim(64) == 64
    assert lib.siglip2_padded_head_dim(96) == 96


def test_metadata_layout():
    lib = L.load()
    hw = np.array([[3, 5], [16, 16], [1, 1], [20, 7]], dtype=np.int32)
    n_tok, n_tiles = ctypes.c_int(), ctypes.c_int()
    size = lib.siglip2_metadata_size(hw.ctypes.data, 4, ctypes.byref(n_tok), ctypes.byref(n_tiles))
    assert n_tok.value == 15 + 256 + 1 + 140
    assert n_tiles.value == 1 + 2 + 1 + 2
    buf = np.full(size, -7, dtype=np.int32)
    assert lib.siglip2_metadata(hw.ctypes.data, 4, buf.ctypes.data, size) == 0
    cu = buf[:5]
    assert list(cu) == [0, 15, 271, 272, 412]
    assert list(buf[5:13]) == hw.reshape(-1).tolist()
    off = (3 * 4 + 1 + 1) & ~1
    tiles = buf[off:off + 2 * n_tiles.value].reshape(-1, 2)
    assert tiles[0, 0] == 1  # longest image first
    assert sorted(map(tuple, tiles.tolist())) == sorted([(0, 0), (1, 0), (1, 1), (2, 0), (3, 0), (3, 1)])
    bad = np.array([[0, 5]], dtype=np.int32)
    assert lib.siglip2_metadata_size(bad.ctypes.data, 1, None, None) == -3
    assert b"non-positive" in lib.siglip2_last_error()


def test_workspace_size_monotone():
    lib = L.load()
    cfg = L.Config(hidden=1152, intermediate=4304, layers=27, heads=16, head_dim=72, patch_dim=768, pos_grid=16,
                   eps=1e-6, dtype=1, has_head=1)
    a = lib.siglip2_workspace_size(ctypes.byref(cfg), 64, 30000)
    b = lib.siglip2_workspace_size(ctypes.byref(cfg), 64, 40000)
    assert 0 < a < b


def test_rowsum_slots_follow_the_tile_widths():
    """Row-sum slots are half a GEMM tile wide (256-wide tiles, 128-column
    slots) on the tensor-core path and 128 wide on the fp32 path; bad widths
    are rejected without a GPU."""
    lib = L.load()
    bf16, f32 = 1, 0
    assert lib.siglip2_rowsum_slots(bf16, 1152) == 9
    assert lib.siglip2_rowsum_slots(bf16, 768) == 6
    assert lib.siglip2_rowsum_slots(bf16, 1536) == 12
    assert lib.siglip2_rowsum_slots(bf16, 4304) == 34
    assert lib.siglip2_rowsum_slots(f32, 768) == 6
    assert lib.siglip2_rowsum_slots(bf16, 0) < 0
    assert lib.siglip2_rowsum_block(bf16, 1152) == 128
    assert lib.siglip2_rowsum_block(bf16, 4304) == 128  # the last of the 34 slots holds 80 columns
    assert lib.siglip2_rowsum_block(f32, 4304) == 128
