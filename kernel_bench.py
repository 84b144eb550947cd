"""Per-kernel timing driver at the tower's shapes (CUDA events), also the
command the ncu summaries under ``profiles/`` were captured with.

    python kernel_bench.py gemm --epi ln_gelu --m 39178 --n 4304 --k 1152
    python kernel_bench.py gemm_e4m3 --m 39178 --n 4304 --k 1152 --epi bias_gelu
    python kernel_bench.py fmha --preset so400m --images 64 --max-patches 1024
    python kernel_bench.py layer --preset so400m --images 64 --max-patches 1024
    python kernel_bench.py patch_embed --preset so400m --images 64 --max-patches 1024
    python kernel_bench.py patchify --images 64 --height 768 --width 1024 --max-patches 1024

Prints one JSON line per measurement: milliseconds per launch, the
algorithmic TFLOP/s (dense contractions only) and the median SM clock seen
through NVML while the launches ran.  ``gemm --cublas`` adds torch.matmul
(cuBLAS, no epilogue) on the same operands as a library reference point.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from siglip2_b200 import _lib as L  # noqa: E402
from siglip2_b200 import ops  # noqa: E402
from siglip2_b200 import workloads as W  # noqa: E402
from siglip2_b200.clocks import ClockSampler  # noqa: E402

EPIS = {"bias": L.EPI_BIAS, "bias_res": L.EPI_BIAS_RES, "ln": L.EPI_LN, "ln_gelu": L.EPI_LN_GELU,
        "bias_gelu": L.EPI_BIAS_GELU, "lnrs": L.EPI_LN_ROWSUMS, "lnrs_gelu": L.EPI_LN_ROWSUMS_GELU,
        "bias_res_rs": L.EPI_BIAS_RES_ROWSUMS}


_LAST_CLOCK = {}


def _time(fn, reps: int, warmup: int = 3) -> float:
    """Milliseconds per call over ``reps`` back-to-back calls (CUDA events on
    the current stream); the SM clock seen meanwhile goes to ``_LAST_CLOCK``."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device(), period=0.005) as clk:
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
    _LAST_CLOCK.clear()
    _LAST_CLOCK.update(clk.summary())
    return s.elapsed_time(e) / reps


def _clock():
    return {"sm_mhz": _LAST_CLOCK.get("sm_mhz"), "reasons": _LAST_CLOCK.get("reasons")}


def bench_gemm(m, n, k, epi, reps, dtype=torch.bfloat16, warmup=3, cublas=False):
    a = torch.randn(m, k, device="cuda").to(dtype)
    w = (torch.randn(n, k, device="cuda") * 0.02).to(dtype)
    vec = torch.randn(n, device="cuda") * 0.1
    res = torch.randn(m, n, device="cuda").to(dtype) if epi in ("bias_res", "bias_res_rs") else None
    out = torch.empty(m, n, device="cuda", dtype=dtype)
    if epi in ("lnrs", "lnrs_gelu", "bias_res_rs"):
        acc = torch.zeros(m, ops.rowsum_slots(dtype, n), 2, device="cuda") if epi == "bias_res_rs" else None
        rs_in = ops.rowsums_reference(a) if epi != "bias_res_rs" else None
        fn = lambda: ops.gemm_rowsums(a, w, EPIS[epi], bias=vec, res=res, c1=vec, c2=vec, rs_in=rs_in, rs_acc=acc,  # noqa: E731
                                      out=out)
    else:
        fn = lambda: ops.gemm(a, w, EPIS[epi], bias=vec, res=res, c1=vec, c2=vec, out=out)  # noqa: E731
    ms = _time(fn, reps, warmup)
    r = {"kernel": "gemm", "epi": epi, "M": m, "N": n, "K": k, "ms": ms, "tflops": 2 * m * n * k / ms / 1e9,
         **_clock()}
    if cublas:
        wt = w.t()
        ms_c = _time(lambda: torch.matmul(a, wt, out=out), reps, warmup)
        r["cublas"] = {"ms": ms_c, "tflops": 2 * m * n * k / ms_c / 1e9, **_clock()}
    return r


def _shapes(preset, images, max_patches, seed=1337):
    return W.sample_spatial_shapes("area_aspect" if max_patches > 256 else "full", images, max_patches, seed)


def bench_fmha(preset, images, max_patches, reps, dtype=torch.bfloat16, warmup=3):
    D, _, _, H = W.PRESETS[preset]
    hd = D // H
    shapes = _shapes(preset, images, max_patches)
    lens = (shapes[:, 0] * shapes[:, 1]).tolist()
    N = sum(lens)
    qkv = torch.randn(N, 3 * H * hd, device="cuda").to(dtype)  # q | k | v
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device="cuda")
    tiles = ops.attention_tiles(lens).cuda()
    out = torch.empty(N, D, device="cuda", dtype=dtype)
    ms = _time(lambda: ops.fmha_varlen(qkv, cu, tiles, H, hd, out=out), reps, warmup)
    fl = sum(4 * L_ * L_ * D for L_ in lens)
    return {"kernel": "fmha", "preset": preset, "images": images, "tokens": N, "ms": ms, "tflops": fl / ms / 1e9,
            **_clock()}


def bench_gemm_e4m3(m, n, k, epi, reps, warmup=3, cublas=False):
    """The e4m3 GEMM (siglip2_gemm_e4m3, kind::f8f6f4 on SM pairs) against the
    bf16 GEMM of the same shape and epilogue; 2 m n k FLOPs each.  The
    per-row quantisation of A (siglip2_quantize_e4m3) is timed on its own:
    bytes = m k (2 read + 1 written) + 4 m."""
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.03).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    qa, sa = ops.quantize_e4m3(a)
    qw, sw = ops.quantize_e4m3(w)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    r_in = torch.randn(m, n, device="cuda", generator=g).bfloat16() if epi == "bias_res" else None
    code = EPIS[epi]
    fl = 2 * m * n * k
    res = []
    ms = _time(lambda: ops.gemm_e4m3(qa, sa, qw, sw, code, bias, res=r_in, out=out), reps, warmup)
    res.append({"kernel": "gemm_e4m3", "epi": epi, "M": m, "N": n, "K": k, "ms": ms, "tflops": fl / ms / 1e9, **_clock()})
    ms = _time(lambda: ops.gemm(a, w, code, bias=bias, res=r_in, out=out), reps, warmup)
    res.append({"kernel": "gemm_bf16", "epi": epi, "M": m, "N": n, "K": k, "ms": ms, "tflops": fl / ms / 1e9, **_clock()})
    qo = torch.empty(m, k, device="cuda", dtype=torch.float8_e4m3fn)
    so = torch.empty(m, device="cuda")
    ms = _time(lambda: L.call("siglip2_quantize_e4m3", L.DTYPE_BF16, a.data_ptr(), k, m, k, qo.data_ptr(), k,
                              so.data_ptr(), torch.cuda.current_stream().cuda_stream), reps, warmup)
    res.append({"kernel": "quantize_e4m3", "rows": m, "cols": k, "ms": ms, "gbs": (3 * m * k + 4 * m) / ms / 1e6,
                **_clock()})
    if cublas:
        one = torch.ones((), device="cuda")
        ms = _time(lambda: torch._scaled_mm(qa, qw.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16), reps,
                   warmup)
        res.append({"kernel": "torch._scaled_mm (cuBLAS, tensor-wise scales, no epilogue)", "M": m, "N": n, "K": k,
                    "ms": ms, "tflops": fl / ms / 1e9, **_clock()})
    return res


def bench_backward_gemms(m, n, k, reps, warmup=3):
    """dgrad dA = dY W and wgrad dW = dY^T A of y = A W^T (A [m, k], W [n, k])
    on the transposed-operand tensor-core GEMM (siglip2_gemm_t), and the
    GELU-gradient recompute GEMM; algorithmic 2 m n k FLOPs each."""
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.03).bfloat16()
    dy = torch.randn(m, n, device="cuda", generator=g).bfloat16()
    bias = torch.zeros(n, device="cuda")
    out = []
    for name, fn in (("dgrad", lambda: ops.gemm_t(dy, w, False, True)),
                     ("wgrad", lambda: ops.gemm_t(dy, a, True, True)),
                     ("wgrad_splitk", lambda: ops.gemm_t_splitk(dy, a, True)),
                     ("gelu_grad_recompute", lambda: ops.gemm(a, w, L.EPI_BIAS_GELU_GRAD, bias=bias, res=dy))):
        ms = _time(fn, reps, warmup)
        out.append({"kernel": name, "m": m, "n": n, "k": k, "ms": ms, "tflops": 2 * m * n * k / ms / 1e9, **_clock()})
    return out


def bench_layer(preset, images, max_patches, reps):
    D, I, _, H = W.PRESETS[preset]
    N = int((lambda s: (s[:, 0] * s[:, 1]).sum())(_shapes(preset, images, max_patches)))
    out = []
    # the epilogues the forward uses
    for name, n, k, epi in (("qkv", 3 * D, D, "lnrs"), ("out", D, D, "bias_res_rs"), ("fc1", I, D, "lnrs_gelu"),
                            ("fc2", D, I, "bias_res_rs")):
        r = bench_gemm(N, n, k, epi, reps)
        r["name"] = name
        out.append(r)
    out.append(bench_fmha(preset, images, max_patches, reps))
    return out


def bench_patch_embed(preset, images, max_patches, reps, warmup=3):
    """``siglip2_patch_embed`` (patch Linear + antialiased resize of the 16x16
    position table in the epilogue + slot statistics) on the seeded NaFlex
    grids; 2 N 768 D FLOPs per launch (the resize is not counted)."""
    D = W.PRESETS[preset][0]
    shapes = _shapes(preset, images, max_patches)
    lens = (shapes[:, 0] * shapes[:, 1]).tolist()
    N = sum(lens)
    g = torch.Generator(device="cuda").manual_seed(0)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device="cuda")
    hw = shapes.to(torch.int32).flatten().cuda()
    tok = ops.token_image(cu, N)
    patches = (torch.rand(N, 768, device="cuda", generator=g) * 2 - 1).bfloat16()
    w = (torch.randn(D, 768, device="cuda", generator=g) * 0.02).bfloat16()
    bias = torch.randn(D, device="cuda", generator=g) * 0.02
    table = torch.randn(256, D, device="cuda", generator=g) * 0.02
    rs = torch.empty((N, ops.rowsum_slots(torch.bfloat16, D), 2), device="cuda")
    ms = _time(lambda: ops.patch_embed(patches, w, bias, table, hw, cu, tok, rs), reps, warmup)
    return {"kernel": "patch_embed", "preset": preset, "images": images, "tokens": N, "ms": ms,
            "tflops": 2 * N * 768 * D / ms / 1e9, **_clock()}


def bench_patchify(images: int, height: int, width: int, max_patches: int, reps: int, warmup: int = 3,
                   channels_last: bool = True) -> dict:
    """``siglip2_patchify`` on ``images`` random uint8 images of one size
    already on the device (the kernel alone: the grids are computed and the
    metadata uploaded once).  HBM bytes: the uint8 source read once plus the
    bf16 ``pixel_values`` written."""
    import ctypes as ct

    import numpy as np

    from siglip2_b200.image_processor import image_grid
    g = torch.Generator(device="cuda").manual_seed(0)
    shape = (images, height, width, 3) if channels_last else (images, 3, height, width)
    pix = torch.randint(0, 256, shape, dtype=torch.uint8, device="cuda", generator=g)
    gh, gw = image_grid(height, width, 16, max_patches)
    src = np.tile(np.array([height, width], dtype=np.int32), images)
    grid = np.tile(np.array([gh, gw], dtype=np.int32), images)
    offs = np.arange(images, dtype=np.int64) * (height * width * 3)
    meta = torch.from_numpy(np.concatenate([offs.view(np.int32), src, grid])).cuda()
    out = torch.empty((images, max_patches, 768), dtype=torch.bfloat16, device="cuda")
    mask = torch.empty((images, max_patches), dtype=torch.int32, device="cuda")
    mean = np.full(3, 127.5, dtype=np.float32)
    std = np.full(3, 127.5, dtype=np.float32)
    stream = torch.cuda.current_stream().cuda_stream

    def run():
        L.call("siglip2_patchify", L.DTYPE_BF16, pix.data_ptr(), meta.data_ptr(), src.ctypes.data,
               meta[2 * images:].data_ptr(), grid.ctypes.data, meta[4 * images:].data_ptr(), images, 3, 16,
               int(channels_last), mean.ctypes.data, std.ctypes.data, max_patches, out.data_ptr(),
               mask.data_ptr(), ct.c_void_p(stream))

    ms = _time(run, reps, warmup)
    nbytes = pix.numel() + out.numel() * 2 + mask.numel() * 4
    return {"kernel": "patchify", "images": images, "src": [height, width], "grid": [gh, gw],
            "max_patches": max_patches, "resize": (gh * 16, gw * 16) != (height, width), "ms": ms,
            "gbs": nbytes / ms / 1e6, **_LAST_CLOCK}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=39178)
    g.add_argument("--n", type=int, default=4304)
    g.add_argument("--k", type=int, default=1152)
    g.add_argument("--epi", default="ln_gelu", help="one of %s, or several separated by commas" % ",".join(sorted(EPIS)))
    g.add_argument("--cublas", action="store_true", help="also time torch.matmul (cuBLAS) on the same operands")
    g.add_argument("--reps", type=int, default=20)
    g.add_argument("--warmup", type=int, default=3)
    e8 = sub.add_parser("gemm_e4m3")
    e8.add_argument("--m", type=int, default=39178)
    e8.add_argument("--n", type=int, default=4304)
    e8.add_argument("--k", type=int, default=1152)
    e8.add_argument("--epi", default="bias_gelu", help="bias, bias_res or bias_gelu")
    e8.add_argument("--cublas", action="store_true", help="also time torch._scaled_mm on the same codes")
    e8.add_argument("--reps", type=int, default=20)
    e8.add_argument("--warmup", type=int, default=3)
    e8.add_argument("--variant", type=int, default=0)
    f = sub.add_parser("fmha")
    f.add_argument("--preset", default="so400m")
    f.add_argument("--images", type=int, default=64)
    f.add_argument("--max-patches", type=int, default=1024)
    f.add_argument("--reps", type=int, default=20)
    f.add_argument("--warmup", type=int, default=3)
    y = sub.add_parser("layer")
    y.add_argument("--preset", default="so400m")
    y.add_argument("--images", type=int, default=64)
    y.add_argument("--max-patches", type=int, default=1024)
    y.add_argument("--reps", type=int, default=20)
    for sp in (g, f, y):
        sp.add_argument("--variant", type=int, default=0, help="GEMM kernel: 0 auto, 1 one SM, 2 SM pairs")
    f.add_argument("--fmha-variant", type=int, default=0,
                   help="attention kernel: 0 auto, 1 one query tile per CTA, 2 query-tile pairs")
    bw = sub.add_parser("bwd")
    bw.add_argument("--m", type=int, default=39178)
    bw.add_argument("--n", type=int, default=4304)
    bw.add_argument("--k", type=int, default=1152)
    bw.add_argument("--reps", type=int, default=20)
    bw.add_argument("--variant", type=int, default=0)
    pe = sub.add_parser("patch_embed")
    pe.add_argument("--preset", default="so400m")
    pe.add_argument("--images", type=int, default=64)
    pe.add_argument("--max-patches", type=int, default=1024)
    pe.add_argument("--reps", type=int, default=20)
    pe.add_argument("--warmup", type=int, default=3)
    pe.add_argument("--variant", type=int, default=0)
    pz = sub.add_parser("patchify")
    pz.add_argument("--images", type=int, default=64)
    pz.add_argument("--height", type=int, default=512)
    pz.add_argument("--width", type=int, default=512)
    pz.add_argument("--max-patches", type=int, default=1024)
    pz.add_argument("--channels-first", action="store_true")
    pz.add_argument("--reps", type=int, default=20)
    pz.add_argument("--warmup", type=int, default=3)
    pz.add_argument("--variant", type=int, default=0)
    a = ap.parse_args()
    L.check(L.load().siglip2_set_gemm_variant(a.variant))
    if a.cmd == "gemm":
        for epi in a.epi.split(","):
            if epi not in EPIS:
                raise SystemExit(f"unknown epilogue {epi!r}")
            print(json.dumps(bench_gemm(a.m, a.n, a.k, epi, a.reps, warmup=a.warmup, cublas=a.cublas)))
    elif a.cmd == "gemm_e4m3":
        for r in bench_gemm_e4m3(a.m, a.n, a.k, a.epi, a.reps, a.warmup, a.cublas):
            print(json.dumps(r))
    elif a.cmd == "patch_embed":
        print(json.dumps(bench_patch_embed(a.preset, a.images, a.max_patches, a.reps, a.warmup)))
    elif a.cmd == "patchify":
        print(json.dumps(bench_patchify(a.images, a.height, a.width, a.max_patches, a.reps, a.warmup,
                                        channels_last=not a.channels_first)))
    elif a.cmd == "bwd":
        for r in bench_backward_gemms(a.m, a.n, a.k, a.reps):
            print(json.dumps(r))
    elif a.cmd == "fmha":
        L.check(L.load().siglip2_set_fmha_variant(a.fmha_variant))
        r = bench_fmha(a.preset, a.images, a.max_patches, a.reps, warmup=a.warmup)
        r["fmha_variant"] = a.fmha_variant
        print(json.dumps(r))
    else:
        for r in bench_layer(a.preset, a.images, a.max_patches, a.reps):
            print(json.dumps(r))


if __name__ == "__main__":
    main()
