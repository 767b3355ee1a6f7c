"""Fixed-input profiling harness (the role of the reference's
scripts/profile_lsq_inference.py with ``--reuse-single-batch``), shaped for
Nsight Compute: every sub-command builds its inputs once, runs a few
warm-up launches, then ``--iters`` timed launches with CUDA events, and
prints one JSON line. To capture individual launches, run the same command
(after it has exited 0 on its own) under
``ncu --clock-control none --metrics gpu__time_duration.sum -k regex:w4a8
-s <warmup> -c <n>``; without ``--clock-control none`` ncu locks the GPU
clocks, a setting that outlasts the process. A fuller capture (``--set
full`` or several sections) should cover one kernel and one to three
launches of a small case.

  python -m quant_pipeline.runtime.profile_cli conv  --n 256 --h 56 --c 64 --o 64 --k 3 --stride 1
  python -m quant_pipeline.runtime.profile_cli gemm  --m 4096 --n 8192 --k 8192
  python -m quant_pipeline.runtime.profile_cli resnet --batch 256 [--arch resnet18] [--eager]
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

import int4_int8_ext as ext  # noqa: E402


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / max(iters, 1)


def conv(a) -> dict:
    """One conv launch. --ho overrides the output size (the space-to-depth
    stem pads 2 top/left, 1 bottom/right); --out f32 writes float32 (stem);
    --residual adds a float32 identity and a float32 side output (the last
    conv of a residual block)."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    ho = a.ho if a.ho else (a.h + 2 * a.pad - a.k) // a.stride + 1
    x = torch.randint(0, 128, (a.n, a.h, a.h, a.c), dtype=torch.int8, device=dev, generator=g)
    ktot = a.k * a.k * a.c
    wb = ktot // 2 if a.wbits == 4 else ktot
    ldw = -(-wb // 16) * 16
    w = torch.randint(0, 256 if a.wbits == 4 else 127, (a.o, ldw), dtype=torch.uint8, device=dev, generator=g)
    alpha = torch.rand(a.o, device=dev, generator=g) * 1e-3
    beta = torch.randn(a.o, device=dev, generator=g) * 1e-2
    kind = ext.OUT_F32 if a.out == "f32" else ext.OUT_S8
    out = torch.empty((a.n, ho, ho, a.o), dtype=torch.float32 if a.out == "f32" else torch.int8, device=dev)
    res = aux = None
    if a.residual:
        res = torch.randn((a.n, ho, ho, a.o), device=dev, generator=g)
        aux = torch.empty_like(res)
    if a.pool:
        ph = (ho - 1) // 2 + 1
        out = torch.empty((a.n, ph, ph, a.o), dtype=out.dtype, device=dev)
        aux = torch.empty((a.n, ph, ph, a.o), dtype=torch.float32, device=dev)
    geom = ext.ConvGeom(a.n, a.h, a.h, a.c, a.k, a.k, a.stride, a.pad, a.pad, ho, ho, a.o, ext.LAYOUT_NHWC, a.o,
                        int(a.pool))
    epi = ext.make_epilogue(kind, alpha=alpha, beta=beta, relu=True, out_scale=0.05, qn=0, qp=127,
                            residual=res, res_ld=a.o, aux=aux, aux_ld=a.o)
    wkind = ext.W_INT4 if a.wbits == 4 else ext.W_INT8
    ms = _time(lambda: ext.conv2d_nhwc(x, w, wkind, geom, epi, out), a.iters, a.warmup)
    ops = 2.0 * a.n * ho * ho * a.o * ktot
    nbytes = x.numel() + out.numel() * out.element_size() + a.o * wb
    if a.residual:
        nbytes += 2 * res.numel() * 4
    return {"op": "conv", "shape": vars(a), "ms": ms, "tops": ops / ms / 1e9, "gbs": nbytes / ms / 1e6,
            "alg_ops": ops, "alg_bytes": nbytes}


def gemm(a) -> dict:
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randint(-128, 128, (a.m, a.k), dtype=torch.int8, device=dev, generator=g)
    if a.wbits == 4:
        w = torch.randint(0, 256, (a.n, a.k // 2), dtype=torch.uint8, device=dev, generator=g)
    else:
        w = torch.randint(-128, 128, (a.n, a.k), dtype=torch.int8, device=dev, generator=g)
    out = torch.empty((a.m, a.n), dtype=torch.int32, device=dev)
    epi = ext.make_epilogue(ext.OUT_S32)
    wkind = ext.W_INT4 if a.wbits == 4 else ext.W_INT8
    ms = _time(lambda: ext.gemm(x, w, wkind, a.k, epi, out), a.iters, a.warmup)
    ops = 2.0 * a.m * a.n * a.k
    nbytes = x.numel() + w.numel() + out.numel() * 4
    return {"op": "gemm", "shape": vars(a), "ms": ms, "tops": ops / ms / 1e9, "gbs": nbytes / ms / 1e6}


def resnet(a) -> dict:
    from quant_pipeline.runtime.engine import W4A8ResNetEngine
    from quant_pipeline.runtime.lsq_resnet import build_lsq_resnet, synthetic_images

    dev = torch.device("cuda")
    eng = W4A8ResNetEngine(build_lsq_resnet(a.arch), a.batch, device=dev, use_graph=not a.eager)
    eng.images.copy_(synthetic_images(a.batch).to(dev))
    ms = _time(lambda: eng.forward(), a.iters, a.warmup)
    eng.release()
    return {"op": "resnet", "shape": vars(a), "ms": ms, "images_per_s": a.batch / ms * 1e3}


def main() -> None:
    p = argparse.ArgumentParser()
    sub = p.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("conv")
    for k, v in dict(n=256, h=56, c=64, o=64, k=3, stride=1, pad=1, ho=0, wbits=4).items():
        c.add_argument(f"--{k}", type=int, default=v)
    c.add_argument("--out", choices=["s8", "f32"], default="s8")
    c.add_argument("--residual", action="store_true")
    c.add_argument("--pool", action="store_true", help="fuse the 3x3/s2/p1 max pool (float32 side output)")
    gm = sub.add_parser("gemm")
    for k, v in dict(m=4096, n=8192, k=8192, wbits=4).items():
        gm.add_argument(f"--{k}", type=int, default=v)
    r = sub.add_parser("resnet")
    r.add_argument("--batch", type=int, default=256)
    r.add_argument("--arch", default="resnet18")
    r.add_argument("--eager", action="store_true")
    for sp in (c, gm, r):
        sp.add_argument("--iters", type=int, default=3)
        sp.add_argument("--warmup", type=int, default=2)
    a = p.parse_args()
    res = {"conv": conv, "gemm": gemm, "resnet": resnet}[a.cmd](a)
    if ext.device_error():
        raise RuntimeError("device-side wait timeout recorded")
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
