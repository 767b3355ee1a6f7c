#!/usr/bin/env python
"""Benchmark: W4A8 LSQ-converted ResNet-18 inference, batch 256 per GPU.

One step = one forward of the converted ResNet-18 over a batch of 256
synthetic 224x224 images (N(0,1), seeded per rank) on each GPU, plus the
NCCL all-gather of the logits when N > 1 (batch sharded data-parallel,
weak scaling). Prints one JSON line (rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the CPU oracle (a numpy port of the reference's
integer path) on the host cores; the reference's own code is Python over a
CUDA extension with no sm_100 path and is not installed on the GPU box.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "lsq-lowbit-optimization_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "W4A8 ResNet-18 images/s (bs256) @1/2/4/8 B200; GEMM int8 TOPS vs peak"
WORKLOAD = "LSQ-converted ResNet-18 W4A8 inference (int8 first conv and fc), 224x224"
BATCH = 256
# Nominal dense int8 tensor peak of one B200, for context only.
INT8_NOMINAL_TOPS = 4500.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=BATCH, help="images per GPU")
    p.add_argument("--arch", default="resnet18", choices=["resnet18", "resnet50"])
    p.add_argument("--no-extras", action="store_true", help="skip roofline/GEMM/CPU side measurements")
    return p.parse_args()


def measured_peaks() -> dict:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.tmp = None

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.index)], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: the timed region (a few hundred ms at
        # the default step count) begins only once the first sample is written.
        t0 = time.time()
        while time.time() - t0 < 5.0 and self.proc.poll() is None:
            try:
                if Path(self.tmp.name).read_text().count("\n") >= 1:
                    break
            except OSError:
                pass
            time.sleep(0.02)
        return self

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.tmp.flush()
        rows = []
        for line in Path(self.tmp.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.tmp.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        load = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def time_events(fn, iters: int, warmup: int = 2) -> float:
    """Average ms per call of ``fn`` with CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def cpu_oracle_rate(model, images: int, seed: int = 7) -> dict:
    """Images/s of the CPU oracle (numpy integer port) on this host."""
    from oracle import resnet_oracle as ro
    from quant_pipeline.runtime.lsq_resnet import synthetic_images

    x = synthetic_images(images, seed=seed).numpy()
    t0 = time.perf_counter()
    ro.resnet_forward(model, x)
    dt = time.perf_counter() - t0
    return {"value": images / dt, "unit": "images/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{images} images per call, numpy integer oracle (exact float32/float64 BLAS, "
                      f"{os.cpu_count()} host threads)", "seconds": round(dt, 2)}


def cpu_fakequant_rate(model, images: int, seed: int = 7) -> dict:
    """The reference's CPU path for the whole network: the LSQ fake-quant
    float32 forward (clamp(round(x/s))*s on activations and weights, float
    conv / linear, BatchNorm, ReLU, pooling in torch) on the host cores,
    after one warm-up call."""
    from quant_pipeline.runtime.lsq_resnet import synthetic_images

    torch.set_num_threads(os.cpu_count())
    x = synthetic_images(images, seed=seed)
    with torch.no_grad():
        model(x[:2])
        t0 = time.perf_counter()
        model(x)
        dt = time.perf_counter() - t0
    return {"value": images / dt, "unit": "images/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"one batch of {images} images: LSQ fake-quant float32 forward in torch on the host "
                      f"(the LSQ native model of the reference's flow), {torch.get_num_threads()} threads",
            "seconds": round(dt, 2)}


def cpu_baseline_leg(model, images: torch.Tensor, logits: torch.Tensor) -> tuple:
    """The CPU leg: times the reference's CPU path (LSQ fake-quant forward)
    on a bounded sample, and checks the engine's logits for the whole timed
    batch against the integer oracle (the checker; exact by construction).
    Returns (cpu_baseline, parity)."""
    import numpy as np
    from oracle import resnet_oracle as ro

    base = cpu_fakequant_rate(model, int(images.shape[0]))
    t0 = time.perf_counter()
    want = ro.resnet_forward(model, images.numpy())
    dt = time.perf_counter() - t0
    got = logits.cpu().numpy()
    parity = {"images": int(got.shape[0]), "checker": "CPU integer oracle (oracle/resnet_oracle.py)",
              "bit_exact": bool(np.array_equal(got, want)), "rel_err": float(ro.rel_err(got, want)),
              "top1_agreement": float(ro.top1_agreement(got, want)), "gate": "rel_err <= 1e-3, top-1 >= 0.999"}
    parity["pass"] = parity["rel_err"] <= 1e-3 and parity["top1_agreement"] >= 0.999
    base["oracle_port_images_per_s"] = round(got.shape[0] / dt, 2)
    return base, parity


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    from quant_pipeline.runtime.lsq_resnet import build_lsq_resnet

    torch.set_num_threads(os.cpu_count())
    model = build_lsq_resnet(args.arch, seed=0)
    per_step = 2 if args.steps + args.warmup > 50 else 8
    for _ in range(args.warmup):
        cpu_oracle_rate(model, per_step)
    t0 = time.perf_counter()
    for i in range(args.steps):
        cpu_oracle_rate(model, per_step, seed=100 + i)
    dt = time.perf_counter() - t0
    value = per_step * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch_per_step": per_step, "arch": args.arch,
                   "note": "CPU oracle (numpy port of the reference's integer path), bounded sample per step"},
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{per_step} images per step x {args.steps} steps"},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def gemm_tops(device) -> dict:
    """Large W4A8 GEMM (M=4096, N=K=8192, int32 out) on the tcgen05 kernel."""
    import int4_int8_ext as ext

    m = n = k = 8192
    m = 4096
    gen = torch.Generator(device=device).manual_seed(0)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=device, generator=gen)
    w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=device, generator=gen)
    c = torch.empty((m, n), dtype=torch.int32, device=device)
    epi = ext.make_epilogue(ext.OUT_S32)
    ms = time_events(lambda: ext.gemm(a, w, ext.W_INT4, k, epi, c), iters=20, warmup=3)
    tops = 2.0 * m * n * k / (ms * 1e-3) / 1e12
    return {"shape_mnk": [m, n, k], "ms": round(ms, 4), "tops": round(tops, 1)}


def small_m_gemm_hbm(device, hbm_gbs: float) -> list:
    """Memory-bound W4A8 GEMMs (N = K = 8192, packed weights 32 MiB): M = 1
    on the CUDA-core GEMV, M = 32 on swapped-operand split-K. L2 (126 MB) is
    flushed before every timed call by reading a 256 MiB buffer (clean lines,
    so no write-back lands inside the timed call) and the weights stream from
    HBM; only the GEMM itself is inside the events."""
    import int4_int8_ext as ext

    n = k = 8192
    gen = torch.Generator(device=device).manual_seed(1)
    w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=device, generator=gen)
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=device)
    out = []
    for m in (1, 32):
        a = torch.randint(-128, 128, (m, k), dtype=torch.int8, device=device, generator=gen)
        c = torch.empty((m, n), dtype=torch.int32, device=device)
        epi = ext.make_epilogue(ext.OUT_S32)
        for _ in range(3):
            ext.gemm(a, w, ext.W_INT4, k, epi, c)
        total = 0.0
        iters = 20
        for _ in range(iters):
            flush_sum = flush.max()  # noqa: F841 (read-only L2 flush)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            ext.gemm(a, w, ext.W_INT4, k, epi, c)
            e1.record()
            torch.cuda.synchronize()
            total += e0.elapsed_time(e1)
        ms = total / iters
        nbytes = w.numel() + a.numel() + c.numel() * 4
        gbs = nbytes / (ms * 1e-3) / 1e9
        # The same calls replayed from a CUDA graph, each after the flush: the
        # device time a GEMM adds to a stream of kernels, without the per-call
        # launch and event overhead (an empty kernel timed alone with events
        # measures about 6 us here). Graph of `reps` x (flush, GEMM) minus a
        # graph of `reps` x flush, best of three replays each.
        reps = 20
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            ext.gemm(a, w, ext.W_INT4, k, epi, c)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g_both, g_flush = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_both):
            for _ in range(reps):
                flush.max()
                ext.gemm(a, w, ext.W_INT4, k, epi, c)
        with torch.cuda.graph(g_flush):
            for _ in range(reps):
                flush.max()

        def replay_ms(graph):
            best = float("inf")
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                e1.record()
                torch.cuda.synchronize()
                best = min(best, e0.elapsed_time(e1))
            return best

        ms_graph = (replay_ms(g_both) - replay_ms(g_flush)) / reps
        del g_both, g_flush
        gbs_graph = nbytes / (ms_graph * 1e-3) / 1e9 if ms_graph > 0 else None
        out.append({"shape_mnk": [m, n, k], "path": "gemv" if m <= 8 else "split-k",
                    "us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm_gbs, 4),
                    "us_in_graph": round(ms_graph * 1e3, 2),
                    "hbm_frac_in_graph": round(gbs_graph / hbm_gbs, 4) if gbs_graph else None,
                    "l2": "flushed before each call (256 MiB read)",
                    "timing": "us: per call between CUDA events; us_in_graph: per call inside a CUDA graph "
                              "of (flush, GEMM) pairs minus a graph of flushes"})
    return out


def int8_library_marker(device) -> dict:
    """torch._int_mm (cuBLASLt int8, int32 out) at 8192^3: an achievable-library
    marker beside the nominal dense int8 peak, not a roofline denominator."""
    n = 8192
    gen = torch.Generator(device=device).manual_seed(2)
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=device, generator=gen)
    b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=device, generator=gen)
    try:
        ms = time_events(lambda: torch._int_mm(a, b), iters=10, warmup=3)
    except RuntimeError as exc:  # no int8 cuBLASLt kernel for this build
        return {"unavailable": str(exc).splitlines()[0][:120]}
    return {"op": "torch._int_mm 8192^3", "ms": round(ms, 4), "tops": round(2.0 * n ** 3 / (ms * 1e-3) / 1e12, 1)}


def fc_cfg0(device, hbm_gbs: float) -> dict:
    """ResNet-18 classifier shape (X int8 [256, 512] x W int4 [1000, 512],
    per-channel scale + bias, float32 out): latency and GB/s."""
    import int4_int8_ext as ext

    gen = torch.Generator(device=device).manual_seed(0)
    x = torch.randint(-128, 128, (256, 512), dtype=torch.int8, device=device, generator=gen)
    w = torch.randint(0, 256, (1000, 256), dtype=torch.uint8, device=device, generator=gen)
    alpha = torch.rand(1000, device=device, generator=gen) * 1e-4
    bias = torch.randn(1000, device=device, generator=gen) * 0.01
    out = torch.empty((256, 1000), dtype=torch.float32, device=device)
    epi = ext.make_epilogue(ext.OUT_F32, alpha=alpha, beta=bias)
    ext.gemm(x, w, ext.W_INT4, 512, epi, out)
    torch.cuda.synchronize()
    reps = 20  # CUDA-graph replay of 20 calls: device time without host launch overhead
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            ext.gemm(x, w, ext.W_INT4, 512, epi, out)
    ms = time_events(lambda: g.replay(), iters=10, warmup=2) / reps
    del g
    nbytes = x.numel() + w.numel() + out.numel() * 4 + 8 * 1000
    return {"shape_mnk": [256, 1000, 512], "us": round(ms * 1e3, 2), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm_gbs, 4),
            "timing": "CUDA-graph replay of 20 calls; 1.4 MB of work, inputs L2-resident across calls"}


def gemm_sweep(device, int8_peak: float, hbm_gbs: float) -> list:
    """Config 1: W4A8 GEMM (int32 out) over M in {1, 32, 256, 4096} x N = K in
    {1024, 4096, 8192}, per call with CUDA events after a read-only 256 MiB
    L2 flush; TOPS against the int8 peak and GB/s against HBM."""
    import int4_int8_ext as ext

    gen = torch.Generator(device=device).manual_seed(3)
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=device)
    out = []
    for nk in (1024, 4096, 8192):
        w = torch.randint(0, 256, (nk, nk // 2), dtype=torch.uint8, device=device, generator=gen)
        for m in (1, 32, 256, 4096):
            a = torch.randint(-128, 128, (m, nk), dtype=torch.int8, device=device, generator=gen)
            c = torch.empty((m, nk), dtype=torch.int32, device=device)
            epi = ext.make_epilogue(ext.OUT_S32)
            for _ in range(3):
                ext.gemm(a, w, ext.W_INT4, nk, epi, c)
            total, iters = 0.0, 10
            for _ in range(iters):
                flush.max()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                ext.gemm(a, w, ext.W_INT4, nk, epi, c)
                e1.record()
                torch.cuda.synchronize()
                total += e0.elapsed_time(e1)
            ms = total / iters
            tops = 2.0 * m * nk * nk / (ms * 1e-3) / 1e12
            gbs = (a.numel() + w.numel() + c.numel() * 4) / (ms * 1e-3) / 1e9
            out.append({"mnk": [m, nk, nk], "us": round(ms * 1e3, 2), "tops": round(tops, 1),
                        "tensor_frac": round(tops / int8_peak, 4), "gbs": round(gbs, 1),
                        "hbm_frac": round(gbs / hbm_gbs, 4)})
    return out


def conv_cfg2(device, int8_peak: float, hbm_gbs: float) -> list:
    """Config 2 at full size: NHWC int8 [256, 56, 56, 64] post-ReLU codes, int4
    weights, per-channel weight scale, bias, ReLU and int8 requant (scale
    0.05) fused; the stride-2 64->128 variant and its 1x1 stride-2 shortcut
    (float32 identity out). Per launch with CUDA events (inputs and outputs
    exceed L2 together)."""
    import int4_int8_ext as ext

    gen = torch.Generator(device=device).manual_seed(4)
    n, h, w, c = 256, 56, 56, 64
    x = torch.randint(0, 128, (n, h, w, c), dtype=torch.int8, device=device, generator=gen)
    out = []
    for name, o, k, s, pad, kind in (("3x3s1", 64, 3, 1, 1, ext.OUT_S8), ("3x3s2", 128, 3, 2, 1, ext.OUT_S8),
                                     ("1x1s2", 128, 1, 2, 0, ext.OUT_F32)):
        ho = (h + 2 * pad - k) // s + 1
        wt = torch.randint(0, 256, (o, (k * k * c) // 2), dtype=torch.uint8, device=device, generator=gen)
        alpha = torch.rand(o, device=device, generator=gen) * 9e-3 * 0.05 + 1e-3 * 0.05
        bias = torch.randn(o, device=device, generator=gen) * 0.01
        y = torch.empty((n, ho, ho, o), dtype=torch.int8 if kind == ext.OUT_S8 else torch.float32, device=device)
        epi = (ext.make_epilogue(kind, alpha=alpha, beta=bias, relu=True, out_scale=0.05, qn=0, qp=127)
               if kind == ext.OUT_S8 else ext.make_epilogue(kind, alpha=alpha, beta=bias))
        geom = ext.ConvGeom(n, h, w, c, k, k, s, pad, pad, ho, ho, o, ext.LAYOUT_NHWC, o)
        ms = time_events(lambda: ext.conv2d_nhwc(x, wt, ext.W_INT4, geom, epi, y), iters=20, warmup=3)
        ops = 2.0 * n * ho * ho * o * c * k * k
        nbytes = x.numel() + y.numel() * y.element_size() + wt.numel() + 8 * o
        tops, gbs = ops / (ms * 1e-3) / 1e12, nbytes / (ms * 1e-3) / 1e9
        out.append({"conv": name, "ms": round(ms, 4), "tops": round(tops, 1),
                    "tensor_frac": round(tops / int8_peak, 4), "gbs": round(gbs, 1),
                    "hbm_frac": round(gbs / hbm_gbs, 4)})
    return out


def cpu_cfg012() -> dict:
    """The reference's CPU integer path for configs 0-2, timed on the host
    cores with torch: its own check pattern A.int32 @ unpack(Bp).int32.T
    (benchmarks/benchmark_inference.py:67-76) for the fc layer and a GEMM
    sample, and quantised unfold + the same int32 matmul for the conv
    (quant_pipeline/ops/int4_conv2d.py:171-191), on bounded samples."""
    import torch.nn.functional as F
    from quant_pipeline.quantization.int4_pack import unpack_int4_weights

    torch.set_num_threads(os.cpu_count())
    gen = torch.Generator().manual_seed(5)

    def best(fn, reps=3):
        fn()
        t = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            t.append(time.perf_counter() - t0)
        return min(t)

    res = {"cores": torch.get_num_threads()}
    x = torch.randint(-128, 128, (256, 512), dtype=torch.int8, generator=gen)
    wp = torch.randint(0, 256, (1000, 256), dtype=torch.uint8, generator=gen)
    dt = best(lambda: x.to(torch.int32) @ unpack_int4_weights(wp).to(torch.int32).t())
    res["cfg0_fc"] = {"mnk": [256, 1000, 512], "us": round(dt * 1e6, 1), "gops": round(2 * 256 * 1000 * 512 / dt / 1e9, 2)}
    m, nk = 32, 4096
    a = torch.randint(-128, 128, (m, nk), dtype=torch.int8, generator=gen)
    wp = torch.randint(0, 256, (nk, nk // 2), dtype=torch.uint8, generator=gen)
    dt = best(lambda: a.to(torch.int32) @ unpack_int4_weights(wp).to(torch.int32).t())
    res["cfg1_gemm_sample"] = {"mnk": [m, nk, nk], "us": round(dt * 1e6, 1), "gops": round(2 * m * nk * nk / dt / 1e9, 2)}
    imgs = 4
    xq = torch.randint(0, 128, (imgs, 64, 56, 56), dtype=torch.int8, generator=gen)
    wq = torch.randint(0, 256, (64, 288), dtype=torch.uint8, generator=gen)

    def conv():
        cols = F.unfold(xq.to(torch.float32), 3, padding=1).transpose(1, 2).reshape(-1, 576).to(torch.int32)
        return cols @ unpack_int4_weights(wq).to(torch.int32).t()

    dt = best(conv, reps=2)
    res["cfg2_conv3x3_sample"] = {"images": imgs, "shape": "[n,56,56,64] 3x3 s1 64->64", "ms": round(dt * 1e3, 1),
                                  "images_per_s": round(imgs / dt, 2),
                                  "gops": round(2 * imgs * 56 * 56 * 64 * 576 / dt / 1e9, 2)}
    res["note"] = "reported CPU baselines (unpacked int32 torch matmul, not BLAS), not optimisation targets"
    return res


def resnet50_rate(device, batch: int) -> dict:
    """Config 4 on one GPU: the LSQ-converted ResNet-50 W4A8 engine at the
    per-GPU batch (CUDA-graph replay, CUDA events), beside the FP16 cuDNN
    torchvision ResNet-50."""
    from quant_pipeline.runtime.engine import W4A8ResNetEngine
    from quant_pipeline.runtime.lsq_resnet import build_lsq_resnet, synthetic_images

    model = build_lsq_resnet("resnet50", seed=0)
    eng = W4A8ResNetEngine(model, batch, device=device, use_graph=True)
    eng.forward(synthetic_images(batch, seed=1).to(device))
    ms = time_events(lambda: eng.forward(), iters=30, warmup=5)
    launches = eng.launches
    eng.release()
    fp16 = fp16_cudnn_rate(device, batch, "resnet50")
    return {"value": batch / (ms * 1e-3), "unit": "images/s", "ms_per_batch": round(ms, 4), "batch": batch,
            "launches_per_batch": launches, "fp16_cudnn": round(fp16["value"], 1),
            "w4a8_speedup": round(batch / (ms * 1e-3) / fp16["value"], 3)}


def fp16_cudnn_rate(device, batch: int, arch: str) -> dict:
    """The same network in FP16 through torchvision + cuDNN (channels_last,
    cudnn.benchmark, CUDA graph): the library path the W4A8 model must beat."""
    import torchvision

    torch.backends.cudnn.benchmark = True
    net = getattr(torchvision.models, arch)(weights=None).to(device).half().eval()
    net = net.to(memory_format=torch.channels_last)
    x = torch.randn((batch, 3, 224, 224), device=device, dtype=torch.float16).to(memory_format=torch.channels_last)
    with torch.no_grad():
        for _ in range(3):
            net(x)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            net(x)
        torch.cuda.current_stream(device).wait_stream(s)
        with torch.cuda.graph(g):
            net(x)
        ms = time_events(g.replay, iters=30, warmup=3)
    del g
    return {"value": batch / (ms * 1e-3), "unit": "images/s", "ms_per_batch": round(ms, 4),
            "config": f"torchvision {arch}, fp16, channels_last, cudnn.benchmark, CUDA graph, bs{batch}"}


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import int4_int8_ext as ext
    from quant_pipeline.runtime.engine import W4A8ResNetEngine
    from quant_pipeline.runtime.lsq_resnet import build_lsq_resnet, synthetic_images

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = torch.distributed if world > 1 else None
    B = args.batch
    model = build_lsq_resnet(args.arch, seed=0)
    engine = W4A8ResNetEngine(model, B, device=device, use_graph=True)
    host_images = synthetic_images(B, seed=1000 + rank).pin_memory()
    dev_images = host_images.to(device)
    classes = engine.logits.shape[1]
    gathered = torch.empty((B * world, classes), dtype=torch.float32, device=device) if world > 1 else None
    host_logits = torch.empty((B, classes), dtype=torch.float32).pin_memory()
    engine.forward(dev_images)  # builds the CUDA graph
    torch.cuda.synchronize()

    from quant_pipeline.runtime.dp import gather_logits

    def step():
        logits = engine.forward()
        if world > 1:
            gather_logits(logits, gathered)

    post = (lambda logits: gather_logits(logits, gathered)) if world > 1 else None
    copy_stream = torch.cuda.Stream(device)
    outs = [torch.empty((B, classes), dtype=torch.float32).pin_memory() for _ in range(2)]

    def run_e2e(steps: int):
        """Public serving API over host buffers: every step uploads its
        pinned fp32 images (overlapped with the previous batch's compute on
        a copy stream), runs the forward and reads the logits back."""
        engine.infer_host([host_images] * steps, out=[outs[i % 2] for i in range(steps)],
                          copy_stream=copy_stream, post=post)

    def timed(fn, steps: int, warm=None) -> float:
        if warm is not None:
            warm()
        else:
            for _ in range(args.warmup):
                fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        if warm is not None:
            fn(steps)
        else:
            for _ in range(steps):
                fn()
        e.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([s.elapsed_time(e)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    engine.images.copy_(dev_images)
    sampler = ClockSampler(local_rank).start() if rank == 0 else None
    total_ms = timed(step, args.steps)
    clocks = sampler.stop() if sampler else None
    e2e_ms = timed(run_e2e, args.steps, warm=lambda: run_e2e(args.warmup))
    if ext.device_error():
        raise RuntimeError("a kernel recorded a device-side wait timeout")

    line = None
    if rank == 0:
        ms_step = total_ms / args.steps
        value = B * world / (ms_step * 1e-3)
        peaks = measured_peaks()
        int8_peak = 2.0 * peaks["bf16_tflops"]
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "arch": args.arch, "global_batch": B * world, "batch_per_gpu": B,
                       "seq_len": None, "parallelism": f"dp{world}",
                       "l2": "no flush: each step streams inputs and activations far larger than L2 "
                             "(images 154 MB, pooled stem outputs 256 MB)",
                       "timing": "CUDA graph replay of the whole forward (+ NCCL all-gather of logits when N>1)"},
            "gpu_launches": engine.launches * args.steps,
            "e2e": {"value": B * world / (e2e_ms / args.steps * 1e-3), "unit": "images/s",
                    "h2d_bytes_per_step": host_images.numel() * 4, "d2h_bytes_per_step": host_logits.numel() * 4,
                    "api": "W4A8ResNetEngine.infer_host (pinned host images in, host logits out; upload of "
                           "batch i+1 overlapped with batch i on a copy stream)"},
            "clocks": clocks,
        }
        if not args.no_extras and world == 1:
            prof = engine.profile_steps(iters=5)
            convs = [p for p in prof if p["ops"] > 0]
            top = max(convs, key=lambda p: p["ms"])
            tot = sum(p["ms"] for p in prof)
            tflops = top["ops"] / (top["ms"] * 1e-3) / 1e12
            gbs = top["bytes"] / (top["ms"] * 1e-3) / 1e9
            t_frac, h_frac = tflops / int8_peak, gbs / peaks["hbm_gbs"]
            traffic = None
            tf = ROOT / "profiles" / "traffic.json"
            if tf.exists():
                traffic = json.loads(tf.read_text()).get(top["name"])
            line["roofline"] = {
                "kernel": f"w4a8_mma_kernel ({top['name']})", "bound": "tensor" if t_frac >= h_frac else "hbm",
                "achieved": round(tflops if t_frac >= h_frac else gbs, 2),
                "peak": round(int8_peak if t_frac >= h_frac else peaks["hbm_gbs"], 1),
                "unit": "TFLOP/s" if t_frac >= h_frac else "GB/s",
                "frac": round(max(t_frac, h_frac), 4), "traffic": traffic,
                "peak_source": f"{peaks['source']}: int8 = 2 x measured bf16 {peaks['bf16_tflops']} TF/s; "
                               f"HBM {peaks['hbm_gbs']} GB/s",
                "tensor_frac": round(t_frac, 4), "hbm_frac": round(h_frac, 4),
                "launch_ms": round(top["ms"], 4), "share_of_step": round(top["ms"] / tot, 4),
                "alg_ops_per_launch": top["ops"], "alg_bytes_per_launch": top["bytes"],
            }
            line["layers"] = [{"name": p["name"], "ms": round(p["ms"], 4),
                               "tops": round(p["ops"] / (p["ms"] * 1e-3) / 1e12, 1) if p["ops"] else None,
                               "gbs": round(p["bytes"] / (p["ms"] * 1e-3) / 1e9, 1) if p["bytes"] else None}
                              for p in prof]
            g = gemm_tops(device)
            g.update(frac_of_int8_peak=round(g["tops"] / int8_peak, 4),
                     frac_of_nominal=round(g["tops"] / INT8_NOMINAL_TOPS, 4))
            line["gemm_int8"] = g
            line["gemm_small_m"] = small_m_gemm_hbm(device, peaks["hbm_gbs"])
            line["fc_cfg0"] = fc_cfg0(device, peaks["hbm_gbs"])
            lib_mark = int8_library_marker(device)
            if "tops" in lib_mark:
                lib_mark["frac_of_nominal"] = round(lib_mark["tops"] / INT8_NOMINAL_TOPS, 4)
            line["int8_library_marker"] = lib_mark
            fp16 = fp16_cudnn_rate(device, B, args.arch)
            fp16["w4a8_speedup"] = round(value / fp16["value"], 3)
            line["fp16_cudnn"] = fp16
            line["gemm_sweep_cfg1"] = gemm_sweep(device, int8_peak, peaks["hbm_gbs"])
            line["conv_cfg2"] = conv_cfg2(device, int8_peak, peaks["hbm_gbs"])
            if args.arch == "resnet18":
                line["resnet50_cfg4"] = resnet50_rate(device, B)
            # The CPU leg: the reference's CPU path on the host cores, and the
            # engine's logits for the timed batch checked against the oracle.
            engine.forward(dev_images)
            torch.cuda.synchronize()
            line["cpu_baseline"], line["parity"] = cpu_baseline_leg(model, host_images, engine.logits)
            line["cpu_baselines_cfg012"] = cpu_cfg012()
    engine.release()
    if line is not None:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        torch.cuda.set_device(local_rank)
        # NCCL prints its version line to stdout when the communicator is
        # created (eagerly here, device_id given); it goes to stderr so that
        # rank 0's stdout carries the one JSON line.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120),
                                                 device_id=torch.device("cuda", local_rank))
            torch.distributed.barrier()
            torch.cuda.synchronize()
        finally:
            import ctypes

            ctypes.CDLL(None).fflush(None)  # C stdio buffers (NCCL's printf) go out before fd 1 is restored
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
