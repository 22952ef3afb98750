"""Benchmark driver for the vdn_b200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload vda|gemm|block]
                    [--impl ours|reference]

One JSON line on rank 0.  A "step" is one pass of the hot path over one batch of
synthetic input of the BASELINE shapes (seeded; no dataset).  Device timing uses
CUDA events on the launching stream between a barrier + synchronize on both
sides; the value is the max over ranks.  `e2e` repeats the measurement through
the public API with pinned host inputs copied in and the result copied out
inside the timed region.  `--impl reference` times the CPU oracle (the
reference algorithm restated in numpy) on a bounded sample of the same workload
on the host cores.

Workloads:
  block (default)  BASELINE config 3: one hybrid DiT block (hidden 5120, 40 x 128
        heads, GELU FFN 13824, MXFP8 projections, VDA + window softmax +-1 frame)
        over 21 frames x 1560 tokens = 32760 tokens; metric = tokens/s of the
        whole job.  N > 1: Ulysses sequence parallelism (sequence shards, heads
        around attention) with the exchange done by the producers over NVLink
        peer memory (the QKV GEMM's scatter epilogue and the scatter quantiser,
        device fences; NCCL carries only setup and the timing reductions):
        strong scaling, the same 32760-token block split over N GPUs.  Each rank
        then recomputes the unsharded block outside the timed region and the line
        carries `parity` (max over ranks of the relative L2 of its rows).  N = 1:
        the line also carries `vda` (config 2), `gemm_sweep` (config 1) and
        `quantiser` sub-records, each timed on its own after the block.
  vda   BASELINE config 2: the VDA branch, H=40, d=128, 21 frames x 1560 tokens,
        metric = algorithmic HBM GB/s (q, k, v, gate, beta, alpha in; out).
        N > 1: independent replicas (heads are independent; no collective).
        --frames F shrinks the clip (small profiling case).
  gemm  BASELINE config 1: the MXFP8 GEMM sweep, M = 32760, (N, K) in
        (15360, 5120), (5120, 5120), (13824, 5120), (5120, 13824); each step
        quantises the bf16 activation and runs the four GEMMs; metric = TFLOP/s.
        --rows M shrinks M (small profiling case).  N > 1: replicas.
  stack BASELINE config 4: one denoise step = a 40-block stack of the config-3
        block over 512 text rows (packed first, dense softmax) + 60 x 1560 video
        rows, then the Euler update; --steps 8 is the 8-step loop; metric = video
        tokens/s.  N > 1: Ulysses over the packed rows (all-to-all exchange).
        --depth / --frames shrink it (small case).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    try:
        data = json.loads(PEAKS_FILE.read_text())
        return data, "measured"
    except Exception:
        return FALLBACK, "fallback"


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# DRAM bytes (read + write) per launch of the dominant kernels, from separate ncu
# captures of small cases of the same kernels (not measured in this run; summarised
# under profiles/), scaled to the full BASELINE shapes by the units processed:
# the QKV GEMM from 4096 rows (x 32760 / 4096), the VDA kernels from 5 frames
# (x 21 / 5).  Reported as roofline "traffic" with "traffic_source" saying so.
NCU_TRAFFIC_BYTES = {
    "mxfp8_gemm_qkv": (104.2e6 + 97.6e6) * 32760 / 4096,
    "statistics": 164.3e6 * 21 / 5,
    "factors": 13.2e6 * 21 / 5,
    "scan": 26.4e6 * 21 / 5,
    "gather": 15.8e6 * 21 / 5,
    "readout": 213.6e6 * 21 / 5,
}

TRAFFIC_SOURCE = ("from a separate ncu capture of a small case of this kernel (profiles/), scaled to "
                  "this shape by the units processed; not measured in this run")


# ------------------------------------------------------------------ timing
def time_steps(torch, fn, steps, warmup, dist, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        ms = float(t.item())
    return ms


def kernel_times(torch, launches, reps, stream):
    """Average device ms of each named launch (CUDA events on `stream`)."""
    out = {}
    for name, fn in launches:
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        out[name] = a.elapsed_time(b) / reps
    return out


def cublas_fp8_ms(torch, m, n, k, dev, stream, reps=10):
    """Device ms of the same-box cuBLAS per-tensor E4M3 GEMM [m, k] x [n, k]^T -> bf16:
    the reference's B200 FP8 path, Fp8Linear.forward_quantized (src/models/ops/
    fp8_linear.py:269-273: torch._scaled_mm, scalar scales, use_fast_accum=True)."""
    g = torch.Generator(device=dev).manual_seed(99)
    a = torch.randn(m, k, device=dev, generator=g).to(torch.float8_e4m3fn)
    b = torch.randn(n, k, device=dev, generator=g).to(torch.float8_e4m3fn)
    one = torch.ones((), device=dev)
    fn = lambda: torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16,
                                  use_fast_accum=True)
    return kernel_times(torch, [("cublas", fn)], reps, stream)["cublas"]


def torch_mxfp8_ms(torch, xq, xs, wq, ws, stream, reps=10):
    """Device ms of torch's block-scaled MXFP8 GEMM on the same codes and swizzled scales:
    the call the reference's MXFP8Linear makes (src/models/ops/mxfp8_linear.py:89-94,
    F.scaled_mm with BlockWise1x32 / SWIZZLE_32_4_4; gated to SM120 there).  Raises if
    this torch / cuBLAS build does not run it on this GPU."""
    import torch.nn.functional as Fn
    e4, e8 = torch.float8_e4m3fn, torch.float8_e8m0fnu
    fn = lambda: Fn.scaled_mm(xq.view(e4), wq.view(e4).T, xs.view(e8), Fn.ScalingType.BlockWise1x32,
                              ws.view(e8), Fn.ScalingType.BlockWise1x32, Fn.SwizzleType.SWIZZLE_32_4_4,
                              Fn.SwizzleType.SWIZZLE_32_4_4, output_dtype=torch.bfloat16)
    return kernel_times(torch, [("mx", fn)], reps, stream)["mx"]


# ------------------------------------------------------------------ VDA
VDA_CFG = dict(F=21, S=1560, H=40, d=128)


def vda_bytes(F, S, H, d):
    n = F * S
    return 4 * n * H * d * 2 + n * H * 2 + F * H * d * 4 + n * H * d * 2


def vda_inputs(torch, device, F, S, H, d, seed=0):
    import torch.nn.functional as Fn
    g = torch.Generator(device=device).manual_seed(seed)
    n = F * S
    q = Fn.normalize(torch.randn(n, H, d, device=device, generator=g), dim=-1).bfloat16()
    k = Fn.normalize(torch.randn(n, H, d, device=device, generator=g), dim=-1).bfloat16()
    v = torch.randn(n, H, d, device=device, generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(n, H, device=device, generator=g)).bfloat16()
    gate = torch.rand(n, H, d, device=device, generator=g).bfloat16()
    alpha = torch.exp(-Fn.softplus(torch.randn(F, H, 1, device=device, generator=g))).expand(F, H, d).contiguous()
    return q, k, v, beta, gate, alpha


def bench_vda(args, torch, dist, rank, world):
    from vdn_b200 import _lib
    from vdn_b200.linear_attention import vda_forward, window_bounds
    F, S, H, d = (VDA_CFG[k] for k in ("F", "S", "H", "d"))
    F = args.frames or F
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    q, k, v, beta, gate, alpha = vda_inputs(torch, dev, F, S, H, d, seed=rank)
    w = torch.ones(d, device=dev)
    bounds = window_bounds(F, 1)
    n = F * S
    out = torch.empty(n, H * d, device=dev, dtype=torch.bfloat16)
    ws_bytes = _lib.load().vdn_vda_workspace_size(F, S, H, d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    buf = (_lib.C.c_int32 * (2 * F))(*[x for b in bounds for x in b])
    st = _lib.stream_of(dev)

    def step():
        _lib.call("vdn_vda_forward", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), q.stride(0), q.stride(1),
                  _lib.ptr(beta), beta.stride(0), beta.stride(1), _lib.ptr(gate), gate.stride(0),
                  gate.stride(1), _lib.ptr(alpha), _lib.ptr(w), 1e-6, buf, None, 1, F, S, H, d,
                  _lib.ptr(out), _lib.ptr(ws), ws_bytes, st)

    with ClockSampler(dev.index) as clk:
        ms = time_steps(torch, step, args.steps, args.warmup, dist, stream)
    per_step_ms = ms / args.steps
    nbytes = vda_bytes(F, S, H, d)
    value = world * nbytes / (per_step_ms * 1e-3) / 1e9

    # Per-kernel device times of the five stage launches (same stream), on the regions of
    # the forward's own workspace (d = 128: A then the forward bank over it, B, the split
    # inverses, the reverse bank, the gathered state).  The scan is timed in the bf16-B
    # form the forward runs (the statistics stage API writes fp32 B, so its bytes feed the
    # scan as arbitrary bf16 values here: timing only).
    plane = F * H * d * d
    up = lambda b: (b + 255) // 256 * 256
    A = ws[: plane * 4].view(torch.float32)
    B = ws[up(plane * 4): up(plane * 4) + plane * 4].view(torch.float32)
    planes = ws[2 * up(plane * 4): 2 * up(plane * 4) + plane * 6]
    pre = A
    suf = ws[2 * up(plane * 4) + up(plane * 6): 2 * up(plane * 4) + up(plane * 6) + plane * 4].view(torch.float32)
    state = ws[3 * up(plane * 4) + up(plane * 6): 3 * up(plane * 4) + up(plane * 6) + plane * 2]
    sf = S * q.stride(0)
    launches = [
        ("statistics", lambda: _lib.call("vdn_vda_statistics", _lib.ptr(k), sf, q.stride(0), q.stride(1),
                                         _lib.ptr(v), sf, q.stride(0), q.stride(1), _lib.ptr(beta),
                                         S * beta.stride(0), beta.stride(0), beta.stride(1), 0, F, S, H,
                                         d, _lib.ptr(A), _lib.ptr(B), st)),
        ("factors", lambda: _lib.call("vdn_vda_factor_inverse", _lib.ptr(A), F * H, _lib.ptr(planes), st)),
        ("scan", lambda: _lib.call("vdn_vda_scan_tc_bf16", _lib.ptr(planes), _lib.ptr(B), _lib.ptr(alpha), None, F, H,
                                   _lib.ptr(pre), _lib.ptr(suf), None, st)),
        ("gather", lambda: _lib.call("vdn_vda_gather", _lib.ptr(pre), _lib.ptr(suf), _lib.ptr(alpha), buf,
                                     None, 1, F, H, d, _lib.ptr(state), _lib.DTYPE_BF16, st)),
        ("readout", lambda: _lib.call("vdn_vda_readout", _lib.ptr(q), sf, q.stride(0), q.stride(1),
                                      _lib.ptr(state), _lib.ptr(gate), S * gate.stride(0), gate.stride(0),
                                      gate.stride(1), _lib.ptr(w), 1e-6, F, S, H, d, _lib.ptr(out), st)),
    ]
    kt = kernel_times(torch, launches, 5, stream)
    n_tok_h_d = n * H * d
    algo = {  # algorithmic bytes per launch
        "statistics": 2 * n_tok_h_d * 2 + n * H * 2 + 2 * F * H * d * d * 4,
        "factors": F * H * d * d * 4 + F * H * d * d * 6,
        "scan": F * H * d * d * 6 * 2 + F * H * d * d * 4 * 2 + 2 * F * H * d * d * 4,
        "gather": 2 * F * H * d * d * 4 + F * H * d * d * 2,
        "readout": 2 * n_tok_h_d * 2 + F * H * d * d * 2 + n_tok_h_d * 2,
    }
    top = max(kt, key=kt.get)
    pk, src = peaks()
    achieved = algo[top] / (kt[top] * 1e-3) / 1e9

    # End to end through the public API: pinned host inputs in, result out.
    host = [t.cpu().pin_memory() for t in (q, k, v, beta, gate, alpha)]
    out_host = torch.empty(n, H * d, dtype=torch.bfloat16).pin_memory()
    dq = [torch.empty_like(t) for t in (q, k, v, beta, gate, alpha)]

    def e2e_step():
        for dst, src_t in zip(dq, host):
            dst.copy_(src_t, non_blocking=True)
        y = vda_forward(dq[0], dq[1], dq[2], dq[3], dq[4], dq[5], bounds, F, S, w)
        out_host.copy_(y, non_blocking=True)

    e2e_ms = time_steps(torch, e2e_step, max(2, args.steps // 2), 1, dist, stream) / max(2, args.steps // 2)
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = out_host.numel() * 2
    rec = {
        "metric": "VDA branch HBM GB/s (algorithmic bytes), BASELINE config 2",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "vda_config2", "frames": F, "tokens_per_frame": S, "heads": H,
                   "head_dim": d, "window": "+-1 frame", "calls_per_step": 1,
                   "parallelism": f"replicated x{world} (heads independent, no collective)",
                   "l2": "inputs (1.68 GB/step) larger than L2"},
        "e2e": {"value": round(world * nbytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": 5 * args.steps,
        "roofline": {"bound": "hbm", "kernel": top, "achieved": round(achieved, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "traffic": NCU_TRAFFIC_BYTES.get(top) if F == VDA_CFG["F"] else None,
                     "traffic_unit": "bytes per launch (ncu dram read + write)",
                     "traffic_source": TRAFFIC_SOURCE, "peak_source": src,
                     "algorithmic_bytes_per_launch": algo[top]},
        "kernels_ms": {k_: round(v_, 4) for k_, v_ in kt.items()},
        "clocks": clk.summary(),
    }
    return rec


def cpu_baseline_vda(threads):
    """Oracle VDA on 1 head of config 2 (full frames/tokens), scaled to 40 heads."""
    import numpy as np
    import torch
    from oracle import vda as ovda
    F, S, H, d = (VDA_CFG[k] for k in ("F", "S", "H", "d"))
    q, k, v, beta, gate, alpha = vda_inputs(torch, torch.device("cpu"), F, S, 1, d)
    args = [t.float().numpy() for t in (q, k, v, beta, gate)] + [alpha.numpy()]
    bounds = ovda.window_bounds(F, 1)
    t0 = time.perf_counter()
    ovda.readout(*args, bounds, F, S)
    dt = (time.perf_counter() - t0) * H
    return {"value": round(vda_bytes(F, S, H, d) / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "port", "sample": "oracle VDA body, 1 of 40 heads at 21x1560 tokens, time x40"}


# ---------------------------------------------------------------------- gemm
GEMM_SHAPES = (("qkv", 15360, 5120), ("o", 5120, 5120), ("ffn_up", 13824, 5120), ("ffn_down", 5120, 13824))
GEMM_ROWS = 32760


def gemm_activation(torch, device, rows, k, seed):
    """bf16 N(0,1) with 1% of the K channels (a fixed seeded set) scaled x50."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(rows, k, device=device, generator=g)
    cols = torch.randperm(k, generator=torch.Generator().manual_seed(seed))[: max(1, k // 100)]
    x[:, cols.to(device)] *= 50.0
    return x.bfloat16()


def bench_gemm(args, torch, dist, rank, world):
    """MXFP8 GEMM sweep, activation quantised on the fly each step."""
    from vdn_b200.mxfp8_quant import quantize_activation
    from vdn_b200.mxfp8_linear import mxfp8_gemm, check_gemm_status
    M = args.rows or GEMM_ROWS
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    cases = []
    for i, (name, n, k) in enumerate(GEMM_SHAPES):
        x = gemm_activation(torch, dev, M, k, seed=10 + i)
        g = torch.Generator(device=dev).manual_seed(20 + i)
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
        wq, ws = quantize_activation(w)
        del w
        y = torch.empty(M, n, device=dev, dtype=torch.bfloat16)
        cases.append(dict(name=name, n=n, k=k, x=x, wq=wq, ws=ws, y=y, flops=2 * M * n * k))

    def run(c, xq=None, xs=None):
        if xq is None:
            xq, xs = quantize_activation(c["x"], check_finite=False)
        mxfp8_gemm(xq, xs, c["wq"], c["ws"], c["n"], rows=M, out=c["y"])

    def step():
        for c in cases:
            run(c)

    with ClockSampler(dev.index) as clk:
        ms = time_steps(torch, step, args.steps, args.warmup, dist, stream)
    check_gemm_status(dev)
    per_step_ms = ms / args.steps
    total_flops = sum(c["flops"] for c in cases)
    value = world * total_flops / (per_step_ms * 1e-3) / 1e12

    # Kernel-only times: each GEMM on pre-quantised operands, and each quantiser pass.
    launches = []
    for c in cases:
        c["xq"], c["xs"] = quantize_activation(c["x"], check_finite=False)
        launches.append((c["name"], (lambda c=c: run(c, c["xq"], c["xs"]))))
        launches.append((c["name"] + "_quantize", (lambda c=c: quantize_activation(c["x"], check_finite=False))))
    kt = kernel_times(torch, launches, 10, stream)
    pk, src = peaks()
    fp8_peak = 2 * pk["bf16_tflops"]
    per_shape = {}
    for c in cases:
        tf = c["flops"] / (kt[c["name"]] * 1e-3) / 1e12
        try:
            cub = c["flops"] / (cublas_fp8_ms(torch, M, c["n"], c["k"], dev, stream) * 1e-3) / 1e12
        except Exception:  # comparator only
            cub = None
        try:
            tmx = c["flops"] / (torch_mxfp8_ms(torch, c["xq"], c["xs"], c["wq"], c["ws"], stream) * 1e-3) / 1e12
        except Exception as e:  # comparator only
            tmx = repr(e)[:100]
        qbytes = M * c["k"] * 2 + (M + 127) // 128 * 128 * c["k"] * 33 // 32
        per_shape[c["name"]] = {"m": M, "n": c["n"], "k": c["k"], "gemm_ms": round(kt[c["name"]], 4),
                                "tflops": round(tf, 1), "frac_fp8_peak": round(tf / fp8_peak, 4),
                                "cublas_fp8_per_tensor_tflops": None if cub is None else round(cub, 1),
                                "frac_of_cublas": None if cub is None else round(tf / cub, 4),
                                "torch_mxfp8_tflops": round(tmx, 1) if isinstance(tmx, float) else tmx,
                                "quantize_ms": round(kt[c["name"] + "_quantize"], 4),
                                "quantize_gbs": round(qbytes / (kt[c["name"] + "_quantize"] * 1e-3) / 1e9, 1)}
    top = cases[0]
    achieved = top["flops"] / (kt[top["name"]] * 1e-3) / 1e12

    # End to end through the public API: host activations in, bf16 results out.
    xh = [c["x"].cpu().pin_memory() for c in cases]
    yh = [torch.empty(M, c["n"], dtype=torch.bfloat16).pin_memory() for c in cases]
    xd = [torch.empty_like(c["x"]) for c in cases]

    def e2e_step():
        for c, h, d_, o in zip(cases, xh, xd, yh):
            d_.copy_(h, non_blocking=True)
            xq, xs = quantize_activation(d_, check_finite=False)
            mxfp8_gemm(xq, xs, c["wq"], c["ws"], c["n"], rows=M, out=c["y"])
            o.copy_(c["y"], non_blocking=True)

    e2e_steps = max(2, args.steps // 2)
    e2e_ms = time_steps(torch, e2e_step, e2e_steps, 1, dist, stream) / e2e_steps
    return {
        "metric": "MXFP8 GEMM TFLOP/s, BASELINE config 1 sweep (activation quantised each step)",
        "value": round(value, 1), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8 e4m3 x e4m3, e8m0 per 32, fp32 accumulate",
        "data": "synthetic (bf16 N(0,1) activations, 1% of channels x50; N(0,0.02) weights)",
        "config": {"workload": "gemm_config1", "m": M, "shapes": [[n, k] for _, n, k in GEMM_SHAPES],
                   "parallelism": f"replicated x{world}" if world > 1 else "single GPU",
                   "l2": "operands and outputs of every GEMM larger than L2"},
        "e2e": {"value": round(world * total_flops / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                "h2d_bytes_per_step": sum(h.numel() * 2 for h in xh),
                "d2h_bytes_per_step": sum(o.numel() * 2 for o in yh)},
        "gpu_launches": 2 * len(cases) * args.steps,
        "roofline": {"bound": "tensor", "kernel": "mxfp8_gemm (qkv, %d x 15360 x 5120)" % M,
                     "achieved": round(achieved, 1), "peak": round(fp8_peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / fp8_peak, 4),
                     "traffic": NCU_TRAFFIC_BYTES["mxfp8_gemm_qkv"] if M == GEMM_ROWS else None,
                     "traffic_unit": "bytes per launch (ncu dram read + write)",
                     "traffic_source": TRAFFIC_SOURCE,
                     "peak_source": f"2 x {src} bf16 dense ({pk['bf16_tflops']}): the FP8 rate",
                     "algorithmic_flops_per_launch": top["flops"]},
        "shapes": per_shape,
        "clocks": clk.summary(),
    }


def cpu_baseline_gemm(threads):
    """Dequantised fp32 matmul oracle on a 256-row slice of the QKV shape, scaled to the sweep."""
    import torch
    from oracle import mxfp8 as omx
    rows = 256
    total = 0.0
    for i, (name, n, k) in enumerate(GEMM_SHAPES[:1]):
        x = gemm_activation(torch, torch.device("cpu"), rows, k, seed=10 + i)
        w = (torch.randn(n, k, generator=torch.Generator().manual_seed(20 + i)) * 0.02).bfloat16()
        xq, xs = omx.quantize(x.float().numpy())
        wq, wsc = omx.quantize(w.float().numpy())
        t0 = time.perf_counter()
        omx.mxfp8_gemm(xq, xs, wq, wsc, rows, n)
        total += time.perf_counter() - t0
        flops = 2 * rows * n * k
    return {"value": round(flops / total / 1e12, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": "oracle dequantise + fp32 matmul, 256 rows of the QKV shape (15360 x 5120)"}


# ---------------------------------------------------------------------- block
BLOCK_CFG = dict(F=21, S=1560, hidden=5120, heads=40, head_dim=128, ffn=13824)


def bench_block(args, torch, dist, rank, world):
    from vdn_b200.block import HybridBlock
    from vdn_b200.ulysses import init_ulysses
    from vdn_b200.mxfp8_quant import quantize_activation
    F, S = BLOCK_CFG["F"], BLOCK_CFG["S"]
    T = F * S
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    block = HybridBlock(seed=0, device=dev)
    runtime = None
    lo, hi = 0, T
    if world > 1:
        runtime = init_ulysses("nccl")
        if args.softmax_ranks:
            runtime.enable_branch_parallel(args.softmax_ranks)
        runtime.configure(T, BLOCK_CFG["heads"])
        lo, hi = runtime.local_start, runtime.local_end
    if args.softmax_ranks and (world < 2 or not args.eager):
        raise SystemExit("--softmax-ranks needs --gpus >= 2 and --eager (NCCL all-to-alls are not captured)")
    g = torch.Generator(device=dev).manual_seed(1234)
    x_full = torch.randn(T, BLOCK_CFG["hidden"], device=dev, generator=g).bfloat16()
    temb = torch.randn(BLOCK_CFG["hidden"], device=dev, generator=g)
    x = x_full[lo:hi].contiguous()
    if world == 1:
        del x_full  # N > 1 keeps it for the parity check against the unsharded block
    rows = hi - lo

    if args.eager:
        def step():
            return block(x, temb, F, S, runtime)
    else:
        from vdn_b200.block import BlockGraph
        graph = BlockGraph(block, x, temb, F, S, runtime)

        def step():
            return graph.replay()

    with ClockSampler(dev.index) as clk:
        ms = time_steps(torch, step, args.steps, args.warmup, dist, stream)
    per_step_ms = ms / args.steps
    value = T / (per_step_ms * 1e-3)
    # This library's kernels per forward, counted on one eager forward (every rank runs
    # it: the sharded forward has collectives); the graph replays the same launches.
    launches = count_launches(lambda: block(x, temb, F, S, runtime))
    flops = 2 * T * BLOCK_CFG["hidden"] * (3 * BLOCK_CFG["hidden"] + 2 * BLOCK_CFG["hidden"]
                                           + 2 * BLOCK_CFG["ffn"])

    # Dominant kernel: the FFN-up / QKV MXFP8 GEMMs; time the QKV launch on this rank's rows.
    y1 = torch.randn(rows, BLOCK_CFG["hidden"], device=dev).bfloat16()
    q1, s1 = quantize_activation(y1)
    out = torch.empty(rows, 3 * BLOCK_CFG["hidden"], device=dev, dtype=torch.bfloat16)
    kt = kernel_times(torch, [("mxfp8_gemm_qkv", lambda: block._gemm(q1, s1, block.qkv, rows, out,
                                                                    bias=block.qkv.bias))], 10, stream)
    gemm_flops = 2 * rows * 3 * BLOCK_CFG["hidden"] * BLOCK_CFG["hidden"]
    achieved = gemm_flops / (kt["mxfp8_gemm_qkv"] * 1e-3) / 1e12
    pk, src = peaks()
    fp8_peak = 2 * pk["bf16_tflops"]
    comp = {}
    try:
        cub = gemm_flops / (cublas_fp8_ms(torch, rows, 3 * BLOCK_CFG["hidden"], BLOCK_CFG["hidden"], dev,
                                          stream) * 1e-3) / 1e12
        comp["cublas_fp8_per_tensor_tflops"] = round(cub, 1)
        comp["cublas_call"] = "torch._scaled_mm, scalar scales, use_fast_accum=True (Fp8Linear)"
        comp["frac_of_cublas"] = round(achieved / cub, 4)
    except Exception as e:  # comparator only
        comp["cublas_fp8_per_tensor_error"] = repr(e)[:120]

    # End to end through the public API: pinned host rows in, block output back to the host,
    # every step.  Graph launch (default): BlockPipeline overlaps batch i's compute with the
    # host copies of its neighbours; eager: copy in, forward, copy out, in order.
    x_host = [x.cpu().pin_memory() for _ in range(2)]
    out_host = [torch.empty_like(x_host[0]).pin_memory() for _ in range(2)]
    e2e_steps = max(2, args.steps)
    if args.eager:
        x_dev = torch.empty_like(x)

        def e2e_step():
            x_dev.copy_(x_host[0], non_blocking=True)
            y = block(x_dev, temb, F, S, runtime)
            out_host[0].copy_(y, non_blocking=True)

        e2e_ms = time_steps(torch, e2e_step, e2e_steps, 1, dist, stream) / e2e_steps
    else:
        # Two captured forwards alternate; each batch's host-to-device and device-to-host
        # copies run on the copy engines while the neighbouring batches compute (under
        # Ulysses every rank streams its own rows; the graphs share the peer exchange,
        # whose replays are serialised on the compute stream).
        from vdn_b200.block import BlockPipeline
        pipe = BlockPipeline(block, rows, temb, F, S, runtime)
        ins = [x_host[i & 1] for i in range(e2e_steps)]
        outs = [out_host[i & 1] for i in range(e2e_steps)]
        e2e_ms = time_steps(torch, lambda: pipe.run(ins, outs), 1, 1, dist, stream) / e2e_steps
        del pipe
    rec = {
        "metric": "hybrid-block tokens/s (BASELINE config 3, 32760 tokens)",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "mxfp8 GEMMs (fp32 accumulate), bf16 activations",
        "data": "synthetic (seeded N(0,1) tokens and timestep embedding, random-init weights)",
        "config": {"workload": "hybrid_block_config3", "frames": F, "tokens_per_frame": S,
                   "hidden": BLOCK_CFG["hidden"], "heads": BLOCK_CFG["heads"],
                   "head_dim": BLOCK_CFG["head_dim"], "ffn": BLOCK_CFG["ffn"], "window": "+-1 frame",
                   "lora_rank": 32, "parallelism": f"ulysses sp{world}" if world > 1 else "single GPU",
                   "l2": "per-step working set (activations > 1 GB) larger than L2",
                   "gemm_tflops_per_step": round(flops / 1e12, 3)},
        "e2e": {"value": round(T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": x_host[0].numel() * 2, "d2h_bytes_per_step": out_host[0].numel() * 2,
                "steps": e2e_steps, "copies": "per step; overlapped with neighbouring steps"
                if not args.eager else "per step; serial"},
        "gpu_launches": launches * args.steps,
        "launch": "eager" if args.eager else "cuda_graph",
        "roofline": {"bound": "tensor", "kernel": "mxfp8_gemm (QKV, %d x 15360 x 5120)" % rows,
                     "achieved": round(achieved, 1), "peak": round(fp8_peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / fp8_peak, 4),
                     "traffic": NCU_TRAFFIC_BYTES["mxfp8_gemm_qkv"] if world == 1 else None,
                     "traffic_unit": "bytes per launch (ncu dram read + write)",
                     "traffic_source": TRAFFIC_SOURCE,
                     "peak_source": f"2 x {src} bf16 dense ({pk['bf16_tflops']}): the FP8 rate",
                     "algorithmic_flops_per_launch": gemm_flops},
        "comparators": comp,
        "kernels_ms": {k_: round(v_, 4) for k_, v_ in kt.items()},
        "clocks": clk.summary(),
    }
    if world > 1:
        rec["parity"] = block_parity(torch, dist, block, step, x_full, temb, F, S, lo, hi)
        del x_full
        if runtime.exchange_mode == "peer" and not runtime.branch_parallel:
            rec["phases"] = block_phases(torch, dist, block, x, temb, F, S, runtime)
    elif not args.no_sub:
        rec.update(sub_records(args, torch))
    if runtime is not None:
        rec["config"]["exchange"] = runtime.exchange_mode
        if runtime.branch_parallel:
            rec["config"]["exchange"] = "nccl all-to-all (two dispatch communicators)"
            rec["config"]["parallelism"] = (f"ulysses branch-parallel {runtime.softmax_ranks} softmax + "
                                            f"{world - runtime.softmax_ranks} VDA ranks")
        runtime.close()
    return rec


def block_parity(torch, dist, block, step, x_full, temb, F, S, lo, hi, tol=2e-3):
    """This rank's rows of the sharded forward against the unsharded block computed on
    the same rank (same weights, same inputs), outside the timed region; the relative
    L2 and max-abs differences are reduced by MAX over ranks.  The bar (2e-3) is the
    multi-GPU block test's: alpha sees the frame sums added in another order."""
    y = step().clone()                       # every rank replays its shard (peer fences)
    torch.cuda.synchronize()
    ref = block(x_full, temb, F, S, None)[lo:hi]
    torch.cuda.synchronize()
    rel = float((y.double() - ref.double()).norm() / ref.double().norm())
    mx = float((y.float() - ref.float()).abs().max())
    t = torch.tensor([rel, mx], device=y.device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    rel, mx = float(t[0]), float(t[1])
    return {"rel_l2_max": rel, "max_abs": mx, "tol_rel_l2": tol, "ok": bool(rel < tol),
            "reference": "unsharded block on each rank (same seeded weights and input)"}


PEER_PHASES = ("adaln_prenorm", "gates_and_side_rows", "qkv_gemm_scatter", "fence_heads", "window_softmax",
               "softmax_quantize_scatter", "vda_branch", "vda_quantize_scatter", "fence_rows", "out_gemm", "ffn")


def block_phases(torch, dist, block, x, temb, F, S, runtime):
    """One eager forward with CUDA events around the phases of the peer-exchange block
    (the softmax phases on the caller's stream, the VDA phases on the side stream,
    which overlap them), max over ranks; plus the bytes each rank moves over NVLink."""
    runtime.reset_profile()
    runtime.profile_enabled = True
    block(x, temb, F, S, runtime)
    ms = runtime.profile_milliseconds()
    runtime.profile_enabled = False
    runtime.reset_profile()
    t = torch.tensor([ms.get(k, 0.0) for k in PEER_PHASES], device=x.device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    P, T = runtime.world_size, F * S
    cfg = block.cfg
    hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
    rows = runtime.local_end - runtime.local_start
    r = block.output_gate.down.weight.shape[0]
    remote = (P - 1) / P
    out_bytes = {  # bytes this rank stores into other ranks' memory per block
        "qkv_scatter": int(rows * 3 * hd * 2 * remote),
        "side_rows_and_frame_sums": int((rows * (2 * H + r) * 2 + F * hd * 4) * (P - 1)),
        "results_mxfp8_scatter": int(2 * T * (H // P) * d * (1 + 1 / 32) * remote),
    }
    phases = {k: round(float(v), 4) for k, v in zip(PEER_PHASES, t.tolist())}
    ret_ms = phases["softmax_quantize_scatter"] + phases["vda_quantize_scatter"]
    return {"ms_max_over_ranks": phases, "launch": "eager, one forward after the timed region",
            "nvlink_bytes_out_per_rank": out_bytes,
            "result_scatter_gbs": round(out_bytes["results_mxfp8_scatter"] / (ret_ms * 1e-3) / 1e9, 1)
            if ret_ms > 0 else None}


def sub_records(args, torch):
    """BASELINE configs 2 and 1 timed on their own after the block (N = 1): the VDA
    branch (8 calls), the four-GEMM sweep and the activation quantiser.  Each keeps
    its metric, roofline, kernel times, e2e and clocks."""
    sub = argparse.Namespace(**vars(args))
    sub.steps, sub.warmup, sub.frames, sub.rows = 8, 3, 0, 0
    keep = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "e2e", "roofline",
            "kernels_ms", "clocks", "config", "gpu_launches")
    torch.cuda.empty_cache()
    v = bench_vda(sub, torch, None, 0, 1)
    torch.cuda.empty_cache()
    g = bench_gemm(sub, torch, None, 0, 1)
    torch.cuda.empty_cache()
    pk, src = peaks()
    qkv = g["shapes"]["qkv"]
    qbytes = GEMM_ROWS * 5120 * 2 + (GEMM_ROWS + 127) // 128 * 128 * 5120 * 33 // 32
    quant = {"metric": "MXFP8 activation quantiser GB/s (32760 x 5120 bf16 -> E4M3 codes + E8M0 scales)",
             "value": qkv["quantize_gbs"], "unit": "GB/s", "ms": qkv["quantize_ms"],
             "algorithmic_bytes": qbytes,
             "roofline": {"bound": "hbm", "achieved": qkv["quantize_gbs"], "peak": pk["hbm_gbs"],
                          "unit": "GB/s", "frac": round(qkv["quantize_gbs"] / pk["hbm_gbs"], 4),
                          "peak_source": src},
             "clocks": g["clocks"]}
    return {"vda": {k: v[k] for k in keep if k in v},
            "gemm_sweep": {**{k: g[k] for k in keep if k in g}, "shapes": g["shapes"]},
            "quantiser": quant}


def cpu_baseline_block(threads):
    """Reference block composition (oracle/block.py) on the CPU for 3 of 21 frames."""
    import torch
    from oracle import block as oblock
    from vdn_b200.block import BlockConfig
    cfg = BlockConfig()
    frames, tokens = 3, BLOCK_CFG["S"]
    hd, ffn = cfg.hidden, cfg.ffn
    g = torch.Generator().manual_seed(0)
    w = dict(adaln_w=torch.randn(6 * hd, hd, generator=g) * 0.02, adaln_b=torch.zeros(6 * hd),
             norm1=torch.ones(hd), norm2=torch.ones(hd),
             qkv=torch.randn(3 * hd, hd, generator=g) * 0.02, qkv_b=torch.zeros(3 * hd),
             o=torch.randn(hd, hd, generator=g) * 0.02, ol=torch.randn(hd, hd, generator=g) * 0.02,
             o_b=torch.zeros(hd), up=torch.randn(ffn, hd, generator=g) * 0.02, up_b=torch.zeros(ffn),
             down=torch.randn(hd, ffn, generator=g) * 0.02, down_b=torch.zeros(hd),
             sg_w=torch.zeros(cfg.heads, hd), sg_b=torch.full((cfg.heads,), 4.595),
             beta_w=torch.randn(cfg.heads, hd, generator=g) * 0.02,
             og_down=torch.randn(cfg.head_dim, hd, generator=g) * 0.02,
             og_up=torch.randn(hd, cfg.head_dim, generator=g) * 0.02, og_b=torch.zeros(hd))
    x = torch.randn(frames * tokens, hd, generator=g).bfloat16()
    temb = torch.randn(hd, generator=g)
    alpha = lambda fm: torch.exp(-torch.nn.functional.softplus(torch.zeros(frames, cfg.heads, cfg.head_dim)))
    t0 = time.perf_counter()
    oblock.block_reference(x, temb, w, frames, tokens, cfg, alpha)
    dt = time.perf_counter() - t0
    return {"value": round(frames * tokens / dt, 2), "unit": "tokens/s", "cores": threads,
            "kind": "port", "sample": "reference block composition (fp32 torch CPU + numpy oracle), "
            "3 frames x 1560 tokens (per-token work is constant in the frame count)"}


# ---------------------------------------------------------------------- stack
STACK_CFG = dict(F=60, S=1560, text_rows=512, depth=40, denoise_steps=8)

# Kernels of this library each entry point launches (default 1; setup calls launch none).
KERNELS_PER_CALL = {"vdn_vda_forward": 5, "vdn_frame_alpha": 2, "vdn_sepconv": 2,
                    "vdn_peer_alloc": 0, "vdn_peer_free": 0, "vdn_ipc_handle": 0, "vdn_ipc_open": 0,
                    "vdn_ipc_close": 0, "vdn_copy_async": 0, "vdn_mxfp8_quantize_host": 0,
                    "vdn_last_error": 0, "vdn_mxfp8_padded_shape": 0, "vdn_vda_workspace_size": 0}


def count_launches(fn):
    """Run fn() once and count the kernels of this library it launches (by entry point)."""
    from vdn_b200 import _lib
    real = _lib.call
    count = [0]

    def counting(name, *a, **k):
        count[0] += KERNELS_PER_CALL.get(name, 1)
        return real(name, *a, **k)

    _lib.call = counting
    try:
        fn()
    finally:
        _lib.call = real
    return count[0]


def bench_stack(args, torch, dist, rank, world):
    """the 8-step denoise loop of a 40-block stack over 512 text rows +
    60 x 1560 video rows (text packed first as global rows); N > 1 shards the packed rows
    with Ulysses (all-to-all exchange)."""
    from vdn_b200.block import BlockConfig
    from vdn_b200.mxfp8_quant import quantize_activation
    from vdn_b200.stack import HybridStack, denoise, local_rows
    from vdn_b200.ulysses import init_ulysses
    F = args.frames or STACK_CFG["F"]
    S, L = STACK_CFG["S"], STACK_CFG["text_rows"]
    depth = args.depth or STACK_CFG["depth"]
    cfg = BlockConfig()
    hd = cfg.hidden
    T = F * S
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    runtime = None
    if world > 1:  # Ulysses over the packed [text | video] rows, all-to-all exchange
        runtime = init_ulysses("nccl")
        runtime.exchange_mode = "alltoall"
        runtime.configure(L + T, cfg.heads)
    (ta, tb), (va, vb) = local_rows(L, runtime, L + T)
    stack = HybridStack(cfg, depth, seed=0, device=dev, init="device")
    g = torch.Generator(device=dev).manual_seed(4321)
    video = torch.randn(T, hd, device=dev, generator=g).bfloat16()[va:vb].contiguous()
    text = torch.randn(L, hd, device=dev, generator=g).bfloat16()
    nsteps = STACK_CFG["denoise_steps"]
    tembs = torch.randn(nsteps, hd, device=dev, generator=g)
    rows = (tb - ta) + (vb - va)
    packed = torch.empty(rows, hd, device=dev, dtype=torch.bfloat16)
    i = [0]

    def step():  # one denoise step: the whole stack over [text | video], then the Euler update
        j = i[0] % nsteps
        denoise(stack, video, text, tembs[j:j + 1], F, S, packed=packed, dt=-1.0 / nsteps, runtime=runtime)
        i[0] += 1

    launches = count_launches(step)
    with ClockSampler(dev.index) as clk:
        ms = time_steps(torch, step, args.steps, args.warmup, dist, stream)
    finite = bool(torch.isfinite(video).all())
    per_step_ms = ms / args.steps
    value = T / (per_step_ms * 1e-3)

    # e2e: each step copies its inputs (latent + text context) in from pinned host memory
    # and reads the updated latent back.
    v_host = video.cpu().pin_memory()
    t_host = text.cpu().pin_memory()
    out_host = torch.empty_like(v_host).pin_memory()

    def e2e_step():
        video.copy_(v_host, non_blocking=True)
        text.copy_(t_host, non_blocking=True)
        step()
        out_host.copy_(video, non_blocking=True)

    e2e_steps = 2
    e2e_ms = time_steps(torch, e2e_step, e2e_steps, 1, dist, stream) / e2e_steps

    blk = stack.blocks[0]
    n = rows
    y1 = torch.randn(n, hd, device=dev).bfloat16()
    q1, s1 = quantize_activation(y1)
    out = torch.empty(n, 3 * hd, device=dev, dtype=torch.bfloat16)
    kt = kernel_times(torch, [("mxfp8_gemm_qkv", lambda: blk._gemm(q1, s1, blk.qkv, n, out,
                                                                  bias=blk.qkv.bias))], 5, stream)
    gemm_flops = 2 * n * 3 * hd * hd
    achieved = gemm_flops / (kt["mxfp8_gemm_qkv"] * 1e-3) / 1e12
    pk, src = peaks()
    fp8_peak = 2 * pk["bf16_tflops"]
    rec = {
        "metric": "denoise-loop tokens/s (BASELINE config 4: 40-block stack, 60 x 1560 video + 512 text rows)",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "mxfp8 GEMMs (fp32 accumulate), bf16 activations",
        "data": "synthetic (seeded N(0,1) latent, text context and timestep embeddings; random-init "
                "weights drawn on the device)",
        "config": {"workload": "denoise_stack_config4", "frames": F, "tokens_per_frame": S, "text_rows": L,
                   "depth": depth, "denoise_steps": nsteps, "step": "one denoise step (whole stack + Euler update)",
                   "hidden": hd, "heads": cfg.heads, "head_dim": cfg.head_dim, "ffn": cfg.ffn,
                   "window": "+-1 frame, text rows dense",
                   "parallelism": f"ulysses sp{world} (all-to-all exchange)" if world > 1 else "single GPU",
                   "l2": "per-step working set (weights 23 GB, activations > 1 GB) larger than L2",
                   "latent_finite_after_timing": finite},
        "e2e": {"value": round(T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": v_host.numel() * 2 + t_host.numel() * 2,
                "d2h_bytes_per_step": out_host.numel() * 2, "steps": e2e_steps, "copies": "per step; serial"},
        "gpu_launches": launches * args.steps,
        "launch": "eager",
        "roofline": {"bound": "tensor", "kernel": "mxfp8_gemm (QKV, %d x 15360 x 5120)" % n,
                     "achieved": round(achieved, 1), "peak": round(fp8_peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / fp8_peak, 4), "traffic": None,
                     "peak_source": f"2 x {src} bf16 dense ({pk['bf16_tflops']}): the FP8 rate",
                     "algorithmic_flops_per_launch": gemm_flops},
        "kernels_ms": {k_: round(v_, 4) for k_, v_ in kt.items()},
        "clocks": clk.summary(),
    }
    if runtime is not None:
        runtime.close()
    return rec


def cpu_baseline_stack(threads):
    """The block CPU baseline divided over the stack's depth (per-token work of one step)."""
    base = cpu_baseline_block(threads)
    base["value"] = round(base["value"] / STACK_CFG["depth"], 3)
    base["sample"] = ("reference block composition, 3 frames x 1560 tokens, divided by the 40 blocks "
                      "of one denoise step (text rows not included)")
    return base


CPU_BASELINES = {"block": cpu_baseline_block, "vda": cpu_baseline_vda, "gemm": cpu_baseline_gemm,
                 "stack": cpu_baseline_stack}


# ---------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="block", choices=["block", "vda", "gemm", "stack"])
    ap.add_argument("--rows", type=int, default=0, help="gemm: M override (small profiling case)")
    ap.add_argument("--frames", type=int, default=0, help="vda / stack: frame-count override (small case)")
    ap.add_argument("--depth", type=int, default=0, help="stack: block-count override (small case)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="block, N = 1: skip the config-2 / config-1 sub-records")
    ap.add_argument("--eager", action="store_true", help="block: launch eagerly instead of a CUDA graph")
    ap.add_argument("--softmax-ranks", type=int, default=0,
                    help="block, N > 1: branch-parallel layout with this many softmax ranks (needs --eager)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    threads = os.cpu_count() or 1

    if args.impl == "reference":
        if rank != 0:
            return
        import torch
        torch.set_num_threads(threads)
        fn = CPU_BASELINES[args.workload]
        steps, warmup = max(1, min(args.steps, 3)), 1
        for _ in range(warmup):
            fn(threads)
        vals = sorted(fn(threads)["value"] for _ in range(steps))
        base = fn(threads)
        base["value"] = vals[len(vals) // 2]
        if args.workload == "block":
            meta = dict(metric="hybrid-block tokens/s (BASELINE config 3, 32760 tokens)",
                        unit="tokens/s", scaling="strong",
                        config={"workload": "hybrid_block_config3", **BLOCK_CFG})
        elif args.workload == "stack":
            meta = dict(metric="denoise-loop tokens/s (BASELINE config 4: 40-block stack, 60 x 1560 video + "
                               "512 text rows)", unit="tokens/s", scaling="strong",
                        config={"workload": "denoise_stack_config4", **STACK_CFG})
        elif args.workload == "gemm":
            meta = dict(metric="MXFP8 GEMM TFLOP/s, BASELINE config 1 sweep (activation quantised each step)",
                        unit="TFLOP/s", scaling="weak",
                        config={"workload": "gemm_config1", "m": GEMM_ROWS,
                                "shapes": [[n, k] for _, n, k in GEMM_SHAPES]})
        else:
            meta = dict(metric="VDA branch HBM GB/s (algorithmic bytes), BASELINE config 2",
                        unit="GB/s", scaling="weak", config={"workload": "vda_config2", **VDA_CFG})
        print(json.dumps({
            "impl": "reference", "metric": meta["metric"], "value": base["value"], "unit": meta["unit"],
            "n_gpus": args.gpus, "steps": steps, "warmup": warmup, "higher_is_better": True,
            "scaling": meta["scaling"], "vs_baseline": None, "dtype": "fp32 (CPU reference port)",
            "data": "synthetic", "config": meta["config"], "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": meta["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return

    import torch
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        from datetime import timedelta
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist_mod.init_process_group("nccl", timeout=timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        dist = dist_mod
    else:
        torch.cuda.set_device(0)
    if args.workload == "block":
        rec = bench_block(args, torch, dist, rank, world)
    elif args.workload == "stack":
        rec = bench_stack(args, torch, dist, rank, world)
    elif args.workload == "gemm":
        rec = bench_gemm(args, torch, dist, rank, world)
    else:
        rec = bench_vda(args, torch, dist, rank, world)
    if rank == 0:
        if not args.no_cpu_baseline:
            torch.set_num_threads(threads)
            rec["cpu_baseline"] = CPU_BASELINES[args.workload](threads)
        print(json.dumps(rec))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
