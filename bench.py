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
  vda   BASELINE config 2: the VDA branch, H=40, d=128, 21 frames x 1560 tokens,
        metric = algorithmic HBM GB/s (q, k, v, gate, beta, alpha in; out).
        Multi-GPU: heads are independent, each rank runs its head shard (no
        collective on the data path): weak scaling over 40/N heads... per rank
        the full 40 heads (replica-free weak scaling: fixed work per GPU).
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

    # Per-kernel device times of the five stage launches (same stream).
    plane = F * H * d * d
    up = lambda b: (b + 255) // 256 * 256
    A = ws[: plane * 4].view(torch.float32)
    B = ws[up(plane * 4): up(plane * 4) + plane * 4].view(torch.float32)
    pre = ws[2 * up(plane * 4): 2 * up(plane * 4) + plane * 4].view(torch.float32)
    suf = ws[3 * up(plane * 4): 3 * up(plane * 4) + plane * 4].view(torch.float32)
    state = ws[4 * up(plane * 4): 4 * up(plane * 4) + plane * 2]
    sf = S * q.stride(0)
    launches = [
        ("statistics", lambda: _lib.call("vdn_vda_statistics", _lib.ptr(k), sf, q.stride(0), q.stride(1),
                                         _lib.ptr(v), sf, q.stride(0), q.stride(1), _lib.ptr(beta),
                                         S * beta.stride(0), beta.stride(0), beta.stride(1), 0, F, S, H,
                                         d, _lib.ptr(A), _lib.ptr(B), st)),
        ("factors", lambda: _lib.call("vdn_delta_factors", _lib.ptr(A), _lib.ptr(B), _lib.ptr(alpha),
                                      F * H, d, _lib.ptr(pre), _lib.ptr(suf), st)),
        ("scan", lambda: _lib.call("vdn_vda_scan", _lib.ptr(pre), _lib.ptr(suf), None, F, H, d,
                                   _lib.ptr(A), _lib.ptr(B), st)),
        ("gather", lambda: _lib.call("vdn_vda_gather", _lib.ptr(A), _lib.ptr(B), _lib.ptr(alpha), buf,
                                     None, 1, F, H, d, _lib.ptr(state), _lib.DTYPE_BF16, st)),
        ("readout", lambda: _lib.call("vdn_vda_readout", _lib.ptr(q), sf, q.stride(0), q.stride(1),
                                      _lib.ptr(state), _lib.ptr(gate), S * gate.stride(0), gate.stride(0),
                                      gate.stride(1), _lib.ptr(w), 1e-6, F, S, H, d, _lib.ptr(out), st)),
    ]
    kt = kernel_times(torch, launches, 5, stream)
    n_tok_h_d = n * H * d
    algo = {  # algorithmic bytes per launch
        "statistics": 2 * n_tok_h_d * 2 + n * H * 2 + 2 * F * H * d * d * 4,
        "factors": 2 * F * H * d * d * 4 + F * H * d * 4 + 2 * F * H * d * d * 4,
        "scan": 2 * F * H * d * d * 4 + 2 * F * H * d * d * 4,
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
                     "traffic": None, "peak_source": src,
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


# ---------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="vda", choices=["vda"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    threads = os.cpu_count() or 1

    if args.impl == "reference":
        if rank != 0:
            return
        import numpy as np  # noqa: F401
        os.environ.setdefault("OMP_NUM_THREADS", str(threads))
        times = []
        for _ in range(args.warmup):
            cpu_baseline_vda(threads)
        for _ in range(args.steps):
            times.append(cpu_baseline_vda(threads)["value"])
        value = sorted(times)[len(times) // 2]
        base = cpu_baseline_vda(threads)
        base["value"] = value
        print(json.dumps({
            "impl": "reference", "metric": "VDA branch HBM GB/s (algorithmic bytes), BASELINE config 2",
            "value": value, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp64/fp32 (numpy oracle)", "data": "synthetic",
            "config": {"workload": "vda_config2", **VDA_CFG},
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        from datetime import timedelta
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist_mod.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        dist = dist_mod
    else:
        torch.cuda.set_device(0)
    rec = bench_vda(args, torch, dist, rank, world)
    if rank == 0:
        if not args.no_cpu_baseline:
            rec["cpu_baseline"] = cpu_baseline_vda(threads)
        print(json.dumps(rec))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
