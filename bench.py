"""Benchmark: retrieval block-sparse decode attention on B200.

Metric: sparse decode-attention microseconds per layer, with
the achieved HBM GB/s of the decode kernel against the measured roofline.

Workload (N = 1): config 1, Qwen3-4B-shaped decode attention -- bf16 KV,
batch 1, 32 query heads, 8 kv heads, head_dim 128, context 32768 tokens,
block 64 (512 blocks), top-64 blocks + the recent block, 36 independent
layers per decode step, 16 planted needle blocks. Each layer's step is the
sparse branch of attentionWithCacheUpdate: append the new token (row 32767),
score 511 candidate blocks, select, attend, write out. After a step the
cache is trimmed by one token (host bookkeeping), so every step sees the
same context. Inputs are synthetic (seeded) and device-resident; a step
moves 36 x 18.1 MB, larger than the 126 MB L2, so no flush is needed.

N > 1 (torchrun, one process per GPU): the same workload sequence-sharded
(block j on rank j % N) through the fused peer-memory step -- one launch per
layer and GPU that exchanges the top-K candidates and the (m, l, o) partials
with the other shards over NVLink: strong scaling of the per-layer latency.

`--impl reference` times the CPU restatement of the path (oracle/, all host
threads) on the same workload: the reference's own implementation (Swift +
MLX) cannot run on this machine.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "mlx-swift-lm_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "sparse decode-attn us/layer (achieved HBM GB/s vs roofline in `roofline`)"
UNIT = "us/layer"


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    f = ROOT / "profiles" / f"{kernel}_{workload}.txt"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
def build_layers(w, n_layers: int, rank: int, world: int, seed0: int = 1000):
    """One SparseIndex per layer holding T-1 prefilled rows; plus each layer's
    step inputs (q, k_new, v_new) on the device."""
    import torch
    from sparse_decode import SparseIndex
    from sparse_decode.synth import make_case_torch
    layers = []
    for l in range(n_layers):
        case = make_case_torch(w, seed=seed0 + l)
        idx = SparseIndex(w.B, w.Hq, w.Hkv, w.D, w.S, w.K, w.T, w.dtype, w.bits, shard_rank=rank, shard_count=world)
        k, v = case["k"], case["v"]
        idx.append(k[:, :, : w.T - 1].contiguous(), v[:, :, : w.T - 1].contiguous())
        idx.set_launch_overlap(True)
        layers.append({"idx": idx, "q": case["q"].contiguous(), "k_new": k[:, :, w.T - 1].contiguous(),
                       "v_new": v[:, :, w.T - 1].contiguous(), "out": torch.empty_like(case["q"])})
        del case, k, v
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return layers


def cpu_sample(w, seconds: float, threads: int):
    """Time the oracle's fp32 decode of one config-shaped layer on the host."""
    import numpy as np

    import oracle
    from sparse_decode.synth import DTYPE_CODE, make_case
    c = make_case(w, seed=77)
    dt = DTYPE_CODE[w.dtype]
    BH = w.B * w.Hkv
    ks = oracle.to_storage(c["k"].reshape(BH, w.T, w.D), dt)
    vs = oracle.to_storage(c["v"].reshape(BH, w.T, w.D), dt)
    qs = oracle.to_storage(c["q"], dt)
    Kc, Vc = oracle.Cache(dt, w.D, ks), oracle.Cache(dt, w.D, vs)
    oracle.lib().orc_set_threads(threads)
    summ = oracle.summaries(Kc, w.T, w.S, dt)
    scale = 1.0 / math.sqrt(w.D)
    oracle.decode_f32(qs, dt, Kc, Vc, summ, dt, w.B, w.Hq, w.Hkv, w.T, w.S, w.K, scale, threads)
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.decode_f32(qs, dt, Kc, Vc, summ, dt, w.B, w.Hq, w.Hkv, w.T, w.S, w.K, scale, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return el / n * 1e6, n


def run_reference(args, w, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    per = max(1.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_sample(w, 0.0, threads)
    vals = []
    for _ in range(args.steps):
        us, _ = cpu_sample(w, per, threads)
        vals.append(us)
    v = statistics.median(vals)
    line = {"metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(v * w.layers / 1000, 4), "higher_is_better": False,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": w.dtype,
            "data": "synthetic (seeded N(0,1) Q/K/V, planted needle blocks)", "impl": "reference",
            "config": {"workload": w.name, "batch": w.B, "q_heads": w.Hq, "kv_heads": w.Hkv, "head_dim": w.D,
                       "context": w.T, "block": w.S, "top_k": w.K, "layers_per_step": w.layers},
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"one layer per timed repetition, median of {args.steps} samples of ~{per:.0f}s; "
                                       "the reference (Swift + MLX) cannot run here, so the CPU restatement "
                                       "of the path (oracle/sd_oracle.cpp, fp32, all host threads) stands in"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c1")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    from sparse_decode.synth import CONFIGS, algorithmic_bytes
    w = CONFIGS[args.config]
    if args.layers:
        w = w.with_(layers=args.layers)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")

    if args.impl == "reference":
        run_reference(args, w, rank, world)
        return

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import sparse_decode
    sparse_decode.lib()

    layers = build_layers(w, w.layers, rank, world)
    stream = torch.cuda.current_stream()
    scale = 1.0 / math.sqrt(w.D)
    # Several GPUs: the fused sequence-sharded step, one launch per layer and
    # GPU that exchanges candidates and partials through peer memory (all
    # layers share one exchange area).
    comm = sparse_decode.ShardComm(layers[0]["idx"]) if world > 1 else None
    if dist:
        dist.barrier()

    def decode_layer(L, q, kn, vn, out):
        if comm is None:
            L["idx"].decode(q, kn, vn, scale, out=out)
        else:
            L["idx"].shard_decode(comm, q, kn, vn, scale, out=out)

    # Capture the 36 single-layer launches of one step in a CUDA graph; the
    # launches are identical every step because the step's token is trimmed
    # again afterwards.
    for L in layers:
        decode_layer(L, L["q"], L["k_new"], L["v_new"], L["out"])
    for L in layers:
        L["idx"].trim(1)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for L in layers:
            decode_layer(L, L["q"], L["k_new"], L["v_new"], L["out"])
    for L in layers:
        L["idx"].trim(1)

    def run_step():
        graph.replay()

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            run_step()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / args.steps
    us_layer = ms_step * 1000.0 / w.layers
    err = sum(L["idx"].check_device() for L in layers)
    if err:
        raise SystemExit(f"device error word set: {err}")

    # ---- end to end through the public API with host buffers ----
    import numpy as np
    esz = 2 if w.dtype != "f32" else 4
    n_in = sum(L["q"].numel() + L["k_new"].numel() + L["v_new"].numel() for L in layers)
    n_out = sum(L["q"].numel() for L in layers)
    h_in = torch.empty(n_in, dtype=layers[0]["q"].dtype, pin_memory=True)
    h_out = torch.empty(n_out, dtype=layers[0]["q"].dtype, pin_memory=True)
    d_in = torch.empty(n_in, dtype=layers[0]["q"].dtype, device="cuda")
    d_out = torch.empty(n_out, dtype=layers[0]["q"].dtype, device="cuda")
    views, o = [], 0
    for L in layers:
        parts = []
        for name in ("q", "k_new", "v_new"):
            n = L[name].numel()
            parts.append(d_in[o:o + n].view(L[name].shape))
            h_in[o:o + n].copy_(L[name].reshape(-1).cpu())
            o += n
        views.append(parts)
    outs, o = [], 0
    for L in layers:
        n = L["q"].numel()
        outs.append(d_out[o:o + n].view(L["q"].shape))
        o += n

    def e2e_step():
        d_in.copy_(h_in, non_blocking=True)
        for L, (q, kn, vn), out in zip(layers, views, outs):
            decode_layer(L, q, kn, vn, out)
        h_out.copy_(d_out, non_blocking=True)
        for L in layers:
            L["idx"].trim(1)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e_us = ems / args.steps * 1000.0 / w.layers

    # ---- roofline of the decode kernel ----
    peak, peak_kind = _peaks()
    bytes_layer = algorithmic_bytes(w)
    achieved = bytes_layer / (us_layer * 1e-6) / 1e9  # GB/s (whole job, all ranks' bytes)
    traffic = _traffic("decode_kernel", w.name)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        cpu_us, reps = cpu_sample(w, args.cpu_seconds, threads)
        cpu = {"value": round(cpu_us, 2), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{reps} single-layer decodes of the same workload shape (one layer, ~{args.cpu_seconds:.0f}s) "
                         "through oracle/sd_oracle.cpp in fp32 on all host threads; the reference (Swift + MLX) "
                         "cannot run here"}
    if rank == 0:
        line = {"metric": METRIC, "value": round(us_layer, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": False,
                "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": w.dtype,
                "data": "synthetic (seeded N(0,1) Q/K/V, planted needle blocks)",
                "config": {"workload": w.name, "batch": w.B, "q_heads": w.Hq, "kv_heads": w.Hkv, "head_dim": w.D,
                           "context": w.T, "block": w.S, "top_k": w.K, "layers_per_step": w.layers,
                           "parallelism": f"sequence-sharded x{world} (fused peer-memory exchange)" if world > 1
                           else "single GPU",
                           "l2": f"inputs larger than L2 ({w.layers} layers x {bytes_layer / 1e6:.1f} MB per step)"
                                 if w.layers * bytes_layer > 126e6 else
                                 f"inputs smaller than L2 ({w.layers} layers x {bytes_layer / 1e6:.1f} MB): not a bench line",
                           "cuda_graph": True},
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                             "algorithmic_bytes_per_layer": bytes_layer,
                             "note": "per-layer time includes inter-launch gaps inside the CUDA graph"},
                "e2e": {"value": round(e2e_us, 4), "unit": UNIT,
                        "h2d_bytes_per_step": n_in * esz, "d2h_bytes_per_step": n_out * esz},
                "gpu_launches": args.steps * w.layers,
                "clocks": clk.summary()}
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graph
    if comm is not None:
        comm.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
