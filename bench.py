"""Benchmark: retrieval block-sparse decode attention on B200.

Metric: sparse decode-attention microseconds per layer, with
the achieved HBM GB/s of the decode kernel against the measured roofline.

Workload (every N): config 4, the 1M-token configuration the scaling target
is quoted on -- batch 1, 32 query heads, 8 kv heads, head_dim 128, context
1,048,576 tokens, 8-bit affine group-64 KV with bf16 scales and biases, block
64 (16384 blocks), top-256 blocks + the recent block, 64 planted needle blocks
and a slow drift of the mean key, 36 independent layers per decode step. Each
layer's step is the sparse branch of attentionWithCacheUpdate: append the new
token (row 1,048,575), score 16383 candidate blocks, select, attend, write
out. After a step the cache is trimmed by one token (host bookkeeping), so
every step sees the same context. Inputs are synthetic (seeded) and
device-resident; a step moves 36 x 69.4 MB, far more than the 126 MB L2, so no
flush is needed.

N > 1 (torchrun, one process per GPU): the same workload sequence-sharded
(block j on rank j % N) through the fused peer-memory step -- one launch per
layer and GPU that exchanges the top-K candidates and the (m, l, o) partials
with the other shards over NVLink. The total work is fixed: strong scaling of
the per-layer latency. Outside the timed region every rank's selection and
output of layer 0 are gathered and compared with each other and with a
single-GPU decode of the same layer on rank 0; a mismatch exits non-zero.

`--impl reference` times the CPU implementation of the path
(oracle/sd_cpu_baseline.cpp, every host thread) on the same workload: the
reference's own implementation (Swift + MLX) cannot run on this machine.
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
import threading
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


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled about every
    millisecond during the timed region by a host thread through NVML
    (read-only queries); nvidia-smi at 100 ms when NVML is unavailable."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.cuda_index).uuid)
        want = uuid.replace("GPU-", "")
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            u = pynvml.nvmlDeviceGetUUID(h)
            u = u.decode() if isinstance(u, bytes) else u
            if u.replace("GPU-", "") == want:
                return h
        return pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        try:
            import pynvml
            h = self._handle()
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def loop():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        why = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((float(mhz), int(why)))
                    except Exception:
                        pass
                    time.sleep(0.001)

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
            try:
                q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                     "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                     "clocks_event_reasons.sw_power_cap")
                self._proc = subprocess.Popen(["nvidia-smi", "-i", str(self.cuda_index), f"--query-gpu={q}",
                                               "--format=csv,noheader,nounits", "-lms", "100"],
                                              stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except (FileNotFoundError, OSError):
                self._proc = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
        if self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            for l in out.splitlines():
                f = [x.strip() for x in l.split(",")]
                if len(f) < 6:
                    continue
                try:
                    bits = sum(self.REASONS[n] for n, v in zip(self.REASONS, f[2:6]) if v.lower() == "active")
                    self.samples.append((float(f[0]), bits))
                    self.max_mhz = float(f[1])
                except ValueError:
                    continue

    def summary(self) -> dict:
        sm = [m for m, _ in self.samples]
        reasons = sorted(n for n, bit in self.REASONS.items() if any(w & bit for _, w in self.samples))
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "source": "nvml" if self._proc is None else "nvidia-smi"}


# ---------------------------------------------------------------------------
def build_layers(w, n_layers: int, rank: int, world: int, seed0: int = 1000):
    """One SparseIndex per layer holding T-1 prefilled rows (this rank's
    blocks), plus each layer's step inputs (q, k_new, v_new) on the device."""
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
                       "v_new": v[:, :, w.T - 1].contiguous(), "out": torch.empty_like(case["q"]),
                       "seed": seed0 + l})
        del case, k, v
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return layers


# ---------------------------------------------------------------------------
# CPU implementation (oracle/sd_cpu_baseline.cpp) on the same workload
# ---------------------------------------------------------------------------
def _np_from_dev(t):
    """Device tensor -> numpy storage array (bf16/fp16 as uint16 bits, int32 codes as uint32)."""
    import numpy as np
    import torch
    t = t.contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).cpu().numpy().view(np.uint16 if t.dtype == torch.bfloat16 else np.float16)
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().numpy()


def cpu_inputs_from_index(w, idx, q) -> dict:
    """The oracle's view of a GPU layer: its arena arrays copied to the host."""
    import oracle
    from sparse_decode.synth import DTYPE_CODE
    dt = DTYPE_CODE[w.dtype]
    v = idx.views()
    if w.bits:
        Kc = oracle.Cache(dt, w.D, _np_from_dev(v["k"]), w.bits, _np_from_dev(v["k_scales"]),
                          _np_from_dev(v["k_biases"]))
        Vc = oracle.Cache(dt, w.D, _np_from_dev(v["v"]), w.bits, _np_from_dev(v["v_scales"]),
                          _np_from_dev(v["v_biases"]))
    else:
        Kc, Vc = oracle.Cache(dt, w.D, _np_from_dev(v["k"])), oracle.Cache(dt, w.D, _np_from_dev(v["v"]))
    return {"q": _np_from_dev(q), "K": Kc, "V": Vc, "summ": _np_from_dev(v["summaries"]), "dt": dt}


def cpu_inputs_generated(w, seed: int) -> dict:
    """The same recipe generated on the host (torch's CPU generator), for the
    CPU-only reference arm: quantized and summarised by the oracle."""
    import numpy as np
    import torch

    import oracle
    from sparse_decode.synth import DTYPE_CODE, make_case_torch
    oracle.lib().orc_set_threads(0)
    dt = DTYPE_CODE[w.dtype]
    c = make_case_torch(w, seed, device="cpu")
    BH = w.B * w.Hkv

    def st(t):
        t = t.contiguous()
        return t.view(torch.int16).numpy().view(np.uint16) if w.dtype == "bf16" else t.numpy()

    ks = st(c["k"]).reshape(BH, w.T, w.D)
    vs = st(c["v"]).reshape(BH, w.T, w.D)
    if w.bits:
        kq, vq = oracle.quantize(ks, dt, w.D, w.bits), oracle.quantize(vs, dt, w.D, w.bits)
        Kc = oracle.Cache(dt, w.D, kq[0], w.bits, kq[1], kq[2])
        Vc = oracle.Cache(dt, w.D, vq[0], w.bits, vq[1], vq[2])
    else:
        Kc, Vc = oracle.Cache(dt, w.D, ks), oracle.Cache(dt, w.D, vs)
    return {"q": st(c["q"]), "K": Kc, "V": Vc, "summ": oracle.summaries(Kc, w.T, w.S, dt), "dt": dt}


def cpu_time(w, inp: dict, seconds: float, threads: int):
    """Repeat the CPU decode of one layer for about `seconds`; returns
    (us per layer, repetitions, threads that ran tasks, out, sel)."""
    import oracle
    scale = 1.0 / math.sqrt(w.D)
    args = (inp["q"], inp["dt"], inp["K"], inp["V"], inp["summ"], inp["dt"], w.B, w.Hq, w.Hkv, w.T, w.S, w.K, scale)
    out, sel = oracle.decode_f32(*args, threads=threads)
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.decode_f32(*args, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return el / n * 1e6, n, oracle.last_threads(), out, sel


def cpu_sample(w, seconds: float, threads: int):
    """Time the CPU decode of one generated layer of `w` (small configs and the
    reference arm's fallback); returns (us per layer, repetitions)."""
    us, n, _, _, _ = cpu_time(w, cpu_inputs_generated(w, 77), seconds, threads)
    return us, n


def run_reference(args, w, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = _host_threads()
    t0 = time.time()
    inp = cpu_inputs_generated(w, 1000)
    setup_s = time.time() - t0
    per = max(1.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_time(w, inp, 0.0, threads)
    vals, used = [], 0
    for _ in range(args.steps):
        us, _, used, _, _ = cpu_time(w, inp, per, threads)
        vals.append(us)
    v = statistics.median(vals)
    line = {"metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(v * w.layers / 1000, 4), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
            "data": "synthetic (seeded N(0,1) Q/K/V, planted needle blocks)", "impl": "reference",
            "config": _config(w, world, gpu=False),
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": used, "kind": "port",
                             "sample": f"one layer per repetition ({w.name}), median of {args.steps} samples of "
                                       f"~{per:.0f}s after {setup_s:.0f}s of input set-up; the reference (Swift + "
                                       "MLX) cannot run here, so the CPU implementation of the path "
                                       "(oracle/sd_cpu_baseline.cpp, fp32, AVX2, thread pool) stands in"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _config(w, world: int = 1, gpu: bool = True) -> dict:
    """The workload keys (both arms) plus, for the GPU arm, how it ran."""
    from sparse_decode.synth import algorithmic_bytes
    b = algorithmic_bytes(w)
    c = {"workload": w.name, "batch": w.B, "q_heads": w.Hq, "kv_heads": w.Hkv, "head_dim": w.D,
         "context": w.T, "block": w.S, "top_k": w.K, "kv_bits": w.bits, "layers_per_step": w.layers}
    if gpu:
        c["parallelism"] = f"sequence-sharded x{world} (fused peer-memory exchange)" if world > 1 else "single GPU"
        c["l2"] = (f"inputs larger than L2 ({w.layers} layers x {b / 1e6:.1f} MB per step)"
                   if w.layers * b > 126e6 else
                   f"inputs smaller than L2 ({w.layers} layers x {b / 1e6:.1f} MB): not a bench line")
        c["cuda_graph"] = True
    return c


def _rel_err(a, b) -> float:
    import numpy as np
    a = np.asarray(a, np.float64).reshape(-1, b.shape[-1])
    b = np.asarray(b, np.float64).reshape(-1, b.shape[-1])
    return float((np.sqrt(((a - b) ** 2).sum(-1)) / np.maximum(np.sqrt((b ** 2).sum(-1)), 1e-30)).max())


def _to_f32(t):
    return t.float().cpu().numpy()


# ---------------------------------------------------------------------------
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4")
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

    def decode_layer(L, q, kn, vn, out, sel=None):
        if comm is None:
            L["idx"].decode(q, kn, vn, scale, out=out, sel_out=sel)
        else:
            L["idx"].shard_decode(comm, q, kn, vn, scale, out=out, sel_out=sel)

    # Capture the single-layer launches of one step in a CUDA graph; the
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

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
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

    # ---- layer 0 once more, eagerly, with its selection (outside the timed regions) ----
    L0 = layers[0]
    sel0 = torch.full((w.B * w.Hkv, w.K + 1), -7, dtype=torch.int32, device="cuda")
    out0 = torch.empty_like(L0["q"])
    decode_layer(L0, L0["q"], L0["k_new"], L0["v_new"], out0, sel0)
    torch.cuda.synchronize()
    L0["idx"].trim(1)
    check = None
    if world > 1:
        check = _check_shards(w, dist, rank, world, L0, sel0, out0, scale)
        if not check["ok"]:
            if rank == 0:
                print(json.dumps({"error": "sharded decode disagrees", "check": check}), flush=True)
            graph = None
            comm.close()
            dist.destroy_process_group()
            raise SystemExit(3)

    # ---- roofline of the decode kernel ----
    peak1, peak_kind = _peaks()
    peak = peak1 * world
    bytes_layer = algorithmic_bytes(w)
    achieved = bytes_layer / (us_layer * 1e-6) / 1e9  # GB/s (whole job, all ranks' bytes)
    traffic = _traffic("decode_kernel", w.name)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = _host_threads()
        inp = cpu_inputs_from_index(w, L0["idx"], L0["q"])
        cpu_us, reps, used, cout, csel = cpu_time(w, inp, args.cpu_seconds, threads)
        import numpy as np
        n_sel = w.n_sel
        cpu = {"value": round(cpu_us, 2), "unit": UNIT, "cores": used, "kind": "port",
               "sample": f"{reps} single-layer decodes of layer 0 of the same workload (its arrays copied from "
                         f"the GPU, ~{args.cpu_seconds:.0f}s) through oracle/sd_cpu_baseline.cpp in fp32 on "
                         f"{used} host threads; the reference (Swift + MLX) cannot run here",
               "selection_equal_to_gpu": bool(np.array_equal(csel, sel0.cpu().numpy()[:, :n_sel])),
               "output_rel_err_vs_gpu": round(_rel_err(_to_f32(out0), cout.astype(np.float32)
                                                       if cout.dtype != np.uint16 else
                                                       (cout.astype(np.uint32) << 16).view(np.float32)), 6)}
    if rank == 0:
        line = {"metric": METRIC, "value": round(us_layer, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
                "data": "synthetic (seeded N(0,1) Q/K/V, planted needle blocks)",
                "config": _config(w, world),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "GB/s",
                             "frac": round(achieved / peak, 4), "traffic": traffic,
                             "peak_kind": f"{peak_kind}" + (f" x {world} GPUs" if world > 1 else ""),
                             "algorithmic_bytes_per_layer": bytes_layer,
                             "note": "per-layer time includes inter-launch gaps inside the CUDA graph"},
                "e2e": {"value": round(e2e_us, 4), "unit": UNIT,
                        "h2d_bytes_per_step": n_in * esz, "d2h_bytes_per_step": n_out * esz},
                "gpu_launches": args.steps * w.layers,
                "clocks": clk.summary()}
        if check is not None:
            line["multi_gpu_check"] = check
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graph
    if comm is not None:
        comm.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def _check_shards(w, dist, rank: int, world: int, L0, sel0, out0, scale) -> dict:
    """Every rank's selection and output of layer 0 must be identical, and
    equal to what the timed graph replays left in layer 0's output; rank 0
    also decodes layer 0 on one GPU (a single-shard index of the same data)
    and compares: selection equal, output within 2e-3 (normwise)."""
    import numpy as np
    import torch
    from sparse_decode import SparseIndex
    from sparse_decode.synth import make_case_torch
    sels = [torch.empty_like(sel0) for _ in range(world)]
    outs = [torch.empty_like(out0) for _ in range(world)]
    dist.all_gather(sels, sel0)
    dist.all_gather(outs, out0)
    same_sel = all(torch.equal(s, sels[0]) for s in sels)
    same_out = all(torch.equal(o, outs[0]) for o in outs)
    # the timed CUDA-graph replays (launches overlapping across layers) left
    # layer 0's output of the same token: the same bits as the eager decode
    graph_ok = torch.tensor([1 if torch.equal(L0["out"], out0) else 0], device="cuda")
    dist.all_reduce(graph_ok, op=dist.ReduceOp.MIN)
    graph_same = bool(graph_ok.item())
    ref_sel_ok, ref_err = True, 0.0
    if rank == 0:
        case = make_case_torch(w, seed=L0["seed"])
        one = SparseIndex(w.B, w.Hq, w.Hkv, w.D, w.S, w.K, w.T, w.dtype, w.bits)
        one.append(case["k"][:, :, : w.T - 1].contiguous(), case["v"][:, :, : w.T - 1].contiguous())
        s1 = torch.full_like(sel0, -7)
        o1 = one.decode(case["q"].contiguous(), case["k"][:, :, w.T - 1].contiguous(),
                        case["v"][:, :, w.T - 1].contiguous(), scale, sel_out=s1)
        torch.cuda.synchronize()
        ref_sel_ok = bool(torch.equal(s1, sel0))
        ref_err = _rel_err(_to_f32(out0), _to_f32(o1))
        del one, case
        torch.cuda.empty_cache()
    flag = torch.tensor([1 if (same_sel and same_out and graph_same and ref_sel_ok and ref_err <= 2e-3) else 0],
                        device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return {"ok": bool(flag.item()), "ranks_same_selection": same_sel, "ranks_same_output": same_out,
            "graph_replay_equal_to_eager": graph_same,
            "selection_equal_to_single_gpu": ref_sel_ok, "output_rel_err_vs_single_gpu": round(ref_err, 6),
            "layer": 0}


if __name__ == "__main__":
    main()
