"""Per-phase timing of the decode kernel inside CUDA-graph replays.

Uses the phase-timing build of the library (libsparse_decode_phases.so, see
sparse_decode.build): thread 0 of every CTA stamps %globaltimer at entry and
exit and clock64 at the phase boundaries (entry, scoring start, scoring end,
selection end, attention end, merge end). This module builds `layers`
independent single-layer indexes of a workload exactly as bench.py does,
captures one decode step of all of them in a CUDA graph, replays it, and
reports per phase the median and maximum over CTAs (microseconds, clock64
cycles converted with each CTA's own cycles-per-ns), sub-phases of the
selection, attention and merge (medians; a sub-phase whose stamps a path
does not write is left out), plus the layer cadence seen by %globaltimer.

    python -m sparse_decode.phase_profile --config c1 --layers 36

Run from mlx-swift-lm_b200/ (or with it on sys.path); needs a GPU. Under
torchrun (WORLD_SIZE > 1) every rank profiles its shard of the layers through
the fused peer-memory step, and rank 0 reports its own CTAs:

    torchrun --nproc-per-node 2 -m sparse_decode.phase_profile --config c4 --layers 8
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
from pathlib import Path

PHASES = ["prologue", "score", "select", "attend", "merge"]
# sub-phases: (name, from slot, to slot) -- see SD_STAMP_* in csrc/sd_device.cuh
SUBPHASES = [("select.local_or_cluster_wait", 3, 15), ("select.exchange_or_topk", 15, 14), ("select.rest", 14, 4),
             ("attend.first_fill_issued", 4, 8), ("attend.warp0_first_tile", 4, 9), ("attend.warp0_tiles", 9, 10),
             ("attend.tail", 10, 5), ("merge.cta_partial", 5, 11), ("merge.store", 11, 12),
             ("merge.gather", 12, 13), ("merge.output", 13, 6),
             ("sliced.keys64", 3, 16), ("sliced.local_list", 16, 15), ("sliced.union_hist", 14, 17),
             ("sliced.union_kth", 17, 18), ("sliced.list_check", 18, 19), ("sliced.picks", 19, 20),
             ("sliced.after_picks", 20, 4), ("attend.proxy_fences", 4, 21), ("attend.first_issue", 21, 22),
             ("attend.warp0_unit0", 9, 23), ("attend.warp0_unit8_on", 23, 10)]


def _load_phase_lib():
    from . import build as b
    # SPARSE_DECODE_LIB may name another phase-timing build to profile
    path = os.environ.get("SPARSE_DECODE_LIB") or (b.LIB_PHASES if b.LIB_PHASES.exists()
                                                   else b.build(phase_timing=True))
    os.environ["SPARSE_DECODE_LIB"] = str(path)
    import sparse_decode
    if sparse_decode._lib is not None and not hasattr(sparse_decode._lib, "sd_debug_set_phase_buffer"):
        raise RuntimeError("the product library is already loaded in this process")
    L = sparse_decode.lib()
    L.sd_debug_set_phase_buffer.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    L.sd_debug_set_phase_buffer.restype = ctypes.c_int32
    L.sd_debug_grid.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]
    L.sd_debug_grid.restype = ctypes.c_int32
    L.sd_debug_set_l2_plain.argtypes = [ctypes.c_void_p, ctypes.c_int32]
    L.sd_debug_set_l2_plain.restype = ctypes.c_int32
    return L


def profile(config: str, layers: int, warmup: int = 3, overlap: bool = True, l2_plain: bool = False) -> dict:
    import torch

    L = _load_phase_lib()
    from sparse_decode import ShardComm, SparseIndex, _check
    from sparse_decode.synth import CONFIGS, algorithmic_bytes, make_case_torch

    # under torchrun: this rank's shard of every layer, the fused peer-memory step
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    w = CONFIGS[config].with_(layers=layers)
    scale = 1.0 / math.sqrt(w.D)
    items = []
    for l in range(layers):
        case = make_case_torch(w, seed=1000 + l)
        idx = SparseIndex(w.B, w.Hq, w.Hkv, w.D, w.S, w.K, w.T, w.dtype, w.bits, shard_rank=rank,
                          shard_count=world)
        k, v = case["k"], case["v"]
        idx.append(k[:, :, : w.T - 1].contiguous(), v[:, :, : w.T - 1].contiguous())
        idx.set_launch_overlap(overlap)
        _check(L.sd_debug_set_l2_plain(idx._h, 1 if l2_plain else 0))
        gx, gy = ctypes.c_int32(), ctypes.c_int32()
        _check(L.sd_debug_grid(idx._h, ctypes.byref(gx), ctypes.byref(gy)))
        buf = torch.zeros((gy.value, gx.value, 24), dtype=torch.int64, device="cuda")
        _check(L.sd_debug_set_phase_buffer(idx._h, ctypes.c_void_p(buf.data_ptr())))
        items.append({"idx": idx, "q": case["q"].contiguous(), "k": k[:, :, w.T - 1].contiguous(),
                      "v": v[:, :, w.T - 1].contiguous(), "out": torch.empty_like(case["q"]), "buf": buf})
        del case, k, v
    torch.cuda.synchronize()
    comm = ShardComm(items[0]["idx"]) if world > 1 else None
    if dist:
        dist.barrier()

    def step(it):
        if comm is None:
            it["idx"].decode(it["q"], it["k"], it["v"], scale, out=it["out"])
        else:
            it["idx"].shard_decode(comm, it["q"], it["k"], it["v"], scale, out=it["out"])

    for it in items:
        step(it)
    for it in items:
        it["idx"].trim(1)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for it in items:
            step(it)
    for it in items:
        it["idx"].trim(1)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us_layer = e0.elapsed_time(e1) * 1000.0 / layers
    err = sum(it["idx"].check_device() for it in items)

    per_phase = {p: [] for p in PHASES}
    per_phase_max = {p: [] for p in PHASES}
    per_sub = {n: [] for n, _, _ in SUBPHASES}
    spans, entries, exits, skews = [], [], [], []
    for it in items:
        a = it["buf"].cpu().reshape(-1, 24).tolist()
        ph = {p: [] for p in PHASES}
        sub = {n: [] for n, _, _ in SUBPHASES}
        for r in a:
            gt0, c1, c2, c3, c4, c5, c6, gt7 = r[:8]
            ns = gt7 - gt0
            cyc = c6 - c1
            cpn = cyc / ns if ns > 0 else 1.965
            for p_, (x, y) in zip(PHASES, [(c1, c2), (c2, c3), (c3, c4), (c4, c5), (c5, c6)]):
                ph[p_].append((y - x) / cpn / 1000.0)
            for n_, x, y in SUBPHASES:
                if r[x] and r[y]:
                    sub[n_].append((r[y] - r[x]) / cpn / 1000.0)
        for p_ in PHASES:
            per_phase[p_].append(statistics.median(ph[p_]))
            per_phase_max[p_].append(max(ph[p_]))
        for n_, _, _ in SUBPHASES:
            if sub[n_]:
                per_sub[n_].append(statistics.median(sub[n_]))
        t0 = min(r[0] for r in a)
        t1 = max(r[7] for r in a)
        entries.append(t0)
        exits.append(t1)
        spans.append((t1 - t0) / 1000.0)
        skews.append((max(r[0] for r in a) - t0) / 1000.0)
    cad = [(entries[i + 1] - entries[i]) / 1000.0 for i in range(len(entries) - 1)]
    gaps = [(entries[i + 1] - exits[i]) / 1000.0 for i in range(len(entries) - 1)]
    res = {
        "config": w.name, "layers": layers, "shards": world, "rank": rank, "l2_evict_first_hint": not l2_plain, "grid": list(items[0]["buf"].shape[:2][::-1]),
        "us_per_layer_events": round(us_layer, 3), "device_error": err,
        "algorithmic_bytes_per_layer": algorithmic_bytes(w),
        "phase_us_median_over_ctas": {p: round(statistics.median(per_phase[p]), 3) for p in PHASES},
        "phase_us_max_over_ctas": {p: round(statistics.median(per_phase_max[p]), 3) for p in PHASES},
        "subphase_us_median": {n: round(statistics.median(v), 3) for n, v in per_sub.items() if v},
        "layer_span_us": round(statistics.median(spans), 3),
        "cta_start_skew_us": round(statistics.median(skews), 3),
        "layer_cadence_us": round(statistics.median(cad), 3) if cad else None,
        "gap_next_entry_minus_exit_us": round(statistics.median(gaps), 3) if gaps else None,
    }
    del graph
    if comm is not None:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c1")
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--no-overlap", action="store_true")
    ap.add_argument("--l2-plain", action="store_true", help="streamed loads without the L2 evict_first hint")
    args = ap.parse_args()
    import torch
    if int(os.environ.get("WORLD_SIZE", "1")) == 1:
        torch.cuda.set_device(0)
    res = profile(args.config, args.layers, args.warmup, not args.no_overlap, args.l2_plain)
    if res["rank"] == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    here = Path(__file__).resolve().parent.parent
    if str(here) not in sys.path:
        sys.path.insert(0, str(here))
    main()
