"""World-size-2 `gloo` run of the sequence-sharded decode step on CPU.

`sparse_decode.sharded_decode` is the host choreography of the multi-GPU
path: local candidates -> all-gather -> global top-K and attention over this
rank's stripe -> all-gather of (m, l, o) partials -> log-sum-exp merge. Here
the three device steps are played by the CPU oracle (test infrastructure
only), so what is checked is the host logic around them -- stripe ownership
(block j on rank j % P), the gathers' layout and the merge -- against the
unsharded oracle decode. Both ranks must return the same output, and the
global selection must equal the single-device one.
"""
from __future__ import annotations

import math
import socket
from datetime import timedelta

import numpy as np
import pytest

import oracle
from sparse_decode.synth import Workload

from _util import assert_close, host_case

CASES = [
    Workload("sh_bf16", B=2, Hq=8, Hkv=2, D=64, T=1000, S=32, K=8, dtype="bf16", needles=3),
    Workload("sh_q8", B=1, Hq=8, Hkv=2, D=128, T=1500, S=64, K=6, dtype="bf16", bits=8, needles=2),
    Workload("sh_f32_allk", B=1, Hq=4, Hkv=1, D=64, T=300, S=32, K=20, dtype="f32"),   # K > candidates
    Workload("sh_f16_k0", B=1, Hq=8, Hkv=4, D=64, T=700, S=64, K=0, dtype="f16"),       # recent block only
]


def _storage(t, dt: int) -> np.ndarray:
    import torch
    if dt == oracle.BF16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _tensor(a: np.ndarray, dt: int):
    import torch
    if dt == oracle.BF16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a))


class OracleShard:
    """One rank's shard with the device steps of SparseIndex.shard_* done by
    the CPU oracle over the blocks this rank owns."""

    def __init__(self, w: Workload, c: dict, rank: int, P: int):
        self.w, self.c, self.pr, self.P = w, c, rank, P
        self.B, self.Hq, self.Hkv, self.D, self.K = w.B, w.Hq, w.Hkv, w.D, w.K
        self.sel = None

    def _bh_cache(self, cache: oracle.Cache, bh: int) -> oracle.Cache:
        sl = slice(bh, bh + 1)
        return oracle.Cache(cache.dtype, cache.D, cache.data[sl], cache.bits,
                            None if cache.scales is None else cache.scales[sl],
                            None if cache.biases is None else cache.biases[sl])

    def shard_candidates(self, q, cs, cb, k_new=None, v_new=None, scale=None):
        import torch
        w, c = self.w, self.c
        sc = oracle.scores(_storage(q, c["dt"]), c["dt"], c["summ"], c["dt"], w.B, w.Hq, w.Hkv, w.D, w.NB,
                           c["scale"])
        mine = np.arange(self.pr, w.NB - 1, self.P, dtype=np.int32)
        cs.fill_(-math.inf)
        cb.fill_(-1)
        for bh in range(w.B * w.Hkv):
            blk, s = oracle.topk(sc[bh, mine], mine, w.K)
            cs[bh, : len(blk)] = torch.from_numpy(s)
            cb[bh, : len(blk)] = torch.from_numpy(blk)

    def shard_attend(self, q, all_cs, all_cb, ml, po, scale=None, sel_out=None):
        import torch
        w, c = self.w, self.c
        G, NB = w.G, w.NB
        qs = _storage(q, c["dt"]).reshape(w.B, w.Hq, w.D)
        sels = []
        for bh in range(w.B * w.Hkv):
            blk = all_cb[:, bh].reshape(-1).numpy()
            s = all_cs[:, bh].reshape(-1).numpy()
            keep = blk >= 0
            chosen, _ = oracle.topk(s[keep], blk[keep], w.K)
            full = np.append(np.sort(chosen), NB - 1).astype(np.int32)
            sels.append(full)
            own = full[full % self.P == self.pr]
            rows = slice(bh * G, (bh + 1) * G)
            if len(own) == 0:
                ml[rows, 0] = -math.inf
                ml[rows, 1] = 0.0
                po[rows] = 0.0
                continue
            b, h = divmod(bh, w.Hkv)
            qg = np.ascontiguousarray(qs[b, h * G:(h + 1) * G][None])
            m, l_, o = oracle.attend_f64(qg, c["dt"], self._bh_cache(c["Kc"], bh), self._bh_cache(c["Vc"], bh), 1, G,
                                         1, w.T, w.S, own[None], c["scale"], normalise=False)
            ml[rows, 0] = torch.from_numpy((m / math.log(2.0)).astype(np.float32))   # log2 units, as on the GPU
            ml[rows, 1] = torch.from_numpy(l_.astype(np.float32))
            po[rows] = torch.from_numpy(o.astype(np.float32))
        self.sel = np.stack(sels)

    def shard_merge(self, all_ml, all_po, out):
        import torch
        m = all_ml[..., 0].double().numpy() * math.log(2.0)
        l_ = all_ml[..., 1].double().numpy()
        merged = oracle.merge_f64(m, l_, all_po.double().numpy())
        out.copy_(torch.from_numpy(merged.astype(np.float32)).reshape(out.shape).to(out.dtype))


def _rank_main(rank: int, world: int, port: int, results):
    import torch
    import torch.distributed as dist
    from sparse_decode import sharded_decode
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        res = []
        for i, w in enumerate(CASES):
            c = host_case(w, 100 + i)
            shard = OracleShard(w, c, rank, world)
            out = sharded_decode(shard, _tensor(c["qs"], c["dt"]).reshape(w.B, w.Hq, w.D))
            res.append((out.float().numpy(), shard.sel))
        results.put((rank, res))
    except BaseException as e:  # reported to the parent, which fails the test
        results.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_decode_two_ranks_gloo(oracle_lib):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in procs:
            rank, res = results.get(timeout=240)
            got[rank] = res
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert not isinstance(got[r], str), f"rank {r}: {got[r]}"
    for i, w in enumerate(CASES):
        c = host_case(w, 100 + i)
        out0, sel0 = got[0][i]
        out1, sel1 = got[1][i]
        assert np.array_equal(out0, out1), w.name
        assert np.array_equal(sel0, c["sel"]) and np.array_equal(sel1, c["sel"]), w.name
        assert_close(out0.reshape(-1, w.D), c["out"], w.dtype)
