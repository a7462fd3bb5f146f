"""Sequence-sharded decode across real GPUs (one process per GPU, NCCL): the
output of `sparse_decode.sharded_decode` on every rank matches the oracle and
the selection is the single-device one, through NCCL all-gathers and through
the fused peer-memory step (ShardComm), which must give the same bits. The
multi-GPU case needs at least two GPUs and is skipped otherwise; the fused
step with a single shard runs on one GPU."""
from __future__ import annotations

import socket
from datetime import timedelta

import numpy as np
import pytest

from sparse_decode.synth import Workload

pytestmark = pytest.mark.gpu

CASES = [
    Workload("mg_bf16", B=2, Hq=8, Hkv=2, D=128, T=64 * 40 + 9, S=64, K=8, dtype="bf16", needles=4),
    Workload("mg_q8", B=1, Hq=32, Hkv=8, D=128, T=128 * 20 + 1, S=128, K=5, dtype="bf16", bits=8, needles=3),
    # K = 256 over 4200 candidates: the sliced selection, whose CTAs' lists
    # meet across the shards in one exchange
    Workload("mg_k256_q8", B=1, Hq=8, Hkv=2, D=128, T=64 * 4200 + 7, S=64, K=256, dtype="bf16", bits=8,
             needles=20),
    # every candidate block scores the same: the K lowest block indices win,
    # so the lists of the first CTAs of every shard are cut and fully taken
    # (the exact two-level path decides)
    Workload("mg_ties", B=1, Hq=4, Hkv=1, D=128, T=64 * 3001, S=64, K=256, dtype="bf16"),
]


def _case(i: int):
    from _util import host_case
    w = CASES[i]
    c = host_case(w, 300 + i)
    if w.name == "mg_ties":
        from test_gpu_parity import _recompute
        ks = c["ks"].reshape(1, w.T, w.D)
        for j in range(1, w.NB - 1):
            ks[0, j * w.S:(j + 1) * w.S] = ks[0, 0:w.S]
        c = _recompute(w, c, ks)
        assert list(c["sel"][0]) == list(range(w.K)) + [w.NB - 1]
    return c


def _rank_main(rank: int, world: int, port: int, results):
    import torch
    import torch.distributed as dist
    from gpu_cases import to_dev, to_host
    from sparse_decode import ShardComm, SparseIndex, sharded_decode
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        res = []
        for i, w in enumerate(CASES):
            c = _case(i)
            B, Hkv, T, D = w.B, w.Hkv, w.T, w.D
            idx = SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, T, w.dtype, w.bits, shard_rank=rank, shard_count=world)
            k = to_dev(c["ks"].reshape(B, Hkv, T, D), w.dtype)
            v = to_dev(c["vs"].reshape(B, Hkv, T, D), w.dtype)
            q = to_dev(c["qs"], w.dtype)
            idx.append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
            outs, sels = [], []
            for rep in range(2):  # decode, trim, decode again: same result
                sel = torch.full((B * Hkv, w.K + 1), -7, dtype=torch.int32, device="cuda")
                out = sharded_decode(idx, q, k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(), c["scale"],
                                     sel_out=sel)
                torch.cuda.synchronize()
                outs.append(to_host(out, w.dtype))
                sels.append(sel.cpu().numpy()[:, : w.n_sel])
                assert idx.trim(1) == 1
            # the fused peer-memory step: the same selection, the same output bits
            comm = ShardComm(idx)
            for rep in range(2):
                sel = torch.full((B * Hkv, w.K + 1), -7, dtype=torch.int32, device="cuda")
                out = sharded_decode(idx, q, k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(), c["scale"],
                                     sel_out=sel, comm=comm)
                torch.cuda.synchronize()
                outs.append(to_host(out, w.dtype))
                sels.append(sel.cpu().numpy()[:, : w.n_sel])
                assert idx.trim(1) == 1
            comm.close()
            res.append((outs, sels, idx.check_device()))
            idx.close()
        results.put((rank, res))
    except BaseException as e:  # reported to the parent, which fails the test
        results.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_across_gpus(cuda, world):
    import torch
    import torch.multiprocessing as mp
    from _util import assert_close
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in procs:
            rank, res = results.get(timeout=300)
            got[rank] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(got[r], str), f"rank {r}: {got[r]}"
    for i, w in enumerate(CASES):
        c = _case(i)
        ref_out = None
        for r in range(world):
            outs, sels, err = got[r][i]
            assert err == 0, (w.name, r)
            for o, s in zip(outs, sels):
                assert np.array_equal(s, c["sel"]), (w.name, r)
                assert_close(o.reshape(-1, w.D), c["out"], w.dtype)
                if ref_out is None:
                    ref_out = o
                assert np.array_equal(o, ref_out), (w.name, r)  # identical on every rank and step


def test_peer_wait_expires_without_the_other_shard(cuda):
    """Failure detection of the fused sharded step: shard 0 of 2 runs alone
    (shard 1's kernel is never launched, so its flags are never set). Both of
    the kernel's waits for shard 1 give up after the comm's limit, the error
    bit 4 is reported, and the GPU context stays usable."""
    import time
    import torch
    from gpu_cases import to_dev
    from _util import host_case
    from sparse_decode import ShardComm, SparseIndex
    w = Workload("lonely", B=1, Hq=8, Hkv=2, D=128, T=64 * 20 + 3, S=64, K=4, dtype="bf16", needles=1)
    c = host_case(w, 500)
    B, Hkv, T, D = w.B, w.Hkv, w.T, w.D
    shards = [SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, T, w.dtype, 0, shard_rank=r, shard_count=2) for r in range(2)]
    comms = [ShardComm(s, local=True) for s in shards]
    ShardComm.open_local(comms)
    comms[0].set_wait_limit(0.2)
    k = to_dev(c["ks"].reshape(B, Hkv, T, D), w.dtype)
    v = to_dev(c["vs"].reshape(B, Hkv, T, D), w.dtype)
    q = to_dev(c["qs"], w.dtype)
    shards[0].append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
    torch.cuda.synchronize()
    t0 = time.time()
    shards[0].shard_decode(comms[0], q)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert shards[0].check_device() & 4
    assert 0.3 < dt < 5.0, dt  # two expired waits of 0.2 s
    # the context still works
    one = SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, T, w.dtype, 0)
    one.append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
    one.decode(q, k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(), c["scale"])
    torch.cuda.synchronize()
    assert one.check_device() == 0
    for cm in comms:
        cm.close()


def test_peer_step_single_shard_matches_decode(cuda):
    """The fused peer-memory step with one shard (the exchange goes to the
    shard's own area): bit-identical to sd_decode over several steps, also
    when the steps of three layers are replayed from a CUDA graph (the epoch
    lives on the device)."""
    import torch
    from gpu_cases import to_dev
    from _util import host_case
    from sparse_decode import ShardComm, SparseIndex
    w = Workload("peer1", B=1, Hq=32, Hkv=8, D=128, T=64 * 50 + 5, S=64, K=16, dtype="bf16", needles=4)
    cases = [host_case(w, 400 + i) for i in range(3)]
    B, Hkv, T, D = w.B, w.Hkv, w.T, w.D

    def make(c):
        idx = SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, T, w.dtype, 0)
        k = to_dev(c["ks"].reshape(B, Hkv, T, D), w.dtype)
        v = to_dev(c["vs"].reshape(B, Hkv, T, D), w.dtype)
        idx.append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
        return idx, to_dev(c["qs"], w.dtype), k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous()

    ref, peer = [make(c) for c in cases], [make(c) for c in cases]
    comm = ShardComm(peer[0][0])
    want = []
    for (idx, q, kn, vn), c in zip(ref, cases):
        want.append(idx.decode(q, kn, vn, c["scale"]).clone())
        idx.trim(1)
    outs = [torch.empty_like(q) for (_, q, _, _) in peer]
    sels = [torch.empty((B * Hkv, w.K + 1), dtype=torch.int32, device="cuda") for _ in peer]
    for rep in range(2):  # eager launches
        for (idx, q, kn, vn), c, o, s in zip(peer, cases, outs, sels):
            idx.shard_decode(comm, q, kn, vn, c["scale"], out=o, sel_out=s)
            idx.trim(1)
        torch.cuda.synchronize()
        for o, wnt, s, c in zip(outs, want, sels, cases):
            assert torch.equal(o, wnt)
            assert np.array_equal(s.cpu().numpy()[:, : w.n_sel], c["sel"])
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for (idx, q, kn, vn), c, o in zip(peer, cases, outs):
            idx.shard_decode(comm, q, kn, vn, c["scale"], out=o)
    for (idx, _, _, _) in peer:
        idx.trim(1)
    for rep in range(3):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for o, wnt in zip(outs, want):
            assert torch.equal(o, wnt)
    for (idx, _, _, _) in peer:
        assert idx.check_device() == 0
    del g
    comm.close()
