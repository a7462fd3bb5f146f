"""GPU parity of the selection paths for large candidate sets.

The decode kernel selects the top-K blocks in one of two ways. When a
group has at most 2048 candidate blocks and K <= 128, every CTA of the group
holds all candidate keys and runs a block-wide bitonic top-K. Otherwise
(config 4: 16383 candidates, K = 256) the candidates are split over all the
group's CTAs, each CTA reduces its share to a list of its best keys, and the
lists are combined through L2 (a second round with full lists when a cut
list was fully taken). These cases force the second path -- K > 128 alone,
more than 2048 candidates alone, both, 17000 candidates over 64 CTAs, ties
across CTAs, and a reduced config 4 -- and compare block scores and selected
blocks with the oracle bit for bit, outputs within the tolerance of
tests/_util.py.
Selection semantics: top-K blocks by (score desc, block index asc) plus the
recent block, ascending.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from sparse_decode.synth import CONFIGS, Workload

from _util import host_case
from gpu_cases import run_decode, to_dev
from test_gpu_parity import _check, _recompute

pytestmark = pytest.mark.gpu

LARGE = [
    # K > 128 with ~600 candidates
    Workload("sel_k129_n601", B=1, Hq=8, Hkv=2, D=128, T=64 * 601 + 10, S=64, K=129, dtype="bf16", needles=20),
    # more than 2048 candidates with K = 64
    Workload("sel_k64_n2101", B=1, Hq=8, Hkv=2, D=128, T=64 * 2101 + 5, S=64, K=64, dtype="bf16", needles=10),
    # both, 4-bit codes
    Workload("sel_k200_n3000_q4", B=1, Hq=16, Hkv=2, D=128, T=64 * 3000 + 1, S=64, K=200, dtype="bf16", bits=4,
             needles=30),
    # config 4's shape at a quarter of its context: 8-bit, K = 256, 4095 candidates, drift
    CONFIGS["c4"].with_(name="c4_reduced_T262144", T=262144, layers=1),
    # 17000 candidates in one group, spread over 64 CTAs
    Workload("sel_k100_n17000", B=1, Hq=4, Hkv=1, D=128, T=64 * 17000 + 3, S=64, K=100, dtype="bf16",
             bits=8, needles=12),
]


@pytest.mark.parametrize("w", LARGE, ids=[w.name for w in LARGE])
def test_large_selection_parity(cuda, w):
    c, idx, res = run_decode(w, seed=4242)
    _check(w, c, res, idx)
    for bh in range(w.B * w.Hkv):
        assert set(c["needles"][bh // w.Hkv].tolist()) <= set(res["sel"][bh].tolist())


@pytest.mark.parametrize("n_cand,K", [(600, 200), (2500, 64), (3000, 256)])
def test_large_selection_ties(cuda, n_cand, K):
    """All candidate blocks are copies of block 0 (equal scores): the K lowest
    block indices win. Every candidate of the lowest-index share of the group
    is selected, which the lists combined through L2 must still resolve
    exactly."""
    w = Workload("ties_large", B=1, Hq=4, Hkv=1, D=128, T=64 * (n_cand + 1), S=64, K=K, dtype="bf16")
    c = host_case(w, seed=71)
    ks = c["ks"].reshape(1, w.T, w.D)
    for j in range(1, n_cand):
        ks[0, j * 64:(j + 1) * 64] = ks[0, 0:64]
    c = _recompute(w, c, ks)
    assert len(set(c["scores"][0, :-1].tolist())) == 1
    _, idx, res = run_decode(w, 71, c=c)
    assert list(res["sel"][0]) == list(range(K)) + [n_cand]
    _check(w, c, res)


def test_large_selection_ties_in_tail(cuda):
    """A run of equal scores at the boundary of the top-K, spread over several
    CTAs' shares: the lower block indices among the tied ones win."""
    w = Workload("ties_tail", B=1, Hq=4, Hkv=1, D=128, T=64 * 2601, S=64, K=150, dtype="bf16", needles=100)
    c = host_case(w, seed=72)
    ks = c["ks"].reshape(1, w.T, w.D)
    tied = np.arange(5, 2600, 7)  # 372 blocks spread over the whole sequence
    for j in tied:
        ks[0, j * 64:(j + 1) * 64] = ks[0, 3 * 64:4 * 64]
    c = _recompute(w, c, ks)
    _, idx, res = run_decode(w, 72, c=c)
    _check(w, c, res)


@pytest.mark.parametrize("cluster", [1, 2, 4, 8, 16])
def test_large_selection_cluster_sizes(cuda, cluster):
    w = Workload("sel_clusters", B=1, Hq=8, Hkv=2, D=128, T=64 * 2500 + 17, S=64, K=160, dtype="bf16", needles=12)
    c, idx, res = run_decode(w, seed=73, cluster=cluster)
    assert idx.cluster_size == cluster
    _check(w, c, res)


def test_large_selection_decode_steps(cuda):
    """Several decode steps on the large path (K = 140, 2100+ candidates),
    crossing a block boundary: every step matches the oracle."""
    import torch
    from sparse_decode import SparseIndex
    from gpu_cases import to_host
    from _util import assert_close
    w = Workload("sel_steps", B=1, Hq=8, Hkv=2, D=128, T=64 * 2110 + 60, S=64, K=140, dtype="bf16", bits=8,
                 needles=9)
    steps = 8
    wf = w.with_(T=w.T + steps)
    c = host_case(wf, seed=74)
    idx = SparseIndex(1, w.Hq, w.Hkv, w.D, w.S, w.K, wf.T, w.dtype, w.bits)
    k = to_dev(c["ks"].reshape(1, w.Hkv, wf.T, w.D), w.dtype)
    v = to_dev(c["vs"].reshape(1, w.Hkv, wf.T, w.D), w.dtype)
    idx.append(k[:, :, : w.T - 1].contiguous(), v[:, :, : w.T - 1].contiguous())
    q = to_dev(c["qs"], w.dtype)
    dt = c["dt"]
    for s in range(steps):
        T = w.T + s
        sel = torch.zeros((w.Hkv, w.K + 1), dtype=torch.int32, device="cuda")
        out = idx.decode(q, k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(), c["scale"], sel_out=sel)
        summ = oracle.summaries(c["Kc"], T, w.S, dt)
        sc = oracle.scores(c["qs"], dt, summ, dt, 1, w.Hq, w.Hkv, w.D, (T + 63) // 64, c["scale"])
        osel = oracle.select(sc, w.K)
        ref = oracle.attend_f64(c["qs"], dt, c["Kc"], c["Vc"], 1, w.Hq, w.Hkv, T, w.S, osel, c["scale"])
        assert np.array_equal(sel.cpu().numpy()[:, : osel.shape[1]], osel), f"step {s}"
        assert_close(to_host(out, w.dtype).reshape(-1, w.D), ref, w.dtype)
    assert idx.check_device() == 0


def test_peer_step_single_shard_large_union(cuda):
    """The fused peer-memory step with one shard and K = 256 (> 128), so the
    union of the shards' candidates is selected by the large-union path:
    bit-identical to sd_decode and equal to the oracle's selection."""
    import torch
    from sparse_decode import ShardComm, SparseIndex
    from _util import assert_close
    from gpu_cases import to_host
    w = Workload("peer_k256", B=1, Hq=32, Hkv=8, D=128, T=64 * 900 + 5, S=64, K=256, dtype="bf16", bits=8,
                 needles=20)
    c = host_case(w, 410)
    B, Hkv, T, D = w.B, w.Hkv, w.T, w.D
    k = to_dev(c["ks"].reshape(B, Hkv, T, D), w.dtype)
    v = to_dev(c["vs"].reshape(B, Hkv, T, D), w.dtype)
    q = to_dev(c["qs"], w.dtype)
    kn, vn = k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous()
    ref = SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, T, w.dtype, w.bits)
    ref.append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
    want_sel = torch.empty((B * Hkv, w.K + 1), dtype=torch.int32, device="cuda")
    want = ref.decode(q, kn, vn, c["scale"], sel_out=want_sel).clone()
    peer = SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, T, w.dtype, w.bits)
    peer.append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
    comm = ShardComm(peer)
    for rep in range(2):
        sel = torch.full((B * Hkv, w.K + 1), -7, dtype=torch.int32, device="cuda")
        out = peer.shard_decode(comm, q, kn, vn, c["scale"], sel_out=sel)
        torch.cuda.synchronize()
        assert torch.equal(out, want), rep
        assert np.array_equal(sel.cpu().numpy(), want_sel.cpu().numpy())
        assert np.array_equal(sel.cpu().numpy()[:, : w.n_sel], c["sel"])
        assert_close(to_host(out, w.dtype).reshape(-1, D), c["out"], w.dtype)
        peer.trim(1)
    assert peer.check_device() == 0 and ref.check_device() == 0
    comm.close()


def test_c2q8_full_size_layer(cuda):
    """Config 2 (8-bit, B = 4, T = 131072, S = 128, top-32 + recent) at full size."""
    w = CONFIGS["c2q8"]
    c, idx, res = run_decode(w, seed=2025)
    _check(w, c, res, idx)


def test_c3_shaped_layer(cuda):
    """Config 3's single-GPU shape (bf16, B = 16, T = 131072, S = 64, 2047
    candidates, top-128 + recent): 128 groups, more than fit on the GPU at once."""
    w = CONFIGS["c3"]
    c, idx, res = run_decode(w, seed=2026)
    _check(w, c, res)


def test_c1_full_size_layer(cuda):
    """Config 1 (bf16, T = 32768, S = 64, top-64 + recent) at full size."""
    w = CONFIGS["c1"]
    c, idx, res = run_decode(w, seed=2024)
    _check(w, c, res, idx)
