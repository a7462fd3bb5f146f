"""Parity of the CUDA library (through its C ABI) with the CPU oracle.

Bar: block scores and selected blocks bit-exact (the kernels use the
oracle's canonical fp32 order), summaries and quantized codes bit-exact,
outputs within the tolerance of tests/_util.py (normwise 2e-3 per head for
fp16/bf16 and within one output ulp element-wise; 1e-5 for fp32).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from sparse_decode.synth import CONFIGS, Workload

from _util import assert_close, host_case
from gpu_cases import run_decode, to_dev, to_host

pytestmark = pytest.mark.gpu

SMALL = [
    CONFIGS["c0"],                                                     # fp32 D64 G4, the reference CPU-sized case
    CONFIGS["c1"].with_(name="c1_reduced_T8192", T=8192),             # bf16 D128 G4 S64 K64
    Workload("f16_d64_g2", B=2, Hq=4, Hkv=2, D=64, T=3000, S=32, K=16, dtype="f16", needles=5),
    Workload("bf16_g8_s128", B=1, Hq=16, Hkv=2, D=128, T=5000, S=128, K=8, dtype="bf16", needles=3),
    Workload("bf16_g1_s256", B=1, Hq=4, Hkv=4, D=128, T=3333, S=256, K=4, dtype="bf16", needles=2),
    CONFIGS["c2q8"].with_(name="c2q8_reduced_B2_T8192", B=2, T=8192),  # 8-bit bf16 scales, outliers
    CONFIGS["c2q4"].with_(name="c2q4_reduced_B2_T8192", B=2, T=8192),  # 4-bit
    Workload("q8_f16_d64", B=1, Hq=4, Hkv=2, D=64, T=2000, S=64, K=10, dtype="f16", bits=8, needles=3),
    Workload("q4_f32_d64", B=1, Hq=8, Hkv=2, D=64, T=1500, S=32, K=12, dtype="f32", bits=4, needles=3),
    Workload("q4_bf16_d64_g8", B=1, Hq=16, Hkv=2, D=64, T=2500, S=64, K=9, dtype="bf16", bits=4, needles=3),
    Workload("q8_f16_d128_g1", B=2, Hq=2, Hkv=2, D=128, T=2100, S=32, K=14, dtype="f16", bits=8, needles=2),
    Workload("q4_f16_d128_g2", B=1, Hq=4, Hkv=2, D=128, T=3100, S=128, K=5, dtype="f16", bits=4, needles=2),
    Workload("q8_bf16_d64_g8", B=1, Hq=16, Hkv=2, D=64, T=1700, S=64, K=7, dtype="bf16", bits=8, needles=2),
]


def _check(w, c, res, idx=None):
    assert res["err"] == 0, f"device error word {res['err']}"
    n_sel = w.n_sel
    # scores: bit-exact for every block but the recent one
    assert np.array_equal(res["scores"][:, : w.NB - 1], c["scores"][:, : w.NB - 1])
    # selection: bit-exact (and equal to the fp64 selection where the K-th gap > 1e-3)
    assert np.array_equal(res["sel"][:, :n_sel], c["sel"])
    assert (res["sel"][:, n_sel:] == -1).all()
    assert_close(res["out"], c["out"], w.dtype)
    if idx is not None:
        v = idx.views()
        dt = c["dt"]
        g = v["summaries"][:, : w.NB - 1]
        assert np.array_equal(to_host(g.contiguous(), w.dtype), oracle.to_f32(c["summ"][:, : w.NB - 1], dt))
        if w.bits:
            kq = v["k"][:, : w.T].cpu().numpy().view(np.uint32)
            assert np.array_equal(kq, c["Kc"].data[:, : w.T])
            assert np.array_equal(to_host(v["k_scales"][:, : w.T].contiguous(), w.dtype),
                                  oracle.to_f32(c["Kc"].scales[:, : w.T], dt))


@pytest.mark.parametrize("w", SMALL, ids=[w.name for w in SMALL])
def test_decode_parity(cuda, w):
    c, idx, res = run_decode(w, seed=100)
    _check(w, c, res, idx)
    # the planted needles are retrieved
    for bh in range(w.B * w.Hkv):
        assert set(c["needles"][bh // w.Hkv].tolist()) <= set(res["sel"][bh].tolist())


def test_c1_full_size_layer(cuda):
    """Config 1 (Qwen3-4B shape, T=32768, 512 blocks, top-64 + recent) at full size."""
    w = CONFIGS["c1"]
    c, idx, res = run_decode(w, seed=2024)
    _check(w, c, res, idx)


@pytest.mark.parametrize("bits", [0, 8, 4])
def test_many_tiles_per_cta(cuda, bits):
    """One CTA per group (cluster 1, no replicas) walks hundreds of 32-token
    tiles through the TMA ring, so every stage is reused many times by
    different consumer warps (the shape of config 3, where 128 groups fill the
    GPU with one CTA each)."""
    w = Workload("many", B=2, Hq=8, Hkv=2, D=128, T=64 * 140 + 33, S=64, K=128, dtype="bf16", bits=bits,
                 needles=5)
    c, idx, res = run_decode(w, seed=31, cluster=1)
    assert idx.cluster_size == 1 and idx.replicas == 1
    assert res["err"] == 0
    _check(w, c, res, idx)


@pytest.mark.parametrize("cluster", [1, 2, 4, 8, 16])
def test_cluster_sizes_agree(cuda, cluster):
    w = CONFIGS["c1"].with_(name="c1_reduced_T6000_K20", T=6000, K=20)
    c, idx, res = run_decode(w, seed=5, cluster=cluster)
    assert idx.cluster_size == cluster
    _check(w, c, res)


@pytest.mark.parametrize("bits", [0, 8])
def test_all_blocks_is_dense_attention(cuda, bits):
    w = Workload("dense_eq", B=1, Hq=8, Hkv=2, D=128, T=1000, S=64, K=40, dtype="bf16", bits=bits)
    c, idx, res = run_decode(w, seed=6)
    assert (res["sel"][:, : w.NB] == np.arange(w.NB)).all()
    _check(w, c, res)


def test_ties_take_the_lower_block(cuda):
    """Blocks with identical keys score identically; the lower index wins."""
    w = Workload("ties", B=1, Hq=4, Hkv=1, D=128, T=64 * 40, S=64, K=5, dtype="bf16")
    c = host_case(w, seed=7)
    ks = c["ks"].reshape(1, w.T, w.D)
    for j in range(1, 39):            # every block a copy of block 0 -> all scores equal
        ks[0, j * 64:(j + 1) * 64] = ks[0, 0:64]
    c = _recompute(w, c, ks)
    assert len(set(c["scores"][0, :-1].tolist())) == 1
    _, idx, res = run_decode(w, 7, c=c)
    assert list(res["sel"][0]) == [0, 1, 2, 3, 4, 39]
    _check(w, c, res)


def _recompute(w, c, ks):
    """Oracle results for edited key storage."""
    dt = c["dt"]
    Kc = oracle.Cache(dt, w.D, ks.reshape(w.B * w.Hkv, w.T, w.D))
    summ = oracle.summaries(Kc, w.T, w.S, dt)
    sc = oracle.scores(c["qs"], dt, summ, dt, w.B, w.Hq, w.Hkv, w.D, w.NB, c["scale"])
    sel = oracle.select(sc, w.K)
    out = oracle.attend_f64(c["qs"], dt, Kc, c["Vc"], w.B, w.Hq, w.Hkv, w.T, w.S, sel, c["scale"])
    c = dict(c)
    c.update(ks=Kc.data, Kc=Kc, summ=summ, scores=sc, sel=sel, out=out)
    return c


@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 130])
def test_short_contexts(cuda, T):
    w = Workload("short", B=1, Hq=8, Hkv=2, D=64, T=T, S=64, K=3, dtype="bf16")
    c, idx, res = run_decode(w, seed=T)
    _check(w, c, res)


def test_top_k_zero_keeps_only_recent(cuda):
    w = Workload("k0", B=2, Hq=8, Hkv=2, D=128, T=1000, S=64, K=0, dtype="bf16")
    c, idx, res = run_decode(w, seed=9)
    assert (res["sel"][:, 0] == w.NB - 1).all()
    _check(w, c, res)


@pytest.mark.parametrize("bits", [0, 8, 4])
def test_decode_steps_across_blocks(cuda, bits):
    """Prefill, then 70 single-token steps crossing block boundaries: every
    step's selection and output match the oracle, and the summaries of blocks
    completed during decode are bit-exact."""
    import torch
    w = Workload("steps", B=1, Hq=8, Hkv=2, D=128, T=64 * 10 + 60, S=64, K=4, dtype="bf16", bits=bits)
    steps = 70
    wf = w.with_(T=w.T + steps)
    c = host_case(wf, seed=11)
    from sparse_decode import SparseIndex
    idx = SparseIndex(1, w.Hq, w.Hkv, w.D, w.S, w.K, wf.T, w.dtype, bits)
    k = to_dev(c["ks"].reshape(1, w.Hkv, wf.T, w.D), w.dtype)
    v = to_dev(c["vs"].reshape(1, w.Hkv, wf.T, w.D), w.dtype)
    idx.append(k[:, :, : w.T - 1].contiguous(), v[:, :, : w.T - 1].contiguous())
    q = to_dev(c["qs"], w.dtype)
    dt = c["dt"]
    for s in range(steps):
        T = w.T + s
        sel = torch.zeros((w.Hkv, w.K + 1), dtype=torch.int32, device="cuda")
        out = idx.decode(q, k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(), c["scale"], sel_out=sel)
        assert idx.offset == T
        summ = oracle.summaries(c["Kc"], T, w.S, dt)
        sc = oracle.scores(c["qs"], dt, summ, dt, 1, w.Hq, w.Hkv, w.D, (T + 63) // 64, c["scale"])
        osel = oracle.select(sc, w.K)
        ref = oracle.attend_f64(c["qs"], dt, c["Kc"], c["Vc"], 1, w.Hq, w.Hkv, T, w.S, osel, c["scale"])
        assert np.array_equal(sel.cpu().numpy()[:, : osel.shape[1]], osel), f"step {s}"
        assert_close(to_host(out, w.dtype).reshape(-1, w.D), ref, w.dtype)
    full = (w.T + steps) // 64
    g = to_host(idx.views()["summaries"][:, :full].contiguous(), w.dtype)
    assert np.array_equal(g, oracle.to_f32(oracle.summaries(c["Kc"], full * 64, 64, dt), dt)[:, :full])
    assert idx.check_device() == 0


def test_trim_then_decode(cuda):
    import torch
    w = Workload("trim", B=1, Hq=8, Hkv=2, D=128, T=64 * 8, S=64, K=3, dtype="bf16", needles=2)
    c, idx, res = run_decode(w, seed=12)
    _check(w, c, res)
    assert idx.trim(70) == 70
    assert idx.offset == w.T - 70
    # re-append the same rows one decode step at a time and land on the same result
    k = to_dev(c["ks"].reshape(1, w.Hkv, w.T, w.D), w.dtype)
    v = to_dev(c["vs"].reshape(1, w.Hkv, w.T, w.D), w.dtype)
    q = to_dev(c["qs"], w.dtype)
    sel = torch.zeros((w.Hkv, w.K + 1), dtype=torch.int32, device="cuda")
    for t in range(w.T - 70, w.T):
        out = idx.decode(q, k[:, :, t].contiguous(), v[:, :, t].contiguous(), c["scale"], sel_out=sel)
    assert np.array_equal(sel.cpu().numpy(), c["sel"])
    assert_close(to_host(out, w.dtype).reshape(-1, w.D), c["out"], w.dtype)


@pytest.mark.parametrize("P", [2, 3, 4])
@pytest.mark.parametrize("bits", [0, 8])
def test_sharded_steps_on_one_gpu(cuda, P, bits):
    """The sequence-sharded path with P shards held on one GPU (the
    all-gathers done by concatenation): same selection and output as the
    single-shard decode and the oracle."""
    import torch
    from sparse_decode import SparseIndex
    w = Workload("shard", B=2, Hq=8, Hkv=2, D=128, T=64 * 30 + 17, S=64, K=6, dtype="bf16", bits=bits, needles=4)
    c = host_case(w, seed=13)
    B, Hkv, T, D, K = w.B, w.Hkv, w.T, w.D, w.K
    k = to_dev(c["ks"].reshape(B, Hkv, T, D), w.dtype)
    v = to_dev(c["vs"].reshape(B, Hkv, T, D), w.dtype)
    q = to_dev(c["qs"], w.dtype)
    shards = [SparseIndex(B, w.Hq, Hkv, D, w.S, K, T, w.dtype, bits, shard_rank=r, shard_count=P) for r in range(P)]
    for s in shards:
        s.append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
    cs = [torch.empty((B * Hkv, K), device="cuda") for _ in range(P)]
    cb = [torch.empty((B * Hkv, K), device="cuda", dtype=torch.int32) for _ in range(P)]
    scores = torch.full((B * Hkv, w.NB), float("nan"), device="cuda")
    for r, s in enumerate(shards):
        s.shard_candidates(q, cs[r], cb[r], k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(), c["scale"],
                           scores_out=scores)
    all_cs, all_cb = torch.stack(cs), torch.stack(cb)
    mls, pos, sels = [], [], []
    for s in shards:
        ml = torch.empty((B * w.Hq, 2), device="cuda")
        po = torch.empty((B * w.Hq, D), device="cuda")
        sel = torch.empty((B * Hkv, K + 1), device="cuda", dtype=torch.int32)
        s.shard_attend(q, all_cs, all_cb, ml, po, c["scale"], sel)
        mls.append(ml); pos.append(po); sels.append(sel)
    out = torch.empty_like(q)
    shards[0].shard_merge(torch.stack(mls), torch.stack(pos), out)
    torch.cuda.synchronize()
    assert np.array_equal(scores.cpu().numpy()[:, : w.NB - 1], c["scores"][:, : w.NB - 1])
    for sel in sels:
        assert np.array_equal(sel.cpu().numpy()[:, : w.n_sel], c["sel"])
    assert_close(to_host(out, w.dtype).reshape(-1, D), c["out"], w.dtype)
    for s in shards:
        assert s.check_device() == 0


@pytest.mark.parametrize("bits", [0, 8])
def test_trim_one_then_other_token(cuda, bits):
    """Decode the token that fills a block, trim it, decode a different token
    in its place (the running block sums are restored by the one-step undo):
    summaries, selection and output match the oracle for the second token."""
    import torch
    from sparse_decode import SparseIndex
    w = Workload("undo", B=1, Hq=8, Hkv=2, D=128, T=64 * 12, S=64, K=4, dtype="bf16", bits=bits, needles=2)
    c = host_case(w, seed=21)
    idx = SparseIndex(1, w.Hq, w.Hkv, w.D, w.S, w.K, w.T, w.dtype, bits)
    k = to_dev(c["ks"].reshape(1, w.Hkv, w.T, w.D), w.dtype)
    v = to_dev(c["vs"].reshape(1, w.Hkv, w.T, w.D), w.dtype)
    q = to_dev(c["qs"], w.dtype)
    idx.append(k[:, :, : w.T - 2].contiguous(), v[:, :, : w.T - 2].contiguous())
    idx.decode(q, k[:, :, w.T - 2].contiguous(), v[:, :, w.T - 2].contiguous(), c["scale"])  # rebuilds the sums
    rng = np.random.default_rng(5)
    other = rng.standard_normal((w.Hkv, w.D)).astype(np.float32)
    for rep in range(3):
        idx.decode(q, k[:, :, w.T - 1].contiguous(), v[:, :, w.T - 1].contiguous(), c["scale"])
        assert idx.trim(1) == 1
        ks2 = c["ks"].reshape(w.Hkv, w.T, w.D).copy()
        ks2[:, w.T - 1] = oracle.to_storage(other * (rep + 1), c["dt"])
        c2 = _recompute_k(w, c, ks2)
        kn = to_dev(ks2[:, w.T - 1].reshape(1, w.Hkv, w.D), w.dtype)
        sel = torch.zeros((w.Hkv, w.K + 1), dtype=torch.int32, device="cuda")
        out = idx.decode(q, kn, v[:, :, w.T - 1].contiguous(), c["scale"], sel_out=sel)
        assert np.array_equal(sel.cpu().numpy(), c2["sel"])
        assert_close(to_host(out, w.dtype).reshape(-1, w.D), c2["out"], w.dtype)
        g = to_host(idx.views()["summaries"][:, : w.NB].contiguous(), w.dtype)
        assert np.array_equal(g, oracle.to_f32(c2["summ"], c["dt"]).reshape(g.shape))
        assert idx.trim(1) == 1
    assert idx.check_device() == 0


def _recompute_k(w, c, ks):
    """Oracle results with key storage `ks` [BH, T, D] (re-quantized when needed)."""
    dt = c["dt"]
    if w.bits:
        kq = oracle.quantize(ks, dt, w.D, w.bits)
        Kc = oracle.Cache(dt, w.D, kq[0], w.bits, kq[1], kq[2])
    else:
        Kc = oracle.Cache(dt, w.D, ks)
    summ = oracle.summaries(Kc, w.T, w.S, dt)
    sc = oracle.scores(c["qs"], dt, summ, dt, w.B, w.Hq, w.Hkv, w.D, w.NB, c["scale"])
    sel = oracle.select(sc, w.K)
    out = oracle.attend_f64(c["qs"], dt, Kc, c["Vc"], w.B, w.Hq, w.Hkv, w.T, w.S, sel, c["scale"])
    return {"summ": summ, "scores": sc, "sel": sel, "out": out}


def test_overlapped_launches_across_layers(cuda):
    """Two layers decoded alternately with launch overlap enabled (each
    kernel may start while the other layer's kernel finishes), and the same
    layer twice in a row (no early reads then): every step matches the oracle."""
    import torch
    from sparse_decode import SparseIndex
    w = Workload("pdl", B=1, Hq=8, Hkv=2, D=128, T=64 * 20 + 40, S=64, K=6, dtype="bf16", needles=3)
    steps = 30
    wf = w.with_(T=w.T + steps)
    cases = [host_case(wf, seed=31 + l) for l in range(2)]
    idxs, dev = [], []
    for c in cases:
        idx = SparseIndex(1, w.Hq, w.Hkv, w.D, w.S, w.K, wf.T, w.dtype)
        k = to_dev(c["ks"].reshape(1, w.Hkv, wf.T, w.D), w.dtype)
        v = to_dev(c["vs"].reshape(1, w.Hkv, wf.T, w.D), w.dtype)
        idx.append(k[:, :, : w.T - 1].contiguous(), v[:, :, : w.T - 1].contiguous())
        idx.set_launch_overlap(True)
        idxs.append(idx)
        dev.append((k, v, to_dev(c["qs"], w.dtype)))
    outs = []
    for s in range(steps):
        T = w.T + s
        step_out = {}
        # alternating order: layer 1 runs twice in a row across steps 0/1, layer 0 across 1/2, ...
        for l in ((0, 1) if s % 2 == 0 else (1, 0)):
            k, v, q = dev[l]
            sel = torch.zeros((w.Hkv, w.K + 1), dtype=torch.int32, device="cuda")
            step_out[l] = (idxs[l].decode(q, k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(),
                                          cases[l]["scale"], sel_out=sel), sel)
        outs.append((T, step_out))
    torch.cuda.synchronize()
    for T, step_out in outs:
        for l, (out, sel) in step_out.items():
            c = cases[l]
            dt = c["dt"]
            summ = oracle.summaries(c["Kc"], T, w.S, dt)
            sc = oracle.scores(c["qs"], dt, summ, dt, 1, w.Hq, w.Hkv, w.D, (T + 63) // 64, c["scale"])
            osel = oracle.select(sc, w.K)
            ref = oracle.attend_f64(c["qs"], dt, c["Kc"], c["Vc"], 1, w.Hq, w.Hkv, T, w.S, osel, c["scale"])
            assert np.array_equal(sel.cpu().numpy()[:, : osel.shape[1]], osel)
            assert_close(to_host(out, w.dtype).reshape(-1, w.D), ref, w.dtype)
    for idx in idxs:
        assert idx.check_device() == 0
