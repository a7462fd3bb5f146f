"""CPU checks of the oracle (no GPU): the C++ restatement against its
independent numpy twin, known-answer cases, and the committed golden fixtures.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from sparse_decode.synth import CONFIGS, DTYPE_CODE, make_case

from _util import assert_close, boundary_gap_ok, host_case

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_quantize_matches_numpy_twin(oracle_lib, bits, dtype):
    dt = DTYPE_CODE[dtype]
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 128)).astype(np.float32) * rng.uniform(0.01, 10, (64, 1)).astype(np.float32)
    x[0] = 0.0                       # all zero
    x[1] = 1.5                       # constant
    x[2, :64] = -np.abs(x[2, :64])   # all negative group
    xs = oracle.to_storage(x, dt)
    xf = oracle.to_f32(xs, dt).reshape(x.shape)
    wq, sc, bi = oracle.quantize(xs, dt, 128, bits)
    codes, s_np, b_np = oracle.np_quantize(xf, bits)
    assert np.array_equal(oracle.np_unpack(wq, bits), codes)
    assert np.array_equal(wq, oracle.np_pack(codes, bits))
    assert np.array_equal(oracle.to_f32(sc, dt).reshape(s_np.shape), oracle.round_to(s_np, dt).reshape(s_np.shape))
    assert np.array_equal(oracle.to_f32(bi, dt).reshape(b_np.shape), oracle.round_to(b_np, dt).reshape(b_np.shape))


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_roundtrip_bound(oracle_lib, bits):
    dt = DTYPE_CODE["bf16"]
    rng = np.random.default_rng(5)
    x = rng.standard_normal((256, 128)).astype(np.float32)
    x[:, :4] *= 8.0
    xs = oracle.to_storage(x, dt)
    xf = oracle.to_f32(xs, dt).reshape(x.shape)
    wq, sc, bi = oracle.quantize(xs, dt, 128, bits)
    c = oracle.Cache(dt, 128, wq.reshape(1, 256, -1), bits, sc.reshape(1, 256, -1), bi.reshape(1, 256, -1))
    deq = c.floats()[0]
    codes, s32, b32 = oracle.np_quantize(xf, bits)
    s_st = oracle.to_f32(sc, dt).reshape(s32.shape)
    b_st = oracle.to_f32(bi, dt).reshape(b32.shape)
    n_max = 2 ** bits - 1
    # The edge-anchored scale s = edge / round(edge / s0) can be a little
    # smaller than the range needs, so the far end of a group may clip:
    # |x - deq| <= max(|s|/2, range - n_max*|s|) + n_max*|s - s_stored| + |b - b_stored|
    g = xf.reshape(256, 2, 64)
    rng_ = g.max(-1) - g.min(-1)
    quant = np.maximum(np.abs(s32) / 2, rng_ - n_max * np.abs(s32))
    bound = (quant + n_max * np.abs(s32 - s_st) + np.abs(b32 - b_st)) * 1.0001 + 1e-6
    err = np.abs(xf - deq).reshape(256, 2, 64).max(-1)
    assert (err <= bound).all()
    # the clipping stays small: within 1.5 quantization steps of the group
    assert (err <= 1.5 * np.abs(s32) + n_max * np.abs(s32 - s_st) + np.abs(b32 - b_st) + 1e-6).all()
    # zeros stay exactly representable
    z = np.zeros((4, 128), np.float32)
    wz, sz, bz = oracle.quantize(oracle.to_storage(z, dt), dt, 128, bits)
    cz = oracle.Cache(dt, 128, wz.reshape(1, 4, -1), bits, sz.reshape(1, 4, -1), bz.reshape(1, 4, -1))
    assert np.array_equal(cz.floats(), np.zeros((1, 4, 128), np.float32))


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_summaries_match_numpy_twin(oracle_lib, dtype):
    dt = DTYPE_CODE[dtype]
    rng = np.random.default_rng(7)
    T, S, D = 1000, 64, 64
    k = oracle.to_storage(rng.standard_normal((3, T, D)).astype(np.float32), dt)
    Kc = oracle.Cache(dt, D, k)
    summ = oracle.summaries(Kc, T, S, dt)
    ref = oracle.np_summaries(Kc.floats(), T, S, dt)
    assert np.array_equal(oracle.to_f32(summ, dt).reshape(ref.shape), ref)


def test_scores_and_selection_vs_fp64(oracle_lib):
    w = CONFIGS["c1"].with_(name="c1_reduced_T8192", T=8192)
    c = host_case(w, seed=11)
    sf = oracle.to_f32(c["summ"], c["dt"]).reshape(w.B * w.Hkv, w.NB, w.D)
    s64 = oracle.np_scores_f64(c["q"], sf, w.Hkv, c["scale"])
    assert np.allclose(c["scores"], s64, rtol=1e-5, atol=1e-6 * np.abs(s64).max())
    # selection from fp64 scores agrees wherever the K-th boundary gap > 1e-3
    ok = boundary_gap_ok(c["scores"], w.K)
    sel64 = oracle.np_select(s64, w.K)
    assert ok.any()
    assert np.array_equal(c["sel"][ok], sel64[ok])


def test_select_matches_numpy_and_breaks_ties_low_index(oracle_lib):
    rng = np.random.default_rng(1)
    sc = rng.integers(-3, 4, size=(5, 40)).astype(np.float32)  # many exact ties
    sc[0, :] = 1.0                                               # all equal
    sc[1, 5] = -0.0
    sc[1, 6] = 0.0
    got = oracle.select(sc, 7)
    assert np.array_equal(got, oracle.np_select(sc, 7))
    assert list(got[0]) == [0, 1, 2, 3, 4, 5, 6, 39]
    # the recent block is present even when it has the lowest score
    sc2 = np.arange(10, dtype=np.float32)[::-1].copy()[None]
    assert list(oracle.select(sc2, 3)[0]) == [0, 1, 2, 9]
    # NB - 1 <= K: everything is taken
    assert list(oracle.select(sc2, 20)[0]) == list(range(10))


def test_attend_f64_matches_numpy(oracle_lib):
    w = CONFIGS["c0"].with_(name="c0_T1000_K4", T=1000, K=4)
    c = host_case(w, seed=2)
    ref = oracle.np_attend_f64(c["q"], c["Kc"].floats(), c["Vc"].floats(), w.Hkv, w.T, w.S, c["sel"], c["scale"])
    assert np.allclose(c["out"], ref, rtol=1e-12, atol=1e-12)


def test_all_blocks_equals_dense_attention(oracle_lib):
    w = CONFIGS["c0"].with_(name="c0_T777_K64", T=777, K=64)  # K >= NB - 1: every block
    c = host_case(w, seed=4)
    assert c["sel"].shape[1] == w.NB
    B, Hq, D = w.B, w.Hq, w.D
    kf, vf = c["Kc"].floats(), c["Vc"].floats()
    dense = np.zeros((B * Hq, D))
    for hq in range(Hq):
        s = kf[hq // w.G, :w.T].astype(np.float64) @ c["q"][0, hq].astype(np.float64) * c["scale"]
        p = np.exp(s - s.max())
        dense[hq] = p @ vf[hq // w.G, :w.T].astype(np.float64) / p.sum()
    assert np.allclose(c["out"], dense, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", ["c0", "c1"])
def test_needles_are_retrieved(oracle_lib, name):
    w = CONFIGS[name]
    if name == "c1":
        w = w.with_(T=8192)
    c = host_case(w, seed=21)
    for bh in range(w.B * w.Hkv):
        chosen = set(c["sel"][bh].tolist())
        assert set(c["needles"][bh // w.Hkv].tolist()) <= chosen
        assert c["sel"][bh][-1] == w.NB - 1


@pytest.mark.parametrize("bits", [0, 8, 4])
def test_cpu_baseline_matches_f64(oracle_lib, bits):
    w = CONFIGS["c2q8"].with_(name=f"c2_reduced_B1_T4096_q{bits}", B=1, T=4096, bits=bits)
    c = host_case(w, seed=8)
    out, sel = oracle.decode_f32(c["qs"], c["dt"], c["Kc"], c["Vc"], c["summ"], c["dt"], w.B, w.Hq, w.Hkv, w.T,
                                 w.S, w.K, c["scale"], threads=2)
    assert np.array_equal(sel, c["sel"])
    assert_close(oracle.to_f32(out, c["dt"]).reshape(-1, w.D), c["out"], w.dtype)


def test_sharded_topk_equals_global(oracle_lib):
    """Local top-K per stripe, then top-K of the union == global top-K."""
    rng = np.random.default_rng(9)
    NB, K, P = 300, 20, 4
    sc = rng.standard_normal(NB).astype(np.float32)
    sc[[10, 50, 90]] = sc[5]  # ties across stripes
    glob, _ = oracle.topk(sc[:-1], np.arange(NB - 1, dtype=np.int32), K)
    cands_s, cands_i = [], []
    for p in range(P):
        idx = np.arange(p, NB - 1, P, dtype=np.int32)
        i, s = oracle.topk(sc[idx], idx, K)
        cands_s.append(s)
        cands_i.append(i)
    merged, _ = oracle.topk(np.concatenate(cands_s), np.concatenate(cands_i), K)
    assert np.array_equal(merged, glob)


def test_golden_fixtures(oracle_lib):
    files = sorted(GOLDEN.glob("*.npz"))
    assert files, "golden fixtures missing (tests/golden/make_golden.py)"
    for f in files:
        g = np.load(f)
        dt = int(g["dtype"])
        B, Hq, Hkv, D, T, S, K, bits = (int(g[n]) for n in ("B", "Hq", "Hkv", "D", "T", "S", "K", "bits"))
        if bits:
            Kc = oracle.Cache(dt, D, g["k_wq"], bits, g["k_scales"], g["k_biases"])
            Vc = oracle.Cache(dt, D, g["v_wq"], bits, g["v_scales"], g["v_biases"])
        else:
            Kc, Vc = oracle.Cache(dt, D, g["k"]), oracle.Cache(dt, D, g["v"])
        summ = oracle.summaries(Kc, T, S, dt)
        assert np.array_equal(summ, g["summaries"]), f.name
        sc = oracle.scores(g["q"], dt, summ, dt, B, Hq, Hkv, D, (T + S - 1) // S, float(g["scale"]))
        assert np.array_equal(sc, g["scores"]), f.name
        sel = oracle.select(sc, K)
        assert np.array_equal(sel, g["sel"]), f.name
        out = oracle.attend_f64(g["q"], dt, Kc, Vc, B, Hq, Hkv, T, S, sel, float(g["scale"]))
        assert np.allclose(out, g["out"], rtol=1e-12, atol=1e-12), f.name
        if bits:
            x = g["k_src"]
            wq, s_, b_ = oracle.quantize(x, dt, D, bits)
            assert np.array_equal(wq, g["k_wq"]) and np.array_equal(s_, g["k_scales"]), f.name
