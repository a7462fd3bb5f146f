"""Shared helpers for the parity tests: tolerances and case construction."""
from __future__ import annotations

import numpy as np

import oracle
from sparse_decode.synth import DTYPE_CODE, Workload

# Output tolerances. TOL is the relative error of each head's output row,
# ||out - ref||_2 / ||ref||_2: 2e-3 for fp16/bf16 outputs, 1e-5 for fp32.
# For 16-bit outputs `ref` is the fp64 oracle rounded to the output type --
# the output an exact implementation would return -- because the rounding of
# a bf16 output by itself already costs ~1.6e-3 normwise (and up to 3.9e-3
# element-wise just above a power of two). Element-wise, 16-bit outputs must
# also lie within one unit in the last place of the unrounded fp64 value plus
# ABS_FLOOR * rms(head row) -- the floor covers components that nearly cancel
# to zero, where a 1e-5 absolute fp32 accumulation error is already more than
# one ulp of the tiny value; fp32 outputs within 1e-4 of max(|ref|, row rms)
# (EL_TOL_F32).
TOL = {"bf16": 2e-3, "f16": 2e-3, "f32": 1e-5}
ULPS = 1.0
ABS_FLOOR = 2e-4
EL_TOL_F32 = 1e-4
MANT_BITS = {"bf16": 7, "f16": 10}


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """Largest per-row normwise relative error ||out - ref|| / ||ref||."""
    out = np.asarray(out, np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    num = np.sqrt(((out - ref) ** 2).sum(-1))
    den = np.maximum(np.sqrt((ref ** 2).sum(-1)), 1e-30)
    return float((num / den).max())


def ulp_err(out: np.ndarray, ref: np.ndarray, dtype: str) -> float:
    """Largest (|out - ref| - ABS_FLOOR * rms(row)) in units of the output
    type's ulp at |ref| (<= 1 passes)."""
    out = np.asarray(out, np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    rms = np.sqrt((ref ** 2).mean(-1, keepdims=True))
    e = np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -14)))
    ulp = 2.0 ** (e - MANT_BITS[dtype])
    return float((np.maximum(np.abs(out - ref) - ABS_FLOOR * rms, 0.0) / ulp).max())


def el_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max |out - ref| / max(|ref|, row rms) (element-wise, floored)."""
    out = np.asarray(out, np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    den = np.maximum(np.abs(ref), np.sqrt((ref ** 2).mean(-1, keepdims=True)))
    return float((np.abs(out - ref) / den).max())


def assert_close(out: np.ndarray, ref: np.ndarray, dtype: str) -> None:
    """The output tolerance of this path (see TOL / ULPS / EL_TOL_F32)."""
    ref_out = ref if dtype == "f32" else oracle.round_to(np.asarray(ref, np.float32), oracle.F16 if dtype == "f16" else oracle.BF16)
    r = rel_err(out, np.asarray(ref_out, np.float64).reshape(np.shape(ref)))
    assert r <= TOL[dtype], f"normwise relative error {r:.3g} > {TOL[dtype]}"
    if dtype == "f32":
        e = el_err(out, ref)
        assert e <= EL_TOL_F32, f"element-wise error {e:.3g} > {EL_TOL_F32}"
    else:
        u = ulp_err(out, ref, dtype)
        assert u <= ULPS, f"element-wise error {u:.3g} ulp > {ULPS}"


# The oracle's parallel loops use every host thread (rows and groups are
# independent, so the results do not depend on the thread count).
oracle.lib().orc_set_threads(0)

# Above this many K elements host_case draws its inputs with torch's CPU
# generator (many threads) instead of numpy's; same recipe, another stream.
FAST_ELEMS = 1 << 27


def _storage_from_torch(t, dtype: str) -> np.ndarray:
    import torch
    t = t.contiguous()
    if dtype == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def host_case(w: Workload, seed: int) -> dict:
    """Synthetic case plus its oracle caches (all T rows filled), summaries,
    canonical scores, selection and fp64 outputs."""
    from sparse_decode.synth import make_case, make_case_torch
    dt = DTYPE_CODE[w.dtype]
    B, Hkv, T, D = w.B, w.Hkv, w.T, w.D
    if B * Hkv * T * D > FAST_ELEMS:
        c = make_case_torch(w, seed, device="cpu")
        ks = _storage_from_torch(c["k"], w.dtype).reshape(B * Hkv, T, D)
        vs = _storage_from_torch(c["v"], w.dtype).reshape(B * Hkv, T, D)
        c["q"] = oracle.to_f32(_storage_from_torch(c["q"], w.dtype), dt)
        del c["k"], c["v"]
    else:
        c = make_case(w, seed)
        k = c["k"].reshape(B * Hkv, T, D)
        v = c["v"].reshape(B * Hkv, T, D)
        ks, vs = oracle.to_storage(k, dt), oracle.to_storage(v, dt)
    if w.bits:
        kq = oracle.quantize(ks, dt, D, w.bits)
        vq = oracle.quantize(vs, dt, D, w.bits)
        Kc = oracle.Cache(dt, D, kq[0], w.bits, kq[1], kq[2])
        Vc = oracle.Cache(dt, D, vq[0], w.bits, vq[1], vq[2])
    else:
        Kc, Vc = oracle.Cache(dt, D, ks), oracle.Cache(dt, D, vs)
    summ = oracle.summaries(Kc, T, w.S, dt)
    qs = oracle.to_storage(c["q"], dt)
    scale = 1.0 / np.sqrt(D)
    sc = oracle.scores(qs, dt, summ, dt, B, w.Hq, Hkv, D, w.NB, scale)
    sel = oracle.select(sc, w.K)
    out = oracle.attend_f64(qs, dt, Kc, Vc, B, w.Hq, Hkv, T, w.S, sel, scale)
    c.update(dict(ks=ks, vs=vs, Kc=Kc, Vc=Vc, summ=summ, qs=qs, scale=scale, scores=sc, sel=sel, out=out, dt=dt))
    return c


def boundary_gap_ok(scores: np.ndarray, K: int, tol: float = 1e-3) -> np.ndarray:
    """Per row: True when the K-th and (K+1)-th best candidate scores differ by
    more than `tol` relative, i.e. the selection is well defined."""
    cand = scores[:, :-1]
    if cand.shape[1] <= K:
        return np.ones(scores.shape[0], bool)
    s = -np.sort(-cand, axis=1)
    a, b = s[:, K - 1], s[:, K]
    return np.abs(a - b) > tol * np.maximum(np.abs(a), 1e-30)
