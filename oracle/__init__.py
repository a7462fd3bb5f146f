"""CPU oracle for the retrieval block-sparse decode path -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this package; the product path (mlx-swift-lm_b200) never does.

PARITY UNPINNED: the reference snapshot holds no implementation of this path
and no golden vectors for it, and MLX (which holds the quantization and SDPA
arithmetic the reference calls) is not vendored. This package exposes:

* `sd_oracle.cpp` (built into liboracle.so) through ctypes -- the canonical-order
  restatement used for bit-exact selection checks and fp64 attention;
* `sd_cpu_baseline.cpp` (same library) -- the timed fp32 CPU implementation of
  the whole path (thread pool, AVX2), checked against the fp64 oracle;
* a pure-numpy twin of each stage (`np_*`), written independently, used at
  small sizes to cross-check the C++ restatement.

Arrays: bf16 tensors are numpy uint16 bit patterns, fp16 are float16, fp32
float32. dtype codes: 0 = f32, 1 = f16, 2 = bf16.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

F32, F16, BF16 = 0, 1, 2
NP_STORAGE = {F32: np.float32, F16: np.float16, BF16: np.uint16}


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (g++ only)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


class KVView(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int32), ("dtype", ctypes.c_int32), ("group_size", ctypes.c_int32),
                ("cap", ctypes.c_int32), ("D", ctypes.c_int32), ("data", ctypes.c_void_p),
                ("scales", ctypes.c_void_p), ("biases", ctypes.c_void_p)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64, f32, f64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_double
        kvp = ctypes.POINTER(KVView)
        L.orc_set_threads.argtypes = [i32]
        L.orc_quantize.argtypes = [vp, i32, i64, i32, i32, i32, vp, vp, vp]
        L.orc_dequantize.argtypes = [vp, vp, vp, i32, i64, i32, i32, i32, vp]
        L.orc_summaries.argtypes = [kvp, i64, i32, i32, i32, i32, i32, vp, i32]
        L.orc_scores.argtypes = [vp, i32, vp, i32, i32, i32, i32, i32, i32, i32, f32, vp]
        L.orc_select.argtypes = [vp, i64, i32, i32, vp, i32]
        L.orc_select.restype = i32
        L.orc_topk.argtypes = [vp, vp, i32, i32, vp, vp]
        L.orc_topk.restype = i32
        L.orc_attend_f64.argtypes = [vp, i32, kvp, kvp, i32, i32, i32, i32, i32, vp, i32, i32, f64, i32, vp, vp, vp]
        L.orc_merge_f64.argtypes = [i32, i64, i32, vp, vp, vp, vp]
        L.orc_base_set_threads.argtypes = [i32]
        L.orc_base_last_threads.restype = i32
        L.orc_base_decode.argtypes = [vp, i32, kvp, kvp, vp, i32, i32, i32, i32, i32, i32, i32, i32, f32, vp, vp]
        L.orc_base_decode.restype = i32
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------------------
# dtype helpers (bf16 as uint16 bit patterns, round half to even)
# ---------------------------------------------------------------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_storage(x: np.ndarray, dtype: int) -> np.ndarray:
    """fp32 values -> storage array of `dtype` (RNE)."""
    if dtype == F32:
        return np.ascontiguousarray(x, dtype=np.float32)
    if dtype == F16:
        return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16)
    return f32_to_bf16_bits(x)


def to_f32(a: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == BF16:
        return bf16_bits_to_f32(a)
    return np.ascontiguousarray(a).astype(np.float32)


def round_to(x: np.ndarray, dtype: int) -> np.ndarray:
    return to_f32(to_storage(x, dtype), dtype)


# ---------------------------------------------------------------------------
# Cache views for the C++ oracle
# ---------------------------------------------------------------------------
class Cache:
    """One K or V cache on the host: dense storage [BH, cap, D] of dtype, or
    quantized (wq uint32 [BH, cap, D*bits/32], scales/biases [BH, cap, D/64])."""

    def __init__(self, dtype: int, D: int, data: np.ndarray, bits: int = 0, scales=None, biases=None):
        self.dtype, self.D, self.bits = dtype, D, bits
        self.data = np.ascontiguousarray(data)
        self.scales = None if scales is None else np.ascontiguousarray(scales)
        self.biases = None if biases is None else np.ascontiguousarray(biases)
        self.cap = self.data.shape[1]

    def view(self) -> KVView:
        return KVView(self.bits, self.dtype, 64, self.cap, self.D, _p(self.data), _p(self.scales), _p(self.biases))

    def floats(self) -> np.ndarray:
        """All rows as fp32 values [BH, cap, D] (dequantized when quantized)."""
        if self.bits == 0:
            return to_f32(self.data, self.dtype).reshape(self.data.shape)
        BH, cap = self.data.shape[:2]
        out = np.empty((BH, cap, self.D), np.float32)
        lib().orc_dequantize(_p(self.data), _p(self.scales), _p(self.biases), self.dtype, BH * cap, self.D, 64,
                             self.bits, _p(out))
        return out


def quantize(x_storage: np.ndarray, dtype: int, D: int, bits: int):
    """Affine group-64 quantization of rows [..., D] -> (wq, scales, biases)."""
    rows = x_storage.size // D
    lead = x_storage.shape[:-1]
    wq = np.empty(lead + (D * bits // 32,), np.uint32)
    sc = np.empty(lead + (D // 64,), NP_STORAGE[dtype])
    bi = np.empty(lead + (D // 64,), NP_STORAGE[dtype])
    lib().orc_quantize(_p(np.ascontiguousarray(x_storage)), dtype, rows, D, 64, bits, _p(wq), _p(sc), _p(bi))
    return wq, sc, bi


def summaries(K: Cache, T: int, S: int, sdtype: int, nb: int | None = None) -> np.ndarray:
    BH = K.data.shape[0]
    NB = (T + S - 1) // S
    nb = nb or NB
    out = np.zeros((BH, nb, K.D), NP_STORAGE[sdtype])
    v = K.view()
    lib().orc_summaries(ctypes.byref(v), BH, T, S, 0, NB, sdtype, _p(out), nb)
    return out


def scores(q: np.ndarray, qdtype: int, summ: np.ndarray, sdtype: int, B: int, Hq: int, Hkv: int, D: int, NB: int,
           scale: float) -> np.ndarray:
    out = np.empty((B * Hkv, NB), np.float32)
    lib().orc_scores(_p(np.ascontiguousarray(q)), qdtype, _p(summ), sdtype, B, Hq, Hkv, D, NB, summ.shape[1],
                     np.float32(scale), _p(out))
    return out


def select(sc: np.ndarray, K: int) -> np.ndarray:
    """[BH, NB] scores -> [BH, n_sel] blocks: top-K of [0, NB-1) ascending, then NB-1."""
    BH, NB = sc.shape
    n_sel = min(K, NB - 1) + 1
    out = np.empty((BH, n_sel), np.int32)
    lib().orc_select(_p(np.ascontiguousarray(sc, dtype=np.float32)), BH, NB, K, _p(out), n_sel)
    return out


def topk(sc: np.ndarray, idx: np.ndarray, K: int):
    """Top-K of candidate (score, block) pairs by (score desc, block asc), sorted by block."""
    sc = np.ascontiguousarray(sc, dtype=np.float32)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    oi = np.empty(min(K, len(sc)), np.int32)
    os_ = np.empty(min(K, len(sc)), np.float32)
    m = lib().orc_topk(_p(sc), _p(idx), len(sc), K, _p(oi), _p(os_))
    return oi[:m], os_[:m]


def attend_f64(q, qdtype, Kc: Cache, Vc: Cache, B, Hq, Hkv, T, S, sel: np.ndarray, scale: float,
               normalise: bool = True):
    """fp64 attention over the selected blocks. Returns out [B*Hq, D] (and m, l
    in natural-log units when normalise is False, with o unnormalised)."""
    D = Kc.D
    sel = np.ascontiguousarray(sel, dtype=np.int32)
    o = np.empty((B * Hq, D), np.float64)
    m = np.empty(B * Hq, np.float64)
    l_ = np.empty(B * Hq, np.float64)
    kv, vv = Kc.view(), Vc.view()
    lib().orc_attend_f64(_p(np.ascontiguousarray(q)), qdtype, ctypes.byref(kv), ctypes.byref(vv), B, Hq, Hkv, T, S,
                         _p(sel), sel.shape[1], sel.shape[1], float(scale), 1 if normalise else 0, _p(m), _p(l_),
                         _p(o))
    return o if normalise else (m, l_, o)


def merge_f64(m: np.ndarray, l_: np.ndarray, o: np.ndarray) -> np.ndarray:
    P, BQ, D = o.shape
    out = np.empty((BQ, D), np.float64)
    lib().orc_merge_f64(P, BQ, D, _p(np.ascontiguousarray(m)), _p(np.ascontiguousarray(l_)),
                        _p(np.ascontiguousarray(o)), _p(out))
    return out


def decode_f32(q, qdtype, Kc: Cache, Vc: Cache, summ, sdtype, B, Hq, Hkv, T, S, K, scale, threads=0):
    """Whole path in fp32 on host threads: the timed CPU implementation
    (sd_cpu_baseline.cpp; threads=0 uses every hardware thread). Returns
    (out, sel); `last_threads()` tells how many threads ran tasks."""
    D = Kc.D
    out = np.empty((B, Hq, D), NP_STORAGE[qdtype])
    n_sel = min(K, (T + S - 1) // S - 1) + 1
    sel = np.empty((B * Hkv, n_sel), np.int32)
    kv, vv = Kc.view(), Vc.view()
    lib().orc_base_set_threads(threads)
    lib().orc_base_decode(_p(np.ascontiguousarray(q)), qdtype, ctypes.byref(kv), ctypes.byref(vv), _p(summ), sdtype,
                          summ.shape[1], B, Hq, Hkv, T, S, K, np.float32(scale), _p(out), _p(sel))
    return out, sel


def last_threads() -> int:
    """Threads that ran at least one task in the last decode_f32 call."""
    return int(lib().orc_base_last_threads())


# ---------------------------------------------------------------------------
# numpy twin (independent restatement, small sizes)
# ---------------------------------------------------------------------------
def np_quantize(x: np.ndarray, bits: int):
    """x: fp32 values [..., D] -> (codes uint8 [..., D], scale fp32 [..., D/64], bias fp32)."""
    D = x.shape[-1]
    g = x.reshape(x.shape[:-1] + (D // 64, 64)).astype(np.float32)
    n_bins = np.float32(2 ** bits - 1)
    wmax, wmin = g.max(-1), g.min(-1)
    scale = np.maximum((wmax - wmin) / n_bins, np.float32(1e-7)).astype(np.float32)
    mask = np.abs(wmin) > np.abs(wmax)
    scale = np.where(mask, scale, -scale).astype(np.float32)
    edge = np.where(mask, wmin, wmax).astype(np.float32)
    q0 = np.rint(edge / scale).astype(np.float32)
    scale = np.where(q0 != 0, edge / np.where(q0 != 0, q0, 1), scale).astype(np.float32)
    bias = np.where(q0 == 0, np.float32(0), edge).astype(np.float32)
    c = np.clip(np.rint((g - bias[..., None]) / scale[..., None]), 0, n_bins)
    return c.reshape(x.shape).astype(np.uint8), scale, bias


def np_pack(codes: np.ndarray, bits: int) -> np.ndarray:
    per = 32 // bits
    c = codes.astype(np.uint32).reshape(codes.shape[:-1] + (codes.shape[-1] // per, per))
    sh = (np.arange(per, dtype=np.uint32) * bits)
    return np.bitwise_or.reduce(c << sh, axis=-1).astype(np.uint32)


def np_unpack(wq: np.ndarray, bits: int) -> np.ndarray:
    per = 32 // bits
    sh = (np.arange(per, dtype=np.uint32) * bits)
    c = (wq[..., None] >> sh) & np.uint32(2 ** bits - 1)
    return c.reshape(wq.shape[:-1] + (wq.shape[-1] * per,)).astype(np.uint8)


def np_summaries(Kf: np.ndarray, T: int, S: int, sdtype: int) -> np.ndarray:
    """Kf: fp32 [BH, >=T, D] -> summaries as fp32 values rounded to sdtype."""
    BH, _, D = Kf.shape
    NB = (T + S - 1) // S
    out = np.zeros((BH, NB, D), np.float32)
    for j in range(NB):
        t0, t1 = j * S, min((j + 1) * S, T)
        acc = Kf[:, t0].astype(np.float32).copy()
        for t in range(t0 + 1, t1):
            acc = (acc + Kf[:, t]).astype(np.float32)
        out[:, j] = acc / np.float32(t1 - t0)
    return round_to(out, sdtype)


def np_scores_f64(qf: np.ndarray, summ_f: np.ndarray, Hkv: int, scale: float) -> np.ndarray:
    """fp64 block scores: qf [B, Hq, D], summ_f [B*Hkv, NB, D] -> [B*Hkv, NB]."""
    B, Hq, D = qf.shape
    G = Hq // Hkv
    qs = qf.astype(np.float64).reshape(B, Hkv, G, D).sum(2).reshape(B * Hkv, D)
    return np.einsum("bd,bnd->bn", qs, summ_f.astype(np.float64)) * scale


def np_select(sc: np.ndarray, K: int) -> np.ndarray:
    BH, NB = sc.shape
    n = NB - 1
    out = []
    for r in range(BH):
        order = sorted(range(n), key=lambda j: (-float(sc[r, j]), j))[:K]
        out.append(sorted(order) + [NB - 1])
    return np.array(out, np.int32)


def np_attend_f64(qf, Kf, Vf, Hkv, T, S, sel, scale):
    """qf [B, Hq, D]; Kf/Vf fp32 [B*Hkv, >=T, D]; sel [B*Hkv, n] -> out [B*Hq, D] fp64."""
    B, Hq, D = qf.shape
    G = Hq // Hkv
    out = np.zeros((B * Hq, D))
    for b in range(B):
        for hq in range(Hq):
            bh = b * Hkv + hq // G
            toks = np.concatenate([np.arange(j * S, min((j + 1) * S, T)) for j in sel[bh] if j >= 0])
            k = Kf[bh, toks].astype(np.float64)
            v = Vf[bh, toks].astype(np.float64)
            s = k @ qf[b, hq].astype(np.float64) * scale
            p = np.exp(s - s.max())
            out[b * Hq + hq] = p @ v / p.sum()
    return out
