"""Seeded synthetic decode workloads (no datasets are involved in this path).

Each case is one attention layer's decode step: a context of T tokens whose
first T-1 rows are prefilled and whose last row (k_new, v_new) is appended by
the step itself, plus the step's queries. Q, K, V ~ N(0, 1); "needle" blocks
get +0.5*sqrt(D)*q_hat added to every key, q_hat being the unit sum of the
query heads of the kv group, so that they must be retrieved. Config 2 scales
key channels 0-3 by 8 (outliers) before quantizing; config 4 adds a slow drift
0.1*sin(2*pi*t/T)*u_h of the mean key (u_h a seeded unit vector per kv head).

Two generators with the same recipe: `make_case` (numpy PCG64, any size the
host can hold; used where the CPU oracle must see the same inputs) and
`make_case_torch` (torch CUDA generator, for full-size benchmark layers).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    Hq: int
    Hkv: int
    D: int
    T: int
    S: int
    K: int
    dtype: str          # "f32" | "f16" | "bf16"
    bits: int = 0       # 0 dense, 4/8 affine group-64
    needles: int = 0
    outlier_channels: int = 0
    outlier_scale: float = 1.0
    drift: float = 0.0
    layers: int = 1

    @property
    def G(self) -> int:
        return self.Hq // self.Hkv

    @property
    def NB(self) -> int:
        return (self.T + self.S - 1) // self.S

    @property
    def n_sel(self) -> int:
        return min(self.K, self.NB - 1) + 1

    def with_(self, **kw) -> "Workload":
        return replace(self, **kw)


CONFIGS = {
    "c0": Workload("c0_fp32_T4096", B=1, Hq=8, Hkv=2, D=64, T=4096, S=64, K=8, dtype="f32", needles=6),
    "c1": Workload("c1_qwen3_4b_bf16_T32768", B=1, Hq=32, Hkv=8, D=128, T=32768, S=64, K=64, dtype="bf16",
                   needles=16, layers=36),
    "c2q8": Workload("c2_llama3_8b_q8_T131072_B4", B=4, Hq=32, Hkv=8, D=128, T=131072, S=128, K=32, dtype="bf16",
                     bits=8, needles=8, outlier_channels=4, outlier_scale=8.0),
    "c2q4": Workload("c2_llama3_8b_q4_T131072_B4", B=4, Hq=32, Hkv=8, D=128, T=131072, S=128, K=32, dtype="bf16",
                     bits=4, needles=8, outlier_channels=4, outlier_scale=8.0),
    "c3": Workload("c3_serving_bf16_T131072_B16", B=16, Hq=32, Hkv=8, D=128, T=131072, S=64, K=128, dtype="bf16",
                   needles=32),
    "c4": Workload("c4_q8_T1048576", B=1, Hq=32, Hkv=8, D=128, T=1048576, S=64, K=256, dtype="bf16", bits=8,
                   needles=64, drift=0.1, layers=36),
}

DTYPE_CODE = {"f32": 0, "f16": 1, "bf16": 2}


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to `dtype` (RNE), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    return r.view(np.float32)


def needle_blocks(w: Workload, seed: int, b: int) -> np.ndarray:
    """Seed-chosen needle blocks of sequence b (never the recent block)."""
    rng = np.random.Generator(np.random.PCG64([seed, 7919, b]))
    n = min(w.needles, w.NB - 1)
    return np.sort(rng.choice(w.NB - 1, size=n, replace=False)) if n > 0 else np.zeros(0, np.int64)


def make_case(w: Workload, seed: int) -> dict:
    """numpy case: q [B,Hq,D], k/v [B,Hkv,T,D] (fp32 values already rounded to
    the dtype; rows T-1 are the step's k_new / v_new), needles {b: blocks}."""
    rng = np.random.Generator(np.random.PCG64(seed))
    q = _round(rng.standard_normal((w.B, w.Hq, w.D), dtype=np.float32), w.dtype)
    k = rng.standard_normal((w.B, w.Hkv, w.T, w.D), dtype=np.float32)
    v = rng.standard_normal((w.B, w.Hkv, w.T, w.D), dtype=np.float32)
    if w.outlier_channels:
        k[..., : w.outlier_channels] *= np.float32(w.outlier_scale)
    if w.drift:
        u = rng.standard_normal((w.Hkv, w.D), dtype=np.float32)
        u /= np.linalg.norm(u, axis=-1, keepdims=True)
        ph = np.float32(w.drift) * np.sin(2 * np.pi * np.arange(w.T, dtype=np.float64) / w.T).astype(np.float32)
        k += ph[None, None, :, None] * u[None, :, None, :]
    needles = {}
    qg = q.reshape(w.B, w.Hkv, w.G, w.D).sum(2)
    qhat = qg / np.maximum(np.linalg.norm(qg, axis=-1, keepdims=True), 1e-30)
    for b in range(w.B):
        blocks = needle_blocks(w, seed, b)
        needles[b] = blocks
        for j in blocks:
            k[b, :, j * w.S:(j + 1) * w.S, :] += np.float32(0.5 * math.sqrt(w.D)) * qhat[b, :, None, :]
    k = _round(k, w.dtype)
    v = _round(v, w.dtype)
    return {"q": q, "k": k, "v": v, "needles": needles}


def make_case_torch(w: Workload, seed: int, device="cuda", T_rows: int | None = None):
    """torch case on `device` in the workload dtype: q [B,Hq,D], k/v
    [B,Hkv,T,D]. Same recipe as make_case, different random stream."""
    import torch

    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[w.dtype]
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    T = w.T if T_rows is None else T_rows
    q = torch.randn((w.B, w.Hq, w.D), generator=g, device=device, dtype=torch.float32).to(tdt)
    k = torch.randn((w.B, w.Hkv, T, w.D), generator=g, device=device, dtype=torch.float32)
    if w.outlier_channels:
        k[..., : w.outlier_channels] *= w.outlier_scale
    if w.drift:
        u = torch.randn((w.Hkv, w.D), generator=g, device=device)
        u /= u.norm(dim=-1, keepdim=True)
        t = torch.arange(T, device=device, dtype=torch.float64)
        ph = (w.drift * torch.sin(2 * math.pi * t / w.T)).float()
        k += ph[None, None, :, None] * u[None, :, None, :]
    qg = q.float().reshape(w.B, w.Hkv, w.G, w.D).sum(2)
    qhat = qg / qg.norm(dim=-1, keepdim=True).clamp_min(1e-30)
    needles = {}
    for b in range(w.B):
        blocks = needle_blocks(w, seed, b)
        needles[b] = blocks
        for j in blocks:
            if j * w.S < T:
                k[b, :, j * w.S:(j + 1) * w.S, :] += 0.5 * math.sqrt(w.D) * qhat[b, :, None, :]
    k = k.to(tdt)
    v = torch.randn((w.B, w.Hkv, T, w.D), generator=g, device=device, dtype=torch.float32).to(tdt)
    return {"q": q, "k": k, "v": v, "needles": needles}


def algorithmic_bytes(w: Workload) -> int:
    """Bytes one decode step of one layer must move: every candidate summary,
    the selected blocks' K and V (codes, scales, biases), q and the output."""
    esz = 4 if w.dtype == "f32" else 2
    BH = w.B * w.Hkv
    summ = BH * (w.NB - 1) * w.D * esz
    row = (w.D * w.bits // 8 + 2 * (w.D // 64) * esz) if w.bits else w.D * esz
    n_recent = w.T - (w.NB - 1) * w.S
    sel_tokens = (w.n_sel - 1) * w.S + n_recent
    kv = BH * sel_tokens * 2 * row
    qo = 2 * w.B * w.Hq * w.D * esz
    return summ + kv + qo
