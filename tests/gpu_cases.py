"""Builders shared by the GPU tests: put a host case into a SparseIndex
through the C ABI and collect the GPU results next to the oracle's."""
from __future__ import annotations

import numpy as np

import oracle
from sparse_decode import SparseIndex
from sparse_decode.synth import Workload

from _util import host_case


def to_dev(a: np.ndarray, dtype: str):
    """Host storage array (uint16 bits for bf16) -> CUDA tensor of `dtype`."""
    import torch
    if dtype == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def to_host(t, dtype: str) -> np.ndarray:
    """CUDA tensor -> fp32 numpy values."""
    import torch
    if dtype == "bf16":
        return oracle.bf16_bits_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))
    return t.float().cpu().numpy()


def run_decode(w: Workload, seed: int, cluster: int = 0, c: dict | None = None, capacity: int | None = None):
    """Prefill T-1 rows with sd_append, then one sd_decode step that appends
    row T-1. Returns (case, index, gpu results)."""
    import torch
    c = c or host_case(w, seed)
    B, Hkv, T, D = w.B, w.Hkv, w.T, w.D
    idx = SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, capacity or T, w.dtype, w.bits, cluster_size=cluster)
    k = to_dev(c["ks"].reshape(B, Hkv, T, D), w.dtype)
    v = to_dev(c["vs"].reshape(B, Hkv, T, D), w.dtype)
    if T > 1:
        idx.append(k[:, :, : T - 1].contiguous(), v[:, :, : T - 1].contiguous())
    q = to_dev(c["qs"], w.dtype)
    sel = torch.full((B * Hkv, w.K + 1), -7, dtype=torch.int32, device="cuda")
    scores = torch.full((B * Hkv, w.NB), float("nan"), dtype=torch.float32, device="cuda")
    out = idx.decode(q, k[:, :, T - 1].contiguous(), v[:, :, T - 1].contiguous(), c["scale"], sel_out=sel,
                     scores_out=scores)
    torch.cuda.synchronize()
    res = {"out": to_host(out, w.dtype).reshape(B * w.Hq, D), "sel": sel.cpu().numpy(),
           "scores": scores.cpu().numpy(), "err": idx.check_device()}
    return c, idx, res
