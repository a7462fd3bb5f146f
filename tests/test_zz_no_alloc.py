"""The decode entry point that allocates no device memory (sd_decode_noalloc).

Some callers own all of the GPU's memory -- e.g. a serving runtime that
reserves the device's memory pool at start-up and lends slices of it to its
plug-ins -- and cannot let a library call cudaMalloc. For them the library
offers one decode call that takes the caller's own cache arrays and keeps its
scratch (the message words through which a group's CTAs merge their partial
results, and the groups' epochs) in a fixed device array compiled into the
library. This file is collected last on purpose.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [0, 8])
def test_noalloc_decode_matches_sd_decode_twice(cuda, bits):
    """bits 8: the caller's scale/bias arrays reach the kernel as four 1-D
    bulk copies per tile (the index's own arena uses one tiled copy)."""
    import torch

    import sparse_decode as sd
    from sparse_decode.synth import CONFIGS

    from _util import assert_close, host_case
    from gpu_cases import to_dev, to_host

    # 8 (batch, kv-head) groups: several replicas, so the scratch holds partials
    w = CONFIGS["c1"].with_(name=f"c1_reduced_T8192_q{bits}", T=8192, bits=bits)
    c = host_case(w, seed=77)
    B, Hkv, T, D = w.B, w.Hkv, w.T, w.D
    idx = sd.SparseIndex(B, w.Hq, Hkv, D, w.S, w.K, T, w.dtype, w.bits)
    assert idx.replicas > 1
    k = to_dev(c["ks"].reshape(B, Hkv, T, D), w.dtype)
    v = to_dev(c["vs"].reshape(B, Hkv, T, D), w.dtype)
    idx.append(k, v)
    q = to_dev(c["qs"], w.dtype)

    # the existing entry point, decoding the same token without an append
    ref_sel = torch.full((B * Hkv, w.K + 1), -7, dtype=torch.int32, device="cuda")
    ref = idx.decode(q, scale=c["scale"], sel_out=ref_sel)
    torch.cuda.synchronize()
    ref_h = to_host(ref, w.dtype).reshape(-1, D)
    assert_close(ref_h, c["out"], w.dtype)

    lib = sd.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # the second call sees the scratch the first one left behind
        out = torch.empty_like(q)
        sel = torch.full((B * Hkv, w.K + 1), -7, dtype=torch.int32, device="cuda")
        flags = torch.zeros(1, dtype=torch.int32, device="cuda")
        rc = lib.sd_decode_noalloc(ctypes.byref(idx.cfg), ctypes.byref(idx._arrays), T, q.data_ptr(), c["scale"],
                                   out.data_ptr(), sel.data_ptr(), flags.data_ptr(), stream)
        assert rc == 0, lib.sd_last_error().decode()
        torch.cuda.synchronize()
        assert int(flags.item()) == 0, f"call {call}: device error bits {int(flags.item())}"
        assert np.array_equal(sel.cpu().numpy(), ref_sel.cpu().numpy()), f"call {call}"
        got = to_host(out, w.dtype).reshape(-1, D)
        assert_close(got, ref_h.astype(np.float64), w.dtype)  # against the existing entry point
        assert_close(got, c["out"], w.dtype)                   # and against the fp64 oracle


def _noalloc(idx, T, q, scale, K1):
    import torch

    import sparse_decode as sd
    lib = sd.lib()
    out = torch.empty_like(q)
    sel = torch.full((idx.cfg.batch * idx.cfg.n_kv_heads, K1), -7, dtype=torch.int32, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.sd_decode_noalloc(ctypes.byref(idx.cfg), ctypes.byref(idx._arrays), T, q.data_ptr(), scale,
                               out.data_ptr(), sel.data_ptr(), flags.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.sd_last_error().decode()
    torch.cuda.synchronize()
    assert int(flags.item()) == 0, f"device error bits {int(flags.item())}"
    return out, sel


def test_noalloc_large_scratch_uses_a_smaller_launch(cuda):
    """G = 8 heads of D = 128 per group: the group merge's message words of the
    index's own launch shape need more than the 1 MiB scratch, so the entry
    point takes fewer CTAs per group (fewer replicas, then smaller clusters
    with replicas raised again where they fit). The selection must equal the
    index's own decode and the oracle's, the output both within tolerance;
    then a call of another configuration, right after, still matches."""
    import torch

    import sparse_decode as sd
    from sparse_decode.synth import Workload

    from _util import assert_close, host_case
    from gpu_cases import to_dev, to_host

    w = Workload("noalloc_g8_d128", B=1, Hq=64, Hkv=8, D=128, T=6000, S=64, K=16, dtype="bf16", needles=3)
    w2 = Workload("noalloc_q8_small", B=1, Hq=8, Hkv=2, D=128, T=3000, S=64, K=8, dtype="bf16", bits=8, needles=2)
    done = []
    for i, x in enumerate((w, w2)):
        c = host_case(x, seed=91 + i)
        B, Hkv, T, D = x.B, x.Hkv, x.T, x.D
        idx = sd.SparseIndex(B, x.Hq, Hkv, D, x.S, x.K, T, x.dtype, x.bits)
        k = to_dev(c["ks"].reshape(B, Hkv, T, D), x.dtype)
        v = to_dev(c["vs"].reshape(B, Hkv, T, D), x.dtype)
        idx.append(k, v)
        q = to_dev(c["qs"], x.dtype)
        ref_sel = torch.full((B * Hkv, x.K + 1), -7, dtype=torch.int32, device="cuda")
        ref = idx.decode(q, scale=c["scale"], sel_out=ref_sel)
        torch.cuda.synchronize()
        out, sel = _noalloc(idx, T, q, c["scale"], x.K + 1)
        assert np.array_equal(sel.cpu().numpy(), ref_sel.cpu().numpy()), x.name
        assert np.array_equal(sel.cpu().numpy()[:, : x.n_sel], c["sel"]), x.name
        got = to_host(out, x.dtype).reshape(-1, D)
        assert_close(got, to_host(ref, x.dtype).reshape(-1, D).astype(np.float64), x.dtype)
        assert_close(got, c["out"], x.dtype)
        done.append(idx)


def test_noalloc_rejects_bad_arguments(cuda):
    import sparse_decode as sd

    lib = sd.lib()
    cfg = sd.SDConfig(1, 8, 2, 128, 64, 8, 1024, 2, 0, 0, 0, 1, 0)
    arrays = sd.SDArrays()
    rc = lib.sd_decode_noalloc(ctypes.byref(cfg), ctypes.byref(arrays), 10, None, 0.1, None, None, None, None)
    assert rc == 1  # SD_ERR_INVALID_ARG: NULL queries/output/arrays
