"""Attention sinks (sd_set_sinks): a per-head logit that joins the softmax
denominator without contributing a value, as the reference's sink-attention
models compute it (MLXFast.scaledDotProductAttention(..., sinks:),
Libraries/MLXLLM/Models/GPTOSS.swift:228-261, MiMoV2Flash.swift:14-56).
The fp64 reference is the oracle's unnormalised attention (m, l, o) over the
same selected blocks: out = o / (l + e^(sink - m))."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from sparse_decode.synth import Workload

from _util import assert_close, host_case
from gpu_cases import to_dev, to_host

pytestmark = pytest.mark.gpu

W = Workload("sinks", B=2, Hq=8, Hkv=2, D=128, T=64 * 24 + 9, S=64, K=6, dtype="bf16", needles=3)


def _sinks(w, seed=7):
    rng = np.random.default_rng(seed)
    return rng.uniform(-2.0, 6.0, w.Hq).astype(np.float32)


def _reference(w, c, sinks):
    m, l_, o = oracle.attend_f64(c["qs"], c["dt"], c["Kc"], c["Vc"], w.B, w.Hq, w.Hkv, w.T, w.S, c["sel"], c["scale"],
                                 normalise=False)
    s = np.tile(sinks.astype(np.float64), w.B)
    return o / (l_ + np.exp(s - m))[:, None]


def _index(w, c, **kw):
    import torch
    from sparse_decode import SparseIndex
    idx = SparseIndex(w.B, w.Hq, w.Hkv, w.D, w.S, w.K, w.T, w.dtype, w.bits, **kw)
    k = to_dev(c["ks"].reshape(w.B, w.Hkv, w.T, w.D), w.dtype)
    v = to_dev(c["vs"].reshape(w.B, w.Hkv, w.T, w.D), w.dtype)
    idx.append(k[:, :, : w.T - 1].contiguous(), v[:, :, : w.T - 1].contiguous())
    return idx, to_dev(c["qs"], w.dtype), k[:, :, w.T - 1].contiguous(), v[:, :, w.T - 1].contiguous()


@pytest.mark.parametrize("bits", [0, 8])
def test_decode_with_sinks_matches_oracle(cuda, bits):
    import torch
    w = W.with_(bits=bits)
    c = host_case(w, 11)
    sinks = _sinks(w)
    idx, q, kn, vn = _index(w, c)
    idx.set_sinks(torch.from_numpy(sinks).cuda())
    out = idx.decode(q, kn, vn, c["scale"])
    torch.cuda.synchronize()
    assert idx.check_device() == 0
    assert_close(to_host(out, w.dtype).reshape(-1, w.D), _reference(w, c, sinks), w.dtype)
    # off again: the plain output
    idx.trim(1)
    idx.set_sinks(None)
    out = idx.decode(q, kn, vn, c["scale"])
    torch.cuda.synchronize()
    assert_close(to_host(out, w.dtype).reshape(-1, w.D), c["out"], w.dtype)


def test_sharded_merge_and_peer_step_apply_sinks(cuda):
    """The NCCL-path merge (sd_shard_merge, shards on one GPU, gathers by
    concatenation) and the fused step with one shard apply the same sinks."""
    import torch
    from sparse_decode import ShardComm
    w = W
    c = host_case(w, 12)
    sinks = torch.from_numpy(_sinks(w, 8)).cuda()
    ref = _reference(w, c, sinks.cpu().numpy())
    P = 2
    shards = [_index(w, c, shard_rank=r, shard_count=P) for r in range(P)]
    cs, cb = [], []
    for idx, q, kn, vn in shards:
        s_ = torch.empty((w.B * w.Hkv, w.K), device="cuda")
        b_ = torch.empty((w.B * w.Hkv, w.K), device="cuda", dtype=torch.int32)
        idx.shard_candidates(q, s_, b_, kn, vn, c["scale"])
        cs.append(s_)
        cb.append(b_)
    mls, pos = [], []
    for idx, q, _, _ in shards:
        ml = torch.empty((w.B * w.Hq, 2), device="cuda")
        po = torch.empty((w.B * w.Hq, w.D), device="cuda")
        idx.shard_attend(q, torch.stack(cs), torch.stack(cb), ml, po, c["scale"])
        mls.append(ml)
        pos.append(po)
    out = torch.empty_like(shards[0][1])
    shards[0][0].set_sinks(sinks)
    shards[0][0].shard_merge(torch.stack(mls), torch.stack(pos), out)
    torch.cuda.synchronize()
    assert_close(to_host(out, w.dtype).reshape(-1, w.D), ref, w.dtype)

    one, q, kn, vn = _index(w, c)
    one.set_sinks(sinks)
    want = one.decode(q, kn, vn, c["scale"]).clone()
    one.trim(1)
    comm = ShardComm(one)
    got = one.shard_decode(comm, q, kn, vn, c["scale"])
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    comm.close()


def test_router_with_sinks_prefill_and_decode(cuda):
    """attention_with_cache_update(..., sinks=): prefill (dense over the
    cache) and the sparse single-token step both honour the sinks."""
    import torch
    from sparse_decode import SparseKVCache, attention_with_cache_update
    w = Workload("rsinks", B=1, Hq=8, Hkv=2, D=128, T=64 * 3, S=64, K=8, dtype="bf16")
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(1, 8, 4, 128, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(1, 2, 4, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(1, 2, 4, 128, generator=g, device="cuda").to(torch.bfloat16)
    sinks = torch.tensor(_sinks(w, 9), device="cuda")
    cache = SparseKVCache(8, block_size=64, top_k=8)
    out = attention_with_cache_update(q, k, v, cache, 128 ** -0.5, mask="causal", sinks=sinks)
    kk = k.float().repeat_interleave(4, dim=1)
    vv = v.float().repeat_interleave(4, dim=1)
    s = torch.einsum("bhld,bhtd->bhlt", q.float(), kk) * 128 ** -0.5
    s = s.masked_fill(torch.ones(4, 4, device="cuda").triu(1).bool(), float("-inf"))
    p = torch.softmax(torch.cat([s, sinks.view(1, 8, 1, 1).expand(1, 8, 4, 1)], -1), -1)[..., :-1]
    ref = torch.einsum("bhlt,bhtd->bhld", p, vv)
    assert torch.allclose(out.float(), ref, rtol=2e-2, atol=2e-2)
    # single-token step through the sparse path: all blocks selected here, so
    # it must equal dense attention with the sinks over the 5 cached tokens
    q1 = torch.randn(1, 8, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
    k1 = torch.randn(1, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
    v1 = torch.randn(1, 2, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
    out1 = attention_with_cache_update(q1, k1, v1, cache, 128 ** -0.5, sinks=sinks)
    kc, vc = cache.state
    s1 = torch.einsum("bhd,bhtd->bht", q1[:, :, 0].float(), kc.float().repeat_interleave(4, dim=1)) * 128 ** -0.5
    p1 = torch.softmax(torch.cat([s1, sinks.view(1, 8, 1)], -1), -1)[..., :-1]
    ref1 = torch.einsum("bht,bhtd->bhd", p1, vc.float().repeat_interleave(4, dim=1))
    assert torch.allclose(out1[:, :, 0].float(), ref1, rtol=1e-2, atol=1e-2)
