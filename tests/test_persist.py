"""Prompt-cache files (the reference's savePromptCache / loadPromptCache
layout: tensors "i.j", metadata "0.i.j" / "1.key" / "2.i" in one safetensors
file). CPU: the container and the layout, written and read back; GPU: a
SparseKVCache saved and loaded decodes exactly like the original, and the
reference's dense / quantized cache entries load as SparseKVCache."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest

from sparse_decode.persist import read_safetensors, write_safetensors


def test_safetensors_round_trip(tmp_path):
    import torch
    g = torch.Generator().manual_seed(0)
    t = {"0.0": torch.randn(1, 2, 5, 8, generator=g).to(torch.bfloat16),
         "0.1": torch.randn(1, 2, 5, 8, generator=g),
         "1.0": torch.randint(0, 2 ** 31 - 1, (1, 2, 5, 4), generator=g, dtype=torch.int32),
         "1.1": torch.randn(3, generator=g).to(torch.float16)}
    meta = {"0.0.0": "256", "1.model": "x", "2.0": "SparseKVCache"}
    p = tmp_path / "c.safetensors"
    write_safetensors(str(p), t, meta)
    raw = p.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    assert header["__metadata__"] == meta
    assert header["0.0"]["dtype"] == "BF16" and header["1.0"]["dtype"] == "I32"
    assert (8 + n) % 8 == 0
    back, m2 = read_safetensors(str(p))
    assert m2 == meta
    for k in t:
        assert back[k].dtype == t[k].dtype and torch.equal(back[k], t[k]), k


def test_truncated_file_is_rejected(tmp_path):
    import torch
    p = tmp_path / "c.safetensors"
    write_safetensors(str(p), {"0.0": torch.zeros(4, 4)}, {})
    p.write_bytes(p.read_bytes()[:-8])
    with pytest.raises(ValueError):
        read_safetensors(str(p))


def _cache_case(bits):
    import torch
    from sparse_decode import SparseKVCache
    g = torch.Generator(device="cuda").manual_seed(3)
    B, Hq, Hkv, D, T = 1, 8, 2, 128, 64 * 9 + 7
    k = torch.randn(B, Hkv, T, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g, device="cuda").to(torch.bfloat16)
    c = SparseKVCache(Hq, block_size=64, top_k=4, kv_bits=bits or None)
    c._append(k[:, :, : T - 1], v[:, :, : T - 1])
    q = torch.randn(B, Hq, 1, D, generator=g, device="cuda").to(torch.bfloat16)
    return c, q, k[:, :, T - 1:], v[:, :, T - 1:]


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [0, 8])
def test_saved_cache_decodes_like_the_original(cuda, tmp_path, bits):
    import torch
    from sparse_decode import load_prompt_cache, save_prompt_cache
    c, q, kn, vn = _cache_case(bits)
    p = tmp_path / "p.safetensors"
    save_prompt_cache(str(p), [c], {"model": "synthetic"})
    (c2,), meta = load_prompt_cache(str(p))
    assert meta == {"model": "synthetic"}
    assert c2.offset == c.offset and c2.bits == c.bits and c2.top_k == c.top_k
    o1 = c._decode(q, kn, vn, 128 ** -0.5)
    o2 = c2._decode(q, kn, vn, 128 ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


@pytest.mark.gpu
def test_reference_dense_and_quantized_entries_load_as_sparse(cuda, tmp_path):
    """Entries as the reference writes them for KVCacheSimple ("KVCache",
    state [keys, values]) and QuantizedKVCache (6 arrays, metaState [step,
    offset, groupSize, bits]) load into SparseKVCache with summaries built."""
    import torch
    from sparse_decode import load_prompt_cache
    from sparse_decode.persist import write_safetensors
    c, q, kn, vn = _cache_case(0)
    cq, _, _, _ = _cache_case(8)
    k, v = c.state
    tensors = {"0.0": k, "0.1": v}
    for j, a in enumerate(cq.state):
        tensors[f"1.{j}"] = a
    meta = {"0.0.0": "256", "0.0.1": str(c.offset), "2.0": "KVCache",
            "0.1.0": "256", "0.1.1": str(cq.offset), "0.1.2": "64", "0.1.3": "8", "2.1": "QuantizedKVCache"}
    p = tmp_path / "ref.safetensors"
    write_safetensors(str(p), tensors, meta)
    with pytest.raises(ValueError):
        load_prompt_cache(str(p))
    (d, qz), _ = load_prompt_cache(str(p), sparse={"n_q_heads": 8, "block_size": 64, "top_k": 4})
    assert d.offset == c.offset and qz.bits == 8 and qz.offset == cq.offset
    for a, b in ((c, d), (cq, qz)):
        o1 = a._decode(q, kn, vn, 128 ** -0.5)
        o2 = b._decode(q, kn, vn, 128 ** -0.5)
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        sa, sb = a.index.views()["summaries"], b.index.views()["summaries"]
        assert torch.equal(sa, sb)


@pytest.mark.gpu
def test_maybe_quantize_converts_after_the_start(cuda):
    from sparse_decode import make_prompt_cache, maybe_quantize_kv_cache
    caches = make_prompt_cache(2, 8, block_size=64, top_k=4)
    c, q, kn, vn = _cache_case(0)
    caches[0] = c
    maybe_quantize_kv_cache(caches, 8, 64, quantized_kv_start=10_000)
    assert caches[0] is c
    maybe_quantize_kv_cache(caches, 8, 64, quantized_kv_start=100)
    assert caches[0].bits == 8 and caches[0].offset == c.offset
    assert caches[1].offset == 0 and caches[1].bits == 0  # empty caches stay as they are
    o = caches[0]._decode(q, kn, vn, 128 ** -0.5)
    assert o.shape == q.shape
