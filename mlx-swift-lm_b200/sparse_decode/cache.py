"""The reference's cache protocol and attention router over a SparseIndex.

`SparseKVCache` follows `protocol KVCache` (Libraries/MLXLMCommon/
KVCache.swift:38-77) -- offset, maxSize, update, state, metaState,
isTrimmable, trim, makeMask, copy -- and, when created with kv_bits, the
`QuantizedKVCacheProtocol` (KVCache.swift:94-119): groupSize, bits, mode,
updateQuantized, getQuantizedState. Names are snake_case; meanings and error
behaviour follow the Swift originals (`update` on a quantized cache is an
error as in QuantizedKVCache.update, KVCache.swift:893-897).

`attention_with_cache_update` is the router of AttentionUtils.swift:37-77
with one extra branch: a SparseKVCache and a single query token (L == 1)
take the retrieval path (one fused kernel launch: append, score, top-K,
attend). Prefill (L > 1) appends through the index and attends densely over
the cached tokens, as the reference does for every step.
"""
from __future__ import annotations

import math
from typing import Optional

from . import SparseIndex, _torch_dtype


class SparseKVCache:
    """Retrieval KV cache for one attention layer.

    Capacity grows like the reference's (multiples of `step` = 256 tokens,
    KVCache.swift:318, :333-362) but geometrically (at least doubling), so a
    long decode re-allocates O(log T) times instead of every 256 tokens.
    """

    step = 256

    def __init__(self, n_q_heads: int, block_size: int = 64, top_k: int = 64, kv_bits: Optional[int] = None,
                 group_size: int = 64, mode: str = "affine", capacity: int = 0, cluster_size: int = 0):
        if kv_bits is not None and mode != "affine":
            raise ValueError("only affine quantization is supported")
        self.n_q_heads = n_q_heads
        self.block_size = block_size
        self.top_k = top_k
        self.bits = kv_bits or 0
        self.group_size = group_size
        self.mode = mode
        self._initial_capacity = capacity
        self.cluster_size = cluster_size
        self.index: Optional[SparseIndex] = None
        self.dtype: Optional[str] = None

    # -- protocol KVCache ------------------------------------------------------
    @property
    def offset(self) -> int:
        return 0 if self.index is None else self.index.offset

    @property
    def max_size(self):
        return None

    @property
    def is_quantized(self) -> bool:
        return self.bits != 0

    @property
    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        return 0 if self.index is None else self.index.trim(n)

    def make_mask(self, n: int, window_size: Optional[int] = None, return_array: bool = False):
        """BaseKVCache.makeMask (KVCache.swift:160-174): None for a single token,
        'causal' otherwise (an explicit boolean mask when asked for one)."""
        if n == 1:
            return None
        if return_array or (window_size is not None and n > window_size):
            import torch
            off = self.offset
            rinds = torch.arange(off + n)
            linds = torch.arange(off, off + n)[:, None]
            mask = linds >= rinds[None]
            if window_size is not None:
                mask &= linds < rinds[None] + window_size
            return mask
        return "causal"

    def update(self, keys, values):
        """Append keys/values [B, Hkv, L, D]; returns the cached keys/values
        [B, Hkv, offset, D] (views of the device arena)."""
        if self.bits:
            raise RuntimeError("`update` was called on a quantized SparseKVCache. Use `update_quantized` instead.")
        self._append(keys, values)
        return self._dense_state()

    def update_quantized(self, keys, values):
        """QuantizedKVCacheProtocol.updateQuantized: append (quantizing) and
        return ((wq, scales, biases), (wq, scales, biases)) [B, Hkv, offset, .]."""
        if not self.bits:
            raise RuntimeError("update_quantized on a dense SparseKVCache")
        self._append(keys, values)
        return self.get_quantized_state()

    def get_quantized_state(self):
        if self.index is None or not self.bits:
            return None
        s = self.state
        return (s[0], s[1], s[2]), (s[3], s[4], s[5])

    @property
    def state(self):
        """[keys, values] (dense) or [wq_k, scales_k, biases_k, wq_v, scales_v,
        biases_v] (quantized), trimmed to offset, shaped [B, Hkv, offset, .]."""
        if self.index is None:
            return []
        if not self.bits:
            return list(self._dense_state())
        v, n = self._views(), self.offset
        B, Hkv = self.index.B, self.index.Hkv
        r = lambda t: t.view(B, Hkv, t.shape[1], t.shape[2])[:, :, :n]
        return [r(v["k"]), r(v["k_scales"]), r(v["k_biases"]), r(v["v"]), r(v["v_scales"]), r(v["v_biases"])]

    @state.setter
    def state(self, arrays):
        import torch
        want = 6 if self.bits else 2
        if len(arrays) != want:
            raise ValueError(f"SparseKVCache state must have exactly {want} arrays")
        k = arrays[0]
        B, Hkv, n = k.shape[0], k.shape[1], k.shape[2]
        D = arrays[0].shape[3] * 32 // self.bits if self.bits else arrays[0].shape[3]
        dtype = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[
            arrays[1].dtype if self.bits else k.dtype]
        self.index = None
        self._create(B, Hkv, D, dtype, max(n, 1))
        v = self._views()
        names = ["k", "k_scales", "k_biases", "v", "v_scales", "v_biases"] if self.bits else ["k", "v"]
        for name, a in zip(names, arrays):
            dst = v[name].view(B, Hkv, v[name].shape[1], v[name].shape[2])
            dst[:, :, :n].copy_(a.reshape(B, Hkv, n, -1).view(dst.dtype))
        self.index.set_offset(n)
        self.index.rebuild_summaries()

    @property
    def meta_state(self):
        """[step, offset, groupSize, bits] as QuantizedKVCache's metaState
        (KVCache.swift:900-944), then blockSize, topK and nQueryHeads."""
        return [str(self.step), str(self.offset), str(self.group_size), str(self.bits), str(self.block_size),
                str(self.top_k), str(self.n_q_heads)]

    @meta_state.setter
    def meta_state(self, values):
        if len(values) != 7:
            raise ValueError("SparseKVCache metaState must have exactly 7 values")
        if self.index is not None:
            self.index.set_offset(int(values[1]))

    def copy(self) -> "SparseKVCache":
        c = SparseKVCache(self.n_q_heads, self.block_size, self.top_k, self.bits or None, self.group_size, self.mode,
                          self._initial_capacity, self.cluster_size)
        if self.index is not None:
            c.index = self.index.copy()
            c.dtype = self.dtype
        return c

    # -- internals ---------------------------------------------------------------
    def _views(self):
        return self.index.views()

    def _dense_state(self):
        v, n = self._views(), self.offset
        B, Hkv = self.index.B, self.index.Hkv
        k = v["k"].view(B, Hkv, -1, self.index.D)[:, :, :n]
        vv = v["v"].view(B, Hkv, -1, self.index.D)[:, :, :n]
        return k, vv

    def _create(self, B: int, Hkv: int, D: int, dtype: str, need: int) -> None:
        cap = max(need, self._initial_capacity)
        cap = (cap + self.step - 1) // self.step * self.step
        self.index = SparseIndex(B, self.n_q_heads, Hkv, D, self.block_size, self.top_k, cap, dtype, self.bits,
                                 self.group_size, cluster_size=self.cluster_size)
        self.dtype = dtype

    def _grow(self, need: int) -> None:
        old = self.index
        n = old.offset
        cap = max(need, 2 * old.capacity)
        cap = (cap + self.step - 1) // self.step * self.step
        new = SparseIndex(old.B, old.Hq, old.Hkv, old.D, old.S, old.K, cap, old.dtype, old.bits,
                          self.group_size, cluster_size=self.cluster_size)
        ov, nv = old.views(), new.views()
        for name, t in ov.items():
            rows = n if name != "summaries" else (n + old.S - 1) // old.S
            nv[name][:, :rows].copy_(t[:, :rows])
        new.set_offset(n)
        self.index = new
        old.close()

    def _append(self, keys, values) -> None:
        import torch
        B, Hkv, L, D = keys.shape
        dtype = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[keys.dtype]
        if self.index is None:
            self._create(B, Hkv, D, dtype, L)
        elif self.offset + L > self.index.capacity:
            self._grow(self.offset + L)
        self.index.append(keys.contiguous(), values.contiguous())

    def _decode(self, queries, keys, values, scale: float, sinks=None):
        """One fused launch: append the token, score, select, attend."""
        import torch
        B, Hkv, L, D = keys.shape
        dtype = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[keys.dtype]
        if self.index is None:
            self._create(B, Hkv, D, dtype, 1)
        elif self.offset + 1 > self.index.capacity:
            self._grow(self.offset + 1)
        if sinks is not getattr(self.index, "_sinks_src", None):
            self.index.set_sinks(sinks)
            self.index._sinks_src = sinks
        q = queries[:, :, 0, :].contiguous()
        out = self.index.decode(q, keys[:, :, 0, :].contiguous(), values[:, :, 0, :].contiguous(), scale)
        return out[:, :, None, :]


def _dense_attention(queries, keys, values, scale: float, mask, sinks=None):
    """Dense SDPA over cached tokens (prefill only; not the retrieval path).
    `sinks` [Hq]: per-head logits joining the softmax denominator."""
    import torch
    import torch.nn.functional as F
    B, Hq, L, D = queries.shape
    G = Hq // keys.shape[1]
    k = keys.repeat_interleave(G, dim=1).to(queries.dtype)
    v = values.repeat_interleave(G, dim=1).to(queries.dtype)
    if isinstance(mask, str) and mask == "causal":
        T = k.shape[2]
        mask = torch.arange(T - L, T, device=queries.device)[:, None] >= torch.arange(T, device=queries.device)[None]
    elif mask is not None:
        mask = mask.to(queries.device)
    if sinks is None:
        return F.scaled_dot_product_attention(queries, k, v, attn_mask=mask, scale=scale)
    s = torch.einsum("bhld,bhtd->bhlt", queries.float(), k.float()) * scale
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf")) if mask.dtype == torch.bool else s + mask
    sink = sinks.float().view(1, Hq, 1, 1).expand(B, Hq, L, 1)
    p = torch.softmax(torch.cat([s, sink], dim=-1), dim=-1)[..., :-1]
    return torch.einsum("bhlt,bhtd->bhld", p, v.float()).to(queries.dtype)


def _dequantize(wq, scales, biases, bits: int):
    """Dense values of a quantized tuple [B, Hkv, T, .] with fma(scale, code, bias)."""
    import torch
    per = 32 // bits
    shifts = torch.arange(per, device=wq.device, dtype=torch.int32) * bits
    codes = (wq.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)
    codes = codes.reshape(*wq.shape[:-1], wq.shape[-1] * per).float()
    s = scales.float().repeat_interleave(64, dim=-1)
    b = biases.float().repeat_interleave(64, dim=-1)
    return torch.addcmul(b, s, codes).to(scales.dtype)


def attention_with_cache_update(queries, keys, values, cache, scale: float, mask=None, sinks=None):
    """Router (AttentionUtils.swift:37-77; with `sinks`, the sink variant of
    MiMoV2Flash.swift:14-56). queries [B, Hq, L, D]; keys/values
    [B, Hkv, L, D]; sinks [Hq] or None. Returns [B, Hq, L, D]."""
    if cache is None:
        return _dense_attention(queries, keys, values, scale, mask, sinks)
    if isinstance(cache, SparseKVCache):
        if queries.shape[2] == 1:
            out = cache._decode(queries, keys, values, scale, sinks)
            return out
        if cache.bits:
            (kq, ks, kb), (vq, vs, vb) = cache.update_quantized(keys, values)
            k = _dequantize(kq, ks, kb, cache.bits)
            v = _dequantize(vq, vs, vb, cache.bits)
        else:
            k, v = cache.update(keys, values)
        return _dense_attention(queries, k, v, scale, mask, sinks)
    raise TypeError(f"unsupported cache type {type(cache).__name__}")
