"""Prompt-cache persistence and cache construction around SparseKVCache.

* `save_prompt_cache` / `load_prompt_cache` write and read the reference's
  prompt-cache file (savePromptCache / loadPromptCache,
  Libraries/MLXLMCommon/KVCache.swift:1244-1388): one `.safetensors` file whose
  tensors are the caches' `state` arrays under "i.j" (cache i, array j) and
  whose string metadata holds the caches' `metaState` under "0.i.j", the
  caller's metadata under "1.key" and the cache class names under "2.i".
  SparseKVCache entries are stored under the class name "SparseKVCache" with
  the metaState of `SparseKVCache.meta_state`. Entries written by the
  reference for its dense ("KVCache") and quantized ("QuantizedKVCache")
  caches are loaded as SparseKVCache when `sparse` parameters are given: the
  rows are copied into an index and the block summary keys are built from
  them (the prefill-side step of the sparse path).
* `make_prompt_cache` mirrors `LanguageModel.newCache` (LanguageModel.swift:
  215-229) for models whose attention layers use the sparse path, with the
  reference's GenerateParameters knobs (kvBits, kvGroupSize,
  Evaluate.swift:67-73) plus block size and top-K.
* `maybe_quantize_kv_cache` mirrors maybeQuantizeKVCache (KVCache.swift:
  1637-1660): dense caches become quantized ones once their offset passes
  `quantized_kv_start`.

The safetensors container (8-byte little-endian header length, a JSON header
of {name: {dtype, shape, data_offsets}} plus "__metadata__", then the raw
little-endian tensor bytes) is written and read here directly.
"""
from __future__ import annotations

import json
import struct
from typing import Dict, List, Optional, Sequence, Tuple

_DTYPES = {"BF16": 2, "F16": 2, "F32": 4, "U32": 4, "I32": 4, "U8": 1}


def _torch_to_st(t):
    import torch
    return {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.int32: "I32",
            torch.uint8: "U8"}.get(t.dtype) or ("U32" if t.dtype == torch.uint32 else None)


def _tensor_bytes(t) -> Tuple[str, bytes]:
    import torch
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return "BF16", t.view(torch.int16).numpy().tobytes()
    if t.dtype == torch.uint32:
        return "U32", t.view(torch.int32).numpy().tobytes()
    name = _torch_to_st(t)
    if name is None:
        raise TypeError(f"unsupported tensor dtype {t.dtype}")
    return name, t.numpy().tobytes()


def _tensor_from(dtype: str, shape: Sequence[int], raw: bytes, device):
    import numpy as np
    import torch
    np_dt = {"BF16": np.int16, "F16": np.float16, "F32": np.float32, "U32": np.int32, "I32": np.int32,
             "U8": np.uint8}[dtype]
    a = np.frombuffer(raw, dtype=np_dt).reshape(shape).copy()
    t = torch.from_numpy(a)
    if dtype == "BF16":
        t = t.view(torch.bfloat16)
    elif dtype == "U32":
        t = t.view(torch.uint32) if hasattr(torch, "uint32") else t
    return t.to(device) if device is not None else t


def write_safetensors(path: str, tensors: Dict[str, object], metadata: Dict[str, str]) -> None:
    """Write `tensors` (torch tensors, any device) and string `metadata`."""
    header: Dict[str, object] = {"__metadata__": dict(metadata)}
    blobs: List[bytes] = []
    off = 0
    for name in sorted(tensors):
        dt, raw = _tensor_bytes(tensors[name])
        header[name] = {"dtype": dt, "shape": list(tensors[name].shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)  # 8-byte aligned data start
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_safetensors(path: str, device=None) -> Tuple[Dict[str, object], Dict[str, str]]:
    """Read a safetensors file: ({name: tensor}, metadata)."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 8:
        raise ValueError(f"{path}: not a safetensors file")
    (n,) = struct.unpack("<Q", data[:8])
    if 8 + n > len(data):
        raise ValueError(f"{path}: header length {n} exceeds the file")
    header = json.loads(data[8:8 + n].decode())
    meta = header.pop("__metadata__", {}) or {}
    base = 8 + n
    out = {}
    for name, info in header.items():
        b, e = info["data_offsets"]
        dt, shape = info["dtype"], info["shape"]
        size = _DTYPES[dt]
        for s in shape:
            size *= s
        if e - b != size or base + e > len(data):
            raise ValueError(f"{path}: tensor {name} has inconsistent offsets")
        out[name] = _tensor_from(dt, shape, data[base + b:base + e], device)
    return out, meta


def save_prompt_cache(path: str, caches: Sequence[object], metadata: Optional[Dict[str, str]] = None) -> None:
    """savePromptCache (KVCache.swift:1244-1297) for SparseKVCache lists."""
    from .cache import SparseKVCache
    tensors: Dict[str, object] = {}
    meta: Dict[str, str] = {}
    for i, c in enumerate(caches):
        if not isinstance(c, SparseKVCache):
            raise TypeError(f"cache {i} is a {type(c).__name__}; only SparseKVCache is stored here")
        for j, a in enumerate(c.state):
            tensors[f"{i}.{j}"] = a
        for j, v in enumerate(c.meta_state):
            meta[f"0.{i}.{j}"] = v
        meta[f"2.{i}"] = "SparseKVCache"
    for k, v in (metadata or {}).items():
        meta[f"1.{k}"] = str(v)
    write_safetensors(path, tensors, meta)


def load_prompt_cache(path: str, device="cuda", sparse: Optional[dict] = None):
    """loadPromptCache (KVCache.swift:1305-1388). Returns (caches, metadata).

    `sparse` (n_q_heads, block_size, top_k, optionally cluster_size) turns
    the reference's "KVCache" / "KVCacheSimple" and "QuantizedKVCache"
    entries into SparseKVCache; without it they are rejected."""
    from .cache import SparseKVCache
    arrays, meta = read_safetensors(path, device)
    n = 0
    while f"2.{n}" in meta:
        n += 1
    state: List[List[object]] = [[] for _ in range(n)]
    for name, t in arrays.items():
        i, j = (int(x) for x in name.split(".")[:2])
        if i >= n:
            raise ValueError("Mismatch in cache counts")
        while len(state[i]) <= j:
            state[i].append(None)
        state[i][j] = t
    info: List[List[str]] = []
    for i in range(n):
        row, j = [], 0
        while f"0.{i}.{j}" in meta:
            row.append(meta[f"0.{i}.{j}"])
            j += 1
        info.append(row)
    user = {k[2:]: v for k, v in meta.items() if k.startswith("1.")}
    caches = []
    for i in range(n):
        cls = meta[f"2.{i}"]
        if cls == "SparseKVCache":
            if len(info[i]) != 7:
                raise ValueError("SparseKVCache metaState must have exactly 7 values")
            _, _, group, bits, block, top_k, hq = (int(x) for x in info[i])
            c = SparseKVCache(hq, block, top_k, bits or None, group or 64)
        elif cls in ("KVCache", "KVCacheSimple", "QuantizedKVCache"):
            if sparse is None:
                raise ValueError(f"cache {i} is a {cls}; pass `sparse` parameters to load it as a SparseKVCache")
            bits = 0
            group = 64
            if cls == "QuantizedKVCache":
                # QuantizedKVCache.metaState: [step, offset, groupSize, bits] (KVCache.swift:900-944)
                group, bits = int(info[i][2]), int(info[i][3])
            c = SparseKVCache(sparse["n_q_heads"], sparse.get("block_size", 64), sparse.get("top_k", 64),
                              bits or None, group, cluster_size=sparse.get("cluster_size", 0))
        else:
            raise ValueError(f"Unknown cache class: {cls}")
        if any(a is None for a in state[i]):
            raise ValueError(f"cache {i}: missing state arrays")
        if state[i]:
            c.state = state[i]
            if cls == "SparseKVCache":
                c.meta_state = info[i]
        caches.append(c)
    return caches, user


def make_prompt_cache(n_layers: int, n_q_heads: int, kv_bits: Optional[int] = None, kv_group_size: int = 64,
                      block_size: int = 64, top_k: int = 64, capacity: int = 0) -> list:
    """LanguageModel.newCache (LanguageModel.swift:215-229) for a model whose
    attention layers take the sparse path: one SparseKVCache per layer,
    quantized when kv_bits is set (GenerateParameters.kvBits / kvGroupSize)."""
    from .cache import SparseKVCache
    return [SparseKVCache(n_q_heads, block_size, top_k, kv_bits, kv_group_size, capacity=capacity)
            for _ in range(n_layers)]


def maybe_quantize_kv_cache(caches: list, kv_bits: Optional[int], kv_group_size: int = 64,
                            quantized_kv_start: int = 0) -> None:
    """maybeQuantizeKVCache (KVCache.swift:1637-1660): once a dense cache's
    offset passes quantized_kv_start, replace it in place by a quantized one
    holding the same tokens (quantized and summarised on the GPU)."""
    from .cache import SparseKVCache
    if kv_bits is None:
        return
    for i, c in enumerate(caches):
        if not isinstance(c, SparseKVCache) or c.bits or c.offset <= quantized_kv_start:
            continue
        k, v = c.state
        q = SparseKVCache(c.n_q_heads, c.block_size, c.top_k, kv_bits, kv_group_size,
                          capacity=c.index.capacity if c.index is not None else 0, cluster_size=c.cluster_size)
        q._append(k.contiguous(), v.contiguous())
        caches[i] = q
