"""Python host layer of the B200 retrieval block-sparse decode library.

Binds the C ABI of libsparse_decode.so (include/sparse_decode.h) with ctypes
and mirrors the reference's cache/attention API on top of it:

* `SparseIndex`          -- one layer's index (sd_index*): KV arenas, summaries,
                            decode launches, sharded decode steps.
* `SparseKVCache`        -- the `KVCache` protocol (Libraries/MLXLMCommon/
                            KVCache.swift:38-77) and, when kv_bits is set,
                            `QuantizedKVCacheProtocol` (KVCache.swift:94-119),
                            with the reference's 256-token capacity growth
                            (KVCache.swift:318, :333-362).
* `attention_with_cache_update` -- the router
                            (Libraries/MLXLMCommon/AttentionUtils.swift:37-77)
                            with the sparse branch for single-token decode.

torch is used for device memory and streams only. There is no CPU fallback:
the native library must be built (`__graft_entry__.build()`), and every
compute call goes through it.
"""
from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path
from typing import Optional

PKG_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_DIR / "libsparse_decode.so"

SD_OK = 0
STATUS = {0: "SD_OK", 1: "SD_ERR_INVALID_ARG", 2: "SD_ERR_SHAPE", 3: "SD_ERR_CAPACITY", 4: "SD_ERR_STATE",
          5: "SD_ERR_CUDA", 6: "SD_ERR_DEVICE"}
DTYPES = {"f32": 0, "f16": 1, "bf16": 2}

EXPORTED = ["sd_abi_version", "sd_status_string", "sd_last_error", "sd_index_create", "sd_index_destroy",
            "sd_index_config", "sd_index_arrays", "sd_index_offset", "sd_index_copy", "sd_append", "sd_trim",
            "sd_set_offset", "sd_rebuild_summaries", "sd_decode", "sd_shard_candidates", "sd_shard_attend",
            "sd_shard_merge", "sd_check_device", "sd_set_launch_overlap", "sd_decode_noalloc", "sd_comm_create",
            "sd_comm_handle", "sd_comm_open", "sd_comm_open_local", "sd_comm_set_wait_limit", "sd_comm_destroy",
            "sd_shard_decode", "sd_set_sinks"]
COMM_HANDLE_BYTES = 128


class SDError(RuntimeError):
    """A non-zero sd_status from the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class SDConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "batch", "n_q_heads", "n_kv_heads", "head_dim", "block_size", "top_k", "capacity", "dtype", "kv_bits",
        "group_size", "shard_rank", "shard_count", "cluster_size")] + [("reserved", ctypes.c_int32 * 3)]


class SDArrays(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "k_data", "v_data", "k_scales", "k_biases", "v_scales", "v_biases", "summaries")] + [
        ("cap_local", ctypes.c_int64), ("nb_local", ctypes.c_int64), ("row_bytes", ctypes.c_int32),
        ("cluster_size", ctypes.c_int32), ("smem_bytes", ctypes.c_int32), ("replicas", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 4)]


_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load libsparse_decode.so; raises when it has not been built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("SPARSE_DECODE_LIB", str(LIB_PATH)))
        if not path.exists():
            raise RuntimeError(f"{path} is missing: build it with __graft_entry__.build() "
                               "(the CUDA path has no fallback)")
        L = ctypes.CDLL(str(path))
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        pp = ctypes.POINTER(ctypes.c_void_p)
        sig = {
            "sd_abi_version": ([], i32),
            "sd_status_string": ([i32], ctypes.c_char_p),
            "sd_last_error": ([], ctypes.c_char_p),
            "sd_index_create": ([ctypes.POINTER(SDConfig), pp], i32),
            "sd_index_destroy": ([vp], i32),
            "sd_index_config": ([vp, ctypes.POINTER(SDConfig)], i32),
            "sd_index_arrays": ([vp, ctypes.POINTER(SDArrays)], i32),
            "sd_index_offset": ([vp, ctypes.POINTER(ctypes.c_int64)], i32),
            "sd_index_copy": ([vp, pp, vp], i32),
            "sd_append": ([vp, vp, vp, i32, vp], i32),
            "sd_trim": ([vp, i32, ctypes.POINTER(ctypes.c_int32)], i32),
            "sd_set_offset": ([vp, i64], i32),
            "sd_rebuild_summaries": ([vp, vp], i32),
            "sd_decode": ([vp, vp, vp, vp, f32, vp, vp, vp, vp], i32),
            "sd_shard_candidates": ([vp, vp, vp, vp, f32, vp, vp, vp, vp], i32),
            "sd_shard_attend": ([vp, vp, vp, vp, f32, vp, vp, vp, vp], i32),
            "sd_shard_merge": ([vp, vp, vp, vp, vp], i32),
            "sd_check_device": ([vp, ctypes.POINTER(ctypes.c_int32), vp], i32),
            "sd_set_launch_overlap": ([vp, i32], i32),
            "sd_decode_noalloc": ([ctypes.POINTER(SDConfig), ctypes.POINTER(SDArrays), i64, vp, f32, vp, vp, vp, vp],
                                  i32),
            "sd_comm_create": ([vp, pp], i32),
            "sd_comm_handle": ([vp, vp], i32),
            "sd_comm_open": ([vp, vp], i32),
            "sd_comm_open_local": ([vp, ctypes.POINTER(ctypes.c_void_p)], i32),
            "sd_comm_set_wait_limit": ([vp, i64], i32),
            "sd_comm_destroy": ([vp], i32),
            "sd_shard_decode": ([vp, vp, vp, vp, vp, f32, vp, vp, vp], i32),
            "sd_set_sinks": ([vp, vp], i32),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status != SD_OK:
        raise SDError(status, lib().sd_last_error().decode())


def _ptr(t) -> Optional[int]:
    """Device pointer of a torch tensor (None passes NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("sparse_decode arguments must be CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("sparse_decode arguments must be contiguous")
    return t.data_ptr()


def _stream(stream) -> Optional[int]:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _torch_dtype(name: str):
    import torch
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


class _DevArray:
    """__cuda_array_interface__ wrapper so torch can view library-owned memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class SparseIndex:
    """One layer's retrieval index on one GPU (one shard of a sharded sequence)."""

    def __init__(self, batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int, block_size: int, top_k: int,
                 capacity: int, dtype: str = "bf16", kv_bits: int = 0, group_size: int = 64, shard_rank: int = 0,
                 shard_count: int = 1, cluster_size: int = 0, _handle: Optional[int] = None):
        self.dtype = dtype
        self._sinks = None
        self.cfg = SDConfig(batch, n_q_heads, n_kv_heads, head_dim, block_size, top_k, capacity, DTYPES[dtype],
                            kv_bits, group_size if kv_bits else 0, shard_rank, shard_count, cluster_size)
        if _handle is None:
            h = ctypes.c_void_p()
            _check(lib().sd_index_create(ctypes.byref(self.cfg), ctypes.byref(h)))
            self._h = h
        else:
            self._h = ctypes.c_void_p(_handle)
        got = SDConfig()
        _check(lib().sd_index_config(self._h, ctypes.byref(got)))
        self.cluster_size = got.cluster_size
        arr = SDArrays()
        _check(lib().sd_index_arrays(self._h, ctypes.byref(arr)))
        self._arrays = arr
        self.replicas = arr.replicas

    # -- geometry -----------------------------------------------------------
    B = property(lambda s: s.cfg.batch)
    Hq = property(lambda s: s.cfg.n_q_heads)
    Hkv = property(lambda s: s.cfg.n_kv_heads)
    D = property(lambda s: s.cfg.head_dim)
    S = property(lambda s: s.cfg.block_size)
    K = property(lambda s: s.cfg.top_k)
    bits = property(lambda s: s.cfg.kv_bits)
    P = property(lambda s: s.cfg.shard_count)
    rank = property(lambda s: s.cfg.shard_rank)

    @property
    def capacity(self) -> int:
        return (self.cfg.capacity + 255) // 256 * 256

    @property
    def offset(self) -> int:
        v = ctypes.c_int64()
        _check(lib().sd_index_offset(self._h, ctypes.byref(v)))
        return v.value

    @property
    def cap_local(self) -> int:
        return self._arrays.cap_local

    @property
    def nb_local(self) -> int:
        return self._arrays.nb_local

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().sd_index_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- arrays (views over the library's arenas) ----------------------------
    def views(self) -> dict:
        """torch views of the device arrays: k/v [B*Hkv, cap_local, D] (dense, in
        the index dtype) or k/v codes [B*Hkv, cap_local, D*bits/32] int32 plus
        k/v scales and biases [B*Hkv, cap_local, D/64]; summaries
        [B*Hkv, nb_local, D]."""
        import torch
        a, BH, D = self._arrays, self.B * self.Hkv, self.D
        tdt = _torch_dtype(self.dtype)
        es = "<f4" if self.dtype == "f32" else "<i2"

        def t(ptr, shape, ts=es, dt=tdt):
            x = torch.as_tensor(_DevArray(ptr, shape, ts), device="cuda")
            return x.view(dt) if ts == "<i2" else x

        out = {"summaries": t(a.summaries, (BH, a.nb_local, D))}
        if self.bits:
            W = D * self.bits // 32
            out["k"] = t(a.k_data, (BH, a.cap_local, W), "<i4", None)
            out["v"] = t(a.v_data, (BH, a.cap_local, W), "<i4", None)
            for n in ("k_scales", "k_biases", "v_scales", "v_biases"):
                out[n] = t(getattr(a, n), (BH, a.cap_local, D // 64))
        else:
            out["k"] = t(a.k_data, (BH, a.cap_local, D))
            out["v"] = t(a.v_data, (BH, a.cap_local, D))
        return out

    # -- cache writes ----------------------------------------------------------
    def append(self, keys, values, stream=None) -> None:
        """keys/values [B, Hkv, n, D] in the index dtype."""
        n = keys.shape[2]
        _check(lib().sd_append(self._h, _ptr(keys), _ptr(values), n, _stream(stream)))

    def trim(self, n: int) -> int:
        t = ctypes.c_int32()
        _check(lib().sd_trim(self._h, n, ctypes.byref(t)))
        return t.value

    def set_offset(self, offset: int) -> None:
        _check(lib().sd_set_offset(self._h, offset))

    def rebuild_summaries(self, stream=None) -> None:
        _check(lib().sd_rebuild_summaries(self._h, _stream(stream)))

    def copy(self, stream=None) -> "SparseIndex":
        h = ctypes.c_void_p()
        _check(lib().sd_index_copy(self._h, ctypes.byref(h), _stream(stream)))
        c = self.cfg
        dup = SparseIndex(c.batch, c.n_q_heads, c.n_kv_heads, c.head_dim, c.block_size, c.top_k, c.capacity,
                          self.dtype, c.kv_bits, c.group_size or 64, c.shard_rank, c.shard_count, c.cluster_size,
                          _handle=h.value)
        if self._sinks is not None:
            dup.set_sinks(self._sinks)
        return dup

    # -- decode ----------------------------------------------------------------
    def decode(self, q, k_new=None, v_new=None, scale: Optional[float] = None, out=None, sel_out=None,
               scores_out=None, stream=None):
        """Single-token decode step (appends k_new/v_new first when given).
        q [B, Hq, D] -> out [B, Hq, D]."""
        import torch
        if scale is None:
            scale = 1.0 / math.sqrt(self.D)
        if out is None:
            out = torch.empty_like(q)
        _check(lib().sd_decode(self._h, _ptr(q), _ptr(k_new), _ptr(v_new), scale, _ptr(out), _ptr(sel_out),
                               _ptr(scores_out), _stream(stream)))
        return out

    def shard_candidates(self, q, cand_score, cand_block, k_new=None, v_new=None, scale=None, scores_out=None,
                         stream=None) -> None:
        scale = 1.0 / math.sqrt(self.D) if scale is None else scale
        _check(lib().sd_shard_candidates(self._h, _ptr(q), _ptr(k_new), _ptr(v_new), scale, _ptr(cand_score),
                                         _ptr(cand_block), _ptr(scores_out), _stream(stream)))

    def shard_attend(self, q, all_cand_score, all_cand_block, part_ml, part_o, scale=None, sel_out=None,
                     stream=None) -> None:
        scale = 1.0 / math.sqrt(self.D) if scale is None else scale
        _check(lib().sd_shard_attend(self._h, _ptr(q), _ptr(all_cand_score), _ptr(all_cand_block), scale,
                                     _ptr(part_ml), _ptr(part_o), _ptr(sel_out), _stream(stream)))

    def shard_merge(self, all_part_ml, all_part_o, out, stream=None) -> None:
        _check(lib().sd_shard_merge(self._h, _ptr(all_part_ml), _ptr(all_part_o), _ptr(out), _stream(stream)))

    def shard_decode(self, comm: "ShardComm", q, k_new=None, v_new=None, scale: Optional[float] = None, out=None,
                     sel_out=None, stream=None):
        """One fused sequence-sharded decode step over peer memory (see
        ShardComm); every shard calls it with the same arguments and gets the
        full output."""
        import torch
        scale = 1.0 / math.sqrt(self.D) if scale is None else scale
        out = torch.empty_like(q) if out is None else out
        _check(lib().sd_shard_decode(self._h, comm._h, _ptr(q), _ptr(k_new), _ptr(v_new), scale, _ptr(out),
                                     _ptr(sel_out), _stream(stream)))
        return out

    def set_sinks(self, sinks) -> None:
        """Attention-sink logits [n_q_heads] (fp32 CUDA tensor, kept alive by
        the index) joining every head's softmax denominator; None turns them
        off. See sd_set_sinks."""
        if sinks is not None:
            import torch
            sinks = sinks.detach().to(torch.float32).contiguous()
            if sinks.numel() != self.Hq or not sinks.is_cuda:
                raise ValueError(f"sinks must be a CUDA tensor of {self.Hq} values")
        self._sinks = sinks
        _check(lib().sd_set_sinks(self._h, _ptr(sinks)))

    def set_launch_overlap(self, enable: bool = True) -> None:
        """Let decode launches overlap the previous kernel on the stream
        (programmatic dependent launch); see sd_set_launch_overlap."""
        _check(lib().sd_set_launch_overlap(self._h, 1 if enable else 0))

    def check_device(self, stream=None) -> int:
        f = ctypes.c_int32()
        _check(lib().sd_check_device(self._h, ctypes.byref(f), _stream(stream)))
        return f.value


class ShardComm:
    """This shard's exchange area for the fused sharded step (sd_comm*).

    Created from an index (any index of the same configuration can use it);
    the shards' handles are exchanged with an all-gather over `group` (or by
    `exchange(my_handle_bytes) -> all handles in shard order`), then opened.
    Every shard must construct it at the same point of its program. `close()`
    waits at a barrier of the group before the area is freed, because the
    other shards map it."""

    def __init__(self, index: "SparseIndex", group=None, exchange=None, local: bool = False):
        h = ctypes.c_void_p()
        _check(lib().sd_comm_create(index._h, ctypes.byref(h)))
        self._h = h
        self.P = index.P
        self.group = group
        self.local = local
        if local:  # opened later with open_local (shards of this process)
            return
        buf = (ctypes.c_uint8 * COMM_HANDLE_BYTES)()
        _check(lib().sd_comm_handle(self._h, buf))
        mine = bytes(buf)
        if self.P == 1:
            handles = mine
        elif exchange is not None:
            handles = exchange(mine)
        else:
            handles = _all_gather_bytes(mine, group)
        if len(handles) != self.P * COMM_HANDLE_BYTES:
            raise ValueError(f"expected {self.P} handles of {COMM_HANDLE_BYTES} bytes")
        _check(lib().sd_comm_open(self._h, handles))

    @staticmethod
    def open_local(comms) -> None:
        """Open the comms of all shards driven by this process (shard order)."""
        arr = (ctypes.c_void_p * len(comms))(*[c._h.value for c in comms])
        for c in comms:
            _check(lib().sd_comm_open_local(c._h, arr))

    def set_wait_limit(self, seconds: float) -> None:
        _check(lib().sd_comm_set_wait_limit(self._h, int(seconds * 1e9)))

    def close(self, barrier: bool = True) -> None:
        if self._h is not None:
            if barrier and self.P > 1 and not self.local:
                import torch
                import torch.distributed as dist
                torch.cuda.synchronize()
                dist.barrier(group=self.group)
            lib().sd_comm_destroy(self._h)
            self._h = None


def _all_gather_bytes(data: bytes, group=None) -> bytes:
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    mine = torch.tensor(list(data), dtype=torch.uint8, device=dev)
    world = dist.get_world_size(group)
    allb = torch.empty(world * len(data), dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(allb, mine, group=group)
    return bytes(allb.cpu().tolist())


def sharded_decode(index, q, k_new=None, v_new=None, scale=None, group=None, sel_out=None, comm=None):
    """Sequence-sharded decode step over torch.distributed (NCCL over NVLink):
    local candidates -> all-gather -> global top-K + local attention ->
    all-gather of (m, l, o) partials -> log-sum-exp merge. Every rank calls it
    with the same q / k_new / v_new; returns out [B, Hq, D] on every rank.

    `index` is a SparseIndex (or anything with its shard_* methods and P, B,
    Hq, Hkv, D, K attributes). The gathers use flat views, the form that every
    torch.distributed backend accepts. With `comm` (a ShardComm) the whole
    step is one fused launch per shard that exchanges through peer memory
    instead (SparseIndex.shard_decode)."""
    import torch
    import torch.distributed as dist
    if comm is not None:
        return index.shard_decode(comm, q, k_new, v_new, scale, sel_out=sel_out)
    P, BH, K = index.P, index.B * index.Hkv, index.K
    BQ, D = index.B * index.Hq, index.D
    dev = q.device
    KK = max(K, 1)
    cs = torch.empty((BH, KK), device=dev, dtype=torch.float32)
    cb = torch.empty((BH, KK), device=dev, dtype=torch.int32)
    index.shard_candidates(q, cs, cb, k_new, v_new, scale)
    all_cs = torch.empty((P, BH, KK), device=dev, dtype=torch.float32)
    all_cb = torch.empty((P, BH, KK), device=dev, dtype=torch.int32)
    dist.all_gather_into_tensor(all_cs.view(-1), cs.view(-1), group=group)
    dist.all_gather_into_tensor(all_cb.view(-1), cb.view(-1), group=group)
    ml = torch.empty((BQ, 2), device=dev, dtype=torch.float32)
    po = torch.empty((BQ, D), device=dev, dtype=torch.float32)
    index.shard_attend(q, all_cs, all_cb, ml, po, scale, sel_out)
    all_ml = torch.empty((P, BQ, 2), device=dev, dtype=torch.float32)
    all_po = torch.empty((P, BQ, D), device=dev, dtype=torch.float32)
    dist.all_gather_into_tensor(all_ml.view(-1), ml.view(-1), group=group)
    dist.all_gather_into_tensor(all_po.view(-1), po.view(-1), group=group)
    out = torch.empty_like(q)
    index.shard_merge(all_ml, all_po, out)
    return out


from .cache import SparseKVCache, attention_with_cache_update  # noqa: E402,F401
from .persist import (load_prompt_cache, make_prompt_cache, maybe_quantize_kv_cache,  # noqa: E402,F401
                      save_prompt_cache)
