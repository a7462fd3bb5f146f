// sd_device.cuh -- device-side building blocks for the sm_100a sparse decode
// kernels: element conversion, PTX wrappers for mbarriers, TMA bulk copies and
// thread-block clusters, CTA-wide scans and a radix select over 64-bit keys.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sd {

// ---------------------------------------------------------------------------
// Element types. A format is (E, BITS): E is the dense element type, or the
// type of the per-group scales/biases when BITS is 4 or 8.
// ---------------------------------------------------------------------------
template <typename E> struct Elt;
template <> struct Elt<float> {
  static __device__ __forceinline__ float to_f32(float x) { return x; }
  static __device__ __forceinline__ float from_f32(float x) { return x; }
};
template <> struct Elt<__half> {
  static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f32(float x) { return __float2half_rn(x); }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
};

// Unpack one 32-bit word holding 32/sizeof(E)/8 elements of E into floats.
template <typename E> __device__ __forceinline__ void unpack_word(uint32_t w, float* f);
template <> __device__ __forceinline__ void unpack_word<float>(uint32_t w, float* f) {
  f[0] = __uint_as_float(w);
}
template <> __device__ __forceinline__ void unpack_word<__nv_bfloat16>(uint32_t w, float* f) {
  f[0] = __uint_as_float(w << 16);
  f[1] = __uint_as_float(w & 0xffff0000u);
}
template <> __device__ __forceinline__ void unpack_word<__half>(uint32_t w, float* f) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  float2 x = __half22float2(h);
  f[0] = x.x;
  f[1] = x.y;
}

// Byte-code -> float without an int->float conversion: 0x4B000000 | c is the
// float 2^23 + c, exact for c < 2^23; subtracting 2^23 leaves c exactly.
__device__ __forceinline__ float code_u8(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4Bu, 0x4550u + i)) - 8388608.0f;
}
__device__ __forceinline__ float code_u4(uint32_t w, int i) {
  return __uint_as_float(((w >> (4 * i)) & 0xFu) | 0x4B000000u) - 8388608.0f;
}

// Order-preserving 32-bit key of a score (larger = better). NaN ranks lowest,
// -0.0 is folded onto +0.0.
__device__ __forceinline__ uint32_t score_key(float s) {
  if (s != s) return 0u;
  if (s == 0.0f) s = 0.0f;
  uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_score(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
// Composite key: score first, then the lower block index wins. All distinct.
__device__ __forceinline__ uint64_t full_key(uint32_t k32, int32_t j) {
  return (uint64_t(k32) << 32) | uint64_t(0xffffffffu - uint32_t(j));
}

// ---------------------------------------------------------------------------
// Shared-memory and global access helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
// Streaming 16-byte global load that does not allocate in L1 (L2 policy `pol`).
__device__ __forceinline__ uint4 ldg_stream(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(pol));
  return v;
}

// Byte offset inside a TMA box written with the 128B/64B/32B swizzle modes:
// the 16-byte chunk index is XORed with address bits [7, 7+log2(cpb)).
// Box bases are 1024-byte aligned, so offsets inside the box are enough.
__device__ __forceinline__ uint32_t swz(uint32_t off, uint32_t cpb) {
  return off ^ (((off >> 7) & (cpb - 1u)) << 4);
}

// ---------------------------------------------------------------------------
// Time-bounded waiting. Every spin in these kernels gives up after this many
// nanoseconds of %globaltimer, records an error and lets the kernel finish.
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr int kErrTimeout = 1;
constexpr int kErrBadIndex = 2;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Phase stamps of the decode kernel, compiled only into the phase-timing
// build (-DSD_PHASE_TIMING): 24 u64 per CTA in DecodeParams::dbg. Thread 0
// writes [0] %globaltimer at entry and [7] at exit, and clock64 at [1] entry,
// [2] scoring start, [3] scoring end, [4] selection end, [5] attention end,
// [6] merge end; [14]/[15] inside the selection (the local list / the
// exchange). One thread of the producer warp writes [8] (first ring fill
// issued), consumer warp 0's lane 0 [9] (its first tile arrived) and [10]
// (its last tile done), thread 0 [11] (partials written), [12] (merge
// records stored) and [13] (merge records gathered); in the sliced
// selection thread 0 writes [16] (64-bit keys built), [17] (union
// histogram), [18] (union threshold), [19] (list check) and [20] (picks).
// The product build has no stamps.
#ifdef SD_PHASE_TIMING
__device__ __forceinline__ unsigned long long clock_u64() {
  unsigned long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}
#define SD_DBG_SLOT(p, k) (p).dbg[(size_t(blockIdx.y) * gridDim.x + blockIdx.x) * 24 + (k)]
#define SD_STAMP_T(p, k)                                             \
  do {                                                               \
    if (threadIdx.x == 0 && (p).dbg) SD_DBG_SLOT(p, k) = ::sd::globaltimer(); \
  } while (0)
#define SD_STAMP_C(p, k)                                             \
  do {                                                               \
    if (threadIdx.x == 0 && (p).dbg) SD_DBG_SLOT(p, k) = ::sd::clock_u64(); \
  } while (0)
// clock64 from the calling thread (the caller picks one thread)
#define SD_STAMP_HERE(p, k)                                          \
  do {                                                               \
    if ((p).dbg) SD_DBG_SLOT(p, k) = ::sd::clock_u64();              \
  } while (0)
#else
#define SD_STAMP_T(p, k) do { } while (0)
#define SD_STAMP_C(p, k) do { } while (0)
#define SD_STAMP_HERE(p, k) do { } while (0)
#endif

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase; false (and the error word set) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u && globaltimer() - t0 > kWaitLimitNs) {
      if (err) atomicOr(err, kErrTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// Messages between GPUs (peer memory over NVLink). Every 8-byte word carries
// 32 bits of payload and the launch's epoch: an aligned 8-byte store is
// single-copy atomic, so a reader that sees the current epoch in a word also
// sees that word's payload, with no fence and no separate flag (one NVLink
// trip per message). Waits are bounded like the mbarrier waits, with a
// longer, configurable limit because the shards' launches are only loosely
// aligned in time.
// ---------------------------------------------------------------------------
constexpr int kErrPeerTimeout = 4;

__device__ __forceinline__ void st_msg(unsigned long long* p, uint32_t payload, uint32_t epoch) {
  const unsigned long long v = (static_cast<unsigned long long>(epoch) << 32) | payload;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_msg_raw(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The same between the CTAs of one GPU (device scope).
__device__ __forceinline__ void st_msg_gpu(unsigned long long* p, uint32_t payload, uint32_t epoch) {
  const unsigned long long v = (static_cast<unsigned long long>(epoch) << 32) | payload;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// The payload of a message word once it carries `epoch`; on expiry of
// limit_ns the error word is set, *ok cleared, and 0 returned.
__device__ __forceinline__ uint32_t ld_msg(const unsigned long long* p, uint32_t epoch, uint64_t limit_ns, int* err,
                                           bool* ok) {
  unsigned long long v = ld_msg_raw(p);
  if (uint32_t(v >> 32) == epoch) return uint32_t(v);
  if (!*ok) return 0u;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    v = ld_msg_raw(p);
    if (uint32_t(v >> 32) == epoch) return uint32_t(v);
    if ((it & 15u) == 0u && globaltimer() - t0 > limit_ns) {
      if (err) atomicOr(err, kErrPeerTimeout);
      *ok = false;
      return 0u;
    }
  }
}

// Gather the payloads (as floats) of the message words w[i], i < n, for
// which want(i) holds, into dst[i], with a batch of loads in flight per thread
// before any is checked; words not yet carrying `epoch` are polled again
// (bounded). All threads of the CTA call; the caller synchronises after.
// kSys: the words are written by other GPUs (system scope) rather than by
// other CTAs of this GPU.
template <bool kSys, class Addr, class Want>
__device__ __noinline__ void gather_msgs(Addr addr, int n, uint32_t epoch, uint64_t limit_ns, int* err, float* dst,
                                            int tid, int nthreads, Want want) {
  constexpr int BATCH = 8;
#pragma unroll 1
  for (int base = tid; base < n; base += nthreads * BATCH) {
    bool need[BATCH];
#pragma unroll
    for (int j = 0; j < BATCH; ++j) need[j] = base + j * nthreads < n && want(base + j * nthreads);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
      unsigned long long v[BATCH];
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        v[j] = 0ull;
        if (need[j]) {
          if constexpr (kSys)
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v[j]) : "l"(addr(base + j * nthreads)) : "memory");
          else
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v[j]) : "l"(addr(base + j * nthreads)) : "memory");
        }
      }
      bool left = false;
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        if (!need[j]) continue;
        if (uint32_t(v[j] >> 32) == epoch) {
          dst[base + j * nthreads] = __uint_as_float(uint32_t(v[j]));
          need[j] = false;
        } else {
          left = true;
        }
      }
      if (!left) break;
      if (it == 0) t0 = globaltimer();
      else if ((it & 15u) == 0u && globaltimer() - t0 > limit_ns) {
        if (err) atomicOr(err, kSys ? kErrPeerTimeout : kErrTimeout);
#pragma unroll
        for (int j = 0; j < BATCH; ++j)
          if (need[j]) dst[base + j * nthreads] = 0.0f;
        break;
      }
    }
  }
}

// L2 policy of the data a launch streams once (block summaries, K/V tiles):
// evict_first, so that the streamed bytes -- tens of MB per layer -- are
// replaced before the lines every launch reuses (the kernel's code, message
// words, per-group state). `plain` gives the default policy instead.
__device__ __forceinline__ uint64_t stream_policy(bool plain) {
  uint64_t pol;
  if (plain)
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  else
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 16-byte asynchronous global -> shared copy (L2 only, L2 policy `pol`); the
// issuing thread waits for its own copies with cp_async_wait<N> (groups of
// cp_async_commit).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Bulk L2 prefetch of [p, p + bytes) (16-byte aligned, bytes % 16 == 0) by the
// TMA unit: one instruction for a long contiguous range.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(p), "r"(bytes), "l"(pol)
               : "memory");
}

// Generic-proxy writes -> async-proxy (TMA) reads ordering.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch: let the next kernel on the stream start its
// prologue, and wait for the previous kernel's results (no-ops when the
// launch carries no programmatic dependency).
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Fetch a tensor map (kernel parameter) into the descriptor cache early.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Tiled TMA loads of one box into this CTA's shared memory (no multicast),
// with L2 policy `pol`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            int32_t w, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core pieces (m16n8k16, fp32 accumulation)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
// c += A(16x16, row-major) * B(16x8, col-major); the A registers of rows
// 8..15 are passed as zero (at most 8 query heads per group).
template <typename E>
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* c, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* c, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
// c += A(16x16, row-major) * B(16x8, col-major), all four A registers (fp16).
__device__ __forceinline__ void mma16816_f16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Transpose of an 8x8 16-bit matrix held one row pair per lane (lane l:
// row l/4, elements 2(l%4), 2(l%4)+1) into the same layout.
__device__ __forceinline__ uint32_t movm_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// Two floats -> packed 16-bit pair (x in the low half), round to nearest even.
template <typename E> __device__ __forceinline__ uint32_t pack2(float x, float y);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float x, float y) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}
// (x, y) = hi + lo with hi, lo packed 16-bit pairs: ~16 significant bits.
template <typename E> __device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  hi = pack2<E>(x, y);
  float hx[2];
  unpack_word<E>(hi, hx);
  lo = pack2<E>(x - hx[0], y - hx[1]);
}
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Thread-block clusters
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Softmax normalisation of a merged (m, l, o) in the exp2 domain, with an
// optional attention sink: a per-head logit that joins the denominator and
// contributes no value (out = o / (l + 2^(sink*log2e - m))).
__device__ __forceinline__ float normalise_out(float O, float Ls, float M, const float* sinks, int head) {
  if (!(Ls > 0.0f)) return 0.0f;
  if (sinks) Ls += exp2f(__fmaf_rn(sinks[head], 1.4426950408889634f, -M));
  return O / Ls;
}

// Split cluster barrier: arrive early, wait right before the first access to
// a peer's shared memory (every CTA of the cluster has started by then).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// ---------------------------------------------------------------------------
// Warp / CTA reductions and scans
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sort 32 keys held one per lane into descending lane order (bitonic network
// over shuffles; no shared memory, no barriers).
__device__ __forceinline__ unsigned long long warp_sort_desc(unsigned long long x, int lane) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, x, j);
      const bool up = (lane & k) == 0, lower = (lane & j) == 0;
      x = (lower == up) ? (x > y ? x : y) : (x < y ? x : y);
    }
  }
  return x;
}

// Bitonic network over L = 32*RR keys held by one warp (register r of lane l
// holds element r*32 + l): sorts descending.
template <int RR>
__device__ __forceinline__ void warp_bitonic_sort_desc(unsigned long long (&v)[RR], int lane) {
  constexpr int L = 32 * RR;
#pragma unroll
  for (int k = 2; k <= L; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int jr = j >> 5;
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          if ((r & jr) == 0) {
            const int rp = r | jr;
            const bool desc = ((r * 32 + lane) & k) == 0;
            const unsigned long long x = v[r], y = v[rp];
            const unsigned long long hi = x > y ? x : y, lo = x > y ? y : x;
            v[r] = desc ? hi : lo;
            v[rp] = desc ? lo : hi;
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          const unsigned long long y = __shfl_xor_sync(0xffffffffu, v[r], j);
          const bool desc = ((r * 32 + lane) & k) == 0, lower = (lane & j) == 0;
          v[r] = (lower == desc) ? (v[r] > y ? v[r] : y) : (v[r] < y ? v[r] : y);
        }
      }
    }
  }
}

// The last stage of the network: sorts a bitonic sequence descending.
template <int RR>
__device__ __forceinline__ void warp_bitonic_merge_desc(unsigned long long (&v)[RR], int lane) {
  constexpr int L = 32 * RR;
#pragma unroll
  for (int j = L >> 1; j > 0; j >>= 1) {
    if (j >= 32) {
      const int jr = j >> 5;
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        if ((r & jr) == 0) {
          const int rp = r | jr;
          const unsigned long long x = v[r], y = v[rp];
          v[r] = x > y ? x : y;
          v[rp] = x > y ? y : x;
        }
      }
    } else {
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        const unsigned long long y = __shfl_xor_sync(0xffffffffu, v[r], j);
        v[r] = ((lane & j) == 0) ? (v[r] > y ? v[r] : y) : (v[r] < y ? v[r] : y);
      }
    }
  }
}

// Top L = 32*RR of n distinct keys keyf(i) (key 0 never occurs): runs of L
// keys are sorted by the warps, then merged pairwise -- max of run A and the
// reversed run B is bitonic and holds the top L of both, and one bitonic
// merge sorts it -- until runs[0 .. min(L, n)) holds the top keys,
// descending. All CTA threads call. runs: ceil(n / L) * L u64 of shared memory.
template <int RR, class KeyF>
__device__ __forceinline__ void block_topk(KeyF keyf, int n, unsigned long long* runs, int lane, int warp,
                                           int nwarps) {
  constexpr int L = 32 * RR;
  const int nrun = (n + L - 1) / L;
  for (int run = warp; run < nrun; run += nwarps) {
    unsigned long long v[RR];
#pragma unroll
    for (int r = 0; r < RR; ++r) {
      const int i = run * L + r * 32 + lane;
      v[r] = i < n ? keyf(i) : 0ull;
    }
    warp_bitonic_sort_desc<RR>(v, lane);
#pragma unroll
    for (int r = 0; r < RR; ++r) runs[run * L + r * 32 + lane] = v[r];
  }
  __syncthreads();
  for (int s = 1; s < nrun; s <<= 1) {
    for (int a = warp * 2 * s; a < nrun; a += nwarps * 2 * s) {
      const int b = a + s;
      if (b < nrun) {
        unsigned long long v[RR];
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          const int e = r * 32 + lane;
          const unsigned long long x = runs[a * L + e], y = runs[b * L + (L - 1 - e)];
          v[r] = x > y ? x : y;
        }
        warp_bitonic_merge_desc<RR>(v, lane);
#pragma unroll
        for (int r = 0; r < RR; ++r) runs[a * L + r * 32 + lane] = v[r];
      }
    }
    __syncthreads();
  }
}

// The top L keys of nrun runs that are each already sorted descending
// (runs[r*L .. r*L + L), 0-padded): the merge levels of block_topk alone.
template <int RR, class Sync>
__device__ __forceinline__ void block_merge_runs(unsigned long long* runs, int nrun, int lane, int warp, int nwarps,
                                                 Sync sync) {
  constexpr int L = 32 * RR;
  for (int s = 1; s < nrun; s <<= 1) {
    for (int a = warp * 2 * s; a < nrun; a += nwarps * 2 * s) {
      const int b = a + s;
      if (b < nrun) {
        unsigned long long v[RR];
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          const int e = r * 32 + lane;
          const unsigned long long x = runs[a * L + e], y = runs[b * L + (L - 1 - e)];
          v[r] = x > y ? x : y;
        }
        warp_bitonic_merge_desc<RR>(v, lane);
#pragma unroll
        for (int r = 0; r < RR; ++r) runs[a * L + r * 32 + lane] = v[r];
      }
    }
    sync();
  }
}

// Number of entries of a descending list of distinct keys that exceed x.
__device__ __forceinline__ int count_greater(const unsigned long long* a, int len, unsigned long long x) {
  int lo = 0, hi = len;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] > x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Exclusive scan of one int per thread over the whole CTA (all threads call).
// `scratch` holds at least 33 ints. Returns the exclusive prefix; *total gets the sum.
__device__ __forceinline__ int cta_exclusive_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) scratch[lane] = w;  // inclusive warp totals
    if (lane == 31) scratch[32] = w;
  }
  __syncthreads();
  const int before = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[32];
  const int r = before + x - v;
  __syncthreads();
  return r;
}

// State of a radix select, kept in shared memory.
struct RadixState {
  unsigned long long prefix;
  unsigned long long mask;
  int rem;
  int digit;
  int exact;
  int pad;
};

// Radix select over n distinct 64-bit keys produced by keyf(i): finds
// (prefix, mask) such that exactly k keys satisfy (key & mask) >= prefix,
// i.e. the k largest keys. Requires 0 < k < n. All CTA threads call it.
// hist: 256 u32 of shared memory.
template <class KeyF>
__device__ __noinline__ void radix_select(KeyF keyf, int n, int k, uint32_t* hist, RadixState* st) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  unsigned long long prefix = 0ull, mask = 0ull;
  int rem = k;
  for (int pb = 7; pb >= 0; --pb) {
#pragma unroll 1
    for (int i = tid; i < 256; i += nthr) hist[i] = 0u;
    __syncthreads();
    const int shift = 8 * pb;
#pragma unroll 1
    for (int base = warp * 32; base < n; base += nthr) {
      const int i = base + lane;
      bool active = false;
      uint32_t digit = 0;
      if (i < n) {
        const unsigned long long key = keyf(i);
        active = (key & mask) == prefix;
        digit = uint32_t(key >> shift) & 255u;
      }
      const unsigned amask = __ballot_sync(0xffffffffu, active);
      if (active) {
        const unsigned peers = __match_any_sync(amask, digit);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[digit], uint32_t(__popc(peers)));
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l covers digits 255-8l .. 248-8l (descending)
      uint32_t c[8];
      uint32_t s = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) { c[e] = hist[255 - 8 * lane - e]; s += c[e]; }
      uint32_t incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const uint32_t excl = incl - s;
      if (excl < uint32_t(rem) && uint32_t(rem) <= incl) {
        uint32_t above = excl;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (above + c[e] >= uint32_t(rem)) {
            st->digit = 255 - 8 * lane - e;
            st->rem = rem - int(above);
            st->exact = (c[e] == uint32_t(rem) - above) ? 1 : 0;
            break;
          }
          above += c[e];
        }
      }
    }
    __syncthreads();
    prefix |= (unsigned long long)(st->digit) << shift;
    mask |= 0xffull << shift;
    rem = st->rem;
    const bool done = st->exact != 0;
    __syncthreads();
    if (done) break;
  }
  if (tid == 0) { st->prefix = prefix; st->mask = mask; }
  __syncthreads();
}

// Buckets of the top-K threshold search over a CTA's own large chunk: the
// top 10 bits of a 64-bit key (sign, exponent and 1 mantissa bit of the score).
constexpr int kBuckets = 1024;
__device__ __forceinline__ uint32_t key_bucket(unsigned long long x) { return uint32_t(x >> 54); }

// The k-th largest of n distinct 64-bit keys keyf(i) (0 < k < n), i.e. the
// threshold tau with exactly k keys >= tau. A histogram of the keys' buckets
// (`h`, kBuckets u32 of shared memory; filled here unless the caller built it
// already) finds the bucket that holds the k-th key; the keys of that bucket
// (usually a few dozen) are compacted into bidx (room for cap / 2 keys) and
// ranked against each other by counting. When the bucket holds more than
// min(cap / 2, 256) keys
// (equal scores, say) a radix select over all n keys decides instead. All CTA
// threads call; scratch: cta_exclusive_scan's 33 ints plus [120, 124).
template <class KeyF>
__device__ __noinline__ unsigned long long topk_threshold(KeyF keyf, int n, int k, uint32_t* h, bool have_hist, int* bidx,
                                             int cap, int* scratch, uint32_t* hist256, RadixState* rs) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  unsigned long long* tau = reinterpret_cast<unsigned long long*>(scratch + 122);
  if (!have_hist) {
#pragma unroll 1
    for (int i = tid; i < kBuckets; i += nthr) h[i] = 0u;
    __syncthreads();
#pragma unroll 1
    for (int i = tid; i < n; i += nthr) atomicAdd(&h[key_bucket(keyf(i))], 1u);
  }
  __syncthreads();
  // each thread sums a run of buckets from the top; the run holding the k-th
  // key finds its bucket b and the count above it
  const int per = (kBuckets + nthr - 1) / nthr;
  const int top = kBuckets - 1 - tid * per;
  int cnt = 0;
#pragma unroll 1
  for (int j = 0; j < per; ++j)
    if (top - j >= 0) cnt += int(h[top - j]);
  int total;
  const int before = cta_exclusive_scan(cnt, scratch, &total);
  if (before < k && before + cnt >= k) {
    int acc = before;
#pragma unroll 1
    for (int j = 0; j < per && top - j >= 0; ++j) {
      const int c = int(h[top - j]);
      if (acc + c >= k) {
        scratch[120] = top - j;
        scratch[121] = acc;
        break;
      }
      acc += c;
    }
  }
  if (tid == 0) *tau = ~0ull;
  __syncthreads();
  const uint32_t b = uint32_t(scratch[120]);
  const int r = k - scratch[121];  // keys still needed from bucket b (>= 1)
  const int nb = int(h[b]);
  if (nb <= min(cap / 2, 256)) {
    // the bucket's keys, compacted as keys (bidx holds 2 ints per key)
    unsigned long long* bk = reinterpret_cast<unsigned long long*>(bidx);
    cta_compact(n, [&](int i) { return key_bucket(keyf(i)) == b; }, [&](int pos, int i) { bk[pos] = keyf(i); },
                scratch);
#pragma unroll 1
    for (int a = tid; a < nb; a += nthr) {
      const unsigned long long x = bk[a];
      int rank = 0;
#pragma unroll 8
      for (int c = 0; c < nb; ++c) rank += bk[c] > x ? 1 : 0;  // every thread reads the same word: broadcast
      if (rank == r - 1) *tau = x;
    }
  } else {
    radix_select(keyf, n, k, hist256, rs);
    const unsigned long long pre = rs->prefix, msk = rs->mask;
    unsigned long long m = ~0ull;
#pragma unroll 1
    for (int i = tid; i < n; i += nthr) {
      const unsigned long long x = keyf(i);
      if ((x & msk) >= pre && x < m) m = x;
    }
    atomicMin(tau, m);
  }
  __syncthreads();
  const unsigned long long t = *tau;
  __syncthreads();
  return t;
}

// ---------------------------------------------------------------------------
// Top-K building blocks over 64-bit keys in shared memory (the sliced
// selection): keys are distinct, 0 marks padding. All CTA threads call each
// function; scratch: cta_exclusive_scan's 33 ints, [118, 124).
// ---------------------------------------------------------------------------

// A slot in a buffer with counter *ctr for every lane whose `want` holds, one
// shared atomic per warp (atomics aimed at one address serialise across a
// warp); all lanes of the warp call it.
__device__ __forceinline__ int warp_slot(bool want, int* ctr) {
  const unsigned m = __ballot_sync(0xffffffffu, want);
  const int lane = threadIdx.x & 31;
  int base = 0;
  if (m && lane == __ffs(m) - 1) base = atomicAdd(ctr, __popc(m));
  base = __shfl_sync(0xffffffffu, base, __ffs(m ? m : 1u) - 1);
  return base + __popc(m & ((1u << lane) - 1u));
}
// Buckets of the keys' histogram, by the distance d = hi - key of the 32-bit
// score key from the largest one (hi, kept in scratch[113] by hist_keys): d's
// binary exponent and 5 mantissa bits, i.e. buckets 1/32 of d wide -- fine
// near the top, where the K-th key lies, whatever the scores' magnitude and
// however far outliers sit above the rest. Monotonic: bucket order is key
// order (bucket kBuckets - 1 holds the largest key).
__device__ __forceinline__ uint32_t range_bucket(unsigned long long x, uint32_t hi) {
  static_assert(kBuckets == 32 * 32, "32 binary exponents x 5 mantissa bits");
  const uint32_t d = hi - uint32_t(x >> 32);
  const uint32_t f = __float_as_uint(__uint2float_rz(d));  // d >= 1: exponent 127..158
  const uint32_t idx = d == 0u ? 0u : 1u + ((f >> 23) - 127u) * 32u + ((f >> 18) & 31u);
  return uint32_t(kBuckets - 1) - min(idx, uint32_t(kBuckets - 1));
}
// Bucket histogram of the non-zero keys x[0, n) by their distance from the
// largest; returns their number.
static __device__ __noinline__ int hist_keys(const unsigned long long* x, int n, uint32_t* h, int* scratch) {
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int i = threadIdx.x; i < kBuckets; i += blockDim.x) h[i] = 0u;
  if (threadIdx.x == 0) {
    scratch[118] = 0;
    scratch[113] = 0;
  }
  uint32_t hi = 0u;
  int c = 0;
#pragma unroll 4
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long v = x[i];
    if (v != 0ull) {
      hi = max(hi, uint32_t(v >> 32));
      ++c;
    }
  }
  hi = __reduce_max_sync(0xffffffffu, hi);
  c = __reduce_add_sync(0xffffffffu, c);
  __syncthreads();  // the counters above are initialised
  if (lane == 0) {
    atomicMax(reinterpret_cast<unsigned*>(&scratch[113]), hi);
    if (c) atomicAdd(&scratch[118], c);
  }
  __syncthreads();
  hi = uint32_t(scratch[113]);
#pragma unroll 4
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long v = x[i];
    if (v != 0ull) atomicAdd(&h[range_bucket(v, hi)], 1u);
  }
  __syncthreads();
  const int total = scratch[118];
  __syncthreads();
  return total;
}

// The k-th largest non-zero key of x[0, n) (1 <= k <= number of non-zero
// keys), h being the bucket histogram of x made by hist_keys (whose largest
// score key is still in scratch): the bucket holding it is found from h; that
// bucket's keys (usually a few) are gathered into bk (256 entries) and ranked
// by counting. A bucket of more than 256 keys (equal scores) is resolved by a
// radix select over x instead.
static __device__ __noinline__ unsigned long long kth_key(const unsigned long long* x, int n, int k, const uint32_t* h,
                                                   unsigned long long* bk, int* scratch, uint32_t* hist256,
                                                   RadixState* rs) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  unsigned long long* tau = reinterpret_cast<unsigned long long*>(scratch + 122);
  const int per = (kBuckets + nthr - 1) / nthr;
  const int top = kBuckets - 1 - tid * per;
  int cnt = 0;
#pragma unroll 1
  for (int j = 0; j < per; ++j)
    if (top - j >= 0) cnt += int(h[top - j]);
  int total;
  const int before = cta_exclusive_scan(cnt, scratch, &total);
  if (before < k && before + cnt >= k) {
    int acc = before;
#pragma unroll 1
    for (int j = 0; j < per && top - j >= 0; ++j) {
      const int c = int(h[top - j]);
      if (acc + c >= k) {
        scratch[120] = top - j;
        scratch[121] = acc;
        break;
      }
      acc += c;
    }
  }
  if (tid == 0) {
    *tau = ~0ull;
    scratch[119] = 0;
  }
  __syncthreads();
  const uint32_t b = uint32_t(scratch[120]);
  const int r = k - scratch[121];  // keys still needed from bucket b (>= 1)
  const int nb = int(h[b]);
  if (nb <= 256) {
    const uint32_t hi = uint32_t(scratch[113]);
#pragma unroll 4
    for (int b0 = tid & ~31; b0 < n; b0 += nthr) {
      const int i = b0 + (tid & 31);
      const unsigned long long v = i < n ? x[i] : 0ull;
      const bool in = v != 0ull && range_bucket(v, hi) == b;
      const int slot = warp_slot(in, &scratch[119]);
      if (in) bk[slot] = v;
    }
    __syncthreads();
#pragma unroll 1
    for (int a = tid; a < nb; a += nthr) {
      const unsigned long long v = bk[a];
      int rank = 0;
#pragma unroll 8
      for (int c = 0; c < nb; ++c) rank += bk[c] > v ? 1 : 0;  // the same word for every thread: broadcast
      if (rank == r - 1) *tau = v;
    }
  } else {
    radix_select([x](int i) { return x[i]; }, n, k, hist256, rs);
    const unsigned long long pre = rs->prefix, msk = rs->mask;
    unsigned long long m = ~0ull;
#pragma unroll 1
    for (int i = tid; i < n; i += nthr) {
      const unsigned long long v = x[i];
      if (v && (v & msk) >= pre && v < m) m = v;
    }
    atomicMin(tau, m);
  }
  __syncthreads();
  const unsigned long long t = *tau;
  __syncthreads();
  return t;
}

// The m largest keys of the distinct non-zero keys x[0, n) into out, in no
// particular order; returns min(n, m). h: the bucket histogram of x when
// have_hist (it is built here otherwise).
static __device__ __noinline__ int top_keys(const unsigned long long* x, int n, int m, uint32_t* h, bool have_hist,
                                     unsigned long long* out, unsigned long long* bk, int* scratch,
                                     uint32_t* hist256, RadixState* rs) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  if (n <= m) {
#pragma unroll 1
    for (int i = tid; i < n; i += nthr) out[i] = x[i];
    __syncthreads();
    return n;
  }
  if (m <= 0) return 0;
  if (!have_hist) hist_keys(x, n, h, scratch);
  const unsigned long long t = kth_key(x, n, m, h, bk, scratch, hist256, rs);
  if (tid == 0) scratch[119] = 0;
  __syncthreads();
#pragma unroll 4
  for (int b0 = tid & ~31; b0 < n; b0 += nthr) {
    const int i = b0 + (tid & 31);
    const unsigned long long v = i < n ? x[i] : 0ull;
    const bool in = i < n && v >= t;
    const int slot = warp_slot(in, &scratch[119]);
    if (in) out[slot] = v;
  }
  __syncthreads();
  return m;
}

}  // namespace sd
