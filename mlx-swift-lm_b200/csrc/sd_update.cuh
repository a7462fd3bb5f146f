// sd_update.cuh -- cache writes: appending token rows (with affine
// quantization for 4/8-bit caches) and (re)building block summary keys.
//
// Storage follows the reference's KV layout [B, Hkv, cap, D]
// (Libraries/MLXLMCommon/KVCache.swift:328-371) and its quantized tuple
// (wq, scales, biases) with scales/biases in the key dtype
// (KVCache.swift:816-889). With sequence sharding, block j of the sequence is
// stored on shard j % P as local block j / P.
#pragma once

#include "sd_device.cuh"
#include "sd_format.h"
#include "sd_params.h"

namespace sd {

// Quantize one row of D elements (one warp) with the affine group-64 rule
// (scale from the group's range, the larger-magnitude edge placed exactly on a
// code, round-half-even codes clamped to [0, 2^bits-1], codes packed
// little-endian in uint32 words). The fp32 operations match the CPU
// restatement in oracle/sd_oracle.cpp (orc_quantize) one for one.
template <typename E, int BITS, int D>
__device__ __forceinline__ void quantize_row_regs(const float (&w)[D / 32], uint32_t* wq, E* sc, E* bi, int lane,
                                                  float (&deq)[D / 32]) {
  constexpr int EPL = D / 32;            // elements per lane (lane holds elements lane*EPL ..)
  constexpr int LPG = 64 / EPL;          // lanes per quantization group
  constexpr int PER_WORD = 32 / BITS;    // codes per uint32
  constexpr int LPW = PER_WORD / EPL;    // lanes sharing one word (>= 1)
  static_assert(EPL * BITS <= 32, "lane codes exceed one word");
  const float n_bins = float((1 << BITS) - 1);
  float wmax = w[0], wmin = w[0];
#pragma unroll
  for (int e = 1; e < EPL; ++e) { wmax = fmaxf(wmax, w[e]); wmin = fminf(wmin, w[e]); }
#pragma unroll
  for (int o = 1; o < LPG; o <<= 1) {
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
    wmin = fminf(wmin, __shfl_xor_sync(0xffffffffu, wmin, o));
  }
  float scale = fmaxf(__fdiv_rn(__fsub_rn(wmax, wmin), n_bins), 1e-7f);
  const bool mask = fabsf(wmin) > fabsf(wmax);
  if (!mask) scale = -scale;
  const float edge = mask ? wmin : wmax;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  if (q0 != 0.0f) scale = __fdiv_rn(edge, q0);
  const float bias = (q0 == 0.0f) ? 0.0f : edge;
  // what a reader of the cache sees: the stored (rounded) scale and bias
  const float s_st = Elt<E>::to_f32(Elt<E>::from_f32(scale)), b_st = Elt<E>::to_f32(Elt<E>::from_f32(bias));
  uint32_t bits = 0;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    float c = rintf(__fdiv_rn(__fsub_rn(w[e], bias), scale));
    c = fminf(fmaxf(c, 0.0f), n_bins);
    bits |= uint32_t(c) << (BITS * ((lane * EPL + e) % PER_WORD));
    deq[e] = __fmaf_rn(s_st, c, b_st);
  }
#pragma unroll
  for (int o = 1; o < LPW; o <<= 1) bits |= __shfl_xor_sync(0xffffffffu, bits, o);
  if (lane % LPW == 0) wq[(lane * EPL) / PER_WORD] = bits;
  if (lane % LPG == 0) {
    const int g = (lane * EPL) / 64;
    sc[g] = Elt<E>::from_f32(scale);
    bi[g] = Elt<E>::from_f32(bias);
  }
}

template <typename E, int BITS, int D>
__device__ __forceinline__ void quantize_row_warp(const E* src, uint32_t* wq, E* sc, E* bi, int lane) {
  constexpr int EPL = D / 32;
  float w[EPL], deq[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) w[e] = Elt<E>::to_f32(src[lane * EPL + e]);
  quantize_row_regs<E, BITS, D>(w, wq, sc, bi, lane, deq);
}


// Element d of key row `row` as fp32 (dequantized with fma(scale, code, bias)).
template <typename E, int BITS, int D>
__device__ __forceinline__ float load_key_elt(const void* data, const void* scales, const void* biases,
                                              size_t row, int d) {
  // L2-only loads (ld.global.cg): rows may have been written by another CTA
  // of the cluster earlier in the same launch.
  if constexpr (BITS == 0) {
    return Elt<E>::to_f32(__ldcg(static_cast<const E*>(data) + row * D + d));
  } else {
    constexpr int PER_WORD = 32 / BITS, WORDS = D / PER_WORD, NG = D / 64;
    const uint32_t w = __ldcg(static_cast<const uint32_t*>(data) + row * WORDS + d / PER_WORD);
    const float code = float((w >> (BITS * (d % PER_WORD))) & ((1u << BITS) - 1u));
    const float s = Elt<E>::to_f32(__ldcg(static_cast<const E*>(scales) + row * NG + d / 64));
    const float b = Elt<E>::to_f32(__ldcg(static_cast<const E*>(biases) + row * NG + d / 64));
    return __fmaf_rn(s, code, b);
  }
}

// Summary of one block: column mean over its n filled token rows starting at
// `row0`, sequential fp32 adds in token order, IEEE division, rounded to E.
// Threads [t0, t0 + nthr) of the caller cooperate over the D columns.
template <typename E, int BITS, int D>
__device__ __forceinline__ void block_summary(const void* data, const void* scales, const void* biases,
                                              size_t row0, int n, E* dst, int t, int nthr) {
  for (int d = t; d < D; d += nthr) {
    float acc = load_key_elt<E, BITS, D>(data, scales, biases, row0, d);
#pragma unroll 8
    for (int i = 1; i < n; ++i) acc = __fadd_rn(acc, load_key_elt<E, BITS, D>(data, scales, biases, row0 + i, d));
    dst[d] = Elt<E>::from_f32(__fdiv_rn(acc, float(n)));
  }
}

// Sum of column d over n >= 1 rows starting at `row0` in the canonical order
// (start from row 0, sequential fp32 adds). Loads are issued 64 rows at a
// time before the adds, so a block of up to 64 rows costs one memory round
// trip plus the add chain.
template <typename E, int BITS, int D>
__device__ __forceinline__ float column_sum(const void* data, const void* scales, const void* biases, size_t row0,
                                            int n, int d) {
  constexpr int BATCH = 64;
  float acc = 0.0f;
  for (int i0 = 0; i0 < n; i0 += BATCH) {
    float v[BATCH];
#pragma unroll
    for (int i = 0; i < BATCH; ++i)
      v[i] = (i0 + i < n) ? load_key_elt<E, BITS, D>(data, scales, biases, row0 + i0 + i, d) : 0.0f;
#pragma unroll
    for (int i = 0; i < BATCH; ++i)
      if (i0 + i < n) acc = (i0 + i == 0) ? v[i] : __fadd_rn(acc, v[i]);
  }
  return acc;
}

// Column sums of the lane's D/32 columns over n rows from `row0` (the
// canonical order of column_sum) into out -- the rare rebuild of a decode
// step's running sums, kept out of line.
template <typename E, int BITS, int D>
__device__ __noinline__ void rebuild_sums(const void* data, const void* scales, const void* biases, size_t row0,
                                          int n, int lane, float* out) {
  for (int e = 0; e < D / 32; ++e) out[e] = column_sum<E, BITS, D>(data, scales, biases, row0, n, lane * (D / 32) + e);
}

// Write one token row of K and V (warp 0: K, warp 1: V) at local row `row`.
template <typename E, int BITS, int D>
__device__ __forceinline__ void write_token_row(const E* src, void* data, void* scales, void* biases,
                                                size_t row, int lane) {
  if constexpr (BITS == 0) {
    E* dst = static_cast<E*>(data) + row * D;
    for (int d = lane; d < D; d += 32) dst[d] = src[d];
  } else {
    constexpr int WORDS = D * BITS / 32, NG = D / 64;
    quantize_row_warp<E, BITS, D>(src, static_cast<uint32_t*>(data) + row * WORDS,
                                  static_cast<E*>(scales) + row * NG, static_cast<E*>(biases) + row * NG, lane);
  }
}

// The decode step's own token, one warp: the K and V rows arrive in registers
// (loaded by append_load as early as possible), are stored (quantized for
// 4/8-bit caches), and the returned key values are the row as the cache
// holds it (dequantized codes for 4/8-bit) -- the input of the running sums.
template <typename E, int BITS, int D>
struct TokenRows {
  float k[D / 32], v[D / 32];
};
template <typename E, int BITS, int D>
__device__ __forceinline__ void append_load(TokenRows<E, BITS, D>& t, const E* k_src, const E* v_src, int lane) {
  constexpr int EPL = D / 32;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    t.k[e] = Elt<E>::to_f32(k_src[lane * EPL + e]);
    t.v[e] = Elt<E>::to_f32(v_src[lane * EPL + e]);
  }
}
template <typename E, int BITS, int D>
__device__ __forceinline__ void append_store(const TokenRows<E, BITS, D>& t, void* k_data, void* k_scales,
                                             void* k_biases, void* v_data, void* v_scales, void* v_biases,
                                             size_t row, int lane, float (&kdeq)[D / 32]) {
  constexpr int EPL = D / 32;
  if constexpr (BITS == 0) {
    E* kd = static_cast<E*>(k_data) + row * D + lane * EPL;
    E* vd = static_cast<E*>(v_data) + row * D + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      kd[e] = Elt<E>::from_f32(t.k[e]);
      vd[e] = Elt<E>::from_f32(t.v[e]);
      kdeq[e] = t.k[e];
    }
  } else {
    constexpr int WORDS = D * BITS / 32, NG = D / 64;
    float vdeq[EPL];
    quantize_row_regs<E, BITS, D>(t.k, static_cast<uint32_t*>(k_data) + row * WORDS,
                                  static_cast<E*>(k_scales) + row * NG, static_cast<E*>(k_biases) + row * NG, lane,
                                  kdeq);
    quantize_row_regs<E, BITS, D>(t.v, static_cast<uint32_t*>(v_data) + row * WORDS,
                                  static_cast<E*>(v_scales) + row * NG, static_cast<E*>(v_biases) + row * NG, lane,
                                  vdeq);
  }
}

// Append n_tok tokens [B, Hkv, n_tok, D] at global positions t0.. : one warp
// per (token, K or V). Tokens whose block lives on another shard are skipped.
template <typename E, int BITS, int D>
__global__ void __launch_bounds__(256) append_kernel(const __grid_constant__ AppendParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int i = blockIdx.x * 4 + (warp >> 1);
  const int bh = blockIdx.y;
  if (i >= p.n_tok) return;
  const int t = p.t0 + i;
  const int j = t / p.S;
  if (j % p.P != p.pr) return;
  const size_t row = size_t(bh) * p.cap_local + size_t(j / p.P) * p.S + (t % p.S);
  const size_t src = (size_t(bh) * p.n_tok + i) * D;
  if ((warp & 1) == 0)
    write_token_row<E, BITS, D>(static_cast<const E*>(p.k_src) + src, p.k_data, p.k_scales, p.k_biases, row, lane);
  else
    write_token_row<E, BITS, D>(static_cast<const E*>(p.v_src) + src, p.v_data, p.v_scales, p.v_biases, row, lane);
}

// Rebuild the summaries of local blocks jl0 + blockIdx.x for every (b, kv-head).
template <typename E, int BITS, int D>
__global__ void __launch_bounds__(128) summary_kernel(const __grid_constant__ SummaryParams p) {
  const int jl = p.jl0 + blockIdx.x;
  const int bh = blockIdx.y;
  const int j = jl * p.P + p.pr;
  const int n = min(p.S, p.T - j * p.S);
  if (n <= 0) return;
  const size_t row0 = size_t(bh) * p.cap_local + size_t(jl) * p.S;
  E* dst = static_cast<E*>(p.summ) + (size_t(bh) * p.nb_stride + jl) * D;
  block_summary<E, BITS, D>(p.k_data, p.k_scales, p.k_biases, row0, n, dst, threadIdx.x, blockDim.x);
}

}  // namespace sd
