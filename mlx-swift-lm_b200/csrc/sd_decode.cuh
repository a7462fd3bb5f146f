// sd_decode.cuh -- the retrieval block-sparse decode kernel for sm_100a.
//
// Q CTAs serve one (batch, kv-head) group: C CTAs of a thread-block cluster
// times R replica clusters (Q = C * R, all resident at once).
//   phase 0  queries of the group -> shared memory; the group's summary rows
//            are bulk-prefetched to L2 (evict_first) and the first cp.async
//            batches of them are staged before the query barrier; the producer
//            warp loads the new
//            token (the cache.update half of attentionWithCacheUpdate,
//            Libraries/MLXLMCommon/AttentionUtils.swift:54-66 / :67-76).
//   phase 1  score: 8 warps score this CTA's candidate rows, score[j] =
//            scale * (sum_g q_g) . summary[j], one 16-byte load of a summary
//            row per lane and a fixed fp32 reduction order (the CPU oracle
//            restates it); meanwhile the producer warp appends the token
//            (quantizing 4/8-bit rows) and keeps the recent block's running
//            column sums.
//   phase 2  select (top-K by score, lower block index wins; then the recent
//            block), one of two ways:
//            whole  -- at most 2048 candidates and K <= 128 with clusters of
//                      several CTAs (or one CTA per group): the cluster's CTAs
//                      score chunks and push the keys into every peer's copy
//                      (DSMEM); every CTA runs the same block-wide bitonic
//                      top-K (replica clusters repeat this);
//            sliced -- otherwise: CTA q of Q scores chunk q, keeps its best MT
//                      keys (bitonic top-K for MT <= 128 of at most 2048,
//                      else a bucket-histogram threshold), the lists meet in L2
//                      as epoch-tagged message words, every CTA finds the
//                      union's K-th key the same way and takes the union's keys
//                      above it in gathered order; a CTA whose MT keys were all
//                      taken makes every CTA repeat with full top-K lists.
//   phase 3  attend: the selected blocks are cut into stages of LT tokens
//            (64 for 4/8-bit codes with 16-bit scales, else 32) spread evenly
//            over the group's Q CTAs; a producer warp stages them with TMA
//            (one 4-D copy for K and V where V lies a fixed stride after K,
//            one copy for the scale/bias pieces; no multicast) into a ring of
//            mbarrier-guarded stages; 8 consumer warps run online softmax in
//            the exp2 domain on tensor cores (mma.sync m16n8k16) for 16-bit
//            K/V and for 4/8-bit codes with 16-bit scales (exact codes as fp16
//            operands; 8-bit codes with the tokens as the tile's rows), on FMA
//            pipes otherwise.
//   phase 4  merge: warp partials -> CTA partial -> a few owner CTAs each
//            gather every CTA's record of their output slice (L2 message words
//            tagged with the group's epoch) and merge them by log-sum-exp; the
//            other CTAs exit once their records are out.
// Sharded decode: MODE_PEER exchanges the CTAs' lists (sliced groups; the
// shards' top-K candidates otherwise) and the partial records through peer
// memory in the same launch; MODE_CANDIDATES /
// MODE_ATTEND run phases 0-2 and 2-4 around the caller's all-gathers.
// Stage-4 semantics follow quantizedScaledDotProductAttention
// (Libraries/MLXLMCommon/KVCache.swift:1544-1618) restricted to the gathered
// tokens.
#pragma once

#include "sd_device.cuh"
#include "sd_format.h"
#include "sd_params.h"
#include "sd_update.cuh"

namespace sd {

// Ordered stream compaction over [0, n): emit(pos, i) for every i with pred(i),
// pos ascending with i. All CTA threads call. Returns the number emitted.
template <class Pred, class Emit>
__device__ __noinline__ int cta_compact(int n, Pred pred, Emit emit, int* scratch) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int i0 = min(n, int(threadIdx.x) * per), i1 = min(n, i0 + per);
  int cnt = 0;
#pragma unroll 4
  for (int i = i0; i < i1; ++i) cnt += pred(i) ? 1 : 0;
  int total;
  int pos = cta_exclusive_scan(cnt, scratch, &total);
#pragma unroll 4
  for (int i = i0; i < i1; ++i)
    if (pred(i)) emit(pos++, i);
  __syncthreads();
  return total;
}

// A consumer waits on a stage's full barrier for a reused stage only once the
// producer has issued its unit: several warps share a stage (the stage count
// need not be a multiple of the warp count), and a warp waiting two phases
// ahead of a stage would see the phase of the same parity before it as
// complete. (A stage's first use waits for phase 0 of a fresh barrier, which
// cannot be mistaken.)
__device__ __forceinline__ bool wait_issued(const volatile int* issued, int i, int* err) {
  if (*issued > i) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (*issued > i) return true;
    if ((it & 255u) == 0u && globaltimer() - t0 > kWaitLimitNs) {
      if (err) atomicOr(err, kErrTimeout);
      return false;
    }
  }
}

// What a consumer warp needs to walk its tiles.
struct TileWalk {
  uint8_t* ring;       // stage s at ring + s * stage bytes
  uint64_t* full;
  uint64_t* empty;
  const volatile int* issued;  // units the producer has issued so far
  const int* own;      // selected blocks of this shard, recent last
  int u0, nmine, tpb;  // this CTA's units [u0, u0 + nmine), tiles per block
  float* mw;           // per-warp partial slots (m[G], l[G], o[G][D])
};

// FMA consumer (fp32 K/V, or 4/8-bit codes). Lane = token row for q.k; for
// p.v each lane owns kPiece bytes (kDpl head dims) of a row.
template <typename E, int BITS, int D, int G>
__device__ __forceinline__ void consume_tiles_fma(const DecodeParams& p, const TileWalk& tw, const float* qf,
                                                  const float* qs, float* ps, int warp, int lane) {
  using F = Fmt<int(sizeof(E)), BITS, D>;
  constexpr int NG = F::kGroups, TS = kTileTokens;
  const int S = p.S, T = p.T;
  float m_run[G], l_run[G], o_acc[G][F::kDpl], ob[G][NG];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m_run[g] = -INFINITY;
    l_run[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < F::kDpl; ++e) o_acc[g][e] = 0.0f;
#pragma unroll
    for (int r = 0; r < NG; ++r) ob[g][r] = 0.0f;
  }
  const uint32_t ps_a = smem_u32(ps);
  const uint32_t qf_a = smem_u32(qf);
  for (int i = warp; i < tw.nmine; i += kConsumerWarps) {
    const int s = i % F::kStages;
    if ((i < F::kStages || wait_issued(tw.issued, i, p.err)) &&
        mbar_wait(tw.full + s, uint32_t(i / F::kStages) & 1u, p.err)) {
      if (i == warp && warp == 0 && lane == 0) SD_STAMP_HERE(p, 9);
      const int u = tw.u0 + i, li = u / tw.tpb, tile = u % tw.tpb, j = tw.own[li];
      const int nv = min(TS, T - (j * S + tile * TS));
      uint8_t* stage = tw.ring + s * F::kStageBytes;
      const uint32_t kb = smem_u32(stage);
      const uint32_t vb = kb + F::kKvTileBytes;
      // --- q.k: lane = token row ---
      const int t = lane;
      float sc[G], acc[G][NG];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sc[g] = 0.0f;
#pragma unroll
        for (int r = 0; r < NG; ++r) acc[g][r] = 0.0f;
      }
#pragma unroll
      for (int ch = 0; ch < F::kNChunk; ++ch) {
        const int bx = ch / F::kCpb, cc = ch % F::kCpb;
        const uint4 raw = lds128(kb + bx * TS * F::kBoxBytes + swz(uint32_t(t * F::kBoxBytes + cc * 16), F::kCpb));
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          constexpr int EPW = F::kEpc / 4;  // elements per 32-bit word
          float f[EPW];
          if constexpr (BITS == 8) {
#pragma unroll
            for (int e = 0; e < EPW; ++e) f[e] = code_u8(wv[wi], e);
          } else if constexpr (BITS == 4) {
#pragma unroll
            for (int e = 0; e < EPW; ++e) f[e] = code_u4(wv[wi], e);
          } else {
            unpack_word<E>(wv[wi], f);
          }
#pragma unroll
          for (int e = 0; e < EPW; ++e) {
            const int d = ch * F::kEpc + wi * EPW + e;
            float qv[G];
            if constexpr (G % 4 == 0) {
#pragma unroll
              for (int g4 = 0; g4 < G; g4 += 4) {
                const float4 x = lds_f4(qf_a + (d * G + g4) * 4);
                qv[g4] = x.x; qv[g4 + 1] = x.y; qv[g4 + 2] = x.z; qv[g4 + 3] = x.w;
              }
            } else {
#pragma unroll
              for (int g = 0; g < G; ++g) qv[g] = qf[d * G + g];
            }
            if constexpr (BITS == 0) {
#pragma unroll
              for (int g = 0; g < G; ++g) sc[g] = fmaf(qv[g], f[e], sc[g]);
            } else {
              const int grp = d / 64;
#pragma unroll
              for (int g = 0; g < G; ++g) acc[g][grp] = fmaf(qv[g], f[e], acc[g][grp]);
            }
          }
        }
      }
      float vsc[NG], vbi[NG];
      if constexpr (BITS != 0) {
        const E* ksc = reinterpret_cast<const E*>(stage + 2 * F::kKvTileBytes);
        const E* kbi = ksc + TS * NG;
        const E* vs = ksc + 2 * TS * NG;
        const E* vbp = ksc + 3 * TS * NG;
#pragma unroll
        for (int r = 0; r < NG; ++r) {
          const float s_ = Elt<E>::to_f32(ksc[t * NG + r]);
          const float b_ = Elt<E>::to_f32(kbi[t * NG + r]);
#pragma unroll
          for (int g = 0; g < G; ++g) sc[g] = fmaf(s_, acc[g][r], fmaf(b_, qs[g * NG + r], sc[g]));
          vsc[r] = Elt<E>::to_f32(vs[t * NG + r]);
          vbi[r] = Elt<E>::to_f32(vbp[t * NG + r]);
        }
      }
      // --- online softmax over the tile (log2 domain) ---
      const bool valid = t < nv;
      float pv[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float s_ = valid ? sc[g] : -INFINITY;
        const float mx = warp_max(s_);
        const float mn = fmaxf(m_run[g], mx);
        const float alpha = exp2f(m_run[g] - mn);
        pv[g] = valid ? exp2f(s_ - mn) : 0.0f;
        l_run[g] = l_run[g] * alpha + warp_sum(pv[g]);
#pragma unroll
        for (int e = 0; e < F::kDpl; ++e) o_acc[g][e] *= alpha;
        m_run[g] = mn;
        if constexpr (BITS != 0) {
#pragma unroll
          for (int r = 0; r < NG; ++r) ob[g][r] = ob[g][r] * alpha + warp_sum(valid ? pv[g] * vbi[r] : 0.0f);
        }
      }
      if constexpr (BITS == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) ps[t * G + g] = pv[g];
      } else {
#pragma unroll
        for (int r = 0; r < NG; ++r)
#pragma unroll
          for (int g = 0; g < G; ++g) ps[(t * NG + r) * G + g] = pv[g] * vsc[r];
      }
      __syncwarp();
      // --- p.v: lane owns kPiece bytes (kDpl dims) of rows rr, rr + kRpp, ... ---
      const int rr = lane / F::kLpr, pi = lane % F::kLpr;
      const int byte0 = pi * F::kPiece;
      const int chunk = byte0 / 16, within = byte0 % 16;
      const int bx = chunk / F::kCpb, cc = chunk % F::kCpb;
      const int grp = (pi * F::kDpl) / 64;
      for (int r = rr; r < nv; r += F::kRpp) {
        float pg[G];
        const uint32_t pa = ps_a + ((BITS == 0 ? r : r * NG + grp) * G) * 4;
        if constexpr (G % 4 == 0) {
#pragma unroll
          for (int g4 = 0; g4 < G; g4 += 4) {
            const float4 x = lds_f4(pa + g4 * 4);
            pg[g4] = x.x; pg[g4 + 1] = x.y; pg[g4 + 2] = x.z; pg[g4 + 3] = x.w;
          }
        } else {
#pragma unroll
          for (int g = 0; g < G; ++g) pg[g] = ps[(BITS == 0 ? r : r * NG + grp) * G + g];
        }
        const uint32_t va = vb + bx * TS * F::kBoxBytes + swz(uint32_t(r * F::kBoxBytes + cc * 16), F::kCpb) + within;
        float v[F::kDpl];
        if constexpr (F::kPiece == 16) {
          const uint4 x = lds128(va);
          unpack_word<E>(x.x, v);
          unpack_word<E>(x.y, v + F::kDpl / 4);
          unpack_word<E>(x.z, v + F::kDpl / 2);
          unpack_word<E>(x.w, v + 3 * F::kDpl / 4);
        } else if constexpr (F::kPiece == 8) {
          const uint2 x = lds64(va);
          unpack_word<E>(x.x, v);
          unpack_word<E>(x.y, v + F::kDpl / 2);
        } else {
          const uint32_t x = lds32(va);
          if constexpr (BITS == 8) {
#pragma unroll
            for (int e = 0; e < F::kDpl; ++e) v[e] = code_u8(x, e);
          } else if constexpr (BITS == 4) {
#pragma unroll
            for (int e = 0; e < F::kDpl; ++e) v[e] = code_u4(x, e);
          } else {
            unpack_word<E>(x, v);
          }
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int e = 0; e < F::kDpl; ++e) o_acc[g][e] = fmaf(pg[g], v[e], o_acc[g][e]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(tw.empty + s);
  }
  // Fold the row groups of the p.v mapping together.
#pragma unroll
  for (int o = F::kLpr; o < 32; o <<= 1)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < F::kDpl; ++e) o_acc[g][e] += __shfl_xor_sync(0xffffffffu, o_acc[g][e], o);
  if constexpr (BITS != 0) {
    const int grp = ((lane % F::kLpr) * F::kDpl) / 64;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < F::kDpl; ++e) o_acc[g][e] += ob[g][grp];
  }
  if (warp == 0 && lane == 0) SD_STAMP_HERE(p, 10);
  named_barrier(1, kConsumerWarps * 32);  // all consumers are done with the ring
  float* w = tw.mw + warp * (G * D + 2 * G);
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) { w[g] = m_run[g]; w[G + g] = l_run[g]; }
  }
  if (lane < F::kLpr) {
    const int d0 = lane * F::kDpl;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < F::kDpl; ++e) w[2 * G + g * D + d0 + e] = o_acc[g][e];
  }
}

// Tensor-core consumer for 16-bit dense K/V. Rows of the m16n8k16 tiles are
// the G query heads of the group (rows >= G are zero); columns are tokens
// (q.k^T) or head dims (p.v).
//   q.k^T: A = q (registers, loaded once), B = K rows through ldmatrix from
//          the 128B-swizzled tile; fp32 accumulation, then * scale*log2(e).
//   softmax: per head over the tile (exp2 domain), running (m, l) per lane.
//   p.v:   A = P taken from the q.k^T accumulators (the C fragment of two
//          8-token column tiles is the A fragment of one 16-token k-step),
//          split into hi + lo 16-bit halves so the weights keep ~16
//          significant bits; B = V rows through ldmatrix.trans.
template <typename E, int D, int G>
__device__ __forceinline__ void consume_tiles_mma(const DecodeParams& p, const TileWalk& tw, const E* qg, int warp,
                                                  int lane) {
  using F = Fmt<2, 0, D>;
  constexpr int TS = kTileTokens, KSTEPS = D / 16, NT = TS / 8, ND = D / 8;
  const int g = lane >> 2, tq = lane & 3;
  const int S = p.S, T = p.T;
  uint32_t qa0[KSTEPS], qa2[KSTEPS];
  {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(qg + size_t(g < G ? g : 0) * D);
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      qa0[ks] = g < G ? qw[8 * ks + tq] : 0u;
      qa2[ks] = g < G ? qw[8 * ks + 4 + tq] : 0u;
    }
  }
  float m_run = -INFINITY, l_run = 0.0f;
  float o[ND][4];
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
  const int mq = lane >> 3, r8 = lane & 7;
  for (int i = warp; i < tw.nmine; i += kConsumerWarps) {
    const int s = i % F::kStages;
    if ((i < F::kStages || wait_issued(tw.issued, i, p.err)) &&
        mbar_wait(tw.full + s, uint32_t(i / F::kStages) & 1u, p.err)) {
      if (i == warp && warp == 0 && lane == 0) SD_STAMP_HERE(p, 9);
      const int u = tw.u0 + i, li = u / tw.tpb, tile = u % tw.tpb, j = tw.own[li];
      const int nv = min(TS, T - (j * S + tile * TS));
      const uint32_t kb = smem_u32(tw.ring + s * F::kStageBytes);
      const uint32_t vb = kb + F::kKvTileBytes;
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
        for (int kp = 0; kp < KSTEPS / 2; ++kp) {
          const int chunk = 4 * kp + mq, bx = chunk >> 3, cc = chunk & 7;
          const int row = 8 * nt + r8;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + bx * TS * 128 + swz(uint32_t(row * 128 + cc * 16), 8u), b0, b1, b2, b3);
          mma16816<E>(sc[nt], qa0[2 * kp], qa2[2 * kp], b0, b1);
          mma16816<E>(sc[nt], qa0[2 * kp + 1], qa2[2 * kp + 1], b2, b3);
        }
      }
      // online softmax over the tile per head (lanes 4g..4g+3 share head g)
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = 8 * nt + 2 * tq + e;
          sc[nt][e] = t < nv ? sc[nt][e] * p.scale_log2 : -INFINITY;
          mx = fmaxf(mx, sc[nt][e]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m_run, mx);
      const float alpha = exp2f(m_run - mn);
      float rs = 0.0f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sc[nt][e] = exp2f(sc[nt][e] - mn);  // exp2(-inf) = 0 for padding tokens
          rs += sc[nt][e];
        }
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l_run = l_run * alpha + rs;
      m_run = mn;
#pragma unroll
      for (int nd = 0; nd < ND; ++nd) { o[nd][0] *= alpha; o[nd][1] *= alpha; }
      // p.v: two k-steps of 16 tokens
#pragma unroll
      for (int kt = 0; kt < NT / 2; ++kt) {
        uint32_t h0, l0, h2, l2;
        split2<E>(sc[2 * kt][0], sc[2 * kt][1], h0, l0);
        split2<E>(sc[2 * kt + 1][0], sc[2 * kt + 1][1], h2, l2);
        const int tok = 16 * kt + r8 + 8 * (mq & 1);
#pragma unroll
        for (int dp = 0; dp < ND / 2; ++dp) {
          const int chunk = 2 * dp + (mq >> 1), bx = chunk >> 3, cc = chunk & 7;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vb + bx * TS * 128 + swz(uint32_t(tok * 128 + cc * 16), 8u), b0, b1, b2, b3);
          mma16816<E>(o[2 * dp], h0, h2, b0, b1);
          mma16816<E>(o[2 * dp], l0, l2, b0, b1);
          mma16816<E>(o[2 * dp + 1], h0, h2, b2, b3);
          mma16816<E>(o[2 * dp + 1], l0, l2, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(tw.empty + s);
  }
  if (warp == 0 && lane == 0) SD_STAMP_HERE(p, 10);
  named_barrier(1, kConsumerWarps * 32);  // all consumers are done with the ring
  float* w = tw.mw + warp * (G * D + 2 * G);
  if (g < G) {
    if (tq == 0) { w[g] = m_run; w[G + g] = l_run; }
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
      w[2 * G + g * D + 8 * nd + 2 * tq] = o[nd][0];
      w[2 * G + g * D + 8 * nd + 2 * tq + 1] = o[nd][1];
    }
  }
}

// Tensor-core consumer for 4/8-bit K/V with 16-bit scales (fp16 or bf16
// caches). The codes stay exact: ldmatrix brings a 16-byte piece of a row
// into registers, a byte permute puts each code in the mantissa of the fp16
// 1024 + c, and a packed subtraction leaves c itself. q . k over one
// quantization group of 64 dims is then one fp16 product per k-step
// (q.c, accumulated in fp32) and k's affine form is applied per token in
// fp32: q.k = s * (q.c) + b * sum(q). The order of the dims inside a k-step
// is permuted on both operands alike (a dot product does not care), which is
// what lets one 32-bit register of ldmatrix output feed the mma directly. For
// p.v the codes of two consecutive tokens are paired the same way from
// ldmatrix.trans, and p' = p * s_v (per token and group, as hi + lo fp16) is
// the A operand; the bias part sum_t p * b_v is accumulated on the side. q is scaled by 2^-eq
// so that its fp16 form cannot overflow; eq is undone on the product.
__device__ __forceinline__ uint32_t code_pair_u8(uint32_t r, uint32_t sel) {
  const uint32_t h = __byte_perm(r, 0x6464u, sel);  // fp16 1024 + c in each half
  uint32_t out;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(out) : "r"(h), "r"(0x64006400u));
  return out;
}
__device__ __forceinline__ uint32_t code_pair_u4(uint32_t r, int j) {
  const uint32_t h = ((r >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
  uint32_t out;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(out) : "r"(h), "r"(0x64006400u));
  return out;
}

template <typename E, int BITS, int D, int G>
__device__ __forceinline__ void consume_tiles_qmma(const DecodeParams& p, const TileWalk& tw, const E* qg,
                                                   const float* qs, int warp, int lane) {
  using F = Fmt<2, BITS, D>;
  constexpr int TS = kTileTokens, NT = TS / 8, NG = F::kGroups, NCH = F::kNChunk;
  constexpr int KSTEPS = D / 16;                 // 16-dim k-steps of q.k
  constexpr int CPG = 64 / F::kEpc;              // 16-byte chunks per quantization group
  constexpr int NPC = BITS == 8 ? 2 : 4;         // p.v n-tiles (8 dims each) per chunk
  constexpr int ND = NCH * NPC;                  // p.v n-tiles = D / 8
  static_assert(ND == D / 8, "n-tile count");
  const int g = lane >> 2, tq = lane & 3;
  const int S = p.S, T = p.T;
  // q of head g (rows 8..15 are zero), scaled by 2^-eq, in the permuted order
  float qmax = 0.0f;
  for (int i = lane; i < G * D; i += 32) qmax = fmaxf(qmax, fabsf(Elt<E>::to_f32(qg[i])));
  qmax = warp_max(qmax);
  const int eq = qmax > 16384.0f ? (ilogbf(qmax) - 13) : 0;
  const float qscale = ldexpf(1.0f, -eq);
  auto qv = [&](int d) { return g < G ? Elt<E>::to_f32(qg[g * D + d]) * qscale : 0.0f; };
  uint32_t qa0[KSTEPS], qa2[KSTEPS];
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    if constexpr (BITS == 8) {
      const int d = 16 * ks + 4 * tq;  // chunk ks: dims 4tq..4tq+3 of this lane's register
      qa0[ks] = pack2<__half>(qv(d), qv(d + 1));
      qa2[ks] = pack2<__half>(qv(d + 2), qv(d + 3));
    } else {
      const int c = ks >> 1, h = ks & 1;  // chunk c holds 32 dims; k-step h of it
      const int d = 32 * c + 8 * tq + 2 * h;
      qa0[ks] = pack2<__half>(qv(d), qv(d + 4));
      qa2[ks] = pack2<__half>(qv(d + 1), qv(d + 5));
    }
  }
  const float qfac = ldexpf(p.scale_log2, eq);  // undoes 2^-eq and applies scale * log2(e)
  float m_run = -INFINITY, l_run = 0.0f, ob[NG];
  float o[ND][4];
#pragma unroll
  for (int r = 0; r < NG; ++r) ob[r] = 0.0f;
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
  const int mq = lane >> 3, r8 = lane & 7;
  auto chunk_addr = [&](uint32_t base, int row, int c) {
    const int bx = c / F::kCpb, cc = c % F::kCpb;
    return base + bx * TS * F::kBoxBytes + swz(uint32_t(row * F::kBoxBytes + cc * 16), F::kCpb);
  };
  for (int i = warp; i < tw.nmine; i += kConsumerWarps) {
    const int s = i % F::kStages;
    if ((i < F::kStages || wait_issued(tw.issued, i, p.err)) &&
        mbar_wait(tw.full + s, uint32_t(i / F::kStages) & 1u, p.err)) {
      if (i == warp && warp == 0 && lane == 0) SD_STAMP_HERE(p, 9);
      if (i == warp + kConsumerWarps && warp == 0 && lane == 0) SD_STAMP_HERE(p, 23);
      const int u = tw.u0 + i, li = u / tw.tpb, tile = u % tw.tpb, j = tw.own[li];
      const int LT = p.lt;  // the stage holds LT tokens: LT / 32 halves
      uint8_t* stage = tw.ring + s * F::kStageBytes;
      for (int hf = 0; hf < LT / TS; ++hf) {
      const int nv = min(TS, T - (j * S + tile * LT + hf * TS));
      if (nv <= 0) break;
      const uint32_t kb = smem_u32(stage) + uint32_t(hf * TS * F::kBoxBytes);
      const uint32_t vb = smem_u32(stage) + uint32_t(LT * F::kRowBytes + hf * TS * F::kBoxBytes);
      const E* ksc = reinterpret_cast<const E*>(stage + 2 * LT * F::kRowBytes) + hf * TS * NG;
      const E* kbi = ksc + LT * NG;
      const E* vsc = ksc + 2 * LT * NG;
      const E* vbi = ksc + 3 * LT * NG;
      // --- q.c per group: lane m of the x4 load supplies row r8 of token block mq ---
      float acc[NG][NT][4];
#pragma unroll
      for (int r = 0; r < NG; ++r)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[r][nt][0] = acc[r][nt][1] = acc[r][nt][2] = acc[r][nt][3] = 0.0f;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint32_t rk[4];
        ldsm_x4(chunk_addr(kb, 8 * mq + r8, c), rk[0], rk[1], rk[2], rk[3]);
        const int grp = c / CPG;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if constexpr (BITS == 8) {
            mma16816<__half>(acc[grp][nt], qa0[c], qa2[c], code_pair_u8(rk[nt], 0x4140u),
                             code_pair_u8(rk[nt], 0x4342u));
          } else {
            mma16816<__half>(acc[grp][nt], qa0[2 * c], qa2[2 * c], code_pair_u4(rk[nt], 0),
                             code_pair_u4(rk[nt], 1));
            mma16816<__half>(acc[grp][nt], qa0[2 * c + 1], qa2[2 * c + 1], code_pair_u4(rk[nt], 2),
                             code_pair_u4(rk[nt], 3));
          }
        }
      }
      // scores (log2 units) of head g for tokens 8nt + 2tq + e
      float sc[NT][2];
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = 8 * nt + 2 * tq + e;
          float v = 0.0f;
          if (t < nv && g < G) {
#pragma unroll
            for (int r = 0; r < NG; ++r) {
              const float s_ = Elt<E>::to_f32(ksc[t * NG + r]), b_ = Elt<E>::to_f32(kbi[t * NG + r]);
              v = fmaf(s_, acc[r][nt][e] * qfac, fmaf(b_, qs[g * NG + r], v));
            }
          }
          sc[nt][e] = t < nv ? v : -INFINITY;
          mx = fmaxf(mx, sc[nt][e]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m_run, mx);
      const float alpha = exp2f(m_run - mn);
      float rs = 0.0f, bsum[NG];
#pragma unroll
      for (int r = 0; r < NG; ++r) bsum[r] = 0.0f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = 8 * nt + 2 * tq + e;
          sc[nt][e] = t < nv ? exp2f(sc[nt][e] - mn) : 0.0f;
          rs += sc[nt][e];
          if (t < nv) {
#pragma unroll
            for (int r = 0; r < NG; ++r) bsum[r] = fmaf(sc[nt][e], Elt<E>::to_f32(vbi[t * NG + r]), bsum[r]);
          }
        }
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
#pragma unroll
      for (int r = 0; r < NG; ++r) {
        bsum[r] += __shfl_xor_sync(0xffffffffu, bsum[r], 1);
        bsum[r] += __shfl_xor_sync(0xffffffffu, bsum[r], 2);
        ob[r] = ob[r] * alpha + bsum[r];
      }
      l_run = l_run * alpha + rs;
      m_run = mn;
#pragma unroll
      for (int nd = 0; nd < ND; ++nd) { o[nd][0] *= alpha; o[nd][1] *= alpha; }
      // --- p'.c: k-steps of 16 tokens; A = p * s_v per group (fp16) ---
#pragma unroll
      for (int kt = 0; kt < NT / 2; ++kt) {
        // p' as hi + lo fp16 pairs (~22 significant bits): the code and bias
        // parts of p.v can nearly cancel, so p' must not lose more than fp32
        // would in the sum
        uint32_t pa0[NG], pa2[NG], pl0[NG], pl2[NG];
#pragma unroll
        for (int r = 0; r < NG; ++r) {
          const int t0 = 16 * kt + 2 * tq, t2 = t0 + 8;
          auto sv = [&](int t) { return t < nv ? Elt<E>::to_f32(vsc[t * NG + r]) : 0.0f; };
          split2<__half>(sc[2 * kt][0] * sv(t0), sc[2 * kt][1] * sv(t0 + 1), pa0[r], pl0[r]);
          split2<__half>(sc[2 * kt + 1][0] * sv(t2), sc[2 * kt + 1][1] * sv(t2 + 1), pa2[r], pl2[r]);
        }
#pragma unroll
        for (int c = 0; c < NCH; c += 2) {
          // matrices: tokens 16kt + {0..7, 8..15} of chunks c and c + 1
          uint32_t rv[4];
          ldsm_x4_t(chunk_addr(vb, 16 * kt + 8 * (mq & 1) + r8, c + (mq >> 1)), rv[0], rv[1], rv[2], rv[3]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int cc = c + h, grp = cc / CPG;
            const uint32_t lo = rv[2 * h], hi = rv[2 * h + 1];
#pragma unroll
            for (int jn = 0; jn < NPC; ++jn) {
              uint32_t b0, b1;
              if constexpr (BITS == 8) {
                const uint32_t sel = jn == 0 ? 0x4240u : 0x4341u;
                b0 = code_pair_u8(lo, sel);
                b1 = code_pair_u8(hi, sel);
              } else {
                b0 = code_pair_u4(lo, jn);
                b1 = code_pair_u4(hi, jn);
              }
              mma16816<__half>(o[cc * NPC + jn], pa0[grp], pa2[grp], b0, b1);
              mma16816<__half>(o[cc * NPC + jn], pl0[grp], pl2[grp], b0, b1);
            }
          }
        }
      }
      }  // halves of the stage
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(tw.empty + s);
  }
  if (warp == 0 && lane == 0) SD_STAMP_HERE(p, 10);
  named_barrier(1, kConsumerWarps * 32);  // all consumers are done with the ring
  float* w = tw.mw + warp * (G * D + 2 * G);
  if (g < G) {
    if (tq == 0) { w[g] = m_run; w[G + g] = l_run; }
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
      const int c = nd / NPC, jn = nd % NPC;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = 2 * tq + e;  // column of the n-tile
        const int d = BITS == 8 ? 16 * c + 2 * n + jn : 32 * c + 4 * n + jn;
        w[2 * G + g * D + d] = o[nd][e] + ob[d / 64];
      }
    }
  }
}

// 8-bit codes on tensor cores with the tokens as the rows of the m16n8k16
// tile: S^T = K q^T and O^T = V^T P^T, so the G <= 8 query heads fill the
// tile's 8 columns (rather than G of its 16 rows): half the mma instructions
// and accumulators of consume_tiles_qmma. The codes enter as exact fp16
// values (code_pair_u8); q.k = s_k * (q.c) + b_k * sum(q) per 64-dim group,
// and p.v = (p * s_v) . c + sum(p * b_v), with p * s_v split into hi + lo
// fp16 halves. TS token rows per pass (a whole 64-row stage, or 32).
// Fragments: lane (g, tq) = (lane / 4, lane % 4).
//   S^T tile (16 tokens x 8 heads): rows g, g + 8 = tokens, columns 2tq, 2tq + 1 = heads.
//   A of S^T: K codes by ldmatrix; k-slots {2tq, 2tq+1, 2tq+8, 2tq+9} = dims 4tq..4tq+3 of
//     the 16-dim chunk (q^T, the B operand, is packed in the same order).
//   B of O^T: P^T by movmatrix from the S^T accumulators (k-slot = token).
//   A of O^T: V codes by ldmatrix.trans; row g = dim 2g, row g + 8 = dim 2g + 1 of the chunk.
template <typename E, int D, int G, int TS>
__device__ __forceinline__ void consume_tiles_q8t(const DecodeParams& p, const TileWalk& tw, const E* qg,
                                                  const float* qs, int warp, int lane) {
  using F = Fmt<2, 8, D>;
  constexpr int MT = TS / 16, NG = F::kGroups, NCH = F::kNChunk;  // NCH = D / 16
  constexpr int CPG = 4;  // 16-dim chunks per 64-dim quantization group
  static_assert(G <= 8 && NCH % 2 == 0 && F::kEpc == 16, "8-bit codes, at most 8 heads");
  static_assert(F::kNBox == 1, "8-bit rows of at most 128 bytes: one box column");
  const int g = lane >> 2, tq = lane & 3;
  const int S = p.S, T = p.T;
  float qmax = 0.0f;
  for (int i = lane; i < G * D; i += 32) qmax = fmaxf(qmax, fabsf(Elt<E>::to_f32(qg[i])));
  qmax = warp_max(qmax);
  const int eq = qmax > 16384.0f ? (ilogbf(qmax) - 13) : 0;
  const float qscale = ldexpf(1.0f, -eq);
  auto qv = [&](int d) { return g < G ? Elt<E>::to_f32(qg[g * D + d]) * qscale : 0.0f; };
  uint32_t qb0[NCH], qb1[NCH];  // q^T of head g: dims 16c + 4tq + {0, 1} and {2, 3}
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int d = 16 * c + 4 * tq;
    qb0[c] = pack2<__half>(qv(d), qv(d + 1));
    qb1[c] = pack2<__half>(qv(d + 2), qv(d + 3));
  }
  const float qfac = ldexpf(p.scale_log2, eq);  // undoes 2^-eq and applies scale * log2(e)
  // this lane's heads: 2tq + h
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f}, ob[2][NG];
  float o[NCH][4];  // O^T of chunk c: (dim 16c + 2g, heads 2tq, 2tq + 1), (dim 16c + 2g + 1, ...)
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int r = 0; r < NG; ++r) ob[h][r] = 0.0f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) o[c][0] = o[c][1] = o[c][2] = o[c][3] = 0.0f;
  const int mq = lane >> 3, r8 = lane & 7;
  auto chunk_addr = [&](uint32_t base, int row, int c) {
    return base + swz(uint32_t(row * F::kBoxBytes + c * 16), F::kCpb);
  };
  for (int i = warp; i < tw.nmine; i += kConsumerWarps) {
    const int s = i % F::kStages;
    if ((i < F::kStages || wait_issued(tw.issued, i, p.err)) &&
        mbar_wait(tw.full + s, uint32_t(i / F::kStages) & 1u, p.err)) {
      if (i == warp && warp == 0 && lane == 0) SD_STAMP_HERE(p, 9);
      if (i == warp + kConsumerWarps && warp == 0 && lane == 0) SD_STAMP_HERE(p, 23);
      const int u = tw.u0 + i, li = u / tw.tpb, tile = u % tw.tpb, j = tw.own[li];
      const int LT = p.lt;  // the stage holds LT tokens: LT / TS passes
      uint8_t* stage = tw.ring + s * F::kStageBytes;
      for (int hf = 0; hf < LT / TS; ++hf) {
      const int nv = min(TS, T - (j * S + tile * LT + hf * TS));
      if (nv <= 0) break;
      const uint32_t kb = smem_u32(stage) + uint32_t(hf * TS * F::kBoxBytes);
      const uint32_t vb = smem_u32(stage) + uint32_t(LT * F::kRowBytes + hf * TS * F::kBoxBytes);
      const E* ksc = reinterpret_cast<const E*>(stage + 2 * LT * F::kRowBytes) + hf * TS * NG;
      const E* kbi = ksc + LT * NG;
      const E* vsc = ksc + 2 * LT * NG;
      const E* vbi = ksc + 3 * LT * NG;
      // --- S^T = K q^T per group: m-tile mt = tokens 16mt .. 16mt + 15 ---
      float acc[NG][MT][4];
#pragma unroll
      for (int r = 0; r < NG; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) acc[r][mt][0] = acc[r][mt][1] = acc[r][mt][2] = acc[r][mt][3] = 0.0f;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int c = 0; c < NCH; c += 2) {
          // matrices: tokens 16mt + {0..7, 8..15} of chunks c and c + 1
          uint32_t r0, r1, r2, r3;
          ldsm_x4(chunk_addr(kb, 16 * mt + 8 * (mq & 1) + r8, c + (mq >> 1)), r0, r1, r2, r3);
          mma16816_f16(acc[c / CPG][mt], code_pair_u8(r0, 0x4140u), code_pair_u8(r1, 0x4140u),
                       code_pair_u8(r0, 0x4342u), code_pair_u8(r1, 0x4342u), qb0[c], qb1[c]);
          mma16816_f16(acc[(c + 1) / CPG][mt], code_pair_u8(r2, 0x4140u), code_pair_u8(r3, 0x4140u),
                       code_pair_u8(r2, 0x4342u), code_pair_u8(r3, 0x4342u), qb0[c + 1], qb1[c + 1]);
        }
      }
      // scores (log2 units): token 16mt + g + 8e, head 2tq + h
      float sc[MT][2][2];
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = 16 * mt + g + 8 * e;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int hd = 2 * tq + h;
            float v = 0.0f;
            if (t < nv && hd < G) {
#pragma unroll
              for (int r = 0; r < NG; ++r) {
                const float s_ = Elt<E>::to_f32(ksc[t * NG + r]), b_ = Elt<E>::to_f32(kbi[t * NG + r]);
                v = fmaf(s_, acc[r][mt][2 * e + h] * qfac, fmaf(b_, qs[hd * NG + r], v));
              }
            }
            sc[mt][e][h] = t < nv ? v : -INFINITY;
            mx[h] = fmaxf(mx[h], sc[mt][e][h]);
          }
        }
      }
      float mn[2], alpha[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 4));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 8));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 16));
        mn[h] = fmaxf(m_run[h], mx[h]);
        alpha[h] = exp2f(m_run[h] - mn[h]);
      }
      float rs[2] = {0.0f, 0.0f}, bsum[2][NG];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int r = 0; r < NG; ++r) bsum[h][r] = 0.0f;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = 16 * mt + g + 8 * e;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            sc[mt][e][h] = t < nv ? exp2f(sc[mt][e][h] - mn[h]) : 0.0f;
            rs[h] += sc[mt][e][h];
            if (t < nv) {
#pragma unroll
              for (int r = 0; r < NG; ++r)
                bsum[h][r] = fmaf(sc[mt][e][h], Elt<E>::to_f32(vbi[t * NG + r]), bsum[h][r]);
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int o_ = 4; o_ <= 16; o_ <<= 1) {
          rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], o_);
#pragma unroll
          for (int r = 0; r < NG; ++r) bsum[h][r] += __shfl_xor_sync(0xffffffffu, bsum[h][r], o_);
        }
        l_run[h] = l_run[h] * alpha[h] + rs[h];
        m_run[h] = mn[h];
#pragma unroll
        for (int r = 0; r < NG; ++r) ob[h][r] = ob[h][r] * alpha[h] + bsum[h][r];
      }
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        o[c][0] *= alpha[0];
        o[c][1] *= alpha[1];
        o[c][2] *= alpha[0];
        o[c][3] *= alpha[1];
      }
      // --- O^T += V^T P'^T: k-step kt = tokens 16kt .. 16kt + 15 ---
#pragma unroll
      for (int kt = 0; kt < MT; ++kt) {
        // P' = p * s_v per group as hi + lo fp16 in the S^T layout (tokens
        // 16kt + g, + 8; heads 2tq, 2tq + 1), transposed into B fragments
        // (tokens 2tq, 2tq + 1 and 8 + 2tq, 8 + 2tq + 1 of head g); the code
        // and bias parts of p.v can nearly cancel, so p' keeps ~22 bits
        uint32_t bh0[NG], bh1[NG], bl0[NG], bl1[NG];
        const int t0 = 16 * kt + g, t1 = t0 + 8;
#pragma unroll
        for (int r = 0; r < NG; ++r) {
          const float s0 = t0 < nv ? Elt<E>::to_f32(vsc[t0 * NG + r]) : 0.0f;
          const float s1 = t1 < nv ? Elt<E>::to_f32(vsc[t1 * NG + r]) : 0.0f;
          uint32_t h0, l0, h1, l1;
          split2<__half>(sc[kt][0][0] * s0, sc[kt][0][1] * s0, h0, l0);
          split2<__half>(sc[kt][1][0] * s1, sc[kt][1][1] * s1, h1, l1);
          bh0[r] = movm_trans(h0);
          bl0[r] = movm_trans(l0);
          bh1[r] = movm_trans(h1);
          bl1[r] = movm_trans(l1);
        }
#pragma unroll
        for (int c = 0; c < NCH; c += 2) {
          // matrices (transposed): tokens 16kt + {0..7, 8..15} of chunks c and c + 1
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(chunk_addr(vb, 16 * kt + 8 * (mq & 1) + r8, c + (mq >> 1)), r0, r1, r2, r3);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int cc = c + hh, grp = cc / CPG;
            const uint32_t ra = hh ? r2 : r0, rb = hh ? r3 : r1;
            const uint32_t a0 = code_pair_u8(ra, 0x4240u), a1 = code_pair_u8(ra, 0x4341u);
            const uint32_t a2 = code_pair_u8(rb, 0x4240u), a3 = code_pair_u8(rb, 0x4341u);
            mma16816_f16(o[cc], a0, a1, a2, a3, bh0[grp], bh1[grp]);
            mma16816_f16(o[cc], a0, a1, a2, a3, bl0[grp], bl1[grp]);
          }
        }
      }
      }  // passes over the stage
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(tw.empty + s);
  }
  if (warp == 0 && lane == 0) SD_STAMP_HERE(p, 10);
  named_barrier(1, kConsumerWarps * 32);  // all consumers are done with the ring
  float* w = tw.mw + warp * (G * D + 2 * G);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int hd = 2 * tq + h;
    if (hd < G) {
      if (g == 0) { w[hd] = m_run[h]; w[G + hd] = l_run[h]; }
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int d = 16 * c + 2 * g + e;
          w[2 * G + hd * D + d] = o[c][2 * e + h] + ob[h][d / 64];
        }
      }
    }
  }
}

template <typename E, int BITS, int D, int G>
__global__ void __launch_bounds__(kThreads, 1)
decode_kernel(const __grid_constant__ DecodeParams p, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmS) {
  using F = Fmt<int(sizeof(E)), BITS, D>;
  constexpr int NG = F::kGroups;
  constexpr int TS = kTileTokens;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  const Layout L = make_layout(D, G, NG);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  SD_STAMP_T(p, 0);
  SD_STAMP_C(p, 1);
  const int C = p.C, R = p.R;
  const int crank = C > 1 ? int(cluster_ctarank()) : 0;
  const int rep = blockIdx.x / C;  // replica cluster of this CTA
  const int Q = C * R, qrank = rep * C + crank;
  const int bh = blockIdx.y, b = bh / p.Hkv, h = bh % p.Hkv;
  const int K = p.K, P = p.P, pr = p.pr, S = p.S, T = p.T, NB = p.NB;
  const bool peer = p.mode == MODE_PEER;

  float* qf = reinterpret_cast<float*>(sm + L.qf);
  float* qsum = reinterpret_cast<float*>(sm + L.qsum);
  float* qs = reinterpret_cast<float*>(sm + L.qs);
  int* sel = reinterpret_cast<int*>(sm + L.sel);
  uint32_t* hist = reinterpret_cast<uint32_t*>(sm + L.hist);
  int* scratch = reinterpret_cast<int*>(sm + L.scratch);
  RadixState* rs = reinterpret_cast<RadixState*>(scratch + 40);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint64_t* empty = full + 16;
  // Ring aliases (only one is live at a time): candidate keys [0, 64K);
  // sorted runs [64K, 72K); radix-reduced candidates [72K, 80K); the
  // cluster's sorted lists [80K, 144K); selection flags [144K, 152K); the
  // selection result over the keys; sharded-attend union [64K, 128K).
  uint32_t* keys = reinterpret_cast<uint32_t*>(sm + L.ring);
  uint2* uni = reinterpret_cast<uint2*>(sm + L.ring + L.union_off);
  uint2* pick = reinterpret_cast<uint2*>(sm + L.ring);

  // ---------------- phase 0: barriers, queries, append ----------------
  // With a programmatic launch, the next kernel may start its own prologue
  // now; everything that the previous kernel may have produced (queries, the
  // new token, and this index unless pdl_early says otherwise) is read only
  // after griddep_wait.
  if (tid == 0) griddep_launch_dependents();
  // Cluster start-up barrier: arrived here, waited for before the first key
  // is pushed into a peer's shared memory.
  if (C > 1) cluster_arrive_relaxed();
  if (!p.pdl_early) griddep_wait();
  if (tid == 0) {
    for (int s = 0; s < F::kStages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    fence_mbar_init();
    scratch[124] = 0;  // units issued by the producer
  }
  if (warp == kConsumerWarps && lane == 0 && p.mode != MODE_CANDIDATES) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    if (BITS != 0 && p.sb_fused) prefetch_tensormap(&tmS);
  }
  const bool owner_recent = ((NB - 1) % P) == pr;
  // The new token is appended by the group's last CTA (qrank Q - 1): it attends
  // the last unit, the recent block's last tile, which holds the new row, and
  // it keeps the recent block's running column sums.
  const bool appending = p.k_new != nullptr && p.mode != MODE_ATTEND && owner_recent && qrank == Q - 1;
  // The appended token fills its block: its summary key is written in this
  // launch (from the running column sums).
  const bool completing = p.k_new != nullptr && p.mode != MODE_ATTEND && owner_recent && (T % S) == 0;

  const int ncand = NB - 1;  // candidate blocks [0, NB-1); the recent block is always taken
  const int nloc = ncand > pr ? (ncand - pr + P - 1) / P : 0;
  // Whole selection (the host sets it for at most kAllKeysMax candidates,
  // K <= 128 and clusters of several CTAs, or one CTA per group): each CTA of
  // a cluster scores chunk crank of C and pushes the keys into every cluster
  // peer's copy of the group's key array; after one cluster barrier every CTA
  // selects by the same block-wide bitonic top-K (replica clusters repeat
  // this; the keys are few). Otherwise the selection is sliced: every CTA of
  // the group scores chunk qrank of Q, keeps its best keys, and the lists
  // meet in L2.
  const bool whole = p.mode != MODE_ATTEND && !p.sliced;
  const int NCH = whole ? C : Q, ich = whole ? crank : qrank;
  // 32-bit: r * nloc <= 64 * 2^19 (the host bounds capacity and group size)
  auto chunk_lo = [&](int r) { return r * nloc / NCH; };
  const int c0 = chunk_lo(ich), c1 = chunk_lo(ich + 1);
  const int n = c1 - c0;
  auto jglob = [&](int i) { return (c0 + i) * P + pr; };
  uint32_t* allk = reinterpret_cast<uint32_t*>(sm + L.allk);
  if (whole) keys = allk + c0;
  else if (n <= kAllKeysMax) keys = allk;  // the ring stays free for the lists
  const int sc0 = c0, sn = n;  // the rows this CTA scores

  // Score-phase loads go out before the query barrier so that the two memory
  // latencies overlap. Warps 0..7 score; the producer warp does not.
  constexpr int LPB = F::kSumLanes, EPC = F::kSumEpc, BPW = 32 / LPB, UNR = 8, NWS = kConsumerWarps;
  const int sub = lane / LPB, cch = lane % LPB;
  const bool scorer = warp < NWS && p.mode != MODE_ATTEND;
  const uint8_t* sbase = static_cast<const uint8_t*>(p.summ) + (size_t(bh) * p.nb_stride + sc0) * D * sizeof(E);
  const uint64_t spol = stream_policy(p.l2_plain != 0);  // L2 policy of the streamed summaries and K/V tiles
  // The CTA's summary rows go to L2 at once: one bulk prefetch per 64 KB
  // (thread 0; safe before the grid-dependency wait -- L2 is coherent and a
  // prefetch never returns data), so the register batches below stream from
  // L2 and HBM works on the whole chunk from the start.
  if (p.mode != MODE_ATTEND && tid == 0 && sn > 0) {
    constexpr int SROW = D * int(sizeof(E));
    for (size_t off = 0; off < size_t(sn) * SROW; off += 65536)
      bulk_prefetch_l2(sbase + off, uint32_t(min(size_t(65536), size_t(sn) * SROW - off)), spol);
  }
  // bucket histogram of the sliced selection's threshold searches (in the ring)
  uint32_t* hbk = reinterpret_cast<uint32_t*>(sm + L.ring + 128 * 1024);
  const uint8_t* srow0 = sbase + cch * 16;
  // Lane-staged scoring (the keys do not live in the ring): every lane copies
  // its own 16-byte chunks of NBQ batches ahead into a slot of the ring with
  // cp.async (128 KB in flight per CTA instead of a register batch), and
  // reads back only what it copied itself -- no waits between lanes.
  constexpr int NBQ = 4;                                 // batches in flight per warp
  constexpr int BATCH_ROWS = NWS * BPW * UNR;            // rows of one batch of the CTA
  const bool lstage = p.mode != MODE_ATTEND && keys != reinterpret_cast<uint32_t*>(sm + L.ring);
  const uint32_t lslot = smem_u32(sm + L.ring) + uint32_t(warp * NBQ * UNR * 512 + lane * 16);
  auto stage_batch = [&](int bt) {  // batch bt of this warp into slot bt % NBQ, one commit group
    const int it = warp * BPW + bt * BATCH_ROWS;
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int i = it + u * NWS * BPW + sub;
      if (i < sn) cp_async16(lslot + uint32_t(((bt % NBQ) * UNR + u) * 512), srow0 + size_t(i) * D * sizeof(E), spol);
    }
    cp_async_commit();
  };
  uint4 raw[UNR];
  if (scorer && lstage) {
    for (int bt = 0; bt < NBQ; ++bt) stage_batch(bt);
  } else if (scorer) {
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int i = warp * BPW + u * NWS * BPW + sub;
      raw[u] = i < sn ? ldg_stream(srow0 + size_t(i) * D * sizeof(E), spol) : make_uint4(0u, 0u, 0u, 0u);
    }
  }

  if (p.pdl_early) griddep_wait();
  // The producer warp appends the new token during phase 1; its inputs are
  // loaded now, next to the queries.
  constexpr int EPL = D / 32;
  TokenRows<E, BITS, D> tok;
  float rin[EPL];
  const int apos = (T - 1) % S;  // position of the new token in its block
  const bool keep_sums = appending;
  if (warp == kConsumerWarps && appending) {
    append_load<E, BITS, D>(tok, static_cast<const E*>(p.k_new) + size_t(bh) * D,
                            static_cast<const E*>(p.v_new) + size_t(bh) * D, lane);
    if (keep_sums && apos > 0 && !p.racc_rebuild) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) rin[e] = p.racc_in[size_t(bh) * D + lane * EPL + e];
    }
  }
  // Peer mode: this launch's epoch, read after the grid-dependency wait (the
  // previous launch is complete). The control word changes only after every
  // CTA of the previous launch has finished, so all CTAs read the same value;
  // nothing touches an exchange area before this point.
  const uint32_t epoch = peer ? *reinterpret_cast<const volatile uint32_t*>(p.peer[pr] + p.x_ctl) + 1u : 0u;
  // this launch's epoch of the group merge (the previous launch is complete)
  const uint32_t gep = Q > 1 ? __ldcg(p.gep + bh) + 1u : 0u;
  const E* qg = static_cast<const E*>(p.q) + (size_t(b) * p.Hq + size_t(h) * G) * D;
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    qf[d * G + g] = __fmul_rn(Elt<E>::to_f32(qg[i]), p.scale_log2);
  }
  if (tid < D) {
    float a = Elt<E>::to_f32(qg[tid]);
#pragma unroll
    for (int g = 1; g < G; ++g) a = __fadd_rn(a, Elt<E>::to_f32(qg[g * D + tid]));
    qsum[tid] = a;
  }
  __syncthreads();
  if constexpr (BITS != 0) {
    if (tid < G * NG) {
      const int g = tid / NG, grp = tid % NG;
      float a = 0.0f;
      for (int d = grp * 64; d < grp * 64 + 64; ++d) a += qf[d * G + g];
      qs[g * NG + grp] = a;
    }
  }

  // ---------------- phase 1: block scores ----------------
  SD_STAMP_C(p, 2);
  // (the producer warp appends the new token meanwhile)
  if (C > 1) cluster_wait();
  if (warp == kConsumerWarps && appending) {
    // The token's K and V rows, ordered before this CTA's own TMA loads of
    // them by the proxy fence here and a barrier before the loads.
    const size_t row0 = size_t(bh) * p.cap_local + size_t((NB - 1) / P) * S;
    float kdeq[EPL];
    append_store<E, BITS, D>(tok, p.k_data, p.k_scales, p.k_biases, p.v_data, p.v_scales, p.v_biases, row0 + apos,
                             lane, kdeq);
    fence_proxy_async_global();
    // Running column sums of the recent block (fp32, rows in order -- the
    // canonical summary order): acc = acc_before + appended row as stored;
    // when the appended row fills the block, its summary key is acc / S.
    if (keep_sums) {
      // the sums before this row: carried over, or (after a prefill, a load
      // or a trim of more than one token) summed again from the cache
      float before[EPL];
      if (apos > 0 && p.racc_rebuild) {
        rebuild_sums<E, BITS, D>(p.k_data, p.k_scales, p.k_biases, row0, apos, lane, before);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) before[e] = rin[e];
      }
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const int d = lane * EPL + e;
        float acc = kdeq[e];
        if (apos > 0) acc = __fadd_rn(before[e], kdeq[e]);
        p.racc_out[size_t(bh) * D + d] = acc;
        if (completing)
          static_cast<E*>(p.summ)[(size_t(bh) * p.nb_stride + (NB - 1) / P) * D + d] =
              Elt<E>::from_f32(__fdiv_rn(acc, float(S)));
      }
    }
  }
  // one summary row's score (16-byte chunk per lane, canonical order) -> key
  auto score_row = [&](const uint4& raw16, const float (&qr)[EPC], int i, bool valid) {
    float f[EPC];
    unpack_word<E>(raw16.x, f);
    unpack_word<E>(raw16.y, f + EPC / 4);
    unpack_word<E>(raw16.z, f + EPC / 2);
    unpack_word<E>(raw16.w, f + 3 * EPC / 4);
    float a = 0.0f;
#pragma unroll
    for (int e = 0; e < EPC; ++e) a = __fmaf_rn(qr[e], f[e], a);
#pragma unroll
    for (int o = LPB / 2; o >= 1; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (cch == 0 && valid) {
      const float sc = __fmul_rn(a, p.scale);
      keys[i] = score_key(sc);
      if (p.scores_out) p.scores_out[size_t(bh) * NB + size_t(sc0 + i) * P + pr] = sc;
    }
  };
  if (scorer && lstage) {
    float qr[EPC];
#pragma unroll
    for (int e = 0; e < EPC; ++e) qr[e] = qsum[cch * EPC + e];
    for (int bt = 0, it = warp * BPW; it < sn; ++bt, it += BATCH_ROWS) {
      cp_async_wait<NBQ - 1>();  // this lane's copies of batch bt have landed
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int i = it + u * NWS * BPW + sub;
        const uint4 v = lds128(lslot + uint32_t(((bt % NBQ) * UNR + u) * 512));
        score_row(v, qr, i, i < sn);
      }
      stage_batch(bt + NBQ);  // into the slot just read (this lane's own chunks)
    }
    cp_async_wait<0>();
  } else if (scorer) {
    float qr[EPC];
#pragma unroll
    for (int e = 0; e < EPC; ++e) qr[e] = qsum[cch * EPC + e];
    for (int it = warp * BPW; it < sn; it += NWS * BPW * UNR) {
      uint4 cur[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) cur[u] = raw[u];
      const int nx = it + NWS * BPW * UNR;
      if (nx < sn) {
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const int i = nx + u * NWS * BPW + sub;
          raw[u] = i < sn ? ldg_stream(srow0 + size_t(i) * D * sizeof(E), spol) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int i = it + u * NWS * BPW + sub;
        score_row(cur[u], qr, i, i < sn);
      }
    }
  }
  __syncthreads();

  // This CTA's keys into every cluster peer's copy of the group's key array.
  if (whole && C > 1) {
    for (int idx = tid; idx < n * (C - 1); idx += kThreads) {
      const int i = idx % n, rr = idx / n, r = rr < crank ? rr : rr + 1;
      st_cluster_u32(map_rank(smem_u32(keys + i), uint32_t(r)), keys[i]);
    }
  }

  // ---------------- phase 2: selection ----------------
  SD_STAMP_C(p, 3);
  int kk;  // blocks chosen by top-K
  bool global_done = false;  // peer mode: pick[0, kk) is already the top-K of every shard
  if (whole) {
    if (C > 1) cluster_sync();  // every peer's pushed keys have landed
    SD_STAMP_C(p, 15);
    kk = min(K, nloc);
    if (nloc <= K || K == 0) {
      for (int i = tid; i < kk; i += kThreads) pick[i] = make_uint2(allk[i], uint32_t(i * P + pr));
    } else {
      unsigned long long* runs = reinterpret_cast<unsigned long long*>(sm + L.ring + 32 * 1024);
      auto akey = [&](int i) -> unsigned long long { return full_key(allk[i], i * P + pr); };
      if (K <= 64) block_topk<2>(akey, nloc, runs, lane, warp, kThreads / 32);
      else block_topk<4>(akey, nloc, runs, lane, warp, kThreads / 32);
      SD_STAMP_C(p, 14);
      for (int i = tid; i < kk; i += kThreads) {
        const unsigned long long x = runs[i];
        pick[i] = make_uint2(uint32_t(x >> 32), 0xffffffffu - uint32_t(x));
      }
    }
    __syncthreads();
  } else if (p.mode != MODE_ATTEND) {
    // Sliced selection. (1) This CTA's best min(n, MT) keys of its chunk
    // (radix select when it holds more), in index order. (2) The list goes to
    // L2 as message words tagged with the group's launch epoch. (3) Every CTA
    // gathers the group's Q lists, drops the padding and finds the top-K of
    // their union by radix select: the same set on every CTA. (4) The union
    // holds the group's top-K unless some CTA had more than MT candidates and
    // all MT of them made the union's top-K (its next key might belong too);
    // then every CTA publishes its full top-K list and the selection is made
    // again over those. The decision depends only on the gathered lists, so
    // every CTA takes the same branch.
    const int MT = p.mt;
    // ring map of this path: [0, 16K) local keys as 64-bit keys (or the u32
    // keys of a large chunk below 64K) -- later the picks; [16K, 32K) sorted
    // runs of the bitonic local list; [64K, 128K) the gathered lists;
    // [128K, 144K) bucket histogram; [144K, 146K) a bucket's keys;
    // [146K, 154K) this CTA's list.
    unsigned long long* lk = reinterpret_cast<unsigned long long*>(sm + L.ring);
    unsigned long long* g = reinterpret_cast<unsigned long long*>(sm + L.ring + 64 * 1024);
    unsigned long long* bk = reinterpret_cast<unsigned long long*>(sm + L.ring + 144 * 1024);
    unsigned long long* lst = reinterpret_cast<unsigned long long*>(sm + L.ring + 146 * 1024);
    const uint32_t* keys_c = keys;
    const int cb = c0, Pc = P, prc = pr;
    auto keyf = [=](int i) -> unsigned long long { return full_key(keys_c[i], (cb + i) * Pc + prc); };
    const bool small_n = n <= kAllKeysMax;  // the keys live in allk
    SD_STAMP_C(p, 16);
    bool lk_ready = false;
    // this CTA's best m keys into lst, in no particular order; returns how many
    auto local_list = [&](int m) -> int {
      if (small_n && m <= 128) {
        // bitonic: runs of 64 (m <= 64) or 128 keys sorted in registers by
        // the warps, merged pairwise; runs[0, m) = the top m, descending
        unsigned long long* runs = reinterpret_cast<unsigned long long*>(sm + L.ring + 16 * 1024);
        if (m <= 64) block_topk<2>(keyf, n, runs, lane, warp, kThreads / 32);
        else block_topk<4>(keyf, n, runs, lane, warp, kThreads / 32);
        const int c = min(n, m);
        for (int i = tid; i < c; i += kThreads) lst[i] = runs[i];
        __syncthreads();
        return c;
      }
      if (small_n) {
        if (!lk_ready) {  // the keys as 64-bit keys, once
          for (int i = tid; i < n; i += kThreads) lk[i] = keyf(i);
          __syncthreads();
          lk_ready = true;
        }
        return top_keys(lk, n, m, hbk, false, lst, bk, scratch, hist, rs);
      }
      if (n <= m) {
        for (int i = tid; i < n; i += kThreads) lst[i] = keyf(i);
        __syncthreads();
        return n;
      }
      if (m <= 0) return 0;
      const unsigned long long t =
          topk_threshold(keyf, n, m, hbk, false, reinterpret_cast<int*>(bk), 512, scratch, hist, rs);
      if (tid == 0) scratch[119] = 0;
      __syncthreads();
      for (int i = tid; i < n; i += kThreads) {
        const unsigned long long v = keyf(i);
        if (v >= t) lst[atomicAdd(&scratch[119], 1)] = v;
      }
      __syncthreads();
      return m;
    };
    auto to_pick = [](unsigned long long x) { return make_uint2(uint32_t(x >> 32), 0xffffffffu - uint32_t(x)); };
    if (peer && K > 0 && p.mtp > 0) {
      // One level across the shards: this CTA's best MP keys go to every
      // shard's exchange area (message words tagged with the launch epoch);
      // every CTA of every shard gathers the group's P x Q lists from its own
      // area and takes the top-K of their union -- the same set in the same
      // order everywhere. The union holds the top-K unless a CTA whose list
      // was cut had all MP keys taken; then the two-level path below decides
      // (shard top-K through L2, then the shards' lists).
      const int MP = p.mtp, NLS = P * Q;
      const int nl = local_list(MP);
      SD_STAMP_C(p, 15);
      // area layout [BH][P][Q][MP][2]: the group's lists are contiguous
      const size_t grp = size_t(bh) * NLS * MP * 2;
      for (int r = 0; r < P; ++r) {
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(p.peer[r] + p.x_clst) + grp +
                                  (size_t(pr) * Q + qrank) * MP * 2;
        for (int i = tid; i < MP; i += kThreads) {
          const unsigned long long x = i < nl ? lst[i] : 0ull;
          st_msg(dst + 2 * i, uint32_t(x), epoch);
          st_msg(dst + 2 * i + 1, uint32_t(x >> 32), epoch);
        }
      }
      const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.peer[pr] + p.x_clst) + grp;
      gather_msgs<true>([src](int i) { return src + i; }, NLS * MP * 2, epoch, p.peer_wait_ns, p.err, reinterpret_cast<float*>(g), tid, kThreads, [](int) { return true; });
      __syncthreads();
      SD_STAMP_C(p, 14);
      const int N = NLS * MP;
      const int U = hist_keys(g, N, hbk, scratch);
      SD_STAMP_C(p, 17);
      const unsigned long long tau = U > K ? kth_key(g, N, K, hbk, bk, scratch, hist, rs) : 0ull;
      SD_STAMP_C(p, 18);
      int need = 0;
      for (int li = warp; li < NLS; li += kThreads / 32) {
        const int r = li / Q, q = li - (li / Q) * Q;
        const int nlr = ncand > r ? (ncand - r + P - 1) / P : 0;
        const int nq = (q + 1) * nlr / Q - q * nlr / Q;
        int taken = 0;
        for (int i = lane; i < MP; i += 32) {
          const unsigned long long x = g[size_t(li) * MP + i];
          taken += __popc(__ballot_sync(0xffffffffu, x != 0ull && x >= tau));
        }
        if (lane == 0) need |= (nq > MP && taken == MP);
      }
      const bool cut = __syncthreads_or(need) != 0;
      SD_STAMP_C(p, 19);
      if (!cut) {
        kk = min(K, U);
        const unsigned long long* gc = g;
        uint2* pk = pick;
        cta_compact(N, [gc, tau](int i) { return gc[i] != 0ull && gc[i] >= tau; },
                    [gc, pk, to_pick](int pos, int i) { pk[pos] = to_pick(gc[i]); }, scratch);
        global_done = true;
        SD_STAMP_C(p, 20);
      }
    }
    if (global_done) {
    } else if (K == 0) {
      kk = 0;
    } else if (Q == 1) {
      kk = local_list(K);
      for (int i = tid; i < kk; i += kThreads) pick[i] = to_pick(lst[i]);
      __syncthreads();
    } else {
      // publish this CTA's list (0-padded to m keys; each key as its low and
      // high 32-bit message words) and gather all Q lists into g[0, Q*m)
      auto exchange = [&](unsigned long long* area, int m, int nl) {
        unsigned long long* mine = area + size_t(qrank) * m * 2;
        for (int i = tid; i < m; i += kThreads) {
          const unsigned long long x = i < nl ? lst[i] : 0ull;
          st_msg_gpu(mine + 2 * i, uint32_t(x), gep);
          st_msg_gpu(mine + 2 * i + 1, uint32_t(x >> 32), gep);
        }
        gather_msgs<false>([area](int i) { return area + i; }, Q * m * 2, gep, kWaitLimitNs, p.err,
                           reinterpret_cast<float*>(g), tid, kThreads, [](int) { return true; });
        __syncthreads();
      };
      const int nl1 = local_list(MT);
      SD_STAMP_C(p, 15);
      exchange(p.clist + size_t(bh) * Q * MT * 2, MT, nl1);
      SD_STAMP_C(p, 14);
      int N = Q * MT;
      int U = hist_keys(g, N, hbk, scratch);
      SD_STAMP_C(p, 17);
      unsigned long long tau = U > K ? kth_key(g, N, K, hbk, bk, scratch, hist, rs) : 0ull;
      SD_STAMP_C(p, 18);
      bool fallback = false;
      if (MT < K) {
        // lists whose CTA had more than MT candidates and whose MT entries are
        // all selected: the CTA's next key might belong too
        // (one warp per list: ballots, no shared atomics)
        int need = 0;
        for (int q = warp; q < Q; q += kThreads / 32) {
          int taken = 0;
          for (int i = lane; i < MT; i += 32) {
            const unsigned long long x = g[size_t(q) * MT + i];
            taken += __popc(__ballot_sync(0xffffffffu, x != 0ull && x >= tau));
          }
          if (lane == 0) need |= (chunk_lo(q + 1) - chunk_lo(q) > MT && taken == MT);
        }
        fallback = __syncthreads_or(need) != 0;
      }
      SD_STAMP_C(p, 19);
      if (fallback) {
        // every CTA's full top-K list (the local keys are intact: only the
        // picks, written below, overwrite them)
        const int nl = local_list(K);
        exchange(p.cfall + size_t(bh) * Q * K * 2, K, nl);
        N = Q * K;
        U = hist_keys(g, N, hbk, scratch);
        tau = U > K ? kth_key(g, N, K, hbk, bk, scratch, hist, rs) : 0ull;
      }
      // CANDIDATES mode ends before the group merge, whose owner 0 advances
      // the epoch: CTA 0 holds every list, so every CTA has read the epoch.
      if (p.mode == MODE_CANDIDATES && qrank == 0 && tid == 0) p.gep[bh] = gep;
      kk = min(K, U);
      // the selected keys in the order of the gathered lists: the same order
      // on every CTA of the group
      const unsigned long long* gc = g;
      const unsigned long long tc = tau;
      uint2* pk = pick;
      cta_compact(N, [gc, tc](int i) { return gc[i] != 0ull && gc[i] >= tc; },
                  [gc, pk, to_pick](int pos, int i) { pk[pos] = to_pick(gc[i]); }, scratch);
      SD_STAMP_C(p, 20);
    }
  }
  // The group's top-K of a candidate union uni[0, U) (score key, block):
  // the pairs become 64-bit keys in place, then the bucket histogram finds
  // the K-th key and the keys at or above it are kept in union order; every
  // shard computes the same selection.
  auto select_union = [&](int U) {
    kk = min(K, U);
    unsigned long long* uk64 = reinterpret_cast<unsigned long long*>(uni);
    for (int i = tid; i < U; i += kThreads) {
      const uint2 e = uni[i];
      uk64[i] = full_key(e.x, int32_t(e.y));
    }
    __syncthreads();
    const unsigned long long* ukc = uk64;
    uint2* pk = pick;
    auto emit = [ukc, pk](int pos, int i) {
      pk[pos] = make_uint2(uint32_t(ukc[i] >> 32), 0xffffffffu - uint32_t(ukc[i]));
    };
    if (U > K && K > 0) {
      hist_keys(uk64, U, hbk, scratch);
      const unsigned long long tau = kth_key(uk64, U, K, hbk,
                                             reinterpret_cast<unsigned long long*>(sm + L.ring + 144 * 1024),
                                             scratch, hist, rs);
      cta_compact(U, [ukc, tau](int i) { return ukc[i] >= tau; }, emit, scratch);
    } else {
      for (int i = tid; i < kk; i += kThreads) emit(i, i);
      __syncthreads();
    }
  };
  if (p.mode == MODE_ATTEND) {
    // Sharded attend: the P shards' candidates (gathered by the caller),
    // padding dropped, then the group's top-K by radix select.
    const int tot = P * K;
    const size_t BH = size_t(gridDim.y);
    auto src = [&](int i) { return (size_t(i / K) * BH + bh) * K + (i % K); };
    const int U = cta_compact(
        tot, [&](int i) { return p.cand_block[src(i)] >= 0; },
        [&](int pos, int i) {
          uni[pos] = make_uint2(score_key(p.cand_score[src(i)]), uint32_t(p.cand_block[src(i)]));
        },
        scratch);
    select_union(U);
  } else if (peer && K > 0 && !global_done) {
    // Peer mode: (1) this shard's local top-K (0-padded full keys, two
    // message words each) goes into every shard's exchange area; (2) every
    // shard's candidates of the group are read from this shard's area as
    // their words arrive; (3) the top-K of the P*K union, identical on every
    // shard.
    const int BHn = int(gridDim.y);
    if (crank == 0 && rep == 0) {
      for (int r = 0; r < P; ++r) {
        unsigned long long* dst =
            reinterpret_cast<unsigned long long*>(p.peer[r] + p.x_cand) + (size_t(pr) * BHn + bh) * K * 2;
        for (int i = tid; i < K; i += kThreads) {
          const unsigned long long x = i < kk ? full_key(pick[i].x, int(pick[i].y)) : 0ull;
          st_msg(dst + 2 * i, uint32_t(x >> 32), epoch);
          st_msg(dst + 2 * i + 1, uint32_t(x), epoch);
        }
      }
    }
    const int N = P * K;
    const bool small = N <= kAllKeysMax && K <= 128;
    // When every shard's list is the sorted output of its block top-K (each
    // shard holds more than K candidates and at most kAllKeysMax), the
    // union's top-K is a merge of P sorted runs: the lists land straight in
    // runs of L = 64/128 keys and only the merge levels run. Otherwise the
    // union is staged in shared memory and fully sorted.
    const int RL = K <= 64 ? 64 : 128;
    bool presorted = small && P * RL <= kAllKeysMax;
    for (int r = 0; r < P; ++r) {
      const int nl = ncand > r ? (ncand - r + P - 1) / P : 0;
      presorted = presorted && nl > K && nl <= kAllKeysMax;
    }
    unsigned long long* runs = reinterpret_cast<unsigned long long*>(sm + L.ring + 32 * 1024);
    unsigned long long* uk = reinterpret_cast<unsigned long long*>(sm + L.ring + 80 * 1024);
    const unsigned long long* ck = reinterpret_cast<const unsigned long long*>(p.peer[pr] + p.x_cand);
    auto cword = [&](int i) { return ck + ((size_t(i / K) * BHn + bh) * K + (i % K)) * 2; };
    bool ok = true;
    int nz = 0;
    for (int i = tid; i < N; i += kThreads) {
      const uint32_t hi = ld_msg(cword(i), epoch, p.peer_wait_ns, p.err, &ok);
      const uint32_t lo = ld_msg(cword(i) + 1, epoch, p.peer_wait_ns, p.err, &ok);
      const unsigned long long x = (static_cast<unsigned long long>(hi) << 32) | lo;
      if (presorted) runs[(i / K) * RL + (i % K)] = x;
      else if (small) uk[i] = x;
      nz += x != 0ull;
    }
    if (presorted)
      for (int i = tid; i < P * (RL - K); i += kThreads) runs[(i / (RL - K)) * RL + K + (i % (RL - K))] = 0ull;
    const int U = __syncthreads_count(nz > 0) > 0 ? N : 0;  // any candidate at all
    if (U == 0) {
      kk = 0;
    } else if (small) {
      auto sync_all = [] { __syncthreads(); };
      if (presorted) {
        if (RL == 64) block_merge_runs<2>(runs, P, lane, warp, kThreads / 32, sync_all);
        else block_merge_runs<4>(runs, P, lane, warp, kThreads / 32, sync_all);
      } else {
        auto ukey = [&](int i) -> unsigned long long { return uk[i]; };
        if (K <= 64) block_topk<2>(ukey, N, runs, lane, warp, kThreads / 32);
        else block_topk<4>(ukey, N, runs, lane, warp, kThreads / 32);
      }
      kk = __syncthreads_count(tid < K && runs[tid] != 0ull);
      for (int i = tid; i < kk; i += kThreads) {
        const unsigned long long x = runs[i];
        pick[i] = make_uint2(uint32_t(x >> 32), 0xffffffffu - uint32_t(x));
      }
      __syncthreads();
    } else {
      // larger unions: the words have arrived; compact the non-zero keys into
      // the ring's union area straight from the exchange area
      auto gkey = [&](int i) {
        return (ld_msg_raw(cword(i)) << 32) | (ld_msg_raw(cword(i) + 1) & 0xffffffffull);
      };
      const int Uc = cta_compact(
          N, [&](int i) { return gkey(i) != 0ull; },
          [&](int pos, int i) {
            const unsigned long long x = gkey(i);
            uni[pos] = make_uint2(uint32_t(x >> 32), 0xffffffffu - uint32_t(x));
          },
          scratch);
      select_union(Uc);
    }
  }
  if (p.mode == MODE_CANDIDATES) {
    if (crank == 0 && rep == 0) {
      for (int i = tid; i < K; i += kThreads) {
        const bool v = i < kk;
        p.cand_score[size_t(bh) * K + i] = v ? key_score(pick[i].x) : -INFINITY;
        p.cand_block[size_t(bh) * K + i] = v ? int32_t(pick[i].y) : -1;
      }
    }
    return;
  }

  // Selected blocks (in selection order), then the recent block.
  SD_STAMP_C(p, 4);
  for (int i = tid; i < kk; i += kThreads) sel[i] = int(pick[i].y);
  if (tid == 0) sel[kk] = NB - 1;
  __syncthreads();
  const int n_sel = kk + 1;

  // Blocks of this shard (all of them when P == 1), order kept.
  int* own = reinterpret_cast<int*>(sm + L.own);
  int nown;
  if (P == 1) {
    own = sel;
    nown = n_sel;
  } else {
    // one warp keeps the order with ballots
    if (warp == 0) {
      int base = 0;
      for (int i0 = 0; i0 < n_sel; i0 += 32) {
        const int i = i0 + lane;
        const bool mine = i < n_sel && sel[i] % P == pr;
        const unsigned bal = __ballot_sync(0xffffffffu, mine);
        if (mine) own[base + __popc(bal & ((1u << lane) - 1u))] = sel[i];
        base += __popc(bal);
      }
      if (lane == 0) scratch[126] = base;
    }
    __syncthreads();
    nown = scratch[126];
  }

  // ---------------- phase 3: attention over the staged tiles ----------------
  const int LT = p.lt;  // tokens per staged copy (a unit of the ring)
  const int tpb = S / LT;
  const int recent_tiles = (T - (NB - 1) * S + LT - 1) / LT;
  const int n_units = owner_recent ? (nown - 1) * tpb + recent_tiles : nown * tpb;
  const int u0 = qrank * n_units / Q, u1 = (qrank + 1) * n_units / Q;
  const int nmine = u1 - u0;
  constexpr int WSTRIDE = G * D + 2 * G;
  float* mw = reinterpret_cast<float*>(sm + L.ring);  // per-warp partials, once every stage is consumed
  volatile int* issued = scratch + 124;  // zeroed in phase 0
  const TileWalk tw{sm + L.ring, full, empty, issued, own, u0, nmine, tpb, mw};
  constexpr bool kMma = BITS == 0 && sizeof(E) == 2;
  constexpr bool kQMma = BITS != 0 && sizeof(E) == 2;

  if (warp == kConsumerWarps) {
    auto issue = [&](int i) {
      const int s = i % F::kStages;
      const int u = u0 + i, li = u / tpb, tile = u % tpb, j = own[li];
      const int row = bh * p.cap_local + (j / P) * S + tile * LT;
      uint8_t* st = sm + L.ring + s * F::kStageBytes;
      const uint32_t kvb = uint32_t(LT * F::kRowBytes);                        // K (or V) bytes of the stage
      const uint32_t sbb = F::kQuant ? uint32_t(LT * NG * sizeof(E)) : 0u;     // one scale/bias piece
      mbar_arrive_expect_tx(full + s, 2 * kvb + 4 * sbb);
      // the stage's K and V rows, all column boxes: one copy when the K map
      // covers V too (4-D, V one fixed stride after K), else one each
      if (p.kv_fused) {
        tma_load_4d(st, &tmK, 0, row, 0, 0, full + s, spol);
      } else {
        tma_load_3d(st, &tmK, 0, row, 0, full + s, spol);
        tma_load_3d(st + kvb, &tmV, 0, row, 0, full + s, spol);
      }
      if constexpr (BITS != 0) {
        const size_t so = size_t(row) * NG * sizeof(E);
        uint8_t* sb = st + 2 * kvb;
        if (p.sb_fused) {
          tma_load_2d(sb, &tmS, int32_t(so), 0, full + s, spol);  // so < 2^31 whenever the map is used
        } else {
          bulk_load(sb, static_cast<const uint8_t*>(p.k_scales) + so, sbb, full + s, spol);
          bulk_load(sb + sbb, static_cast<const uint8_t*>(p.k_biases) + so, sbb, full + s, spol);
          bulk_load(sb + 2 * sbb, static_cast<const uint8_t*>(p.v_scales) + so, sbb, full + s, spol);
          bulk_load(sb + 3 * sbb, static_cast<const uint8_t*>(p.v_biases) + so, sbb, full + s, spol);
        }
      }
      *issued = i + 1;
    };
    if (lane == 0) {
      // the ring was last written by generic stores (the selection); the
      // appended token's rows were fenced for the async proxy by the lanes
      // that stored them, before the barriers since (no global fence here:
      // in peer mode it would wait for this thread's stores to other GPUs)
      fence_proxy_async_shared();
      SD_STAMP_HERE(p, 21);
      for (int i = 0; i < min(nmine, F::kStages); ++i) {
        issue(i);
        if (i == 0) SD_STAMP_HERE(p, 22);
      }
      SD_STAMP_HERE(p, 8);
    }
    __syncwarp();
    // sel_out: the selected blocks ascending (rank counting), recent last, -1 padded
    if (p.sel_out && crank == 0 && rep == 0) {
      int32_t* so = p.sel_out + size_t(bh) * (K + 1);
      for (int i = lane; i < kk; i += 32) {
        const int ji = sel[i];
        int pos = 0;
        for (int m = 0; m < kk; ++m) pos += sel[m] < ji ? 1 : 0;
        so[pos] = ji;
      }
      for (int i = kk + lane; i <= K; i += 32) so[i] = i == kk ? NB - 1 : -1;
    }
    if (lane == 0) {
      for (int i = F::kStages; i < nmine; ++i) {
        const int s = i % F::kStages;
        if (!mbar_wait(empty + s, uint32_t((i / F::kStages) - 1) & 1u, p.err)) break;
        issue(i);
      }
    }
    __syncwarp();
  } else if constexpr (kMma) {
    consume_tiles_mma<E, D, G>(p, tw, qg, warp, lane);
  } else if constexpr (kQMma && BITS == 8) {
    // a 64-row stage in one pass (4 m-tiles of tokens: twice the independent
    // mma chains per softmax step), else 32 rows per pass
    if (LT == 64) consume_tiles_q8t<E, D, G, 64>(p, tw, qg, qs, warp, lane);
    else consume_tiles_q8t<E, D, G, kTileTokens>(p, tw, qg, qs, warp, lane);
  } else if constexpr (kQMma) {
    consume_tiles_qmma<E, BITS, D, G>(p, tw, qg, qs, warp, lane);
  } else {
    float* ps = reinterpret_cast<float*>(sm + L.ps + warp * align_up(TS * G * NG * 4, 16));
    consume_tiles_fma<E, BITS, D, G>(p, tw, qf, qs, ps, warp, lane);
  }
  __syncthreads();  // warp partials are in mw
  SD_STAMP_C(p, 5);

  // ---------------- phase 4: merge ----------------
  float* cpart = reinterpret_cast<float*>(sm + L.cpart);  // [G] m, [G] l, [G][D] o
  // the warps' rescale factors first (one exp2 per warp and head), then o
  float* wf = reinterpret_cast<float*>(sm + L.recv);  // [kConsumerWarps][G]
  if (tid < kConsumerWarps * G) {
    const int w = tid / G, g = tid % G;
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < kConsumerWarps; ++w2) M = fmaxf(M, mw[w2 * WSTRIDE + g]);
    wf[tid] = M == -INFINITY ? 0.0f : exp2f(mw[w * WSTRIDE + g] - M);
    if (w == 0) cpart[g] = M;
  }
  __syncthreads();
  if (tid < G) {
    float Ls = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) Ls += mw[w * WSTRIDE + G + tid] * wf[w * G + tid];
    cpart[G + tid] = Ls;
  }
  for (int idx = tid; idx < G * D; idx += kThreads) {
    const int g = idx / D;
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) O += mw[w * WSTRIDE + 2 * G + idx] * wf[w * G + g];
    cpart[2 * G + idx] = O;
  }
  // The group's Q = C*R CTAs merge through L2: output elements are cut into
  // NO slices (NO = p.nown <= Q, host-chosen so that an owner gathers its
  // records in one batch of loads), CTA q < NO owns slice q. Every CTA sends
  // each owner a record -- the (m, l) of every head, then its partial o over
  // the owner's slice -- as message words tagged with the group's launch
  // epoch; each owner reads the Q records of its slice as their words arrive
  // and merges them in CTA order. The other CTAs are done once their records
  // are out: they exit early, and a programmatically dependent next launch
  // can start its prologue on their SMs. All Q CTAs are resident at once
  // (clusters, or replica clusters chosen so that all fit), so the owners'
  // bounded waits always end.
  constexpr int GD = G * D;
  const int NO = Q > 1 ? p.nown : 1;
  const int SL = (GD + NO - 1) / NO;  // slice length
  const int RS = 2 * G + SL;          // record length (words)
  const bool owner = qrank < NO;
  const int e0 = owner ? min(GD, qrank * SL) : GD, e1 = owner ? min(GD, e0 + SL) : GD;
  const int g0 = e0 / D, g1 = (e1 - 1) / D;  // heads this slice touches
  auto emit = [&](int idx, float M, float Ls, float O) {
    const int g = idx / D, d = idx % D;
    const size_t bq = size_t(b) * p.Hq + size_t(h) * G + g;
    if (p.mode == MODE_FUSED) {
      static_cast<E*>(p.out)[bq * D + d] = Elt<E>::from_f32(normalise_out(O, Ls, M, p.sinks, int(bq % p.Hq)));
    } else if (peer) {
      // this shard's record of (group, slice) -- [2G (m, l)][slice of o] as
      // message words -- into every shard's exchange area
      const size_t ro = ((size_t(pr) * gridDim.y + bh) * NO + qrank) * RS;
      for (int r = 0; r < P; ++r) {
        unsigned long long* rec = reinterpret_cast<unsigned long long*>(p.peer[r] + p.x_part) + ro;
        st_msg(rec + 2 * G + idx - e0, __float_as_uint(O), epoch);
        if (idx == e0 || d == 0) {
          st_msg(rec + g, __float_as_uint(M), epoch);
          st_msg(rec + G + g, __float_as_uint(Ls), epoch);
        }
      }
    } else {
      p.part_o[bq * D + d] = O;
      if (d == 0) { p.part_ml[bq * 2] = M; p.part_ml[bq * 2 + 1] = Ls; }
    }
  };
  __syncthreads();  // cpart is complete
  SD_STAMP_C(p, 11);
  if (Q == 1) {
    for (int idx = e0 + tid; idx < e1; idx += kThreads) {
      const int g = idx / D;
      emit(idx, cpart[g], cpart[G + g], cpart[2 * G + idx]);
    }
  } else {
    unsigned long long* slots = p.gslot + size_t(bh) * NO * Q * RS;  // [owner][source][RS]
    for (int i = tid; i < NO * RS; i += kThreads) {
      const int o = i / RS, k = i - o * RS;
      const int e = o * SL + (k - 2 * G);
      if (k >= 2 * G && e >= GD) continue;
      st_msg_gpu(slots + (size_t(o) * Q + qrank) * RS + k, __float_as_uint(k < 2 * G ? cpart[k] : cpart[2 * G + e]),
                 gep);
    }
    SD_STAMP_C(p, 12);
    // as the owner of [e0, e1): every source's record, gathered into shared
    // memory with all loads of a batch in flight at once (the ring is free)
    const unsigned long long* mine = slots + size_t(qrank) * Q * RS;
    float* rq = reinterpret_cast<float*>(sm + L.ring);  // [Q][RS]
    const int nw = e1 - e0;
    auto needed = [&](int k) {
      if (k >= 2 * G) return k - 2 * G < nw;
      const int g = k % G;
      return nw > 0 && g >= g0 && g <= g1;
    };
    if (owner)
      gather_msgs<false>([&](int i) { return mine + i; }, Q * RS, gep, kWaitLimitNs, p.err, rq, tid, kThreads,
                         [&](int i) { return needed(i % RS); });
    __syncthreads();
    SD_STAMP_C(p, 13);
    for (int idx = e0 + tid; idx < e1; idx += kThreads) {
      const int g = idx / D;
      float M = -INFINITY;
      for (int q = 0; q < Q; ++q) M = fmaxf(M, rq[q * RS + g]);
      float Ls = 0.0f, O = 0.0f;
      if (M != -INFINITY) {
        for (int q = 0; q < Q; ++q) {
          const float f = exp2f(rq[q * RS + g] - M);
          Ls += rq[q * RS + G + g] * f;
          O += rq[q * RS + 2 * G + idx - e0] * f;
        }
      }
      emit(idx, M, Ls, O);
    }
    // Owner 0 has every CTA's record, so every CTA of the group has read the
    // epoch: the next launch may use the next one.
    __syncthreads();
    if (qrank == 0 && tid == 0) p.gep[bh] = gep;
  }
  SD_STAMP_C(p, 6);
  SD_STAMP_T(p, 7);
  if (!peer) return;

  // ---------------- peer mode: merge the shards ----------------
  // After this shard's record of the slice went out: read every shard's
  // record of it from this shard's area as its words arrive and merge them in
  // shard order (the same output on every shard). Then every CTA counts
  // itself finished in its own area; the last one of the launch resets the
  // count and publishes the epoch.
  {
    const int BHn = int(gridDim.y);
    const unsigned long long* recs = reinterpret_cast<const unsigned long long*>(p.peer[pr] + p.x_part);
    auto rec = [&](int r) { return recs + ((size_t(r) * BHn + bh) * NO + qrank) * RS; };
    float* rp = reinterpret_cast<float*>(sm + L.ring + 32 * 1024);  // [P][RS] (the ring is free)
    const int nw = e1 - e0;
    __syncthreads();  // the group merge above may still read the ring
    if (owner)
      gather_msgs<true>([&](int i) { return rec(i / RS) + (i % RS); }, P * RS, epoch, p.peer_wait_ns, p.err, rp, tid,
                        kThreads, [&](int i) {
                        const int k = i % RS;
                        if (k >= 2 * G) return k - 2 * G < nw;
                        const int g = k % G;
                        return nw > 0 && g >= g0 && g <= g1;
                      });
    __syncthreads();
    for (int idx = e0 + tid; idx < e1; idx += kThreads) {
      const int g = idx / D, d = idx % D;
      float M = -INFINITY;
      for (int r = 0; r < P; ++r) M = fmaxf(M, rp[r * RS + g]);
      float Ls = 0.0f, O = 0.0f;
      if (M != -INFINITY) {
        for (int r = 0; r < P; ++r) {
          const float f = exp2f(rp[r * RS + g] - M);
          Ls += rp[r * RS + G + g] * f;
          O += rp[r * RS + 2 * G + idx - e0] * f;
        }
      }
      const size_t bq = size_t(b) * p.Hq + size_t(h) * G + g;
      static_cast<E*>(p.out)[bq * D + d] = Elt<E>::from_f32(normalise_out(O, Ls, M, p.sinks, int(bq % p.Hq)));
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t* ctl = reinterpret_cast<uint32_t*>(p.peer[pr] + p.x_ctl);
      __threadfence();
      if (atomicAdd(ctl + 1, 1u) == gridDim.x * gridDim.y - 1u) {
        ctl[1] = 0u;
        __threadfence();
        ctl[0] = epoch;
      }
    }
    SD_STAMP_C(p, 6);
    SD_STAMP_T(p, 7);
  }
}

// LSE merge of P shard partials (rank order) into the output [B, Hq, D].
template <typename E>
__global__ void merge_kernel(int P, int BQ, int D, const float* __restrict__ ml, const float* __restrict__ o,
                             E* __restrict__ out, const float* __restrict__ sinks, int Hq) {
  const int i = blockIdx.x;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float M = -INFINITY;
    for (int r = 0; r < P; ++r) M = fmaxf(M, ml[(size_t(r) * BQ + i) * 2]);
    float Ls = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int r = 0; r < P; ++r) {
        const float f = exp2f(ml[(size_t(r) * BQ + i) * 2] - M);
        Ls += ml[(size_t(r) * BQ + i) * 2 + 1] * f;
        O += o[(size_t(r) * BQ + i) * D + d] * f;
      }
    }
    out[size_t(i) * D + d] = Elt<E>::from_f32(normalise_out(O, Ls, M, sinks, i % Hq));
  }
}

}  // namespace sd
