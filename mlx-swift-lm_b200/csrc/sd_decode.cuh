// sd_decode.cuh -- the retrieval block-sparse decode kernel for sm_100a.
//
// One thread-block cluster of C CTAs serves one (batch, kv-head) group:
//   phase 0  queries of the group -> shared memory; optional append of the new
//            token (the decode half of attentionWithCacheUpdate,
//            Libraries/MLXLMCommon/AttentionUtils.swift:54-66 / :67-76).
//   phase 1  score: every CTA scores its slice of the candidate blocks,
//            score[j] = scale * (sum_g q_g) . summary[j], with half-warp /
//            warp groups of 16-byte streaming loads (one chunk per lane) and a
//            fixed fp32 reduction order (see oracle/sd_oracle.cpp).
//   phase 2  select: per-CTA top-K by radix select on 64-bit keys
//            (score, then lower block index), candidates pushed into every CTA
//            of the cluster through distributed shared memory, then the
//            group's top-K, ascending, plus the most recent block.
//   phase 3  attend: selected blocks are cut into 32-token tiles, spread
//            evenly over the cluster; a producer warp stages K and V tiles
//            with TMA (128B/64B/32B swizzle, no multicast) into a ring of
//            mbarrier-guarded stages; 8 consumer warps run online softmax
//            (exp2 domain) with 4/8-bit codes dequantized in registers.
//   phase 4  merge: warp partials -> CTA partial -> cluster-wide log-sum-exp
//            merge over DSMEM, each CTA writing a slice of the output.
// Sharded decode (MODE_CANDIDATES / MODE_ATTEND) runs phases 0-2 and 2-4 as
// two launches around the caller's all-gather of candidates.
// Semantics of stage 4 follow quantizedScaledDotProductAttention
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
__device__ __forceinline__ int cta_compact(int n, Pred pred, Emit emit, int* scratch) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int i0 = min(n, int(threadIdx.x) * per), i1 = min(n, i0 + per);
  int cnt = 0;
  for (int i = i0; i < i1; ++i) cnt += pred(i) ? 1 : 0;
  int total;
  int pos = cta_exclusive_scan(cnt, scratch, &total);
  for (int i = i0; i < i1; ++i)
    if (pred(i)) emit(pos++, i);
  __syncthreads();
  return total;
}

template <typename E, int BITS, int D, int G>
__global__ void __launch_bounds__(kThreads, 1)
decode_kernel(const __grid_constant__ DecodeParams p, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV) {
  using F = Fmt<int(sizeof(E)), BITS, D>;
  constexpr int NG = F::kGroups;
  constexpr int TS = kTileTokens;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  const Layout L = make_layout(D, G, NG);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = p.C;
  const int crank = C > 1 ? int(cluster_ctarank()) : 0;
  const int bh = blockIdx.y, b = bh / p.Hkv, h = bh % p.Hkv;
  const int K = p.K, P = p.P, pr = p.pr, S = p.S, T = p.T, NB = p.NB;

  float* qf = reinterpret_cast<float*>(sm + L.qf);
  float* qsum = reinterpret_cast<float*>(sm + L.qsum);
  float* qs = reinterpret_cast<float*>(sm + L.qs);
  int* sel = reinterpret_cast<int*>(sm + L.sel);
  uint32_t* hist = reinterpret_cast<uint32_t*>(sm + L.hist);
  int* scratch = reinterpret_cast<int*>(sm + L.scratch);
  RadixState* rs = reinterpret_cast<RadixState*>(scratch + 40);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint64_t* empty = full + 16;
  uint32_t* keys = reinterpret_cast<uint32_t*>(sm + L.ring);
  uint2* uni = reinterpret_cast<uint2*>(sm + L.ring + L.union_off);
  uint2* pick = reinterpret_cast<uint2*>(sm + L.ring);  // selection result (keys are dead by then)

  // ---------------- phase 0: barriers, queries, append ----------------
  if (tid == 0) {
    for (int s = 0; s < F::kStages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    fence_mbar_init();
  }
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
  const bool owner_recent = ((NB - 1) % P) == pr;
  const bool appending = p.k_new != nullptr && p.mode != MODE_ATTEND && owner_recent && crank == C - 1;
  if (appending && warp < 2) {
    const int t = T - 1;
    const size_t row = size_t(bh) * p.cap_local + size_t((NB - 1) / P) * S + (t % S);
    if (warp == 0)
      write_token_row<E, BITS, D>(static_cast<const E*>(p.k_new) + size_t(bh) * D, p.k_data, p.k_scales,
                                  p.k_biases, row, lane);
    else
      write_token_row<E, BITS, D>(static_cast<const E*>(p.v_new) + size_t(bh) * D, p.v_data, p.v_scales,
                                  p.v_biases, row, lane);
    fence_proxy_async_global();
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
  const int ncand = NB - 1;  // candidate blocks [0, NB-1); the recent block is always taken
  const int nloc = ncand > pr ? (ncand - pr + P - 1) / P : 0;
  auto chunk_lo = [&](int r) { return int((long long)r * nloc / C); };
  const int c0 = chunk_lo(crank), c1 = chunk_lo(crank + 1);
  const int n = c1 - c0;
  if (p.mode != MODE_ATTEND) {
    constexpr int LPB = F::kSumLanes, EPC = F::kSumEpc, BPW = 32 / LPB, U = 4;
    constexpr int NW = kThreads / 32;
    const int sub = lane / LPB, c = lane % LPB;
    float qr[EPC];
#pragma unroll
    for (int e = 0; e < EPC; ++e) qr[e] = qsum[c * EPC + e];
    const uint8_t* srow0 =
        static_cast<const uint8_t*>(p.summ) + (size_t(bh) * p.nb_stride + c0) * D * sizeof(E) + c * 16;
    for (int it = warp * BPW; it < n; it += NW * BPW * U) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = it + u * NW * BPW + sub;
        raw[u] = i < n ? ldg_stream(srow0 + size_t(i) * D * sizeof(E)) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = it + u * NW * BPW + sub;
        float f[EPC];
        unpack_word<E>(raw[u].x, f);
        unpack_word<E>(raw[u].y, f + EPC / 4);
        unpack_word<E>(raw[u].z, f + EPC / 2);
        unpack_word<E>(raw[u].w, f + 3 * EPC / 4);
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < EPC; ++e) a = __fmaf_rn(qr[e], f[e], a);
#pragma unroll
        for (int o = LPB / 2; o >= 1; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (c == 0 && i < n) {
          const float sc = __fmul_rn(a, p.scale);
          keys[i] = score_key(sc);
          if (p.scores_out) p.scores_out[size_t(bh) * NB + size_t(c0 + i) * P + pr] = sc;
        }
      }
    }
  }
  __syncthreads();

  // ---------------- phase 2: selection ----------------
  int U = 0;  // entries in the union
  if (p.mode != MODE_ATTEND) {
    int my_off = 0;
    for (int r = 0; r < C; ++r) {
      const int cr = min(K, chunk_lo(r + 1) - chunk_lo(r));
      if (r < crank) my_off += cr;
      U += cr;
    }
    auto jglob = [&](int i) { return (c0 + i) * P + pr; };
    auto put = [&](int pos, int i) {
      const uint32_t k32 = keys[i];
      const int32_t j = jglob(i);
      if (C == 1) {
        uni[my_off + pos] = make_uint2(k32, uint32_t(j));
      } else {
        const uint32_t a = smem_u32(&uni[my_off + pos]);
        for (int r = 0; r < C; ++r) st_cluster_v2(map_rank(a, uint32_t(r)), k32, uint32_t(j));
      }
    };
    if (K > 0 && n > K) {
      auto keyf = [&](int i) -> unsigned long long { return full_key(keys[i], jglob(i)); };
      radix_select(keyf, n, K, hist, rs);
      const unsigned long long pre = rs->prefix, msk = rs->mask;
      cta_compact(n, [&](int i) { return (keyf(i) & msk) >= pre; }, put, scratch);
    } else if (K > 0) {
      for (int i = tid; i < n; i += kThreads) put(i, i);
    }
    if (C > 1) cluster_sync(); else __syncthreads();
  } else {
    // Sharded attend: gather the P shards' candidates, dropping padding.
    const int tot = P * K;
    const size_t BH = size_t(gridDim.y);
    auto src = [&](int i) { return (size_t(i / K) * BH + bh) * K + (i % K); };
    U = cta_compact(
        tot, [&](int i) { return p.cand_block[src(i)] >= 0; },
        [&](int pos, int i) {
          uni[pos] = make_uint2(score_key(p.cand_score[src(i)]), uint32_t(p.cand_block[src(i)]));
        },
        scratch);
  }

  const int kk = min(K, U);
  {
    auto ukey = [&](int i) -> unsigned long long { return full_key(uni[i].x, int32_t(uni[i].y)); };
    if (U > K && K > 0) {
      radix_select(ukey, U, K, hist, rs);
      const unsigned long long pre = rs->prefix, msk = rs->mask;
      cta_compact(U, [&](int i) { return (ukey(i) & msk) >= pre; }, [&](int pos, int i) { pick[pos] = uni[i]; },
                  scratch);
    } else {
      for (int i = tid; i < kk; i += kThreads) pick[i] = uni[i];
      __syncthreads();
    }
  }

  if (p.mode == MODE_CANDIDATES) {
    if (crank == 0) {
      for (int i = tid; i < K; i += kThreads) {
        const bool v = i < kk;
        p.cand_score[size_t(bh) * K + i] = v ? key_score(pick[i].x) : -INFINITY;
        p.cand_block[size_t(bh) * K + i] = v ? int32_t(pick[i].y) : -1;
      }
    }
    if (appending && warp == 0 && (T % S) == 0) {
      const size_t row0 = size_t(bh) * p.cap_local + size_t((NB - 1) / P) * S;
      E* dst = static_cast<E*>(p.summ) + (size_t(bh) * p.nb_stride + (NB - 1) / P) * D;
      block_summary<E, BITS, D>(p.k_data, p.k_scales, p.k_biases, row0, S, dst, lane, 32);
    }
    return;
  }

  // Selected blocks ascending, then the recent block.
  if (p.mode == MODE_FUSED) {
    for (int i = tid; i < kk; i += kThreads) sel[i] = int(pick[i].y);
  } else {
    for (int i = tid; i < kk; i += kThreads) {
      const int ji = int(pick[i].y);
      int pos = 0;
      for (int m = 0; m < kk; ++m) pos += int(pick[m].y) < ji ? 1 : 0;
      sel[pos] = ji;
    }
  }
  if (tid == 0) sel[kk] = NB - 1;
  __syncthreads();
  const int n_sel = kk + 1;
  if (p.sel_out && crank == 0)
    for (int i = tid; i <= K; i += kThreads) p.sel_out[size_t(bh) * (K + 1) + i] = i < n_sel ? sel[i] : -1;

  // Blocks of this shard (all of them when P == 1), order kept.
  int* own = reinterpret_cast<int*>(sm + L.own);
  int nown;
  if (P == 1) {
    own = sel;
    nown = n_sel;
  } else {
    __syncthreads();
    nown = cta_compact(n_sel, [&](int i) { return sel[i] % P == pr; }, [&](int pos, int i) { own[pos] = sel[i]; },
                       scratch);
  }

  // ---------------- phase 3: attention over the staged tiles ----------------
  const int tpb = S / TS;
  const int recent_tiles = (T - (NB - 1) * S + TS - 1) / TS;
  const int n_units = owner_recent ? (nown - 1) * tpb + recent_tiles : nown * tpb;
  const int u0 = int((long long)crank * n_units / C), u1 = int((long long)(crank + 1) * n_units / C);
  const int nmine = u1 - u0;

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

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      fence_proxy_async_shared();
      fence_proxy_async_global();
      for (int i = 0; i < nmine; ++i) {
        const int s = i % F::kStages;
        if (i >= F::kStages && !mbar_wait(empty + s, uint32_t((i / F::kStages) - 1) & 1u, p.err)) break;
        const int u = u0 + i, li = u / tpb, tile = u % tpb, j = own[li];
        const int row = bh * p.cap_local + (j / P) * S + tile * TS;
        uint8_t* st = sm + L.ring + s * F::kStageBytes;
        mbar_arrive_expect_tx(full + s, 2 * F::kKvTileBytes + 4 * F::kSbTileBytes);
#pragma unroll
        for (int bx = 0; bx < F::kNBox; ++bx) {
          tma_load_2d(st + bx * TS * F::kBoxBytes, &tmK, bx * F::kBoxBytes, row, full + s);
          tma_load_2d(st + F::kKvTileBytes + bx * TS * F::kBoxBytes, &tmV, bx * F::kBoxBytes, row, full + s);
        }
        if constexpr (BITS != 0) {
          const size_t so = size_t(row) * NG * sizeof(E);
          uint8_t* sb = st + 2 * F::kKvTileBytes;
          bulk_load(sb, static_cast<const uint8_t*>(p.k_scales) + so, F::kSbTileBytes, full + s);
          bulk_load(sb + F::kSbTileBytes, static_cast<const uint8_t*>(p.k_biases) + so, F::kSbTileBytes, full + s);
          bulk_load(sb + 2 * F::kSbTileBytes, static_cast<const uint8_t*>(p.v_scales) + so, F::kSbTileBytes,
                    full + s);
          bulk_load(sb + 3 * F::kSbTileBytes, static_cast<const uint8_t*>(p.v_biases) + so, F::kSbTileBytes,
                    full + s);
        }
      }
    }
    __syncwarp();
    // A block that just filled up gets its summary key now (it stops being the
    // recent block at the next step). The producer warp is otherwise idle.
    if (appending && (T % S) == 0) {
      const size_t row0 = size_t(bh) * p.cap_local + size_t((NB - 1) / P) * S;
      E* dst = static_cast<E*>(p.summ) + (size_t(bh) * p.nb_stride + (NB - 1) / P) * D;
      block_summary<E, BITS, D>(p.k_data, p.k_scales, p.k_biases, row0, S, dst, lane, 32);
    }
  } else {
    float* ps = reinterpret_cast<float*>(sm + L.ps + warp * align_up(TS * G * NG * 4, 16));
    const uint32_t ps_a = smem_u32(ps);
    const uint32_t qf_a = smem_u32(qf);
    for (int i = warp; i < nmine; i += kConsumerWarps) {
      const int s = i % F::kStages;
      const bool ok = mbar_wait(full + s, uint32_t(i / F::kStages) & 1u, p.err);
      if (ok) {
        const int u = u0 + i, li = u / tpb, tile = u % tpb, j = own[li];
        const int nv = min(TS, T - (j * S + tile * TS));
        const uint32_t kb = smem_u32(sm + L.ring + s * F::kStageBytes);
        const uint32_t vb = kb + F::kKvTileBytes;
        const uint32_t sbb = kb + 2 * F::kKvTileBytes;
        // --- QK: lane = token row ---
        const int t = lane;
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = 0.0f;
        float acc[G][NG];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int r = 0; r < NG; ++r) acc[g][r] = 0.0f;
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
          const E* ksc = reinterpret_cast<const E*>(sm + (sbb - smem_u32(sm)));
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
        // --- PV: lane owns kPiece bytes (kDpl dims) of rows rr, rr+kRpp, ... ---
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
      if (lane == 0) mbar_arrive(empty + s);
    }
    // Fold the row groups of the PV mapping together.
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
  }
  __syncthreads();  // every stage consumed: the ring is free for the merge

  // ---------------- phase 4: merge ----------------
  constexpr int WSTRIDE = G * D + 2 * G;
  float* mw = reinterpret_cast<float*>(sm + L.ring);
  if (warp < kConsumerWarps) {
    float* w = mw + warp * WSTRIDE;
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
  __syncthreads();
  float* cpart = reinterpret_cast<float*>(sm + L.cpart);  // [G] m, [G] l, [G][D] o
  for (int idx = tid; idx < G * D; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mw[w * WSTRIDE + g]);
    float Ls = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float f = exp2f(mw[w * WSTRIDE + g] - M);
        Ls += mw[w * WSTRIDE + G + g] * f;
        O += mw[w * WSTRIDE + 2 * G + g * D + d] * f;
      }
    }
    if (d == 0) { cpart[g] = M; cpart[G + g] = Ls; }
    cpart[2 * G + g * D + d] = O;
  }
  if (C > 1) cluster_sync(); else __syncthreads();

  const int tot = G * D;
  const int e0 = int((long long)crank * tot / C), e1 = int((long long)(crank + 1) * tot / C);
  const uint32_t cp_a = smem_u32(cpart);
  for (int idx = e0 + tid; idx < e1; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int r = 0; r < C; ++r) M = fmaxf(M, C > 1 ? ld_cluster_f32(map_rank(cp_a + g * 4, r)) : cpart[g]);
    float Ls = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int r = 0; r < C; ++r) {
        const float mr = C > 1 ? ld_cluster_f32(map_rank(cp_a + g * 4, r)) : cpart[g];
        const float lr = C > 1 ? ld_cluster_f32(map_rank(cp_a + (G + g) * 4, r)) : cpart[G + g];
        const float orr = C > 1 ? ld_cluster_f32(map_rank(cp_a + (2 * G + g * D + d) * 4, r)) : cpart[2 * G + g * D + d];
        const float f = exp2f(mr - M);
        Ls += lr * f;
        O += orr * f;
      }
    }
    const size_t bq = size_t(b) * p.Hq + size_t(h) * G + g;
    if (p.mode == MODE_FUSED) {
      static_cast<E*>(p.out)[bq * D + d] = Elt<E>::from_f32(Ls > 0.0f ? O / Ls : 0.0f);
    } else {
      p.part_o[bq * D + d] = O;
      if (d == 0) { p.part_ml[bq * 2] = M; p.part_ml[bq * 2 + 1] = Ls; }
    }
  }
  if (C > 1) cluster_sync();
}

// LSE merge of P shard partials (rank order) into the output [B, Hq, D].
template <typename E>
__global__ void merge_kernel(int P, int BQ, int D, const float* __restrict__ ml, const float* __restrict__ o,
                             E* __restrict__ out) {
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
    out[size_t(i) * D + d] = Elt<E>::from_f32(Ls > 0.0f ? O / Ls : 0.0f);
  }
}

}  // namespace sd
