// sd_oracle.cpp -- CPU restatement of retrieval block-sparse decode attention.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA library in
// mlx-swift-lm_b200/csrc: only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py load it. The product path
// never calls it and has no CPU fallback.
//
// PARITY UNPINNED. The reference snapshot (TheTom/mlx-swift-lm) contains no
// block-sparse / retrieval decode path and no golden vectors for one, and the
// library that holds its arithmetic (mlx-swift 0.31.3, MLX C++ core; pinned at
// Package.swift:39) is not vendored and cannot be built or run here. What this
// oracle restates, and from where:
//
//   * KV layout [B, Hkv, cap, D], D contiguous
//       -- Libraries/MLXLMCommon/KVCache.swift:328-371 (KVCacheSimple.update).
//   * Quantized KV tuple (wq uint32-packed, scales, biases) with scales and
//     biases in the key dtype, group size 64 along D
//       -- KVCache.swift:816-889 (updateQuantized), :776-783 (initQuant).
//     The affine rule itself lives in MLX's `quantize` (un-vendored); it is
//     restated here from MLX's published algorithm: per group, scale from the
//     min/max range, the larger-magnitude edge anchored exactly on a code so
//     that 0.0 stays representable, round-half-even codes clamped to
//     [0, 2^bits-1], codes packed little-endian inside each uint32.
//   * Attention math: queries scaled, GQA grouping hq -> hq / G, softmax over
//     keys, weighted sum of values -- KVCache.swift:1544-1618
//     (quantizedScaledDotProductAttention). Sparsity is expressed by gathering
//     the selected blocks, never by the reference's bool-mask path, which
//     fills with Float.leastNormalMagnitude (+1.2e-38) and so excludes nothing
//     (KVCache.swift:1583,1587,1596).
//   * Stages 1-3 (summary = per-block key mean, GQA score, top-K + recent,
//     tie-break lower index wins) have no reference code; they follow the
//     build's specification of this path, restated in canonical fp32 order so
//     the GPU selection can be checked bit for bit.
//
// Canonical fp32 orders (the CUDA kernels use the same operations):
//   summary[j][d] = RNE_dtype( (((k[t0][d] + k[t0+1][d]) + ...) + k[t1-1][d]) / n )
//       sequential fp32 adds over the filled tokens of block j, IEEE division.
//   qsum[d] = ((q[hG][d] + q[hG+1][d]) + ...) + q[hG+G-1][d]
//   score[j] = scale * tree( chunk partials ), where the D elements are cut into
//       16-byte chunks of E = 16/elt elements, partial[c] = fma chain over the
//       chunk starting from 0, and tree(p) folds p[c] += p[c + off] for
//       off = nc/2, nc/4, ..., 1.
//   dequant(code) = fma(scale, code, bias) in fp32.

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };

inline float bits_to_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f32_to_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

inline float bf16_to_f32(uint16_t b) { return bits_to_f32(uint32_t(b) << 16); }
inline uint16_t f32_to_bf16(float f) {
  uint32_t u = f32_to_bits(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40u);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);                                          // round half to even
  return uint16_t(u >> 16);
}
inline float f16_to_f32(uint16_t h) { _Float16 x; std::memcpy(&x, &h, 2); return float(x); }
inline uint16_t f32_to_f16(float f) { _Float16 x = (_Float16)f; uint16_t h; std::memcpy(&h, &x, 2); return h; }

inline int elt_bytes(int dtype) { return dtype == ORC_F32 ? 4 : 2; }

// Host threads used by the parallel loops (0 = all hardware threads).
int g_threads = 1;

// Dynamic parallel loop over [0, n) on g_threads std::threads.
template <class Fn>
void parallel_for(int64_t n, Fn fn) {
  int nt = g_threads > 0 ? g_threads : int(std::max(1u, std::thread::hardware_concurrency()));
  nt = int(std::min<int64_t>(nt, n));
  if (nt <= 1) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next(0);
  std::vector<std::thread> pool;
  for (int t = 0; t < nt; ++t)
    pool.emplace_back([&] {
      for (int64_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
    });
  for (auto& th : pool) th.join();
}

inline float load_elt(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case ORC_F32: return static_cast<const float*>(p)[i];
    case ORC_F16: return f16_to_f32(static_cast<const uint16_t*>(p)[i]);
    default: return bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
  }
}
inline void store_elt(void* p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case ORC_F32: static_cast<float*>(p)[i] = v; break;
    case ORC_F16: static_cast<uint16_t*>(p)[i] = f32_to_f16(v); break;
    default: static_cast<uint16_t*>(p)[i] = f32_to_bf16(v); break;
  }
}
inline float round_to(float v, int dtype) {
  switch (dtype) {
    case ORC_F32: return v;
    case ORC_F16: return f16_to_f32(f32_to_f16(v));
    default: return bf16_to_f32(f32_to_bf16(v));
  }
}

// Order-preserving key of a score; larger key = better. NaN ranks lowest and
// -0.0 is folded onto +0.0 so that equal scores compare equal.
inline uint32_t score_key(float s) {
  if (s != s) return 0u;
  if (s == 0.0f) s = 0.0f;
  uint32_t u = f32_to_bits(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace

extern "C" {

// A view of one K or V cache: dense elements of `dtype`, or affine-quantized
// codes with per-group scales and biases of `dtype`.
typedef struct {
  int32_t bits;        // 0 = dense; 4 or 8 = quantized
  int32_t dtype;       // dense element dtype, or scales/biases dtype
  int32_t group_size;  // quantization group along D
  int32_t cap;         // token capacity per (b, kv-head)
  int32_t D;
  const void* data;    // dense [BH, cap, D]; quantized wq [BH, cap, D*bits/32] (uint32)
  const void* scales;  // quantized only: [BH, cap, D/group_size]
  const void* biases;  // quantized only: [BH, cap, D/group_size]
} orc_kv_view;

int orc_version(void) { return 1; }

// Host threads for the parallel loops of this library (0 = all).
void orc_set_threads(int n) { g_threads = n; }

void orc_to_float(const void* src, int dtype, int64_t n, float* dst) {
  for (int64_t i = 0; i < n; ++i) dst[i] = load_elt(src, dtype, i);
}

void orc_from_float(const float* src, int dtype, int64_t n, void* dst) {
  for (int64_t i = 0; i < n; ++i) store_elt(dst, dtype, i, src[i]);
}

// Affine quantization of rows of D dtype elements, groups of gs along D.
// Restates MLX's affine `quantize` (see file header): computed in fp32,
// scales and biases stored in `dtype` after the codes are chosen.
void orc_quantize(const void* x, int dtype, int64_t rows, int D, int gs, int bits,
                  uint32_t* wq, void* scales, void* biases) {
  const int ng = D / gs;
  const float n_bins = float((1 << bits) - 1);
  const int per_word = 32 / bits;
  const int words = D / per_word;
  // rows are independent: runs of 4096 rows in parallel
  const int64_t RUN = 4096;
  parallel_for((rows + RUN - 1) / RUN, [&](int64_t run) {
    std::vector<float> w(gs);
    std::vector<uint32_t> codes(D);
    for (int64_t r = run * RUN; r < std::min(rows, (run + 1) * RUN); ++r) {
      for (int g = 0; g < ng; ++g) {
        float wmax = -INFINITY, wmin = INFINITY;
        for (int i = 0; i < gs; ++i) {
          w[i] = load_elt(x, dtype, r * D + g * gs + i);
          wmax = std::max(wmax, w[i]);
          wmin = std::min(wmin, w[i]);
        }
        float scale = std::max((wmax - wmin) / n_bins, 1e-7f);
        const bool mask = std::fabs(wmin) > std::fabs(wmax);
        if (!mask) scale = -scale;
        const float edge = mask ? wmin : wmax;
        const float q0 = std::rint(edge / scale);
        if (q0 != 0.0f) scale = edge / q0;
        const float bias = (q0 == 0.0f) ? 0.0f : edge;
        for (int i = 0; i < gs; ++i) {
          float c = std::rint((w[i] - bias) / scale);
          c = std::min(std::max(c, 0.0f), n_bins);
          codes[g * gs + i] = uint32_t(c);
        }
        store_elt(scales, dtype, r * ng + g, scale);
        store_elt(biases, dtype, r * ng + g, bias);
      }
      for (int k = 0; k < words; ++k) {
        uint32_t word = 0;
        for (int i = 0; i < per_word; ++i) word |= codes[k * per_word + i] << (bits * i);
        wq[r * words + k] = word;
      }
    }
  });
}

void orc_dequantize(const uint32_t* wq, const void* scales, const void* biases, int dtype,
                    int64_t rows, int D, int gs, int bits, float* out) {
  const int ng = D / gs;
  const int per_word = 32 / bits;
  const int words = D / per_word;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t r = 0; r < rows; ++r) {
    for (int d = 0; d < D; ++d) {
      const uint32_t word = wq[r * words + d / per_word];
      const float code = float((word >> (bits * (d % per_word))) & mask);
      const float s = load_elt(scales, dtype, r * ng + d / gs);
      const float b = load_elt(biases, dtype, r * ng + d / gs);
      out[r * D + d] = std::fma(s, code, b);
    }
  }
}

}  // extern "C"

namespace {

// Row t of (b, kv-head) `bh` as fp32 values (dequantized when quantized).
inline void load_row(const orc_kv_view* v, int64_t bh, int64_t t, float* out) {
  const int D = v->D;
  const int64_t row = bh * v->cap + t;
  if (v->bits == 0) {
    for (int d = 0; d < D; ++d) out[d] = load_elt(v->data, v->dtype, row * D + d);
    return;
  }
  const int bits = v->bits, gs = v->group_size, ng = D / gs;
  const int per_word = 32 / bits, words = D / per_word;
  const uint32_t mask = (1u << bits) - 1u;
  const uint32_t* wq = static_cast<const uint32_t*>(v->data) + row * words;
  for (int d = 0; d < D; ++d) {
    const float code = float((wq[d / per_word] >> (bits * (d % per_word))) & mask);
    const float s = load_elt(v->scales, v->dtype, row * ng + d / gs);
    const float b = load_elt(v->biases, v->dtype, row * ng + d / gs);
    out[d] = std::fma(s, code, b);
  }
}

inline bool better(uint32_t ka, int32_t ia, uint32_t kb, int32_t ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Top-k of (score, index) pairs by (score desc, index asc); result sorted by index asc.
int topk_sorted(const float* scores, const int32_t* idx, int n, int k, int32_t* out_idx,
                float* out_scores) {
  std::vector<int> order(n);
  std::vector<uint32_t> keys(n);
  for (int i = 0; i < n; ++i) { order[i] = i; keys[i] = score_key(scores[i]); }
  const int m = std::min(k, n);
  std::partial_sort(order.begin(), order.begin() + m, order.end(), [&](int a, int b) {
    return better(keys[a], idx[a], keys[b], idx[b]);
  });
  std::sort(order.begin(), order.begin() + m, [&](int a, int b) { return idx[a] < idx[b]; });
  for (int i = 0; i < m; ++i) {
    out_idx[i] = idx[order[i]];
    if (out_scores) out_scores[i] = scores[order[i]];
  }
  return m;
}

}  // namespace

extern "C" {

// Summaries of blocks [j0, j1) for every (b, kv-head): mean over the filled
// tokens of the block, canonical sequential fp32 sum, IEEE division, rounded to
// sdtype. summ is [BH, nb_stride, D] of sdtype.
void orc_summaries(const orc_kv_view* K, int64_t BH, int T, int S, int j0, int j1, int sdtype,
                   void* summ, int nb_stride) {
  const int D = K->D;
  parallel_for(BH, [&](int64_t bh) {
    std::vector<float> row(D), acc(D);
    for (int j = j0; j < j1; ++j) {
      const int t0 = j * S, t1 = std::min((j + 1) * S, T);
      if (t1 <= t0) continue;
      for (int t = t0; t < t1; ++t) {
        load_row(K, bh, t, row.data());
        if (t == t0) { for (int d = 0; d < D; ++d) acc[d] = row[d]; }
        else { for (int d = 0; d < D; ++d) acc[d] = acc[d] + row[d]; }
      }
      const float n = float(t1 - t0);
      for (int d = 0; d < D; ++d)
        store_elt(summ, sdtype, (bh * nb_stride + j) * D + d, acc[d] / n);
    }
  });
}

// Block scores in canonical fp32 order (file header). q [B, Hq, D] of qdtype;
// summ [B*Hkv, nb_stride, D] of sdtype; scores [B*Hkv, NB].
void orc_scores(const void* q, int qdtype, const void* summ, int sdtype, int B, int Hq, int Hkv,
                int D, int NB, int nb_stride, float scale, float* scores) {
  const int G = Hq / Hkv;
  const int E = 16 / elt_bytes(sdtype);
  const int nc = D / E;
  parallel_for(int64_t(B) * Hkv, [&](int64_t bh) {
    const int64_t b = bh / Hkv, h = bh % Hkv;
    std::vector<float> qsum(D), part(nc);
    for (int d = 0; d < D; ++d) {
      float a = load_elt(q, qdtype, (b * Hq + h * G) * D + d);
      for (int g = 1; g < G; ++g) a = a + load_elt(q, qdtype, (b * Hq + h * G + g) * D + d);
      qsum[d] = a;
    }
    for (int j = 0; j < NB; ++j) {
      const int64_t base = (bh * nb_stride + j) * D;
      for (int c = 0; c < nc; ++c) {
        float a = 0.0f;
        for (int e = 0; e < E; ++e) a = std::fma(qsum[c * E + e], load_elt(summ, sdtype, base + c * E + e), a);
        part[c] = a;
      }
      for (int off = nc / 2; off >= 1; off /= 2)
        for (int c = 0; c < off; ++c) part[c] = part[c] + part[c + off];
      scores[bh * NB + j] = part[0] * scale;
    }
  });
}

// Selection per (b, kv-head): the top-k of blocks [0, NB-1) by (score desc,
// block index asc), sorted ascending, followed by the recent block NB-1.
// Returns the number of selected blocks, min(k, NB-1) + 1.
int orc_select(const float* scores, int64_t BH, int NB, int k, int32_t* sel, int sel_stride) {
  const int n = NB - 1;
  int n_sel = std::min(k, n) + 1;
  std::vector<int32_t> idx(std::max(n, 1));
  for (int i = 0; i < n; ++i) idx[i] = i;
  for (int64_t bh = 0; bh < BH; ++bh) {
    const int m = topk_sorted(scores + bh * NB, idx.data(), n, k, sel + bh * sel_stride, nullptr);
    sel[bh * sel_stride + m] = NB - 1;
  }
  return n_sel;
}

// Generic top-k of candidate (score, global block index) pairs, result sorted
// by block index ascending. Used for local and global (sharded) selection.
int orc_topk(const float* scores, const int32_t* idx, int n, int k, int32_t* out_idx,
             float* out_scores) {
  return topk_sorted(scores, idx, n, k, out_idx, out_scores);
}

// Attention of every query head over the tokens of its group's selected
// blocks (tokens < T only). fp64 accumulation. Writes, per (b, hq), the
// running max m (natural-log domain, scaled logits), the sum l = sum exp(s-m)
// and the unnormalised o = sum exp(s-m) v, or the normalised output when
// `normalise` is set (then m and l may be null).
void orc_attend_f64(const void* q, int qdtype, const orc_kv_view* K, const orc_kv_view* V, int B,
                    int Hq, int Hkv, int T, int S, const int32_t* sel, int n_sel, int sel_stride,
                    double scale, int normalise, double* m_out, double* l_out, double* o_out) {
  const int G = Hq / Hkv, D = K->D;
  parallel_for(int64_t(B) * Hq, [&](int64_t bq) {
    const int64_t b = bq / Hq, hq = bq % Hq, bh = b * Hkv + hq / G;
    std::vector<double> qv(D), o(D, 0.0), logits;
    std::vector<int64_t> toks;
    std::vector<float> row(D);
    for (int d = 0; d < D; ++d) qv[d] = load_elt(q, qdtype, bq * D + d);
    for (int i = 0; i < n_sel; ++i) {
      const int j = sel[bh * sel_stride + i];
      if (j < 0) continue;
      for (int t = j * S; t < std::min((j + 1) * S, T); ++t) {
        load_row(K, bh, t, row.data());
        double s = 0.0;
        for (int d = 0; d < D; ++d) s += qv[d] * double(row[d]);
        logits.push_back(s * scale);
        toks.push_back(t);
      }
    }
    double m = -INFINITY, l = 0.0;
    for (double s : logits) m = std::max(m, s);
    for (size_t i = 0; i < logits.size(); ++i) {
      const double p = std::exp(logits[i] - m);
      l += p;
      load_row(V, bh, toks[i], row.data());
      for (int d = 0; d < D; ++d) o[d] += p * double(row[d]);
    }
    if (m_out) m_out[bq] = m;
    if (l_out) l_out[bq] = l;
    for (int d = 0; d < D; ++d) o_out[bq * D + d] = normalise ? (l > 0 ? o[d] / l : 0.0) : o[d];
  });
}

// Log-sum-exp merge of P partials (m, l, o unnormalised) in rank order.
void orc_merge_f64(int P, int64_t BQ, int D, const double* m, const double* l, const double* o,
                   double* out) {
  for (int64_t i = 0; i < BQ; ++i) {
    double M = -INFINITY;
    for (int p = 0; p < P; ++p) if (l[p * BQ + i] > 0) M = std::max(M, m[p * BQ + i]);
    double L = 0.0;
    for (int p = 0; p < P; ++p) if (l[p * BQ + i] > 0) L += l[p * BQ + i] * std::exp(m[p * BQ + i] - M);
    for (int d = 0; d < D; ++d) {
      double acc = 0.0;
      for (int p = 0; p < P; ++p)
        if (l[p * BQ + i] > 0) acc += o[(p * BQ + i) * D + d] * std::exp(m[p * BQ + i] - M);
      out[i * D + d] = L > 0 ? acc / L : 0.0;
    }
  }
}

}  // extern "C"
