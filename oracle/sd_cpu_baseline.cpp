// sd_cpu_baseline.cpp -- the timed fp32 CPU implementation of the decode path.
//
// TEST INFRASTRUCTURE ONLY: bench.py's cpu_baseline and --impl reference legs
// time it; nothing in the product library calls it. The reference's own CPU
// implementation of this path (MLX's CPU backend under mlx-swift) cannot run
// here, so this file stands in for it: the same four stages as sd_oracle.cpp
// (summaries are given), written to run fast on the host cores.
//
//   scoring     parallel over (b, kv-head, run of 512 blocks); each score in
//               the canonical fp32 order of sd_oracle.cpp (per 16-byte chunk
//               an fma chain from 0, a fixed tree over chunks, * scale), so
//               the selection equals the oracle's bit for bit.
//   selection   per (b, kv-head): top-K of blocks [0, NB-1) by (score desc,
//               block index asc) with std::nth_element, then the recent block
//               (Evaluate.swift:283-290 is the nearest reference idiom).
//   attention   parallel over (b, kv-head, selected block): the block's K and
//               V rows are converted (dequantized with fma(scale, code, bias)
//               for 4/8-bit caches, KVCache.swift:1544-1618 for the math) into
//               a float tile, q.k and p.v run as 8-wide AVX2 FMA loops, and
//               each task leaves a partial (m, l, o) per query head; the
//               partials are merged per group in block order (log-sum-exp).
//
// Threads: a persistent pool of worker threads (created on first use, sized by
// orc_base_set_threads); orc_base_last_threads() reports how many distinct
// threads ran at least one task in the last call.
#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace {

enum { F32 = 0, F16 = 1, BF16 = 2 };

inline float bits_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f32_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float bf16_f32(uint16_t b) { return bits_f32(uint32_t(b) << 16); }
inline uint16_t f32_bf16(float f) {
  uint32_t u = f32_bits(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
inline float f16_f32(uint16_t h) { _Float16 x; std::memcpy(&x, &h, 2); return float(x); }
inline uint16_t f32_f16(float f) { _Float16 x = (_Float16)f; uint16_t h; std::memcpy(&h, &x, 2); return h; }

inline float ld(const void* p, int dt, int64_t i) {
  if (dt == F32) return static_cast<const float*>(p)[i];
  const uint16_t h = static_cast<const uint16_t*>(p)[i];
  return dt == F16 ? f16_f32(h) : bf16_f32(h);
}
inline void st(void* p, int dt, int64_t i, float v) {
  if (dt == F32) static_cast<float*>(p)[i] = v;
  else static_cast<uint16_t*>(p)[i] = dt == F16 ? f32_f16(v) : f32_bf16(v);
}
inline uint32_t score_key(float s) {
  if (s != s) return 0u;
  if (s == 0.0f) s = 0.0f;
  const uint32_t u = f32_bits(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// Persistent thread pool: parallel_for(n, fn) runs fn(i) for i in [0, n) on the
// workers and the calling thread, dynamic scheduling by an atomic counter.
// ---------------------------------------------------------------------------
class Pool {
 public:
  void resize(int n) {
    stop();
    n_ = std::max(1, n);
    quit_ = false;
    for (int t = 1; t < n_; ++t) workers_.emplace_back([this, t] { loop(t); });
  }
  int size() const { return n_; }
  int run(int64_t n, const std::function<void(int64_t)>& fn) {
    if (n <= 0) return 0;
    used_.assign(size_t(n_), 0);
    {
      std::unique_lock<std::mutex> lk(mu_);
      fn_ = &fn;
      total_ = n;
      next_.store(0);
      busy_ = n_ - 1;
      ++gen_;
    }
    cv_.notify_all();
    work(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return busy_ == 0; });
    fn_ = nullptr;
    int c = 0;
    for (char u : used_) c += u ? 1 : 0;
    return c;
  }
  ~Pool() { stop(); }

 private:
  void work(int t) {
    for (int64_t i = next_.fetch_add(1); i < total_; i = next_.fetch_add(1)) {
      (*fn_)(i);
      used_[size_t(t)] = 1;
    }
  }
  void loop(int t) {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
        if (quit_) return;
        seen = gen_;
      }
      work(t);
      std::lock_guard<std::mutex> lk(mu_);
      if (--busy_ == 0) done_cv_.notify_one();
    }
  }
  void stop() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
    workers_.clear();
  }
  int n_ = 1;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int64_t)>* fn_ = nullptr;
  std::atomic<int64_t> next_{0};
  int64_t total_ = 0;
  int busy_ = 0;
  uint64_t gen_ = 0;
  bool quit_ = false;
  std::vector<char> used_;
};

Pool& pool() {
  static Pool p;
  return p;
}
int g_last_threads = 0;

inline float dot8(const float* a, const float* b, int D) {
  __m256 acc = _mm256_setzero_ps();
  for (int d = 0; d < D; d += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + d), _mm256_loadu_ps(b + d), acc);
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
  s = _mm_hadd_ps(s, s);
  s = _mm_hadd_ps(s, s);
  return _mm_cvtss_f32(s);
}
inline void axpy8(float a, const float* x, float* y, int D) {
  const __m256 va = _mm256_set1_ps(a);
  for (int d = 0; d < D; d += 8)
    _mm256_storeu_ps(y + d, _mm256_fmadd_ps(va, _mm256_loadu_ps(x + d), _mm256_loadu_ps(y + d)));
}
inline void scale8(float a, float* y, int D) {
  const __m256 va = _mm256_set1_ps(a);
  for (int d = 0; d < D; d += 8) _mm256_storeu_ps(y + d, _mm256_mul_ps(va, _mm256_loadu_ps(y + d)));
}

struct View {  // layout of sd_oracle.cpp's orc_kv_view
  int32_t bits, dtype, group_size, cap, D;
  const void* data;
  const void* scales;
  const void* biases;
};

// n rows of (bh, t0..t0+n) as floats into out[n][D].
void load_rows(const View* v, int64_t bh, int64_t t0, int n, float* out) {
  const int D = v->D;
  if (v->bits == 0) {
    const int64_t base = (bh * v->cap + t0) * D;
    if (v->dtype == F32) {
      std::memcpy(out, static_cast<const float*>(v->data) + base, sizeof(float) * size_t(n) * D);
    } else if (v->dtype == BF16) {
      const uint16_t* s = static_cast<const uint16_t*>(v->data) + base;
      for (int64_t i = 0; i < int64_t(n) * D; i += 8) {
        const __m128i h = _mm_loadu_si128(reinterpret_cast<const __m128i*>(s + i));
        _mm256_storeu_ps(out + i, _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_cvtepu16_epi32(h), 16)));
      }
    } else {
      const uint16_t* s = static_cast<const uint16_t*>(v->data) + base;
      for (int64_t i = 0; i < int64_t(n) * D; i += 8)
        _mm256_storeu_ps(out + i, _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(s + i))));
    }
    return;
  }
  const int bits = v->bits, gs = v->group_size, ng = D / gs;
  const int per_word = 32 / bits, words = D / per_word;
  const uint32_t mask = (1u << bits) - 1u;
  for (int r = 0; r < n; ++r) {
    const int64_t row = bh * v->cap + t0 + r;
    const uint32_t* wq = static_cast<const uint32_t*>(v->data) + row * words;
    float* o = out + int64_t(r) * D;
    for (int g = 0; g < ng; ++g) {
      const float s = ld(v->scales, v->dtype, row * ng + g), b = ld(v->biases, v->dtype, row * ng + g);
      for (int d = g * gs; d < (g + 1) * gs; ++d) {
        const float code = float((wq[d / per_word] >> (bits * (d % per_word))) & mask);
        o[d] = std::fma(s, code, b);
      }
    }
  }
}

}  // namespace

extern "C" {

void orc_base_set_threads(int n) {
  if (n < 1) n = int(std::max(1u, std::thread::hardware_concurrency()));
  if (n != pool().size()) pool().resize(n);
}

int orc_base_last_threads(void) { return g_last_threads; }

// fp32 decode of one layer: q [B, Hq, D] (qdtype); K, V caches (View);
// summaries [B*Hkv, nb_stride, D] (sdtype); out [B, Hq, D] (qdtype); sel_out
// [B*Hkv, n_sel] or null. Returns n_sel = min(k, NB-1) + 1.
int orc_base_decode(const void* q, int qdtype, const View* K, const View* V, const void* summ, int sdtype,
                    int nb_stride, int B, int Hq, int Hkv, int T, int S, int k, float scale, void* out,
                    int32_t* sel_out) {
  const int G = Hq / Hkv, D = K->D;
  const int NB = (T + S - 1) / S;
  const int64_t BH = int64_t(B) * Hkv;
  const int n_sel = std::min(k, NB - 1) + 1;
  const int E = sdtype == F32 ? 4 : 8, nc = D / E;
  constexpr int RUN = 512;
  const int nrun = (NB + RUN - 1) / RUN;
  std::vector<float> qsum(size_t(BH) * D);
  for (int64_t bh = 0; bh < BH; ++bh) {
    const int64_t b = bh / Hkv, h = bh % Hkv;
    for (int d = 0; d < D; ++d) {
      float a = ld(q, qdtype, (b * Hq + h * G) * D + d);
      for (int g = 1; g < G; ++g) a = a + ld(q, qdtype, (b * Hq + h * G + g) * D + d);
      qsum[size_t(bh) * D + d] = a;
    }
  }
  std::vector<float> scores(size_t(BH) * NB);
  int used = pool().run(BH * nrun, [&](int64_t task) {
    const int64_t bh = task / nrun;
    const int j0 = int(task % nrun) * RUN, j1 = std::min(NB, j0 + RUN);
    const float* qs = qsum.data() + size_t(bh) * D;
    float part[64];
    for (int j = j0; j < j1; ++j) {
      const int64_t base = (bh * nb_stride + j) * D;
      for (int c = 0; c < nc; ++c) {
        float a = 0.0f;
        for (int e = 0; e < E; ++e) a = std::fma(qs[c * E + e], ld(summ, sdtype, base + c * E + e), a);
        part[c] = a;
      }
      for (int off = nc / 2; off >= 1; off /= 2)
        for (int c = 0; c < off; ++c) part[c] = part[c] + part[c + off];
      scores[size_t(bh) * NB + j] = part[0] * scale;
    }
  });
  // selection: per group, top-k of the candidates, ascending, then the recent block
  std::vector<int32_t> sel(size_t(BH) * n_sel);
  used = std::max(used, pool().run(BH, [&](int64_t bh) {
    const int n = NB - 1;
    std::vector<uint64_t> key(size_t(std::max(n, 1)));
    for (int j = 0; j < n; ++j)
      key[size_t(j)] = (uint64_t(score_key(scores[size_t(bh) * NB + j])) << 32) | uint64_t(0xffffffffu - uint32_t(j));
    const int m = std::min(k, n);
    if (m > 0 && m < n) std::nth_element(key.begin(), key.begin() + m, key.begin() + n, std::greater<uint64_t>());
    int32_t* s = sel.data() + size_t(bh) * n_sel;
    for (int i = 0; i < m; ++i) s[i] = int32_t(0xffffffffu - uint32_t(key[size_t(i)]));
    std::sort(s, s + m);
    s[m] = NB - 1;
  }));
  // attention: one task per (group, selected block) -> partial (m, l, o) per head
  const int64_t ntask = BH * n_sel;
  const int PS = 2 * G + G * D;
  std::vector<float> part(size_t(ntask) * PS);
  used = std::max(used, pool().run(ntask, [&](int64_t task) {
    const int64_t bh = task / n_sel, b = bh / Hkv, h = bh % Hkv;
    const int j = sel[size_t(task)];
    const int t0 = j * S, n = std::min((j + 1) * S, T) - t0;
    thread_local std::vector<float> kt, vt, qv, sc;
    kt.resize(size_t(S) * D);
    vt.resize(size_t(S) * D);
    qv.resize(size_t(G) * D);
    sc.resize(size_t(S));
    load_rows(K, bh, t0, n, kt.data());
    load_rows(V, bh, t0, n, vt.data());
    float* P = part.data() + size_t(task) * PS;
    for (int g = 0; g < G; ++g) {
      for (int d = 0; d < D; ++d) qv[size_t(g) * D + d] = ld(q, qdtype, (b * Hq + h * G + g) * D + d) * scale;
      float mx = -INFINITY;
      for (int t = 0; t < n; ++t) {
        sc[size_t(t)] = dot8(qv.data() + size_t(g) * D, kt.data() + size_t(t) * D, D);
        mx = std::max(mx, sc[size_t(t)]);
      }
      float* o = P + 2 * G + g * D;
      std::fill(o, o + D, 0.0f);
      float l = 0.0f;
      for (int t = 0; t < n; ++t) {
        const float p = std::exp(sc[size_t(t)] - mx);
        l += p;
        axpy8(p, vt.data() + size_t(t) * D, o, D);
      }
      P[g] = mx;
      P[G + g] = l;
    }
  }));
  // merge the block partials of each (group, head) in block order
  used = std::max(used, pool().run(BH * G, [&](int64_t t) {
    const int64_t bh = t / G, g = t % G, b = bh / Hkv, h = bh % Hkv;
    float M = -INFINITY;
    for (int i = 0; i < n_sel; ++i) M = std::max(M, part[size_t(bh * n_sel + i) * PS + g]);
    thread_local std::vector<float> acc;
    acc.assign(size_t(D), 0.0f);
    float L = 0.0f;
    for (int i = 0; i < n_sel; ++i) {
      const float* P = part.data() + size_t(bh * n_sel + i) * PS;
      const float f = std::exp(P[g] - M);
      L += P[G + g] * f;
      axpy8(f, P + 2 * G + g * D, acc.data(), D);
    }
    scale8(1.0f / L, acc.data(), D);
    for (int d = 0; d < D; ++d) st(out, qdtype, (b * Hq + h * G + g) * D + d, acc[size_t(d)]);
  }));
  g_last_threads = used;
  if (sel_out) std::memcpy(sel_out, sel.data(), sel.size() * sizeof(int32_t));
  return n_sel;
}

}  // extern "C"
