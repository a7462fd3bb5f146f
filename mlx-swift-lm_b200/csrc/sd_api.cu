// sd_api.cu -- the C ABI (include/sparse_decode.h): index lifetime, cache
// writes, decode launches and the sharded decode steps. Host code only; the
// kernels live in sd_decode.cuh / sd_update.cuh, instantiated by sd_inst.cu.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/sparse_decode.h"
#include "sd_format.h"
#include "sd_kernels.h"
#include "sd_params.h"

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

#define SD_CUDA(call)                                                                              \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess) return fail(SD_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                       __FILE__, __LINE__);                                        \
  } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int elt_size(int dtype) { return dtype == SD_F32 ? 4 : 2; }

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

sd::KernelSet lookup(int dtype, int bits, int D, int G) {
  const int key = dtype * 16 + bits;
  switch (key) {
    case 0 * 16 + 0: return sd::kernels_e0_b0(D, G);
    case 1 * 16 + 0: return sd::kernels_e1_b0(D, G);
    case 2 * 16 + 0: return sd::kernels_e2_b0(D, G);
    case 0 * 16 + 4: return sd::kernels_e0_b4(D, G);
    case 1 * 16 + 4: return sd::kernels_e1_b4(D, G);
    case 2 * 16 + 4: return sd::kernels_e2_b4(D, G);
    case 0 * 16 + 8: return sd::kernels_e0_b8(D, G);
    case 1 * 16 + 8: return sd::kernels_e1_b8(D, G);
    case 2 * 16 + 8: return sd::kernels_e2_b8(D, G);
    default: return sd::KernelSet{nullptr, nullptr, nullptr, nullptr};
  }
}

// Last index whose work was launched on each stream: a decode that overlaps
// its predecessor may read its own index state early only when that
// predecessor belongs to another index.
std::mutex g_stream_mu;
std::unordered_map<cudaStream_t, const void*> g_stream_last;

bool note_stream(cudaStream_t st, const void* idx) {
  std::lock_guard<std::mutex> lk(g_stream_mu);
  auto it = g_stream_last.find(st);
  const bool other = it == g_stream_last.end() || it->second != idx;
  g_stream_last[st] = idx;
  return other;
}

void forget_index(const void* idx) {
  std::lock_guard<std::mutex> lk(g_stream_mu);
  for (auto it = g_stream_last.begin(); it != g_stream_last.end();)
    it = it->second == idx ? g_stream_last.erase(it) : std::next(it);
}

}  // namespace

struct sd_index {
  sd_config cfg;
  int device;
  int G, groups, esize, row_bytes;
  int64_t cap_global, nb_global;
  int64_t cap_local, nb_local;
  int64_t offset;
  int C, R;             // cluster size and replica clusters per (b, kv-head)
  size_t smem;
  void* arena;
  size_t arena_bytes;
  void *k_data, *v_data, *k_scales, *k_biases, *v_scales, *v_biases, *summ;
  unsigned long long* gslot;  // C*R > 1: the group merge's message words
  uint32_t* gep;        // C*R > 1: epoch of each group's last merged launch
  int mt;               // sliced selection: list length per CTA (0: the index never slices)
  unsigned long long* clist;  // sliced selection, C*R > 1: [BH][C*R][mt][2] message words
  unsigned long long* cfall;  // ... and [BH][C*R][top_k][2] for the full lists
  float* racc;          // 2 x [BH, D] running sums of the recent block's rows
  int racc_cur;         // buffer holding the current sums
  bool racc_valid;      // the current buffer matches the cache
  bool racc_undo;       // the other buffer holds the sums before the last single-token append
  int* d_err;
  int overlap;          // launch decodes with programmatic stream serialization
  const float* sinks;   // [Hq] attention-sink logits (device), or null
  CUtensorMap tmK, tmV, tmS;
  int sb_fused;         // tmS covers the four scale/bias arrays
  int lt;               // tokens per staged copy
  int kv_fused;         // tmK covers V too (4-D)
  sd::KernelSet ks;
  bool attrs_set;
  unsigned long long* dbg;  // phase-timing build: stamp buffer of the decode launches
  int l2_plain;  // phase-timing build: 1 drops the L2 evict_first hint (comparison runs)
};

// Exchange area of one shard for the fused sharded step (sd_shard_decode);
// the layout is described with DecodeParams::peer.
struct sd_comm {
  int device;
  int P, pr, BH, K, C, R, G, D, RS;
  int resident;                     // every cluster of a launch fits on the GPU at once
  size_t bytes;
  int64_t off_cand, off_part, off_ctl, off_clst;
  int MP;                           // sliced selection: keys per CTA list across the shards (0: unused)
  uint8_t* local;
  uint8_t* peers[sd::kMaxShards];   // own area at [pr]
  bool opened;
  bool ipc[sd::kMaxShards];         // peers[r] was opened from an IPC handle
  uint64_t wait_ns;                 // bound of the kernel's waits for other shards
};

namespace {

int32_t validate(const sd_config* c) {
  if (!c) return fail(SD_ERR_INVALID_ARG, "config is NULL");
  if (c->batch < 1 || c->n_q_heads < 1 || c->n_kv_heads < 1 || c->capacity < 1)
    return fail(SD_ERR_INVALID_ARG, "batch, n_q_heads, n_kv_heads and capacity must be positive");
  if (c->n_q_heads % c->n_kv_heads != 0)
    return fail(SD_ERR_SHAPE, "n_q_heads (%d) is not a multiple of n_kv_heads (%d)", c->n_q_heads, c->n_kv_heads);
  const int G = c->n_q_heads / c->n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return fail(SD_ERR_SHAPE, "query heads per kv head must be 1, 2, 4 or 8 (got %d)", G);
  if (c->head_dim != 64 && c->head_dim != 128) return fail(SD_ERR_SHAPE, "head_dim must be 64 or 128 (got %d)", c->head_dim);
  if (c->block_size != 32 && c->block_size != 64 && c->block_size != 128 && c->block_size != 256)
    return fail(SD_ERR_SHAPE, "block_size must be 32, 64, 128 or 256 (got %d)", c->block_size);
  if (c->top_k < 0 || c->top_k > sd::kMaxTopK) return fail(SD_ERR_SHAPE, "top_k must be in [0, %d] (got %d)", sd::kMaxTopK, c->top_k);
  if (c->dtype != SD_F32 && c->dtype != SD_F16 && c->dtype != SD_BF16) return fail(SD_ERR_INVALID_ARG, "unknown dtype %d", c->dtype);
  if (c->kv_bits != 0 && c->kv_bits != 4 && c->kv_bits != 8) return fail(SD_ERR_SHAPE, "kv_bits must be 0, 4 or 8 (got %d)", c->kv_bits);
  if (c->kv_bits != 0 && c->group_size != 64) return fail(SD_ERR_SHAPE, "group_size must be 64 for quantized caches (got %d)", c->group_size);
  if (c->shard_count < 1 || c->shard_count > 64) return fail(SD_ERR_INVALID_ARG, "shard_count must be in [1, 64]");
  if (c->shard_rank < 0 || c->shard_rank >= c->shard_count) return fail(SD_ERR_INVALID_ARG, "shard_rank out of range");
  if (c->cluster_size < 0 || c->cluster_size > 16)
    return fail(SD_ERR_INVALID_ARG, "cluster_size must be in [0, 16]");
  for (int r : c->reserved)
    if (r != 0) return fail(SD_ERR_INVALID_ARG, "reserved config fields must be 0");
  if (c->shard_count * c->top_k > sd::kUnionMax)
    return fail(SD_ERR_SHAPE, "shard_count * top_k must be <= %d", sd::kUnionMax);
  return SD_OK;
}

// The K or V arena as a 3-D byte tensor (column box, row, box index): a row
// of row_bytes is cut into boxes of min(row_bytes, 128) bytes, the widest the
// swizzle allows, and one copy moves a whole tile of kTileTokens rows with all
// its boxes, landing as [box][row][box bytes] in shared memory. One TMA
// operation per tile rather than one per box: the SM's TMA unit spends a fixed
// time on each operation, which dominates copies of a few KB.
int32_t encode_map(CUtensorMap* map, void* base, int row_bytes, int64_t rows, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SD_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int box_bytes = std::min(row_bytes, 128);
  const int nbox = row_bytes / box_bytes;
  CUtensorMapSwizzle sw = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_32B;
  cuuint64_t dims[3] = {cuuint64_t(box_bytes), cuuint64_t(rows), cuuint64_t(nbox)};
  cuuint64_t strides[2] = {cuuint64_t(row_bytes), cuuint64_t(box_bytes)};
  cuuint32_t box[3] = {cuuint32_t(box_bytes), cuuint32_t(box_rows), cuuint32_t(nbox)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return SD_OK;
}

// K and V as one 4-D byte tensor (column box, row, box index, K/V) when V
// starts a positive multiple of 16 bytes after K: one copy moves a stage's K
// rows and then its V rows, landing as [K|V][box][row][box bytes] -- what the
// consumers expect with V box_rows * row_bytes after K. False if the layout
// or the encoder does not allow it.
bool encode_kv_map(CUtensorMap* map, void* k, void* v, int row_bytes, int64_t rows, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  const intptr_t dist = reinterpret_cast<intptr_t>(v) - reinterpret_cast<intptr_t>(k);
  if (!fn || dist <= 0 || dist % 16 != 0 || dist >= (intptr_t(1) << 40)) return false;
  const int box_bytes = std::min(row_bytes, 128);
  const int nbox = row_bytes / box_bytes;
  CUtensorMapSwizzle sw = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_32B;
  cuuint64_t dims[4] = {cuuint64_t(box_bytes), cuuint64_t(rows), cuuint64_t(nbox), 2};
  cuuint64_t strides[3] = {cuuint64_t(row_bytes), cuuint64_t(box_bytes), cuuint64_t(dist)};
  cuuint32_t box[4] = {cuuint32_t(box_bytes), cuuint32_t(box_rows), cuuint32_t(nbox), 2};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, k, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tokens per staged copy for a format (Fmt::kLoadTokens), or 32 when blocks
// hold 32 tokens.
int load_tokens(const sd_config& c) {
  const int lt = (c.kv_bits && elt_size(c.dtype) == 2) ? 64 : sd::kTileTokens;
  return std::min(lt, c.block_size);
}

// The four scale/bias arrays of a quantized index (k_scales, k_biases,
// v_scales, v_biases, each `bytes` long, one every `stride` bytes) as a 2-D
// byte tensor: one copy moves the tile's four pieces of tile_bytes, stacked
// as the kernel's stage expects. The byte coordinate is a signed 32-bit
// number, so arrays of 2 GiB or more keep the 1-D bulk copies.
bool encode_sb_map(CUtensorMap* map, void* base, size_t stride, size_t bytes, int tile_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || stride % 16 != 0 || bytes >= (size_t(1) << 31) || tile_bytes % 16 != 0 || tile_bytes > 256) return false;
  cuuint64_t dims[2] = {cuuint64_t(bytes), 4};
  cuuint64_t strides[1] = {cuuint64_t(stride)};
  cuuint32_t box[2] = {cuuint32_t(tile_bytes), 4};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Number of clusters of size C the device can hold at once (0 = not launchable).
int max_active_clusters(const sd_index* x, int C) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(C), unsigned(x->cfg.batch * x->cfg.n_kv_heads), 1);
  cfg.blockDim = dim3(sd::kThreads, 1, 1);
  cfg.dynamicSmemBytes = x->smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, x->ks.decode, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Candidate blocks of the largest shard (rank 0) when the cache is full: the
// same on every shard, so every shard of a sequence picks the same launch
// shape and selection path.
int64_t max_local_candidates(const sd_index* x) {
  const sd_config& c = x->cfg;
  const int64_t ncand = x->nb_global - 1;
  return ncand > 0 ? (ncand + c.shard_count - 1) / c.shard_count : 0;
}

// Whether a launch with nloc candidate blocks per group takes the sliced
// selection (see decode_kernel): more than kAllKeysMax candidates, K > 128,
// or several CTAs per group that are not one cluster.
bool sliced_launch(const sd_index* x, int64_t nloc) {
  return x->cfg.top_k > 128 || nloc > sd::kAllKeysMax || (x->C == 1 && x->R > 1);
}

// Length of each CTA's list in the sliced selection with Q CTAs per group:
// about four times a CTA's share of the top-K (at least 32, at most K), so
// that the lists hold the group's top-K unless one share is very uneven (then
// the kernel falls back to full lists); Q * mt <= 4096 (the kernel's buffer).
int list_len(int K, int Q) {
  if (K <= 0) return 0;
  int m = 4 * ((K + Q - 1) / Q);
  m = std::max(32, (m + 31) / 32 * 32);
  m = std::min(m, K);
  return std::max(1, std::min(m, 4096 / Q));
}

// CTAs of a group (of Q) that own a slice of the output in the group merge:
// about one per 128 outputs, and enough that an owner's Q records fit one
// batch of loads (8 words per thread of the decode kernel).
int merge_owners(int Q, int G, int D) {
  if (Q <= 1) return 1;
  const int GD = G * D;
  int n = std::max(1, (GD + 127) / 128);
  while (n < Q && int64_t(Q) * (2 * G + (GD + n - 1) / n) > 8 * sd::kThreads) ++n;
  return std::min(n, Q);
}

// Words of one merge record: the (m, l) of every head, then an owner's slice.
int merge_record(int Q, int G, int D) {
  const int no = merge_owners(Q, G, D);
  return 2 * G + (G * D + no - 1) / no;
}

int32_t setup_kernels(sd_index* x) {
  if (x->attrs_set) return SD_OK;
  SD_CUDA(cudaFuncSetAttribute(x->ks.decode, cudaFuncAttributeMaxDynamicSharedMemorySize, int(x->smem)));
  SD_CUDA(cudaFuncSetAttribute(x->ks.decode, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  x->attrs_set = true;
  return SD_OK;
}

// Choose the cluster size (CTAs per (batch, kv-head)). Automatic choice: the
// largest C <= 16 for which every group's cluster is resident at once (one
// wave: a cluster must fit in one GPC, so with one CTA per SM a B200 holds 7
// clusters of 16 but 8 of 10), with B*Hkv*C <= SMs, C*top_k within the union
// buffer and at most kLocalKeysMax candidate blocks per CTA at full capacity.
int32_t choose_cluster(sd_index* x) {
  const sd_config& c = x->cfg;
  const int64_t BH = int64_t(c.batch) * c.n_kv_heads;
  int n_sm = 148;
  cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, x->device);
  auto fits = [&](int C) {
    return int64_t(C) * c.top_k <= sd::kUnionMax && (x->nb_local + C - 1) / C <= sd::kLocalKeysMax;
  };
  if (c.cluster_size != 0) {
    if (!fits(c.cluster_size))
      return fail(SD_ERR_SHAPE, "cluster_size %d is too small for this capacity or top_k", c.cluster_size);
    x->C = c.cluster_size;
    x->R = 1;
    if (max_active_clusters(x, x->C) < 1)
      return fail(SD_ERR_SHAPE, "cluster size %d cannot be scheduled with %zu bytes of shared memory", x->C, x->smem);
    return SD_OK;
  }
  // Sliced selection at full capacity (K > 128 or more than kAllKeysMax
  // candidates per group): single-CTA "clusters", Q = R CTAs per group, as
  // many as the SMs hold at once (one CTA per SM) -- every CTA scores 1/Q of
  // the candidates and attends 1/Q of the tiles; Q * K stays within the
  // kernel's union buffer.
  if (c.top_k > 128 || max_local_candidates(x) > sd::kAllKeysMax) {
    int Q = int(std::min<int64_t>(sd::kMaxGroupCtas, std::max<int64_t>(1, n_sm / BH)));
    if (c.top_k > 0) Q = std::min(Q, std::max(1, sd::kUnionMax / c.top_k));
    const int mac = max_active_clusters(x, 1);
    while (Q > 1 && mac < BH * Q) --Q;
    if (mac < 1) return fail(SD_ERR_SHAPE, "the decode kernel cannot be scheduled with %zu bytes of shared memory", x->smem);
    x->C = 1;
    x->R = Q;
    return SD_OK;
  }
  // Replicas (R <= 4 clusters per group, each attending 1/R of the tiles)
  // raise the number of CTAs that pull from HBM: pick the largest
  // B*Hkv*C*R <= SMs whose clusters are all resident at once, larger C first.
  int best_c = 0, best_r = 0;
  for (int C = 16; C >= 1; --C) {
    if (!fits(C)) continue;
    const int mac = max_active_clusters(x, C);
    for (int R = 1; R <= 4; ++R) {
      if (BH * C * R > n_sm || mac < BH * R) break;
      if (C * R > best_c * best_r) { best_c = C; best_r = R; }
    }
  }
  if (best_c) {
    x->C = best_c;
    x->R = best_r;
    return SD_OK;
  }
  // More groups than the GPU holds at once: the smallest feasible cluster.
  for (int C = 1; C <= 16; ++C)
    if (fits(C) && max_active_clusters(x, C) >= 1) {
      x->C = C;
      x->R = 1;
      return SD_OK;
    }
  return fail(SD_ERR_SHAPE, "no schedulable cluster size for this configuration");
}

int32_t launch_decode(sd_index* x, int mode, int T, const void* q, const void* k_new, const void* v_new,
                      float scale, void* out, int32_t* sel_out, float* scores_out, float* cand_score,
                      int32_t* cand_block, float* part_ml, float* part_o, cudaStream_t st,
                      const sd_comm* comm = nullptr) {
  const sd_config& c = x->cfg;
  sd::DecodeParams p{};
  p.B = c.batch; p.Hq = c.n_q_heads; p.Hkv = c.n_kv_heads; p.S = c.block_size; p.K = c.top_k;
  p.T = T;
  p.NB = (T + c.block_size - 1) / c.block_size;
  p.P = c.shard_count; p.pr = c.shard_rank;
  p.cap_local = int(x->cap_local);
  p.nb_stride = int(x->nb_local);
  p.C = x->C;
  p.mode = mode;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = q; p.k_new = k_new; p.v_new = v_new;
  p.k_data = x->k_data; p.v_data = x->v_data;
  p.k_scales = x->k_scales; p.k_biases = x->k_biases; p.v_scales = x->v_scales; p.v_biases = x->v_biases;
  p.summ = x->summ;
  p.out = out; p.sel_out = sel_out; p.scores_out = scores_out;
  p.cand_score = cand_score; p.cand_block = cand_block; p.part_ml = part_ml; p.part_o = part_o;
  p.err = x->d_err;
  {
    const int64_t BHD = int64_t(c.batch) * c.n_kv_heads * c.head_dim;
    p.racc_in = x->racc + int64_t(x->racc_cur) * BHD;
    p.racc_out = x->racc + int64_t(1 - x->racc_cur) * BHD;
    p.racc_rebuild = x->racc_valid ? 0 : 1;
  }
  p.R = x->R;
  p.nown = merge_owners(x->C * x->R, x->G, c.head_dim);
  p.sinks = x->sinks;
  p.gslot = x->gslot;
  p.gep = x->gep;
  const bool other_before = note_stream(st, x);
  // Peer mode overlaps too: the kernel reads the launch epoch and touches
  // the exchange areas only after its grid-dependency wait, and a shard's
  // launch finishes only once every CTA of every other shard has read this
  // launch's lists (the shards' records it waits for come after them).
  const bool overlap = x->overlap != 0;
  p.pdl_early = (overlap && other_before) ? 1 : 0;
  if (mode == sd::MODE_PEER) {
    for (int r = 0; r < comm->P; ++r) p.peer[r] = comm->peers[r];
    p.x_cand = comm->off_cand;
    p.x_clst = comm->off_clst;
    p.mtp = comm->MP;
    p.x_part = comm->off_part;
    p.x_ctl = comm->off_ctl;
    p.peer_wait_ns = comm->wait_ns;
  }
  const int64_t ncand = p.NB - 1;
  const int64_t nloc = ncand > p.pr ? (ncand - p.pr + p.P - 1) / p.P : 0;
  p.sliced = sliced_launch(x, nloc) ? 1 : 0;
  // The one-level exchange across the shards needs every shard on the sliced
  // path: the shard with the fewest candidates (the last) decides, the same
  // answer on every shard.
  if (mode == sd::MODE_PEER) {
    const int64_t nmin = ncand > p.P - 1 ? (ncand - (p.P - 1) + p.P - 1) / p.P : 0;
    if (!sliced_launch(x, nmin)) p.mtp = 0;
  }
  const int64_t chunks = p.sliced ? int64_t(x->C) * x->R : x->C;
  if ((nloc + chunks - 1) / chunks > sd::kLocalKeysMax)
    return fail(SD_ERR_SHAPE, "too many blocks per CTA (%lld) for %lld CTAs per group",
                (long long)((nloc + chunks - 1) / chunks), (long long)chunks);
  if (p.sliced && x->C * x->R > 1 && c.top_k > 0 && mode != sd::MODE_ATTEND && (!x->clist || !x->cfall))
    return fail(SD_ERR_STATE, "index has no sliced-selection buffers");
  p.mt = x->mt;
  p.clist = x->clist;
  p.cfall = x->cfall;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(x->C * x->R), unsigned(c.batch * c.n_kv_heads), 1);
  cfg.blockDim = dim3(sd::kThreads, 1, 1);
  cfg.dynamicSmemBytes = x->smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(x->C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap ? 2 : 1;
  p.sb_fused = x->sb_fused;
  p.lt = x->lt;
  p.kv_fused = x->kv_fused;
  p.dbg = x->dbg;
  p.l2_plain = x->l2_plain;
  void* args[4] = {&p, &x->tmK, &x->tmV, &x->tmS};
  SD_CUDA(cudaLaunchKernelExC(&cfg, x->ks.decode, args));
  return SD_OK;
}

int32_t launch_summaries(sd_index* x, int64_t jl0, int64_t jl1, int64_t T, cudaStream_t st) {
  if (jl1 <= jl0) return SD_OK;
  const sd_config& c = x->cfg;
  sd::SummaryParams sp{};
  sp.Hkv = c.n_kv_heads; sp.S = c.block_size; sp.P = c.shard_count; sp.pr = c.shard_rank;
  sp.cap_local = int(x->cap_local); sp.nb_stride = int(x->nb_local);
  sp.T = int(T);
  sp.jl0 = int(jl0);
  sp.k_data = x->k_data; sp.k_scales = x->k_scales; sp.k_biases = x->k_biases; sp.summ = x->summ;
  void* args[1] = {&sp};
  note_stream(st, x);
  SD_CUDA(cudaLaunchKernel(x->ks.summary, dim3(unsigned(jl1 - jl0), unsigned(c.batch * c.n_kv_heads)), dim3(128),
                           args, 0, st));
  return SD_OK;
}

// A single-token append went through a decode launch: the running sums
// moved to the other buffer; the old one still holds the sums before it.
void appended_one(sd_index* x) {
  // only the shard that stores the recent block keeps its sums
  const int64_t j = (x->offset - 1) / x->cfg.block_size;
  if ((j % x->cfg.shard_count) == x->cfg.shard_rank) {
    x->racc_cur = 1 - x->racc_cur;
    x->racc_valid = true;
    x->racc_undo = true;
  } else {
    x->racc_valid = false;
    x->racc_undo = false;
  }
}

// Local blocks [jl0, jl1) of this shard whose global index falls in [jg0, jg1].
void local_range(const sd_index* x, int64_t jg0, int64_t jg1, int64_t* jl0, int64_t* jl1) {
  const int64_t P = x->cfg.shard_count, pr = x->cfg.shard_rank;
  int64_t a = jg0 <= pr ? 0 : (jg0 - pr + P - 1) / P;
  int64_t b = jg1 < pr ? -1 : (jg1 - pr) / P;
  *jl0 = a;
  *jl1 = std::max(a, b + 1);
}

}  // namespace

extern "C" {

int32_t sd_abi_version(void) { return 1; }

const char* sd_status_string(int32_t s) {
  switch (s) {
    case SD_OK: return "SD_OK";
    case SD_ERR_INVALID_ARG: return "SD_ERR_INVALID_ARG";
    case SD_ERR_SHAPE: return "SD_ERR_SHAPE";
    case SD_ERR_CAPACITY: return "SD_ERR_CAPACITY";
    case SD_ERR_STATE: return "SD_ERR_STATE";
    case SD_ERR_CUDA: return "SD_ERR_CUDA";
    case SD_ERR_DEVICE: return "SD_ERR_DEVICE";
    default: return "SD_ERR_UNKNOWN";
  }
}

const char* sd_last_error(void) { return g_last_error.c_str(); }

int32_t sd_index_create(const sd_config* cfg, sd_index** out) {
  if (!out) return fail(SD_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  int32_t rc = validate(cfg);
  if (rc != SD_OK) return rc;
  const sd_config& c = *cfg;
  int device = 0;
  SD_CUDA(cudaGetDevice(&device));
  sd_index* x = new sd_index();
  x->cfg = c;
  x->device = device;
  x->G = c.n_q_heads / c.n_kv_heads;
  x->esize = elt_size(c.dtype);
  x->groups = c.kv_bits ? c.head_dim / 64 : 1;
  x->row_bytes = c.kv_bits ? c.head_dim * c.kv_bits / 8 : c.head_dim * x->esize;
  x->cap_global = (int64_t(c.capacity) + 255) / 256 * 256;
  x->nb_global = x->cap_global / c.block_size;
  x->nb_local = (x->nb_global + c.shard_count - 1) / c.shard_count;
  x->cap_local = x->nb_local * c.block_size;
  x->offset = 0;
  const int64_t BH = int64_t(c.batch) * c.n_kv_heads;
  if (BH * x->cap_local >= (int64_t(1) << 31) || BH > 65535) {
    delete x;
    return fail(SD_ERR_SHAPE, "cache too large: batch*kv_heads*capacity rows must stay below 2^31");
  }
  x->ks = lookup(c.dtype, c.kv_bits, c.head_dim, x->G);
  if (!x->ks.decode) {
    const int G = x->G;
    delete x;
    return fail(SD_ERR_SHAPE, "no kernel for dtype %d, bits %d, head_dim %d, G %d", c.dtype, c.kv_bits, c.head_dim, G);
  }
  const sd::Layout L = sd::make_layout(c.head_dim, x->G, x->groups);
  x->smem = size_t(L.total) + 1024;
  rc = setup_kernels(x);
  if (rc == SD_OK) rc = choose_cluster(x);
  if (rc != SD_OK) {
    delete x;
    return rc;
  }

  const size_t kv = align256(size_t(BH) * x->cap_local * x->row_bytes);
  const size_t sb = c.kv_bits ? align256(size_t(BH) * x->cap_local * x->groups * x->esize) : 0;
  const size_t su = align256(size_t(BH) * x->nb_local * c.head_dim * x->esize);
  const int Q = x->C * x->R;
  const size_t rp =
      Q > 1 ? align256(size_t(BH) * merge_owners(Q, x->G, c.head_dim) * Q * merge_record(Q, x->G, c.head_dim) * 8) : 0;
  const size_t rcn = Q > 1 ? align256(size_t(BH) * 4) : 0;
  const size_t ra = align256(size_t(2) * BH * c.head_dim * 4);
  const bool slices = Q > 1 && (c.top_k > 128 || max_local_candidates(x) > sd::kAllKeysMax || x->C == 1);
  x->mt = slices ? list_len(c.top_k, Q) : 0;
  const size_t cl = slices ? align256(size_t(BH) * Q * x->mt * 2 * 8) : 0;
  const size_t cf = slices ? align256(size_t(BH) * Q * c.top_k * 2 * 8) : 0;
  x->arena_bytes = 2 * kv + 4 * sb + su + rp + rcn + cl + cf + ra + 256;
  cudaError_t e = cudaMalloc(&x->arena, x->arena_bytes);
  if (e != cudaSuccess) {
    const size_t bytes = x->arena_bytes;
    delete x;
    return fail(SD_ERR_CUDA, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
  }
  uint8_t* a = static_cast<uint8_t*>(x->arena);
  x->k_data = a; a += kv;
  x->v_data = a; a += kv;
  if (c.kv_bits) {
    x->k_scales = a; a += sb;
    x->k_biases = a; a += sb;
    x->v_scales = a; a += sb;
    x->v_biases = a; a += sb;
  }
  x->summ = a; a += su;
  x->gslot = rp ? reinterpret_cast<unsigned long long*>(a) : nullptr; a += rp;
  x->gep = rcn ? reinterpret_cast<uint32_t*>(a) : nullptr; a += rcn;
  x->clist = cl ? reinterpret_cast<unsigned long long*>(a) : nullptr; a += cl;
  x->cfall = cf ? reinterpret_cast<unsigned long long*>(a) : nullptr; a += cf;
  x->racc = reinterpret_cast<float*>(a); a += ra;
  x->d_err = reinterpret_cast<int*>(a);
  e = cudaMemset(x->arena, 0, x->arena_bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(x->arena);
    delete x;
    return fail(SD_ERR_CUDA, "cudaMemset failed: %s", cudaGetErrorString(e));
  }
  // One copy per tile for the four scale/bias pieces: the arena keeps the
  // four arrays sb bytes apart.
  std::memset(&x->tmS, 0, sizeof(x->tmS));
  x->lt = load_tokens(c);
  x->sb_fused = c.kv_bits && encode_sb_map(&x->tmS, x->k_scales, sb, size_t(BH) * x->cap_local * x->groups * x->esize,
                                           x->lt * x->groups * x->esize) ? 1 : 0;
  rc = SD_OK;
  x->kv_fused = encode_kv_map(&x->tmK, x->k_data, x->v_data, x->row_bytes, BH * x->cap_local, x->lt) ? 1 : 0;
  if (!x->kv_fused) {
    rc = encode_map(&x->tmK, x->k_data, x->row_bytes, BH * x->cap_local, x->lt);
    if (rc == SD_OK) rc = encode_map(&x->tmV, x->v_data, x->row_bytes, BH * x->cap_local, x->lt);
  }
  if (rc != SD_OK) {
    cudaFree(x->arena);
    delete x;
    return rc;
  }
  *out = x;
  return SD_OK;
}

int32_t sd_index_destroy(sd_index* x) {
  if (!x) return SD_OK;
  forget_index(x);
  cudaError_t e = cudaFree(x->arena);
  delete x;
  if (e != cudaSuccess) return fail(SD_ERR_CUDA, "cudaFree failed: %s", cudaGetErrorString(e));
  return SD_OK;
}

int32_t sd_index_config(const sd_index* x, sd_config* out) {
  if (!x || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  *out = x->cfg;
  out->cluster_size = x->C;
  return SD_OK;
}

int32_t sd_index_arrays(const sd_index* x, sd_arrays* out) {
  if (!x || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  std::memset(out, 0, sizeof(*out));
  out->k_data = x->k_data; out->v_data = x->v_data;
  out->k_scales = x->k_scales; out->k_biases = x->k_biases; out->v_scales = x->v_scales; out->v_biases = x->v_biases;
  out->summaries = x->summ;
  out->cap_local = x->cap_local;
  out->nb_local = x->nb_local;
  out->row_bytes = x->row_bytes;
  out->cluster_size = x->C;
  out->replicas = x->R;
  out->smem_bytes = int32_t(x->smem);
  return SD_OK;
}

int32_t sd_index_offset(const sd_index* x, int64_t* offset) {
  if (!x || !offset) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  *offset = x->offset;
  return SD_OK;
}

int32_t sd_index_copy(const sd_index* src, sd_index** out, sd_stream stream) {
  if (!src || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  int32_t rc = sd_index_create(&src->cfg, out);
  if (rc != SD_OK) return rc;
  sd_index* x = *out;
  SD_CUDA(cudaMemcpyAsync(x->arena, src->arena, src->arena_bytes - 256, cudaMemcpyDeviceToDevice,
                          static_cast<cudaStream_t>(stream)));
  x->offset = src->offset;
  x->racc_cur = src->racc_cur;
  x->racc_valid = src->racc_valid;
  x->racc_undo = src->racc_undo;
  return SD_OK;
}

int32_t sd_append(sd_index* x, const void* keys, const void* values, int32_t n, sd_stream stream) {
  if (!x || !keys || !values) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  if (n < 0) return fail(SD_ERR_INVALID_ARG, "n_tokens must be >= 0");
  if (n == 0) return SD_OK;
  if (x->offset + n > x->cap_global)
    return fail(SD_ERR_CAPACITY, "append of %d tokens at offset %lld exceeds capacity %lld", n,
                (long long)x->offset, (long long)x->cap_global);
  const sd_config& c = x->cfg;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  sd::AppendParams ap{};
  ap.Hkv = c.n_kv_heads; ap.S = c.block_size; ap.P = c.shard_count; ap.pr = c.shard_rank;
  ap.cap_local = int(x->cap_local);
  ap.n_tok = n;
  ap.t0 = int(x->offset);
  ap.k_src = keys; ap.v_src = values;
  ap.k_data = x->k_data; ap.v_data = x->v_data;
  ap.k_scales = x->k_scales; ap.k_biases = x->k_biases; ap.v_scales = x->v_scales; ap.v_biases = x->v_biases;
  void* args[1] = {&ap};
  note_stream(st, x);
  SD_CUDA(cudaLaunchKernel(x->ks.append, dim3(unsigned((n + 3) / 4), unsigned(c.batch * c.n_kv_heads)), dim3(256),
                           args, 0, st));
  const int64_t T = x->offset + n;
  int64_t jl0, jl1;
  local_range(x, x->offset / c.block_size, (T - 1) / c.block_size, &jl0, &jl1);
  int32_t rc = launch_summaries(x, jl0, jl1, T, st);
  if (rc != SD_OK) return rc;
  x->offset = T;
  x->racc_valid = false;
  x->racc_undo = false;
  return SD_OK;
}

int32_t sd_trim(sd_index* x, int32_t n, int32_t* trimmed) {
  if (!x) return fail(SD_ERR_INVALID_ARG, "NULL index");
  if (n < 0) return fail(SD_ERR_INVALID_ARG, "n must be >= 0");
  const int64_t t = std::min<int64_t>(x->offset, n);
  if (t == 1 && x->racc_undo) {
    x->racc_cur = 1 - x->racc_cur;  // the sums before the last appended row
    x->racc_valid = true;
  } else if (t > 0) {
    x->racc_valid = false;
  }
  x->racc_undo = false;
  x->offset -= t;
  if (trimmed) *trimmed = int32_t(t);
  return SD_OK;
}

int32_t sd_set_offset(sd_index* x, int64_t offset) {
  if (!x) return fail(SD_ERR_INVALID_ARG, "NULL index");
  if (offset < 0 || offset > x->cap_global) return fail(SD_ERR_CAPACITY, "offset %lld out of range", (long long)offset);
  x->offset = offset;
  x->racc_valid = false;
  x->racc_undo = false;
  return SD_OK;
}

int32_t sd_rebuild_summaries(sd_index* x, sd_stream stream) {
  if (!x) return fail(SD_ERR_INVALID_ARG, "NULL index");
  if (x->offset == 0) return SD_OK;
  int64_t jl0, jl1;
  local_range(x, 0, (x->offset - 1) / x->cfg.block_size, &jl0, &jl1);
  return launch_summaries(x, jl0, jl1, x->offset, static_cast<cudaStream_t>(stream));
}

int32_t sd_decode(sd_index* x, const void* q, const void* k_new, const void* v_new, float scale, void* out,
                  int32_t* sel_out, float* scores_out, sd_stream stream) {
  if (!x || !q || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(SD_ERR_INVALID_ARG, "k_new and v_new must both be given or both NULL");
  if (x->cfg.shard_count != 1) return fail(SD_ERR_STATE, "sd_decode needs a single-shard index; use sd_shard_*");
  if (!std::isfinite(scale)) return fail(SD_ERR_INVALID_ARG, "scale must be finite");
  const int64_t T = x->offset + (k_new ? 1 : 0);
  if (T > x->cap_global) return fail(SD_ERR_CAPACITY, "decode append exceeds capacity %lld", (long long)x->cap_global);
  if (T < 1) return fail(SD_ERR_STATE, "decode on an empty cache");
  int32_t rc = launch_decode(x, sd::MODE_FUSED, int(T), q, k_new, v_new, scale, out, sel_out, scores_out, nullptr,
                             nullptr, nullptr, nullptr, static_cast<cudaStream_t>(stream));
  if (rc == SD_OK) {
    x->offset = T;
    if (k_new) appended_one(x);
  }
  return rc;
}

int32_t sd_shard_candidates(sd_index* x, const void* q, const void* k_new, const void* v_new, float scale,
                            float* cand_score, int32_t* cand_block, float* scores_out, sd_stream stream) {
  if (!x || !q || !cand_score || !cand_block) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(SD_ERR_INVALID_ARG, "k_new and v_new must both be given or both NULL");
  if (!std::isfinite(scale)) return fail(SD_ERR_INVALID_ARG, "scale must be finite");
  const int64_t T = x->offset + (k_new ? 1 : 0);
  if (T > x->cap_global) return fail(SD_ERR_CAPACITY, "decode append exceeds capacity %lld", (long long)x->cap_global);
  if (T < 1) return fail(SD_ERR_STATE, "decode on an empty cache");
  int32_t rc = launch_decode(x, sd::MODE_CANDIDATES, int(T), q, k_new, v_new, scale, nullptr, nullptr, scores_out,
                             cand_score, cand_block, nullptr, nullptr, static_cast<cudaStream_t>(stream));
  if (rc == SD_OK) {
    x->offset = T;
    if (k_new) appended_one(x);
  }
  return rc;
}

int32_t sd_shard_attend(sd_index* x, const void* q, const float* all_cand_score, const int32_t* all_cand_block,
                        float scale, float* part_ml, float* part_o, int32_t* sel_out, sd_stream stream) {
  if (!x || !q || !part_ml || !part_o) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  if (x->cfg.top_k > 0 && (!all_cand_score || !all_cand_block)) return fail(SD_ERR_INVALID_ARG, "NULL candidates");
  if (!std::isfinite(scale)) return fail(SD_ERR_INVALID_ARG, "scale must be finite");
  if (x->offset < 1) return fail(SD_ERR_STATE, "attend on an empty cache");
  return launch_decode(x, sd::MODE_ATTEND, int(x->offset), q, nullptr, nullptr, scale, nullptr, sel_out, nullptr,
                       const_cast<float*>(all_cand_score), const_cast<int32_t*>(all_cand_block), part_ml, part_o,
                       static_cast<cudaStream_t>(stream));
}

int32_t sd_shard_merge(sd_index* x, const float* all_ml, const float* all_o, void* out, sd_stream stream) {
  if (!x || !all_ml || !all_o || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  const sd_config& c = x->cfg;
  int P = c.shard_count, BQ = c.batch * c.n_q_heads, D = c.head_dim;
  int Hq = c.n_q_heads;
  const float* sinks = x->sinks;
  void* args[8] = {&P, &BQ, &D, const_cast<float**>(&all_ml), const_cast<float**>(&all_o), &out,
                   const_cast<float**>(&sinks), &Hq};
  SD_CUDA(cudaLaunchKernel(x->ks.merge, dim3(unsigned(BQ)), dim3(128), args, 0, static_cast<cudaStream_t>(stream)));
  return SD_OK;
}

namespace {
// Shards of one process on different GPUs: let this comm's device access
// every other shard's device (already-enabled access is fine).
int32_t enable_peer_access(const sd_comm* m, sd_comm* const* shards) {
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return fail(SD_ERR_CUDA, "cudaGetDevice failed");
  for (int r = 0; r < m->P; ++r) {
    const int d = shards[r]->device;
    if (d == m->device) continue;
    int ok = 0;
    cudaDeviceCanAccessPeer(&ok, m->device, d);
    if (!ok) return fail(SD_ERR_CUDA, "device %d cannot access device %d", m->device, d);
    cudaSetDevice(m->device);
    cudaError_t e = cudaDeviceEnablePeerAccess(d, 0);
    cudaSetDevice(cur);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();
    } else if (e != cudaSuccess) {
      return fail(SD_ERR_CUDA, "cudaDeviceEnablePeerAccess(%d -> %d): %s", m->device, d, cudaGetErrorString(e));
    }
  }
  return SD_OK;
}

struct CommHandle {
  cudaIpcMemHandle_t ipc;
  int32_t magic, version, P, pr, BH, K, C, R, G, D;
  uint64_t bytes;
};
static_assert(sizeof(CommHandle) <= SD_COMM_HANDLE_BYTES, "comm handle too large");
constexpr int32_t kCommMagic = 0x53444331;  // "SDC1"
}  // namespace

int32_t sd_comm_create(const sd_index* x, sd_comm** out) {
  if (!x || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  *out = nullptr;
  const sd_config& c = x->cfg;
  if (c.shard_count > sd::kMaxShards)
    return fail(SD_ERR_SHAPE, "peer exchange supports up to %d shards (got %d)", sd::kMaxShards, c.shard_count);
  sd_comm m{};
  m.device = x->device;
  m.P = c.shard_count; m.pr = c.shard_rank;
  m.BH = c.batch * c.n_kv_heads; m.K = c.top_k; m.C = x->C; m.R = x->R; m.G = x->G; m.D = c.head_dim;
  const int Q = m.C * m.R;
  const int NO = merge_owners(Q, m.G, m.D);
  m.RS = merge_record(Q, m.G, m.D);
  m.resident = max_active_clusters(x, x->C) >= int64_t(m.BH) * x->R ? 1 : 0;
  const int64_t P = m.P, BH = m.BH;
  // one-level selection across the shards (indexes that slice): lists of MP
  // keys, about four times a CTA's share of the top-K, P * Q * MP <= 8192
  m.MP = 0;
  if (c.top_k > 0 && (c.top_k > 128 || max_local_candidates(x) > sd::kAllKeysMax || (m.C == 1 && m.R > 1))) {
    int mp = 4 * ((c.top_k + int(P) * Q - 1) / (int(P) * Q));
    mp = std::min(std::max(32, (mp + 31) / 32 * 32), c.top_k);
    mp = std::min(mp, 8192 / (int(P) * Q));
    m.MP = mp >= 1 ? mp : 0;
  }
  m.off_cand = 0;
  m.off_part = m.off_cand + int64_t(align256(size_t(P * BH * std::max(m.K, 1) * 2 * 8)));
  m.off_clst = m.off_part + int64_t(align256(size_t(P * BH * NO * m.RS * 8)));
  m.off_ctl = m.off_clst + int64_t(align256(size_t(P * BH * Q * std::max(m.MP, 1) * 2 * 8)));
  m.bytes = size_t(m.off_ctl) + 256;
  int dev = 0;
  SD_CUDA(cudaGetDevice(&dev));
  if (dev != x->device) return fail(SD_ERR_STATE, "current device %d is not the index's device %d", dev, x->device);
  cudaError_t e = cudaMalloc(&m.local, m.bytes);
  if (e != cudaSuccess) return fail(SD_ERR_CUDA, "cudaMalloc(%zu) failed: %s", m.bytes, cudaGetErrorString(e));
  e = cudaMemset(m.local, 0, m.bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(m.local);
    return fail(SD_ERR_CUDA, "cudaMemset failed: %s", cudaGetErrorString(e));
  }
  m.peers[m.pr] = m.local;
  m.opened = m.P == 1;
  m.wait_ns = sd::kPeerWaitLimitNs;
  *out = new sd_comm(m);
  return SD_OK;
}

int32_t sd_comm_handle(const sd_comm* m, void* handle) {
  if (!m || !handle) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  CommHandle h{};
  if (m->P > 1) SD_CUDA(cudaIpcGetMemHandle(&h.ipc, m->local));
  h.magic = kCommMagic; h.version = 1;
  h.P = m->P; h.pr = m->pr; h.BH = m->BH; h.K = m->K; h.C = m->C; h.R = m->R; h.G = m->G; h.D = m->D;
  h.bytes = m->bytes;
  std::memset(handle, 0, SD_COMM_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  return SD_OK;
}

int32_t sd_comm_open(sd_comm* m, const void* handles) {
  if (!m || !handles) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  if (m->opened) return m->P == 1 ? SD_OK : fail(SD_ERR_STATE, "comm is already open");
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < m->P; ++r) {
    CommHandle h;
    std::memcpy(&h, hb + size_t(r) * SD_COMM_HANDLE_BYTES, sizeof(h));
    if (h.magic != kCommMagic || h.version != 1)
      return fail(SD_ERR_INVALID_ARG, "handle %d is not an sd_comm handle", r);
    if (h.pr != r || h.P != m->P)
      return fail(SD_ERR_INVALID_ARG, "handle %d belongs to shard %d of %d (expected %d of %d)", r, h.pr, h.P, r, m->P);
    if (h.BH != m->BH || h.K != m->K || h.C != m->C || h.R != m->R || h.G != m->G || h.D != m->D ||
        h.bytes != m->bytes)
      return fail(SD_ERR_SHAPE, "shard %d's index configuration (cluster %d, replicas %d) differs from this one's "
                  "(cluster %d, replicas %d)", r, h.C, h.R, m->C, m->R);
  }
  for (int r = 0; r < m->P; ++r) {
    if (r == m->pr) continue;
    CommHandle h;
    std::memcpy(&h, hb + size_t(r) * SD_COMM_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h.ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != m->pr && m->peers[q]) {
          cudaIpcCloseMemHandle(m->peers[q]);
          m->peers[q] = nullptr;
          m->ipc[q] = false;
        }
      return fail(SD_ERR_CUDA, "cudaIpcOpenMemHandle(shard %d) failed: %s", r, cudaGetErrorString(e));
    }
    m->peers[r] = static_cast<uint8_t*>(ptr);
    m->ipc[r] = true;
  }
  m->opened = true;
  return SD_OK;
}

int32_t sd_comm_open_local(sd_comm* m, sd_comm* const* shards) {
  if (!m || !shards) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  if (m->opened) return m->P == 1 ? SD_OK : fail(SD_ERR_STATE, "comm is already open");
  for (int r = 0; r < m->P; ++r) {
    const sd_comm* o = shards[r];
    if (!o) return fail(SD_ERR_INVALID_ARG, "shard %d's comm is NULL", r);
    if (o->pr != r || o->P != m->P)
      return fail(SD_ERR_INVALID_ARG, "comm %d belongs to shard %d of %d (expected %d of %d)", r, o->pr, o->P, r, m->P);
    if (o->BH != m->BH || o->K != m->K || o->C != m->C || o->R != m->R || o->G != m->G || o->D != m->D ||
        o->bytes != m->bytes)
      return fail(SD_ERR_SHAPE, "shard %d's index configuration differs from this one's", r);
  }
  if (enable_peer_access(m, shards) != SD_OK) return SD_ERR_CUDA;
  for (int r = 0; r < m->P; ++r) m->peers[r] = shards[r]->local;
  m->opened = true;
  return SD_OK;
}

int32_t sd_comm_set_wait_limit(sd_comm* m, int64_t limit_ns) {
  if (!m) return fail(SD_ERR_INVALID_ARG, "NULL comm");
  if (limit_ns < 1000000 || limit_ns > 600000000000ll)
    return fail(SD_ERR_INVALID_ARG, "wait limit must be in [1 ms, 600 s] (got %lld ns)", (long long)limit_ns);
  m->wait_ns = uint64_t(limit_ns);
  return SD_OK;
}

int32_t sd_comm_destroy(sd_comm* m) {
  if (!m) return SD_OK;
  cudaError_t e = cudaSuccess;
  for (int r = 0; r < m->P; ++r)
    if (r != m->pr && m->peers[r] && m->ipc[r]) {
      cudaError_t e2 = cudaIpcCloseMemHandle(m->peers[r]);
      if (e == cudaSuccess) e = e2;
    }
  cudaError_t e3 = cudaFree(m->local);
  if (e == cudaSuccess) e = e3;
  delete m;
  if (e != cudaSuccess) return fail(SD_ERR_CUDA, "sd_comm_destroy: %s", cudaGetErrorString(e));
  return SD_OK;
}

int32_t sd_shard_decode(sd_index* x, sd_comm* m, const void* q, const void* k_new, const void* v_new, float scale,
                        void* out, int32_t* sel_out, sd_stream stream) {
  if (!x || !m || !q || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(SD_ERR_INVALID_ARG, "k_new and v_new must both be given or both NULL");
  if (!std::isfinite(scale)) return fail(SD_ERR_INVALID_ARG, "scale must be finite");
  if (!m->opened) return fail(SD_ERR_STATE, "comm is not open (sd_comm_open)");
  const sd_config& c = x->cfg;
  if (m->P != c.shard_count || m->pr != c.shard_rank || m->BH != c.batch * c.n_kv_heads || m->K != c.top_k ||
      m->C != x->C || m->R != x->R || m->G != x->G || m->D != c.head_dim || m->device != x->device)
    return fail(SD_ERR_INVALID_ARG, "comm was created for another index configuration");
  if (!m->resident)
    return fail(SD_ERR_SHAPE, "%d groups x %d replica clusters do not fit on the GPU at once; use sd_shard_candidates, "
                "sd_shard_attend and sd_shard_merge", m->BH, m->R);
  const int64_t T = x->offset + (k_new ? 1 : 0);
  if (T > x->cap_global) return fail(SD_ERR_CAPACITY, "decode append exceeds capacity %lld", (long long)x->cap_global);
  if (T < 1) return fail(SD_ERR_STATE, "decode on an empty cache");
  int32_t rc = launch_decode(x, sd::MODE_PEER, int(T), q, k_new, v_new, scale, out, sel_out, nullptr, nullptr,
                             nullptr, nullptr, nullptr, static_cast<cudaStream_t>(stream), m);
  if (rc == SD_OK) {
    x->offset = T;
    if (k_new) appended_one(x);
  }
  return rc;
}

int32_t sd_set_sinks(sd_index* x, const float* sinks) {
  if (!x) return fail(SD_ERR_INVALID_ARG, "NULL index");
  x->sinks = sinks;
  return SD_OK;
}

int32_t sd_set_launch_overlap(sd_index* x, int32_t enable) {
  if (!x) return fail(SD_ERR_INVALID_ARG, "NULL index");
  x->overlap = enable ? 1 : 0;
  return SD_OK;
}

#ifdef SD_PHASE_TIMING
// Phase-timing build only: decode launches of this index write their phase
// stamps ([grid.y][grid.x][24] u64, see SD_STAMP_* in sd_device.cuh) to buf;
// NULL turns the stamps off.
int32_t sd_debug_set_phase_buffer(sd_index* x, void* buf) {
  if (!x) return fail(SD_ERR_INVALID_ARG, "NULL index");
  x->dbg = static_cast<unsigned long long*>(buf);
  return SD_OK;
}
int32_t sd_debug_set_l2_plain(sd_index* x, int32_t plain) {
  if (!x) return fail(SD_ERR_INVALID_ARG, "NULL index");
  x->l2_plain = plain ? 1 : 0;
  return SD_OK;
}
int32_t sd_debug_grid(const sd_index* x, int32_t* grid_x, int32_t* grid_y) {
  if (!x || !grid_x || !grid_y) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  *grid_x = x->C * x->R;
  *grid_y = x->cfg.batch * x->cfg.n_kv_heads;
  return SD_OK;
}
#endif

int32_t sd_check_device(sd_index* x, int32_t* flags, sd_stream stream) {
  if (!x || !flags) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  SD_CUDA(cudaMemcpyAsync(&h, x->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  SD_CUDA(cudaMemsetAsync(x->d_err, 0, sizeof(int), st));
  SD_CUDA(cudaStreamSynchronize(st));
  *flags = h;
  return SD_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode without device allocation (sd_decode_noalloc).
//
// For callers that own every byte of device memory themselves: the keys,
// values, scales, biases and summary keys are their arrays, and the decode
// kernel's scratch -- the message words through which the CTAs of a group
// merge their partials, and the groups' epochs -- lives in one fixed array of
// device memory that this file defines. Every GPU that loads
// the library holds that array until the process exits; all calls on a GPU
// share it and it keeps the last call's contents, so calls that overlap on
// the GPU (two streams, or two host threads) race with each other.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratch = SD_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratch];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[256] = {};  // device address of g_noalloc_scratch, per device ordinal

// Device address of the scratch array on the current device. The array's
// name is only a host-side stand-in for the symbol; the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
int32_t noalloc_scratch(void** out) {
  int dev = 0;
  SD_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 256) return fail(SD_ERR_STATE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(SD_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev, cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SD_OK;
}

}  // namespace

extern "C" int32_t sd_decode_noalloc(const sd_config* cfg, const sd_arrays* arrays, int64_t offset, const void* q,
                                     float scale, void* out, int32_t* sel_out, int32_t* device_flags,
                                     sd_stream stream) {
  int32_t rc = validate(cfg);
  if (rc != SD_OK) return rc;
  if (!arrays || !q || !out) return fail(SD_ERR_INVALID_ARG, "NULL argument");
  // The error bits have nowhere else to go: the scratch array is cleared by
  // the next call before the caller could read it.
  if (!device_flags) return fail(SD_ERR_INVALID_ARG, "device_flags is required (the kernel's error bits go there)");
  const sd_config& c = *cfg;
  if (c.shard_count != 1) return fail(SD_ERR_STATE, "sd_decode_noalloc serves single-shard caches only");
  if (!std::isfinite(scale)) return fail(SD_ERR_INVALID_ARG, "scale must be finite");
  if (!arrays->k_data || !arrays->v_data || !arrays->summaries)
    return fail(SD_ERR_INVALID_ARG, "k_data, v_data and summaries are required");
  if (c.kv_bits && (!arrays->k_scales || !arrays->k_biases || !arrays->v_scales || !arrays->v_biases))
    return fail(SD_ERR_INVALID_ARG, "quantized caches need scales and biases");
  // The kernel reads these arrays with 16-byte loads and bulk copies, the
  // queries with 4-byte loads; a misaligned pointer would fault on the GPU.
  auto mis = [](const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) != 0; };
  if (mis(arrays->k_data, 16) || mis(arrays->v_data, 16) || mis(arrays->summaries, 16))
    return fail(SD_ERR_INVALID_ARG, "k_data, v_data and summaries must be 16-byte aligned");
  if (c.kv_bits && (mis(arrays->k_scales, 16) || mis(arrays->k_biases, 16) || mis(arrays->v_scales, 16) ||
                    mis(arrays->v_biases, 16)))
    return fail(SD_ERR_INVALID_ARG, "scales and biases must be 16-byte aligned");
  if (mis(q, 4) || mis(out, 2) || mis(sel_out, 4) || mis(device_flags, 4))
    return fail(SD_ERR_INVALID_ARG, "q must be 4-byte, out 2-byte, sel_out and device_flags 4-byte aligned");
  if (arrays->cap_local < 1 || arrays->cap_local % c.block_size != 0 || offset < 1 || offset > arrays->cap_local)
    return fail(SD_ERR_SHAPE, "offset %lld / cap_local %lld do not describe a cache", (long long)offset,
                (long long)arrays->cap_local);
  if (arrays->nb_local < (offset + c.block_size - 1) / c.block_size)
    return fail(SD_ERR_SHAPE, "nb_local %lld is smaller than the blocks in the cache", (long long)arrays->nb_local);

  const int row_bytes = c.kv_bits ? c.head_dim * c.kv_bits / 8 : c.head_dim * elt_size(c.dtype);
  if (arrays->row_bytes != 0 && arrays->row_bytes != row_bytes)
    return fail(SD_ERR_SHAPE, "row_bytes %d does not match the configuration (%d)", arrays->row_bytes, row_bytes);

  // A host-side description of the cache; no device memory is allocated.
  sd_index x{};
  x.cfg = c;
  SD_CUDA(cudaGetDevice(&x.device));
  x.G = c.n_q_heads / c.n_kv_heads;
  x.esize = elt_size(c.dtype);
  x.groups = c.kv_bits ? c.head_dim / 64 : 1;
  x.row_bytes = row_bytes;
  x.cap_local = arrays->cap_local;
  x.nb_local = arrays->nb_local;
  x.cap_global = x.cap_local;
  x.nb_global = x.nb_local;
  x.offset = offset;
  const int64_t BH = int64_t(c.batch) * c.n_kv_heads;
  if (BH * x.cap_local >= (int64_t(1) << 31) || BH > 65535)
    return fail(SD_ERR_SHAPE, "cache too large: batch*kv_heads*cap_local rows must stay below 2^31");
  x.ks = lookup(c.dtype, c.kv_bits, c.head_dim, x.G);
  if (!x.ks.decode) return fail(SD_ERR_SHAPE, "no kernel for this configuration");
  x.smem = size_t(sd::make_layout(c.head_dim, x.G, x.groups).total) + 1024;
  rc = setup_kernels(&x);
  if (rc == SD_OK) rc = choose_cluster(&x);
  if (rc != SD_OK) return rc;

  // Scratch layout: [0, 256) reserved, then the groups' epochs, the group
  // merge's message words and, for the sliced selection, the CTAs' lists.
  // Fewer CTAs per group are used if they do not fit. Everything used is
  // cleared by every call (the array is shared by calls of any configuration,
  // and a word left by another configuration could carry a matching epoch).
  const int64_t nloc = offset > c.block_size ? (offset + c.block_size - 1) / c.block_size - 1 : 0;
  struct Need { size_t slots, lists, falls; int mt; };
  auto need = [&](int C, int R) {
    const int Q = C * R;
    Need n{0, 0, 0, 0};
    if (Q > 1) {
      n.slots = align256(size_t(BH) * merge_owners(Q, x.G, c.head_dim) * Q * merge_record(Q, x.G, c.head_dim) * 8);
      if (c.top_k > 128 || nloc > sd::kAllKeysMax || C == 1) {
        n.mt = list_len(c.top_k, Q);
        n.lists = align256(size_t(BH) * Q * n.mt * 2 * 8);
        n.falls = align256(size_t(BH) * Q * c.top_k * 2 * 8);
      }
    }
    return n;
  };
  const size_t ep_bytes = align256(size_t(BH) * 4);
  auto total = [&](int C, int R) {
    const Need n = need(C, R);
    return 256 + ep_bytes + n.slots + n.lists + n.falls;
  };
  auto fits = [&]() { return total(x.C, x.R) <= kNoAllocScratch; };
  // fewer replicas first, then smaller clusters (one CTA per group needs no message words)
  while (!fits() && x.R > 1) --x.R;
  const int c_chosen = x.C;
  while (!fits() && x.C > 1) {
    int c2 = x.C - 1;
    while (c2 > 1 && ((x.nb_local + c2 - 1) / c2 > sd::kLocalKeysMax || max_active_clusters(&x, c2) < 1)) --c2;
    if ((x.nb_local + c2 - 1) / c2 > sd::kLocalKeysMax) break;
    x.C = c2;
  }
  if (x.C < c_chosen && fits()) {
    // a smaller cluster leaves room for replicas again: raise R while the
    // scratch holds them and every cluster stays resident at once (the rule
    // choose_cluster applies)
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, x.device);
    const int64_t mac = max_active_clusters(&x, x.C);
    while (x.R < 4 && BH * x.C * (x.R + 1) <= n_sm && mac >= BH * (x.R + 1) &&
           total(x.C, x.R + 1) <= kNoAllocScratch)
      ++x.R;
  }
  if (!fits())
    return fail(SD_ERR_CAPACITY, "batch*kv_heads (%lld) needs %zu bytes of scratch; the limit is %zu",
                (long long)BH, total(x.C, x.R), kNoAllocScratch);
  const Need nd = need(x.C, x.R);
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != SD_OK) return rc;
  uint8_t* sb = static_cast<uint8_t*>(scratch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SD_CUDA(cudaMemsetAsync(sb, 0, total(x.C, x.R), st));
  x.mt = nd.mt;
  x.gslot = nd.slots ? reinterpret_cast<unsigned long long*>(sb + 256 + ep_bytes) : nullptr;
  x.clist = nd.lists ? reinterpret_cast<unsigned long long*>(sb + 256 + ep_bytes + nd.slots) : nullptr;
  x.cfall = nd.falls ? reinterpret_cast<unsigned long long*>(sb + 256 + ep_bytes + nd.slots + nd.lists) : nullptr;

  x.k_data = arrays->k_data; x.v_data = arrays->v_data;
  x.k_scales = arrays->k_scales; x.k_biases = arrays->k_biases;
  x.v_scales = arrays->v_scales; x.v_biases = arrays->v_biases;
  x.summ = arrays->summaries;
  x.lt = load_tokens(c);
  x.kv_fused = encode_kv_map(&x.tmK, x.k_data, x.v_data, x.row_bytes, BH * x.cap_local, x.lt) ? 1 : 0;
  if (!x.kv_fused) {
    rc = encode_map(&x.tmK, x.k_data, x.row_bytes, BH * x.cap_local, x.lt);
    if (rc == SD_OK) rc = encode_map(&x.tmV, x.v_data, x.row_bytes, BH * x.cap_local, x.lt);
    if (rc != SD_OK) return rc;
  }

  sd::DecodeParams p{};
  p.B = c.batch; p.Hq = c.n_q_heads; p.Hkv = c.n_kv_heads; p.S = c.block_size; p.K = c.top_k;
  p.T = int(offset);
  p.NB = int((offset + c.block_size - 1) / c.block_size);
  p.P = 1; p.pr = 0;
  p.cap_local = int(x.cap_local);
  p.nb_stride = int(x.nb_local);
  p.C = x.C;
  p.mode = sd::MODE_FUSED;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = q;
  p.k_data = x.k_data; p.v_data = x.v_data;
  p.k_scales = x.k_scales; p.k_biases = x.k_biases; p.v_scales = x.v_scales; p.v_biases = x.v_biases;
  p.summ = x.summ;
  p.out = out;
  p.sel_out = sel_out;
  p.err = device_flags;
  p.R = x.R;
  p.nown = merge_owners(x.C * x.R, x.G, c.head_dim);
  p.gep = reinterpret_cast<uint32_t*>(sb + 256);
  p.gslot = x.gslot;
  p.sliced = sliced_launch(&x, nloc) ? 1 : 0;
  p.mt = x.mt;
  p.clist = x.clist;
  p.cfall = x.cfall;
  const int64_t chunks = p.sliced ? int64_t(x.C) * x.R : x.C;
  if ((nloc + chunks - 1) / chunks > sd::kLocalKeysMax)
    return fail(SD_ERR_SHAPE, "too many blocks per CTA for %lld CTAs per group", (long long)chunks);

  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(unsigned(x.C * x.R), unsigned(BH), 1);
  lc.blockDim = dim3(sd::kThreads, 1, 1);
  lc.dynamicSmemBytes = x.smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(x.C);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  p.sb_fused = 0;  // the caller's arrays: four 1-D bulk scale/bias copies
  p.lt = x.lt;
  p.kv_fused = x.kv_fused;
  void* args[4] = {&p, &x.tmK, &x.tmV, &x.tmS};
  SD_CUDA(cudaLaunchKernelExC(&lc, x.ks.decode, args));
  return SD_OK;
}
