/* sparse_decode.h -- C ABI of the B200 (sm_100a) retrieval block-sparse decode
 * attention library (libsparse_decode.so).
 *
 * The library owns a sequence's KV cache for one attention layer, in the
 * reference's layout [B, Hkv, cap, D] (dense fp32/fp16/bf16) or as the
 * affine-quantized tuple (uint32-packed 4/8-bit codes, per-group-of-64
 * scales and biases in the key dtype), plus one summary key per block of S
 * tokens. A decode step scores every block against the query group, keeps the
 * top-K blocks plus the most recent block, and attends over those tokens.
 *
 * Reference interfaces these entry points stand in for (TheTom/mlx-swift-lm;
 * paths inside that project):
 *   - protocol KVCache             Libraries/MLXLMCommon/KVCache.swift:38-77
 *   - protocol QuantizedKVCacheProtocol               KVCache.swift:94-119
 *   - KVCacheSimple (storage, 256-token growth)       KVCache.swift:315-371
 *   - QuantizedKVCache (tuple storage, state)         KVCache.swift:728-988
 *   - quantizedScaledDotProductAttention              KVCache.swift:1533-1621
 *   - attentionWithCacheUpdate (the router)  Libraries/MLXLMCommon/AttentionUtils.swift:37-77
 *
 * Conventions. Every pointer argument is a DEVICE pointer owned by the caller
 * unless stated otherwise; the KV, scale/bias and summary arenas are owned by
 * the index (allocated on create, freed on destroy). Every call is
 * asynchronous on the given CUDA stream (a cudaStream_t passed as void*;
 * NULL = legacy default stream) and returns an sd_status; no call aborts the
 * process. One index is used by one host thread at a time.
 */
#ifndef SPARSE_DECODE_H
#define SPARSE_DECODE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sd_index sd_index; /* opaque */
typedef void* sd_stream;          /* cudaStream_t */

/* Error codes. The reference traps misuse with fatalError/precondition
 * (KVCache.swift:893-897, :929) and throws on I/O (KVCache.swift:1323); this
 * ABI returns a code instead and keeps a per-thread message (sd_last_error). */
typedef enum {
  SD_OK = 0,
  SD_ERR_INVALID_ARG = 1, /* null pointer, bad enum, non-positive size */
  SD_ERR_SHAPE = 2,       /* shapes this build does not support (D, G, S, K ...) */
  SD_ERR_CAPACITY = 3,    /* append beyond the index capacity */
  SD_ERR_STATE = 4,       /* call not valid in the index's current state */
  SD_ERR_CUDA = 5,        /* a CUDA runtime/driver call failed */
  SD_ERR_DEVICE = 6       /* a kernel reported an error (bounded wait expired ...) */
} sd_status;

typedef enum { SD_F32 = 0, SD_F16 = 1, SD_BF16 = 2 } sd_dtype;

/* Fixed at create time. Mirrors the reference's cache knobs: kv_bits /
 * group_size (GenerateParameters kvBits, kvGroupSize: Evaluate.swift:67-73,
 * QuantizedKVCache(groupSize:bits:) KVCache.swift:736) and adds the retrieval
 * knobs block_size and top_k. */
typedef struct {
  int32_t batch;        /* B */
  int32_t n_q_heads;    /* Hq (multiple of n_kv_heads; Hq/Hkv in {1,2,4,8}) */
  int32_t n_kv_heads;   /* Hkv */
  int32_t head_dim;     /* D in {64, 128} */
  int32_t block_size;   /* S tokens per block, in {32, 64, 128, 256} */
  int32_t top_k;        /* K blocks chosen besides the recent block, 0..1023 */
  int32_t capacity;     /* tokens per sequence; rounded up to a multiple of 256 */
  int32_t dtype;        /* sd_dtype of queries, outputs, dense K/V, scales/biases, summaries */
  int32_t kv_bits;      /* 0 = dense, 4 or 8 = affine-quantized K/V */
  int32_t group_size;   /* quantization group along D; must be 64 when kv_bits != 0 */
  int32_t shard_rank;   /* sequence sharding: block j lives on shard j % shard_count */
  int32_t shard_count;  /* 1 = single GPU */
  int32_t cluster_size; /* CTAs per (batch, kv-head) in decode; 0 = choose */
  int32_t reserved[3];  /* must be 0 */
} sd_config;

/* Device arrays of an index (for state export/import and inspection). */
typedef struct {
  void* k_data;     /* dense [B*Hkv, cap_local, D] dtype; quantized [B*Hkv, cap_local, D*bits/32] uint32 */
  void* v_data;
  void* k_scales;   /* quantized only: [B*Hkv, cap_local, D/64] dtype (else NULL) */
  void* k_biases;
  void* v_scales;
  void* v_biases;
  void* summaries;  /* [B*Hkv, nb_local, D] dtype: mean key of each block */
  int64_t cap_local;   /* token rows per (b, kv-head) on this shard */
  int64_t nb_local;    /* block rows per (b, kv-head) on this shard */
  int32_t row_bytes;   /* bytes of one K (or V) row */
  int32_t cluster_size; /* CTAs per cluster in decode */
  int32_t smem_bytes;   /* dynamic shared memory of the decode kernel */
  int32_t replicas;     /* clusters per (batch, kv-head) in decode */
  int32_t reserved[4];
} sd_arrays;

int32_t sd_abi_version(void);
const char* sd_status_string(int32_t status);
/* Message of the last failed call on this thread ("" if none). */
const char* sd_last_error(void);

/* Create an index on the current CUDA device. Replaces constructing a
 * KVCacheSimple()/QuantizedKVCache(groupSize:bits:) (KVCache.swift:320, :736)
 * inside LanguageModel.newCache (LanguageModel.swift:215-229). */
int32_t sd_index_create(const sd_config* cfg, sd_index** out);
int32_t sd_index_destroy(sd_index* idx);
int32_t sd_index_config(const sd_index* idx, sd_config* out);
int32_t sd_index_arrays(const sd_index* idx, sd_arrays* out);
/* KVCache.offset (KVCache.swift:40): tokens currently in the sequence. */
int32_t sd_index_offset(const sd_index* idx, int64_t* offset);
/* Deep copy on the same device (KVCache.copy, KVCache.swift:76). */
int32_t sd_index_copy(const sd_index* src, sd_index** out, sd_stream stream);

/* Append n_tokens rows: keys/values [B, Hkv, n_tokens, D] of the index dtype.
 * Quantizes when kv_bits != 0 and (re)builds the summary of every block
 * touched. Replaces KVCacheSimple.update / QuantizedKVCache.updateQuantized
 * (KVCache.swift:328-371, :816-889) for prefill (L > 1). */
int32_t sd_append(sd_index* idx, const void* keys, const void* values, int32_t n_tokens, sd_stream stream);

/* KVCache.trim (KVCache.swift:59-60, :394-398): drop up to n tokens from the
 * end; *trimmed (nullable, host pointer) receives the count. Host-only. */
int32_t sd_trim(sd_index* idx, int32_t n, int32_t* trimmed);

/* State import: after writing rows through sd_index_arrays, declare the token
 * count and rebuild the summaries (KVCache.state / metaState setters,
 * KVCache.swift:46-50, :900-944). */
int32_t sd_set_offset(sd_index* idx, int64_t offset);
int32_t sd_rebuild_summaries(sd_index* idx, sd_stream stream);

/* One decode step for L == 1: the sparse branch of attentionWithCacheUpdate
 * (AttentionUtils.swift:37-77). q [B, Hq, D]; k_new / v_new [B, Hkv, D] are
 * appended first when non-NULL (the cache.update half of the router), then
 * out [B, Hq, D] = softmax(scale * q K^T) V over the selected blocks' tokens.
 * sel_out [B*Hkv, top_k+1] int32 (nullable): selected blocks ascending, the
 * recent block last, -1 padded. scores_out [B*Hkv, nblocks] float (nullable):
 * the block scores. Single-shard indexes only. */
int32_t sd_decode(sd_index* idx, const void* q, const void* k_new, const void* v_new, float scale, void* out,
                  int32_t* sel_out, float* scores_out, sd_stream stream);

/* Sequence-sharded decode (shard_count > 1), three steps around two
 * all-gathers that the caller runs (e.g. ncclAllGather over NVLink):
 *  1. sd_shard_candidates: optional append (the owning shard stores the row),
 *     local scores and local top-K -> cand_score/cand_block [B*Hkv, top_k]
 *     (-inf / -1 padded). All shards must call it with the same arguments.
 *  2. all-gather candidates into [shard_count, B*Hkv, top_k].
 *  3. sd_shard_attend: global top-K (identical on every shard) plus the
 *     recent block, attention over this shard's selected blocks ->
 *     part_ml [B*Hq, 2] (running max in log2 units, sum) and part_o [B*Hq, D].
 *  4. all-gather partials into [shard_count, ...].
 *  5. sd_shard_merge: log-sum-exp merge in shard order -> out [B, Hq, D]. */
int32_t sd_shard_candidates(sd_index* idx, const void* q, const void* k_new, const void* v_new, float scale,
                            float* cand_score, int32_t* cand_block, float* scores_out, sd_stream stream);
int32_t sd_shard_attend(sd_index* idx, const void* q, const float* all_cand_score, const int32_t* all_cand_block,
                        float scale, float* part_ml, float* part_o, int32_t* sel_out, sd_stream stream);
int32_t sd_shard_merge(sd_index* idx, const float* all_part_ml, const float* all_part_o, void* out,
                       sd_stream stream);

/* Fused sequence-sharded decode over peer memory (one process per GPU, GPUs
 * of one node with peer access, e.g. NVLink through NVSwitch). One launch
 * per step and shard does all of the sharded path's work: local scores and
 * top-K, the candidates' exchange, the global top-K (identical on every
 * shard), attention over this shard's selected blocks, the exchange of the
 * (m, l, o) partials and their log-sum-exp merge in shard order -- the
 * exchanges are stores into the other shards' memory plus flags, so there is
 * no collective call between kernels and the step can be captured in a CUDA
 * graph. Every shard gets the full output.
 *
 * Setup, per index configuration and shard (the layers of a model that share
 * a configuration share one sd_comm):
 *   1. sd_comm_create(idx, &comm): the exchange area of this shard.
 *   2. sd_comm_handle(comm, h): SD_COMM_HANDLE_BYTES of host bytes describing
 *      it (a CUDA IPC handle plus the configuration).
 *   3. exchange the handles between the shards by any transport (e.g. an
 *      all-gather), in shard order, and pass all of them to sd_comm_open.
 * Then per step, on every shard with the same arguments:
 *   sd_shard_decode(idx, comm, q, k_new, v_new, scale, out, sel_out, stream).
 * All shards must issue the same sequence of sd_shard_decode calls on one
 * comm, on one stream each. The kernel waits for the other shards with a
 * bounded wait (10 s): on expiry it sets error bit 4 (sd_check_device) and
 * finishes. Every cluster of the launch must be resident at once: a
 * configuration with more (b, kv-head) groups than the GPU holds is rejected
 * with SD_ERR_SHAPE (use sd_shard_candidates / attend / merge). Destroy a
 * comm only after every shard has finished using it (e.g. after a barrier).
 * No counterpart in the reference. */
typedef struct sd_comm sd_comm; /* opaque */
#define SD_COMM_HANDLE_BYTES 128
int32_t sd_comm_create(const sd_index* idx, sd_comm** out);
int32_t sd_comm_handle(const sd_comm* comm, void* handle);
int32_t sd_comm_open(sd_comm* comm, const void* handles);
/* Shards driven by one process (one GPU each, or several on one GPU for
 * tests that run a single shard): open with every shard's comm, in shard
 * order, instead of IPC handles; peer access between the devices is enabled
 * here. */
int32_t sd_comm_open_local(sd_comm* comm, sd_comm* const* shards);
/* Bound of the kernel's waits for other shards (default 10 s; 1 ms .. 600 s). */
int32_t sd_comm_set_wait_limit(sd_comm* comm, int64_t limit_ns);
int32_t sd_comm_destroy(sd_comm* comm);
int32_t sd_shard_decode(sd_index* idx, sd_comm* comm, const void* q, const void* k_new, const void* v_new,
                        float scale, void* out, int32_t* sel_out, sd_stream stream);

/* Attention sinks for the decodes of this index (sd_decode, sd_shard_decode,
 * sd_shard_merge): `sinks` is a device array of n_q_heads fp32 logits, in the
 * units of scale * q.k, that join every head's softmax denominator without
 * contributing a value -- out = sum_t e^(s_t) v_t / (sum_t e^(s_t) + e^(sink)),
 * as MLXFast.scaledDotProductAttention(..., sinks:) computes it for the
 * reference's sink-attention models (Libraries/MLXLLM/Models/GPTOSS.swift:
 * 228-261, MiMoV2Flash.swift:14-56). NULL turns them off. The array must stay
 * valid while decodes that use it run. The reference rejects sinks with a
 * quantized cache; this library applies them to every cache format. */
int32_t sd_set_sinks(sd_index* idx, const float* sinks);

/* Decode launches of this index may overlap the previous kernel on the
 * stream (programmatic dependent launch): the decode kernel starts its
 * prologue -- barrier setup and the first loads of this index's summary keys
 * -- while the previous kernel finishes, and waits for it before reading the
 * queries or the new token. The library remembers which index it last
 * launched work for on each stream and never reads an index early after its
 * own work; with overlap enabled, the caller must not write this index's
 * arrays (sd_index_arrays) with its own kernels on the same stream. No
 * counterpart in the reference (MLX schedules lazily evaluated graphs). */
int32_t sd_set_launch_overlap(sd_index* idx, int32_t enable);

/* Read and clear the device error word of the index (synchronises the stream).
 * *flags (host pointer) receives the bits: 1 = a bounded wait expired,
 * 2 = an index out of range, 4 = a wait for another shard expired. */
int32_t sd_check_device(sd_index* idx, int32_t* flags, sd_stream stream);

/* Decode for callers that cannot allocate device memory. Some hosts own all
 * of the GPU's memory themselves -- for example a serving runtime that
 * reserves the device's memory pool when it starts and lends slices of it to
 * plug-ins -- so a library that calls cudaMalloc behind their back can fail
 * or fragment that pool. This entry point allocates nothing: the caller
 * passes its own device arrays in the layout of sd_arrays (k_data, v_data,
 * scales/biases for 4/8-bit caches, summaries, cap_local, nb_local; e.g.
 * arrays filled earlier through an index, or by the caller's own code), the
 * number of tokens `offset`, queries, output and an optional sel_out, and the
 * call decodes one token (no append) like sd_decode. device_flags (required:
 * a caller-owned device int, zeroed by the caller) receives the same error
 * bits as sd_check_device reports; there is no other place where a call's
 * device errors could be read. Alignment: k_data, v_data, summaries and the
 * four scale/bias arrays 16 bytes (the kernel reads them with 16-byte loads
 * and bulk copies), q and device_flags 4 bytes, out 2 bytes; a misaligned
 * pointer is rejected with SD_ERR_INVALID_ARG before anything is launched.
 * The kernel's scratch (the message words through which the CTAs of a
 * (batch, kv-head) group merge their partial results, and the groups' epochs)
 * lives in a fixed array of SD_NOALLOC_SCRATCH_BYTES of device memory inside
 * the library, which every GPU that loads the library keeps until the process
 * exits. The first call on a device looks up that array's device address.
 * All calls on a device share the array and it keeps the last call's
 * contents (every call clears the part it uses), so two calls that overlap on
 * the GPU race with each other: serialise them. When the scratch of the
 * usual launch shape does not fit, fewer CTAs per group are used (down to
 * one, which needs only the epochs); a configuration that still cannot fit
 * is rejected with SD_ERR_CAPACITY. Single-shard caches only.
 * No counterpart in the reference. */
#define SD_NOALLOC_SCRATCH_BYTES (1u << 20)
int32_t sd_decode_noalloc(const sd_config* cfg, const sd_arrays* arrays, int64_t offset, const void* q, float scale,
                          void* out, int32_t* sel_out, int32_t* device_flags, sd_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSE_DECODE_H */
