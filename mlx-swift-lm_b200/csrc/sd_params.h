// sd_params.h -- kernel parameter blocks shared by the host launcher and the
// device kernels. Plain C structs: pointers are device pointers.
#pragma once

#include <stdint.h>

namespace sd {

struct DecodeParams {
  int B, Hq, Hkv, S, K;   // K = blocks chosen by top-K (the recent block is extra)
  int T;                  // tokens in the sequence, after the optional append
  int NB;                 // blocks = ceil(T / S)
  int P, pr;              // sequence shards and this shard's rank (block j lives on j % P)
  int cap_local;          // token rows per (b, kv-head) on this shard
  int nb_stride;          // summary rows per (b, kv-head) on this shard
  int C;                  // cluster size (CTAs per (b, kv-head))
  int mode;               // sd::Mode
  float scale;            // softmax scale applied to q.k
  float scale_log2;       // scale * log2(e)
  const void* q;          // [B, Hq, D]
  const void* k_new;      // [B, Hkv, D] appended before attending, or null
  const void* v_new;
  void* k_data;           // dense [BH, cap_local, D] or codes [BH, cap_local, D*bits/32]
  void* v_data;
  void* k_scales;         // quantized only: [BH, cap_local, D/64]
  void* k_biases;
  void* v_scales;
  void* v_biases;
  void* summ;             // [BH, nb_stride, D] summary keys
  void* out;              // [B, Hq, D] (fused mode)
  int32_t* sel_out;       // [BH, K+1] or null: selected blocks, ascending, recent last, -1 padded
  float* scores_out;      // [BH, NB] or null: block scores of this shard's blocks
  float* cand_score;      // candidates mode: out [BH, K]; attend mode: in [P, BH, K]
  int32_t* cand_block;
  float* part_ml;         // attend mode: out [B*Hq, 2] = (max in log2 units, sum)
  float* part_o;          // attend mode: out [B*Hq, D] unnormalised
  int* err;               // device error word (sd::kErr*)
  int R;                  // replica clusters per (b, kv-head): each attends 1/R of the tiles
  int nown;               // Q = C*R > 1: CTAs of a group that own a slice of the output (the merge)
  unsigned long long* gslot;  // Q = C*R > 1: [BH][nown owners][Q sources][2G + ceil(G*D/nown)] message words
  uint32_t* gep;          // Q > 1: [BH] epoch of each group's last merged launch
  // Sliced selection (more than kAllKeysMax candidates per group, or K > 128)
  // with Q > 1: every CTA's best mt keys [BH][Q][mt][2] and, when a list ran
  // out, every CTA's full top-K [BH][Q][K][2], as message words.
  int sliced;             // 1: the sliced selection (set per launch by the host)
  int mt;
  unsigned long long* clist;
  unsigned long long* cfall;
  int pdl_early;          // 1: this index's summaries may be read before the grid-dependency wait
  const float* racc_in;   // [BH, D] fp32 sum of the recent block's rows before this step
  float* racc_out;        // [BH, D] the same sum after the appended row
  int racc_rebuild;       // 1: racc_in is not valid; sum the recent block's rows from the cache
  const float* sinks;     // [Hq] attention-sink logits (same units as scale * q.k), or null
  // Peer mode: every shard's exchange area mapped into this process (own at
  // [pr]). Area layout, identical on every shard, all message words (32-bit
  // payload | epoch << 32): [P][BH][K][2] candidate keys (hi, lo) at x_cand,
  // [P][BH][nown][RS] partial records ([2G] (m, l), then the slice of o) at
  // x_part; at x_ctl two u32 control words of this shard: the last finished
  // epoch and the count of finished CTAs.
  uint8_t* peer[8];
  int64_t x_cand, x_part, x_ctl;  // byte offsets inside an area
  // Sliced selection in peer mode: every CTA's best mtp keys
  // [P][BH][Q][mtp][2] at x_clst (mtp = 0: the two-level path only).
  int mtp;
  int64_t x_clst;
  uint64_t peer_wait_ns;                   // bound of every wait for another shard
  // 1: the scale/bias tensor map covers the four arrays (k_scales, k_biases,
  // v_scales, v_biases at one fixed stride), one copy per tile. 0: four 1-D
  // bulk copies.
  int sb_fused;
  // Tokens per staged copy (Fmt::kLoadTokens, or 32 for blocks of 32 tokens),
  // and 1 when the K tensor map covers V too (one copy per stage for both).
  int lt;
  int kv_fused;
  unsigned long long* dbg;  // phase-timing build only: [grid.y][grid.x][24] stamps, or null
  int l2_plain;  // 1: streamed loads (summaries, K/V tiles) without the L2 evict_first hint
};

struct AppendParams {
  int Hkv, S, P, pr;
  int cap_local;
  int n_tok;              // tokens in this append
  int t0;                 // global position of the first appended token
  const void* k_src;      // [B, Hkv, n_tok, D]
  const void* v_src;
  void* k_data;
  void* v_data;
  void* k_scales;
  void* k_biases;
  void* v_scales;
  void* v_biases;
};

struct SummaryParams {
  int Hkv, S, P, pr;
  int cap_local, nb_stride;
  int T;                  // tokens in the sequence
  int jl0;                // first local block to rebuild (blockIdx.x offsets from here)
  const void* k_data;
  const void* k_scales;
  const void* k_biases;
  void* summ;
};

}  // namespace sd
