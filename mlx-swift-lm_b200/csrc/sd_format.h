// sd_format.h -- compile-time description of one KV storage format and the
// shared-memory layout of the decode kernel. Included by host and device code.
#pragma once

#include <stdint.h>

namespace sd {

constexpr int kTileTokens = 32;                 // tokens per staged tile (one per lane in QK)
constexpr int kConsumerWarps = 8;               // warps that attend
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + one TMA producer warp
constexpr int kRingBytes = 160 * 1024;          // TMA ring; aliases the selection buffers
constexpr int kLocalKeysMax = 16384;            // candidate blocks scored by one CTA
constexpr int kUnionMax = 8192;                 // candidates gathered for the final top-K
constexpr int kMaxTopK = 1023;                  // K (recent block excluded)
constexpr int kMaxGroupCtas = 64;               // C * R: CTAs of one (b, kv-head) group
constexpr int kAllKeysMax = 2048;               // candidates held whole by every CTA (bitonic top-K)

enum Mode { MODE_FUSED = 0, MODE_CANDIDATES = 1, MODE_ATTEND = 2, MODE_PEER = 3 };
constexpr int kMaxShards = 8;                   // peer mode: shards (GPUs) exchanging over peer memory
constexpr unsigned long long kPeerWaitLimitNs = 10000000000ull;  // peer mode: default bound of a wait (10 s)

__host__ __device__ constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// KV format: ESIZE = bytes of the dense element or of the scale/bias type,
// BITS = 0 (dense) or 4 / 8 (affine group-64 codes), D = head_dim.
template <int ESIZE, int BITS, int D>
struct Fmt {
  static constexpr bool kQuant = BITS != 0;
  static constexpr int kEltBits = kQuant ? BITS : 8 * ESIZE;
  static constexpr int kRowBytes = D * kEltBits / 8;
  static constexpr int kBoxBytes = kRowBytes < 128 ? kRowBytes : 128;
  static constexpr int kNBox = kRowBytes / kBoxBytes;
  static constexpr int kCpb = kBoxBytes / 16;          // 16-byte chunks per box
  static constexpr int kNChunk = kRowBytes / 16;       // chunks per row
  static constexpr int kEpc = 128 / kEltBits;          // elements per 16-byte chunk
  static constexpr int kGroups = kQuant ? D / 64 : 1;  // quantization groups per row
  // Token rows of one staged copy (the TMA box): 64 for 4/8-bit codes with
  // 16-bit scales, whose tensor-core consumer walks a stage as two 32-token
  // halves (fewer, larger copies: the TMA unit's per-copy cost dominates
  // tiles of a few KB); 32 otherwise. Blocks of 32 tokens stage 32 (the
  // host picks the box; the stage is sized for kLoadTokens).
  static constexpr int kLoadTokens = (kQuant && ESIZE == 2) ? 64 : kTileTokens;
  static constexpr int kKvTileBytes = kLoadTokens * kRowBytes;
  static constexpr int kSbTileBytes = kQuant ? kLoadTokens * kGroups * ESIZE : 0;
  static constexpr int kStageBytes = align_up(2 * kKvTileBytes + 4 * kSbTileBytes, 1024);
  static constexpr int kStages = (kRingBytes / kStageBytes) < 16 ? (kRingBytes / kStageBytes) : 16;
  // PV mapping: each lane owns kPiece bytes (kDpl dims) of a row; kRpp rows per pass.
  static constexpr int kPiece = (kRowBytes / 32) >= 4 ? (kRowBytes / 32) : 4;
  static constexpr int kLpr = kRowBytes / kPiece;
  static constexpr int kRpp = 32 / kLpr;
  static constexpr int kDpl = kPiece * 8 / kEltBits;
  // Summary scoring: lanes per block (one 16-byte chunk of the summary each).
  static constexpr int kSumLanes = D * ESIZE / 16;
  static constexpr int kSumEpc = 16 / ESIZE;
  static_assert(kSumLanes <= 32, "summary row wider than a warp");
  static_assert(kRowBytes % 16 == 0, "row must be a whole number of 16-byte chunks");
};

// Shared-memory layout of the decode kernel (byte offsets from a 1024-aligned base).
struct Layout {
  int ring;        // kRingBytes: TMA stages | local keys + union | merge buffers
  int union_off;   // inside the ring: union (key u32, block i32) pairs
  int qf;          // G*D floats: queries scaled by scale*log2(e), [D][G]
  int qsum;        // D floats: unscaled sum of the group's queries (scoring)
  int qs;          // G*groups floats: per-group sums of qf (quantized K bias term)
  int sel;         // (kMaxTopK + 2) ints: selected blocks, ascending, recent last
  int own;         // (kMaxTopK + 2) ints: the selected blocks stored on this shard
  int hist;        // 256 u32
  int scratch;     // 128 ints: scans [0,33), radix state [40,48), largest key [113], selection [118,124), ring/own counters [124,127)
  int ps;          // per consumer warp: kTileTokens * G * groups floats
  int cpart;       // G*(D+2) floats: this CTA's merged (m, l, o)
  int recv;        // (m, l) of every CTA of the group for this CTA's output slice
  int allk;        // kAllKeysMax u32: every candidate key of the group (bitonic top-K)
  int bars;        // 2 * 16 mbarriers
  int total;
};

__host__ __device__ inline Layout make_layout(int D, int G, int groups) {
  Layout L{};
  int off = 0;
  L.ring = off; off += kRingBytes;
  L.union_off = kLocalKeysMax * 4;
  L.qf = off; off += align_up(G * D * 4, 16);
  L.qsum = off; off += align_up(D * 4, 16);
  L.qs = off; off += align_up(G * 2 * 4, 16);
  L.sel = off; off += align_up((kMaxTopK + 2) * 4, 16);
  L.own = off; off += align_up((kMaxTopK + 2) * 4, 16);
  L.hist = off; off += 256 * 4;
  L.scratch = off; off += 128 * 4;
  L.ps = off; off += kConsumerWarps * align_up(kTileTokens * G * groups * 4, 16);
  L.cpart = off; off += align_up(G * (D + 2) * 4, 16);
  L.recv = off; off += align_up(kMaxGroupCtas * 2 * G * 4, 16);
  L.allk = off; off += kAllKeysMax * 4;
  L.bars = off; off += 32 * 8;
  L.total = off;
  return L;
}

}  // namespace sd
