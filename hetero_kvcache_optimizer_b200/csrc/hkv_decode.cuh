// Persistent split-KV GQA decode attention over packed INT4 pages + a dense
// fp16/bf16 segment, with a fused log-sum-exp merge. Included by hetero_kv.cu.
//
// Schedule. The work of every (sequence, KV head) unit is a list of tiles:
// 128-token INT4 body tiles, then 32-token dense tiles. Tiles are weighted by
// their HBM bytes, each segment start adds a fixed charge for its piece start and
// end, and the whole list (all units) is cut into one contiguous, equal-weight
// range per CTA of a persistent grid (one CTA per SM). A CTA's range is a short
// sequence of pieces: runs of tiles of one (unit, segment). Each piece ends in
// an un-normalised partial (m, l, O) for the unit's G query heads; the CTA that
// delivers a unit's last partial merges them.
//
// Pipeline. The loaded HBM latency on B200 is several microseconds, so an SM
// needs ~200 KB of reads in flight: the ring has an even number (up to 12) of
// slots, ten 20 KiB slots for fp16min group 32. Warps 8-9 issue the TMA copies
// (each CTA its own copies), each the loads of one parity: INT4 tiles as one 1-D bulk copy
// of their page block, dense tiles as one 5-D tensor copy per side with 128-byte
// swizzle. fp16min blocks are consumed as stored; for ref blocks warps 10-11
// first expand the group metadata in place into fp32 / f16x2 and zero what lies
// past the sequence length. Warps 0-7 are two consumer groups that take
// alternate tiles; each warp computes 32 tokens of a tile with m16n8k16
// tensor-core MMAs (N = 8 query heads, G <= 8 used):
//   S^T[tok][head] = K[tok][:] . Q^T      (M = 16 tokens, K = dims)
//   O^T[dim][head] += V^T[dim][tok] . P^T (M = 16 dims,   K = tokens)
// INT4 K and V fragments come straight from the packed nibbles (the page
// format's nibble order is the fragment order): a nibble OR-ed into the
// mantissa of 1024.0h is the exact f16 value 1024 + n (or 1024 + 16 n for a
// high nibble).
//   K: half of each k-tile is (1024 + n), half (1024 + 16 n) against Q/16, and
//      the accumulator starts at -1024 * sum(Q), so it ends at sum(n Q):
//      score = sum_g s_g * acc_g + b_g * sum(Q_g)        (b = -z*s or min)
//   V: codes are exact integers n (bias removed in f16), the B operand is
//      s * P / 16, so O = 16 * (acc + sum_t b_t P_t / 16).
// The online softmax is fp32 in the base-2 domain with a lazy rescale: the
// running max only moves (one warp-wide max reduction) when a score beats it by
// more than 2^8.
#pragma once
#include "hkv_common.cuh"

namespace hkv {

constexpr int kGroupWarps = 4;                      // warps per consumer group
constexpr int kConsumerWarps = 2 * kGroupWarps;     // two groups take alternate tiles
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kIssueWarp = kConsumerWarps;          // TMA issue, first of kIssueWarps
constexpr int kIssueWarps = 2;                      // issue warp w feeds the loads n with n % 2 == w
constexpr int kExpandWarp = kIssueWarp + kIssueWarps;  // HKV_FMT_REF metadata expansion, first of 2
// HKV_FMT_REF tiles get their metadata rewritten by two expansion warps (alternate
// tiles); HKV_FMT_FP16MIN blocks are stored in the layout the consumers read.
__host__ __device__ constexpr int expand_warps(int fmt) { return fmt == HKV_FMT_REF ? 2 : 0; }
// The fused decode-step append (APPEND instantiation) runs on warp kAppendWarp:
// a warp of its own for fp16min, the first expansion warp (before it starts
// expanding) for ref, whose 12 warps leave no registers for a 13th. (Run by an
// issue warp while its share of the ring fills, the append's chain of loaded
// round trips held back half the ring: a 32-layer step took 3.07 instead of
// 2.56 ms.)
constexpr int kAppendWarp = kIssueWarp + kIssueWarps;
__host__ __device__ constexpr int append_warps(int fmt, bool append) { return append && fmt != HKV_FMT_REF ? 1 : 0; }
__host__ __device__ constexpr int decode_threads(int fmt, bool append = false) {
  return (kConsumerWarps + kIssueWarps + expand_warps(fmt) + append_warps(fmt, append)) * 32;
}
// Arrivals per CTA on the grid-wide state counter in the APPEND instantiation,
// one by each role once it has read the cache state (sequence lengths, ring
// head) for the last time: the two issue warps, the consumers (as one), and
// the append job.
constexpr int kStateRoles = kIssueWarps + 2;
constexpr int kTileI4 = 128;  // tokens per INT4 tile (32 per consumer warp)
constexpr int kTileD = 32;    // tokens per dense tile (8 per consumer warp)
constexpr int kMaxSlots = 12;
constexpr int kSlotBytes = 24 * 1024;   // HKV_FMT_REF: one page block + expansion room
constexpr int kMetaOff = HKV_META_OFF;
constexpr float kLazyRescale = 8.0f;
// Longest sleep (ns) of one pending mbarrier try_wait: issue warps (waiting for a
// free slot) and consumer warps (waiting for a tile). A sleeping warp is woken by
// the phase completion, so the sleep only saves the spin loop's issue slots.
#ifndef HKV_ISSUE_SLEEP_NS
#define HKV_ISSUE_SLEEP_NS 2000
#endif
#ifndef HKV_CONS_SLEEP_NS
#define HKV_CONS_SLEEP_NS 0
#endif
constexpr int kDenseHalf = kTileD * 128;  // bytes of one 64-dim half of 32 dense rows (swizzled)

// Equal-byte partition of the tile list over the persistent grid.
// Positions are counted in 128-byte steps (every tile is a multiple of 128
// bytes) so that the schedule is 32-bit arithmetic in every warp.
constexpr int kSchedStep = 128;
struct Sched {
  int U;            // units (B * Hkv)
  int Tb, Td;       // body / dense tiles per unit (from the host-side length hints)
  int C;            // CTAs
  int S;            // partial slots per unit in the workspace
  uint32_t tb, td;  // steps per body / dense tile
  uint32_t wb, wd;  // steps charged before a unit's body / dense segment (piece start and end work)
  uint32_t Ub;      // steps per unit
  uint32_t Btot;    // steps in total (< 2^31)
  uint32_t q, r;    // Btot = q * C + r
};

struct DecodeParams {
  CUtensorMap tmk;  // dense K [B][Hkv][cap][128] as 5-D (dim in half, token, half, head, batch), box 64 x 32 x 2
  CUtensorMap tmv;
  const void* q;
  int q_dtype;
  int64_t q_sb, q_sh;
  int q_async;  // q rows 16-byte aligned: consumers prefetch the next piece's rows with cp.async
  hkv_int4_store body;
  hkv_dense_kv dense;
  int B, Hq, Hkv, G;
  float qscale;  // sm_scale * log2(e)
  Sched sc;
  int nslots;
  int page_shift;  // log2(page_tokens) when a power of two, else -1
  float* part_o;   // [U][S][G][128]  un-normalised partial outputs
  float* part_ml;  // [U][S][G][2]    (m, l), base-2 logits
  int* counters;   // [U]             zero before first use, self-resetting
  void* out;       // [B][Hq][128] out_dtype (normalised mode)
  int out_dtype;
  int64_t out_sb, out_sh;
  float* out_o;    // [B][Hq][128] f32 (partial mode, when non-null)
  float* out_ml;   // [B][Hq][2]
  // where the attention mass fell (optional, normalised mode): per INT4 body tile
  // k < stat_tiles of unit u, per consumer warp and head, (sum of the warp's
  // softmax numerators, running max) in tile_stats[u][k][warp][head][2]; the
  // unit's final (max, sum) per head in unit_ml[u][head][2]
  float* tile_stats;
  int stat_tiles;
  float* unit_ml;
  // fused decode-step append (APPEND instantiation): per (b, KV head) the new
  // token's K and V rows [B][Hkv][128] (the dense segment's dtype), the cache
  // state arrays (dense_len and body_len are dense.lengths and body.lengths),
  // and the grid-wide counter of state-reading roles (kStateRoles per CTA)
  const void* k_new;
  const void* v_new;
  int64_t new_sb, new_sh;
  int sink;
  int32_t* dense_len;
  int32_t* ring_head;
  int32_t* body_len;
  int* state_counter;
  int early;  // the cache may be read before griddep_wait (HKV_APPEND_EARLY)
};

// Records one body tile's share of the attention for the unit's heads (see
// DecodeParams::tile_stats). P: this thread's numerators (heads 2j + (i & 1)),
// pre-scaled by 1/16 as INT4 tiles carry them; m: the warp's running max.
__device__ __forceinline__ void record_tile_stats(const DecodeParams& p, int u, int k, int wg,
                                                  const float (&m)[2], const float (&P)[8]) {
  const int lane = threadIdx.x & 31, r = lane >> 2, j = lane & 3;
  float s0 = (P[0] + P[2]) + (P[4] + P[6]), s1 = (P[1] + P[3]) + (P[5] + P[7]);
#pragma unroll
  for (int sft = 4; sft < 32; sft <<= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, sft);
    s1 += __shfl_xor_sync(0xffffffffu, s1, sft);
  }
  if (r == 0)
    *reinterpret_cast<float4*>(p.tile_stats + ((((int64_t)u * p.stat_tiles + k) * 4 + wg) * 8 + 2 * j) * 2) =
        make_float4(16.f * s0, m[0], 16.f * s1, m[1]);
}

// An INT4 tile is one 128-token page block, copied as is: K codes | V codes |
// metadata. The consumers read fp16min metadata as stored (f16: K scales
// [128][NG] | K mins | V scales [64 pairs][NG][2] | V mins). Ref metadata (K
// scales f32 [128][NG] | V scales | K zps u8 [128][NG] | V zps) is first expanded
// in place, with N = 128 NG entries, into these byte ranges:
//   [0, 4N) K scale * qs, f32 [128][NG] | [4N, 8N) K bias -z*s f32 [128][NG] |
//   [10N, 14N) V zero-point constants [64 pairs][NG][2] f16x2 |
//   [14N, 16N) V scale pairs f16x2 [64][NG] (tokens 2p, 2p+1)
// Every expanded entry lands either on the raw entry of the same index (read
// by the same lane just before) or past all raw data: a lane never overwrites
// raw bytes another lane has yet to read.
__host__ __device__ constexpr int dense_slot_bytes() { return 4 * kDenseHalf; }
// Ring slot size: a page block (HKV_FMT_FP16MIN: as stored; HKV_FMT_REF: with room
// for the expanded metadata) or a dense tile, in whole KiB (the dense tiles'
// 128-byte swizzle repeats every 1024 bytes).
__host__ __device__ constexpr int slot_bytes(int fmt, int group) {
  return fmt == HKV_FMT_REF ? kSlotBytes
                            : ((block_bytes(fmt, group) > dense_slot_bytes() ? block_bytes(fmt, group)
                                                                              : dense_slot_bytes()) + 1023) / 1024 * 1024;
}
static_assert(kMetaOff + 16 * kTileI4 * 4 <= kSlotBytes && 12 * kTileI4 * 4 + 1024 <= 16 * kTileI4 * 4,
              "expanded metadata (g32) must fit its slot");
static_assert(2 * kTileI4 * HKV_CODE_BYTES == kMetaOff && dense_slot_bytes() <= kSlotBytes, "slot layout");
static_assert(kTileI4 == HKV_BLOCK_TOKENS && block_bytes(HKV_FMT_REF, 32) <= kSlotBytes, "a tile is one page block");

// ---------------------------------------------------------------- schedule arithmetic (per piece, not per tile)
// CTA c owns steps [floor(c Btot / C), floor((c+1) Btot / C)); c*r < C^2 fits 32 bits.
__device__ __forceinline__ uint32_t cta_begin(const Sched& s, int c) {
  return (uint32_t)c * s.q + ((uint32_t)c * s.r) / (uint32_t)s.C;
}
// First step of tile k of segment seg of unit u. A unit is [wb | Tb body tiles | wd | Td dense tiles].
__device__ __forceinline__ uint32_t tile_byte(const Sched& s, int u, int seg, int k) {
  return (uint32_t)u * s.Ub + s.wb +
         (seg == 0 ? (uint32_t)k * s.tb : (uint32_t)s.Tb * s.tb + s.wd + (uint32_t)k * s.td);
}
// The CTA whose range holds step x: a float estimate, then exact corrections.
__device__ __forceinline__ int owner_of(const Sched& s, uint32_t x) {
  int c = min(s.C - 1, (int)((float)x * (float)s.C / (float)s.Btot));
  while (c > 0 && cta_begin(s, c) > x) --c;
  while (c + 1 < s.C && cta_begin(s, c + 1) <= x) ++c;
  return c;
}

// A piece: tiles [k0, k1) of segment seg of unit u (k1 includes tiles past the
// hint when the true length needs them); tiles at or past kd hold no tokens.
// skip: a dense row the piece must leave out (-1: none), the ring row the fused
// append overwrites in this launch.
struct Piece {
  int u, seg, k0, k1, kd, len, skip;
  bool valid;
};

__device__ __forceinline__ int seg_len(const DecodeParams& p, int u, int seg) {
  const int b = u / p.Hkv;
  if (seg == 0) return p.body.lengths ? p.body.lengths[b] : p.body.len;
  return p.dense.lengths ? p.dense.lengths[b] : p.dense.len;
}
// (length, skipped row) of a segment. With the fused append the attention runs
// over the state before the append: the body without the evicted token and the
// dense segment without the ring row being overwritten (when the ring is full);
// the append warp's own partial covers the evicted token and the new one.
template <bool APPEND>
__device__ __forceinline__ int2 seg_state(const DecodeParams& p, int u, int seg) {
  if (!APPEND || seg == 0) return make_int2(seg_len(p, u, seg), -1);
  // both loads in one round trip (the ring head is read whether or not it is used)
  const int b = u / p.Hkv, cap = p.dense.capacity;
  const int len = p.dense_len[b], head = p.ring_head[b];
  return make_int2(len, len >= cap && cap > p.sink ? p.sink + head : -1);
}

__device__ __forceinline__ void piece_fill_len(const DecodeParams& p, uint32_t end, Piece& pc, int len) {
  const Sched& s = p.sc;
  const int T = pc.seg == 0 ? s.Tb : s.Td;
  const uint32_t ts = pc.seg == 0 ? s.tb : s.td;
  const int tile = pc.seg == 0 ? kTileI4 : kTileD;
  const uint32_t seg0 = tile_byte(s, pc.u, pc.seg, 0);
  const uint32_t kq = (end - 1 - seg0) / ts;
  const int kl = kq < (uint32_t)(T - 1) ? (int)kq : T - 1;  // last hinted tile starting in range
  pc.len = len;
  pc.skip = -1;
  const int kneed = (pc.len + tile - 1) / tile;
  pc.k1 = kl + 1;
  // past its last hinted tile a segment continues while the true length needs it
  // (a stale hint can unbalance the grid, never drop tokens)
  if (kl == T - 1 && kneed > pc.k1) pc.k1 = kneed;
  pc.kd = min(pc.k1, kneed);
}
__device__ __forceinline__ void piece_fill(const DecodeParams& p, uint32_t end, Piece& pc) {
  piece_fill_len(p, end, pc, seg_len(p, pc.u, pc.seg));
}

// The CTA's first piece without its length-dependent fields (see piece_fill_len).
__device__ __forceinline__ Piece first_piece_head(const DecodeParams& p, int c, uint32_t end) {
  const Sched& s = p.sc;
  const uint32_t x = cta_begin(s, c);
  Piece pc;
  pc.u = (int)(x / s.Ub);
  const uint32_t r = x - (uint32_t)pc.u * s.Ub;
  const uint32_t db = s.wb + (uint32_t)s.Tb * s.tb + s.wd;  // first dense step of the unit
  if (s.Tb > 0 && r <= s.wb + (uint32_t)(s.Tb - 1) * s.tb) {
    pc.seg = 0;
    // r may lie inside the charge before the body
    pc.k0 = r > s.wb ? (int)((r - s.wb + s.tb - 1) / s.tb) : 0;
  } else if (s.Td > 0 && r <= db + (uint32_t)(s.Td - 1) * s.td) {
    pc.seg = 1;
    // r may lie inside the last body tile or the charge before the dense segment
    pc.k0 = r > db ? (int)((r - db + s.td - 1) / s.td) : 0;
  } else {
    pc.u += 1;
    pc.seg = s.Tb > 0 ? 0 : 1;
    pc.k0 = 0;
  }
  pc.valid = pc.u < s.U && tile_byte(s, pc.u, pc.seg, pc.k0) < end;
  return pc;
}

// The piece after pc without its length-dependent fields (u, seg, k0, valid only).
__device__ __forceinline__ void next_piece_head(const DecodeParams& p, uint32_t end, Piece& pc) {
  const Sched& s = p.sc;
  const int T = pc.seg == 0 ? s.Tb : s.Td;
  if (pc.k1 < T) {  // the range ended inside this segment
    pc.valid = false;
    return;
  }
  if (pc.seg == 0 && s.Td > 0) {
    pc.seg = 1;
  } else {
    pc.u++;
    pc.seg = s.Tb > 0 ? 0 : 1;
  }
  pc.k0 = 0;
  pc.valid = pc.u < s.U && tile_byte(s, pc.u, pc.seg, 0) < end;
}
__device__ __forceinline__ void next_piece(const DecodeParams& p, uint32_t end, Piece& pc) {
  next_piece_head(p, end, pc);
  if (pc.valid) piece_fill(p, end, pc);
}

// Partials of unit u: one per CTA owning its body tiles, then per CTA owning its dense tiles.
__device__ __forceinline__ void unit_pieces(const Sched& s, int u, int& b0, int& nb, int& d0, int& nd) {
  nb = nd = 0;
  b0 = d0 = 0;
  if (s.Tb > 0) {
    b0 = owner_of(s, tile_byte(s, u, 0, 0));
    nb = owner_of(s, tile_byte(s, u, 0, s.Tb - 1)) - b0 + 1;
  }
  if (s.Td > 0) {
    d0 = owner_of(s, tile_byte(s, u, 1, 0));
    nd = owner_of(s, tile_byte(s, u, 1, s.Td - 1)) - d0 + 1;
  }
}

// Ring position: slot index and the parity of its current use.
struct Ring {
  int slot;
  uint32_t phase;
  __device__ __forceinline__ void advance(int n) {
    if (++slot == n) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// ---------------------------------------------------------------- warp state / softmax
// Thread (r = lane/4, j = lane%4) owns heads 2j and 2j+1 in every accumulator.
// The running max starts at a finite "no score yet" value, so that 2^(x - m)
// is 0 for a masked score (x = -inf) and never NaN, without a test per score.
constexpr float kNoMax = -1.0e30f;

template <int NG>
struct WarpState {
  float o[8][4];      // O^T, m-tile mt: (dim 16mt+r | 16mt+r+8) x (head 2j | 2j+1)
  float zc[4];        // fp16min INT4: sum_t min_r(t) P(t)/16 for group r (lanes r < NG), heads 2j, 2j+1
  float m[2];         // running max (base-2 logits)
  float mo[2];        // m + log2 of the P pre-scale (4 for INT4: P/16; 0 for dense)
  float l[2];         // sum of the pre-scaled P
};

template <int NG>
__device__ __forceinline__ void ws_reset(WarpState<NG>& ws) {
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) ws.o[mt][0] = ws.o[mt][1] = ws.o[mt][2] = ws.o[mt][3] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ws.zc[i] = 0.f;
  ws.m[0] = ws.m[1] = ws.mo[0] = ws.mo[1] = kNoMax;
  ws.l[0] = ws.l[1] = 0.f;
}

// One online-softmax step over this thread's scores x (x[i] belongs to head
// 2j + (i & 1); -inf = masked). The max moves only when some score beats it by
// more than kLazyRescale, so the common step needs one vote and no cross-lane
// max reduction. P = 2^(x - m - off) stays below 2^(8 - off).
template <int NG, int N>
__device__ __forceinline__ void softmax_step(WarpState<NG>& ws, const float (&x)[N], float (&P)[N], float off) {
  const float th0 = ws.m[0] + kLazyRescale, th1 = ws.m[1] + kLazyRescale;
  bool need = false;
#pragma unroll
  for (int i = 0; i < N; i += 2) need |= (x[i] > th0) | (x[i + 1] > th1);
  if (__any_sync(0xffffffffu, need)) {
    float t0 = x[0], t1 = x[1];
#pragma unroll
    for (int i = 2; i < N; i += 2) {
      t0 = fmaxf(t0, x[i]);
      t1 = fmaxf(t1, x[i + 1]);
    }
#pragma unroll
    for (int s = 4; s < 32; s <<= 1) {
      t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, s));
      t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, s));
    }
    const float n0 = fmaxf(ws.m[0], t0), n1 = fmaxf(ws.m[1], t1);
    const float a0 = fast_exp2(ws.m[0] - n0), a1 = fast_exp2(ws.m[1] - n1);
    ws.m[0] = n0;
    ws.m[1] = n1;
    ws.mo[0] = n0 + off;
    ws.mo[1] = n1 + off;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      ws.o[mt][0] *= a0;
      ws.o[mt][1] *= a1;
      ws.o[mt][2] *= a0;
      ws.o[mt][3] *= a1;
    }
    ws.zc[0] *= a0;
    ws.zc[1] *= a1;
    ws.zc[2] *= a0;
    ws.zc[3] *= a1;
    ws.l[0] *= a0;
    ws.l[1] *= a1;
  }
#pragma unroll
  for (int i = 0; i < N; ++i) P[i] = fast_exp2(x[i] - ws.mo[i & 1]);
#pragma unroll
  for (int i = 0; i < N; i += 2) {
    ws.l[0] += P[i];
    ws.l[1] += P[i + 1];
  }
}

// ---------------------------------------------------------------- INT4 consumer pieces
template <int NG>
__device__ __forceinline__ void ld_row(const float* base, int row, float (&v)[NG]) {
  if constexpr (NG == 4) {
    const float4 t = *reinterpret_cast<const float4*>(base + row * 4);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  } else if constexpr (NG == 2) {
    const float2 t = *reinterpret_cast<const float2*>(base + row * 2);
    v[0] = t.x;
    v[1] = t.y;
  } else {
    v[0] = base[row];
  }
}
template <int NG>
__device__ __forceinline__ void ld_row_u(const uint32_t* base, int row, uint32_t (&v)[NG]) {
  if constexpr (NG == 4) {
    const uint4 t = *reinterpret_cast<const uint4*>(base + row * 4);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  } else if constexpr (NG == 2) {
    const uint2 t = *reinterpret_cast<const uint2*>(base + row * 2);
    v[0] = t.x;
    v[1] = t.y;
  } else {
    v[0] = base[row];
  }
}

template <int NG>
__device__ __forceinline__ void ld_row_h(const __half* base, int row, float (&v)[NG]) {
  if constexpr (NG == 4) {
    const uint2 t = *reinterpret_cast<const uint2*>(base + row * 4);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&t.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&t.y));
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  } else if constexpr (NG == 2) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(base + row * 2));
    v[0] = a.x;
    v[1] = a.y;
  } else {
    v[0] = __half2float(base[row]);
  }
}

// Scores of 16 tokens x 8 heads: x = {(r,2j), (r,2j+1), (r+8,2j), (r+8,2j+1)}
// in base-2 logits. kc points at this thread's row r of the tile's K codes, mb at
// the tile's metadata, t at the subtile's first token in the tile. The group
// bias term sum_g b_g * sum(Q_g):
//   ref:     expanded metadata, K scale * qs and b = -z*s in fp32, one FMA per
//            group (qsum carries qs);
//   fp16min: the block's own f16 metadata; b = min, one extra MMA of A = mins
//            [token][group, twice] against B = sum(Q_g) split into f16 hi + lo
//            parts (qbias), so every product is exact and the sum is fp32;
//            qs is applied once at the end.
template <int FMT, int NG>
__device__ __forceinline__ void k_scores(const uint8_t* kc, const uint8_t* mb, int t, const uint32_t (&qf)[8][2],
                                         const float (&nbias)[NG][2], const float (&qsum)[NG][2],
                                         uint32_t qbias, float qs, float (&x)[4]) {
  constexpr int WPG = 4 / NG;  // packed words per group
  const int lane = threadIdx.x & 31, r = lane >> 2, j = lane & 3;
  const uint4 kA = *reinterpret_cast<const uint4*>(kc);
  const uint4 kB = *reinterpret_cast<const uint4*>(kc + 8 * HKV_CODE_BYTES);
  const uint32_t kwa[4] = {kA.x, kA.y, kA.z, kA.w};
  const uint32_t kwb[4] = {kB.x, kB.y, kB.z, kB.w};
  float sA[NG], sB[NG], bA[NG], bB[NG];
  x[0] = x[1] = x[2] = x[3] = 0.f;
  if constexpr (FMT == HKV_FMT_REF) {
    const float* ks = reinterpret_cast<const float*>(mb) + (t + r) * NG;
    const float* kb = reinterpret_cast<const float*>(mb + 4 * kTileI4 * NG) + (t + r) * NG;
    ld_row<NG>(ks, 0, sA);
    ld_row<NG>(ks, 8, sB);
    ld_row<NG>(kb, 0, bA);
    ld_row<NG>(kb, 8, bB);
  } else {
    const __half* ks = reinterpret_cast<const __half*>(mb) + (t + r) * NG;
    ld_row_h<NG>(ks, 0, sA);
    ld_row_h<NG>(ks, 8, sB);
    // A columns 2j, 2j+1 of the bias MMA (rows r and r + 8) meet qbias rows 2j,
    // 2j+1 (f16 hi parts of sum(Q_g) in rows 0..NG-1, lo parts in NG..2NG-1):
    // NG 4: (min_g0, min_g1), (min_g2, min_g3), twice; NG 2: (min_g0, min_g1)
    // twice; NG 1: (min, min)
    const uint8_t* kmin = mb + 256 * NG + t * NG * 2;
    uint32_t m0 = 0u, m1 = 0u;
    if constexpr (NG == 4) {
      m0 = reinterpret_cast<const uint32_t*>(kmin)[2 * r + (j & 1)];
      m1 = reinterpret_cast<const uint32_t*>(kmin)[2 * (r + 8) + (j & 1)];
    } else if constexpr (NG == 2) {
      if (j < 2) {
        m0 = reinterpret_cast<const uint32_t*>(kmin)[r];
        m1 = reinterpret_cast<const uint32_t*>(kmin)[r + 8];
      }
    } else {
      if (j == 0) {
        m0 = reinterpret_cast<const uint16_t*>(kmin)[r] * 0x10001u;
        m1 = reinterpret_cast<const uint16_t*>(kmin)[r + 8] * 0x10001u;
      }
    }
    const uint32_t ab[4] = {m0, m1, 0u, 0u};
    mma16816<__half>(x, ab, qbias, 0u);
  }
  float c[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int g = w / WPG;
    const uint32_t xa8 = kwa[w] >> 8, xb8 = kwb[w] >> 8;
    const uint32_t a0[4] = {biased1(kwa[w]), biased1(kwb[w]), biased16(kwa[w]), biased16(kwb[w])};
    const uint32_t a1[4] = {biased1(xa8), biased1(xb8), biased16(xa8), biased16(xb8)};
    if (w % WPG == 0) {
      const float ci[4] = {nbias[g][0], nbias[g][1], nbias[g][0], nbias[g][1]};
      mma16816_c(c, a0, qf[2 * w][0], qf[2 * w][1], ci);
    } else {
      mma16816<__half>(c, a0, qf[2 * w][0], qf[2 * w][1]);
    }
    mma16816<__half>(c, a1, qf[2 * w + 1][0], qf[2 * w + 1][1]);
    if (w % WPG == WPG - 1) {
      if constexpr (FMT == HKV_FMT_REF) {
        x[0] = fmaf(sA[g], c[0], fmaf(bA[g], qsum[g][0], x[0]));
        x[1] = fmaf(sA[g], c[1], fmaf(bA[g], qsum[g][1], x[1]));
        x[2] = fmaf(sB[g], c[2], fmaf(bB[g], qsum[g][0], x[2]));
        x[3] = fmaf(sB[g], c[3], fmaf(bB[g], qsum[g][1], x[3]));
      } else {
        x[0] = fmaf(sA[g], c[0], x[0]);
        x[1] = fmaf(sA[g], c[1], x[1]);
        x[2] = fmaf(sB[g], c[2], x[2]);
        x[3] = fmaf(sB[g], c[3], x[3]);
      }
    }
  }
  if constexpr (FMT == HKV_FMT_FP16MIN) {
    x[0] *= qs;
    x[1] *= qs;
    x[2] *= qs;
    x[3] *= qs;
  }
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// 8 nibbles of x -> 4 f16x2 of the exact integers n - z, with per-half zero
// points: zlo = (1024 + z_lo, 1024 + z_hi) and zhi = (-64 - z_lo, -64 - z_hi)
// (as nib8_to_h2, whose constants are the z = 0 case).
__device__ __forceinline__ void nib8_to_h2_z(uint32_t x, uint32_t zlo, uint32_t zhi, uint32_t (&h)[4]) {
  constexpr uint32_t kMagic = 0x64006400u;  // (1024, 1024)
  constexpr uint32_t kInv16 = 0x2C002C00u;  // (1/16, 1/16)
  const uint32_t e0 = lop3<0xEA>(x, 0x000F000Fu, kMagic);
  const uint32_t e1 = lop3<0xEA>(x, 0x00F000F0u, kMagic);
  const uint32_t x8 = x >> 8;
  const uint32_t e2 = lop3<0xEA>(x8, 0x000F000Fu, kMagic);
  const uint32_t e3 = lop3<0xEA>(x8, 0x00F000F0u, kMagic);
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[0]) : "r"(e0), "r"(zlo));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[1]) : "r"(e1), "r"(kInv16), "r"(zhi));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[2]) : "r"(e2), "r"(zlo));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[3]) : "r"(e3), "r"(kInv16), "r"(zhi));
}

// O^T += V^T . (s P/16)^T for 16 tokens; P = {(r,2j), (r,2j+1), (r+8,2j), (r+8,2j+1)}
// pre-scaled by 1/16. vc points at this thread's V chunk (pair j, chunk r), vsp
// at the subtile's V scale pairs (pair 0 = its tokens 0, 1), [pair][NG] f16x2.
// P is transposed once into the B layout (token pair 2j, 2j+1 of head r) and
// multiplied by the pair's per-group scales there. The group bias:
//   ref:     codes enter as exact n - z (vz: per pair and group the two
//            zero-point constants of nib8_to_h2_z), so no bias term remains;
//   fp16min: zc += mins [group][token] . P^T, one extra MMA (vz: min pairs).
// fp16min metadata of tokens at or past nv (< 16: the sequence ends inside the
// subtile) may hold any bits and is zeroed, so that P = 0 meets 0, never NaN.
template <int FMT, int NG>
__device__ __forceinline__ void v_accumulate(WarpState<NG>& ws, const uint8_t* vc, const uint32_t* vsp,
                                             const uint32_t* vz, const float (&P)[4], int nv) {
  constexpr int WPG = 4 / NG;
  const int lane = threadIdx.x & 31, r = lane >> 2, j = lane & 3;
  uint32_t sA[NG], sB[NG];
  ld_row_u<NG>(vsp, j, sA);
  ld_row_u<NG>(vsp, 4 + j, sB);
  const uint32_t tA = movmatrix_t(pack2<__half>(P[0], P[1]));
  const uint32_t tB = movmatrix_t(pack2<__half>(P[2], P[3]));
  if constexpr (FMT == HKV_FMT_FP16MIN) {
    uint32_t zA = r < NG ? vz[j * NG + r] : 0u, zB = r < NG ? vz[(4 + j) * NG + r] : 0u;
    if (nv < 16) {
      // keep the halves of tokens t, t + 1 of a pair that lie before nv
      auto keep = [nv](uint32_t w, int t) {
        return w & ((t < nv ? 0x0000FFFFu : 0u) | (t + 1 < nv ? 0xFFFF0000u : 0u));
      };
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        sA[g] = keep(sA[g], 2 * j);
        sB[g] = keep(sB[g], 8 + 2 * j);
      }
      zA = keep(zA, 2 * j);
      zB = keep(zB, 8 + 2 * j);
    }
    const uint32_t ab[4] = {zA, 0u, zB, 0u};
    mma16816<__half>(ws.zc, ab, tA, tB);
  }
  uint32_t pb[NG][2];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    pb[g][0] = hmul2(tA, sA[g]);
    pb[g][1] = hmul2(tB, sB[g]);
  }
  const uint4 vA = *reinterpret_cast<const uint4*>(vc);
  const uint4 vB = *reinterpret_cast<const uint4*>(vc + 8 * HKV_CODE_BYTES);
  const uint32_t vwa[4] = {vA.x, vA.y, vA.z, vA.w};
  const uint32_t vwb[4] = {vB.x, vB.y, vB.z, vB.w};
  // exact integer codes: the B operand carries s * P rounded to f16, so a bias
  // left in A would cancel against fp32 sums of differently rounded products
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int g = k / WPG;
    uint32_t ha[4], hb[4];
    if constexpr (FMT == HKV_FMT_REF) {
      const uint2 za = *reinterpret_cast<const uint2*>(vz + 2 * (j * NG + g));
      const uint2 zb = *reinterpret_cast<const uint2*>(vz + 2 * ((4 + j) * NG + g));
      nib8_to_h2_z(vwa[k], za.x, za.y, ha);
      nib8_to_h2_z(vwb[k], zb.x, zb.y, hb);
    } else {
      nib8_to_h2(vwa[k], ha);
      nib8_to_h2(vwb[k], hb);
    }
    const uint32_t a0[4] = {ha[0], ha[1], hb[0], hb[1]};
    const uint32_t a1[4] = {ha[2], ha[3], hb[2], hb[3]};
    mma16816<__half>(ws.o[2 * k], a0, pb[g][0], pb[g][1]);
    mma16816<__half>(ws.o[2 * k + 1], a1, pb[g][0], pb[g][1]);
  }
}

// ---------------------------------------------------------------- dense consumer piece (8 tokens per warp)
// A dense slot holds 32 rows of K then 32 rows of V, each split in two 64-dim
// halves of [32 rows][128 B] written by TMA with the 128-byte swizzle: the
// 16-byte chunk c of row i sits at i*128 + ((c ^ (i & 7)) << 4).
__device__ __forceinline__ uint32_t swz(uint32_t half_base, int row, int chunk) {
  return half_base + row * 128 + (((chunk ^ (row & 7)) & 7) << 4);
}

template <typename DTy, int NG>
__device__ __forceinline__ void dense_subtile(WarpState<NG>& ws, uint32_t slot, int t0, bool ok,
                                              const uint32_t (&qf)[8][2], float qscale) {
  const int lane = threadIdx.x & 31;
  const int row = t0 + (lane & 7);  // rows r+8 of the 16-row fragments repeat rows r and are masked
  float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kt = 0; kt < 8; ++kt) {
    uint32_t a[4];
    ldsm_x4(a, swz(slot + (kt >> 2) * kDenseHalf, row, 2 * (kt & 3) + (lane >> 4)));
    mma16816<DTy>(c, a, qf[kt][0], qf[kt][1]);
  }
  float x[4];
  x[0] = ok ? c[0] * qscale : -INFINITY;
  x[1] = ok ? c[1] * qscale : -INFINITY;
  x[2] = -INFINITY;
  x[3] = -INFINITY;
  float P[4];
  softmax_step<NG, 4>(ws, x, P, 0.f);
  const uint32_t pb0 = movmatrix_t(pack2<DTy>(P[0], P[1]));
  const uint32_t vb = slot + 2 * kDenseHalf;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    uint32_t a[4];
    ldsm_x4_t(a, swz(vb + (mt >> 2) * kDenseHalf, row, 2 * (mt & 3) + ((lane >> 3) & 1)));
    mma16816<DTy>(ws.o[mt], a, pb0, 0u);
  }
}

// Q^T B fragments for this lane: head r (= lane/4), dims 16kt + 2j + {0,1} in
// qf[kt][0] and 16kt + 2j + {8,9} in qf[kt][1] (divided by 16 when hi_div16).
// qa/qb return the values exactly as the tensor core sees them. Heads r >= G
// get Q = 0: their scores are finite and their results are never stored.
// The rows come from global memory, or (qs != nullptr) from the G x 128 copy of
// them in shared memory that the consumers prefetched.
template <typename T>
__device__ __forceinline__ void load_q_frags(const DecodeParams& p, int b, int hk, bool hi_div16, const void* qs,
                                             uint32_t (&qf)[8][2], float (&qa)[8][2], float (&qb)[8][2]) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const bool live = r < p.G;
  const int hq = hk * p.G + (live ? r : 0);
  const void* src = qs ? qs : p.q;
  const int64_t base = qs ? (int64_t)(live ? r : 0) * HKV_D : (int64_t)b * p.q_sb + (int64_t)hq * p.q_sh;
  const float sc = hi_div16 ? 0.0625f : 1.0f;
#pragma unroll
  for (int kt = 0; kt < 8; ++kt) {
    const int d = 16 * kt + 2 * j;
    float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
    if (live) {
      v0 = load_any(src, p.q_dtype, base + d);
      v1 = load_any(src, p.q_dtype, base + d + 1);
      v2 = load_any(src, p.q_dtype, base + d + 8);
      v3 = load_any(src, p.q_dtype, base + d + 9);
    }
    const float r0 = to_f32(from_f32<T>(v0)), r1 = to_f32(from_f32<T>(v1));
    const float r2 = to_f32(from_f32<T>(to_f32(from_f32<T>(v2)) * sc));
    const float r3 = to_f32(from_f32<T>(to_f32(from_f32<T>(v3)) * sc));
    qf[kt][0] = pack2<T>(r0, r1);
    qf[kt][1] = pack2<T>(r2, r3);
    qa[kt][0] = r0;
    qa[kt][1] = r1;
    qb[kt][0] = r2;
    qb[kt][1] = r3;
  }
}

__device__ __forceinline__ int q_elem_bytes(int dtype) { return dtype == HKV_DT_F32 ? 4 : 2; }

// Consumer threads copy unit u's G query rows (G x 128 elements) into qbuf with
// cp.async, 16 bytes per thread; the caller waits (cp.async.wait_all + a consumer
// barrier) before reading them. Requires p.q_async (16-byte aligned rows).
__device__ __forceinline__ void q_prefetch(const DecodeParams& p, int u, uint8_t* qbuf) {
  const int b = u / p.Hkv, hk = u - b * p.Hkv;
  const int es = q_elem_bytes(p.q_dtype);
  const int chunks = (HKV_D * es) / 16;  // per row
  const int t = threadIdx.x;
  if (t < p.G * chunks) {
    const int row = t / chunks, ch = t - row * chunks;
    const uint8_t* src = static_cast<const uint8_t*>(p.q) +
                         ((int64_t)b * p.q_sb + (int64_t)(hk * p.G + row) * p.q_sh) * es + ch * 16;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(qbuf + row * HKV_D * es + ch * 16)),
                 "l"(src)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ int atom_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// Named barrier 1 over the consumer warps only (the TMA and expansion warps never join it).
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory"); }
// Same barrier, returning whether v held on every consumer thread.
__device__ __forceinline__ bool consumer_sync_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kConsumerThreads)
      : "memory");
  return r != 0;
}

// Bounded mbarrier wait with a warp-uniform outcome: lanes that reach the
// timeout at different moments must not split the warp before the next
// warp-synchronous instruction (mma.sync, shuffles, movmatrix).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t sleep_ns = 0) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, sleep_ns));
}

// One tiled TMA load of a 5-D box (coordinates innermost first; x = 0 here, so
// the 16-byte rule on the innermost coordinate holds), into this CTA alone.
__device__ __forceinline__ void tma_tile_5d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w, int v,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], "
      "[%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- metadata expansion (warps kExpandWarp..)
// Expands one HKV_FMT_REF tile's metadata in place (layout above), streaming:
// lane L handles entries 128 it + 4 L + {0..3} ([token][group] order) one
// iteration at a time. Tokens at or past `valid` (beyond the sequence length)
// may hold uninitialised pool bytes: their scale and bias become 0, so a masked
// token (P = 0) contributes exactly 0 and never NaN. The K scale is multiplied
// by qs (sm_scale * log2 e) so scores come out as base-2 logits.
template <int NG>
__device__ __forceinline__ void expand_meta(uint8_t* meta, int lane, int valid, float qs) {
  constexpr int N = kTileI4 * NG;
  constexpr int IT = N / 128;
  uint32_t* vsp = reinterpret_cast<uint32_t*>(meta + 14 * N);  // [64 pairs][NG] f16x2 scales
  uint32_t* vzc = reinterpret_cast<uint32_t*>(meta + 10 * N);  // [64][NG][2] zero-point constants
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int e = 128 * it + 4 * lane;
    float sk[4], bk[4], sv[4], zf[4];
    {
      const float4 a = *reinterpret_cast<const float4*>(meta + 4 * e);
      const float4 c = *reinterpret_cast<const float4*>(meta + 4 * N + 4 * e);
      const uint32_t zk = *reinterpret_cast<const uint32_t*>(meta + 8 * N + e);
      const uint32_t zv = *reinterpret_cast<const uint32_t*>(meta + 9 * N + e);
      const float av[4] = {a.x, a.y, a.z, a.w}, cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sk[i] = av[i];
        sv[i] = cv[i];
        bk[i] = -static_cast<float>((zk >> (8 * i)) & 0xffu) * av[i];
        zf[i] = static_cast<float>((zv >> (8 * i)) & 0xffu);
        if ((e + i) / NG >= valid) sk[i] = bk[i] = sv[i] = zf[i] = 0.f;
      }
    }
    *reinterpret_cast<float4*>(meta + 4 * e) = make_float4(sk[0] * qs, sk[1] * qs, sk[2] * qs, sk[3] * qs);
    *reinterpret_cast<float4*>(meta + 4 * N + 4 * e) = make_float4(bk[0], bk[1], bk[2], bk[3]);
    // pairs (tokens 2p, 2p+1): scales and zero-point constants
    if constexpr (NG == 4) {
      // lane holds token t = 32 it + lane, groups 0..3; its pair partner is lane ^ 1
      float os[4], oz[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        os[i] = __shfl_xor_sync(0xffffffffu, sv[i], 1);
        oz[i] = __shfl_xor_sync(0xffffffffu, zf[i], 1);
      }
      const int t = 32 * it + lane;
      if ((lane & 1) == 0) {
        const int pair = t >> 1;
        *reinterpret_cast<uint4*>(vsp + pair * 4) =
            make_uint4(pack2<__half>(sv[0], os[0]), pack2<__half>(sv[1], os[1]), pack2<__half>(sv[2], os[2]),
                       pack2<__half>(sv[3], os[3]));
        uint32_t w[8];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          w[2 * g] = pack2<__half>(1024.f + zf[g], 1024.f + oz[g]);
          w[2 * g + 1] = pack2<__half>(-64.f - zf[g], -64.f - oz[g]);
        }
        *reinterpret_cast<uint4*>(vzc + pair * 8) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(vzc + pair * 8 + 4) = make_uint4(w[4], w[5], w[6], w[7]);
      }
    } else if constexpr (NG == 2) {
      // entries: (t, g0), (t, g1), (t+1, g0), (t+1, g1) with t = 64 it + 2 lane
      const int pair = 32 * it + lane;
      *reinterpret_cast<uint2*>(vsp + pair * 2) = make_uint2(pack2<__half>(sv[0], sv[2]), pack2<__half>(sv[1], sv[3]));
      *reinterpret_cast<uint4*>(vzc + pair * 4) =
          make_uint4(pack2<__half>(1024.f + zf[0], 1024.f + zf[2]), pack2<__half>(-64.f - zf[0], -64.f - zf[2]),
                     pack2<__half>(1024.f + zf[1], 1024.f + zf[3]), pack2<__half>(-64.f - zf[1], -64.f - zf[3]));
    } else {
      // tokens 4 lane .. 4 lane + 3: pairs 2 lane, 2 lane + 1
      *reinterpret_cast<uint2*>(vsp + 2 * lane) = make_uint2(pack2<__half>(sv[0], sv[1]), pack2<__half>(sv[2], sv[3]));
      *reinterpret_cast<uint4*>(vzc + 4 * lane) =
          make_uint4(pack2<__half>(1024.f + zf[0], 1024.f + zf[1]), pack2<__half>(-64.f - zf[0], -64.f - zf[1]),
                     pack2<__half>(1024.f + zf[2], 1024.f + zf[3]), pack2<__half>(-64.f - zf[2], -64.f - zf[3]));
    }
  }
  // order these generic-proxy writes before later TMA (async-proxy) writes to the slot
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Zero dense V rows [r0, r1) of a swizzled slot (whole 128-byte rows, so the
// swizzle does not matter); rows past the sequence length may hold any bits.
// The fence orders these generic-proxy writes before later TMA writes to the slot.
__device__ __forceinline__ void zero_dense_v_rows(uint8_t* slot, int r0, int r1, int lane) {
  uint8_t* v = slot + 2 * kDenseHalf;
  for (int i = lane; i < (r1 - r0) * 16; i += 32) {  // 2 halves x 8 chunks of 16 B per row
    const int rr = r0 + i / 16, h = (i >> 3) & 1, ch = i & 7;
    *reinterpret_cast<uint4*>(v + h * kDenseHalf + rr * 128 + ch * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void zero_dense_v_tail(uint8_t* slot, int valid, int lane) {
  if (valid < kTileD) zero_dense_v_rows(slot, valid, kTileD, lane);
}

// Cursor over the CTA's tiles that hold tokens (the loads, in ring order).
struct Cursor {
  Piece pc;
  int k;
  bool valid;
};
__device__ __forceinline__ void cursor_settle(const DecodeParams& p, uint32_t end, Cursor& cu) {
  while (cu.pc.valid && cu.k >= cu.pc.kd) {
    next_piece(p, end, cu.pc);
    cu.k = cu.pc.k0;
  }
  cu.valid = cu.pc.valid;
}
__device__ __forceinline__ void cursor_start(const DecodeParams& p, uint32_t end, const Piece& first, Cursor& cu) {
  cu.pc = first;
  cu.k = cu.pc.k0;
  cursor_settle(p, end, cu);
}
__device__ __forceinline__ void cursor_next(const DecodeParams& p, uint32_t end, Cursor& cu) {
  cu.k++;
  cursor_settle(p, end, cu);
}

// ---------------------------------------------------------------- merge of a unit's partials
// One warp merges head h of unit u over its n partials (slots 0..n-1 of the
// unit in the workspace) and writes the output row (or, in partial mode, the
// merged un-normalised partial). Partials are read from L2 (__ldcg): other CTAs
// wrote them, ordered by the unit counter's release / acquire.
template <bool STATS>
__device__ __forceinline__ void merge_head(const DecodeParams& p, int u, int h, int n) {
  const Sched& sc = p.sc;
  const int lane = threadIdx.x & 31;
  const int b = u / p.Hkv, hk = u - b * p.Hkv;
  const float* ml_u = p.part_ml + (int64_t)u * sc.S * p.G * 2;
  const float* o_u = p.part_o + (int64_t)u * sc.S * p.G * HKV_D;
  // partial k's (m, l) in lane k; the first 8 partials' o rows load in
  // the same round trip (the usual unit has at most 8 partials)
  const float2* mlp = reinterpret_cast<const float2*>(ml_u) + h;
  const float4* op = reinterpret_cast<const float4*>(o_u + h * HKV_D) + lane;
  const int ostep = p.G * HKV_D / 4;  // float4s per partial
  const float2 ml0 = lane < n ? __ldcg(mlp + lane * p.G) : make_float2(kNoMax, 0.f);
  float4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = i < n ? __ldcg(op + i * ostep) : make_float4(0.f, 0.f, 0.f, 0.f);
  float M = ml0.x;
  for (int k = lane + 32; k < n; k += 32) M = fmaxf(M, __ldcg(mlp + k * p.G).x);
#pragma unroll
  for (int sft = 16; sft > 0; sft >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sft));
  float wk = lane < n ? fast_exp2(ml0.x - M) : 0.f;
  float L = wk * ml0.y;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float w = __shfl_sync(0xffffffffu, wk, i);
    acc.x = fmaf(w, v[i].x, acc.x);
    acc.y = fmaf(w, v[i].y, acc.y);
    acc.z = fmaf(w, v[i].z, acc.z);
    acc.w = fmaf(w, v[i].w, acc.w);
  }
  // partials 8.. (8 per batch, all loads in flight before the first use)
  for (int k0 = 8; k0 < n; k0 += 8) {
    if (k0 % 32 == 0) {
      const float2 mlk = k0 + lane < n ? __ldcg(mlp + (k0 + lane) * p.G) : make_float2(kNoMax, 0.f);
      wk = k0 + lane < n ? fast_exp2(mlk.x - M) : 0.f;
      L = fmaf(wk, mlk.y, L);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = k0 + i < n ? __ldcg(op + (k0 + i) * ostep) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float w = __shfl_sync(0xffffffffu, wk, (k0 + i) & 31);
      acc.x = fmaf(w, v[i].x, acc.x);
      acc.y = fmaf(w, v[i].y, acc.y);
      acc.z = fmaf(w, v[i].z, acc.z);
      acc.w = fmaf(w, v[i].w, acc.w);
    }
  }
#pragma unroll
  for (int sft = 16; sft > 0; sft >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sft);
  if (STATS && lane == 0) {
    p.unit_ml[((int64_t)u * 8 + h) * 2] = M;
    p.unit_ml[((int64_t)u * 8 + h) * 2 + 1] = L;
  }
  const int hq = hk * p.G + h;
  if (p.out_o) {
    reinterpret_cast<float4*>(p.out_o + ((int64_t)b * p.Hq + hq) * HKV_D)[lane] = acc;
    if (lane == 0) {
      // a row that attended to no token reports m = -inf
      p.out_ml[((int64_t)b * p.Hq + hq) * 2] = L > 0.f ? M : -INFINITY;
      p.out_ml[((int64_t)b * p.Hq + hq) * 2 + 1] = L;
    }
  } else {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int64_t o = (int64_t)b * p.out_sb + (int64_t)hq * p.out_sh + 4 * lane;
    store_any(p.out, p.out_dtype, o + 0, acc.x * inv);
    store_any(p.out, p.out_dtype, o + 1, acc.y * inv);
    store_any(p.out, p.out_dtype, o + 2, acc.z * inv);
    store_any(p.out, p.out_dtype, o + 3, acc.w * inv);
  }
}

// ---------------------------------------------------------------- fused decode-step append
// A role that has finished reading the cache state (lengths, ring head)
// arrives; a whole warp calls this, lane 0 counts. The kStateRoles roles of a
// CTA meet on a shared-memory counter (acquire-release at CTA scope), and the
// CTA's last role arrives for all of them on the grid-wide counter (release at
// GPU scope, cumulative over the reads the CTA's roles made before their own
// arrivals). The last of the C grid arrivals applies every sequence's state
// transition of the decode step, as the standalone append kernel does
// (HeteroKVManager._decode_update, src/memory/manager.py:621-664): a ring with
// room grows by one row, a full ring evicts its oldest row to the INT4 body
// (body_len + 1, ring head + 1), no ring sends the token to the body. Every
// read of the state in this launch happens before its reader's arrival, so the
// update never races a reader; the next launch sees it after griddep_wait.
// One global atomic per CTA instead of one per role: a launch of 4 x 148 of
// them on one address measured ~1 us slower.
// The arrival is split so that a warp need not wait for the global atomic: its
// old count stays in a register that only state_arrive_finish consumes; the
// last arriver fences (acquire) before it writes the state.
// The fused append's arrival on a unit's merge counter: a count of its own
// above the pipeline pieces' (fewer than 2^16 per unit).
constexpr int kAppendArrival = 1 << 16;
// Bounded wait of the unit's last pipeline piece for the append's arrival.
__device__ __forceinline__ bool wait_append_arrival(const int* addr) {
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    if (v >= kAppendArrival) return true;
    if (globaltimer_ns() - t0 > HKV_WAIT_NS) {
      hkv_flag_error(HKV_DEVERR_TIMEOUT);
      return false;
    }
    __nanosleep(256);
  }
}
__device__ __forceinline__ int atom_add_release_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.add.release.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}
// -1 for lanes other than 0 and for roles that are not their CTA's last.
__device__ __forceinline__ int state_arrive_start(const DecodeParams& p, int* s_roles) {
  __syncwarp();
  int old = -1;
  if ((threadIdx.x & 31) == 0) {
    int local;
    asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], 1;" : "=r"(local) : "r"(smem_u32(s_roles)) : "memory");
    if (local == kStateRoles - 1) old = atom_add_release_gpu(p.state_counter, 1);
  }
  return old;
}
__device__ __forceinline__ void state_arrive_finish(const DecodeParams& p, int old) {
  const int lane = threadIdx.x & 31;
  const int last = __shfl_sync(0xffffffffu, old == p.sc.C - 1, 0);
  if (!last) return;
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  const int cap = p.dense.capacity, cap_r = cap - p.sink;
  for (int b = lane; b < p.B; b += 32) {
    const int dl = p.dense_len[b];
    if (dl < cap) {
      p.dense_len[b] = dl + 1;
    } else {
      p.body_len[b] = p.body_len[b] + 1;
      if (cap_r > 0) p.ring_head[b] = (p.ring_head[b] + 1) % cap_r;
    }
  }
  __syncwarp();
  if (lane == 0) *p.state_counter = 0;
}

// The append of unit u = (b, KV head h) for every unit whose last schedule step
// lies in this CTA's range (the CTA that holds the unit's end: its dense
// segment, whose tiles cost less per byte than INT4 tiles, so those CTAs have
// time to spare), by one warp (lanes 0-15: K, 16-31: V, 8 dims a lane), on the
// state before the step:
//  * the ring row to evict (full ring), or the new token itself (no ring), is
//    quantised into body slot body_len[b] exactly as the standalone append
//    kernel does it, and the new token is written into the ring (or the next
//    free row);
//  * the attention of the unit's G heads over the tokens the streaming pipeline
//    leaves out, the evicted token as dequantised and the new one, becomes the
//    unit's extra partial (slot nb + nd, after the pipeline's), so the merged
//    output is the attention over the cache after the append.
// The unit's last pipeline piece merges it (see the consumers' end of piece).
// Not inlined: its code stays out of the kernel's main body (inlined, the
// launches of a 32-layer step measured ~2.5 us slower each).
template <int FMT, int GROUP, typename DTy>
__device__ __noinline__ void append_units(const DecodeParams& p, int c, int* s_roles) {
  griddep_wait();  // the query and the new token come from the grid before (a no-op if waited)
  const Sched& sc = p.sc;
  const int lane = threadIdx.x & 31, side = lane >> 4, pq = lane & 15;
  const int cap = p.dense.capacity, cap_r = cap - p.sink;
  const uint32_t x0 = cta_begin(sc, c), x1 = cta_begin(sc, c + 1);
  for (int u = (int)(x0 / sc.Ub); u < sc.U; ++u) {
    const uint32_t last = (uint32_t)(u + 1) * sc.Ub - 1u;  // the unit's last step
    if (last < x0) continue;
    if (last >= x1) break;
    const int b = u / p.Hkv, h = u - b * p.Hkv;
    const int dl = p.dense_len[b], head = p.ring_head[b], bl = p.body_len[b];
    const bool fill = dl < cap;                // a free row: nothing is evicted
    const bool direct = !fill && cap_r <= 0;   // no ring: the new token goes to the body
    const int row = fill ? dl : p.sink + head;
    DTy* seg = static_cast<DTy*>(side ? p.dense.v : p.dense.k);
    DTy* rowp = seg + b * p.dense.stride_b + h * p.dense.stride_h + (int64_t)row * p.dense.stride_t + 8 * pq;
    const DTy* src = static_cast<const DTy*>(side ? p.v_new : p.k_new) + b * p.new_sb + h * p.new_sh + 8 * pq;
    float nv[8], dq[8];
    load8(src, nv);
#pragma unroll
    for (int i = 0; i < 8; ++i) dq[i] = 0.f;
    if (!fill) {
      float ev[8];
      if (direct) {
#pragma unroll
        for (int i = 0; i < 8; ++i) ev[i] = nv[i];
      } else {
        load8(rowp, ev);
      }
      bool ok = bl < p.body.max_pages * p.body.page_tokens;
      int64_t page = 0;
      if (!ok) {
        if (lane == 0) hkv_flag_error(HKV_DEVERR_CAPACITY);
      } else {
        page = store_page(p.body, u, bl);
        if (page < 0) {
          ok = false;
          if (lane == 0) hkv_flag_error(HKV_DEVERR_BAD_PAGE);
        }
      }
      quantise_token(ev, ok, side ? HKV_ROLE_V : HKV_ROLE_K, FMT, GROUP, p.body, page,
                     ok ? bl % p.body.page_tokens : 0, dq);
    }
    if (!direct) store8(rowp, nv);
    // scores (base-2 logits) of the evicted and the new token for each head:
    // K lanes dot their 8 dims, the half-warp sums, lane 0 broadcasts
    float xe[8], xn[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      float se = 0.f, sn = 0.f;
      if (side == 0 && g < p.G) {
        const int64_t qo = (int64_t)b * p.q_sb + (int64_t)(h * p.G + g) * p.q_sh + 8 * pq;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float qv = load_any(p.q, p.q_dtype, qo + i);
          se = fmaf(qv, dq[i], se);
          sn = fmaf(qv, nv[i], sn);
        }
      }
#pragma unroll
      for (int s = 1; s < 16; s <<= 1) {
        se += __shfl_xor_sync(0xffffffffu, se, s);
        sn += __shfl_xor_sync(0xffffffffu, sn, s);
      }
      xe[g] = fill ? -INFINITY : __shfl_sync(0xffffffffu, se, 0) * p.qscale;
      xn[g] = direct ? -INFINITY : __shfl_sync(0xffffffffu, sn, 0) * p.qscale;
    }
    int b0, nb, d0, nd;
    unit_pieces(sc, u, b0, nb, d0, nd);
    float* po = p.part_o + ((int64_t)u * sc.S + nb + nd) * p.G * HKV_D;
    float* pml = p.part_ml + ((int64_t)u * sc.S + nb + nd) * p.G * 2;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (g < p.G) {
        const float m = fmaxf(xe[g], xn[g]);  // at least one token is finite
        const float pe = fill ? 0.f : fast_exp2(xe[g] - m), pn = direct ? 0.f : fast_exp2(xn[g] - m);
        if (side == 1) {
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = fmaf(pe, dq[i], pn * nv[i]);
          float4* d = reinterpret_cast<float4*>(po + g * HKV_D + 8 * pq);
          d[0] = make_float4(o[0], o[1], o[2], o[3]);
          d[1] = make_float4(o[4], o[5], o[6], o[7]);
        }
        if (lane == 16) *reinterpret_cast<float2*>(pml + 2 * g) = make_float2(m, pe + pn);
      }
    }
    // publish the partial: the release add of kAppendArrival after the warp's
    // writes. The merge stays with the consumers (one warp per head) even when
    // this partial comes last: a unit split over many CTAs has tens of
    // partials, which one warp merging every head alone took tens of us for.
    // Only a unit without pipeline pieces is merged here.
    __threadfence();
    __syncwarp();
    if (lane == 0) atom_add_release_gpu(&p.counters[u], kAppendArrival);
    if (nb + nd == 0) {
      for (int g = 0; g < p.G; ++g) merge_head<false>(p, u, g, 1);
      __syncwarp();
      if (lane == 0) p.counters[u] = 0;
    }
  }
  state_arrive_finish(p, state_arrive_start(p, s_roles));
}

// ---------------------------------------------------------------- the persistent kernel
// STATS: record where the attention mass falls (DecodeParams::tile_stats); a
// separate instantiation so that the plain kernel's tile loop stays unchanged.
// APPEND: the decode step's append runs in the same launch (append_units).
template <int FMT, int GROUP, typename DTy, bool STATS, bool APPEND>
__global__ void __launch_bounds__(decode_threads(FMT, APPEND), 1)
    decode_kernel(const __grid_constant__ DecodeParams p) {
  static_assert(!(STATS && APPEND), "the statistics and the fused append are separate instantiations");
  constexpr int NG = HKV_D / GROUP;
  constexpr int NM = kTileI4 * NG;  // metadata entries per array of a tile
  constexpr int kSlot = slot_bytes(FMT, GROUP);
  constexpr int kExp = expand_warps(FMT);
  constexpr int kExtra = APPEND ? 1 : 0;  // partials per unit besides the pipeline's: the append's
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxSlots];
  __shared__ __align__(8) uint64_t ready_bar[kMaxSlots];
  __shared__ __align__(8) uint64_t empty_bar[kMaxSlots];
  __shared__ int2 s_info[kMaxSlots];  // ref: per slot, from the issue warp: (segment or -1 = done, valid tokens)
  __shared__ int s_last;
  __shared__ int s_roles;  // APPEND: roles of this CTA done reading the cache state

  // the 128-byte swizzle of the dense tiles repeats every 1024 bytes: align the ring
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const Sched& sc = p.sc;
  const int c = blockIdx.x;
  const uint32_t end = cta_begin(sc, c + 1);
  const int nsl = p.nslots;
  uint8_t* ring = smem;
  float* comb = reinterpret_cast<float*>(ring + nsl * kSlot);  // [8][G][128] + [8][8][2]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // The next grid in the stream may start its prologue now (it waits for this one
  // before touching global memory, as this one does below). In early mode the
  // trigger waits until this grid has waited for the one before it (thread 0,
  // consumer section): a grid then starts only once every grid two or more
  // launches back has completed, which is what lets it read its cache early.
  const bool early = APPEND && p.early;
  if (!early) griddep_launch_dependents();
  Piece first = first_piece_head(p, c, end);  // parameters only
  uint8_t* qbuf = reinterpret_cast<uint8_t*>(comb + kConsumerWarps * p.G * HKV_D + kConsumerWarps * 16);
  if (warp == kConsumerWarps - 1 && lane < nsl) {  // a warp whose first work waits anyway
    mbar_init(&full_bar[lane], 1);
    mbar_init(&ready_bar[lane], 1);
    mbar_init(&empty_bar[lane], kGroupWarps);
    fence_barrier_init();
  }
  if (APPEND && threadIdx.x == 0) s_roles = 0;
  // Global memory from here on. The first piece's sequence length (and, for the
  // consumers, its query rows) load across the barrier. Early mode: the cache
  // (state, page table, pages, dense rows) was completed by a grid two or more
  // launches back, so it is read, and the ring filled, before the wait; every
  // role waits on its own before it reads the query or the new token (made by
  // the grid just before) and before its first global write.
  if (!early) griddep_wait();
  const int2 first_st = first.valid ? seg_state<APPEND>(p, first.u, first.seg) : make_int2(0, -1);
  if (!early && warp < kConsumerWarps && p.q_async && first.valid) q_prefetch(p, first.u, qbuf);
  __syncthreads();
  if (first.valid) {
    piece_fill_len(p, end, first, first_st.x);
    first.skip = first_st.y;
  }

  if (warp >= kConsumerWarps) {
    if (warp < kIssueWarp + kIssueWarps) {
      // ================================================================ TMA issue warps
      // Issue warp w takes the loads n with n % 2 == w: one bulk copy in flight per
      // warp is accepted at a time, so two warps keep more of the ring moving. With
      // an even slot count a slot always belongs to one issue warp (and one
      // consumer group), whose waits on it therefore never alias.
      const int w = warp - kIssueWarp;
      Cursor cu;
      cursor_start(p, end, first, cu);
      if (w == 1 && cu.valid) cursor_next(p, end, cu);
      Ring ri{w, 0u};
      int n = w;
      // page ids of pages [pg0, pg0 + 32) of unit pg_u, one per lane (fetched 32 at a time)
      int pg_u = -1, pg0 = 0, pg_lane = -1;
      constexpr uint32_t kTileBytes = block_bytes(FMT, GROUP);  // one 128-token block = one tile
      bool waited = !early;  // early mode: griddep_wait not yet done by this warp
      while (cu.valid) {
        if (n >= nsl) {
          // early mode: the ring share is full; the consumers free slots only after
          // the wait, so wait here first (a long preceding grid must not run the
          // bounded slot wait out)
          if (!waited) {
            griddep_wait();
            waited = true;
          }
          if (!warp_wait(&empty_bar[ri.slot], ri.phase ^ 1u, HKV_ISSUE_SLEEP_NS)) break;
        }
        uint8_t* sb = ring + ri.slot * kSlot;
        uint64_t* fb = &full_bar[ri.slot];
        const int u = cu.pc.u;
        // ref: what the expansion warp needs to know about this load (published by the arrive below)
        if (kExp > 0 && lane == 0)
          s_info[ri.slot] = make_int2(cu.pc.seg, cu.pc.len - cu.k * (cu.pc.seg == 0 ? kTileI4 : kTileD));
        if (cu.pc.seg == 0) {
          const int t = cu.k * kTileI4;
          const int pi = p.page_shift >= 0 ? t >> p.page_shift : t / p.body.page_tokens;
          if (u != pg_u || pi < pg0 || pi >= pg0 + 32) {
            pg_u = u;
            pg0 = pi;
            const int pl = pi + lane;
            pg_lane = -1;
            if (pl < p.body.max_pages)
              pg_lane = p.body.page_table ? p.body.page_table[(int64_t)u * p.body.max_pages + pl]
                                          : (int)((int64_t)u * p.body.max_pages + pl);
          }
          const int page = __shfl_sync(0xffffffffu, pg_lane, pi - pg0);
          if (lane == 0) {
            if (!page_ok(p.body, page)) {
              hkv_flag_error(HKV_DEVERR_BAD_PAGE);
              mbar_arrive(fb);
            } else {
              const int off = p.page_shift >= 0 ? t & ((1 << p.page_shift) - 1) : t % p.body.page_tokens;
              const uint8_t* src = static_cast<const uint8_t*>(p.body.pages) + (int64_t)page * p.body.page_stride +
                                   (int64_t)(off / kTileI4) * kTileBytes;
              mbar_arrive_expect_tx(fb, kTileBytes);
              bulk_g2s(sb, src, kTileBytes, fb);
            }
          }
        } else if (lane == 0) {
          const int b = u / p.Hkv, hk = u - b * p.Hkv, t = cu.k * kTileD;
          const uint32_t d = smem_u32(sb);
          mbar_arrive_expect_tx(fb, dense_slot_bytes());
          // K then V: one box each, both 64-dim halves of 32 rows
          tma_tile_5d(d, &p.tmk, 0, t, 0, hk, b, fb);
          tma_tile_5d(d + 2 * kDenseHalf, &p.tmv, 0, t, 0, hk, b, fb);
        }
        n += 2;
        ri.advance(nsl);
        ri.advance(nsl);
        cursor_next(p, end, cu);
        if (cu.valid) cursor_next(p, end, cu);
      }
      if constexpr (APPEND) {
        if (!waited) griddep_wait();  // before the first global write (the arrival)
        state_arrive_finish(p, state_arrive_start(p, &s_roles));  // the cursor has read its last length
      }
      // an end-of-work load (a plain arrive, no copy) for expansion warp w, which
      // takes the loads of this warp's parity
      if (kExp > 0 && (n < nsl || warp_wait(&empty_bar[ri.slot], ri.phase ^ 1u))) {
        if (lane == 0) {
          s_info[ri.slot] = make_int2(-1, 0);
          mbar_arrive(&full_bar[ri.slot]);
        }
        n += 2;
      }
      // every copy this warp issued must have landed before the CTA exits
      if (lane == 0) {
        for (int i = max(w, n - nsl); i < n; i += 2) mbar_wait(&full_bar[i % nsl], (i / nsl) & 1);
      }
    } else {
      // ================================================================ fused append (APPEND)
      if constexpr (APPEND) {
        if (warp == kAppendWarp) append_units<FMT, GROUP, DTy>(p, c, &s_roles);
      }
      if constexpr (kExp > 0) {
      // ================================================================ metadata expansion warps (ref)
      // expansion warp x takes the loads n with n % 2 == x (those of issue warp x),
      // until that warp's end-of-work load
      static_assert(expand_warps(HKV_FMT_REF) == kIssueWarps, "one expansion warp per issue warp");
      const int x = warp - kExpandWarp;
      Ring re{0, 0u};
      for (int i = 0; i < x; ++i) re.advance(nsl);
      while (true) {
        if (!warp_wait(&full_bar[re.slot], re.phase)) break;
        const int2 info = s_info[re.slot];
        if (info.x < 0) break;
        uint8_t* sb = ring + re.slot * kSlot;
        if (info.x == 0) {
          expand_meta<NG>(sb + kMetaOff, lane, info.y, p.qscale);
        } else {
          zero_dense_v_tail(sb, info.y, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready_bar[re.slot]);
        for (int i = 0; i < kExp; ++i) re.advance(nsl);
      }
      }
    }
    return;
  }

  // ================================================================== consumer warps
  // Group grp (warps 4 grp .. 4 grp + 3) takes the loads n with n % 2 == grp;
  // warp wg of the group computes tokens [32 wg, 32 wg + 32) of an INT4 tile and
  // [8 wg, 8 wg + 8) of a dense tile.
  // a tile is ready for the consumers once expanded (ref) or once landed (fp16min)
  uint64_t* cons_bar = kExp > 0 ? ready_bar : full_bar;
  WarpState<NG> ws;
  uint32_t qf[8][2];
  float qsum[NG][2], nbias[NG][2];  // qsum: ref only
  uint32_t qbias = 0;                // fp16min: B fragment of the K bias MMA
  const int r = lane >> 2, j = lane & 3;
  const int grp = warp / kGroupWarps, wg = warp % kGroupWarps;
  const bool h0 = 2 * j < p.G, h1 = 2 * j + 1 < p.G;
  const float qs = p.qscale;
  Ring rc{grp, 0u};  // ring position of this group's next load
  int n_next = grp;  // index of this group's next load
  int n_base = 0;    // index of the current piece's first load
  const int t0 = wg * 32;
  const int kc_off = (t0 + r) * HKV_CODE_BYTES + 16 * j;
  // chunk r of pair t0/2 + j (and of pair t0/2 + 8 + j): the block rotates pair q's chunks by 2q
  const int vc_off = HKV_V_CODES_OFF + v_chunk_off(t0 / 2 + j, r);
  const int vs_off = (t0 / 2) * NG;  // f16x2 words
  // the query rows of the current piece's unit (qbuf) are prefetched during the
  // previous piece (the first piece's before the barrier setup)
  if (early) {
    griddep_wait();
    if (threadIdx.x == 0) griddep_launch_dependents();
    if (p.q_async && first.valid) q_prefetch(p, first.u, qbuf);
  }
  Piece pc = first;
  bool state_done = false;   // APPEND: the consumers' arrival on the state counter is made
  bool arr_pending = false;  // ... and its count (arr_old, warp 0) not yet consumed
  int arr_old = 0;
  while (pc.valid) {
    const int u = pc.u, b = u / p.Hkv, hk = u - b * p.Hkv;
    // ---- begin piece: query fragments for this unit
    const void* qsrc = nullptr;
    if (p.q_async) {
      cp_async_wait_all();
      consumer_sync();
      qsrc = qbuf;
    }
    {
      float qa[8][2], qb[8][2];
      if (pc.seg == 0) {
        load_q_frags<__half>(p, b, hk, true, qsrc, qf, qa, qb);
        float ps[NG], pbias[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g) ps[g] = pbias[g] = 0.f;
#pragma unroll
        for (int kt = 0; kt < 8; ++kt) {
          const int g = (kt * 16) / GROUP;
          ps[g] += qa[kt][0] + qa[kt][1] + 16.f * (qb[kt][0] + qb[kt][1]);
          pbias[g] += qa[kt][0] + qa[kt][1] + qb[kt][0] + qb[kt][1];
        }
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          ps[g] += __shfl_xor_sync(0xffffffffu, ps[g], 1);
          ps[g] += __shfl_xor_sync(0xffffffffu, ps[g], 2);
          pbias[g] += __shfl_xor_sync(0xffffffffu, pbias[g], 1);
          pbias[g] += __shfl_xor_sync(0xffffffffu, pbias[g], 2);
          qsum[g][0] = qs * __shfl_sync(0xffffffffu, ps[g], (2 * j) * 4);
          qsum[g][1] = qs * __shfl_sync(0xffffffffu, ps[g], (2 * j + 1) * 4);
          nbias[g][0] = -1024.f * __shfl_sync(0xffffffffu, pbias[g], (2 * j) * 4);
          nbias[g][1] = -1024.f * __shfl_sync(0xffffffffu, pbias[g], (2 * j + 1) * 4);
        }
        if constexpr (FMT == HKV_FMT_FP16MIN) {
          // B of the K bias MMA, head r: rows 0..NG-1 = f16 hi parts of sum(Q_g),
          // rows NG..2NG-1 = the lo parts (this lane holds rows 2j, 2j+1)
          __half hi[NG], lo[NG];
#pragma unroll
          for (int g = 0; g < NG; ++g) {
            const float v = ps[g];
            hi[g] = __float2half_rn(v);
            lo[g] = __float2half_rn(v - __half2float(hi[g]));
          }
          auto h2 = [](__half a, __half b) {
            return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
          };
          if constexpr (NG == 4) {
            qbias = j == 0 ? h2(hi[0], hi[1]) : j == 1 ? h2(hi[2], hi[3]) : j == 2 ? h2(lo[0], lo[1]) : h2(lo[2], lo[3]);
          } else if constexpr (NG == 2) {
            qbias = j == 0 ? h2(hi[0], hi[1]) : j == 1 ? h2(lo[0], lo[1]) : 0u;
          } else {
            qbias = j == 0 ? h2(hi[0], lo[0]) : 0u;
          }
        }
      } else {
        load_q_frags<DTy>(p, b, hk, false, qsrc, qf, qa, qb);
      }
    }
    // the next piece: its length and its query rows load while this piece runs
    Piece nx = pc;
    next_piece_head(p, end, nx);
    const int2 nst = nx.valid ? seg_state<APPEND>(p, nx.u, nx.seg) : make_int2(0, -1);
    if (p.q_async && nx.valid) {
      consumer_sync();  // every consumer has read qbuf
      q_prefetch(p, nx.u, qbuf);
    }
    if constexpr (APPEND) {
      // the consumers' last state read lies behind them (and behind a consumer
      // barrier: the prologue's __syncthreads or the previous piece's end):
      // warp 0 arrives for all of them, the count is consumed after the tiles
      if (!nx.valid && !state_done) {
        if (warp == 0) arr_old = state_arrive_start(p, &s_roles);
        state_done = arr_pending = true;
      }
    }
    ws_reset<NG>(ws);

    // ---- this group's share of the piece's tiles that hold tokens
    bool alive = true;
    const int n_end = n_base + max(0, pc.kd - pc.k0);
    if (pc.seg == 0) {
      for (; n_next < n_end; n_next += 2) {
        const int k = pc.k0 + (n_next - n_base);
        if (!warp_wait(&cons_bar[rc.slot], rc.phase, HKV_CONS_SLEEP_NS)) {
          alive = false;
          break;
        }
        const uint8_t* stg = ring + rc.slot * kSlot;
        // metadata: ref expanded in place (layout above); fp16min as stored
        const uint8_t* mb = stg + kMetaOff;
        const uint32_t* vsp =
            reinterpret_cast<const uint32_t*>(mb + (FMT == HKV_FMT_REF ? 14 * NM : 512 * NG)) + vs_off;
        const uint32_t* vz =
            reinterpret_cast<const uint32_t*>(mb + (FMT == HKV_FMT_REF ? 10 * NM : 768 * NG)) +
            (FMT == HKV_FMT_REF ? 2 : 1) * vs_off;
        float xa[4], xb[4], x[8], P[8];
        k_scores<FMT, NG>(stg + kc_off, mb, t0, qf, nbias, qsum, qbias, qs, xa);
        k_scores<FMT, NG>(stg + kc_off + 16 * HKV_CODE_BYTES, mb, t0 + 16, qf, nbias, qsum, qbias, qs, xb);
        const int tok = k * kTileI4 + t0;
        x[0] = xa[0];
        x[1] = xa[1];
        x[2] = xa[2];
        x[3] = xa[3];
        x[4] = xb[0];
        x[5] = xb[1];
        x[6] = xb[2];
        x[7] = xb[3];
        if (tok + 32 > pc.len) {
          if (tok + r >= pc.len) x[0] = x[1] = -INFINITY;
          if (tok + r + 8 >= pc.len) x[2] = x[3] = -INFINITY;
          if (tok + r + 16 >= pc.len) x[4] = x[5] = -INFINITY;
          if (tok + r + 24 >= pc.len) x[6] = x[7] = -INFINITY;
        }
        softmax_step<NG, 8>(ws, x, P, 4.f);
        if (STATS && k < p.stat_tiles) record_tile_stats(p, u, k, wg, ws.m, P);
        const float pa[4] = {P[0], P[1], P[2], P[3]};
        const float pc4[4] = {P[4], P[5], P[6], P[7]};
        const int nv = pc.len - tok;  // tokens of this warp's 32 that lie in the sequence
        v_accumulate<FMT, NG>(ws, stg + vc_off, vsp, vz, pa, nv);
        v_accumulate<FMT, NG>(ws, stg + vc_off + 16 * HKV_CODE_BYTES, vsp + 8 * NG,
                              vz + (FMT == HKV_FMT_REF ? 2 : 1) * 8 * NG, pc4, nv - 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[rc.slot]);
        rc.advance(nsl);
        rc.advance(nsl);
      }
    } else {
      const int dt0 = wg * 8;
      for (; n_next < n_end; n_next += 2) {
        const int k = pc.k0 + (n_next - n_base);
        if (!warp_wait(&cons_bar[rc.slot], rc.phase, HKV_CONS_SLEEP_NS)) {
          alive = false;
          break;
        }
        uint8_t* sl = ring + rc.slot * kSlot;
        if constexpr (kExp == 0) {
          // no expansion warp zeroes the V rows past the sequence end: this
          // warp zeroes its own rows [dt0, dt0 + 8) that lie there
          const int valid = pc.len - k * kTileD;
          if (dt0 + 8 > valid) {
            zero_dense_v_rows(sl, max(dt0, valid), dt0 + 8, lane);
            __syncwarp();
          }
        }
        const uint32_t slot = smem_u32(sl);
        const int trow = k * kTileD + dt0 + r;  // this thread's score row in the segment
        dense_subtile<DTy, NG>(ws, slot, dt0, trow < pc.len && trow != pc.skip, qf, qs);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[rc.slot]);
        rc.advance(nsl);
        rc.advance(nsl);
      }
    }
    n_base = n_end;
    if (APPEND && arr_pending) {
      if (warp == 0) state_arrive_finish(p, arr_old);
      arr_pending = false;
    }

    // ---- end piece: per-warp partials -> shared memory -> one partial for the piece
    {
      const bool body = pc.seg == 0;
      float l0 = ws.l[0], l1 = ws.l[1];
#pragma unroll
      for (int sft = 4; sft < 32; sft <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, sft);
        l1 += __shfl_xor_sync(0xffffffffu, l1, sft);
      }
      // fp16min V bias of group g, heads 2j, 2j+1: row g of the bias MMA (lane 4g + j)
      float z[NG][2];
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        z[g][0] = __shfl_sync(0xffffffffu, ws.zc[0], 4 * g + j);
        z[g][1] = __shfl_sync(0xffffffffu, ws.zc[1], 4 * g + j);
        if (FMT == HKV_FMT_REF || !body) z[g][0] = z[g][1] = 0.f;
      }
      float* wo = comb + warp * p.G * HKV_D;
      float* cml = comb + kConsumerWarps * p.G * HKV_D;  // [8 warps][8 heads][2]
      const float osc = body ? 16.f : 1.f;                 // INT4 tiles accumulate with P/16
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d0 = 16 * mt + r, d1 = d0 + 8;
        const int g = (16 * mt) / GROUP;
        if (h0) {
          wo[(2 * j) * HKV_D + d0] = osc * (ws.o[mt][0] + z[g][0]);
          wo[(2 * j) * HKV_D + d1] = osc * (ws.o[mt][2] + z[g][0]);
        }
        if (h1) {
          wo[(2 * j + 1) * HKV_D + d0] = osc * (ws.o[mt][1] + z[g][1]);
          wo[(2 * j + 1) * HKV_D + d1] = osc * (ws.o[mt][3] + z[g][1]);
        }
      }
      if (r == 0) {
        cml[(warp * 8 + 2 * j) * 2] = ws.m[0];
        cml[(warp * 8 + 2 * j) * 2 + 1] = l0 * osc;
        cml[(warp * 8 + 2 * j + 1) * 2] = ws.m[1];
        cml[(warp * 8 + 2 * j + 1) * 2 + 1] = l1 * osc;
      }
      // a timed-out wait anywhere ends every consumer warp after this piece
      // (the error word is set; the partials written below are meaningless)
      alive = consumer_sync_and(alive);
      int b0, nb, d0, nd;
      unit_pieces(sc, u, b0, nb, d0, nd);
      const int slot = pc.seg == 0 ? c - b0 : nb + c - d0;
      float* po = p.part_o + ((int64_t)u * sc.S + slot) * p.G * HKV_D;
      float* pml = p.part_ml + ((int64_t)u * sc.S + slot) * p.G * 2;
      for (int idx = threadIdx.x; idx < p.G * HKV_D; idx += kConsumerThreads) {
        const int h = idx / HKV_D, d = idx % HKV_D;
        float M = kNoMax;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, cml[(w * 8 + h) * 2]);
        float acc = 0.f, L = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float e = fast_exp2(cml[(w * 8 + h) * 2] - M);
          acc = fmaf(e, comb[(w * p.G + h) * HKV_D + d], acc);
          L = fmaf(e, cml[(w * 8 + h) * 2 + 1], L);
        }
        po[idx] = acc;
        if (d == 0) {
          pml[2 * h] = M;
          pml[2 * h + 1] = L;
        }
      }
      // The barrier orders every consumer thread's partial stores before thread 0's
      // acq_rel atomic, whose release makes them visible GPU-wide (cumulativity)
      // and whose acquire, followed by the barrier, orders the merge's loads of the
      // other CTAs' partials after their releases.
      consumer_sync();
      if (threadIdx.x == 0) {
        const int old = atom_add_acq_rel_gpu(&p.counters[u], 1);
        bool last = (old & (kAppendArrival - 1)) == nb + nd - 1;
        // APPEND: the last pipeline piece also merges the append's partial, once
        // it is published (a bounded wait; the append warp depends on nothing here)
        if (APPEND && last && old < kAppendArrival) last = wait_append_arrival(&p.counters[u]);
        s_last = last;
      }
      consumer_sync();
      if (s_last) {
        // last piece of the unit: merge all its partials (warp h: head h)
        for (int h = warp; h < p.G; h += kConsumerWarps) merge_head<STATS>(p, u, h, nb + nd + kExtra);
        consumer_sync();
        if (threadIdx.x == 0) p.counters[u] = 0;
      }
      consumer_sync();  // the combine area is free again
    }
    if (!alive) break;
    pc = nx;
    if (pc.valid) {
      piece_fill_len(p, end, pc, nst.x);
      pc.skip = nst.y;
    }
  }
  if constexpr (APPEND) {
    if (!state_done) {  // no piece at all, or a timed-out wait ended the loop early
      consumer_sync();
      if (warp == 0) state_arrive_finish(p, state_arrive_start(p, &s_roles));
    }
  }
  cp_async_wait_all();
}

// ---------------------------------------------------------------- log-sum-exp merge (cross-GPU partials)
// One block of 128 threads per output row (b, hq); partial s of that row at
//   o:  part_o  + row*128 + s*split_o,   ml: part_ml + row*2 + s*split_ml
struct MergeParams {
  const float* part_o;
  const float* part_ml;
  int S, Hq;
  int64_t split_o, split_ml;
  void* out;
  int out_dtype;
  int64_t out_sb, out_sh;
};

__global__ void __launch_bounds__(128) lse_merge_kernel(const MergeParams mp) {
  const int row = blockIdx.x;
  const int b = row / mp.Hq, hq = row % mp.Hq;
  const int d = threadIdx.x;
  const float* po = mp.part_o + (int64_t)row * HKV_D + d;
  const float* pml = mp.part_ml + (int64_t)row * 2;
  float M = -INFINITY;
  for (int s = 0; s < mp.S; ++s) M = fmaxf(M, pml[s * mp.split_ml]);
  float acc = 0.f, L = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < mp.S; ++s) {
      const float ms = pml[s * mp.split_ml];
      if (ms == -INFINITY) continue;
      const float w = fast_exp2(ms - M);
      acc = fmaf(w, po[s * mp.split_o], acc);
      L = fmaf(w, pml[s * mp.split_ml + 1], L);
    }
  }
  const float v = L > 0.f ? acc / L : 0.f;
  store_any(mp.out, mp.out_dtype, (int64_t)b * mp.out_sb + (int64_t)hq * mp.out_sh + d, v);
}

// ---------------------------------------------------------------- attention mass per body tile
// One block of 128 threads per unit u: mass[u][k] = mean over the unit's G heads
// of sum_warps s * 2^(m - M) / L, the softmax probability on tile k's tokens
// (0 for tiles past the body length). Inputs as recorded by decode_kernel.
__global__ void __launch_bounds__(128) tile_scores_kernel(const float* __restrict__ stats,
                                                          const float* __restrict__ unit_ml,
                                                          const int32_t* __restrict__ lengths, int len, int Hkv,
                                                          int G, int stat_tiles, float* __restrict__ mass) {
  const int u = blockIdx.x;
  const int b = u / Hkv;
  const int n = lengths ? lengths[b] : len;
  const int tiles = min(stat_tiles, (n + kTileI4 - 1) / kTileI4);
  for (int k = threadIdx.x; k < stat_tiles; k += blockDim.x) {
    float acc = 0.f;
    if (k < tiles) {
      const float* st = stats + ((int64_t)u * stat_tiles + k) * 4 * 8 * 2;
      for (int h = 0; h < G; ++h) {
        const float M = unit_ml[((int64_t)u * 8 + h) * 2], L = unit_ml[((int64_t)u * 8 + h) * 2 + 1];
        if (!(L > 0.f)) continue;
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) t += st[(w * 8 + h) * 2] * exp2f(st[(w * 8 + h) * 2 + 1] - M);
        acc += t / L;
      }
      acc /= (float)G;
    }
    mass[(int64_t)u * stat_tiles + k] = acc;
  }
}

}  // namespace hkv
