// Persistent split-KV GQA decode attention over packed INT4 pages + a dense
// fp16/bf16 segment, with a fused log-sum-exp merge. Included by hetero_kv.cu.
//
// Schedule. The work of every (sequence, KV head) unit is a list of tiles:
// 128-token INT4 body tiles, then 32-token dense tiles. Tiles are weighted by
// their HBM bytes and the whole list (all units) is cut into one contiguous,
// equal-byte range per CTA of a persistent grid (2 CTAs per SM). A CTA's range
// covers pieces: runs of tiles of one (unit, segment). Each piece ends in an
// un-normalised partial (m, l, O) for the unit's G query heads; the CTA that
// delivers a unit's last partial merges them (log-sum-exp) into the output.
//
// Pipeline. Warp 4 is the producer. It streams tiles into a shared-memory ring
// with 1-D bulk async copies (TMA engine, no multicast) that complete on
// mbarriers, and expands each INT4 tile's group metadata (f16 or u8) into an
// fp32 / f16x2 form the consumers use directly. Warps 0-3 consume with
// m16n8k16 tensor-core MMAs (N = 8 query heads, G <= 8 used):
//   S^T[tok][head] = K[tok][:] . Q^T      (M = 16 tokens, K = dims)
//   O^T[dim][head] += V^T[dim][tok] . P^T (M = 16 dims,   K = tokens)
// K and V fragments come straight from the packed nibbles (the page format's
// nibble order is the fragment order) with integer-only ops: a nibble OR-ed
// into the mantissa of 1024.0h is the exact f16 value 1024 + n (or 1024 + 16 n
// for a high nibble). The biases are folded away in fp32:
//   K: half of each k-tile is (1024 + n), half (1024 + 16 n) against Q/16, and
//      the accumulator starts at -1024 * sum(Q), so it ends at sum(n Q):
//      score = sum_g s_g * acc_g + b_g * sum(Q_g)        (b = -z*s or min)
//   V: codes are exact integers n (bias removed in f16), the B operand is
//      s * P / 16, so O = 16 * (acc + sum_t b_t P_t / 16).
// The online softmax is fp32 in the base-2 domain, one max-reduction per 32
// tokens and warp, with a lazy rescale (the running max only moves when a tile
// beats it by more than 2^8).
#pragma once
#include "hkv_common.cuh"

namespace hkv {

constexpr int kConsumerWarps = 4;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kDecodeThreads = kConsumerThreads + 32;
constexpr int kTileI4 = 128;    // tokens per INT4 tile (32 per consumer warp)
constexpr int kTileD = 32;      // tokens per dense tile (8 per consumer warp)
constexpr int kRowPitch = 272;  // bytes per dense row in shared memory (256 + 16: conflict-free ldmatrix)
constexpr int kMaxSlots = 6;
constexpr int kMetaSlots = 2;
constexpr float kLazyRescale = 8.0f;

// Equal-byte partition of the tile list over the persistent grid.
struct Sched {
  int U;          // units (B * Hkv)
  int Tb, Td;     // body / dense tiles per unit (from the host-side length hints)
  int C;          // CTAs
  int S;          // partial slots per unit in the workspace
  int64_t tb, td; // bytes per body / dense tile
  int64_t Ub;     // bytes per unit
  int64_t Btot;   // bytes in total
};

struct DecodeParams {
  const void* q;
  int q_dtype;
  int64_t q_sb, q_sh;
  hkv_int4_store body;
  hkv_dense_kv dense;
  int has_body, has_dense;
  int B, Hq, Hkv, G;
  float qscale;  // sm_scale * log2(e)
  Sched sc;
  int slot_bytes, nslots, meta_bytes;
  float* part_o;   // [U][S][G][128]  un-normalised partial outputs
  float* part_ml;  // [U][S][G][2]    (m, l), base-2 logits
  int* counters;   // [U]             zero before first use, self-resetting
  void* out;       // [B][Hq][128] out_dtype (normalised mode)
  int out_dtype;
  int64_t out_sb, out_sh;
  float* out_o;    // [B][Hq][128] f32 (partial mode, when non-null)
  float* out_ml;   // [B][Hq][2]
};

__host__ __device__ constexpr int i4_raw_bytes(int fmt, int group) {
  return 2 * kTileI4 * HKV_CODE_BYTES + 2 * kTileI4 * 4 * (HKV_D / group) +
         (fmt == HKV_FMT_REF ? 2 * kTileI4 * (HKV_D / group) : 0);
}
__host__ __device__ constexpr int dense_slot_bytes() { return 2 * kTileD * kRowPitch; }
// expanded metadata of one INT4 tile: K scale f32, K bias f32, V scale f16x2 (s,s), V bias f32
__host__ __device__ constexpr int meta_slot_bytes(int group) { return kTileI4 * (HKV_D / group) * 16; }

// ---------------------------------------------------------------- schedule arithmetic
__device__ __forceinline__ int64_t cta_begin(const Sched& s, int c) { return (int64_t)c * s.Btot / s.C; }
__device__ __forceinline__ int64_t tile_byte(const Sched& s, int u, int seg, int k) {
  return (int64_t)u * s.Ub + (seg == 0 ? (int64_t)k * s.tb : (int64_t)s.Tb * s.tb + (int64_t)k * s.td);
}
__device__ __forceinline__ int owner_of(const Sched& s, int64_t x) {
  int c = (int)(x * s.C / s.Btot);
  if (c + 1 <= s.C && cta_begin(s, c + 1) <= x) ++c;
  return c;
}

struct TileRef {
  int u, seg, k;
  bool valid;
};

// First tile whose byte start lies in [cta_begin(c), cta_begin(c+1)).
__device__ __forceinline__ TileRef first_tile(const Sched& s, int c) {
  const int64_t x = cta_begin(s, c), end = cta_begin(s, c + 1);
  TileRef t;
  t.u = (int)(x / s.Ub);
  const int64_t r = x - (int64_t)t.u * s.Ub;
  if (s.Tb > 0 && r <= (int64_t)(s.Tb - 1) * s.tb) {
    t.seg = 0;
    t.k = (int)((r + s.tb - 1) / s.tb);
  } else if (s.Td > 0 && r <= (int64_t)s.Tb * s.tb + (int64_t)(s.Td - 1) * s.td) {
    t.seg = 1;
    const int64_t rd = r - (int64_t)s.Tb * s.tb;
    t.k = rd > 0 ? (int)((rd + s.td - 1) / s.td) : 0;
  } else {
    t.u += 1;
    t.seg = s.Tb > 0 ? 0 : 1;
    t.k = 0;
  }
  t.valid = t.u < s.U && tile_byte(s, t.u, t.seg, t.k) < end;
  return t;
}

__device__ __forceinline__ int body_len(const DecodeParams& p, int u) {
  return p.body.lengths ? p.body.lengths[u / p.Hkv] : p.body.len;
}
__device__ __forceinline__ int dense_len(const DecodeParams& p, int u) {
  return p.dense.lengths ? p.dense.lengths[u / p.Hkv] : p.dense.len;
}

// Next tile of the CTA's range. Past its last hinted tile, a segment continues
// with extra tiles while the unit's true length needs them (a stale hint can
// unbalance the grid, never drop tokens); those belong to the same CTA.
__device__ __forceinline__ void next_tile(const DecodeParams& p, int64_t end, TileRef& t) {
  const Sched& s = p.sc;
  if (t.seg == 0) {
    if (t.k + 1 < s.Tb) {
      t.k++;
      t.valid = tile_byte(s, t.u, 0, t.k) < end;
      return;
    }
    if ((int64_t)kTileI4 * (t.k + 1) < body_len(p, t.u)) {
      t.k++;
      return;
    }
    if (s.Td > 0) {
      t.seg = 1;
      t.k = 0;
      t.valid = tile_byte(s, t.u, 1, 0) < end;
      return;
    }
  } else {
    if (t.k + 1 < s.Td) {
      t.k++;
      t.valid = tile_byte(s, t.u, 1, t.k) < end;
      return;
    }
    if ((int64_t)kTileD * (t.k + 1) < dense_len(p, t.u)) {
      t.k++;
      return;
    }
  }
  t.u++;
  t.seg = s.Tb > 0 ? 0 : 1;
  t.k = 0;
  t.valid = t.u < s.U && tile_byte(s, t.u, t.seg, 0) < end;
}

__device__ __forceinline__ bool tile_has_data(const DecodeParams& p, const TileRef& t) {
  return t.seg == 0 ? kTileI4 * t.k < body_len(p, t.u) : kTileD * t.k < dense_len(p, t.u);
}

// Pieces (partials) of unit u: CTAs owning its body tiles, then its dense tiles.
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

// ---------------------------------------------------------------- warp state / softmax
// Thread (r = lane/4, j = lane%4) owns heads 2j and 2j+1 in every accumulator.
template <int NG>
struct WarpState {
  float o[8][4];      // O^T, m-tile mt: (dim 16mt+r | 16mt+r+8) x (head 2j | 2j+1)
  float zacc[NG][2];  // sum_t b_g(t) * P(t)/16   (INT4 only)
  float m[2];         // running max (base-2 logits)
  float mo[2];        // m + log2 of the P pre-scale (4 for INT4: P/16; 0 for dense)
  float l[2];         // sum of the pre-scaled P
};

template <int NG>
__device__ __forceinline__ void ws_reset(WarpState<NG>& ws) {
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) ws.o[mt][0] = ws.o[mt][1] = ws.o[mt][2] = ws.o[mt][3] = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) ws.zacc[g][0] = ws.zacc[g][1] = 0.f;
  ws.m[0] = ws.m[1] = ws.mo[0] = ws.mo[1] = -INFINITY;
  ws.l[0] = ws.l[1] = 0.f;
}

template <int NG, int N>
__device__ __forceinline__ void softmax_step(WarpState<NG>& ws, const float (&x)[N], float (&P)[N], float off) {
  float t0 = x[0], t1 = x[1];  // x[i] belongs to head 2j + (i & 1)
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
  const bool need = (t0 > ws.m[0] + kLazyRescale) || (t1 > ws.m[1] + kLazyRescale);
  if (__any_sync(0xffffffffu, need)) {
    const float n0 = fmaxf(ws.m[0], t0), n1 = fmaxf(ws.m[1], t1);
    const float a0 = ws.m[0] == -INFINITY ? 0.f : fast_exp2(ws.m[0] - n0);
    const float a1 = ws.m[1] == -INFINITY ? 0.f : fast_exp2(ws.m[1] - n1);
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
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      ws.zacc[g][0] *= a0;
      ws.zacc[g][1] *= a1;
    }
    ws.l[0] *= a0;
    ws.l[1] *= a1;
  }
#pragma unroll
  for (int i = 0; i < N; ++i) P[i] = x[i] == -INFINITY ? 0.f : fast_exp2(x[i] - ws.mo[i & 1]);
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

struct MetaPtrs {
  const float* ks;
  const float* kb;
  const uint32_t* vs2;
  const float* vb;
};

// Scores of 16 tokens x 8 heads: x = {(r,2j), (r,2j+1), (r+8,2j), (r+8,2j+1)} (unscaled).
template <int NG>
__device__ __forceinline__ void k_scores(const uint8_t* codes, const MetaPtrs& mp, int t0,
                                         const uint32_t (&qf)[8][2], const float (&nbias)[NG][2],
                                         const float (&qsum)[NG][2], float (&x)[4]) {
  constexpr int WPG = 4 / NG;  // packed words per group
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const uint4 kA = *reinterpret_cast<const uint4*>(codes + (t0 + r) * HKV_CODE_BYTES + 16 * j);
  const uint4 kB = *reinterpret_cast<const uint4*>(codes + (t0 + r + 8) * HKV_CODE_BYTES + 16 * j);
  const uint32_t kwa[4] = {kA.x, kA.y, kA.z, kA.w};
  const uint32_t kwb[4] = {kB.x, kB.y, kB.z, kB.w};
  float sA[NG], sB[NG], bA[NG], bB[NG];
  ld_row<NG>(mp.ks, t0 + r, sA);
  ld_row<NG>(mp.ks, t0 + r + 8, sB);
  ld_row<NG>(mp.kb, t0 + r, bA);
  ld_row<NG>(mp.kb, t0 + r + 8, bB);
  x[0] = x[1] = x[2] = x[3] = 0.f;
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
      x[0] = fmaf(sA[g], c[0], fmaf(bA[g], qsum[g][0], x[0]));
      x[1] = fmaf(sA[g], c[1], fmaf(bA[g], qsum[g][1], x[1]));
      x[2] = fmaf(sB[g], c[2], fmaf(bB[g], qsum[g][0], x[2]));
      x[3] = fmaf(sB[g], c[3], fmaf(bB[g], qsum[g][1], x[3]));
    }
  }
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// O^T += V^T . (s P/16)^T for 16 tokens; P = {(r,2j), (r,2j+1), (r+8,2j), (r+8,2j+1)} pre-scaled by 1/16.
// Masked rows must come with P == 0.
template <int NG>
__device__ __forceinline__ void v_accumulate(WarpState<NG>& ws, const uint8_t* codes, const MetaPtrs& mp, int t0,
                                             const float (&P)[4]) {
  constexpr int WPG = 4 / NG;
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  uint32_t sA[NG], sB[NG];
  float bA[NG], bB[NG];
  ld_row_u<NG>(mp.vs2, t0 + r, sA);
  ld_row_u<NG>(mp.vs2, t0 + r + 8, sB);
  ld_row<NG>(mp.vb, t0 + r, bA);
  ld_row<NG>(mp.vb, t0 + r + 8, bB);
  const uint32_t pA = pack2<__half>(P[0], P[1]);
  const uint32_t pB = pack2<__half>(P[2], P[3]);
  uint32_t pb[NG][2];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    pb[g][0] = movmatrix_t(hmul2(pA, sA[g]));
    pb[g][1] = movmatrix_t(hmul2(pB, sB[g]));
    ws.zacc[g][0] = fmaf(bA[g], P[0], fmaf(bB[g], P[2], ws.zacc[g][0]));
    ws.zacc[g][1] = fmaf(bA[g], P[1], fmaf(bB[g], P[3], ws.zacc[g][1]));
  }
  const uint8_t* vc = codes + kTileI4 * HKV_CODE_BYTES;
  const uint4 vA = *reinterpret_cast<const uint4*>(vc + (t0 + 2 * j) * HKV_CODE_BYTES + 16 * r);
  const uint4 vB = *reinterpret_cast<const uint4*>(vc + (t0 + 8 + 2 * j) * HKV_CODE_BYTES + 16 * r);
  const uint32_t vwa[4] = {vA.x, vA.y, vA.z, vA.w};
  const uint32_t vwb[4] = {vB.x, vB.y, vB.z, vB.w};
  // exact integer codes: the B operand carries s * P rounded to f16, so a bias
  // left in A would cancel against fp32 sums of differently rounded products
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int g = k / WPG;
    uint32_t ha[4], hb[4];
    nib8_to_h2(vwa[k], ha);
    nib8_to_h2(vwb[k], hb);
    const uint32_t a0[4] = {ha[0], ha[1], hb[0], hb[1]};
    const uint32_t a1[4] = {ha[2], ha[3], hb[2], hb[3]};
    mma16816<__half>(ws.o[2 * k], a0, pb[g][0], pb[g][1]);
    mma16816<__half>(ws.o[2 * k + 1], a1, pb[g][0], pb[g][1]);
  }
}

// ---------------------------------------------------------------- dense consumer piece (8 tokens per warp)
template <typename DTy, int NG>
__device__ __forceinline__ void dense_subtile(WarpState<NG>& ws, const uint8_t* stg, int t0, int tok0, int hi,
                                              const uint32_t (&qf)[8][2], int G, float qscale) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const uint32_t kb = smem_u32(stg);
  const uint32_t vb = kb + kTileD * kRowPitch;
  // rows r+8 of the 16-row fragments repeat rows r and are masked (P = 0)
  const uint32_t krow = kb + (t0 + (lane & 7)) * kRowPitch + (lane >> 4) * 16;
  float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kt = 0; kt < 8; ++kt) {
    uint32_t a[4];
    ldsm_x4(a, krow + kt * 32);
    mma16816<DTy>(c, a, qf[kt][0], qf[kt][1]);
  }
  const bool ok = tok0 + r < hi;
  float x[4];
  x[0] = (ok && 2 * j < G) ? c[0] * qscale : -INFINITY;
  x[1] = (ok && 2 * j + 1 < G) ? c[1] * qscale : -INFINITY;
  x[2] = -INFINITY;
  x[3] = -INFINITY;
  float P[4];
  softmax_step<NG, 4>(ws, x, P, 0.f);
  const uint32_t pb0 = movmatrix_t(pack2<DTy>(P[0], P[1]));
  const uint32_t pb1 = 0u;  // tokens t0+8..15 are masked
  const uint32_t vrow = vb + (t0 + (lane & 7)) * kRowPitch + ((lane >> 3) & 1) * 16;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    uint32_t a[4];
    ldsm_x4_t(a, vrow + mt * 32);
    mma16816<DTy>(ws.o[mt], a, pb0, pb1);
  }
}

// Q^T B fragments for this lane: head r (= lane/4), dims 16kt + 2j + {0,1} in
// qf[kt][0] and 16kt + 2j + {8,9} in qf[kt][1] (divided by 16 when hi_div16).
// qa/qb return the values exactly as the tensor core sees them.
template <typename T>
__device__ __forceinline__ void load_q_frags(const DecodeParams& p, int b, int hk, bool hi_div16,
                                             uint32_t (&qf)[8][2], float (&qa)[8][2], float (&qb)[8][2]) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const bool live = r < p.G;
  const int hq = hk * p.G + (live ? r : 0);
  const int64_t base = (int64_t)b * p.q_sb + (int64_t)hq * p.q_sh;
  const float sc = hi_div16 ? 0.0625f : 1.0f;
#pragma unroll
  for (int kt = 0; kt < 8; ++kt) {
    const int d = 16 * kt + 2 * j;
    float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
    if (live) {
      v0 = load_any(p.q, p.q_dtype, base + d);
      v1 = load_any(p.q, p.q_dtype, base + d + 1);
      v2 = load_any(p.q, p.q_dtype, base + d + 8);
      v3 = load_any(p.q, p.q_dtype, base + d + 9);
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

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory"); }

// ---------------------------------------------------------------- producer helpers
// Slots at or past `valid` (beyond the sequence length) may hold uninitialised
// pool bytes: their expanded scale and bias are written as zeros, so a masked
// token (P = 0) contributes exactly 0 and never NaN.
template <int FMT, int NG>
__device__ __forceinline__ void expand_meta(const uint8_t* raw, uint8_t* meta, int lane, int valid) {
  // raw: K scales | V scales | K zps | V zps (ref) ; K (s,min) | V (s,min) (fp16min), each [128][NG]
  float* ks = reinterpret_cast<float*>(meta);
  float* kb = ks + kTileI4 * NG;
  uint32_t* vs2 = reinterpret_cast<uint32_t*>(kb + kTileI4 * NG);
  float* vb = reinterpret_cast<float*>(vs2 + kTileI4 * NG);
  constexpr int N = kTileI4 * NG;
#pragma unroll 4
  for (int i = lane; i < N; i += 32) {
    float sk, bk, sv, bv;
    if (FMT == HKV_FMT_REF) {
      const float* sc = reinterpret_cast<const float*>(raw);
      const uint8_t* zp = raw + 2 * N * 4;
      sk = sc[i];
      sv = sc[N + i];
      bk = -static_cast<float>(zp[i]) * sk;
      bv = -static_cast<float>(zp[N + i]) * sv;
    } else {
      const __half2* sm = reinterpret_cast<const __half2*>(raw);
      const float2 fk = __half22float2(sm[i]);
      const float2 fv = __half22float2(sm[N + i]);
      sk = fk.x;
      bk = fk.y;
      sv = fv.x;
      bv = fv.y;
    }
    if (i / NG >= valid) sk = bk = sv = bv = 0.f;
    ks[i] = sk;
    kb[i] = bk;
    vs2[i] = pack2<__half>(sv, sv);
    vb[i] = bv;
  }
}

// ---------------------------------------------------------------- the persistent kernel
template <int FMT, int GROUP, typename DTy>
__global__ void __launch_bounds__(kDecodeThreads, 2) decode_kernel(const DecodeParams p) {
  constexpr int NG = HKV_D / GROUP;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxSlots];
  __shared__ __align__(8) uint64_t ready_bar[kMaxSlots];
  __shared__ __align__(8) uint64_t empty_bar[kMaxSlots];
  __shared__ __align__(8) uint64_t mempty_bar[kMetaSlots];
  __shared__ int s_last;

  const Sched& sc = p.sc;
  const int c = blockIdx.x;
  const int64_t end = cta_begin(sc, c + 1);
  const int nsl = p.nslots;
  uint8_t* ring = smem;
  uint8_t* meta_ring = smem + nsl * p.slot_bytes;
  float* comb = reinterpret_cast<float*>(meta_ring + kMetaSlots * p.meta_bytes);  // [4][G][128] + [4][8][2]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < nsl; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&ready_bar[i], 1);
      mbar_init(&empty_bar[i], kConsumerWarps);
    }
    for (int i = 0; i < kMetaSlots; ++i) mbar_init(&mempty_bar[i], kConsumerWarps);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ================================================================ producer warp
    // Issue walks the tile list ahead of expansion by up to nsl loads.
    TileRef it_issue = first_tile(sc, c), it_exp = it_issue;
    int n_issue = 0, n_exp = 0, nb_exp = 0;
    bool ok = true;
    auto issue_one = [&](void) -> bool {
      // advance to the next tile with data; returns false when the range is exhausted
      while (it_issue.valid && !tile_has_data(p, it_issue)) next_tile(p, end, it_issue);
      if (!it_issue.valid) return false;
      const int slot = n_issue % nsl;
      if (n_issue >= nsl && !mbar_wait(&empty_bar[slot], ((n_issue / nsl) & 1) ^ 1)) {
        ok = false;
        return false;
      }
      uint8_t* sb = ring + slot * p.slot_bytes;
      const int u = it_issue.u;
      if (it_issue.seg == 0) {
        if (lane == 0) {
          const int t = it_issue.k * kTileI4;
          const int64_t page = store_page(p.body, u, t);
          if (page < 0) {
            hkv_flag_error(HKV_DEVERR_BAD_PAGE);
            mbar_arrive(&full_bar[slot]);
          } else {
            const uint32_t codes_b = kTileI4 * HKV_CODE_BYTES;
            const uint32_t sc_b = kTileI4 * 4 * NG;
            const uint32_t zp_b = FMT == HKV_FMT_REF ? kTileI4 * NG : 0;
            const int off = t % p.body.page_tokens;
            const SideAddr ka = side_addr(p.body.k, p.body, page, off);
            const SideAddr va = side_addr(p.body.v, p.body, page, off);
            mbar_arrive_expect_tx(&full_bar[slot], 2 * (codes_b + sc_b + zp_b));
            bulk_g2s(sb, ka.codes, codes_b, &full_bar[slot]);
            bulk_g2s(sb + codes_b, va.codes, codes_b, &full_bar[slot]);
            bulk_g2s(sb + 2 * codes_b, ka.scales, sc_b, &full_bar[slot]);
            bulk_g2s(sb + 2 * codes_b + sc_b, va.scales, sc_b, &full_bar[slot]);
            if (FMT == HKV_FMT_REF) {
              bulk_g2s(sb + 2 * codes_b + 2 * sc_b, ka.zps, zp_b, &full_bar[slot]);
              bulk_g2s(sb + 2 * codes_b + 2 * sc_b + zp_b, va.zps, zp_b, &full_bar[slot]);
            }
          }
        }
      } else {
        const int b = u / p.Hkv, hk = u % p.Hkv;
        const int hi = dense_len(p, u);
        const DTy* kbase = static_cast<const DTy*>(p.dense.k) + b * p.dense.stride_b + hk * p.dense.stride_h;
        const DTy* vbase = static_cast<const DTy*>(p.dense.v) + b * p.dense.stride_b + hk * p.dense.stride_h;
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], 2 * kTileD * HKV_D * 2);
        __syncwarp();
        // rows past the length repeat the last valid row (finite data; masked by P = 0)
        const int64_t src = min(it_issue.k * kTileD + lane, hi - 1);
        bulk_g2s(sb + lane * kRowPitch, kbase + src * p.dense.stride_t, HKV_D * 2, &full_bar[slot]);
        bulk_g2s(sb + kTileD * kRowPitch + lane * kRowPitch, vbase + src * p.dense.stride_t, HKV_D * 2,
                 &full_bar[slot]);
      }
      n_issue++;
      next_tile(p, end, it_issue);
      return true;
    };
    for (int i = 0; i < nsl - 1 && issue_one(); ++i) {
    }
    while (ok) {
      while (it_exp.valid && !tile_has_data(p, it_exp)) next_tile(p, end, it_exp);
      if (!it_exp.valid) break;
      const int slot = n_exp % nsl;
      if (!mbar_wait(&full_bar[slot], (n_exp / nsl) & 1)) break;
      if (it_exp.seg == 0) {
        const int ms = nb_exp % kMetaSlots;
        if (nb_exp >= kMetaSlots && !mbar_wait(&mempty_bar[ms], ((nb_exp / kMetaSlots) & 1) ^ 1)) break;
        expand_meta<FMT, NG>(ring + slot * p.slot_bytes + 2 * kTileI4 * HKV_CODE_BYTES,
                             meta_ring + ms * p.meta_bytes, lane, body_len(p, it_exp.u) - it_exp.k * kTileI4);
        nb_exp++;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready_bar[slot]);
      n_exp++;
      next_tile(p, end, it_exp);
      issue_one();
    }
    // drain: every issued copy must have landed before the CTA exits
    if (lane == 0) {
      for (int i = max(0, n_issue - nsl); i < n_issue; ++i) mbar_wait(&full_bar[i % nsl], (i / nsl) & 1);
    }
    return;
  }

  // ================================================================== consumer warps
  WarpState<NG> ws;
  ws_reset<NG>(ws);
  uint32_t qf[8][2];
  float qsum[NG][2], nbias[NG][2];
  const int r = lane >> 2, j = lane & 3;
  const bool h0 = 2 * j < p.G, h1 = 2 * j + 1 < p.G;
  int n_load = 0, nb_load = 0;
  TileRef it = first_tile(sc, c);
  int cur_u = -1, cur_seg = -1;
  bool alive = true;

  auto begin_piece = [&](int u, int seg) {
    const int b = u / p.Hkv, hk = u % p.Hkv;
    float qa[8][2], qb[8][2];
    if (seg == 0) {
      load_q_frags<__half>(p, b, hk, true, qf, qa, qb);
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
        qsum[g][0] = __shfl_sync(0xffffffffu, ps[g], (2 * j) * 4);
        qsum[g][1] = __shfl_sync(0xffffffffu, ps[g], (2 * j + 1) * 4);
        nbias[g][0] = -1024.f * __shfl_sync(0xffffffffu, pbias[g], (2 * j) * 4);
        nbias[g][1] = -1024.f * __shfl_sync(0xffffffffu, pbias[g], (2 * j + 1) * 4);
      }
    } else {
      load_q_frags<DTy>(p, b, hk, false, qf, qa, qb);
    }
    ws_reset<NG>(ws);
    cur_u = u;
    cur_seg = seg;
  };

  auto end_piece = [&]() {
    // 1. per-warp partials to shared memory
    const bool body = cur_seg == 0;
    float l0 = ws.l[0], l1 = ws.l[1];
#pragma unroll
    for (int sft = 4; sft < 32; sft <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, sft);
      l1 += __shfl_xor_sync(0xffffffffu, l1, sft);
    }
    float z[NG][2];
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      z[g][0] = body ? ws.zacc[g][0] : 0.f;
      z[g][1] = body ? ws.zacc[g][1] : 0.f;
#pragma unroll
      for (int sft = 4; sft < 32; sft <<= 1) {
        z[g][0] += __shfl_xor_sync(0xffffffffu, z[g][0], sft);
        z[g][1] += __shfl_xor_sync(0xffffffffu, z[g][1], sft);
      }
    }
    float* wo = comb + warp * p.G * HKV_D;
    float* cml = comb + kConsumerWarps * p.G * HKV_D;  // [4][8][2]
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d0 = 16 * mt + r, d1 = d0 + 8;
      const int g = (16 * mt) / GROUP;
      const float osc = body ? 16.f : 1.f;  // INT4 tiles accumulate with P/16
      if (h0) {
        wo[(2 * j) * HKV_D + d0] = osc * (ws.o[mt][0] + z[g][0]);
        wo[(2 * j) * HKV_D + d1] = osc * (ws.o[mt][2] + z[g][0]);
      }
      if (h1) {
        wo[(2 * j + 1) * HKV_D + d0] = osc * (ws.o[mt][1] + z[g][1]);
        wo[(2 * j + 1) * HKV_D + d1] = osc * (ws.o[mt][3] + z[g][1]);
      }
    }
    const float lsc = body ? 16.f : 1.f;  // INT4 tiles accumulate P/16
    if (r == 0) {
      cml[(warp * 8 + 2 * j) * 2] = ws.m[0];
      cml[(warp * 8 + 2 * j) * 2 + 1] = l0 * lsc;
      cml[(warp * 8 + 2 * j + 1) * 2] = ws.m[1];
      cml[(warp * 8 + 2 * j + 1) * 2 + 1] = l1 * lsc;
    }
    consumer_sync();
    // 2. combine the four warps into this piece's partial slot
    const int u = cur_u;
    int b0, nb, d0, nd;
    unit_pieces(sc, u, b0, nb, d0, nd);
    const int slot = cur_seg == 0 ? c - b0 : nb + c - d0;
    float* po = p.part_o + ((int64_t)u * sc.S + slot) * p.G * HKV_D;
    float* pml = p.part_ml + ((int64_t)u * sc.S + slot) * p.G * 2;
    for (int idx = threadIdx.x; idx < p.G * HKV_D; idx += kConsumerThreads) {
      const int h = idx / HKV_D, d = idx % HKV_D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, cml[(w * 8 + h) * 2]);
      float acc = 0.f, L = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float mw = cml[(w * 8 + h) * 2];
          if (mw == -INFINITY) continue;
          const float e = fast_exp2(mw - M);
          acc = fmaf(e, comb[(w * p.G + h) * HKV_D + d], acc);
          L = fmaf(e, cml[(w * 8 + h) * 2 + 1], L);
        }
      }
      po[idx] = acc;
      if (d == 0) {
        pml[2 * h] = M;
        pml[2 * h + 1] = L;
      }
    }
    __threadfence();
    consumer_sync();
    if (threadIdx.x == 0) s_last = atomicAdd(&p.counters[u], 1) == nb + nd - 1;
    consumer_sync();
    if (s_last) {
      // 3. last piece of the unit: merge all its partials (warp w: heads w, w+4)
      __threadfence();
      const int n = nb + nd;
      const int b = u / p.Hkv, hk = u % p.Hkv;
      const float* ml_u = p.part_ml + (int64_t)u * sc.S * p.G * 2;
      const float* o_u = p.part_o + (int64_t)u * sc.S * p.G * HKV_D;
      for (int h = warp; h < p.G; h += kConsumerWarps) {
        float M = -INFINITY;
        for (int k = lane; k < n; k += 32) M = fmaxf(M, __ldcg(ml_u + (k * p.G + h) * 2));
#pragma unroll
        for (int sft = 16; sft > 0; sft >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sft));
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k0 = 0; k0 < n; k0 += 32) {
          float wk = 0.f;
          if (k0 + lane < n) {
            const float mk = __ldcg(ml_u + ((k0 + lane) * p.G + h) * 2);
            wk = (mk == -INFINITY || M == -INFINITY) ? 0.f : fast_exp2(mk - M);
            L = fmaf(wk, __ldcg(ml_u + ((k0 + lane) * p.G + h) * 2 + 1), L);
          }
          const int kn = min(32, n - k0);
          for (int kk = 0; kk < kn; ++kk) {
            const float w = __shfl_sync(0xffffffffu, wk, kk);
            if (w == 0.f) continue;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(o_u + ((k0 + kk) * p.G + h) * HKV_D) + lane);
            acc.x = fmaf(w, v.x, acc.x);
            acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z);
            acc.w = fmaf(w, v.w, acc.w);
          }
        }
#pragma unroll
        for (int sft = 16; sft > 0; sft >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sft);
        const int hq = hk * p.G + h;
        if (p.out_o) {
          reinterpret_cast<float4*>(p.out_o + ((int64_t)b * p.Hq + hq) * HKV_D)[lane] = acc;
          if (lane == 0) {
            p.out_ml[((int64_t)b * p.Hq + hq) * 2] = M;
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
      consumer_sync();
      if (threadIdx.x == 0) p.counters[u] = 0;
    }
    consumer_sync();  // the combine area is free again
  };

  const float qs = p.qscale;
  while (it.valid && alive) {
    if (it.u != cur_u || it.seg != cur_seg) {
      if (cur_u >= 0) end_piece();
      begin_piece(it.u, it.seg);
    }
    if (tile_has_data(p, it)) {
      const int slot = n_load % nsl;
      if (!mbar_wait(&ready_bar[slot], (n_load / nsl) & 1)) {
        alive = false;
        break;
      }
      const uint8_t* stg = ring + slot * p.slot_bytes;
      if (it.seg == 0) {
        const int ms = nb_load % kMetaSlots;
        const uint8_t* mbase = meta_ring + ms * p.meta_bytes;
        MetaPtrs mp;
        mp.ks = reinterpret_cast<const float*>(mbase);
        mp.kb = mp.ks + kTileI4 * NG;
        mp.vs2 = reinterpret_cast<const uint32_t*>(mp.kb + kTileI4 * NG);
        mp.vb = reinterpret_cast<const float*>(mp.vs2 + kTileI4 * NG);
        const int hi = body_len(p, it.u);
        const int t0 = warp * 32;
        const int tok = it.k * kTileI4 + t0;
        float xa[4], xb[4], x[8], P[8];
        k_scores<NG>(stg, mp, t0, qf, nbias, qsum, xa);
        k_scores<NG>(stg, mp, t0 + 16, qf, nbias, qsum, xb);
        if (tok + 32 <= hi) {
          x[0] = h0 ? xa[0] * qs : -INFINITY;
          x[1] = h1 ? xa[1] * qs : -INFINITY;
          x[2] = h0 ? xa[2] * qs : -INFINITY;
          x[3] = h1 ? xa[3] * qs : -INFINITY;
          x[4] = h0 ? xb[0] * qs : -INFINITY;
          x[5] = h1 ? xb[1] * qs : -INFINITY;
          x[6] = h0 ? xb[2] * qs : -INFINITY;
          x[7] = h1 ? xb[3] * qs : -INFINITY;
        } else {
          const bool ok0 = tok + r < hi, ok1 = tok + r + 8 < hi;
          const bool ok2 = tok + 16 + r < hi, ok3 = tok + 24 + r < hi;
          x[0] = (ok0 && h0) ? xa[0] * qs : -INFINITY;
          x[1] = (ok0 && h1) ? xa[1] * qs : -INFINITY;
          x[2] = (ok1 && h0) ? xa[2] * qs : -INFINITY;
          x[3] = (ok1 && h1) ? xa[3] * qs : -INFINITY;
          x[4] = (ok2 && h0) ? xb[0] * qs : -INFINITY;
          x[5] = (ok2 && h1) ? xb[1] * qs : -INFINITY;
          x[6] = (ok3 && h0) ? xb[2] * qs : -INFINITY;
          x[7] = (ok3 && h1) ? xb[3] * qs : -INFINITY;
        }
        softmax_step<NG, 8>(ws, x, P, 4.f);
        const float pa[4] = {P[0], P[1], P[2], P[3]};
        const float pc[4] = {P[4], P[5], P[6], P[7]};
        v_accumulate<NG>(ws, stg, mp, t0, pa);
        v_accumulate<NG>(ws, stg, mp, t0 + 16, pc);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty_bar[slot]);
          mbar_arrive(&mempty_bar[ms]);
        }
        nb_load++;
      } else {
        const int hi = dense_len(p, it.u);
        const int t0 = warp * 8;
        dense_subtile<DTy, NG>(ws, stg, t0, it.k * kTileD + t0, hi, qf, p.G, qs);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[slot]);
      }
      n_load++;
    }
    next_tile(p, end, it);
  }
  if (cur_u >= 0) end_piece();
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

}  // namespace hkv
