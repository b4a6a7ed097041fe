// Split-KV GQA decode attention over packed INT4 pages + a dense fp16/bf16
// segment, and the log-sum-exp merge. Included by hetero_kv.cu.
//
// Grid: (splits_body + splits_dense, B*Hkv). Each CTA owns one token range of
// one (sequence, KV head) unit and all G = Hq/Hkv query heads of that unit.
// Warp 4 is the producer: it streams 128-token INT4 stages (or 64-token dense
// stages) into a shared-memory ring with 1-D bulk async copies (TMA engine,
// no multicast) completing on mbarriers. Warps 0-3 consume 16-token
// sub-tiles with m16n8k16 tensor-core MMAs:
//   S^T[tok][head] = K[tok][:] . Q^T      (M = 16 tokens, N = 8 heads, K = dims)
//   O^T[dim][head] += V^T[dim][tok] . P^T (M = 16 dims,   N = 8 heads, K = tokens)
// K and V fragments are produced in registers straight from the packed nibbles
// (the nibble order of the page format is the fragment order), as exact
// integers 0..15 in f16. Per-group scale / zero are applied in fp32:
//   score = sum_g s_g * (codes_g . Q) + b_g * sum(Q_g)      (b = -z*s or min)
//   O    += codes . (s_g * P)  +  b_g * sum(P)              (per group g)
// The online softmax runs in the base-2 domain in fp32 with a lazy rescale
// (the running max only moves when a tile exceeds it by more than 2^8).
#pragma once
#include "hkv_common.cuh"

namespace hkv {

constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;
constexpr int kTileI4 = 128;     // tokens per INT4 stage (32 per consumer warp)
constexpr int kTileD = 64;       // tokens per dense stage (16 per consumer warp)
constexpr int kRowPitch = 272;   // bytes per dense row in shared memory (256 + 16: conflict-free ldmatrix)
constexpr int kStageD = 2 * kTileD * kRowPitch;
constexpr int kMaxStages = 8;
constexpr float kLazyRescale = 8.0f;

struct DecodeParams {
  const void* q;
  int q_dtype;
  int64_t q_sb, q_sh;
  hkv_int4_store body;
  hkv_dense_kv dense;
  int B, Hq, Hkv, G;
  float qscale;  // sm_scale * log2(e)
  int splits_body, splits_dense;
  int chunk_body, chunk_dense;
  int ring_bytes;
  float* part_o;   // [units][S][G][128]
  float* part_ml;  // [units][S][G][2]
};

__host__ __device__ constexpr int i4_stage_bytes(int fmt, int group) {
  return 2 * kTileI4 * HKV_CODE_BYTES + 2 * kTileI4 * 4 * (HKV_D / group) +
         (fmt == HKV_FMT_REF ? 2 * kTileI4 * (HKV_D / group) : 0);
}

// Online-softmax state of one consumer warp. Thread (r = lane/4, j = lane%4)
// owns heads 2j and 2j+1 in every accumulator below.
template <int NG>
struct WarpState {
  float o[8][4];     // O^T accumulators, m-tile mt: (dim 16mt+r | +8) x (head 2j | 2j+1)
  float zacc[NG][2]; // sum_t b_g(t) P(t, head) of the V zero term
  float m[2], l[2];
};

template <int NG>
__device__ __forceinline__ void softmax_step(WarpState<NG>& ws, float (&x)[4], float (&P)[4]) {
  float t0 = fmaxf(x[0], x[2]), t1 = fmaxf(x[1], x[3]);
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
  P[0] = x[0] == -INFINITY ? 0.f : fast_exp2(x[0] - ws.m[0]);
  P[1] = x[1] == -INFINITY ? 0.f : fast_exp2(x[1] - ws.m[1]);
  P[2] = x[2] == -INFINITY ? 0.f : fast_exp2(x[2] - ws.m[0]);
  P[3] = x[3] == -INFINITY ? 0.f : fast_exp2(x[3] - ws.m[1]);
  ws.l[0] += P[0] + P[2];
  ws.l[1] += P[1] + P[3];
}

// ---------------------------------------------------------------- INT4 sub-tile (16 tokens)
template <int FMT, int NG>
__device__ __forceinline__ void int4_subtile(WarpState<NG>& ws, const uint8_t* stg, int t0, int tok0, int hi,
                                             const uint32_t (&qf)[8][2], const float (&qsum)[NG][2], int G,
                                             float qscale) {
  constexpr int WPG = 4 / NG;  // packed words per group
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const uint8_t* kc = stg;
  const uint8_t* vc = stg + kTileI4 * HKV_CODE_BYTES;
  const uint8_t* ks = stg + 2 * kTileI4 * HKV_CODE_BYTES;
  const uint8_t* vs = ks + kTileI4 * 4 * NG;
  const uint8_t* kz = vs + kTileI4 * 4 * NG;
  const uint8_t* vz = kz + kTileI4 * NG;

  // ---- S^T = K . Q^T, one accumulator per group
  const uint4 kA = *reinterpret_cast<const uint4*>(kc + (t0 + r) * HKV_CODE_BYTES + 16 * j);
  const uint4 kB = *reinterpret_cast<const uint4*>(kc + (t0 + r + 8) * HKV_CODE_BYTES + 16 * j);
  const uint32_t kwa[4] = {kA.x, kA.y, kA.z, kA.w};
  const uint32_t kwb[4] = {kB.x, kB.y, kB.z, kB.w};
  float c[NG][4];
#pragma unroll
  for (int g = 0; g < NG; ++g) c[g][0] = c[g][1] = c[g][2] = c[g][3] = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t ha[4], hb[4];
    nib8_to_h2(kwa[w], ha);
    nib8_to_h2(kwb[w], hb);
    const uint32_t a0[4] = {ha[0], hb[0], ha[1], hb[1]};
    const uint32_t a1[4] = {ha[2], hb[2], ha[3], hb[3]};
    mma16816<__half>(c[w / WPG], a0, qf[2 * w][0], qf[2 * w][1]);
    mma16816<__half>(c[w / WPG], a1, qf[2 * w + 1][0], qf[2 * w + 1][1]);
  }
  // ---- K metadata of rows r and r+8
  float sA[NG], sB[NG], bA[NG], bB[NG];
  if (FMT == HKV_FMT_REF) {
    const float* sc = reinterpret_cast<const float*>(ks);
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      sA[g] = sc[(t0 + r) * NG + g];
      sB[g] = sc[(t0 + r + 8) * NG + g];
      bA[g] = -static_cast<float>(kz[(t0 + r) * NG + g]) * sA[g];
      bB[g] = -static_cast<float>(kz[(t0 + r + 8) * NG + g]) * sB[g];
    }
  } else {
    const __half2* sm = reinterpret_cast<const __half2*>(ks);
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const float2 fa = __half22float2(sm[(t0 + r) * NG + g]);
      const float2 fb = __half22float2(sm[(t0 + r + 8) * NG + g]);
      sA[g] = fa.x;
      bA[g] = fa.y;
      sB[g] = fb.x;
      bB[g] = fb.y;
    }
  }
  float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    x[0] = fmaf(sA[g], c[g][0], fmaf(bA[g], qsum[g][0], x[0]));
    x[1] = fmaf(sA[g], c[g][1], fmaf(bA[g], qsum[g][1], x[1]));
    x[2] = fmaf(sB[g], c[g][2], fmaf(bB[g], qsum[g][0], x[2]));
    x[3] = fmaf(sB[g], c[g][3], fmaf(bB[g], qsum[g][1], x[3]));
  }
  const bool okA = tok0 + r < hi, okB = tok0 + r + 8 < hi;
  const bool h0 = 2 * j < G, h1 = 2 * j + 1 < G;
  x[0] = (okA && h0) ? x[0] * qscale : -INFINITY;
  x[1] = (okA && h1) ? x[1] * qscale : -INFINITY;
  x[2] = (okB && h0) ? x[2] * qscale : -INFINITY;
  x[3] = (okB && h1) ? x[3] * qscale : -INFINITY;
  float P[4];
  softmax_step<NG>(ws, x, P);

  // ---- V metadata of rows r and r+8; B fragments s_g * P per group
  float svA[NG], svB[NG], bvA[NG], bvB[NG];
  if (FMT == HKV_FMT_REF) {
    const float* sc = reinterpret_cast<const float*>(vs);
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      svA[g] = okA ? sc[(t0 + r) * NG + g] : 0.f;
      svB[g] = okB ? sc[(t0 + r + 8) * NG + g] : 0.f;
      bvA[g] = -static_cast<float>(vz[(t0 + r) * NG + g]) * svA[g];
      bvB[g] = -static_cast<float>(vz[(t0 + r + 8) * NG + g]) * svB[g];
    }
  } else {
    const __half2* sm = reinterpret_cast<const __half2*>(vs);
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const float2 fa = __half22float2(sm[(t0 + r) * NG + g]);
      const float2 fb = __half22float2(sm[(t0 + r + 8) * NG + g]);
      svA[g] = okA ? fa.x : 0.f;
      bvA[g] = okA ? fa.y : 0.f;
      svB[g] = okB ? fb.x : 0.f;
      bvB[g] = okB ? fb.y : 0.f;
    }
  }
  uint32_t pb[NG][2];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    pb[g][0] = movmatrix_t(pack2<__half>(svA[g] * P[0], svA[g] * P[1]));
    pb[g][1] = movmatrix_t(pack2<__half>(svB[g] * P[2], svB[g] * P[3]));
    ws.zacc[g][0] = fmaf(bvA[g], P[0], fmaf(bvB[g], P[2], ws.zacc[g][0]));
    ws.zacc[g][1] = fmaf(bvA[g], P[1], fmaf(bvB[g], P[3], ws.zacc[g][1]));
  }
  // ---- O^T += V^T . (s P)^T
  const uint4 vA = *reinterpret_cast<const uint4*>(vc + (t0 + 2 * j) * HKV_CODE_BYTES + 16 * r);
  const uint4 vB = *reinterpret_cast<const uint4*>(vc + (t0 + 8 + 2 * j) * HKV_CODE_BYTES + 16 * r);
  const uint32_t vwa[4] = {vA.x, vA.y, vA.z, vA.w};
  const uint32_t vwb[4] = {vB.x, vB.y, vB.z, vB.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t ha[4], hb[4];
    nib8_to_h2(vwa[k], ha);
    nib8_to_h2(vwb[k], hb);
    const uint32_t a0[4] = {ha[0], ha[1], hb[0], hb[1]};
    const uint32_t a1[4] = {ha[2], ha[3], hb[2], hb[3]};
    mma16816<__half>(ws.o[2 * k], a0, pb[k / WPG][0], pb[k / WPG][1]);
    mma16816<__half>(ws.o[2 * k + 1], a1, pb[k / WPG][0], pb[k / WPG][1]);
  }
}

// ---------------------------------------------------------------- dense sub-tile (16 tokens)
template <typename DTy, int NG>
__device__ __forceinline__ void dense_subtile(WarpState<NG>& ws, const uint8_t* stg, int t0, int tok0, int hi,
                                              const uint32_t (&qf)[8][2], int G, float qscale) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const uint32_t kb = smem_u32(stg);
  const uint32_t vb = kb + kTileD * kRowPitch;
  float c[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t krow = kb + (t0 + (lane & 7) + ((lane >> 3) & 1) * 8) * kRowPitch + (lane >> 4) * 16;
#pragma unroll
  for (int kt = 0; kt < 8; ++kt) {
    uint32_t a[4];
    ldsm_x4(a, krow + kt * 32);
    mma16816<DTy>(c, a, qf[kt][0], qf[kt][1]);
  }
  const bool okA = tok0 + r < hi, okB = tok0 + r + 8 < hi;
  const bool h0 = 2 * j < G, h1 = 2 * j + 1 < G;
  float x[4];
  x[0] = (okA && h0) ? c[0] * qscale : -INFINITY;
  x[1] = (okA && h1) ? c[1] * qscale : -INFINITY;
  x[2] = (okB && h0) ? c[2] * qscale : -INFINITY;
  x[3] = (okB && h1) ? c[3] * qscale : -INFINITY;
  float P[4];
  softmax_step<NG>(ws, x, P);
  const uint32_t pb0 = movmatrix_t(pack2<DTy>(P[0], P[1]));
  const uint32_t pb1 = movmatrix_t(pack2<DTy>(P[2], P[3]));
  const uint32_t vrow = vb + (t0 + (lane & 7) + (lane >> 4) * 8) * kRowPitch + ((lane >> 3) & 1) * 16;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    uint32_t a[4];
    ldsm_x4_t(a, vrow + mt * 32);
    mma16816<DTy>(ws.o[mt], a, pb0, pb1);
  }
}

// Q^T B fragments for this lane: head r (= lane/4), dims 16kt + 2j + {0,1,8,9}.
template <typename T>
__device__ __forceinline__ void load_q_frags(const DecodeParams& p, int b, int hk, uint32_t (&qf)[8][2],
                                             float (&qv)[8][4]) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const bool live = r < p.G;
  const int hq = hk * p.G + (live ? r : 0);
  const int64_t base = (int64_t)b * p.q_sb + (int64_t)hq * p.q_sh;
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
    qf[kt][0] = pack2<T>(v0, v1);
    qf[kt][1] = pack2<T>(v2, v3);
    // values as the tensor core sees them (rounded to T)
    qv[kt][0] = to_f32(from_f32<T>(v0));
    qv[kt][1] = to_f32(from_f32<T>(v1));
    qv[kt][2] = to_f32(from_f32<T>(v2));
    qv[kt][3] = to_f32(from_f32<T>(v3));
  }
}

// ---------------------------------------------------------------- the split kernel
template <int FMT, int GROUP, typename DTy>
__global__ void __launch_bounds__(kDecodeThreads, 2) decode_split_kernel(const DecodeParams p) {
  constexpr int NG = HKV_D / GROUP;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];

  const int u = blockIdx.y;
  const int b = u / p.Hkv, hk = u % p.Hkv;
  const int s = blockIdx.x;
  const int S = p.splits_body + p.splits_dense;
  const bool is_body = s < p.splits_body;
  int lo, hi;
  // The last split of each segment runs to the true length, so a stale
  // host-side length hint can only unbalance the grid, never drop tokens.
  if (is_body) {
    const int L = p.body.lengths ? p.body.lengths[b] : p.body.len;
    lo = s * p.chunk_body;
    hi = s == p.splits_body - 1 ? L : min(lo + p.chunk_body, L);
  } else {
    const int L = p.dense.lengths ? p.dense.lengths[b] : p.dense.len;
    const int sd = s - p.splits_body;
    lo = sd * p.chunk_dense;
    hi = sd == p.splits_dense - 1 ? L : min(lo + p.chunk_dense, L);
  }
  float* po = p.part_o + ((int64_t)u * S + s) * p.G * HKV_D;
  float* pml = p.part_ml + ((int64_t)u * S + s) * p.G * 2;
  if (lo >= hi) {  // empty range: neutral partial
    for (int i = threadIdx.x; i < p.G * HKV_D; i += blockDim.x) po[i] = 0.f;
    for (int i = threadIdx.x; i < p.G; i += blockDim.x) {
      pml[2 * i] = -INFINITY;
      pml[2 * i + 1] = 0.f;
    }
    return;
  }
  const int tile = is_body ? kTileI4 : kTileD;
  const int ntiles = (hi - lo + tile - 1) / tile;
  const int stage_bytes = is_body ? i4_stage_bytes(FMT, GROUP) : kStageD;
  const int nst = min(kMaxStages, p.ring_bytes / stage_bytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  WarpState<NG> ws;
  if (warp == kConsumerWarps) {
    // ============================== producer warp
    int issued = 0;
    if (is_body) {
      const int ms = i4_stage_bytes(FMT, GROUP);
      const uint32_t codes_b = kTileI4 * HKV_CODE_BYTES;
      const uint32_t sc_b = kTileI4 * 4 * NG;
      const uint32_t zp_b = FMT == HKV_FMT_REF ? kTileI4 * NG : 0;
      const uint32_t tx = 2 * (codes_b + sc_b + zp_b);
      if (lane == 0) {
        for (int i = 0; i < ntiles; ++i) {
          const int st = i % nst;
          if (i >= nst && !mbar_wait(&empty_bar[st], ((i / nst) & 1) ^ 1)) break;
          const int t = lo + i * kTileI4;
          const int64_t page = store_page(p.body, u, t);
          uint8_t* sb = smem + st * ms;
          issued = i + 1;
          if (page < 0) {
            hkv_flag_error(HKV_DEVERR_BAD_PAGE);
            mbar_arrive(&full_bar[st]);
            continue;
          }
          const int off = t % p.body.page_tokens;
          const SideAddr ka = side_addr(p.body.k, p.body, page, off);
          const SideAddr va = side_addr(p.body.v, p.body, page, off);
          mbar_arrive_expect_tx(&full_bar[st], tx);
          bulk_g2s(sb, ka.codes, codes_b, &full_bar[st]);
          bulk_g2s(sb + codes_b, va.codes, codes_b, &full_bar[st]);
          bulk_g2s(sb + 2 * codes_b, ka.scales, sc_b, &full_bar[st]);
          bulk_g2s(sb + 2 * codes_b + sc_b, va.scales, sc_b, &full_bar[st]);
          if (FMT == HKV_FMT_REF) {
            bulk_g2s(sb + 2 * codes_b + 2 * sc_b, ka.zps, zp_b, &full_bar[st]);
            bulk_g2s(sb + 2 * codes_b + 2 * sc_b + zp_b, va.zps, zp_b, &full_bar[st]);
          }
        }
      }
    } else {
      const DTy* kbase = static_cast<const DTy*>(p.dense.k) + b * p.dense.stride_b + hk * p.dense.stride_h;
      const DTy* vbase = static_cast<const DTy*>(p.dense.v) + b * p.dense.stride_b + hk * p.dense.stride_h;
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % nst;
        if (i >= nst && !mbar_wait(&empty_bar[st], ((i / nst) & 1) ^ 1)) break;
        const int t = lo + i * kTileD;
        uint8_t* sb = smem + st * kStageD;
        issued = i + 1;
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[st], 2 * kTileD * HKV_D * 2);
        __syncwarp();
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int row = lane + 32 * rr;
          const int64_t src = min(t + row, hi - 1);  // rows past the range repeat the last valid row
          bulk_g2s(sb + row * kRowPitch, kbase + src * p.dense.stride_t, HKV_D * 2, &full_bar[st]);
          bulk_g2s(sb + kTileD * kRowPitch + row * kRowPitch, vbase + src * p.dense.stride_t, HKV_D * 2,
                   &full_bar[st]);
        }
      }
    }
    // drain: every issued copy must have landed before the CTA can exit
    if (lane == 0) {
      for (int i = max(0, issued - nst); i < issued; ++i) mbar_wait(&full_bar[i % nst], (i / nst) & 1);
    }
  } else {
    // ============================== consumer warps
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) ws.o[mt][0] = ws.o[mt][1] = ws.o[mt][2] = ws.o[mt][3] = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) ws.zacc[g][0] = ws.zacc[g][1] = 0.f;
    ws.m[0] = ws.m[1] = -INFINITY;
    ws.l[0] = ws.l[1] = 0.f;
    uint32_t qf[8][2];
    float qv[8][4];
    if (is_body) {
      load_q_frags<__half>(p, b, hk, qf, qv);
      // sum of Q over each group for heads 2j, 2j+1 (Q as rounded to f16)
      float qsum[NG][2];
      const int j = lane & 3;
      float part[NG];
#pragma unroll
      for (int g = 0; g < NG; ++g) part[g] = 0.f;
#pragma unroll
      for (int kt = 0; kt < 8; ++kt) part[(kt * 16) / GROUP] += qv[kt][0] + qv[kt][1] + qv[kt][2] + qv[kt][3];
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        part[g] += __shfl_xor_sync(0xffffffffu, part[g], 1);
        part[g] += __shfl_xor_sync(0xffffffffu, part[g], 2);
        qsum[g][0] = __shfl_sync(0xffffffffu, part[g], (2 * j) * 4);
        qsum[g][1] = __shfl_sync(0xffffffffu, part[g], (2 * j + 1) * 4);
      }
      const int ms = i4_stage_bytes(FMT, GROUP);
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % nst;
        if (!mbar_wait(&full_bar[st], (i / nst) & 1)) break;
        const uint8_t* stg = smem + st * ms;
        const int tb = lo + i * kTileI4;
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
          const int t0 = warp * 32 + sub * 16;
          int4_subtile<FMT, NG>(ws, stg, t0, tb + t0, hi, qf, qsum, p.G, p.qscale);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[st]);
      }
    } else {
      load_q_frags<DTy>(p, b, hk, qf, qv);
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % nst;
        if (!mbar_wait(&full_bar[st], (i / nst) & 1)) break;
        const uint8_t* stg = smem + st * kStageD;
        const int tb = lo + i * kTileD;
        const int t0 = warp * 16;
        dense_subtile<DTy, NG>(ws, stg, t0, tb + t0, hi, qf, p.G, p.qscale);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[st]);
      }
    }
  }
  __syncthreads();  // ring no longer in use: reuse it for the cross-warp combine

  float* ep_o = reinterpret_cast<float*>(smem);                       // [4 warps][8 heads][128]
  float* ep_ml = ep_o + kConsumerWarps * 8 * HKV_D;                   // [4 warps][8 heads][2]
  if (warp < kConsumerWarps) {
    const int r = lane >> 2, j = lane & 3;
    float l0 = ws.l[0], l1 = ws.l[1];
#pragma unroll
    for (int sft = 4; sft < 32; sft <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, sft);
      l1 += __shfl_xor_sync(0xffffffffu, l1, sft);
    }
    float z[NG][2];
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      z[g][0] = is_body ? ws.zacc[g][0] : 0.f;
      z[g][1] = is_body ? ws.zacc[g][1] : 0.f;
#pragma unroll
      for (int sft = 4; sft < 32; sft <<= 1) {
        z[g][0] += __shfl_xor_sync(0xffffffffu, z[g][0], sft);
        z[g][1] += __shfl_xor_sync(0xffffffffu, z[g][1], sft);
      }
    }
    float* wo = ep_o + warp * 8 * HKV_D;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d0 = 16 * mt + r, d1 = d0 + 8;
      const int g = (16 * mt) / GROUP;
      wo[(2 * j) * HKV_D + d0] = ws.o[mt][0] + z[g][0];
      wo[(2 * j + 1) * HKV_D + d0] = ws.o[mt][1] + z[g][1];
      wo[(2 * j) * HKV_D + d1] = ws.o[mt][2] + z[g][0];
      wo[(2 * j + 1) * HKV_D + d1] = ws.o[mt][3] + z[g][1];
    }
    if (r == 0) {
      float* wml = ep_ml + warp * 16;
      wml[(2 * j) * 2] = ws.m[0];
      wml[(2 * j) * 2 + 1] = l0;
      wml[(2 * j + 1) * 2] = ws.m[1];
      wml[(2 * j + 1) * 2 + 1] = l1;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.G * HKV_D; idx += blockDim.x) {
    const int h = idx / HKV_D, d = idx % HKV_D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, ep_ml[w * 16 + 2 * h]);
    float acc = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = ep_ml[w * 16 + 2 * h];
        if (mw == -INFINITY) continue;
        const float sc = fast_exp2(mw - M);
        acc = fmaf(sc, ep_o[(w * 8 + h) * HKV_D + d], acc);
        L = fmaf(sc, ep_ml[w * 16 + 2 * h + 1], L);
      }
    }
    po[idx] = acc;
    if (d == 0) {
      pml[2 * h] = M;
      pml[2 * h + 1] = L;
    }
  }
}

// ---------------------------------------------------------------- log-sum-exp merge
// One block of 128 threads per output row (b, hq). Partial s of that row is at
//   o:  part_o  + u*unit_o  + g*128 + s*split_o,   ml: part_ml + u*unit_ml + g*2 + s*split_ml
// with u = b*Hkv + hq/G, g = hq%G.
struct MergeParams {
  const float* part_o;
  const float* part_ml;
  int S, Hq, Hkv, G;
  int64_t unit_o, split_o, unit_ml, split_ml;
  void* out;
  int out_dtype;
  int64_t out_sb, out_sh;
  float* out_o;   // partial-output mode when non-null
  float* out_ml;
};

__global__ void __launch_bounds__(128) lse_merge_kernel(const MergeParams mp) {
  const int row = blockIdx.x;
  const int b = row / mp.Hq, hq = row % mp.Hq;
  const int u = b * mp.Hkv + hq / mp.G, g = hq % mp.G;
  const int d = threadIdx.x;
  const float* po = mp.part_o + u * mp.unit_o + g * HKV_D + d;
  const float* pml = mp.part_ml + u * mp.unit_ml + g * 2;
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
  if (mp.out_o) {
    mp.out_o[(int64_t)row * HKV_D + d] = acc;
    if (d == 0) {
      mp.out_ml[(int64_t)row * 2] = M;
      mp.out_ml[(int64_t)row * 2 + 1] = L;
    }
    return;
  }
  const float v = L > 0.f ? acc / L : 0.f;
  store_any(mp.out, mp.out_dtype, (int64_t)b * mp.out_sb + (int64_t)hq * mp.out_sh + d, v);
}

}  // namespace hkv
