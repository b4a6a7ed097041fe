// Multi-query (prefill) attention over a packed INT4 body on the 5th-generation
// tensor cores (tcgen05). Included by hetero_kv.cu.
//
// One CTA of 128 threads per (sequence, KV head) unit and 128-row query tile;
// rows are (query position, head of the unit's G) pairs, row = s * G + g. Per
// 128-token body tile, in order:
//   1. the raw page block lands in one of two ring slots (1-D bulk copy, issued
//      two tiles ahead by thread 0);
//   2. the 128 threads dequantise it into f16 operand tiles in shared memory
//      (128-byte swizzled, the canonical UMMA layouts): K as [token][dim]
//      (K-major B of S = Q K^T) and V transposed, [dim][token] (K-major B of
//      O = P V); K by thread = token, V by thread = 8 tokens x 16 dims;
//   3. thread 0 issues S = Q K^T (M = 128 rows, N = 128 tokens, 8 x K = 16) into
//      TMEM columns [0, 128) and commits to an mbarrier;
//   4. thread t reads its row of S from TMEM lane t (tcgen05.ld), masks tokens
//      past the body length, runs the online softmax in fp32 (base 2; the
//      running max moves only when a score beats it by more than 2^8, then the
//      thread rescales its own row of O in TMEM) and writes P (f16) as the
//      K-major A operand of the second product;
//   5. thread 0 issues O += P V (N = 128 dims) into TMEM columns [128, 256).
// Finally thread t reads its row of O, divides by the row sum and stores it.
// Every wait is bounded (HKV_WAIT_NS) and sets the device error word on expiry.
#pragma once
#include "hkv_common.cuh"

namespace hkv {

constexpr int kPfRows = 128;                   // query rows per CTA (the MMA's M)
constexpr int kPfTileBytes = 128 * 128 * 2;    // one f16 [128][128] operand tile (two 64-column atoms)
constexpr int kPfRawBytes = 24 * 1024;         // one raw page block (ref g32: 21,504 B)
constexpr int kPfSmem = 4 * kPfTileBytes + 2 * kPfRawBytes + 1024;  // Q | K | Vt | P | 2 raw | alignment
constexpr float kPfLazy = 8.0f;

struct PrefillParams {
  const void* q;      // [B][Hq][Sq][128] f16/bf16
  int q_dtype;
  int64_t q_sb, q_sh, q_ss;  // elements
  hkv_int4_store body;
  int B, Hq, Hkv, G, Sq;
  float qscale;       // sm_scale * log2(e)
  void* out;          // [B][Hq][Sq][128]
  int out_dtype;
  int64_t out_sb, out_sh, out_ss;
};

// Byte offset of the 16-byte chunk (8 columns) c of a row of a [128][128]
// 16-bit tile stored as two 64-column atoms of [128 rows][128 B], the chunks
// swizzled by row & 7 (the 128-byte swizzle of the UMMA canonical layouts).
__device__ __forceinline__ uint32_t pf_chunk(int row, int chunk16) {  // 16-byte chunk (8 columns)
  return (chunk16 >> 3) * (128 * 128) + row * 128 + (((chunk16 & 7) ^ (row & 7)) << 4);
}

// UMMA shared-memory descriptor: 128-byte swizzle, K-major (LBO 16 B, SBO 1024 B).
__device__ __forceinline__ uint64_t pf_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: f32 accumulate, f16 A and B, both K-major, M 128, N 128.
constexpr uint32_t kPfIdesc = (1u << 4) | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ void pf_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kPfIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void pf_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tm_ld32(uint32_t addr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tm_st32(uint32_t addr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Dequantises K of token t (thread t) of the raw block rb into sK ([token][dim]).
// Word 4j + w of a K token holds dims 32w + 8c + 16a + 2j + e at nibble 2a + c + 4e,
// so nib8_to_h2 of a word gives the dim pairs (2j, 2j+1) + 32w + {0, 8, 16, 24}.
template <int FMT, int GROUP>
__device__ __forceinline__ void pf_convert_k(const uint8_t* rb, uint8_t* sK, int t, bool valid) {
  constexpr int NG = HKV_D / GROUP;
  const uint32_t* kw = reinterpret_cast<const uint32_t*>(rb + t * HKV_CODE_BYTES);
  const uint8_t* meta = rb + HKV_META_OFF;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int g = (32 * w) / GROUP;
    __half2 s2, m2;
    uint32_t zlo = 0, zhi = 0;
    if constexpr (FMT == HKV_FMT_FP16MIN) {
      const __half s = reinterpret_cast<const __half*>(meta)[t * NG + g];
      const __half m = reinterpret_cast<const __half*>(meta + 256 * NG)[t * NG + g];
      s2 = __half2half2(s);
      m2 = __half2half2(m);
    } else {
      const float s = reinterpret_cast<const float*>(meta)[t * NG + g];
      const uint32_t z = meta[1024 * NG + t * NG + g];
      s2 = __float2half2_rn(s);
      m2 = __float2half2_rn(0.f);
      const uint32_t zl = h2u(__float2half2_rn(1024.f + (float)z)), zh = h2u(__float2half2_rn(-64.f - (float)z));
      zlo = zl;
      zhi = zh;
    }
    if (!valid) s2 = m2 = __float2half2_rn(0.f);
    uint32_t h[4][4];  // [j][nibble pair]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (FMT == HKV_FMT_FP16MIN) nib8_to_h2(kw[4 * j + w], h[j]);
      else nib8_to_h2_z(kw[4 * j + w], zlo, zhi, h[j]);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // dims 32w + 8c' .. + 7 with c' = {0: +0, 1: +8, 2: +16, 3: +24}
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = h2u(__hfma2(u2h(h[j][c]), s2, m2));
      const int d0 = 32 * w + 8 * c;
      *reinterpret_cast<uint4*>(sK + pf_chunk(t, d0 >> 3)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Dequantises V into sVt ([dim][token]): thread t handles tokens 8o .. 8o + 7
// (o = t % 16: pairs 4o .. 4o + 3), word k = t / 32 of the chunks i in
// [4 * ((t / 16) & 1), + 4). Word k of chunk i of a pair holds dims i + 32k + 8m
// (nibble m) of its two tokens (low / high half-word), so nib8_to_h2 of it gives
// the token pairs of dims i + 32k + {0, 8, 16, 24}. `valid` tokens hold data;
// the rest become zero (their P is zero and their bytes may be any bits).
template <int FMT, int GROUP>
__device__ __forceinline__ void pf_convert_v(const uint8_t* rb, uint8_t* sVt, int t, int valid) {
  constexpr int NG = HKV_D / GROUP;
  const int o = t & 15, k = t >> 5, i0 = 4 * ((t >> 4) & 1);
  const int g = (32 * k) / GROUP;
  const uint8_t* meta = rb + HKV_META_OFF;
  __half2 s2[4], m2[4];
  uint32_t zlo[4], zhi[4];
#pragma unroll
  for (int pp = 0; pp < 4; ++pp) {
    const int p = 4 * o + pp;  // pair: tokens 2p, 2p+1
    if constexpr (FMT == HKV_FMT_FP16MIN) {
      s2[pp] = reinterpret_cast<const __half2*>(meta + 512 * NG)[p * NG + g];
      m2[pp] = reinterpret_cast<const __half2*>(meta + 768 * NG)[p * NG + g];
      zlo[pp] = zhi[pp] = 0;
    } else {
      const float* vs = reinterpret_cast<const float*>(meta + 512 * NG);
      const uint8_t* vz = meta + 1152 * NG;
      const float za = (float)vz[(2 * p) * NG + g], zb = (float)vz[(2 * p + 1) * NG + g];
      s2[pp] = __floats2half2_rn(vs[(2 * p) * NG + g], vs[(2 * p + 1) * NG + g]);
      m2[pp] = __float2half2_rn(0.f);
      zlo[pp] = h2u(__floats2half2_rn(1024.f + za, 1024.f + zb));
      zhi[pp] = h2u(__floats2half2_rn(-64.f - za, -64.f - zb));
    }
    // zero the scale and offset of tokens at or past `valid`
    const uint32_t keep = (2 * p < valid ? 0x0000FFFFu : 0u) | (2 * p + 1 < valid ? 0xFFFF0000u : 0u);
    s2[pp] = u2h(h2u(s2[pp]) & keep);
    m2[pp] = u2h(h2u(m2[pp]) & keep);
  }
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    const int i = i0 + ii;
    uint32_t h[4][4];  // [pair][nibble m]
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const uint32_t wd = *reinterpret_cast<const uint32_t*>(rb + HKV_V_CODES_OFF + v_chunk_off(4 * o + pp, i) + 4 * k);
      if constexpr (FMT == HKV_FMT_FP16MIN) nib8_to_h2(wd, h[pp]);
      else nib8_to_h2_z(wd, zlo[pp], zhi[pp], h[pp]);
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int d = i + 32 * k + 8 * m;
      uint32_t out[4];
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) out[pp] = h2u(__hfma2(u2h(h[pp][m]), s2[pp], m2[pp]));
      *reinterpret_cast<uint4*>(sVt + pf_chunk(d, o)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
  }
}

template <int FMT, int GROUP>
__global__ void __launch_bounds__(128, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t pf_raw[];
  __shared__ __align__(8) uint64_t full_bar[2];
  __shared__ __align__(8) uint64_t s_bar, o_bar;
  __shared__ uint32_t s_tmem;
  uint8_t* sm = pf_raw + ((1024u - (smem_u32(pf_raw) & 1023u)) & 1023u);  // swizzle atoms need 1 KiB alignment
  uint8_t* sQ = sm;
  uint8_t* sK = sm + kPfTileBytes;
  uint8_t* sVt = sm + 2 * kPfTileBytes;
  uint8_t* sP = sm + 3 * kPfTileBytes;
  uint8_t* ring = sm + 4 * kPfTileBytes;
  const int t = threadIdx.x, warp = t >> 5;
  const int u = blockIdx.y, b = u / p.Hkv, hk = u - b * p.Hkv;
  const int row = blockIdx.x * kPfRows + t;  // this thread's query row
  const bool row_ok = row < p.Sq * p.G;
  const int qs = row_ok ? row / p.G : 0, qg = row_ok ? row % p.G : 0;
  constexpr uint32_t kBlock = block_bytes(FMT, GROUP);

  if (t == 0) {
    mbar_init(&full_bar[0], 1);
    mbar_init(&full_bar[1], 1);
    mbar_init(&s_bar, 1);
    mbar_init(&o_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(&s_tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  const int len = p.body.lengths ? p.body.lengths[b] : p.body.len;
  const int ntiles = (len + HKV_BLOCK_TOKENS - 1) / HKV_BLOCK_TOKENS;

  // query row -> Q tile (f16, K-major A operand); rows past the end stay zero
  {
    const int64_t base = (int64_t)b * p.q_sb + (int64_t)(hk * p.G + qg) * p.q_sh + (int64_t)qs * p.q_ss;
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = row_ok ? load_any(p.q, p.q_dtype, base + 8 * c + 2 * e) : 0.f;
        const float bb = row_ok ? load_any(p.q, p.q_dtype, base + 8 * c + 2 * e + 1) : 0.f;
        o[e] = h2u(__floats2half2_rn(a, bb));
      }
      *reinterpret_cast<uint4*>(sQ + pf_chunk(t, c)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem, tS = tmem, tO = tmem + 128;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  // raw block of tile k -> ring slot k & 1 (thread 0, which also counts its
  // copies and commits so that an abnormal exit can wait for them)
  int n_issued = 0, n_s = 0, n_o = 0;
  auto issue = [&](int k) {
    ++n_issued;
    const int tok = k * HKV_BLOCK_TOKENS;
    const int64_t page = store_page(p.body, u, tok);
    uint64_t* fb = &full_bar[k & 1];
    if (page < 0) {
      hkv_flag_error(HKV_DEVERR_BAD_PAGE);
      mbar_arrive(fb);
      return;
    }
    const uint8_t* src = static_cast<const uint8_t*>(p.body.pages) + page * p.body.page_stride +
                         (int64_t)((tok % p.body.page_tokens) / HKV_BLOCK_TOKENS) * kBlock;
    mbar_arrive_expect_tx(fb, kBlock);
    bulk_g2s(ring + (k & 1) * kPfRawBytes, src, kBlock, fb);
  };
  if (t == 0) {
    if (ntiles > 0) issue(0);
    if (ntiles > 1) issue(1);
  }

  float m_run = -1.0e30f, l_run = 0.f;
  bool alive = true;
  for (int k = 0; k < ntiles; ++k) {
    const int valid = min(HKV_BLOCK_TOKENS, len - k * HKV_BLOCK_TOKENS);
    // the previous tile's P V product must be done before K, Vt and P are rewritten
    if (k > 0 && !mbar_wait(&o_bar, (k - 1) & 1)) alive = false;
    if (!mbar_wait(&full_bar[k & 1], (k >> 1) & 1)) alive = false;
    if (!__syncthreads_and(alive)) break;
    const uint8_t* rb = ring + (k & 1) * kPfRawBytes;
    pf_convert_k<FMT, GROUP>(rb, sK, t, t < valid);
    pf_convert_v<FMT, GROUP>(rb, sVt, t, valid);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();  // operands written; the raw slot is free
    if (t == 0) {
      tc_fence_after();
      if (k + 2 < ntiles) issue(k + 2);
      const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
        pf_mma(tS, pf_desc(q0 + off), pf_desc(k0 + off), kk > 0);
      }
      pf_commit(&s_bar);
      ++n_s;
    }
    // softmax of this thread's row
    if (!mbar_wait(&s_bar, k & 1)) alive = false;
    tc_fence_after();
    float s[4][32];
#pragma unroll
    for (int c = 0; c < 4; ++c) tm_ld32(tS + lane_base + 32 * c, s[c]);
    float mx = -1.0e30f;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        s[c][i] = 32 * c + i < valid ? s[c][i] * p.qscale : -INFINITY;
        mx = fmaxf(mx, s[c][i]);
      }
    // The row max moves only when a score beats it by more than 2^8; then the
    // row's O is rescaled in TMEM (tcgen05.ld/st are warp-collective: the whole
    // warp takes part, with factor 1 for rows that keep their max).
    const bool move = mx > m_run + kPfLazy;
    if (__any_sync(0xffffffffu, move)) {
      const float nm = move ? mx : m_run;
      const float a = fast_exp2(m_run - nm);
      if (k > 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tm_ld32(tO + lane_base + 32 * c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= a;
          tm_st32(tO + lane_base + 32 * c, o);
        }
      }
      l_run *= a;
      m_run = nm;
    }
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x0 = s[c >> 2][8 * (c & 3) + 2 * e], x1 = s[c >> 2][8 * (c & 3) + 2 * e + 1];
        const __half2 pv = __floats2half2_rn(fast_exp2(x0 - m_run), fast_exp2(x1 - m_run));
        const float2 pf = __half22float2(pv);
        l_run += pf.x + pf.y;
        o[e] = h2u(pv);
      }
      *reinterpret_cast<uint4*>(sP + pf_chunk(t, c)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    if (t == 0) {
      tc_fence_after();
      const uint32_t p0 = smem_u32(sP), v0 = smem_u32(sVt);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
        pf_mma(tO, pf_desc(p0 + off), pf_desc(v0 + off), (k > 0 || kk > 0) ? 1u : 0u);
      }
      pf_commit(&o_bar);
      ++n_o;
    }
  }
  // every thread leaves the loop at the same tile; a wait that ran out anywhere
  // ends the CTA after thread 0 has waited (bounded) for its copies and products
  alive = __syncthreads_and(alive);
  if (!alive && t == 0) {
    for (int j = max(0, n_issued - 2); j < n_issued; ++j) mbar_wait(&full_bar[j & 1], (j >> 1) & 1);
    if (n_s > 0) mbar_wait(&s_bar, (n_s - 1) & 1);
    if (n_o > 0) mbar_wait(&o_bar, (n_o - 1) & 1);
  }
  // epilogue: O row / l
  if (alive && ntiles > 0 && !mbar_wait(&o_bar, (ntiles - 1) & 1)) alive = false;
  tc_fence_after();
  {
    // tcgen05.ld is warp-collective: every lane reads, lanes with a query row store
    const int64_t ob = (int64_t)b * p.out_sb + (int64_t)(hk * p.G + qg) * p.out_sh + (int64_t)qs * p.out_ss;
    const float inv = (alive && ntiles > 0 && l_run > 0.f) ? 1.f / l_run : 0.f;
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float o[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
      if (ntiles > 0) tm_ld32(tO + lane_base + c0, o);
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i) store_any(p.out, p.out_dtype, ob + c0 + i, o[i] * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

}  // namespace hkv
