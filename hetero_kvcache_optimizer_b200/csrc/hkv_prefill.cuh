// Multi-query (prefill) attention over a packed INT4 body on the 5th-generation
// tensor cores (tcgen05). Included by hetero_kv.cu.
//
// One CTA per (sequence, KV head) unit and 128-row query tile; rows are
// (query position, head of the unit's G) pairs, row = s * G + g. Eight warps in
// two roles of 128 threads run a software pipeline over the body's 128-token tiles:
//   warps 4-7 (converters) copy raw page block j into ring slot j & 1 with
//     16-byte cp.async (two tiles ahead; completion on an mbarrier), dequantise
//     it into f16 operand tiles K[j & 1] ([token][dim], K-major B of S = Q K^T)
//     and Vt[j & 1] ([dim][token], K-major B of O = P V), 128-byte swizzled,
//     meet on a named barrier, and their first thread issues S(j) = Q K(j)^T
//     into TMEM buffer S[j & 1] (M = 128 rows, N = 128 tokens);
//   warps 0-3 (softmax; thread = query row = TMEM lane) read S(j), mask it, run
//     the online softmax in fp32 (base 2) and write P(j) as packed f16 over the
//     first 64 columns of S[j & 1]; after a named barrier their first thread
//     issues O += P(j) V(j) with P read from TMEM (the TS form). The running max
//     moves only when a score beats it by more than 2^8; only then does a warp
//     wait for O(j-1) and rescale its rows of O in TMEM, so softmax(j) normally
//     overlaps the O(j-1) product.
// S(j) is issued only after O(j-2) has completed (the converters wait for it
// before they overwrite K/Vt[j & 1]), which also frees S[j & 1].
// Then warps 0-3 read their rows of O, divide by the row sum, store them, and
// optionally the natural-log sum of exponentials per row. With a body split
// (gridDim.z > 1, to fill the SMs' waves) each CTA takes a contiguous share of
// the tiles and stores its un-normalised partial instead; prefill_merge_kernel
// combines the shares.
// Every wait is bounded (HKV_WAIT_NS) and sets the device error word on expiry;
// each role decides to stop together (barrier AND), and an aborted CTA waits
// (bounded) for its copies and products before it frees TMEM.
#pragma once
#include "hkv_common.cuh"

namespace hkv {

constexpr int kPfRows = 128;                   // query rows per CTA (the MMA's M)
constexpr int kPfTileBytes = 128 * 128 * 2;    // one f16 [128][128] operand tile (two 64-column atoms)
constexpr int kPfRawBytes = 24 * 1024;         // one raw page block (ref g32: 21,504 B)
constexpr int kPfThreads = 256;                // softmax warps 0-3 | converter warps 4-7
constexpr int kPfSmem = 5 * kPfTileBytes + 2 * kPfRawBytes + 1024;  // Q | K[2] | Vt[2] | raw[2] | alignment
constexpr float kPfLazy = 8.0f;

struct PrefillParams {
  const void* q;      // [B][Hq][Sq][128] f16/bf16
  int q_dtype;
  int64_t q_sb, q_sh, q_ss;  // elements
  hkv_int4_store body;
  int B, Hq, Hkv, G, Sq;
  int causal;         // query s sees body tokens t <= len - Sq + s
  float qscale;       // sm_scale * log2(e)
  void* out;          // [B][Hq][Sq][128]
  int out_dtype;
  int out_vec;        // out 16-byte aligned with strides in 16-byte units
  int q_vec;          // q 16-byte aligned with strides in 16-byte units (one vector load per 8 values)
  int64_t out_sb, out_sh, out_ss;
  float* lse;         // optional [B][Hq][Sq]: ln sum_t exp(sm_scale q.k_t)
  // split of the body over gridDim.z CTAs per query tile (nsplit > 1): each
  // writes an un-normalised partial, row r = (b Hq + hq) Sq + s, and
  // prefill_merge_kernel combines them
  int nsplit;
  float* part_o;      // [nsplit][rows][128]  sum_t 2^(x_t - m) v_t
  float* part_ml;     // [nsplit][rows][2]    (m, l), x = score * sm_scale * log2(e)
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
// O += P V with A (P, packed f16 pairs along K) read from TMEM columns [a_tmem, a_tmem + 8)
__device__ __forceinline__ void pf_mma_ts(uint32_t tmem, uint32_t a_tmem, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem),
      "r"(a_tmem), "l"(b), "r"(kPfIdesc), "r"(accumulate)
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
// 32 consecutive columns of this thread's lane, without waiting (tm_wait_ld after a batch).
__device__ __forceinline__ void tm_ld32_nw(uint32_t addr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tm_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tm_st32u(uint32_t addr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tm_st16u(uint32_t addr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
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

// Named barrier over `n` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool bar_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// arrive on `bar` once this thread's earlier cp.async copies have landed
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ __half2 u2h_(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// N consecutive f16 / f16x2 values from shared memory in one vector load
// (N * 2 resp. N * 4 bytes, naturally aligned in the page block's metadata).
template <int N>
__device__ __forceinline__ void vload_h(const uint8_t* p, __half (&v)[N]) {
  if constexpr (N == 4) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    const __half2 a = u2h_(r.x), b = u2h_(r.y);
    v[0] = __low2half(a), v[1] = __high2half(a), v[2] = __low2half(b), v[3] = __high2half(b);
  } else if constexpr (N == 2) {
    const __half2 a = u2h_(*reinterpret_cast<const uint32_t*>(p));
    v[0] = __low2half(a), v[1] = __high2half(a);
  } else {
    v[0] = *reinterpret_cast<const __half*>(p);
  }
}
template <int N>
__device__ __forceinline__ void vload_h2(const uint8_t* p, __half2 (&v)[N]) {
  if constexpr (N == 4) {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    v[0] = u2h_(r.x), v[1] = u2h_(r.y), v[2] = u2h_(r.z), v[3] = u2h_(r.w);
  } else if constexpr (N == 2) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    v[0] = u2h_(r.x), v[1] = u2h_(r.y);
  } else {
    v[0] = u2h_(*reinterpret_cast<const uint32_t*>(p));
  }
}

// Eight query values from element `base` of q as four f16 pairs (bf16 converted).
__device__ __forceinline__ void pf_load_q8(const PrefillParams& p, int64_t base, uint32_t (&o)[4]) {
  if (p.q_vec) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.q) + base));
    if (p.q_dtype == HKV_DT_F16) {
      o[0] = r.x, o[1] = r.y, o[2] = r.z, o[3] = r.w;
    } else {
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = h2u(__float22half2_rn(__bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]))));
    }
    return;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e)
    o[e] = h2u(__floats2half2_rn(load_any(p.q, p.q_dtype, base + 2 * e), load_any(p.q, p.q_dtype, base + 2 * e + 1)));
}

// Ring layout of a raw block: the page block as stored, except that the four
// 16-byte chunks of each K token are XOR-swizzled as they are copied in (chunk
// c of token t at t * 64 + 16 * (c ^ ((t >> 1) & 3))), so that the K
// converter's 16-byte reads (thread = token) hit 8 distinct bank groups per phase.
__device__ __forceinline__ uint32_t pf_ring_off(int gc) {  // ring offset of 16-byte chunk gc of a block
  if (gc < 512) {
    const int t = gc >> 2, c = gc & 3;
    return t * 64 + ((c ^ ((t >> 1) & 3)) << 4);
  }
  return gc * 16;
}

// Dequantises K of token t (thread t) of the ring block rb into sK ([token][dim]).
// Word 4j + w of a K token holds dims 32w + 8c + 16a + 2j + e at nibble 2a + c + 4e,
// so nib8_to_h2 of a word gives the dim pairs (2j, 2j+1) + 32w + {0, 8, 16, 24}.
template <int FMT, int GROUP>
__device__ __forceinline__ void pf_convert_k(const uint8_t* rb, uint8_t* sK, int t, bool valid) {
  constexpr int NG = HKV_D / GROUP;
  uint32_t kw[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 c = *reinterpret_cast<const uint4*>(rb + t * 64 + ((j ^ ((t >> 1) & 3)) << 4));
    kw[4 * j] = c.x;
    kw[4 * j + 1] = c.y;
    kw[4 * j + 2] = c.z;
    kw[4 * j + 3] = c.w;
  }
  const uint8_t* meta = rb + HKV_META_OFF;
  __half ks[NG], km[NG];  // fp16min: this token's scales and mins, one vector load each
  if constexpr (FMT == HKV_FMT_FP16MIN) vload_h<NG>(meta + 2 * NG * t, ks), vload_h<NG>(meta + 256 * NG + 2 * NG * t, km);
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int g = (32 * w) / GROUP;
    __half2 s2, m2;
    uint32_t zlo = 0, zhi = 0;
    if constexpr (FMT == HKV_FMT_FP16MIN) {
      s2 = __half2half2(ks[g]);
      m2 = __half2half2(km[g]);
    } else {
      const float s = reinterpret_cast<const float*>(meta)[t * NG + g];
      const uint32_t z = meta[1024 * NG + t * NG + g];
      s2 = __float2half2_rn(s);
      m2 = __float2half2_rn(0.f);
      zlo = h2u(__float2half2_rn(1024.f + (float)z));
      zhi = h2u(__float2half2_rn(-64.f - (float)z));
    }
    if (!valid) s2 = m2 = __float2half2_rn(0.f);
    uint32_t h[4][4];  // [j][nibble pair]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (FMT == HKV_FMT_FP16MIN) nib8_to_h2(kw[4 * j + w], h[j]);
      else nib8_to_h2_z(kw[4 * j + w], zlo, zhi, h[j]);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // dims 32w + 8c .. + 7
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = h2u(__hfma2(u2h(h[j][c]), s2, m2));
      const int d0 = 32 * w + 8 * c;
      *reinterpret_cast<uint4*>(sK + pf_chunk(t, d0 >> 3)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Dequantises V into sVt ([dim][token]): thread t handles tokens 8o .. 8o + 7
// (o = t / 8: pairs 4o .. 4o + 3) and chunk i = t % 8 of each pair, so the 8
// threads of a load phase read the 8 chunks of one pair (distinct bank groups)
// and share its metadata (broadcast). Word k of
// chunk i of a pair holds dims i + 32k + 8m (nibble m) of its two tokens (low /
// high half-word), so nib8_to_h2 of it gives the token pairs of dims
// i + 32k + {0, 8, 16, 24}. `valid` tokens hold data; the rest become zero
// (their P is zero and their bytes may be any bits).
template <int FMT, int GROUP>
__device__ __forceinline__ void pf_convert_v(const uint8_t* rb, uint8_t* sVt, int t, int valid) {
  constexpr int NG = HKV_D / GROUP;
  const int o = t >> 3, i = t & 7;
  const uint8_t* meta = rb + HKV_META_OFF;
  uint4 cw[4];
#pragma unroll
  for (int pp = 0; pp < 4; ++pp)
    cw[pp] = *reinterpret_cast<const uint4*>(rb + HKV_V_CODES_OFF + v_chunk_off(4 * o + pp, i));
  __half2 vs2[4][NG], vm2[4][NG];  // fp16min: each pair's NG scales and mins, one vector load each
  if constexpr (FMT == HKV_FMT_FP16MIN) {
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      vload_h2<NG>(meta + 512 * NG + 4 * NG * (4 * o + pp), vs2[pp]);
      vload_h2<NG>(meta + 768 * NG + 4 * NG * (4 * o + pp), vm2[pp]);
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int g = (32 * k) / GROUP;
    __half2 s2[4], m2[4];
    uint32_t zlo[4], zhi[4];
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const int p = 4 * o + pp;  // pair: tokens 2p, 2p+1
      if constexpr (FMT == HKV_FMT_FP16MIN) {
        s2[pp] = vs2[pp][g];
        m2[pp] = vm2[pp][g];
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
    uint32_t h[4][4];  // [pair][nibble m]
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const uint32_t wd = k == 0 ? cw[pp].x : k == 1 ? cw[pp].y : k == 2 ? cw[pp].z : cw[pp].w;
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

// One query row's result, read from this thread's lane of the O accumulator
// (tO_lane; `have`: O holds data, warp-uniform): the normalised output and lse,
// or with a body split the un-normalised partial (O, m, l) of this CTA's tiles.
__device__ __forceinline__ void pf_store_row(const PrefillParams& p, uint32_t tO_lane, bool have, bool row_ok,
                                             int b, int hk, int qg, int qs, float m_run, float l_run) {
  if (p.part_o) {  // split: the un-normalised partial of this CTA's tiles
    const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
    const int64_t row = ((int64_t)b * p.Hq + hk * p.G + qg) * p.Sq + qs;
    float4* po = reinterpret_cast<float4*>(p.part_o + ((int64_t)blockIdx.z * rows + row) * HKV_D);
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float o[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
      if (have) tm_ld32(tO_lane + c0, o);
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 8; ++i) po[c0 / 4 + i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
      }
    }
    if (row_ok)
      *reinterpret_cast<float2*>(p.part_ml + ((int64_t)blockIdx.z * rows + row) * 2) =
          have ? make_float2(m_run, l_run) : make_float2(-1.0e30f, 0.f);
  } else {
    const float inv = (have && l_run > 0.f) ? 1.f / l_run : 0.f;
    const int64_t ob = (int64_t)b * p.out_sb + (int64_t)(hk * p.G + qg) * p.out_sh + (int64_t)qs * p.out_ss;
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float o[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
      if (have) tm_ld32(tO_lane + c0, o);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] *= inv;
      if (!row_ok) continue;
      if (p.out_vec && p.out_dtype == HKV_DT_F32) {
        float4* d = reinterpret_cast<float4*>(static_cast<float*>(p.out) + ob + c0);
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
      } else if (p.out_vec && p.out_dtype == HKV_DT_F16) {
        uint4* d = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + ob + c0);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          d[i] = make_uint4(pack2<__half>(o[8 * i], o[8 * i + 1]), pack2<__half>(o[8 * i + 2], o[8 * i + 3]),
                            pack2<__half>(o[8 * i + 4], o[8 * i + 5]), pack2<__half>(o[8 * i + 6], o[8 * i + 7]));
      } else if (p.out_vec && p.out_dtype == HKV_DT_BF16) {
        uint4* d = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + ob + c0);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          d[i] = make_uint4(pack2<__nv_bfloat16>(o[8 * i], o[8 * i + 1]),
                            pack2<__nv_bfloat16>(o[8 * i + 2], o[8 * i + 3]),
                            pack2<__nv_bfloat16>(o[8 * i + 4], o[8 * i + 5]),
                            pack2<__nv_bfloat16>(o[8 * i + 6], o[8 * i + 7]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) store_any(p.out, p.out_dtype, ob + c0 + i, o[i]);
      }
    }
    if (p.lse && row_ok)
      p.lse[((int64_t)b * p.Hq + hk * p.G + qg) * p.Sq + qs] =
          (have && l_run > 0.f) ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
  }
}

template <int FMT, int GROUP>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t pf_raw[];
  __shared__ __align__(8) uint64_t raw_full[2], op_empty[2], s_full[2], vt_full[2], o_done[2], drain_bar[2];
  __shared__ uint32_t s_tmem;
  uint8_t* sm = pf_raw + ((1024u - (smem_u32(pf_raw) & 1023u)) & 1023u);  // swizzle atoms need 1 KiB alignment
  uint8_t* sQ = sm;
  uint8_t* sK = sm + kPfTileBytes;      // K[0], K[1]
  uint8_t* sV = sm + 3 * kPfTileBytes;  // Vt[0], Vt[1]
  uint8_t* ring = sm + 5 * kPfTileBytes;
  const int t = threadIdx.x, warp = t >> 5;
  const int u = blockIdx.y, b = u / p.Hkv, hk = u - b * p.Hkv;
  const int row0 = blockIdx.x * kPfRows, nrows = p.Sq * p.G;
  constexpr uint32_t kBlock = block_bytes(FMT, GROUP);

  const int len = max(0, p.body.lengths ? p.body.lengths[b] : p.body.len);
  // tokens the CTA's rows can see: all of the body, or up to the last row's causal limit
  int span = len;
  if (p.causal) span = min(len, len - p.Sq + 1 + (min(row0 + kPfRows, nrows) - 1) / p.G);
  // this CTA's share of the tiles: [t0, t0 + ntiles) of split blockIdx.z; loop
  // indices (ring slots, barrier phases) count from 0, token positions from t0
  const int tiles_all = span > 0 ? (span + HKV_BLOCK_TOKENS - 1) / HKV_BLOCK_TOKENS : 0;
  const int t0 = (int)(((int64_t)blockIdx.z * tiles_all) / p.nsplit);
  const int ntiles = (int)(((int64_t)(blockIdx.z + 1) * tiles_all) / p.nsplit) - t0;

  if (t == 0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&raw_full[i], 128);  // one cp.async arrival per converter thread
      mbar_init(&op_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&vt_full[i], 1);
      mbar_init(&o_done[i], 1);
      mbar_init(&drain_bar[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s_tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  // query rows -> Q tile (f16, K-major A operand), 16-byte chunk c of row i per
  // step so that neighbouring threads read neighbouring bytes; missing rows are zero
  for (int c = t; c < kPfRows * 16; c += kPfThreads) {
    const int i = c >> 4, ch = c & 15, r = row0 + i;
    uint32_t o[4] = {0u, 0u, 0u, 0u};
    if (r < nrows) {
      const int qs = r / p.G, qg = r - qs * p.G;
      const int64_t base =
          (int64_t)b * p.q_sb + (int64_t)(hk * p.G + qg) * p.q_sh + (int64_t)qs * p.q_ss + 8 * ch;
      pf_load_q8(p, base, o);
    }
    *reinterpret_cast<uint4*>(sQ + pf_chunk(i, ch)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem, tO = tmem + 256;

  if (warp >= 4) {
    // ------------- converters: raw block -> ring -> K[j & 1], Vt[j & 1]; issue S(j) -------------
    const int ct = t - 128;
    auto load = [&](int j) {  // this thread's 16-byte chunks of raw block t0 + j into slot j & 1
      const int tok = (t0 + j) * HKV_BLOCK_TOKENS;
      const int64_t page = store_page(p.body, u, tok);
      if (page >= 0) {
        const uint8_t* src = static_cast<const uint8_t*>(p.body.pages) + page * p.body.page_stride +
                             (int64_t)((tok % p.body.page_tokens) / HKV_BLOCK_TOKENS) * kBlock;
        uint8_t* dst = ring + (j & 1) * kPfRawBytes;
#pragma unroll
        for (int n = 0; n < (int)(kBlock / 16 + 127) / 128; ++n) {
          const int gc = ct + 128 * n;
          if (gc < (int)(kBlock / 16)) cp_async16(dst + pf_ring_off(gc), src + 16 * gc);
        }
      } else if (ct == 0) {
        hkv_flag_error(HKV_DEVERR_BAD_PAGE);
      }
      cp_async_arrive(&raw_full[j & 1]);
    };
    if (ntiles > 0) load(0);
    if (ntiles > 1) load(1);
    bool ok = true;
    int n_s = 0;
    for (int j = 0; j < ntiles; ++j) {
      ok = mbar_wait(&raw_full[j & 1], (j >> 1) & 1);
      if (j >= 2) ok = mbar_wait(&op_empty[j & 1], ((j >> 1) - 1) & 1) && ok;
      const int valid = min(HKV_BLOCK_TOKENS, len - (t0 + j) * HKV_BLOCK_TOKENS);
      const uint8_t* rb = ring + (j & 1) * kPfRawBytes;
      pf_convert_k<FMT, GROUP>(rb, sK + (j & 1) * kPfTileBytes, ct, ct < valid);
      pf_convert_v<FMT, GROUP>(rb, sV + (j & 1) * kPfTileBytes, ct, valid);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      ok = bar_and(2, 128, ok);  // operands written, slot j & 1 read, by all 128 converters
      if (!ok) break;
      if (ct == 0) {
        tc_fence_after();
        const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK + (j & 1) * kPfTileBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          pf_mma(tmem + 128 * (j & 1), pf_desc(q0 + off), pf_desc(k0 + off), kk > 0);
        }
        pf_commit(&s_full[j & 1]);
        mbar_arrive(&vt_full[j & 1]);  // Vt(j) is written: hand it to the thread that issues O(j)
        ++n_s;
      }
      if (j + 2 < ntiles) load(j + 2);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (!ok && ct == 0 && n_s > 0) {  // the products already issued finish before TMEM is freed
      pf_commit(&drain_bar[1]);
      mbar_wait(&drain_bar[1], 0);
    }
  } else {
    // ---------------- softmax: thread = query row = TMEM lane; issue O(j) ----------------
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const int r = row0 + t;
    const bool row_ok = r < nrows;
    const int qs = row_ok ? r / p.G : 0, qg = row_ok ? r - qs * p.G : 0;
    const int lim_row = p.causal ? min(len, len - p.Sq + 1 + qs) : len;  // tokens this row sees
    const float qscale = p.qscale;
    float m_run = -1.0e30f, l_run = 0.f;
    bool ok = true;
    int n_o = 0;
    for (int j = 0; j < ntiles; ++j) {
      ok = mbar_wait(&s_full[j & 1], (j >> 1) & 1) && ok;
      tc_fence_after();
      const uint32_t ts = tmem + 128 * (j & 1) + lane_base;
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tm_ld32_nw(ts + 32 * c, s + 32 * c);
      tm_wait_ld();
      const int lim = lim_row - (t0 + j) * HKV_BLOCK_TOKENS;
      if (lim < HKV_BLOCK_TOKENS) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= lim) s[i] = -INFINITY;
      }
      // row max: four independent chains of three-input max, two scores per step
      float mx4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int i = 4; i < 128; i += 2) mx4[(i >> 1) & 3] = fmax3(mx4[(i >> 1) & 3], s[i], s[i + 1]);
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * qscale;
      // the running max moves only when a score beats it by more than 2^8; the
      // warp then waits for O(j-1) and rescales its rows (ld/st are warp-collective)
      const bool move = mx > m_run + kPfLazy;
      if (__any_sync(0xffffffffu, move)) {
        const float nm = move ? mx : m_run;
        const float a = fast_exp2(m_run - nm);
        if (j > 0) {
          ok = mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1) && ok;
          tc_fence_after();
#pragma unroll 1
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
      // x = s * qscale - m two lanes at a time (packed f32x2 FMA / add)
      const float2 qs2 = make_float2(qscale, qscale), nm2 = make_float2(-m_run, -m_run);
      float2 lsum = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float2 x = __ffma2_rn(make_float2(s[32 * c + 2 * i], s[32 * c + 2 * i + 1]), qs2, nm2);
          x.x = fast_exp2(x.x);
          x.y = fast_exp2(x.y);
          lsum = __fadd2_rn(lsum, x);
          pk[i] = h2u(__floats2half2_rn(x.x, x.y));
        }
        tm_st16u(ts + 16 * c, pk);
      }
      l_run += lsum.x + lsum.y;
      tm_wait_st();
      tc_fence_before();
      ok = bar_and(1, 128, ok);  // P(j) (and any rescale of O) written by all 128 rows
      if (!ok) break;
      if (t == 0) {
        // a failed wait skips the product; the next barrier (or the one below) stops the role
        ok = mbar_wait(&vt_full[j & 1], (j >> 1) & 1);
        if (ok) {
          tc_fence_after();
          const uint32_t v0 = smem_u32(sV + (j & 1) * kPfTileBytes), pa = tmem + 128 * (j & 1);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            pf_mma_ts(tO, pa + 8 * kk, pf_desc(v0 + off), (j > 0 || kk > 0) ? 1u : 0u);
          }
          pf_commit(&op_empty[j & 1]);
          pf_commit(&o_done[j & 1]);
          ++n_o;
        }
      }
    }
    ok = bar_and(1, 128, ok);
    if (!ok && t == 0 && n_o > 0) {  // the products already issued finish before TMEM is freed
      pf_commit(&drain_bar[0]);
      mbar_wait(&drain_bar[0], 0);
    }
    // epilogue: O row / l
    bool have = ok && ntiles > 0;
    if (have) {
      const bool w = mbar_wait(&o_done[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1);
      have = __all_sync(0xffffffffu, w);
      tc_fence_after();
    }
    pf_store_row(p, tO + lane_base, have, row_ok, b, hk, qg, qs, m_run, l_run);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// ----------------------------------------------------------------------------
// Two query tiles per CTA, each with its own softmax warps (prefill2_kernel):
// rows [row0, row0 + 128) are tile A (softmax warps 0-3), [row0 + 128, row0 + 256)
// tile B (warps 4-7); both read the same dequantised K and V tiles (converter
// warps 8-11), so the dequantisation is paid once per 256 rows while the two
// softmax groups run side by side. TMEM: S_A, S_B, O_A, O_B (128 columns each).
// One raw slot, whose K half and V half are refilled as soon as each half has
// been converted. Per body tile j: the converters' first thread issues S_X(j)
// once O_X(j-1) has completed (P_X(j-1) lives in S_X's columns); group X's first
// thread issues O_X(j) after its softmax. S_X(j) lands only after O_X(j-1) has
// completed, so a rescale of O_X needs no wait. Twelve warps leave 168 registers
// a thread, so the softmax reads S twice (row max, then P).

// Global 16-byte chunk that chunk `idx` of side `role`'s share of a page block
// is: the side's 512 code chunks, then its metadata (fp16min: scales + mins,
// 32·NG chunks; ref: fp32 scales 32·NG chunks + zero points 8·NG chunks).
template <int FMT, int GROUP>
__device__ __forceinline__ int pf_side_chunk(int role, int idx) {
  constexpr int NG = HKV_D / GROUP;
  if (idx < 512) return role * 512 + idx;
  const int m = idx - 512;
  if (FMT == HKV_FMT_FP16MIN || m < 32 * NG) return 1024 + role * 32 * NG + m;
  return 1024 + 64 * NG + role * 8 * NG + (m - 32 * NG);
}
template <int FMT, int GROUP>
constexpr int pf_side_chunks() {
  return 512 + (FMT == HKV_FMT_FP16MIN ? 32 : 40) * (HKV_D / GROUP);
}

constexpr int kPf2Rows = 2 * kPfRows;
constexpr int kPf2Threads = 384;  // softmax A warps 0-3 | softmax B warps 4-7 | converters 8-11
constexpr int kPf2Smem = 6 * kPfTileBytes + kPfRawBytes + 1024;  // Q_A | Q_B | K[2] | Vt[2] | raw | alignment

template <int FMT, int GROUP>
__global__ void __launch_bounds__(kPf2Threads, 1) prefill2_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t pf_raw[];
  // raw_full[side]: the side's half of tile j landed (one phase per tile)
  // k_full / vt_full[j & 1]: K(j) / Vt(j) written; kfree / vfree[j & 1]: the
  // products reading K[j & 1] / Vt[j & 1] have completed; s_full[X]: S_X(j)
  // done; o_done[X]: O_X(j) done
  __shared__ __align__(8) uint64_t raw_full[2], kfree[2], vfree[2], vt_full[2], s_full[2], o_done[2], drain_bar[3];
  __shared__ uint32_t s_tmem;
  uint8_t* sm = pf_raw + ((1024u - (smem_u32(pf_raw) & 1023u)) & 1023u);  // swizzle atoms need 1 KiB alignment
  uint8_t* sQ = sm;                     // Q_A, Q_B
  uint8_t* sK = sm + 2 * kPfTileBytes;  // K[0], K[1]
  uint8_t* sV = sm + 4 * kPfTileBytes;  // Vt[0], Vt[1]
  uint8_t* raw = sm + 6 * kPfTileBytes;
  const int t = threadIdx.x, warp = t >> 5;
  const int u = blockIdx.y, b = u / p.Hkv, hk = u - b * p.Hkv;
  const int row0 = blockIdx.x * kPf2Rows, nrows = p.Sq * p.G;
  constexpr uint32_t kBlock = block_bytes(FMT, GROUP);
  static_assert(16 * (2 * pf_side_chunks<FMT, GROUP>()) == (int)kBlock, "the two sides cover the block");

  const int len = max(0, p.body.lengths ? p.body.lengths[b] : p.body.len);
  int span = len;
  if (p.causal) span = min(len, len - p.Sq + 1 + (min(row0 + kPf2Rows, nrows) - 1) / p.G);
  const int tiles_all = span > 0 ? (span + HKV_BLOCK_TOKENS - 1) / HKV_BLOCK_TOKENS : 0;
  const int t0 = (int)(((int64_t)blockIdx.z * tiles_all) / p.nsplit);
  const int ntiles = (int)(((int64_t)(blockIdx.z + 1) * tiles_all) / p.nsplit) - t0;

  if (t == 0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&raw_full[i], 128);  // one cp.async arrival per converter thread
      mbar_init(&kfree[i], 1);
      mbar_init(&vfree[i], 2);  // one commit from each softmax group's O issuer
      mbar_init(&vt_full[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&o_done[i], 1);
      mbar_init(&drain_bar[i], 1);
    }
    mbar_init(&drain_bar[2], 1);  // drain barriers: 0 softmax A, 1 converters, 2 softmax B
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s_tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  for (int c = t; c < kPf2Rows * 16; c += kPf2Threads) {
    const int i = c >> 4, ch = c & 15, r = row0 + i;
    uint32_t o[4] = {0u, 0u, 0u, 0u};
    if (r < nrows) {
      const int qs = r / p.G, qg = r - qs * p.G;
      const int64_t base =
          (int64_t)b * p.q_sb + (int64_t)(hk * p.G + qg) * p.q_sh + (int64_t)qs * p.q_ss + 8 * ch;
      pf_load_q8(p, base, o);
    }
    *reinterpret_cast<uint4*>(sQ + (i >> 7) * kPfTileBytes + pf_chunk(i & 127, ch)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;  // S_A 0, S_B 128, O_A 256, O_B 384

  if (warp >= 8) {
    // ---------------- converters; their first thread issues S_A(j) and S_B(j) ----------------
    const int ct = t - 256;
    auto load = [&](int j, int role) {  // this thread's chunks of side `role` of raw block t0 + j
      const int tok = (t0 + j) * HKV_BLOCK_TOKENS;
      const int64_t page = store_page(p.body, u, tok);
      if (page >= 0) {
        const uint8_t* src = static_cast<const uint8_t*>(p.body.pages) + page * p.body.page_stride +
                             (int64_t)((tok % p.body.page_tokens) / HKV_BLOCK_TOKENS) * kBlock;
#pragma unroll
        for (int n = 0; n < (pf_side_chunks<FMT, GROUP>() + 127) / 128; ++n) {
          const int idx = ct + 128 * n;
          if (idx < pf_side_chunks<FMT, GROUP>()) {
            const int gc = pf_side_chunk<FMT, GROUP>(role, idx);
            cp_async16(raw + pf_ring_off(gc), src + 16 * gc);
          }
        }
      } else if (ct == 0 && role == 0) {
        hkv_flag_error(HKV_DEVERR_BAD_PAGE);
      }
      cp_async_arrive(&raw_full[role]);
    };
    if (ntiles > 0) {
      load(0, 0);
      load(0, 1);
    }
    bool ok = true;
    int n_s = 0;
    const uint32_t q0 = smem_u32(sQ);
    for (int j = 0; j < ntiles; ++j) {
      const int valid = min(HKV_BLOCK_TOKENS, len - (t0 + j) * HKV_BLOCK_TOKENS);
      // K(j)
      ok = mbar_wait(&raw_full[0], j & 1) && ok;
      if (j >= 2) ok = mbar_wait(&kfree[j & 1], ((j >> 1) - 1) & 1) && ok;
      pf_convert_k<FMT, GROUP>(raw, sK + (j & 1) * kPfTileBytes, ct, ct < valid);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      ok = bar_and(2, 128, ok);
      if (!ok) break;
      if (j + 1 < ntiles) load(j + 1, 0);  // the raw K half is read: fetch the next one
      if (ct == 0) {
        const uint32_t k0 = smem_u32(sK + (j & 1) * kPfTileBytes);
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (j > 0) ok = mbar_wait(&o_done[x], (j - 1) & 1) && ok;  // O_X(j-1) read P_X(j-1) from S_X
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            pf_mma(tmem + 128 * x, pf_desc(q0 + x * kPfTileBytes + off), pf_desc(k0 + off), kk > 0);
          }
          pf_commit(&s_full[x]);
        }
        pf_commit(&kfree[j & 1]);
        ++n_s;
      }
      // V(j)
      ok = mbar_wait(&raw_full[1], j & 1) && ok;
      if (j >= 2) ok = mbar_wait(&vfree[j & 1], ((j >> 1) - 1) & 1) && ok;
      pf_convert_v<FMT, GROUP>(raw, sV + (j & 1) * kPfTileBytes, ct, valid);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      ok = bar_and(2, 128, ok);
      if (!ok) break;
      if (j + 1 < ntiles) load(j + 1, 1);
      if (ct == 0) mbar_arrive(&vt_full[j & 1]);  // Vt(j) is written: hand it to the O issuer
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (!ok && ct == 0 && n_s > 0) {  // the products already issued finish before TMEM is freed
      pf_commit(&drain_bar[1]);
      mbar_wait(&drain_bar[1], 0);
    }
  } else {
    // ---------------- softmax group x (warps 4x .. 4x + 3): thread = row of tile x; issue O_x(j) ----------------
    const int x = warp >> 2, st = t - 128 * x;  // group, thread in group
    const int bar_id = 1 + 2 * x;              // named barriers 1 (A) and 3 (B); 2 is the converters'
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t ts = tmem + 128 * x + lane_base, to = tmem + 256 + 128 * x + lane_base;
    const int r = row0 + 128 * x + st;
    const bool row_ok = r < nrows;
    const int qs = row_ok ? r / p.G : 0, qg = row_ok ? r - qs * p.G : 0;
    const int lim_row = p.causal ? min(len, len - p.Sq + 1 + qs) : len;  // tokens this row sees
    const float qscale = p.qscale;
    float m_run = -1.0e30f, l_run = 0.f;
    bool ok = true;
    int n_o = 0;
    for (int j = 0; j < ntiles; ++j) {
      ok = mbar_wait(&s_full[x], j & 1) && ok;
      tc_fence_after();
      const int lim = lim_row - (t0 + j) * HKV_BLOCK_TOKENS;  // columns at or past lim are masked
      // pass 1: the row max, 64 columns at a time
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float a[64];
        tm_ld32_nw(ts + 64 * h, a);
        tm_ld32_nw(ts + 64 * h + 32, a + 32);
        tm_wait_ld();
        if (lim < 64 * (h + 1)) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (64 * h + i >= lim) a[i] = -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < 64; i += 2) mx4[(i >> 1) & 3] = fmax3(mx4[(i >> 1) & 3], a[i], a[i + 1]);
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * qscale;
      // lazy max: rescale this row's O only when a score beats the max by 2^8
      // (O_x(j-1) has completed: S_x(j) was issued after it)
      const bool move = mx > m_run + kPfLazy;
      if (__any_sync(0xffffffffu, move)) {
        const float nm = move ? mx : m_run;
        const float a = fast_exp2(m_run - nm);
        if (j > 0) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tm_ld32(to + 32 * c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= a;
            tm_st32(to + 32 * c, o);
          }
        }
        l_run *= a;
        m_run = nm;
      }
      // pass 2: P = 2^(s * qscale - m) as f16 pairs over the first 64 columns,
      // 32 columns at a time (chunk c's P lands on columns already read)
      const float2 qs2 = make_float2(qscale, qscale), nm2 = make_float2(-m_run, -m_run);
      float2 lsum = make_float2(0.f, 0.f);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float a[32];
        tm_ld32_nw(ts + 32 * c, a);
        tm_wait_ld();
        if (lim < 32 * (c + 1)) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (32 * c + i >= lim) a[i] = -INFINITY;
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float2 xx = __ffma2_rn(make_float2(a[2 * i], a[2 * i + 1]), qs2, nm2);
          xx.x = fast_exp2(xx.x);
          xx.y = fast_exp2(xx.y);
          lsum = __fadd2_rn(lsum, xx);
          pk[i] = h2u(__floats2half2_rn(xx.x, xx.y));
        }
        tm_st16u(ts + 16 * c, pk);
      }
      l_run += lsum.x + lsum.y;
      tm_wait_st();
      tc_fence_before();
      ok = bar_and(bar_id, 128, ok);  // P_x(j) (and any rescale of O_x) written by the group's 128 rows
      if (!ok) break;
      if (st == 0) {
        // a failed wait skips the product; the next barrier (or the one below) stops the group
        ok = mbar_wait(&vt_full[j & 1], (j >> 1) & 1);
        if (ok) {
          tc_fence_after();
          const uint32_t v0 = smem_u32(sV + (j & 1) * kPfTileBytes), pa = tmem + 128 * x;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            pf_mma_ts(tmem + 256 + 128 * x, pa + 8 * kk, pf_desc(v0 + off), (j > 0 || kk > 0) ? 1u : 0u);
          }
          pf_commit(&o_done[x]);
          pf_commit(&vfree[j & 1]);
          ++n_o;
        }
      }
    }
    ok = bar_and(bar_id, 128, ok);
    if (!ok && st == 0 && n_o > 0) {  // the products already issued finish before TMEM is freed
      pf_commit(&drain_bar[2 * x]);
      mbar_wait(&drain_bar[2 * x], 0);
    }
    bool have = ok && ntiles > 0;
    if (have) {
      const bool w = mbar_wait(&o_done[x], (ntiles - 1) & 1);
      have = __all_sync(0xffffffffu, w);
      tc_fence_after();
    }
    pf_store_row(p, to, have, row_ok, b, hk, qg, qs, m_run, l_run);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// Combines the nsplit partials of each prefill row (one warp per row, lane =
// dims 4 lane .. 4 lane + 3): O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
__global__ void __launch_bounds__(256) prefill_merge_kernel(const __grid_constant__ PrefillParams p) {
  const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -1.0e30f;
  for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, p.part_ml[((int64_t)s * rows + row) * 2]);
  float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < p.nsplit; ++s) {
    const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + ((int64_t)s * rows + row) * 2);
    const float w = ml.y > 0.f ? fast_exp2(ml.x - M) : 0.f;
    L += w * ml.y;
    const float4 o = *reinterpret_cast<const float4*>(p.part_o + ((int64_t)s * rows + row) * HKV_D + 4 * lane);
    acc[0] += w * o.x;
    acc[1] += w * o.y;
    acc[2] += w * o.z;
    acc[3] += w * o.w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int64_t hs = (int64_t)p.Hq * p.Sq;
  const int b = (int)(row / hs), hq = (int)((row - (int64_t)b * hs) / p.Sq), qs = (int)(row % p.Sq);
  const int64_t ob = (int64_t)b * p.out_sb + (int64_t)hq * p.out_sh + (int64_t)qs * p.out_ss + 4 * lane;
#pragma unroll
  for (int i = 0; i < 4; ++i) store_any(p.out, p.out_dtype, ob + i, acc[i] * inv);
  if (p.lse && lane == 0) p.lse[row] = L > 0.f ? (M + __log2f(L)) * 0.69314718055994531f : -INFINITY;
}

}  // namespace hkv
