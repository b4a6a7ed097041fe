// INT4 quantise / nibble-pack / append / dequantise kernels. Included by hetero_kv.cu.
#pragma once
#include "hkv_common.cuh"

namespace hkv {

// ------------------------------------------------------------------ group arithmetic
// The reference quantiser (src/quantization/kv_compressor.py:76-88), IEEE fp32:
//   scale = max((max - min) / 15, 1e-8); zp = clamp(rint(-min / scale), 0, 15)
//   q = clamp(rint(x / scale + zp), 0, 15)
// Division is correctly rounded (the library is built without fast-math) and
// the add is not contracted into an fma, so codes match torch bit for bit.
// x / s correctly rounded, given r = RN(1/s): q0 = RN(x r); the remainder
// e = x - q0 s is exact with an fma; RN(q0 + e r) is the correctly rounded
// quotient (Markstein's correction step, IBM J. R&D 34(1), 1990; see Muller et
// al., Handbook of Floating-Point Arithmetic, ch. on division with an FMA).
// Holds away from underflow and overflow of the intermediates; the codes only
// depend on quotients near x.5, far from both. Three operations per element
// instead of a full division: the reciprocal is computed once per group.
__device__ __forceinline__ float div_by(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-q0, s, x);
  return __fmaf_rn(e, r, q0);
}

struct RefParams {
  float scale, zpf, rcp;
};
__device__ __forceinline__ RefParams ref_params(float mn, float mx) {
  RefParams p;
  p.scale = fmaxf((mx - mn) / 15.0f, 1e-8f);
  p.zpf = fminf(fmaxf(rintf(-mn / p.scale), 0.0f), 15.0f);
  p.rcp = __frcp_rn(p.scale);
  return p;
}
__device__ __forceinline__ uint32_t ref_code(float x, const RefParams& p) {
  const float t = __fadd_rn(div_by(x, p.scale, p.rcp), p.zpf);
  return static_cast<uint32_t>(fminf(fmaxf(rintf(t), 0.0f), 15.0f));
}

// fp16min format: scale_h = fp16(min((max-min)/15, 65504)), min_h = fp16(min),
// q = clamp(rint((x - min_h) / scale_h), 0, 15), or 0 when scale_h == 0.
struct MinParams {
  __half sh, mh;
  float sf, mf, rcp;
};
__device__ __forceinline__ MinParams min_params(float mn, float mx) {
  MinParams p;
  p.sh = __float2half_rn(fminf((mx - mn) / 15.0f, 65504.0f));
  p.mh = __float2half_rn(mn);
  p.sf = __half2float(p.sh);
  p.mf = __half2float(p.mh);
  p.rcp = p.sf > 0.0f ? __frcp_rn(p.sf) : 0.0f;
  return p;
}
__device__ __forceinline__ uint32_t min_code(float x, const MinParams& p) {
  if (!(p.sf > 0.0f)) return 0u;
  const float t = div_by(__fsub_rn(x, p.mf), p.sf, p.rcp);
  return static_cast<uint32_t>(fminf(fmaxf(rintf(t), 0.0f), 15.0f));
}

// ------------------------------------------------------------------ 16-lane token packer
// A token of 128 values is held by 16 consecutive lanes (a half-warp), lane p
// holding dims [8p, 8p+8) in v[0..7]. quantise_token() computes the group
// statistics with xor-shuffles inside the half-warp, quantises, and writes the
// packed codes + metadata of the token into the K or V half (role) of store
// slot (page, off).
// All 32 lanes of the warp must call it (the shuffles use the full mask);
// lanes with active == false only take part in the shuffles. With deq != null
// the lane also gets its 8 values back as the dequantiser computes them, in
// fp32: (q - zp) * scale (ref, KVCompressor.decompress) or q * scale + min
// (fp16min).
__device__ __forceinline__ void quantise_token(const float (&v)[8], bool active, int role, int fmt, int group,
                                               const hkv_int4_store& st, int64_t page, int off,
                                               float* deq = nullptr) {
  const int lane = threadIdx.x & 31;
  const int p = lane & 15;
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
  const int lanes_per_group = group / 8;  // 4, 8 or 16
  for (int s = 1; s < lanes_per_group; s <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, s));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
  }
  uint32_t packed = 0;  // 8 codes, code i in bits 4i..4i+3
  RefParams rp;
  MinParams mp;
  if (fmt == HKV_FMT_REF) {
    rp = ref_params(mn, mx);
#pragma unroll
    for (int i = 0; i < 8; ++i) packed |= ref_code(v[i], rp) << (4 * i);
  } else {
    mp = min_params(mn, mx);
#pragma unroll
    for (int i = 0; i < 8; ++i) packed |= min_code(v[i], mp) << (4 * i);
  }
  if (deq) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float c = static_cast<float>((packed >> (4 * i)) & 0xFu);
      deq[i] = fmt == HKV_FMT_REF ? __fmul_rn(__fsub_rn(c, rp.zpf), rp.scale) : __fadd_rn(__fmul_rn(c, mp.sf), mp.mf);
    }
  }
  // Gather: lane (4w + j) collects byte j of the four lanes of its 32-dim block w.
  const int w = p >> 2, j = p & 3;
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t vm = __shfl_sync(0xffffffffu, packed, 4 * w + m, 16);
    const uint32_t by = (vm >> (8 * j)) & 0xFFu;
    lo |= (by & 0xFu) << (4 * m);
    hi |= (by >> 4) << (4 * m);
  }
  if (!active) return;
  const BlockRef br = block_ref(st, page, off);
  if (role == HKV_ROLE_K) {
    reinterpret_cast<uint32_t*>(br.base + br.w * HKV_CODE_BYTES)[4 * j + w] = lo | (hi << 16);
  } else {
    // V token pairs: token parity selects the half-word of each word of the pair's chunks.
    uint8_t* vc = br.base + HKV_V_CODES_OFF;
    const int q = br.w >> 1, tau = br.w & 1;
    *reinterpret_cast<uint16_t*>(vc + v_chunk_off(q, 2 * j) + 4 * w + 2 * tau) = static_cast<uint16_t>(lo);
    *reinterpret_cast<uint16_t*>(vc + v_chunk_off(q, 2 * j + 1) + 4 * w + 2 * tau) = static_cast<uint16_t>(hi);
  }
  if ((p % lanes_per_group) == 0) {
    const int ng = HKV_D / group;
    const int gi = p / lanes_per_group;
    if (fmt == HKV_FMT_REF) {
      *reinterpret_cast<float*>(br.base + meta_off(role, ng) + 4 * (br.w * ng + gi)) = rp.scale;
      br.base[zps_off(role, ng) + br.w * ng + gi] = static_cast<uint8_t>(rp.zpf);
    } else {
      *reinterpret_cast<__half*>(br.base + mn_scale_off(role, br.w, ng, gi)) = mp.sh;
      *reinterpret_cast<__half*>(br.base + mn_min_off(role, br.w, ng, gi)) = mp.mh;
    }
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(src);
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = to_f32(e[i]);
}
template <typename T>
__device__ __forceinline__ void store8(T* dst, const float (&v)[8]) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4*>(dst) = raw;
}

// ------------------------------------------------------------------ quantise + pack (bulk)
// One thread = one token x one 32-dim block w (dims 32w..32w+31): it loads the
// block's 64 bytes, takes the group's min / max (a group of 64 or 128 dims
// spans 2 or 4 neighbouring lanes), quantises its 32 values and writes its
// block's four K code words (K side) or V words (V side) and the group's
// metadata. A CTA = 256 threads = 64 consecutive token POSITIONS of one unit
// and one side, the tile aligned to 64 positions: all its tokens lie in one
// 128-token page block, and the two tokens of a V pair (positions 2q, 2q+1) sit
// in lanes l and l ^ 4 of one warp, which swap their words with a shuffle and
// write whole 32-bit words. Compared with 16 lanes per token (quantise_token),
// the group parameters are computed once per 32 values instead of once per 8,
// no gather shuffles are needed, and the element arithmetic runs two lanes at a
// time in packed f32x2 operations with the same IEEE roundings.
constexpr int kQPTile = 64;
// 1.5 * 2^23: for 0 <= t <= 15, RN(t + 1.5 * 2^23) has rint(t) (ties to even,
// like rintf) in its low mantissa bits, i.e. bits = kMagicBits + rint(t).
constexpr float kMagicF = 12582912.0f;
constexpr uint32_t kMagicBits = 0x4B400000u;
// word_j accumulates bits(c) << shift for 8 codes; the magic parts sum to this
// constant (mod 2^32), removed once per word.
constexpr uint32_t kWordMagic = (kMagicBits << 0) + (kMagicBits << 4) + (kMagicBits << 8) + (kMagicBits << 12) +
                                (kMagicBits << 16) + (kMagicBits << 20) + (kMagicBits << 24) +
                                (kMagicBits << 28);

__device__ __forceinline__ float2 to_f32x2(const __half2 h) { return __half22float2(h); }
__device__ __forceinline__ float2 to_f32x2(const __nv_bfloat162 h) { return __bfloat1622float2(h); }

template <typename T> struct Vec2;
template <> struct Vec2<__half> { using type = __half2; };
template <> struct Vec2<__nv_bfloat16> { using type = __nv_bfloat162; };

template <typename T, int FMT, int GROUP>
__global__ void __launch_bounds__(256) quantize_pack_kernel(const T* __restrict__ x, const T* __restrict__ x2,
                                                            int H, int T_, int tiles, int64_t sb, int64_t sh,
                                                            int64_t st, int role, hkv_int4_store store,
                                                            const int32_t* __restrict__ dst_start, int start) {
  using T2 = typename Vec2<T>::type;
  constexpr int kLanesPerGroup = GROUP / 32;  // 1, 2 or 4
  constexpr int ng = HKV_D / GROUP;
  // Launched with programmatic stream serialization (when enabled): the next
  // launch on the stream may start its blocks as this one's drain, and this one
  // waits for the launch before it before touching global memory.
  griddep_launch_dependents();
  griddep_wait();
  // blockIdx.y 0: x as side `role`; 1: x2 as V
  const T* __restrict__ src = blockIdx.y ? x2 : x;
  if (blockIdx.y) role = HKV_ROLE_V;
  const int u = blockIdx.x / tiles, tile = blockIdx.x - u * tiles;
  const int b = u / H, h = u - b * H;
  const int s0 = dst_start ? dst_start[b] : start;
  const int lane = threadIdx.x & 31, w = threadIdx.x & 3;
  const int pos = (s0 & ~(kQPTile - 1)) + kQPTile * tile + (threadIdx.x >> 2);
  const int t = pos - s0;
  const bool valid = t >= 0 && t < T_;
  if (!__any_sync(0xffffffffu, valid)) return;  // warp-uniform: none of its 8 positions is in the chunk
  // the CTA's positions share one page block: one bounds check and lookup for all
  const int cap = store.max_pages * store.page_tokens;
  const int pos0 = (s0 & ~(kQPTile - 1)) + kQPTile * tile;
  int64_t page = -1;
  bool tile_ok = pos0 >= 0 && pos0 < cap;
  if (tile_ok) {
    page = store_page(store, u, pos0);
    tile_ok = page >= 0;
  }
  if (!tile_ok) {
    if (valid && w == 0) hkv_flag_error(pos0 >= 0 && pos0 < cap ? HKV_DEVERR_BAD_PAGE : HKV_DEVERR_CAPACITY);
    return;  // warp-uniform (tile_ok is uniform over the CTA)
  }

  // ---- load the block's 32 values (four 16-byte loads) and the group's range
  uint4 raw[4];
  if (valid) {
    const uint4* p = reinterpret_cast<const uint4*>(src + b * sb + h * sh + (int64_t)t * st + 32 * w);
#pragma unroll
    for (int i = 0; i < 4; ++i) raw[i] = p[i];
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) raw[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  const T2* v2 = reinterpret_cast<const T2*>(raw);  // 16 pairs: dims 32w + 2i, 32w + 2i + 1
  T2 lo2 = v2[0], hi2 = v2[0];
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    lo2 = __hmin2(lo2, v2[i]);
    hi2 = __hmax2(hi2, v2[i]);
  }
  const float2 lof = to_f32x2(lo2), hif = to_f32x2(hi2);
  float mn = fminf(lof.x, lof.y), mx = fmaxf(hif.x, hif.y);
#pragma unroll
  for (int sft = 1; sft < kLanesPerGroup; sft <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, sft));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, sft));
  }

  // ---- codes: t = x / s + zp (ref) or (x - min) / s (fp16min), the division
  // by Markstein's correction step (div_by), clamped to [0, 15], rounded by the
  // magic add; word j gets codes of dims 8m + 2j (low half) and 8m + 2j + 1
  // (high half), m = 0..3, at nibble m.
  float2 s2, r2, ns2, z2;
  RefParams rp;
  MinParams mp;
  bool zero_scale = false;
  if constexpr (FMT == HKV_FMT_REF) {
    rp = ref_params(mn, mx);
    s2 = make_float2(rp.scale, rp.scale);
    r2 = make_float2(rp.rcp, rp.rcp);
    z2 = make_float2(rp.zpf, rp.zpf);
  } else {
    mp = min_params(mn, mx);
    s2 = make_float2(mp.sf, mp.sf);
    r2 = make_float2(mp.rcp, mp.rcp);
    z2 = make_float2(-mp.mf, -mp.mf);
    zero_scale = !(mp.sf > 0.0f);
  }
  ns2 = make_float2(-s2.x, -s2.y);
  const float2 magic2 = make_float2(kMagicF, kMagicF);
  uint32_t word[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i) {  // pair i = dims 2i, 2i + 1 of the block: m = i / 4, j = i % 4
    float2 a = to_f32x2(v2[i]);
    float2 q;
    if constexpr (FMT == HKV_FMT_REF) {
      const float2 q0 = __fmul2_rn(a, r2);
      const float2 e = __ffma2_rn(q0, ns2, a);
      q = __fadd2_rn(__ffma2_rn(e, r2, q0), z2);
    } else {
      a = __fadd2_rn(a, z2);  // x - min, exact as in __fsub_rn
      const float2 q0 = __fmul2_rn(a, r2);
      const float2 e = __ffma2_rn(q0, ns2, a);
      q = __ffma2_rn(e, r2, q0);
    }
    q.x = fminf(fmaxf(q.x, 0.0f), 15.0f);
    q.y = fminf(fmaxf(q.y, 0.0f), 15.0f);
    const float2 rb = __fadd2_rn(q, magic2);
    const int m = i >> 2, j = i & 3;
    word[j] += (__float_as_uint(rb.x) << (4 * m)) + (__float_as_uint(rb.y) << (16 + 4 * m));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) word[j] = zero_scale ? 0u : word[j] - kWordMagic;

  // ---- stores
  const BlockRef br = block_ref(store, page, pos % store.page_tokens);
  const int gi = w / kLanesPerGroup;
  const bool meta_lane = (w % kLanesPerGroup) == 0;
  uint32_t partner[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) partner[j] = __shfl_xor_sync(0xffffffffu, word[j], 4);
  const bool partner_valid = __shfl_xor_sync(0xffffffffu, valid, 4);
  uint32_t meta16 = 0u, meta16_partner = 0u;  // fp16min V: scale | min << 16 of this token and its partner
  if constexpr (FMT == HKV_FMT_FP16MIN) {
    meta16 = static_cast<uint32_t>(__half_as_ushort(mp.sh)) | (static_cast<uint32_t>(__half_as_ushort(mp.mh)) << 16);
    meta16_partner = __shfl_xor_sync(0xffffffffu, meta16, 4);
  }
  if (!valid) return;
  if (role == HKV_ROLE_K) {
    uint32_t* kw = reinterpret_cast<uint32_t*>(br.base + br.w * HKV_CODE_BYTES);
#pragma unroll
    for (int j = 0; j < 4; ++j) kw[4 * j + w] = word[j];
  } else {
    uint8_t* vc = br.base + HKV_V_CODES_OFF;
    const int q = br.w >> 1, tau = br.w & 1;
    if (partner_valid) {
      // the even token writes the pair's words of chunks 2j (low halves of both
      // tokens), the odd token those of chunks 2j + 1 (high halves)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t v = tau ? __byte_perm(partner[j], word[j], 0x7632) : __byte_perm(word[j], partner[j], 0x5410);
        *reinterpret_cast<uint32_t*>(vc + v_chunk_off(q, 2 * j + tau) + 4 * w) = v;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        *reinterpret_cast<uint16_t*>(vc + v_chunk_off(q, 2 * j) + 4 * w + 2 * tau) = static_cast<uint16_t>(word[j]);
        *reinterpret_cast<uint16_t*>(vc + v_chunk_off(q, 2 * j + 1) + 4 * w + 2 * tau) =
            static_cast<uint16_t>(word[j] >> 16);
      }
    }
  }
  if (!meta_lane) return;
  if constexpr (FMT == HKV_FMT_REF) {
    *reinterpret_cast<float*>(br.base + meta_off(role, ng) + 4 * (br.w * ng + gi)) = rp.scale;
    br.base[zps_off(role, ng) + br.w * ng + gi] = static_cast<uint8_t>(rp.zpf);
  } else if (role == HKV_ROLE_K) {
    *reinterpret_cast<__half*>(br.base + mn_scale_off(0, br.w, ng, gi)) = mp.sh;
    *reinterpret_cast<__half*>(br.base + mn_min_off(0, br.w, ng, gi)) = mp.mh;
  } else if (partner_valid) {
    // the pair's two scales side by side (even token), the two mins (odd token)
    const int tau = br.w & 1, w0 = br.w & ~1;
    const uint32_t v = tau ? __byte_perm(meta16_partner, meta16, 0x7632) : __byte_perm(meta16, meta16_partner, 0x5410);
    *reinterpret_cast<uint32_t*>(br.base + (tau ? mn_min_off(1, w0, ng, gi) : mn_scale_off(1, w0, ng, gi))) = v;
  } else {
    *reinterpret_cast<__half*>(br.base + mn_scale_off(1, br.w, ng, gi)) = mp.sh;
    *reinterpret_cast<__half*>(br.base + mn_min_off(1, br.w, ng, gi)) = mp.mh;
  }
}

// ------------------------------------------------------------------ decode-step append
// One block per sequence b, one warp per KV head: lanes 0-15 handle K, 16-31 V.
template <typename T>
__global__ void __launch_bounds__(1024) append_kv_kernel(const T* __restrict__ k_new, const T* __restrict__ v_new,
                                                         int H, int64_t nsb, int64_t nsh, hkv_dense_kv dense,
                                                         int sink, int32_t* dense_len, int32_t* ring_head,
                                                         hkv_int4_store body, int32_t* body_len) {
  const int b = blockIdx.x;
  const int h = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int side = lane >> 4;  // 0 = K, 1 = V
  const int p = lane & 15;
  griddep_wait();  // all global accesses below
  const int dl = dense_len[b];
  const int head = ring_head[b];
  const int bl = body_len[b];
  const int cap = dense.capacity;
  const int cap_r = cap - sink;
  const bool fill = dl < cap;                // room left: no eviction
  const bool direct = !fill && cap_r <= 0;   // no ring at all: new token goes to the body
  const int row = fill ? dl : sink + head;
  T* seg = static_cast<T*>(side ? dense.v : dense.k);
  T* rowp = seg + b * dense.stride_b + h * dense.stride_h + (int64_t)row * dense.stride_t + 8 * p;
  const T* src = (side ? v_new : k_new) + b * nsb + h * nsh + 8 * p;
  float nv[8];
  load8(src, nv);
  if (!fill) {
    // quantise the evicted ring row (or the new token itself when there is no ring)
    float ev[8];
    if (direct) {
#pragma unroll
      for (int i = 0; i < 8; ++i) ev[i] = nv[i];
    } else {
      load8(rowp, ev);
    }
    const int capb = body.max_pages * body.page_tokens;
    bool ok = bl < capb;
    int64_t page = 0;
    if (!ok) {
      if (lane == 0) hkv_flag_error(HKV_DEVERR_CAPACITY);
    } else {
      page = store_page(body, b * H + h, bl);
      if (page < 0) {
        ok = false;
        if (lane == 0) hkv_flag_error(HKV_DEVERR_BAD_PAGE);
      }
    }
    quantise_token(ev, ok, side ? HKV_ROLE_V : HKV_ROLE_K, body.format, body.group, body, page,
                   bl % body.page_tokens);
  }
  if (!direct) store8(rowp, nv);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (fill) {
      dense_len[b] = dl + 1;
    } else {
      body_len[b] = bl + 1;
      if (!direct) ring_head[b] = (head + 1) % cap_r;
    }
  }
  griddep_launch_dependents();  // after this block's work: the next grid may start its prologue
}

// ------------------------------------------------------------------ legacy flat path
// One warp per group over the flattened tensor; the tail group is zero-padded
// exactly like kv_compressor.py:70-74.
template <typename T>
__global__ void __launch_bounds__(256) quantize_flat_kernel(const T* __restrict__ x, int64_t n, int group,
                                                            int64_t ngroups, uint8_t* __restrict__ codes,
                                                            float* __restrict__ scales, uint8_t* __restrict__ zps) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t g = warp; g < ngroups; g += nwarps) {
    const int64_t base = g * group;
    float mn = INFINITY, mx = -INFINITY;
    for (int i = lane; i < group; i += 32) {
      const int64_t idx = base + i;
      const float v = idx < n ? to_f32(x[idx]) : 0.0f;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, s));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    }
    const RefParams rp = ref_params(mn, mx);
    for (int i = lane; i < group; i += 32) {
      const int64_t idx = base + i;
      if (idx < n) codes[idx] = static_cast<uint8_t>(ref_code(to_f32(x[idx]), rp));
    }
    if (lane == 0) {
      scales[g] = rp.scale;
      zps[g] = static_cast<uint8_t>(rp.zpf);
    }
  }
}

template <typename OT>
__global__ void dequantize_flat_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                                       const uint8_t* __restrict__ zps, int64_t n, int group, OT* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = i / group;
    const float v = (static_cast<float>(codes[i]) - static_cast<float>(zps[g])) * scales[g];
    out[i] = from_f32<OT>(v);
  }
}

// ------------------------------------------------------------------ packed -> dense
// Code of (token br.w of block br, dim d) in the K or V half of the block.
__device__ __forceinline__ uint32_t packed_code(const BlockRef& br, int role, int d) {
  if (role == HKV_ROLE_K) {
    const int w = d >> 5, rem = d & 31;
    const int a = rem >> 4, c = (rem >> 3) & 1, j = (rem & 7) >> 1, e = rem & 1;
    const int k = 2 * a + c + 4 * e;
    const uint32_t word = reinterpret_cast<const uint32_t*>(br.base + br.w * HKV_CODE_BYTES)[4 * j + w];
    return (word >> (4 * k)) & 0xFu;
  }
  // word 4i + k of a V pair = word k of its chunk i
  const int i = d & 7, e = d >> 3, k = e >> 2, m = e & 3;
  const int q = br.w >> 1, tau = br.w & 1;
  const uint32_t word = *reinterpret_cast<const uint32_t*>(br.base + HKV_V_CODES_OFF + v_chunk_off(q, i) + 4 * k);
  return (word >> (4 * m + 16 * tau)) & 0xFu;
}

template <typename OT>
__global__ void dequantize_pack_kernel(hkv_int4_store st, int role, int H, int t0, int T_, int64_t ntok,
                                       OT* __restrict__ out) {
  const int64_t tok = (int64_t)blockIdx.x * 2 + (threadIdx.x >> 7);
  if (tok >= ntok) return;
  const int d = threadIdx.x & 127;
  const int t = t0 + (int)(tok % T_);
  const int u = (int)(tok / T_);
  const int64_t page = store_page(st, u, t);
  if (page < 0) {
    if (d == 0) hkv_flag_error(HKV_DEVERR_BAD_PAGE);
    return;
  }
  const BlockRef br = block_ref(st, page, t % st.page_tokens);
  const uint32_t c = packed_code(br, role, d);
  const int ng = HKV_D / st.group;
  const int gi = d / st.group;
  float v;
  if (st.format == HKV_FMT_REF) {
    const float zp = static_cast<float>(br.base[zps_off(role, ng) + br.w * ng + gi]);
    v = (static_cast<float>(c) - zp) * *reinterpret_cast<const float*>(br.base + meta_off(role, ng) + 4 * (br.w * ng + gi));
  } else {
    const float sc = __half2float(*reinterpret_cast<const __half*>(br.base + mn_scale_off(role, br.w, ng, gi)));
    const float mn = __half2float(*reinterpret_cast<const __half*>(br.base + mn_min_off(role, br.w, ng, gi)));
    v = static_cast<float>(c) * sc + mn;
  }
  out[tok * HKV_D + d] = from_f32<OT>(v);
}

// ------------------------------------------------------------------ legacy unpacked -> packed
// One thread per (token, 16-bit half of the packed token).
__global__ void repack_ref_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                                  const uint8_t* __restrict__ zps, int S, int group, int role,
                                  hkv_int4_store st, int64_t ntok) {
  const int64_t tok = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (tok >= ntok) return;
  const int hx = threadIdx.x & 31;
  const int t = (int)(tok % S);
  const int u = (int)(tok / S);
  const int64_t page = store_page(st, u, t);
  if (t >= st.max_pages * st.page_tokens || page < 0) {
    if (hx == 0) hkv_flag_error(HKV_DEVERR_BAD_PAGE);
    return;
  }
  const BlockRef br = block_ref(st, page, t % st.page_tokens);
  const uint8_t* src = codes + tok * HKV_D;
  uint32_t half = 0;
  if (role == HKV_ROLE_K) {
    const int wi = hx >> 1, part = hx & 1;
    const int j = wi >> 2, w = wi & 3;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int k = 4 * part + m;
      const int dim = 16 * (2 * w + (k % 4) / 2) + 8 * ((k % 4) % 2) + 2 * j + k / 4;
      half |= (uint32_t)(src[dim] & 0xF) << (4 * m);
    }
    reinterpret_cast<uint16_t*>(br.base + br.w * HKV_CODE_BYTES)[hx] = (uint16_t)half;
  } else {
    const int i = hx >> 2, k = hx & 3;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int e = 4 * k + m;
      const int dim = 16 * (e / 2) + 8 * (e % 2) + i;
      half |= (uint32_t)(src[dim] & 0xF) << (4 * m);
    }
    const int q = br.w >> 1, tau = br.w & 1;
    *reinterpret_cast<uint16_t*>(br.base + HKV_V_CODES_OFF + v_chunk_off(q, i) + 4 * k + 2 * tau) = (uint16_t)half;
  }
  const int ng = HKV_D / group;
  if (hx < ng) {
    const int64_t gidx = tok * ng + hx;
    *reinterpret_cast<float*>(br.base + meta_off(role, ng) + 4 * (br.w * ng + hx)) = scales[gidx];
    br.base[zps_off(role, ng) + br.w * ng + hx] = zps[gidx];
  }
}

}  // namespace hkv
