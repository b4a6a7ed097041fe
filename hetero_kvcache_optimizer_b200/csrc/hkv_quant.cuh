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

// ------------------------------------------------------------------ quantise + pack
// Each half-warp quantises kQuantTokens consecutive tokens: their 16-byte loads
// are all issued before the first token is processed (latency overlap), 16
// lanes per token. grid.x covers ceil(B*H*T / (16 * kQuantTokens)) blocks of 256.
constexpr int kQuantTokens = 1;
template <typename T>
__global__ void __launch_bounds__(256) quantize_pack_kernel(const T* __restrict__ x, const T* __restrict__ x2,
                                                            int B, int H, int T_, int64_t sb, int64_t sh,
                                                            int64_t st, int role, hkv_int4_store store,
                                                            const int32_t* dst_start, int start) {
  // grid.y == 2: blockIdx.y 0 quantises x as side `role`, 1 quantises x2 as V
  const T* __restrict__ src = blockIdx.y ? x2 : x;
  if (blockIdx.y) role = HKV_ROLE_V;
  const int ntok = B * H * T_;  // < 2^31 (checked by the host)
  const int tok0 = (blockIdx.x * 16 + (threadIdx.x >> 4)) * kQuantTokens;
  const int p = threadIdx.x & 15;
  const int cap = store.max_pages * store.page_tokens;
  float v[kQuantTokens][8];
  int pos[kQuantTokens], unit[kQuantTokens];
#pragma unroll
  for (int i = 0; i < kQuantTokens; ++i) {
    const int tok = tok0 + i;
    const bool valid = tok < ntok;
    const int tt = valid ? tok : 0;
    const int u = tt / T_, t = tt - u * T_;
    const int b = u / H, h = u - b * H;
    unit[i] = valid ? u : -1;
    pos[i] = (dst_start ? dst_start[b] : start) + t;
    if (valid) {
      load8(src + b * sb + h * sh + (int64_t)t * st + 8 * p, v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
    }
  }
#pragma unroll
  for (int i = 0; i < kQuantTokens; ++i) {
    bool ok = unit[i] >= 0;
    int64_t page = 0;
    if (ok) {
      if (pos[i] < 0 || pos[i] >= cap) {
        if (p == 0) hkv_flag_error(HKV_DEVERR_CAPACITY);
        ok = false;
      } else {
        page = store_page(store, unit[i], pos[i]);
        if (page < 0) {
          if (p == 0) hkv_flag_error(HKV_DEVERR_BAD_PAGE);
          ok = false;
        }
      }
    }
    quantise_token(v[i], ok, role, store.format, store.group, store, page, ok ? pos[i] % store.page_tokens : 0);
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
