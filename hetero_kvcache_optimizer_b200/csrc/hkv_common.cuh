// Shared device helpers for libhetero_kv (sm_100a). Included once, by hetero_kv.cu.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hetero_kv.h"

#define HKV_D 128              // head dim of the packed format
#define HKV_CODE_BYTES 64      // packed bytes per token per side
#define HKV_WAIT_NS 2000000000ull  // bounded device waits give up after 2 s

// Sticky device error word (HKV_DEVERR_* bits); read by hkv_device_error().
__device__ unsigned int g_hkv_dev_error;

__device__ __forceinline__ void hkv_flag_error(unsigned int bits) { atomicOr(&g_hkv_dev_error, bits); }

// ------------------------------------------------------------------ dtype helpers
template <typename T> struct DT;
template <> struct DT<__half> { static constexpr int id = HKV_DT_F16; };
template <> struct DT<__nv_bfloat16> { static constexpr int id = HKV_DT_BF16; };

__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(float x) { return x; }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  if (dtype == HKV_DT_F16) return __half2float(static_cast<const __half*>(p)[i]);
  if (dtype == HKV_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_any(void* p, int dtype, int64_t i, float v) {
  if (dtype == HKV_DT_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dtype == HKV_DT_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<float*>(p)[i] = v;
}

// pack two floats into a b16x2 register of type T (low half = a)
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// As mbar_try_wait, but a thread whose phase is not complete may sleep up to
// `ns` nanoseconds (woken early when the phase completes) instead of returning
// after the hardware's default limit: fewer spin iterations for long waits.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Programmatic dependent launch (kernels launched with the programmatic stream
// serialization attribute): griddep_wait blocks until the preceding grid has
// completed and its memory operations are visible, so it goes before the first
// global access; griddep_launch_dependents lets the next grid in the stream
// start its own prologue early (that grid then waits for this one the same way).
// Both are no-ops for a normal launch.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait on an mbarrier phase. Returns false (and flags the device error
// word) if the phase has not completed within limit_ns. With sleep_ns > 0 a
// pending try_wait may sleep that long (woken by the phase completion).
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, uint32_t sleep_ns,
                                                uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (sleep_ns ? mbar_try_wait_sleep(bar, parity, sleep_ns) : mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      hkv_flag_error(HKV_DEVERR_TIMEOUT);
      return false;
    }
  }
}
// The kernels' bounded wait: gives up after HKV_WAIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t sleep_ns = 0) {
  return mbar_wait_limit(bar, parity, sleep_ns, HKV_WAIT_NS);
}

// 1-D bulk async copy global -> this CTA's shared memory, completion counted on bar.
// src, dst 16-byte aligned; bytes a multiple of 16. Into this CTA alone.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <uint32_t LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return d;
}

// 8 nibbles of x -> 4 f16x2 holding the exact integers:
//   h[0] = (n0, n4), h[1] = (n1, n5), h[2] = (n2, n6), h[3] = (n3, n7)
// Magic-number conversion (Kim et al., "Who Says Elephants Can't Run", 2022):
// OR-ing a nibble into the mantissa of 1024.0h gives 1024 + n (or 1024 + 16 n
// for the upper nibble of a byte); one f16x2 subtract / fma removes the bias.
__device__ __forceinline__ void nib8_to_h2(uint32_t x, uint32_t (&h)[4]) {
  constexpr uint32_t kMagic = 0x64006400u;  // (1024, 1024)
  constexpr uint32_t kInv16 = 0x2C002C00u;  // (1/16, 1/16)
  constexpr uint32_t kM64 = 0xD400D400u;    // (-64, -64)
  const uint32_t e0 = lop3<0xEA>(x, 0x000F000Fu, kMagic);
  const uint32_t e1 = lop3<0xEA>(x, 0x00F000F0u, kMagic);
  const uint32_t x8 = x >> 8;
  const uint32_t e2 = lop3<0xEA>(x8, 0x000F000Fu, kMagic);
  const uint32_t e3 = lop3<0xEA>(x8, 0x00F000F0u, kMagic);
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[0]) : "r"(e0), "r"(kMagic));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[1]) : "r"(e1), "r"(kInv16), "r"(kM64));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[2]) : "r"(e2), "r"(kMagic));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[3]) : "r"(e3), "r"(kInv16), "r"(kM64));
}

// D = A(16x16, row) * B(16x8, col) + D, fp32 accumulate. Register-only, so not
// volatile: the compiler may interleave independent MMAs with other work.
template <typename T> __device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D = A * B + C with separate C (used to seed an accumulator with a bias).
__device__ __forceinline__ void mma16816_c(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                           const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

// Integer-only nibble -> f16 extraction (no f16 arithmetic):
//   biased16(x)  : nibbles at bits 4..7 / 20..23 of x -> f16x2 (1024 + 16 n)
//   biased1(x)   : nibbles at bits 0..3 / 16..19 of x -> f16x2 (1024 + n)
// The bias is removed afterwards in fp32, folded into other terms.
__device__ __forceinline__ uint32_t biased16(uint32_t x) { return lop3<0xEA>(x, 0x00F000F0u, 0x64006400u); }
__device__ __forceinline__ uint32_t biased1(uint32_t x) { return lop3<0xEA>(x, 0x000F000Fu, 0x64006400u); }

// 8x8 b16 matrix transpose across the warp (fragment layout in and out).
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------------ store addressing
// A page is page_tokens/128 blocks of 128 tokens; a block holds, at these byte
// offsets: K codes [128][64] | V codes [64 pairs][128] | metadata (ng groups):
//   HKV_FMT_REF:     K scales f32 [128][ng] | V scales | K zps u8 [128][ng] | V zps
//   HKV_FMT_FP16MIN: K scales f16 [128][ng] | K mins | V scales f16 [64 pairs][ng][2]
//                    | V mins  (the V entries of a token pair side by side, the
//                    layout the decode kernel's fragments read without a rewrite)
#define HKV_BLOCK_TOKENS 128
#define HKV_V_CODES_OFF 8192
#define HKV_META_OFF 16384

__host__ __device__ constexpr int block_bytes(int fmt, int group) {
  return HKV_BLOCK_TOKENS * (2 * HKV_CODE_BYTES + 8 * (HKV_D / group) + (fmt == HKV_FMT_REF ? 2 * (HKV_D / group) : 0));
}
// HKV_FMT_REF: byte offset of the K (role 0) or V (role 1) scales / zps inside a block.
__host__ __device__ constexpr int meta_off(int role, int ng) { return HKV_META_OFF + role * 512 * ng; }
__host__ __device__ constexpr int zps_off(int role, int ng) { return HKV_META_OFF + 1024 * ng + role * 128 * ng; }
// HKV_FMT_FP16MIN: byte offsets of the f16 scale and min of token w (0..127),
// group g of role K (0) or V (1) inside a block.
__host__ __device__ constexpr int mn_index(int role, int w, int ng, int g) {
  return role == 0 ? w * ng + g : ((w >> 1) * ng + g) * 2 + (w & 1);
}
__host__ __device__ constexpr int mn_scale_off(int role, int w, int ng, int g) {
  return HKV_META_OFF + role * 512 * ng + 2 * mn_index(role, w, ng, g);
}
__host__ __device__ constexpr int mn_min_off(int role, int w, int ng, int g) {
  return mn_scale_off(role, w, ng, g) + 256 * ng;
}
// Byte offset, inside the V code area of a block, of the 16-byte chunk c of
// token pair q. Rotating the chunks by 2q makes the decode kernel's fragment
// loads (chunk r of pairs j = 0..3 in one quarter-warp) hit 8 distinct bank groups.
__host__ __device__ constexpr int v_chunk_off(int q, int c) { return q * 128 + (((c + 2 * q) & 7) << 4); }

// Whether a page id may be dereferenced: non-negative, and inside the pool when
// the store declares its size (num_pages > 0).
__device__ __forceinline__ bool page_ok(const hkv_int4_store& s, int64_t page) {
  return page >= 0 && (s.num_pages <= 0 || page < s.num_pages);
}
// Page of token t of unit u, or -1 when the slot is outside the unit's table or
// the table holds an id outside the pool.
__device__ __forceinline__ int64_t store_page(const hkv_int4_store& s, int u, int t) {
  const int pi = t / s.page_tokens;
  if (t < 0 || pi >= s.max_pages) return -1;
  const int64_t page = s.page_table ? (int64_t)s.page_table[(int64_t)u * s.max_pages + pi]
                                    : (int64_t)u * s.max_pages + pi;
  return page_ok(s, page) ? page : -1;
}

// Block holding token slot `off` of page `page`, and the token's index in it.
struct BlockRef {
  uint8_t* base;
  int w;
};
__device__ __forceinline__ BlockRef block_ref(const hkv_int4_store& s, int64_t page, int off) {
  BlockRef r;
  r.base = static_cast<uint8_t*>(s.pages) + page * s.page_stride +
           (int64_t)(off / HKV_BLOCK_TOKENS) * block_bytes(s.format, s.group);
  r.w = off % HKV_BLOCK_TOKENS;
  return r;
}
