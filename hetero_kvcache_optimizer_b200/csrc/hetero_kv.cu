// libhetero_kv.so: the C ABI declared in include/hetero_kv.h.
// Single translation unit (the device error word is shared by every kernel).
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "hkv_common.cuh"
#include "hkv_quant.cuh"   // before the decode kernel: its fused append quantises with it
#include "hkv_decode.cuh"
#include "hkv_prefill.cuh"

#define HKV_VERSION 100

// Scratch of hkv_decode_attn_static (merge counters, then partials), for callers
// that cannot allocate a workspace. Zero at module load; one per device.
static __device__ __align__(256) unsigned char g_hkv_decode_scratch[HKV_STATIC_SCRATCH_BYTES];

namespace {

inline cudaStream_t S(hkv_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Last CUDA runtime error seen by a library call on this host thread (hkv_last_cuda_error).
thread_local int t_last_cuda_error = 0;

inline hkv_status cuda_fail(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return HKV_ERR_CUDA;
}

inline hkv_status launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HKV_OK : cuda_fail(e);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch with programmatic stream serialization (programmatic dependent launch):
// the kernel may start while the previous kernel in the stream finishes, and
// waits for it (griddep_wait) before its first global access. Used for the
// decode kernel (its barrier setup then overlaps the tail of the kernel before
// it: 2.586 -> 2.561 ms per config-1 step) and for the quantise-pack kernel
// (a chunked prefill's launches overlap their start with the previous one's
// drain: 4.82 -> 4.68 ms for config 2's 896 chunk launches); the append kernel,
// whose blocks would wait resident beside the decode kernel's, measured slower
// with it (2.608 ms) and launches normally. HKV_PDL (bit mask: 1 decode,
// 2 append, 4 quantise-pack; default 5) overrides this for experiments.
bool pdl_enabled(int which) {
  static const int mask = [] {
    const char* e = std::getenv("HKV_PDL");
    return e ? std::atoi(e) : 5;
  }();
  return (mask & which) != 0;
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(int which, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled(which) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline int cdiv(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// The workspace starts with a region reserved for the per-unit merge counters
// (one int32 per (sequence, KV head), at most kMaxUnits), so that calls of
// different shapes sharing one workspace never see partials where counters live.
constexpr int kMaxUnits = 65536;
constexpr size_t kCounterBytes = (size_t)kMaxUnits * sizeof(int);

int device_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> g(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool valid_group(int g) { return g == 32 || g == 64 || g == 128; }

hkv_status check_store(const hkv_int4_store* s) {
  if (!s) return HKV_ERR_ARG;
  if (s->format != HKV_FMT_REF && s->format != HKV_FMT_FP16MIN) return HKV_ERR_ARG;
  if (!valid_group(s->group)) return HKV_ERR_UNSUPPORTED;
  if (s->page_tokens <= 0 || s->page_tokens % hkv::kTileI4) return HKV_ERR_ARG;
  if (s->max_pages <= 0) return HKV_ERR_ARG;
  if (!s->pages || !aligned16(s->pages)) return HKV_ERR_ARG;
  const int64_t pb = hkv_page_bytes(s->format, s->group, s->page_tokens);
  if (s->page_stride < pb || s->page_stride % 16) return HKV_ERR_ARG;
  if (s->len < 0) return HKV_ERR_ARG;
  return HKV_OK;
}

hkv_status check_dense(const hkv_dense_kv* d) {
  if (!d) return HKV_ERR_ARG;
  if (d->dtype != HKV_DT_F16 && d->dtype != HKV_DT_BF16) return HKV_ERR_ARG;
  if (!d->k || !d->v || !aligned16(d->k) || !aligned16(d->v)) return HKV_ERR_ARG;
  if (d->stride_t % 8 || d->stride_h % 8 || d->stride_b % 8) return HKV_ERR_ARG;
  if (d->capacity < 0 || d->len < 0 || d->len > d->capacity) return HKV_ERR_ARG;
  return HKV_OK;
}

// The calling thread's current driver context (cuCtxGetCurrent through the
// runtime's entry-point query: no link dependency on libcuda), or nullptr.
CUcontext current_context() {
  typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(f);
  });
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

// Address of g_hkv_decode_scratch on the current device, looked up on the first
// call per device and again whenever the device's current context differs from
// the one the address was taken in (a cudaDeviceReset loads the module anew).
hkv_status static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  static CUcontext ctx[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= 64) return HKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> g(mu);
  const CUcontext cur = current_context();
  if (!addr[dev] || cur != ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_hkv_decode_scratch);
    if (e != cudaSuccess) return cuda_fail(e);
    addr[dev] = p;
    ctx[dev] = current_context();  // the lookup makes the primary context current
  }
  *out = addr[dev];
  return HKV_OK;
}

// --------------------------------------------------------------------------- decode plan
constexpr int kDynSmemBudget = 226 * 1024;  // one CTA per SM (227 KB opt-in, static barriers aside)
// Schedule weights, fitted to per-CTA end times of a config-1 layer (globaltimer
// probes in a copy of the kernel) and then swept on the 32-layer step: a dense
// tile costs ~0.7 of an INT4 tile per byte, so it weighs 75 % of its bytes; a
// segment start (piece start and end: query rows, partial, merge) is charged
// 1,440 steps of 128 B (180 KiB, ~9 fp16min group-32 tiles). Config-1 step:
// 2.522 ms with (100 %, 960) -> 2.489-2.492 ms; the region (70-85 %,
// 1,440-1,760) is flat within 0.5 %.
#ifndef HKV_PIECE_STEPS
#define HKV_PIECE_STEPS 1440
#endif
constexpr int64_t kPieceSteps = HKV_PIECE_STEPS;
constexpr int64_t kDenseWeightPct = 75;
// Schedule weights (HKV_SCHED_DENSE: percent of its bytes a dense tile weighs,
// HKV_SCHED_PIECE: steps charged per segment start) can be overridden for sweeps.
int64_t sched_dense_pct() {
  static const int64_t v = [] {
    const char* e = std::getenv("HKV_SCHED_DENSE");
    const int64_t x = e ? std::atoll(e) : kDenseWeightPct;
    return x > 0 && x <= 400 ? x : kDenseWeightPct;
  }();
  return v;
}
int64_t sched_piece_steps() {
  static const int64_t v = [] {
    const char* e = std::getenv("HKV_SCHED_PIECE");
    const int64_t x = e ? std::atoll(e) : kPieceSteps;
    return x >= 0 && x <= 16384 ? x : kPieceSteps;
  }();
  return v;
}

// cuTensorMapEncodeTiled, fetched from the driver through the runtime (no link
// dependency on libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// Dense K or V [B][Hkv][capacity][128] as a 5-D tensor (dim within a 64-dim
// half, token, half, head, batch): one box of 64 dims x 32 tokens x 2 halves is a
// whole 32-token tile side (8 KiB, one copy), landing in shared memory as
// [half][32 rows][128 B] with the 128-byte swizzle.
hkv_status dense_map(CUtensorMap* m, const void* base, const hkv_dense_kv* d, int B, int Hkv) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return HKV_ERR_CUDA;
  const cuuint64_t es = 2;
  const cuuint64_t dims[5] = {64, (cuuint64_t)std::max(1, d->capacity), 2, (cuuint64_t)Hkv, (cuuint64_t)B};
  const cuuint64_t strides[4] = {(cuuint64_t)d->stride_t * es, 64 * es, (cuuint64_t)d->stride_h * es,
                                 (cuuint64_t)d->stride_b * es};
  const cuuint32_t box[5] = {64, (cuuint32_t)hkv::kTileD, 2, 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = enc(m, d->dtype == HKV_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         5, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? HKV_OK : HKV_ERR_ARG;
}

template <int FMT, int GROUP, typename DTy, bool STATS, bool APPEND>
hkv_status launch_decode_t(const hkv::DecodeParams& p, int smem, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(hkv::decode_kernel<FMT, GROUP, DTy, STATS, APPEND>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmemBudget);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err);
  const cudaError_t e = launch_pdl(1, hkv::decode_kernel<FMT, GROUP, DTy, STATS, APPEND>, dim3(p.sc.C),
                                   dim3(hkv::decode_threads(FMT, APPEND)), smem, st, p);
  if (e != cudaSuccess) return cuda_fail(e);
  return launch_status();
}

template <int FMT, int GROUP, typename DTy>
hkv_status launch_decode_m(const hkv::DecodeParams& p, int smem, cudaStream_t st) {
  if (p.tile_stats) return launch_decode_t<FMT, GROUP, DTy, true, false>(p, smem, st);
  if (p.state_counter) return launch_decode_t<FMT, GROUP, DTy, false, true>(p, smem, st);
  return launch_decode_t<FMT, GROUP, DTy, false, false>(p, smem, st);
}

template <int FMT, int GROUP>
hkv_status launch_decode_g(const hkv::DecodeParams& p, int ddt, int smem, cudaStream_t st) {
  if (ddt == HKV_DT_BF16) return launch_decode_m<FMT, GROUP, __nv_bfloat16>(p, smem, st);
  return launch_decode_m<FMT, GROUP, __half>(p, smem, st);
}

template <int FMT>
hkv_status launch_decode_f(const hkv::DecodeParams& p, int group, int ddt, int smem, cudaStream_t st) {
  switch (group) {
    case 32: return launch_decode_g<FMT, 32>(p, ddt, smem, st);
    case 64: return launch_decode_g<FMT, 64>(p, ddt, smem, st);
    case 128: return launch_decode_g<FMT, 128>(p, ddt, smem, st);
  }
  return HKV_ERR_UNSUPPORTED;
}

// The persistent schedule: tiles per unit from the host length hints, bytes per
// tile, grid size, and an upper bound of the partial slots per unit.
struct Plan {
  hkv::Sched sc;
  int nslots, comb_bytes, smem;
  size_t ws_bytes;
};

hkv_status make_plan(int B, int Hq, int Hkv, const hkv_int4_store* body, const hkv_dense_kv* dense, int ctas,
                     Plan* out) {
  const int G = Hq / Hkv;
  hkv::Sched sc;
  std::memset(&sc, 0, sizeof(sc));
  sc.U = B * Hkv;
  int group = 32, fmt = HKV_FMT_REF;
  if (body) {
    group = body->group;
    fmt = body->format;
    // with per-sequence device lengths a zero hint still gets one tile, so extra
    // tiles can follow it when the true length is longer
    sc.Tb = body->len > 0 ? cdiv(body->len, hkv::kTileI4) : (body->lengths ? 1 : 0);
  }
  if (dense) sc.Td = dense->len > 0 ? cdiv(dense->len, hkv::kTileD) : (dense->lengths ? 1 : 0);
  if (sc.Tb + sc.Td == 0) sc.Td = 1;  // nothing to attend to: one empty tile yields zeros
  // tile weights in 128-byte steps (the kernel's schedule is 32-bit arithmetic)
  const int64_t tb = block_bytes(fmt, group) / hkv::kSchedStep;
  // dense tiles weighted by their bytes times sched_dense_pct() / 100
  const int64_t td = std::max<int64_t>(
      1, (int64_t)hkv::kTileD * 2 * HKV_D * 2 / hkv::kSchedStep * sched_dense_pct() / 100);
  // a segment also costs its piece start and end (query rows, partial, merge):
  // charged as steps before it, so that CTAs whose range holds more segment
  // starts get fewer tiles
  const int64_t wb = sc.Tb > 0 ? sched_piece_steps() : 0, wd = sc.Td > 0 ? sched_piece_steps() : 0;
  const int64_t Ub = wb + sc.Tb * tb + wd + sc.Td * td;
  const int64_t Btot = Ub * sc.U;
  if (Btot >= (int64_t(1) << 31)) return HKV_ERR_UNSUPPORTED;  // > 256 GiB in one call
  const int64_t maxtile = std::max<int64_t>(sc.Tb ? tb : 0, sc.Td ? td : 0);
  int C = ctas > 0 ? ctas : device_sms();
  C = (int)std::max<int64_t>(1, std::min<int64_t>(std::min(C, 65535), Btot / maxtile));  // >= 1 tile per CTA
  sc.C = C;
  sc.tb = (uint32_t)tb;
  sc.td = (uint32_t)td;
  sc.wb = (uint32_t)wb;
  sc.wd = (uint32_t)wd;
  sc.Ub = (uint32_t)Ub;
  sc.Btot = (uint32_t)Btot;
  sc.q = (uint32_t)(Btot / C);
  sc.r = (uint32_t)(Btot % C);
  // partial slots per unit: the CTAs whose ranges meet the unit (with margin),
  // plus one for the fused append's partial
  sc.S = (int)(Ub / (Btot / C)) + 5;
  Plan pl;
  pl.sc = sc;
  // the piece-end combine area, then the prefetched query rows of the next piece (f16/bf16)
  pl.comb_bytes = (hkv::kConsumerWarps * G * HKV_D + hkv::kConsumerWarps * 8 * 2) * 4 + G * HKV_D * 2;
  const int avail = kDynSmemBudget - 1024 - pl.comb_bytes;
  const int slot = hkv::slot_bytes(fmt, group);
  // even, so that every slot always serves the same consumer group (loads n and
  // n + nslots have the same parity): a group's parity wait on a slot can then
  // never match a phase that belongs to the other group's load
  pl.nslots = std::min(hkv::kMaxSlots, avail / slot) & ~1;
  if (pl.nslots < 2) return HKV_ERR_UNSUPPORTED;
  // + 1 KiB so the kernel can align the ring to 1024 bytes
  pl.smem = 1024 + pl.nslots * slot + pl.comb_bytes;
  pl.ws_bytes = kCounterBytes + (size_t)sc.U * sc.S * G * (HKV_D + 2) * sizeof(float);
  *out = pl;
  return HKV_OK;
}

hkv_status check_decode_args(const void* q, int q_dtype, const hkv_int4_store* body, const hkv_dense_kv* dense,
                             int B, int Hq, int Hkv, int D) {
  if (!q || (q_dtype != HKV_DT_F16 && q_dtype != HKV_DT_BF16)) return HKV_ERR_ARG;
  if (D != HKV_D) return HKV_ERR_UNSUPPORTED;
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv) return HKV_ERR_ARG;
  if (Hq / Hkv > 8) return HKV_ERR_UNSUPPORTED;
  if ((int64_t)B * Hkv > kMaxUnits) return HKV_ERR_UNSUPPORTED;
  if (!body && !dense) return HKV_ERR_ARG;
  hkv_status rc;
  if (body && (rc = check_store(body)) != HKV_OK) return rc;
  if (dense && (rc = check_dense(dense)) != HKV_OK) return rc;
  return HKV_OK;
}

// The decode step's new token and cache state for the fused append (hkv_decode_append).
struct AppendArgs {
  const void* k_new;
  const void* v_new;
  int64_t new_sb, new_sh;
  int sink;
  int32_t *dense_len, *ring_head, *body_len;
  int early;
};

hkv_status run_decode(const void* q, int q_dtype, int64_t q_sb, int64_t q_sh, const hkv_int4_store* body,
                      const hkv_dense_kv* dense, int B, int Hq, int Hkv, int D, float sm_scale, int ctas,
                      void* workspace, size_t workspace_bytes, void* out, int out_dtype, int64_t out_sb,
                      int64_t out_sh, float* out_o, float* out_ml, cudaStream_t st, float* tile_stats = nullptr,
                      int stat_tiles = 0, float* unit_ml = nullptr, const AppendArgs* app = nullptr) {
  hkv_status rc = check_decode_args(q, q_dtype, body, dense, B, Hq, Hkv, D);
  if (rc != HKV_OK) return rc;
  if (!(sm_scale > 0.f) || !std::isfinite(sm_scale)) return HKV_ERR_ARG;
  Plan pl;
  if ((rc = make_plan(B, Hq, Hkv, body, dense, ctas, &pl)) != HKV_OK) return rc;
  if (!workspace || workspace_bytes < pl.ws_bytes || !aligned16(workspace)) return HKV_ERR_CAPACITY;
  hkv::DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = q;
  p.q_dtype = q_dtype;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  // 16-byte aligned query rows are prefetched a piece ahead with cp.async
  p.q_async = aligned16(q) && (q_sb * 2) % 16 == 0 && (q_sh * 2) % 16 == 0;
  if (body) p.body = *body;
  if (dense) p.dense = *dense;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.qscale = static_cast<float>(static_cast<double>(sm_scale) * 1.4426950408889634);
  p.sc = pl.sc;
  if (dense) {
    if ((rc = dense_map(&p.tmk, dense->k, dense, B, Hkv)) != HKV_OK) return rc;
    if ((rc = dense_map(&p.tmv, dense->v, dense, B, Hkv)) != HKV_OK) return rc;
  }
  p.page_shift = -1;
  if (body && (body->page_tokens & (body->page_tokens - 1)) == 0) {
    int sh = 0;
    while ((1 << sh) < body->page_tokens) ++sh;
    p.page_shift = sh;
  }
  p.nslots = pl.nslots;
  p.counters = static_cast<int*>(workspace);
  p.part_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  p.part_ml = p.part_o + (size_t)pl.sc.U * pl.sc.S * p.G * HKV_D;
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_sb = out_sb;
  p.out_sh = out_sh;
  p.out_o = out_o;
  p.out_ml = out_ml;
  p.tile_stats = tile_stats;
  p.stat_tiles = stat_tiles;
  p.unit_ml = unit_ml;
  if (app) {
    p.k_new = app->k_new;
    p.v_new = app->v_new;
    p.new_sb = app->new_sb;
    p.new_sh = app->new_sh;
    p.sink = app->sink;
    p.dense_len = app->dense_len;
    p.ring_head = app->ring_head;
    p.body_len = app->body_len;
    p.early = app->early;
    // the last counter of the reserved region (units are limited to kMaxUnits - 1)
    p.state_counter = p.counters + (kMaxUnits - 1);
  }
  const int fmt = body ? body->format : HKV_FMT_REF;
  const int group = body ? body->group : 32;
  const int ddt = dense ? dense->dtype : HKV_DT_F16;
  if (fmt == HKV_FMT_REF) return launch_decode_f<HKV_FMT_REF>(p, group, ddt, pl.smem, st);
  return launch_decode_f<HKV_FMT_FP16MIN>(p, group, ddt, pl.smem, st);
}


// --------------------------------------------------------------------------- prefill
// Query rows per prefill CTA: 256 (two query tiles with their own softmax warps
// sharing each dequantised body tile, prefill2_kernel) when a unit has more than
// 128 rows, else 128. HKV_PREFILL_ROWS=128 forces one tile per CTA (comparisons).
int prefill_rows_per_cta(int64_t unit_rows) {
  static const int forced = [] {
    const char* e = std::getenv("HKV_PREFILL_ROWS");
    return e ? std::atoi(e) : 0;
  }();
  if (forced == hkv::kPfRows) return hkv::kPfRows;
  return unit_rows > hkv::kPfRows ? hkv::kPf2Rows : hkv::kPfRows;
}

template <int FMT, int GROUP>
hkv_status launch_prefill_t(const hkv::PrefillParams& p, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(hkv::prefill_kernel<FMT, GROUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    hkv::kPfSmem);
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(hkv::prefill2_kernel<FMT, GROUP>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, hkv::kPf2Smem);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err);
  const int rpc = prefill_rows_per_cta((int64_t)p.Sq * p.G);
  const dim3 grid((unsigned)cdiv((int64_t)p.Sq * p.G, rpc), (unsigned)(p.B * p.Hkv), (unsigned)p.nsplit);
  if (rpc == hkv::kPf2Rows)
    hkv::prefill2_kernel<FMT, GROUP><<<grid, hkv::kPf2Threads, hkv::kPf2Smem, st>>>(p);
  else
    hkv::prefill_kernel<FMT, GROUP><<<grid, hkv::kPfThreads, hkv::kPfSmem, st>>>(p);
  hkv_status rc = launch_status();
  if (rc != HKV_OK || p.nsplit == 1) return rc;
  const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
  hkv::prefill_merge_kernel<<<(unsigned)cdiv(rows, 8), 256, 0, st>>>(p);
  return launch_status();
}

// Splits of the body per query tile for a prefill: the smallest count that
// fills the SMs' waves best, by a model in units of one tile's time (~1.9 us):
// waves x (tiles per split + 5 for a CTA's fixed start and end, measured) + the
// merge's traffic (each split's partial, 520 B per row, read once at ~6.5 TB/s).
// `forced` > 0 asks for that count (still at most one split per tile, 16 in all).
int prefill_splits(int64_t base_ctas, int tiles, int64_t rows, int forced) {
  if (tiles <= 1) return 1;
  if (forced > 0) return std::min(std::min(forced, tiles), 16);
  const int sms = device_sms();
  double best = 0.0;
  int bs = 1;
  for (int sp = 1; sp <= 16; ++sp) {
    if (sp > 1 && tiles / sp < 8) break;
    const double waves = (double)((base_ctas * sp + sms - 1) / sms);
    double t = waves * ((double)tiles / sp + 5.0);
    if (sp > 1) t += (double)rows * sp * 520.0 / 6.5e12 / 1.9e-6 + 2.0;
    if (sp == 1 || t < 0.98 * best) {
      best = t;
      bs = sp;
    }
  }
  return bs;
}
inline size_t prefill_ws_bytes(int splits, int64_t rows) {
  return splits > 1 ? (size_t)splits * (size_t)rows * (HKV_D + 2) * sizeof(float) : 0;
}

// --------------------------------------------------------------------------- small kernels
// Bounded-wait self-test: one warp initialises an mbarrier that expects one
// arrival, lane 0 arrives only when `arrive` is set, and every lane waits on
// the phase with a limit of limit_ns. Without the arrival the wait gives up,
// flags HKV_DEVERR_TIMEOUT and the kernel returns normally: the same bounded
// wait the decode and prefill kernels use, made to run out on purpose without
// a fault or a hang.
__device__ int g_hkv_selftest_completed;
__global__ void __launch_bounds__(32) selftest_wait_kernel(uint64_t limit_ns, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  if (arrive && threadIdx.x == 0) mbar_arrive(&bar);
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, mbar_wait_limit(&bar, 0, 0, limit_ns));
  if (threadIdx.x == 0) g_hkv_selftest_completed = ok ? 1 : 0;
}

// Pre-softmax scores of one query row against S INT4 keys in the reference's
// unpacked layout (one code per byte, flat fp32 scales / u8 zero-points over
// groups of `group` values): out[s] = sum_d q[d] (c[s][d] - z) * scale, fp32,
// one warp per key.
template <typename QT>
__global__ void __launch_bounds__(256) qk_scores_flat_kernel(const QT* __restrict__ q, const uint8_t* __restrict__ c,
                                                            const float* __restrict__ sc,
                                                            const uint8_t* __restrict__ zp, int64_t S, int D,
                                                            int group, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t s = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < S; s += nw) {
    float acc = 0.f;
    for (int d = lane; d < D; d += 32) {
      const int64_t i = s * D + d;
      const int64_t g = i / group;
      acc = fmaf(to_f32(q[d]), (static_cast<float>(c[i]) - static_cast<float>(zp[g])) * sc[g], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[s] = acc;
  }
}

template <int FMT>
hkv_status launch_prefill_f(const hkv::PrefillParams& p, int group, cudaStream_t st) {
  switch (group) {
    case 32: return launch_prefill_t<FMT, 32>(p, st);
    case 64: return launch_prefill_t<FMT, 64>(p, st);
    case 128: return launch_prefill_t<FMT, 128>(p, st);
  }
  return HKV_ERR_UNSUPPORTED;
}

}  // namespace

// =========================================================================== C ABI
extern "C" {

const char* hkv_status_str(hkv_status s) {
  switch (s) {
    case HKV_OK: return "HKV_OK";
    case HKV_ERR_ARG: return "HKV_ERR_ARG: invalid argument";
    case HKV_ERR_CUDA: return "HKV_ERR_CUDA: CUDA runtime error";
    case HKV_ERR_TIMEOUT: return "HKV_ERR_TIMEOUT: bounded wait expired";
    case HKV_ERR_UNSUPPORTED: return "HKV_ERR_UNSUPPORTED: unsupported configuration";
    case HKV_ERR_CAPACITY: return "HKV_ERR_CAPACITY: destination or workspace too small";
    case HKV_ERR_DEVICE: return "HKV_ERR_DEVICE: a kernel reported a device-side error";
  }
  return "HKV_ERR_UNKNOWN";
}

int hkv_version(void) { return HKV_VERSION; }

hkv_status hkv_device_error(uint32_t* bits, int clear) {
  if (!bits) return HKV_ERR_ARG;
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_hkv_dev_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e);
  *bits = v;
  if (clear) {
    const unsigned int z = 0;
    if ((e = cudaMemcpyToSymbol(g_hkv_dev_error, &z, sizeof(z))) != cudaSuccess) return cuda_fail(e);
  }
  return HKV_OK;
}

int32_t hkv_last_cuda_error(void) { return t_last_cuda_error; }

int64_t hkv_page_bytes(int32_t format, int32_t group, int32_t page_tokens) {
  if (!valid_group(group) || page_tokens <= 0 || page_tokens % HKV_BLOCK_TOKENS) return -1;
  if (format != HKV_FMT_REF && format != HKV_FMT_FP16MIN) return -1;
  return (int64_t)(page_tokens / HKV_BLOCK_TOKENS) * block_bytes(format, group);
}

// --------------------------------------------------------------------------- quantise
hkv_status hkv_quantize_flat(const void* x, int32_t dtype, int64_t n, int32_t group, uint8_t* codes, float* scales,
                             uint8_t* zps, hkv_stream_t stream) {
  if (!x || !codes || !scales || !zps || n <= 0 || group <= 0) return HKV_ERR_ARG;
  const int64_t ngroups = (n + group - 1) / group;
  const int threads = 256;
  const int64_t want = (ngroups + 7) / 8;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)device_sms() * 16));
  switch (dtype) {
    case HKV_DT_F16:
      hkv::quantize_flat_kernel<__half><<<blocks, threads, 0, S(stream)>>>(static_cast<const __half*>(x), n, group,
                                                                           ngroups, codes, scales, zps);
      break;
    case HKV_DT_BF16:
      hkv::quantize_flat_kernel<__nv_bfloat16><<<blocks, threads, 0, S(stream)>>>(
          static_cast<const __nv_bfloat16*>(x), n, group, ngroups, codes, scales, zps);
      break;
    case HKV_DT_F32:
      hkv::quantize_flat_kernel<float><<<blocks, threads, 0, S(stream)>>>(static_cast<const float*>(x), n, group,
                                                                          ngroups, codes, scales, zps);
      break;
    default: return HKV_ERR_ARG;
  }
  return launch_status();
}

hkv_status hkv_dequantize_flat(const uint8_t* codes, const float* scales, const uint8_t* zps, int64_t n,
                               int32_t group, void* out, int32_t out_dtype, hkv_stream_t stream) {
  if (!codes || !scales || !zps || !out || n <= 0 || group <= 0) return HKV_ERR_ARG;
  const int threads = 256;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, (int64_t)device_sms() * 32));
  switch (out_dtype) {
    case HKV_DT_F16:
      hkv::dequantize_flat_kernel<__half><<<blocks, threads, 0, S(stream)>>>(codes, scales, zps, n, group,
                                                                             static_cast<__half*>(out));
      break;
    case HKV_DT_BF16:
      hkv::dequantize_flat_kernel<__nv_bfloat16><<<blocks, threads, 0, S(stream)>>>(
          codes, scales, zps, n, group, static_cast<__nv_bfloat16*>(out));
      break;
    case HKV_DT_F32:
      hkv::dequantize_flat_kernel<float><<<blocks, threads, 0, S(stream)>>>(codes, scales, zps, n, group,
                                                                            static_cast<float*>(out));
      break;
    default: return HKV_ERR_ARG;
  }
  return launch_status();
}

namespace {
hkv_status quantize_pack_launch(const void* x, const void* x2, int32_t dtype, int32_t B, int32_t H, int32_t T,
                                int32_t D, int64_t stride_b, int64_t stride_h, int64_t stride_t, int32_t role,
                                const hkv_int4_store* dst, const int32_t* dst_start, int32_t start,
                                cudaStream_t st) {
  if (!x || B <= 0 || H <= 0 || T < 0) return HKV_ERR_ARG;
  if (D != HKV_D) return HKV_ERR_UNSUPPORTED;
  if (role != HKV_ROLE_K && role != HKV_ROLE_V) return HKV_ERR_ARG;
  hkv_status rc = check_store(dst);
  if (rc != HKV_OK) return rc;
  if (!aligned16(x) || (x2 && !aligned16(x2)) || stride_b % 8 || stride_h % 8 || stride_t % 8) return HKV_ERR_ARG;
  if (!dst_start && (start < 0 || (int64_t)start + T > (int64_t)dst->max_pages * dst->page_tokens))
    return HKV_ERR_CAPACITY;
  if (T == 0) return HKV_OK;
  const int64_t ntok = (int64_t)B * H * T;
  if (ntok >= (int64_t(1) << 31) - 64) return HKV_ERR_UNSUPPORTED;
  // 64-position tiles aligned in position space: a chunk starting mid-tile spans one more
  const int tiles = (T + hkv::kQPTile - 1) / hkv::kQPTile + 1;
  if ((int64_t)tiles * B * H >= (int64_t(1) << 31)) return HKV_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)(tiles * B * H), x2 ? 2u : 1u);
  const bool ref = dst->format == HKV_FMT_REF;
  const int g = dst->group;
  cudaError_t qerr = cudaSuccess;
#define HKV_QP_LAUNCH(TY, FMT, G)                                                                            \
  qerr = launch_pdl(4, hkv::quantize_pack_kernel<TY, FMT, G>, grid, dim3(256), 0, st, static_cast<const TY*>(x), \
                    static_cast<const TY*>(x2), (int)H, (int)T, tiles, stride_b, stride_h, stride_t, (int)role, *dst, \
                    dst_start, (int)start)
#define HKV_QP_GROUPS(TY, FMT)        \
  if (g == 32) HKV_QP_LAUNCH(TY, FMT, 32);      \
  else if (g == 64) HKV_QP_LAUNCH(TY, FMT, 64); \
  else HKV_QP_LAUNCH(TY, FMT, 128)
  if (dtype == HKV_DT_F16) {
    if (ref) { HKV_QP_GROUPS(__half, HKV_FMT_REF); } else { HKV_QP_GROUPS(__half, HKV_FMT_FP16MIN); }
  } else if (dtype == HKV_DT_BF16) {
    if (ref) { HKV_QP_GROUPS(__nv_bfloat16, HKV_FMT_REF); } else { HKV_QP_GROUPS(__nv_bfloat16, HKV_FMT_FP16MIN); }
  } else {
    return HKV_ERR_ARG;
  }
#undef HKV_QP_GROUPS
#undef HKV_QP_LAUNCH
  if (qerr != cudaSuccess) return cuda_fail(qerr);
  return launch_status();
}
}  // namespace

hkv_status hkv_quantize_pack(const void* x, int32_t dtype, int32_t B, int32_t H, int32_t T, int32_t D,
                             int64_t stride_b, int64_t stride_h, int64_t stride_t, int32_t role,
                             const hkv_int4_store* dst, const int32_t* dst_start, int32_t start,
                             hkv_stream_t stream) {
  return quantize_pack_launch(x, nullptr, dtype, B, H, T, D, stride_b, stride_h, stride_t, role, dst, dst_start,
                              start, S(stream));
}

hkv_status hkv_quantize_pack_kv(const void* k, const void* v, int32_t dtype, int32_t B, int32_t H, int32_t T,
                                int32_t D, int64_t stride_b, int64_t stride_h, int64_t stride_t,
                                const hkv_int4_store* dst, const int32_t* dst_start, int32_t start,
                                hkv_stream_t stream) {
  if (!v) return HKV_ERR_ARG;
  return quantize_pack_launch(k, v, dtype, B, H, T, D, stride_b, stride_h, stride_t, HKV_ROLE_K, dst, dst_start,
                              start, S(stream));
}

hkv_status hkv_append_kv(const void* k_new, const void* v_new, int32_t dtype, int32_t B, int32_t H, int32_t D,
                         int64_t stride_b, int64_t stride_h, const hkv_dense_kv* dense, int32_t sink,
                         int32_t* dense_len, int32_t* ring_head, const hkv_int4_store* body, int32_t* body_len,
                         hkv_stream_t stream) {
  if (!k_new || !v_new || B <= 0 || H <= 0 || H > 32) return HKV_ERR_ARG;
  if (D != HKV_D) return HKV_ERR_UNSUPPORTED;
  if (!dense_len || !ring_head || !body_len) return HKV_ERR_ARG;
  hkv_status rc = check_dense(dense);
  if (rc != HKV_OK) return rc;
  if ((rc = check_store(body)) != HKV_OK) return rc;
  if (dense->dtype != dtype) return HKV_ERR_ARG;
  if (sink < 0 || sink > dense->capacity) return HKV_ERR_ARG;
  if (!aligned16(k_new) || !aligned16(v_new) || stride_b % 8 || stride_h % 8) return HKV_ERR_ARG;
  if (dtype == HKV_DT_F16) {
    const cudaError_t e = launch_pdl(2, hkv::append_kv_kernel<__half>, dim3(B), dim3(32 * H), 0, S(stream),
                                     static_cast<const __half*>(k_new), static_cast<const __half*>(v_new), H,
                                     stride_b, stride_h, *dense, sink, dense_len, ring_head, *body, body_len);
    if (e != cudaSuccess) return cuda_fail(e);
  } else if (dtype == HKV_DT_BF16) {
    const cudaError_t e =
        launch_pdl(2, hkv::append_kv_kernel<__nv_bfloat16>, dim3(B), dim3(32 * H), 0, S(stream),
                   static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new), H, stride_b,
                   stride_h, *dense, sink, dense_len, ring_head, *body, body_len);
    if (e != cudaSuccess) return cuda_fail(e);
  } else {
    return HKV_ERR_ARG;
  }
  return launch_status();
}

hkv_status hkv_dequantize_pack(const hkv_int4_store* src, int32_t role, int32_t B, int32_t H, int32_t t0, int32_t T,
                               void* out, int32_t out_dtype, hkv_stream_t stream) {
  hkv_status rc = check_store(src);
  if (rc != HKV_OK) return rc;
  if (!out || B <= 0 || H <= 0 || t0 < 0 || T < 0) return HKV_ERR_ARG;
  if ((int64_t)t0 + T > (int64_t)src->max_pages * src->page_tokens) return HKV_ERR_CAPACITY;
  if (T == 0) return HKV_OK;
  const int64_t ntok = (int64_t)B * H * T;
  const int blocks = (int)((ntok + 1) / 2);
  switch (out_dtype) {
    case HKV_DT_F16:
      hkv::dequantize_pack_kernel<__half><<<blocks, 256, 0, S(stream)>>>(*src, role, H, t0, T, ntok,
                                                                        static_cast<__half*>(out));
      break;
    case HKV_DT_BF16:
      hkv::dequantize_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, S(stream)>>>(*src, role, H, t0, T, ntok,
                                                                               static_cast<__nv_bfloat16*>(out));
      break;
    case HKV_DT_F32:
      hkv::dequantize_pack_kernel<float><<<blocks, 256, 0, S(stream)>>>(*src, role, H, t0, T, ntok,
                                                                       static_cast<float*>(out));
      break;
    default: return HKV_ERR_ARG;
  }
  return launch_status();
}

hkv_status hkv_repack_ref(const uint8_t* codes, const float* scales, const uint8_t* zps, int32_t B, int32_t H,
                          int32_t S_, int32_t group, int32_t role, const hkv_int4_store* dst, hkv_stream_t stream) {
  hkv_status rc = check_store(dst);
  if (rc != HKV_OK) return rc;
  if (!codes || !scales || !zps || B <= 0 || H <= 0 || S_ < 0) return HKV_ERR_ARG;
  if (dst->format != HKV_FMT_REF || dst->group != group) return HKV_ERR_ARG;
  if (S_ > dst->max_pages * dst->page_tokens) return HKV_ERR_CAPACITY;
  if (S_ == 0) return HKV_OK;
  const int64_t ntok = (int64_t)B * H * S_;
  hkv::repack_ref_kernel<<<(int)((ntok + 7) / 8), 256, 0, S(stream)>>>(codes, scales, zps, S_, group, role, *dst,
                                                                       ntok);
  return launch_status();
}

// --------------------------------------------------------------------------- decode
size_t hkv_decode_workspace_bytes(const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B, int32_t Hq,
                                  int32_t Hkv, int32_t D, int32_t ctas) {
  static const uint16_t one = 0x3C00;
  if (check_decode_args(&one, HKV_DT_F16, body, dense, B, Hq, Hkv, D) != HKV_OK) return 0;
  Plan pl;
  if (make_plan(B, Hq, Hkv, body, dense, ctas, &pl) != HKV_OK) return 0;
  return pl.ws_bytes;
}

hkv_status hkv_decode_plan(const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B, int32_t Hq, int32_t Hkv,
                           int32_t ctas, int32_t* grid, int32_t* slots_per_unit) {
  if (!grid || !slots_per_unit) return HKV_ERR_ARG;
  static const uint16_t one = 0x3C00;
  hkv_status rc = check_decode_args(&one, HKV_DT_F16, body, dense, B, Hq, Hkv, HKV_D);
  if (rc != HKV_OK) return rc;
  Plan pl;
  if ((rc = make_plan(B, Hq, Hkv, body, dense, ctas, &pl)) != HKV_OK) return rc;
  *grid = pl.sc.C;
  *slots_per_unit = pl.sc.S;
  return HKV_OK;
}

hkv_status hkv_decode_attn(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                           const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B, int32_t Hq, int32_t Hkv,
                           int32_t D, float sm_scale, int32_t ctas, void* workspace, size_t workspace_bytes,
                           void* out, int32_t out_dtype, int64_t out_stride_b, int64_t out_stride_h,
                           hkv_stream_t stream) {
  if (!out || (out_dtype != HKV_DT_F16 && out_dtype != HKV_DT_BF16 && out_dtype != HKV_DT_F32)) return HKV_ERR_ARG;
  return run_decode(q, q_dtype, q_stride_b, q_stride_h, body, dense, B, Hq, Hkv, D, sm_scale, ctas, workspace,
                    workspace_bytes, out, out_dtype, out_stride_b, out_stride_h, nullptr, nullptr, S(stream));
}

hkv_status hkv_decode_append(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                             const void* k_new, const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
                             const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t sink,
                             int32_t* dense_len, int32_t* ring_head, int32_t* body_len, int32_t B, int32_t Hq,
                             int32_t Hkv, int32_t D, float sm_scale, int32_t ctas, void* workspace,
                             size_t workspace_bytes, void* out, int32_t out_dtype, int64_t out_stride_b,
                             int64_t out_stride_h, int32_t flags, hkv_stream_t stream) {
  if (!out || (out_dtype != HKV_DT_F16 && out_dtype != HKV_DT_BF16 && out_dtype != HKV_DT_F32)) return HKV_ERR_ARG;
  if (!body || !dense || !k_new || !v_new || !dense_len || !ring_head || !body_len) return HKV_ERR_ARG;
  if (flags & ~HKV_APPEND_EARLY) return HKV_ERR_ARG;
  // the attention reads the lengths the append advances: one set of state arrays
  if (body->lengths != body_len || dense->lengths != dense_len) return HKV_ERR_ARG;
  if (!aligned16(k_new) || !aligned16(v_new) || new_stride_b % 8 || new_stride_h % 8) return HKV_ERR_ARG;
  if (sink < 0 || sink > dense->capacity) return HKV_ERR_ARG;
  if ((int64_t)B * Hkv > kMaxUnits - 1) return HKV_ERR_UNSUPPORTED;  // the last counter is the state counter
  // a unit's last pipeline piece waits for the append warp of another CTA, so
  // every CTA must be resident at once: at most one CTA per SM
  if (ctas > device_sms()) return HKV_ERR_ARG;
  AppendArgs app{k_new, v_new, new_stride_b, new_stride_h, sink, dense_len, ring_head, body_len,
                 (flags & HKV_APPEND_EARLY) ? 1 : 0};
  return run_decode(q, q_dtype, q_stride_b, q_stride_h, body, dense, B, Hq, Hkv, D, sm_scale, ctas, workspace,
                    workspace_bytes, out, out_dtype, out_stride_b, out_stride_h, nullptr, nullptr, S(stream), nullptr,
                    0, nullptr, &app);
}

hkv_status hkv_decode_attn_scored(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                  const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B, int32_t Hq,
                                  int32_t Hkv, int32_t D, float sm_scale, int32_t ctas, void* workspace,
                                  size_t workspace_bytes, void* out, int32_t out_dtype, int64_t out_stride_b,
                                  int64_t out_stride_h, float* tile_stats, int32_t stat_tiles, float* unit_ml,
                                  hkv_stream_t stream) {
  if (!out || (out_dtype != HKV_DT_F16 && out_dtype != HKV_DT_BF16 && out_dtype != HKV_DT_F32)) return HKV_ERR_ARG;
  if (!tile_stats || !unit_ml || stat_tiles <= 0 || !aligned16(tile_stats)) return HKV_ERR_ARG;
  return run_decode(q, q_dtype, q_stride_b, q_stride_h, body, dense, B, Hq, Hkv, D, sm_scale, ctas, workspace,
                    workspace_bytes, out, out_dtype, out_stride_b, out_stride_h, nullptr, nullptr, S(stream),
                    tile_stats, stat_tiles, unit_ml);
}

size_t hkv_prefill_workspace_bytes(const hkv_int4_store* body, int32_t B, int32_t Hq, int32_t Hkv, int32_t Sq,
                                   int32_t D, int32_t splits) {
  if (check_store(body) != HKV_OK || B <= 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv || Sq <= 0 || D != HKV_D) return 0;
  const int64_t unit_rows = (int64_t)Sq * (Hq / Hkv);
  const int64_t base = cdiv(unit_rows, prefill_rows_per_cta(unit_rows)) * B * Hkv;
  const int64_t rows = (int64_t)B * Hq * Sq;
  const int tiles = (int)cdiv((int64_t)body->len, hkv::kTileI4);
  return prefill_ws_bytes(prefill_splits(base, tiles, rows, splits), rows);
}

hkv_status hkv_prefill_attn(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                            int64_t q_stride_s, const hkv_int4_store* body, int32_t B, int32_t Hq, int32_t Hkv,
                            int32_t Sq, int32_t D, float sm_scale, int32_t causal, void* out, int32_t out_dtype,
                            int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s, float* lse,
                            int32_t splits, void* workspace, size_t workspace_bytes, hkv_stream_t stream) {
  if (!q || !out || (q_dtype != HKV_DT_F16 && q_dtype != HKV_DT_BF16)) return HKV_ERR_ARG;
  if (out_dtype != HKV_DT_F16 && out_dtype != HKV_DT_BF16 && out_dtype != HKV_DT_F32) return HKV_ERR_ARG;
  if (D != HKV_D) return HKV_ERR_UNSUPPORTED;
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv || Sq < 0 || splits < 0) return HKV_ERR_ARG;
  if ((int64_t)B * Hkv > 65535) return HKV_ERR_UNSUPPORTED;
  if (!(sm_scale > 0.f) || !std::isfinite(sm_scale)) return HKV_ERR_ARG;
  if (workspace && !aligned16(workspace)) return HKV_ERR_ARG;
  hkv_status rc = check_store(body);
  if (rc != HKV_OK) return rc;
  if (Sq == 0) return HKV_OK;
  hkv::PrefillParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = q;
  p.q_dtype = q_dtype;
  p.q_sb = q_stride_b;
  p.q_sh = q_stride_h;
  p.q_ss = q_stride_s;
  p.body = *body;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.Sq = Sq;
  p.qscale = static_cast<float>(static_cast<double>(sm_scale) * 1.4426950408889634);
  p.out = out;
  p.out_dtype = out_dtype;
  p.out_sb = out_stride_b;
  p.out_sh = out_stride_h;
  p.out_ss = out_stride_s;
  p.causal = causal ? 1 : 0;
  p.lse = lse;
  {
    // body splits (wave quantisation): as many as the workspace holds, up to the model's choice
    const int64_t unit_rows = (int64_t)Sq * p.G;
    const int64_t base = cdiv(unit_rows, prefill_rows_per_cta(unit_rows)) * B * Hkv;
    const int64_t rows = (int64_t)B * Hq * Sq;
    int sp = prefill_splits(base, (int)cdiv((int64_t)body->len, hkv::kTileI4), rows, splits);
    while (sp > 1 && (!workspace || prefill_ws_bytes(sp, rows) > workspace_bytes)) --sp;
    p.nsplit = sp;
    if (sp > 1) {
      p.part_o = static_cast<float*>(workspace);
      p.part_ml = p.part_o + (size_t)sp * rows * HKV_D;
    }
  }
  {
    const int64_t e = out_dtype == HKV_DT_F32 ? 4 : 8;  // elements per 16 bytes
    p.out_vec = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && out_stride_b % e == 0 && out_stride_h % e == 0 &&
                out_stride_s % e == 0;
    p.q_vec = (reinterpret_cast<uintptr_t>(q) % 16 == 0) && q_stride_b % 8 == 0 && q_stride_h % 8 == 0 &&
              q_stride_s % 8 == 0;
  }
  if (body->format == HKV_FMT_REF) return launch_prefill_f<HKV_FMT_REF>(p, body->group, S(stream));
  return launch_prefill_f<HKV_FMT_FP16MIN>(p, body->group, S(stream));
}

hkv_status hkv_tile_scores(const float* tile_stats, const float* unit_ml, const hkv_int4_store* body, int32_t B,
                           int32_t Hkv, int32_t G, int32_t stat_tiles, float* mass, hkv_stream_t stream) {
  if (!tile_stats || !unit_ml || !mass || !body || B <= 0 || Hkv <= 0 || G <= 0 || G > 8 || stat_tiles <= 0)
    return HKV_ERR_ARG;
  if ((int64_t)B * Hkv > kMaxUnits) return HKV_ERR_UNSUPPORTED;
  hkv::tile_scores_kernel<<<B * Hkv, 128, 0, S(stream)>>>(tile_stats, unit_ml, body->lengths, body->len, Hkv, G,
                                                         stat_tiles, mass);
  return launch_status();
}

hkv_status hkv_decode_attn_partial(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                   const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B, int32_t Hq,
                                   int32_t Hkv, int32_t D, float sm_scale, int32_t ctas, void* workspace,
                                   size_t workspace_bytes, float* part_o, float* part_ml, hkv_stream_t stream) {
  if (!part_o || !part_ml) return HKV_ERR_ARG;
  return run_decode(q, q_dtype, q_stride_b, q_stride_h, body, dense, B, Hq, Hkv, D, sm_scale, ctas, workspace,
                    workspace_bytes, nullptr, HKV_DT_F32, 0, 0, part_o, part_ml, S(stream));
}

hkv_status hkv_decode_attn_static(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                                  const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B, int32_t Hq,
                                  int32_t Hkv, int32_t D, float sm_scale, int32_t ctas, void* out, int32_t out_dtype,
                                  int64_t out_stride_b, int64_t out_stride_h, hkv_stream_t stream) {
  if (!out || (out_dtype != HKV_DT_F16 && out_dtype != HKV_DT_BF16 && out_dtype != HKV_DT_F32)) return HKV_ERR_ARG;
  // validate and size the request on the host first: an invalid or oversized one
  // fails before any CUDA call (nothing queued on the stream)
  hkv_status rc = check_decode_args(q, q_dtype, body, dense, B, Hq, Hkv, D);
  if (rc != HKV_OK) return rc;
  if (!(sm_scale > 0.f) || !std::isfinite(sm_scale)) return HKV_ERR_ARG;
  Plan pl;
  if ((rc = make_plan(B, Hq, Hkv, body, dense, ctas, &pl)) != HKV_OK) return rc;
  if (pl.ws_bytes > HKV_STATIC_SCRATCH_BYTES) return HKV_ERR_CAPACITY;
  void* scratch = nullptr;
  if ((rc = static_scratch(&scratch)) != HKV_OK) return rc;
  // the merge counters must start at zero; the partials are written before they are read
  const cudaError_t e = cudaMemsetAsync(scratch, 0, (size_t)pl.sc.U * sizeof(int), S(stream));
  if (e != cudaSuccess) return cuda_fail(e);
  return run_decode(q, q_dtype, q_stride_b, q_stride_h, body, dense, B, Hq, Hkv, D, sm_scale, ctas, scratch,
                    HKV_STATIC_SCRATCH_BYTES, out, out_dtype, out_stride_b, out_stride_h, nullptr, nullptr,
                    S(stream));
}

hkv_status hkv_lse_merge(const float* part_o, const float* part_ml, int32_t n, int32_t B, int32_t Hq, int32_t D,
                         void* out, int32_t out_dtype, int64_t out_stride_b, int64_t out_stride_h,
                         hkv_stream_t stream) {
  return hkv_lse_merge_strided(part_o, part_ml, n, (int64_t)B * Hq * HKV_D, (int64_t)B * Hq * 2, B, Hq, D, out,
                               out_dtype, out_stride_b, out_stride_h, stream);
}

hkv_status hkv_lse_merge_strided(const float* part_o, const float* part_ml, int32_t n, int64_t split_o,
                                 int64_t split_ml, int32_t B, int32_t Hq, int32_t D, void* out, int32_t out_dtype,
                                 int64_t out_stride_b, int64_t out_stride_h, hkv_stream_t stream) {
  if (!part_o || !part_ml || !out || n <= 0 || B <= 0 || Hq <= 0) return HKV_ERR_ARG;
  if (D != HKV_D) return HKV_ERR_UNSUPPORTED;
  if (out_dtype != HKV_DT_F16 && out_dtype != HKV_DT_BF16 && out_dtype != HKV_DT_F32) return HKV_ERR_ARG;
  if (split_o < 0 || split_ml < 0) return HKV_ERR_ARG;
  hkv::MergeParams mp;
  std::memset(&mp, 0, sizeof(mp));
  mp.part_o = part_o;
  mp.part_ml = part_ml;
  mp.S = n;
  mp.Hq = Hq;
  mp.split_o = split_o;
  mp.split_ml = split_ml;
  mp.out = out;
  mp.out_dtype = out_dtype;
  mp.out_sb = out_stride_b;
  mp.out_sh = out_stride_h;
  hkv::lse_merge_kernel<<<B * Hq, 128, 0, S(stream)>>>(mp);
  return launch_status();
}

hkv_status hkv_qk_scores_flat(const void* q, int32_t q_dtype, const uint8_t* codes, const float* scales,
                              const uint8_t* zps, int64_t n_keys, int32_t D, int32_t group, float* out,
                              hkv_stream_t stream) {
  if (!q || !codes || !scales || !zps || !out || n_keys < 0 || D <= 0 || group <= 0) return HKV_ERR_ARG;
  if (n_keys == 0) return HKV_OK;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n_keys + 7) / 8, (int64_t)device_sms() * 16));
  switch (q_dtype) {
    case HKV_DT_F16:
      qk_scores_flat_kernel<__half><<<blocks, 256, 0, S(stream)>>>(static_cast<const __half*>(q), codes, scales,
                                                                   zps, n_keys, D, group, out);
      break;
    case HKV_DT_BF16:
      qk_scores_flat_kernel<__nv_bfloat16><<<blocks, 256, 0, S(stream)>>>(
          static_cast<const __nv_bfloat16*>(q), codes, scales, zps, n_keys, D, group, out);
      break;
    case HKV_DT_F32:
      qk_scores_flat_kernel<float><<<blocks, 256, 0, S(stream)>>>(static_cast<const float*>(q), codes, scales, zps,
                                                                  n_keys, D, group, out);
      break;
    default: return HKV_ERR_ARG;
  }
  return launch_status();
}

hkv_status hkv_selftest_bounded_wait(int64_t limit_ns, int32_t arrive, hkv_stream_t stream) {
  if (limit_ns <= 0 || limit_ns > 1000000000LL) return HKV_ERR_ARG;
  selftest_wait_kernel<<<1, 32, 0, S(stream)>>>((uint64_t)limit_ns, arrive ? 1 : 0);
  hkv_status rc = launch_status();
  if (rc != HKV_OK) return rc;
  cudaError_t e = cudaStreamSynchronize(S(stream));
  if (e != cudaSuccess) return cuda_fail(e);
  int completed = 0;
  if ((e = cudaMemcpyFromSymbol(&completed, g_hkv_selftest_completed, sizeof(int))) != cudaSuccess)
    return cuda_fail(e);
  return completed ? HKV_OK : HKV_ERR_DEVICE;
}

// --------------------------------------------------------------------------- prefetch
struct hkv_prefetcher {
  const uint8_t* host;
  const uint8_t* host_dev;  // the host pool as kernels address it (mapped pinned memory), or null
  int64_t host_pages;
  uint8_t* dev;
  int64_t dev_pages;
  int64_t page_bytes;
  std::atomic<int64_t> bytes;
};

namespace {
// Zero-copy page gather: the pages' 16-byte vectors are cut into chunks of
// kGatherThreads * kGatherUnroll; CTAs take chunks blockIdx.x, blockIdx.x +
// gridDim.x, ... and every thread keeps kGatherUnroll loads in flight (16 KB per
// CTA) over the host link from mapped pinned host memory, then writes them to
// the page's device slot. 128 threads of few registers: a CTA fits beside a
// persistent decode CTA on the same SM, so gathers overlap attention.
// Host page of entry k: (src[k] + (step ? (*step + step_add) * step_mul : 0))
// mod host_pages, so a graph can replay a sliding selection whose ids advance
// with a device-side step counter. Ids outside the pools are skipped and
// flagged HKV_DEVERR_BAD_PAGE.
constexpr int kGatherThreads = 128;
constexpr int kGatherUnroll = 8;
__global__ void __launch_bounds__(kGatherThreads) page_gather_kernel(
    const uint4* __restrict__ host, uint4* __restrict__ dev, const int32_t* __restrict__ src,
    const int32_t* __restrict__ dst, int n, int64_t page_vecs, int64_t host_pages, int64_t dev_pages,
    const int64_t* __restrict__ step, int64_t step_mul, int32_t step_add) {
  constexpr int64_t kChunk = (int64_t)kGatherThreads * kGatherUnroll;
  const int64_t shift = step ? (*step + step_add) * step_mul : 0;
  const int64_t cpp = (page_vecs + kChunk - 1) / kChunk;  // chunks per page
  const int64_t items = (int64_t)n * cpp;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int k = (int)(it / cpp);
    const int64_t c0 = (it - (int64_t)k * cpp) * kChunk;
    const int64_t raw = src[k], dp = dst[k];
    int64_t sp = (raw + shift) % host_pages;
    if (sp < 0) sp += host_pages;
    if (raw < 0 || (!step && raw >= host_pages) || dp < 0 || dp >= dev_pages) {
      if (threadIdx.x == 0 && c0 == 0) hkv_flag_error(HKV_DEVERR_BAD_PAGE);
      continue;
    }
    const uint4* s = host + sp * page_vecs + c0;
    uint4* d = dev + dp * page_vecs + c0;
    const int64_t lim = page_vecs - c0;
    uint4 r[kGatherUnroll];
#pragma unroll
    for (int j = 0; j < kGatherUnroll; ++j) {
      const int64_t i = threadIdx.x + (int64_t)j * kGatherThreads;
      if (i < lim) r[j] = s[i];
    }
#pragma unroll
    for (int j = 0; j < kGatherUnroll; ++j) {
      const int64_t i = threadIdx.x + (int64_t)j * kGatherThreads;
      if (i < lim) d[i] = r[j];
    }
  }
}
}  // namespace

hkv_status hkv_prefetcher_create(const void* host_pool, int64_t host_pages, void* dev_pool, int64_t dev_pages,
                                 int64_t page_bytes, hkv_prefetcher** out) {
  if (!out || !host_pool || !dev_pool || host_pages <= 0 || dev_pages <= 0 || page_bytes <= 0) return HKV_ERR_ARG;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, host_pool) != cudaSuccess) {
    cudaGetLastError();
    return HKV_ERR_ARG;
  }
  // the host pool must be page-locked, or every async copy silently serialises
  if (attr.type != cudaMemoryTypeHost) return HKV_ERR_ARG;
  hkv_prefetcher* pf = new (std::nothrow) hkv_prefetcher;
  if (!pf) return HKV_ERR_CAPACITY;
  pf->host = static_cast<const uint8_t*>(host_pool);
  // the kernel-side address of the pinned pool (the same pointer under unified
  // addressing); null when the pool is not mapped, which only disables the gather
  void* hd = nullptr;
  if (cudaHostGetDevicePointer(&hd, const_cast<void*>(host_pool), 0) != cudaSuccess) {
    cudaGetLastError();
    hd = nullptr;
  }
  pf->host_dev = static_cast<const uint8_t*>(hd);
  pf->host_pages = host_pages;
  pf->dev = static_cast<uint8_t*>(dev_pool);
  pf->dev_pages = dev_pages;
  pf->page_bytes = page_bytes;
  pf->bytes.store(0);
  *out = pf;
  return HKV_OK;
}

hkv_status hkv_prefetcher_destroy(hkv_prefetcher* pf) {
  if (!pf) return HKV_ERR_ARG;
  delete pf;
  return HKV_OK;
}

hkv_status hkv_prefetch_submit(hkv_prefetcher* pf, const int32_t* src_pages, const int32_t* dst_slots, int32_t n,
                               hkv_stream_t stream, hkv_event_t done) {
  if (!pf || n < 0 || (n > 0 && (!src_pages || !dst_slots))) return HKV_ERR_ARG;
  for (int i = 0; i < n; ++i) {
    if (src_pages[i] < 0 || src_pages[i] >= pf->host_pages) return HKV_ERR_ARG;
    if (dst_slots[i] < 0 || dst_slots[i] >= pf->dev_pages) return HKV_ERR_ARG;
  }
  int64_t total = 0;
  int i = 0;
  while (i < n) {
    int run = 1;  // coalesce consecutive (src, dst) pairs into one copy
    while (i + run < n && src_pages[i + run] == src_pages[i] + run && dst_slots[i + run] == dst_slots[i] + run) ++run;
    const size_t bytes = (size_t)run * pf->page_bytes;
    const cudaError_t e = cudaMemcpyAsync(pf->dev + (int64_t)dst_slots[i] * pf->page_bytes,
                                          pf->host + (int64_t)src_pages[i] * pf->page_bytes, bytes,
                                          cudaMemcpyHostToDevice, S(stream));
    if (e != cudaSuccess) return cuda_fail(e);
    total += (int64_t)bytes;
    i += run;
  }
  pf->bytes.fetch_add(total);
  if (done) {
    const cudaError_t e = cudaEventRecord(reinterpret_cast<cudaEvent_t>(done), S(stream));
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return HKV_OK;
}

int64_t hkv_prefetch_bytes(const hkv_prefetcher* pf) { return pf ? pf->bytes.load() : -1; }

hkv_status hkv_prefetch_gather(hkv_prefetcher* pf, const int32_t* src_pages, const int32_t* dst_slots, int32_t n,
                               const int64_t* step, int64_t step_mul, int32_t step_add, int32_t ctas,
                               hkv_stream_t stream) {
  if (!pf || n < 0 || (n > 0 && (!src_pages || !dst_slots)) || ctas < 0) return HKV_ERR_ARG;
  if (!pf->host_dev) return HKV_ERR_UNSUPPORTED;
  if (pf->page_bytes % 16 || reinterpret_cast<uintptr_t>(pf->host_dev) % 16 ||
      reinterpret_cast<uintptr_t>(pf->dev) % 16)
    return HKV_ERR_UNSUPPORTED;
  if (n == 0) return HKV_OK;
  const int64_t chunks = (int64_t)n * ((pf->page_bytes / 16 + kGatherThreads * kGatherUnroll - 1) /
                                        (kGatherThreads * kGatherUnroll));
  const int grid = (int)std::min<int64_t>(chunks, ctas > 0 ? ctas : 64);
  page_gather_kernel<<<grid, kGatherThreads, 0, S(stream)>>>(
      reinterpret_cast<const uint4*>(pf->host_dev), reinterpret_cast<uint4*>(pf->dev), src_pages, dst_slots, n,
      pf->page_bytes / 16, pf->host_pages, pf->dev_pages, step, step_mul, step_add);
  const hkv_status rc = launch_status();
  if (rc == HKV_OK) pf->bytes.fetch_add((int64_t)n * pf->page_bytes);
  return rc;
}

hkv_status hkv_graph_copy_nodes(void* graph, int32_t max_nodes, void** nodes, void** dsts, int32_t* n) {
  if (!graph || !n || max_nodes < 0 || (max_nodes > 0 && (!nodes || !dsts))) return HKV_ERR_ARG;
  cudaGraph_t g = static_cast<cudaGraph_t>(graph);
  size_t count = 0;
  cudaError_t e = cudaGraphGetNodes(g, nullptr, &count);
  if (e != cudaSuccess) return cuda_fail(e);
  std::vector<cudaGraphNode_t> all(count);
  if (count && (e = cudaGraphGetNodes(g, all.data(), &count)) != cudaSuccess) return cuda_fail(e);
  int32_t k = 0;
  for (size_t i = 0; i < count; ++i) {
    cudaGraphNodeType t;
    if ((e = cudaGraphNodeGetType(all[i], &t)) != cudaSuccess) return cuda_fail(e);
    if (t != cudaGraphNodeTypeMemcpy) continue;
    cudaMemcpy3DParms prm;
    std::memset(&prm, 0, sizeof(prm));
    if ((e = cudaGraphMemcpyNodeGetParams(all[i], &prm)) != cudaSuccess) return cuda_fail(e);
    if (k < max_nodes) {
      nodes[k] = all[i];
      dsts[k] = static_cast<char*>(prm.dstPtr.ptr) + prm.dstPos.x +
                (prm.dstPos.y + prm.dstPos.z * prm.dstPtr.ysize) * prm.dstPtr.pitch;
    }
    ++k;
  }
  *n = k;
  return k > max_nodes ? HKV_ERR_CAPACITY : HKV_OK;
}

hkv_status hkv_graph_exec_set_copy_srcs(void* graph_exec, int32_t n, void* const* nodes, void* const* dsts,
                                        const void* const* srcs, const int64_t* bytes) {
  if (!graph_exec || n < 0 || (n > 0 && (!nodes || !dsts || !srcs || !bytes))) return HKV_ERR_ARG;
  cudaGraphExec_t x = static_cast<cudaGraphExec_t>(graph_exec);
  for (int32_t i = 0; i < n; ++i) {
    if (!nodes[i] || !dsts[i] || !srcs[i] || bytes[i] <= 0) return HKV_ERR_ARG;
    const cudaError_t e = cudaGraphExecMemcpyNodeSetParams1D(x, static_cast<cudaGraphNode_t>(nodes[i]), dsts[i],
                                                             srcs[i], (size_t)bytes[i], cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return HKV_OK;
}

hkv_status hkv_event_wait(hkv_event_t ev, int64_t timeout_us) {
  if (!ev) return HKV_ERR_ARG;
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    const cudaError_t q = cudaEventQuery(reinterpret_cast<cudaEvent_t>(ev));
    if (q == cudaSuccess) return HKV_OK;
    if (q != cudaErrorNotReady) {
      cudaGetLastError();
      return cuda_fail(q);
    }
    const auto el = std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0);
    if (el.count() >= timeout_us) return HKV_ERR_TIMEOUT;
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

}  // extern "C"
