/*
 * hetero_kv.h — C ABI of libhetero_kv.so, the B200 (sm_100a) INT4 KV-cache hot path.
 *
 * Three parts, each replacing a reference (kldxg123/Hetero-KVCache-Optimizer)
 * interface on the same path:
 *   1. quantise + nibble-pack K/V into an INT4 page pool   (replaces KVCompressor.compress,
 *      src/quantization/kv_compressor.py:50-98, and the tail eviction in
 *      HeteroKVManager._decode_update, src/memory/manager.py:640-664)
 *   2. split-KV GQA decode attention straight from packed INT4 + an fp16/bf16
 *      sink/recent segment, with a log-sum-exp merge     (replaces fused_dequant_attn_decode,
 *      src/quantization/fused_dequant_attn.py:254-331 and its twin
 *      src/quantization/kernels/fused_dequant_attn.py:301-368)
 *   3. DRAM->HBM page prefetch on a side stream with per-page events
 *                                                          (replaces AsyncPrefetcher,
 *      src/policy/prefetcher.py:47-111, and the per-chunk .to(device) swap-in of
 *      HeteroKVManager.swap_in_quantized, src/memory/manager.py:233-263)
 *
 * Conventions
 *  - Every device pointer is caller-owned; nothing on these paths allocates.
 *  - Every launch is stream-ordered on the cudaStream_t passed as `stream`
 *    (NULL = legacy default stream). No call synchronises the device, except the
 *    diagnostic hkv_device_error(), the bounded hkv_event_wait() and the
 *    self-test hkv_selftest_bounded_wait() (its own stream).
 *  - Strides are in ELEMENTS; the last (head-dim) axis must be contiguous.
 *  - Errors are integer statuses; no exception crosses the ABI.
 *  - Kernels never trap: a bounded wait that expires, or a page id outside the
 *    pool, sets a sticky device error word read back by hkv_device_error().
 *
 * Packed INT4 page layout (head_dim D = 128, G = D/group groups per token).
 * A page of P tokens (P a multiple of 128) is P/128 contiguous 128-token blocks,
 * each holding K and V together so that one bulk copy moves a decode tile:
 *     offset 0        K codes [128][64]     u8, two 4-bit codes per byte, in the
 *                                           mma-fragment nibble order documented
 *                                           in oracle/kv_oracle.py (per token)
 *     offset 8192     V codes [64][128]     u8, per token pair; the 16-byte chunk
 *                                           c of pair q is stored at chunk position
 *                                           (c + 2q) mod 8 of the pair's 128 bytes
 *   HKV_FMT_REF metadata:
 *     offset 16384    K scales [128][G]     f32
 *     +   512*G       V scales [128][G]     f32
 *     +  1024*G       K zps    [128][G]     u8
 *     +  1152*G       V zps    [128][G]     u8
 *   HKV_FMT_FP16MIN metadata (f16; V entries of a token pair side by side):
 *     offset 16384    K scales [128][G]
 *     +   256*G       K mins   [128][G]
 *     +   512*G       V scales [64 pairs][G][2]
 *     +   768*G       V mins   [64 pairs][G][2]
 *   => 168 B per token (ref, group 32) or 160 B per token (fp16min, group 32)
 *      for K and V together; hkv_page_bytes() gives the page size.
 */
#ifndef HETERO_KV_H_
#define HETERO_KV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default) /* the library is built with -fvisibility=hidden */
#endif

typedef int hkv_status;
#define HKV_OK 0
#define HKV_ERR_ARG 1          /* bad argument (shape, alignment, null pointer) */
#define HKV_ERR_CUDA 2         /* a CUDA runtime call failed */
#define HKV_ERR_TIMEOUT 3      /* a bounded wait expired */
#define HKV_ERR_UNSUPPORTED 4  /* valid request this build does not implement */
#define HKV_ERR_CAPACITY 5     /* destination too small */
#define HKV_ERR_DEVICE 6       /* a kernel reported an error through the device error word */

#define HKV_DT_F16 0
#define HKV_DT_BF16 1
#define HKV_DT_F32 2

#define HKV_FMT_REF 0      /* fp32 scale, u8 zero-point: bit-exact with KVCompressor */
#define HKV_FMT_FP16MIN 1  /* fp16 scale = (max-min)/15, fp16 zero = min */

#define HKV_ROLE_K 0
#define HKV_ROLE_V 1

/* device error word bits (hkv_device_error) */
#define HKV_DEVERR_TIMEOUT 1u
#define HKV_DEVERR_BAD_PAGE 2u
#define HKV_DEVERR_CAPACITY 4u

typedef void* hkv_stream_t; /* cudaStream_t */
typedef void* hkv_event_t;  /* cudaEvent_t */

/* Packed INT4 body of a KV cache: a pool of pages, page p at
 * pages + p*page_stride. Token t of unit u = b*Hkv + h lives in page
 *   page_table ? page_table[u*max_pages + t/P] : u*max_pages + t/P
 * at slot t % P. A dense per-unit buffer is the special case page_table == NULL. */
typedef struct hkv_int4_store {
  void* pages;               /* device page pool, 16-byte aligned */
  int64_t page_stride;       /* bytes between pages: >= hkv_page_bytes(), multiple of 16 */
  int32_t format;            /* HKV_FMT_* */
  int32_t group;             /* 32, 64 or 128 */
  int32_t page_tokens;       /* P: multiple of 128 */
  int32_t max_pages;         /* pages per unit (row length of page_table) */
  const int32_t* page_table; /* [units][max_pages] int32 on device, or NULL */
  const int32_t* lengths;    /* [B] int32 on device (tokens per sequence), or NULL */
  int32_t len;               /* tokens when lengths == NULL; else an upper bound */
  int32_t num_pages;         /* pages in the pool: a page id outside [0, num_pages) is
                                skipped and flagged HKV_DEVERR_BAD_PAGE; 0 = ids are
                                trusted (only negative ids are caught) */
} hkv_int4_store;

/* Dense fp16/bf16 K/V segment [B][Hkv][capacity][D] (e.g. sink + recent ring). */
typedef struct hkv_dense_kv {
  void* k;
  void* v;
  int32_t dtype;          /* HKV_DT_F16 or HKV_DT_BF16 */
  int32_t capacity;       /* rows allocated per unit */
  int64_t stride_b;       /* elements */
  int64_t stride_h;
  int64_t stride_t;
  const int32_t* lengths; /* [B] int32 on device, or NULL */
  int32_t len;            /* rows when lengths == NULL; else an upper bound */
  int32_t reserved;
} hkv_dense_kv;

/* ---------------------------------------------------------------- misc */
const char* hkv_status_str(hkv_status s);
int hkv_version(void);
/* Reads and optionally clears the sticky device error word (synchronises the device). */
hkv_status hkv_device_error(uint32_t* bits, int clear);
/* cudaError_t value behind the last HKV_ERR_CUDA returned to this host thread
 * (0 if none). No counterpart in the reference (it raises Python exceptions). */
int32_t hkv_last_cuda_error(void);
/* Bytes of one page (K and V) for a format/group/page size; -1 if invalid. */
int64_t hkv_page_bytes(int32_t format, int32_t group, int32_t page_tokens);

/* ---------------------------------------------------------------- 1. quantise
 * Legacy flat quantiser, bit-exact with KVCompressor.compress
 * (src/quantization/kv_compressor.py:66-98): x is a contiguous tensor of n
 * elements (fp16/bf16/fp32), groups of `group` run over the flattened order,
 * the last group is zero-padded. codes: n bytes (one code per byte),
 * scales: ceil(n/group) f32, zps: ceil(n/group) u8. */
hkv_status hkv_quantize_flat(const void* x, int32_t dtype, int64_t n, int32_t group,
                             uint8_t* codes, float* scales, uint8_t* zps, hkv_stream_t stream);

/* Legacy flat dequantiser, KVCompressor.decompress (kv_compressor.py:119-132):
 * out[i] = (codes[i] - zps[i/group]) * scales[i/group], written as out_dtype. */
hkv_status hkv_dequantize_flat(const uint8_t* codes, const float* scales, const uint8_t* zps,
                               int64_t n, int32_t group, void* out, int32_t out_dtype,
                               hkv_stream_t stream);

/* Quantise x[B][H][T][128] (fp16/bf16, strides in elements) into the K or V
 * half (role) of the blocks of `dst`: token t of unit (b,h) is written at body slot
 * (dst_start ? dst_start[b] : start) + t. Per-group min/max, scale and
 * zero-point are computed exactly as KVCompressor.compress does for a
 * [.., 128] tensor (HKV_FMT_REF, bit-exact) or as the fp16min spec says.
 * Replaces the compress() calls in HeteroKVManager._evict_to_dram
 * (src/memory/manager.py:1231-1257). */
hkv_status hkv_quantize_pack(const void* x, int32_t dtype, int32_t B, int32_t H, int32_t T,
                             int32_t D, int64_t stride_b, int64_t stride_h, int64_t stride_t,
                             int32_t role, const hkv_int4_store* dst, const int32_t* dst_start,
                             int32_t start, hkv_stream_t stream);

/* hkv_quantize_pack of a K chunk and its V chunk (same dtype, shape and strides)
 * in one launch: the chunked prefill quantises both per chunk, and at 4,096-token
 * chunks the launch latency, not HBM, bounds two separate calls. */
hkv_status hkv_quantize_pack_kv(const void* k, const void* v, int32_t dtype, int32_t B, int32_t H,
                                int32_t T, int32_t D, int64_t stride_b, int64_t stride_h,
                                int64_t stride_t, const hkv_int4_store* dst,
                                const int32_t* dst_start, int32_t start, hkv_stream_t stream);

/* One decode step of the KV cache state machine of HeteroKVManager._decode_update
 * (src/memory/manager.py:621-664), for K and V in one launch: per sequence b,
 * if the recent ring (rows [sink, capacity) of `dense`) is full, its oldest row
 * is quantised into the INT4 body at body_len[b] (which then advances); the
 * new token is written into the ring. State arrays are [B] int32 on device and
 * are updated in place: dense_len = sink + filled ring rows, ring_head = next
 * ring slot. k_new/v_new: [B][H][128] with strides (elements). */
hkv_status hkv_append_kv(const void* k_new, const void* v_new, int32_t dtype, int32_t B,
                         int32_t H, int32_t D, int64_t stride_b, int64_t stride_h,
                         const hkv_dense_kv* dense, int32_t sink, int32_t* dense_len,
                         int32_t* ring_head, const hkv_int4_store* body, int32_t* body_len,
                         hkv_stream_t stream);

/* Dequantise tokens [t0, t0+T) of the K or V half (role) of every unit to a dense
 * [B][H][T][128] tensor (out_dtype, contiguous). Serves the BF16-returning
 * AsyncPrefetcher.fetch_if_ready contract (src/policy/prefetcher.py:81-84). */
hkv_status hkv_dequantize_pack(const hkv_int4_store* src, int32_t role, int32_t B, int32_t H,
                               int32_t t0, int32_t T, void* out, int32_t out_dtype,
                               hkv_stream_t stream);

/* Convert the reference's unpacked representation (codes [B][H][S][128] u8
 * one code per byte, scales f32 and zps u8 flat over groups of `group`) into
 * tokens [0, S) of the K or V half (role) of an HKV_FMT_REF store. Used when the legacy
 * fused_dequant_attn_decode signature is called with KVCompressor outputs. */
hkv_status hkv_repack_ref(const uint8_t* codes, const float* scales, const uint8_t* zps,
                          int32_t B, int32_t H, int32_t S, int32_t group, int32_t role,
                          const hkv_int4_store* dst, hkv_stream_t stream);

/* ---------------------------------------------------------------- 2. decode attention
 * One persistent launch: the (sequence, KV head) units' tile lists (128-token
 * INT4 tiles, 32-token dense tiles) are cut into equal-byte ranges, one per CTA
 * (`ctas` <= 0: one per SM); the last CTA to finish a unit merges its partials.
 * The len fields of body/dense size the schedule; device lengths may exceed them
 * (tokens are never dropped) at the cost of balance.
 *
 * Workspace: a 256 KiB region of per-unit int32 merge counters (B*Hkv <= 65536)
 * followed by the split partials. The counter region must be zero-filled before
 * the first call; every completed call leaves it at zero again, so one
 * workspace serves calls of any shape. Calls that overlap on the GPU must use
 * different workspaces. A call whose bounded wait expired (hkv_device_error
 * reports HKV_DEVERR_TIMEOUT) may leave counters non-zero: zero the counter
 * region again before the workspace's next use. */
size_t hkv_decode_workspace_bytes(const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B,
                                  int32_t Hq, int32_t Hkv, int32_t D, int32_t ctas);

/* The grid and the partial slots per unit a call with these arguments uses. */
hkv_status hkv_decode_plan(const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t B,
                           int32_t Hq, int32_t Hkv, int32_t ctas, int32_t* grid,
                           int32_t* slots_per_unit);

/* out[b][hq][:] = softmax(q[b][hq] . K^T * sm_scale) V over the union of the
 * INT4 body and the dense segment of KV head hq / (Hq/Hkv) (G = Hq/Hkv <= 8).
 * q: [B][Hq][128] fp16/bf16; out: [B][Hq][128] in out_dtype (f32/f16/bf16).
 * Either body or dense may be NULL.
 * Precision: the INT4 tiles multiply on the f16 tensor cores with fp32
 * accumulation, so a bf16 query is rounded to f16 for them (|q| must stay below
 * the f16 range, 65504, or its products overflow to inf); the dense tiles use
 * the dense segment's dtype (a query is rounded to it: use bf16 queries with a
 * bf16 cache) and P is rounded to that dtype for P.V. The tests hold
 * max |out - ref| <= 2e-3 * ||ref||_2 per row against fp32 attention. */
hkv_status hkv_decode_attn(const void* q, int32_t q_dtype, int64_t q_stride_b,
                           int64_t q_stride_h, const hkv_int4_store* body,
                           const hkv_dense_kv* dense, int32_t B, int32_t Hq, int32_t Hkv,
                           int32_t D, float sm_scale, int32_t ctas, void* workspace,
                           size_t workspace_bytes, void* out, int32_t out_dtype,
                           int64_t out_stride_b, int64_t out_stride_h, hkv_stream_t stream);

/* One whole decode step of a layer in ONE launch: hkv_append_kv followed by
 * hkv_decode_attn (replaces HeteroKVManager._decode_update,
 * src/memory/manager.py:588-664, plus the attention over the updated cache,
 * fused_dequant_attn_decode, src/quantization/fused_dequant_attn.py:254-331).
 * The new token k_new/v_new [B][Hkv][128] (the dense segment's dtype, strides in
 * elements, 16-byte aligned rows) enters the cache exactly as hkv_append_kv
 * would put it there (same codes, same ring row, same state transition of
 * dense_len / ring_head / body_len), and `out` is the attention of q over the
 * cache after the append. The attention streams the cache as it was before the
 * step (the ring row the step overwrites is left out) and folds the evicted
 * token (as quantised) and the new token in as one extra partial per unit.
 * body->lengths must be body_len and dense->lengths dense_len (device arrays,
 * updated in place once every CTA has read them). Workspace as
 * hkv_decode_attn (same size); B*Hkv < 65536.
 * flags: 0, or HKV_APPEND_EARLY: the caller guarantees that the kernel
 * launched on `stream` just before this call does not write this cache (body
 * pages, dense rows, the three state arrays); e.g. the layers of a
 * multi-layer step, each layer's cache touched once per step. The launch then
 * reads its cache and streams the first tiles while that kernel finishes
 * (programmatic dependent launch), and only the query, the new token and its
 * own writes wait for it. Without the guarantee pass 0. */
#define HKV_APPEND_EARLY 1
hkv_status hkv_decode_append(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                             const void* k_new, const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
                             const hkv_int4_store* body, const hkv_dense_kv* dense, int32_t sink,
                             int32_t* dense_len, int32_t* ring_head, int32_t* body_len, int32_t B, int32_t Hq,
                             int32_t Hkv, int32_t D, float sm_scale, int32_t ctas, void* workspace,
                             size_t workspace_bytes, void* out, int32_t out_dtype, int64_t out_stride_b,
                             int64_t out_stride_h, int32_t flags, hkv_stream_t stream);

/* hkv_decode_attn, plus where the attention mass fell, for the prefetch policy
 * (the reference aggregates accumulated token scores into block means on the
 * host side of a sync, oracle_triton.py:16-79 and manager.py:931-1056).
 * tile_stats [B*Hkv][stat_tiles][4][8][2] f32 (16-byte aligned) receives, for
 * every INT4 body tile k < stat_tiles (128 tokens) of every (sequence, KV head)
 * unit, per consumer warp and query head of the unit, the sum of the warp's
 * softmax numerators and its running max (base-2 logits); unit_ml
 * [B*Hkv][8][2] f32 the unit's final (max, sum) per head. hkv_tile_scores turns
 * them into attention mass per tile. */
hkv_status hkv_decode_attn_scored(const void* q, int32_t q_dtype, int64_t q_stride_b,
                                  int64_t q_stride_h, const hkv_int4_store* body,
                                  const hkv_dense_kv* dense, int32_t B, int32_t Hq, int32_t Hkv,
                                  int32_t D, float sm_scale, int32_t ctas, void* workspace,
                                  size_t workspace_bytes, void* out, int32_t out_dtype,
                                  int64_t out_stride_b, int64_t out_stride_h, float* tile_stats,
                                  int32_t stat_tiles, float* unit_ml, hkv_stream_t stream);

/* mass [B*Hkv][stat_tiles] f32: for each unit, the mean over its G query heads
 * of the softmax probability on tile k's 128 body tokens (0 past the body
 * length, read from body->lengths or body->len), from the buffers of
 * hkv_decode_attn_scored over the same store. Stream-ordered, no host sync. */
hkv_status hkv_tile_scores(const float* tile_stats, const float* unit_ml, const hkv_int4_store* body,
                           int32_t B, int32_t Hkv, int32_t G, int32_t stat_tiles, float* mass,
                           hkv_stream_t stream);

/* Multi-query attention over the INT4 body (chunked prefill against offloaded
 * context; replaces fused_dequant_attn_forward,
 * src/quantization/fused_dequant_attn.py:158-247 and its twin
 * kernels/fused_dequant_attn.py:371-435): out[b][hq][s] = softmax(q[b][hq][s] .
 * K^T * sm_scale) V over the body tokens of unit (b, hq / (Hq/Hkv)); with
 * causal != 0 query s sees only tokens t <= len - Sq + s (the queries are the
 * last Sq positions), and a query that sees none gets zeros. q and out
 * [B][Hq][Sq][128] with element strides; q f16/bf16 (computed in f16), out
 * f16/bf16/f32. lse (optional, [B][Hq][Sq] f32) receives ln sum_t
 * exp(sm_scale q.k_t) (-inf for an empty row), for merging with attention over
 * other segments. Runs on the tcgen05 tensor cores: 128 (query, head) rows of
 * one KV head per CTA, the body dequantised tile by tile into shared memory.
 * splits: 0 = choose how many CTAs share each query tile's body (to fill the
 * SMs' waves), n > 0 = use n; more than one needs a workspace of
 * hkv_prefill_workspace_bytes (16-byte aligned; NULL or too small = fewer or
 * no splits) for the partials, merged by a second launch on `stream`. */
size_t hkv_prefill_workspace_bytes(const hkv_int4_store* body, int32_t B, int32_t Hq, int32_t Hkv,
                                   int32_t Sq, int32_t D, int32_t splits);
hkv_status hkv_prefill_attn(const void* q, int32_t q_dtype, int64_t q_stride_b, int64_t q_stride_h,
                            int64_t q_stride_s, const hkv_int4_store* body, int32_t B, int32_t Hq,
                            int32_t Hkv, int32_t Sq, int32_t D, float sm_scale, int32_t causal, void* out,
                            int32_t out_dtype, int64_t out_stride_b, int64_t out_stride_h,
                            int64_t out_stride_s, float* lse, int32_t splits, void* workspace,
                            size_t workspace_bytes, hkv_stream_t stream);

/* Same attention, but stops at one un-normalised partial per (b, hq):
 * part_o [B][Hq][128] f32 = sum_t 2^(x_t - m) v_t, part_ml [B][Hq][2] f32 =
 * (m, l) with x = score * sm_scale * log2(e) and l = sum_t 2^(x_t - m).
 * For sequence-split attention across GPUs (partials all-gathered, then merged
 * with hkv_lse_merge). */
hkv_status hkv_decode_attn_partial(const void* q, int32_t q_dtype, int64_t q_stride_b,
                                   int64_t q_stride_h, const hkv_int4_store* body,
                                   const hkv_dense_kv* dense, int32_t B, int32_t Hq,
                                   int32_t Hkv, int32_t D, float sm_scale, int32_t ctas,
                                   void* workspace, size_t workspace_bytes, float* part_o,
                                   float* part_ml, hkv_stream_t stream);

/* Largest workspace hkv_decode_attn_static can serve from its built-in scratch. */
#define HKV_STATIC_SCRATCH_BYTES (8u << 20)

/* hkv_decode_attn without a caller workspace: the merge counters and partials
 * live in one library-owned device array of HKV_STATIC_SCRATCH_BYTES per GPU,
 * so the call allocates nothing. For callers that have no device allocator to
 * hand over a workspace (a plain C or FFI host without a tensor library), or
 * that must not allocate inside a decode step. No counterpart in the reference
 * (its Python path allocates freely).
 * - The first call on a device looks up the array's address (and sets the
 *   kernel's shared-memory attribute); make that first call before any stream
 *   capture. The address is looked up again when the device's current context
 *   changes (after a cudaDeviceReset the module, and the array, are new); a
 *   call that would do so inside a capture fails with HKV_ERR_CUDA.
 * - Every call on a device shares the one array: calls whose kernels may
 *   overlap (different streams, or threads without ordering) race on it.
 *   Each call clears the merge counters it uses on `stream` before its kernel.
 * - Argument errors, and a request whose workspace (hkv_decode_workspace_bytes)
 *   exceeds HKV_STATIC_SCRATCH_BYTES (HKV_ERR_CAPACITY), return before anything
 *   is queued on `stream`. */
hkv_status hkv_decode_attn_static(const void* q, int32_t q_dtype, int64_t q_stride_b,
                                  int64_t q_stride_h, const hkv_int4_store* body,
                                  const hkv_dense_kv* dense, int32_t B, int32_t Hq, int32_t Hkv,
                                  int32_t D, float sm_scale, int32_t ctas, void* out,
                                  int32_t out_dtype, int64_t out_stride_b, int64_t out_stride_h,
                                  hkv_stream_t stream);

/* Merge n partial sets laid out [n][B][Hq][128] / [n][B][Hq][2] (as produced by
 * hkv_decode_attn_partial) into out [B][Hq][128] (out_dtype, strides in elements). */
hkv_status hkv_lse_merge(const float* part_o, const float* part_ml, int32_t n, int32_t B,
                         int32_t Hq, int32_t D, void* out, int32_t out_dtype,
                         int64_t out_stride_b, int64_t out_stride_h, hkv_stream_t stream);
/* hkv_lse_merge over partial sets spaced split_o / split_ml floats apart (partial
 * set s of row (b, hq) at part_o + s*split_o + (b*Hq + hq)*128 and part_ml +
 * s*split_ml + (b*Hq + hq)*2): merges straight from an all-gather buffer that
 * holds every rank's o and (m, l) side by side, with no copy. */
hkv_status hkv_lse_merge_strided(const float* part_o, const float* part_ml, int32_t n, int64_t split_o,
                                 int64_t split_ml, int32_t B, int32_t Hq, int32_t D, void* out,
                                 int32_t out_dtype, int64_t out_stride_b, int64_t out_stride_h,
                                 hkv_stream_t stream);

/* ---------------------------------------------------------------- 3. prefetch
 * A prefetcher moves whole pages from a caller-owned pinned host pool to a
 * caller-owned device pool, one cudaMemcpyAsync per run of consecutive page
 * ids, on a caller-given side stream, and records an event when the batch has
 * landed. Replaces AsyncPrefetcher (src/policy/prefetcher.py:21-122). */
typedef struct hkv_prefetcher hkv_prefetcher;

hkv_status hkv_prefetcher_create(const void* host_pool, int64_t host_pages, void* dev_pool,
                                 int64_t dev_pages, int64_t page_bytes, hkv_prefetcher** out);
hkv_status hkv_prefetcher_destroy(hkv_prefetcher* pf);
/* Copy host pages src_pages[i] -> device slots dst_slots[i] (host int32 arrays)
 * on `stream`, then record `done` (may be NULL) on it. */
hkv_status hkv_prefetch_submit(hkv_prefetcher* pf, const int32_t* src_pages,
                               const int32_t* dst_slots, int32_t n, hkv_stream_t stream,
                               hkv_event_t done);
/* Bytes submitted so far (for H2D GB/s accounting). */
int64_t hkv_prefetch_bytes(const hkv_prefetcher* pf);
/* Zero-copy gather: one kernel on `stream` reads n host pages over the host
 * link (the pinned pool mapped into the device address space) and writes them
 * to device slots. src_pages / dst_slots are DEVICE int32 arrays, so the page
 * set can be chosen on the device and the launch captured in a CUDA graph;
 * host page of entry k = (src_pages[k] + (*step + step_add) * step_mul) mod
 * host_pages when `step` (a device int64 counter) is given, else src_pages[k].
 * ctas = 0: 64 CTAs of 128 threads (a small grid whose CTAs fit beside a
 * persistent decode kernel's).
 * Ids outside the pools are skipped and set HKV_DEVERR_BAD_PAGE.
 * HKV_ERR_UNSUPPORTED when the host pool is not mapped. Replaces the six
 * per-chunk copies of AsyncPrefetcher.submit_prefetch_task
 * (src/policy/prefetcher.py:74-79) for scattered page sets. */
hkv_status hkv_prefetch_gather(hkv_prefetcher* pf, const int32_t* src_pages, const int32_t* dst_slots,
                               int32_t n, const int64_t* step, int64_t step_mul, int32_t step_add,
                               int32_t ctas, hkv_stream_t stream);
/* Page copies inside a CUDA graph whose host source moves between replays (a
 * sliding window over a host arena): hkv_graph_copy_nodes lists the memcpy
 * nodes of a captured graph (a cudaGraph_t) and their destination addresses
 * (at most max_nodes; *n = how many exist, HKV_ERR_CAPACITY if more), and
 * hkv_graph_exec_set_copy_srcs points n of those nodes of the instantiated
 * graph (a cudaGraphExec_t) at new host sources (host -> device, bytes[i]
 * each) for every later launch; a launch already queued keeps its copies. The
 * copies stay on the copy engines at full host-link bandwidth, and a step is
 * one graph launch. */
hkv_status hkv_graph_copy_nodes(void* graph, int32_t max_nodes, void** nodes, void** dsts, int32_t* n);
hkv_status hkv_graph_exec_set_copy_srcs(void* graph_exec, int32_t n, void* const* nodes, void* const* dsts,
                                        const void* const* srcs, const int64_t* bytes);
/* Host-side bounded wait: polls the event until it completes or timeout_us
 * elapses (HKV_ERR_TIMEOUT). Never blocks forever. */
hkv_status hkv_event_wait(hkv_event_t ev, int64_t timeout_us);

/* ---------------------------------------------------------------- 4. legacy scores, self-test
 * Pre-softmax scores of one query row against n_keys keys in the reference's
 * unpacked INT4 layout: out[s] = sum_d q[d] * (codes[s*D+d] - zps[g]) * scales[g],
 * g = (s*D+d) / group, fp32 (replaces the score-only fused_dequant_attention,
 * src/quantization/fused_dequant_attn.py:338-381, and its twin
 * kernels/fused_dequant_attn.py:283-298). q: D elements (f16/bf16/f32). */
hkv_status hkv_qk_scores_flat(const void* q, int32_t q_dtype, const uint8_t* codes, const float* scales,
                              const uint8_t* zps, int64_t n_keys, int32_t D, int32_t group, float* out,
                              hkv_stream_t stream);

/* Failure-detection self-test of the bounded device wait the kernels use: a
 * one-warp kernel waits on an mbarrier phase with a limit of limit_ns
 * (0 < limit_ns <= 1e9). With arrive != 0 the phase completes and the call
 * returns HKV_OK; with arrive == 0 nothing completes it, the wait gives up,
 * sets HKV_DEVERR_TIMEOUT in the device error word and the call returns
 * HKV_ERR_DEVICE, the context still usable. Synchronises `stream`. No
 * counterpart in the reference (it has no device-side waits). */
hkv_status hkv_selftest_bounded_wait(int64_t limit_ns, int32_t arrive, hkv_stream_t stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* HETERO_KV_H_ */
