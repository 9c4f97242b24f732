/*
 * rkv.h -- C ABI of the B200 (sm_100a) implementation of RocketKV's two
 * kernels: stage-1 prefill eviction and stage-2 hybrid sparse decode.
 *
 * Every entry point is extern "C", takes plain pointers and sizes, and
 * returns an rkv_status (0 = success).  None of them aborts the process.
 * "stream" arguments are cudaStream_t values passed as void* (NULL = the
 * legacy default stream), so this header needs no CUDA include.
 *
 * Each entry point names the reference interface it replaces
 * (Rishit2000/RocketKV-cpp, rocket.h / rocket.cpp).  The reference is a CPU
 * C++ library with no FFI of its own; rocket.h (next to this file) keeps its
 * C++ API unchanged and is implemented on top of this ABI.
 *
 * Layouts (row-major, as the reference reads them):
 *   stage 1: Q [num_heads][len_q][dim_head], K [num_heads_kv][len_k][dim_head]
 *   stage 2: Q [num_heads][dim_head],        K, V [num_heads_kv][len_k][dim_head]
 * Batched device entry points take `batch` such items, `*_item_stride`
 * bytes apart.  Element types: rkv_dtype.  q8_0 rows are dim_head/32 blocks
 * of {fp16 scale; int8 q[32]} (34 bytes), the ggml block_q8_0 layout.
 *
 * Device pointers must be 16-byte aligned, and so must every item stride and
 * (for stage 2) every K/V row.
 */
#ifndef RKV_H
#define RKV_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RKV_ABI_VERSION 1

typedef enum rkv_status {
    RKV_OK = 0,
    RKV_ERR_INVALID_ARG = 1,    /* bad size, pointer, alignment or config      */
    RKV_ERR_UNSUPPORTED = 2,    /* valid for the reference, not built here      */
    RKV_ERR_CUDA = 3,           /* a CUDA runtime call failed                   */
    RKV_ERR_WORKSPACE = 4,      /* workspace missing or too small               */
    RKV_ERR_DEVICE_TIMEOUT = 5, /* a bounded in-kernel wait ran out             */
    RKV_ERR_NO_DEVICE = 6       /* no CUDA device / library built without one   */
} rkv_status;

typedef enum rkv_dtype {
    RKV_F32 = 0,
    RKV_BF16 = 1,
    RKV_Q8_0 = 2,
    RKV_F16 = 3   /* source type of rkv_capture_rows only */
} rkv_dtype;

/* Stage-1 scoring engine. */
typedef enum rkv_evict_engine {
    RKV_EVICT_AUTO = 0,   /* the fastest engine built for the inputs          */
    RKV_EVICT_SIMT = 1,   /* fp32 CUDA-core scoring                            */
    RKV_EVICT_TENSOR = 2, /* tcgen05 tensor-core scoring: fp32 K/Q as three
                             TF32 products per step, bf16 directly, q8_0 as
                             exact int8 block products (kind::i8, one int32
                             accumulator per 32-value block, the fp16 scales
                             applied exactly afterwards; q8_0 K tiles that are
                             not 16-byte aligned are dequantised to fp32 and
                             run as three TF32 products).  The persistent
                             kernel (one CTA per SM, K tiles staged by bulk or
                             tensor copies, window queries resident) takes
                             G * window <= 128 with fp32/bf16 rows 16-byte
                             aligned and a multiple of 32 bytes, or q8_0 at
                             dim_head 128; other fp32/bf16 shapes with such
                             rows run the per-tile kernel; anything else is
                             RKV_ERR_UNSUPPORTED.  AUTO takes it whenever it
                             applies                                         */
    RKV_EVICT_TENSOR_TILES = 3 /* the per-tile tcgen05 kernel only (one CTA
                             per 128-key tile; fp32 and bf16), kept as the
                             fallback of RKV_EVICT_TENSOR and for
                             comparison                                      */
} rkv_evict_engine;

/* Field-for-field image of RocketConfig (rocket.h:18-34). */
typedef struct rkv_config {
    int num_heads;
    int num_heads_kv;
    int dim_head;
    int window_size;        /* rocket.h:25, default 32 */
    int kernel_size;        /* rocket.h:26, default 63 */
    int prompt_budget;
    int topk_decode;
    int chunk_size;
    int r_dim;
    float compression_ratio;
} rkv_config;

/* Field-for-field image of RocketBudgetParams (rocket.h:5-15). */
typedef struct rkv_budget_params {
    int token_budget;
    int sequence_length;
    int max_new_tokens;
    int capacity_budget;
    int prompt_budget;
    int chunk_size;
    int r;
    int k;
    float compression_ratio;
} rkv_budget_params;

/* ---- library ------------------------------------------------------------ */
int rkv_abi_version(void);
const char* rkv_status_string(int status);

/* Fills cfg with the rocket.h defaults (window_size 32, kernel_size 63) and
 * zeros elsewhere, as `RocketConfig cfg{};` does. */
void rkv_config_init(rkv_config* cfg);

/* ---- budget derivation ----------------------------------------------------
 * Replaces compute_rocket_params (rocket.h:36-41, rocket.cpp:14-59).
 * Host arithmetic only; no device is touched. */
int rkv_compute_params(int token_budget, int sequence_length, int max_new_tokens,
                       int head_dim, int window_size, rkv_budget_params* out);

/* ---- stage 1: prefill eviction -------------------------------------------
 * Replaces compute_prefill_eviction (rocket.h:43-46, rocket.cpp:61-169).
 * Output: ascending kept token indices, ONE set shared by all KV heads (the
 * pooled scores are summed over KV heads, rocket.cpp:142-148).  Score ties
 * go to the lower token index. */

/* Number of ints one item's kept list can need (the kept_stride minimum). */
int rkv_evict_max_kept(const rkv_config* cfg, int len_q, int len_k);

/* Workspace bytes rkv_evict needs for `batch` items. */
int rkv_evict_workspace_size(const rkv_config* cfg, int dtype, int len_q, int len_k,
                             int batch, size_t* bytes);

/* Device-resident, batched stage 1.  kept: [batch][kept_stride] ints,
 * n_kept: [batch] ints, both device memory.  Asynchronous on `stream`. */
int rkv_evict(const void* Q, const void* K, int dtype, int len_q, int len_k, int batch,
              long long q_item_stride, long long k_item_stride, const rkv_config* cfg,
              int* kept, int kept_stride, int* n_kept,
              void* workspace, size_t workspace_bytes, int engine, void* stream);

/* Head-sharded stage 1, part 1 (rocket.cpp:82-130 for KV heads
 * [head_begin, head_begin+head_count)): pooled scores
 * pooled[batch][head_count][len_k - min(window_size, len_q)] (device). */
int rkv_evict_pool_heads(const void* Q, const void* K, int dtype, int len_q, int len_k,
                         int batch, long long q_item_stride, long long k_item_stride,
                         const rkv_config* cfg, int head_begin, int head_count,
                         float* pooled, void* workspace, size_t workspace_bytes,
                         int engine, void* stream);

/* Head-sharded stage 1, part 2 (rocket.cpp:132-168): sums all num_heads_kv
 * pooled rows in head order 0..HK-1 (pooled[batch][HK][nk], device) and
 * selects.  Bit-identical to rkv_evict on the same pooled rows. */
int rkv_evict_select_pooled(const float* pooled, int len_q, int len_k, int batch,
                            const rkv_config* cfg, int* kept, int kept_stride, int* n_kept,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Capture side (the device analogue of the reference runner's eval callback,
 * runner.cpp:25-92, which copies each micro-batch's post-RoPE Q or K tensor
 * of the last layer to the host, converts it to fp32 and scatters it into
 * [heads][prompt tokens][dim_head]).  Scatters one micro-batch of n_tokens
 * rows as the producing attention left them -- element (t, h, d) at
 * src + t * token_stride + h * head_stride + d * element size, strides in
 * bytes, src_dtype RKV_F32, RKV_F16 or RKV_BF16 -- into item `item` of dst,
 * laid out [n_heads][dst_tokens][dim_head] in dst_dtype (RKV_F32 from any
 * source, exactly; RKV_BF16 from a BF16 source).  Row t of the micro-batch is
 * global token token_offset + t and lands in dst row
 * token_offset + t - dst_first; tokens outside [dst_first, dst_first +
 * dst_tokens) are skipped (for Q, dst_first = prompt length - window keeps
 * only the window rows stage 1 reads).  Items (layers) are dst_item_stride
 * bytes apart, so every layer can be captured and scored in one batched
 * rkv_evict call.  Device pointers; asynchronous on `stream`; no host copy. */
int rkv_capture_rows(const void* src, int src_dtype, int n_tokens, int n_heads, int dim_head,
                     long long token_stride, long long head_stride, int token_offset, void* dst,
                     int dst_dtype, int dst_first, int dst_tokens, long long dst_item_stride, int item,
                     void* stream);

/* Host-buffer stage 1, the rocket.h drop-in path: fp32 host Q and K as
 * compute_prefill_eviction takes them; copies in, runs on the current
 * device, copies the kept indices back (kept_out holds kept_capacity ints).
 * Synchronous. */
int rkv_prefill_eviction_host(const float* Q, const float* K, int len_q, int len_k,
                              const rkv_config* cfg, int* kept_out, int kept_capacity,
                              int* n_kept);

/* ---- stage 2: hybrid sparse decode ----------------------------------------
 * Replaces compute_hybrid_sparse_decode (rocket.h:48-50, rocket.cpp:171-382).
 * recent_window = 0 is the reference behaviour.  recent_window = w > 0 runs
 * the reference selection over the first len_k - w tokens and always attends
 * the last w tokens as well.  Selected indices (ascending) are reported per
 * KV head; the reference computes them but does not return them. */

/* Selected tokens per KV head: min(topk_decode, len_k - w) + w (w clamped). */
int rkv_hsa_sel_capacity(const rkv_config* cfg, int len_k, int recent_window);

int rkv_hsa_workspace_size(const rkv_config* cfg, int len_k, int recent_window,
                           int batch, int head_count, size_t* bytes);

/* Device-resident, batched stage 2 for KV heads [head_begin, head_begin+head_count).
 * O: [batch][num_heads][dim_head] fp32 (only the query heads of the listed KV
 * heads are written); sel: nullable [batch][head_count][sel_stride] ints;
 * n_sel: nullable [batch][head_count] ints.  dtype: RKV_F32 or RKV_BF16. */
int rkv_hsa_decode(const void* Q, const void* K, const void* V, int dtype, int len_k,
                   int recent_window, int batch, long long q_item_stride,
                   long long kv_item_stride, const rkv_config* cfg, int head_begin,
                   int head_count, float* O, int* sel, int sel_stride, int* n_sel,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Host-buffer stage 2, the rocket.h drop-in path: fp32 host Q [H][D] and
 * K, V [HK][len_k][D]; O receives [H][D] (zeros where the reference leaves
 * zeros).  Synchronous. */
int rkv_hybrid_sparse_decode_host(const float* Q, const float* K, const float* V,
                                  int len_k, const rkv_config* cfg, float* O);

/* Host-buffer stage 2, general form (any dtype, batch, recent window): the
 * inputs are host buffers laid out as for rkv_hsa_decode; copies in, runs,
 * copies O (and sel/n_sel when non-NULL) back.  Synchronous.  When V is
 * pinned host memory mapped into the device's address space (cudaHostAlloc,
 * or cudaHostRegister with mapping), V is not copied: the attention reads the
 * selected rows in place, so only those cross the bus. */
int rkv_hsa_decode_host_ex(const void* Q, const void* K, const void* V, int dtype,
                           int len_k, int recent_window, int batch,
                           long long q_item_stride, long long kv_item_stride,
                           const rkv_config* cfg, float* O, int* sel, int sel_stride,
                           int* n_sel);

/* ---- stage 2 with persistent page summaries --------------------------------
 * The page scoring of stage 2 (rocket.cpp:252-289) needs, per page of C
 * tokens of the compressed cache and per selected dimension, the max (or, for
 * a negative query sign, the min) of K over the page.  A cache that does not
 * change between decode steps (the compressed part; new tokens go to the
 * recent window) can keep these extrema as state, so that each step reads
 * only the selected dimensions' sign-chosen extrema instead of every K row:
 * 27.7 % of the K bytes at the headline geometry (C 2, r 71 of 128).  The
 * selected tokens and O are the same as rkv_hsa_decode's, bit for bit.
 *
 * rkv_hsa_summary_size: bytes of the summaries of `batch` items (every KV
 * head) for (cfg, dtype, len_k, recent_window).
 * rkv_hsa_build_summary: writes them from K (the layout rkv_hsa_decode takes;
 * all num_heads_kv heads of each item); summary: device memory, 16-byte
 * aligned, items back to back.  Asynchronous on `stream`.  Rebuild after the
 * compressed part of K changes.
 * rkv_hsa_decode_summary: rkv_hsa_decode with the page scoring read from the
 * summaries built for the same cfg, dtype, len_k and recent_window (the K
 * rows are still read for the selected tokens and the window). */
int rkv_hsa_summary_size(const rkv_config* cfg, int dtype, int len_k, int recent_window, int batch,
                         size_t* bytes);
int rkv_hsa_build_summary(const void* K, int dtype, int len_k, int recent_window, int batch,
                          long long kv_item_stride, const rkv_config* cfg, void* summary, void* stream);
int rkv_hsa_decode_summary(const void* Q, const void* K, const void* V, const void* summary, int dtype,
                           int len_k, int recent_window, int batch, long long q_item_stride,
                           long long kv_item_stride, const rkv_config* cfg, int head_begin, int head_count,
                           float* O, int* sel, int sel_stride, int* n_sel, void* workspace,
                           size_t workspace_bytes, void* stream);

/* No-allocation stage 2.  This entry point has no counterpart in the
 * reference; it exists for callers that cannot allocate device memory (an
 * inference server or plugin host whose allocator owns the device heap, or a
 * hot loop that cannot take cudaMalloc's implicit synchronisation).  Same
 * arguments and results as rkv_hsa_decode, without the workspace: the scratch
 * is a fixed 4 MiB array of device memory inside the library, present on
 * every GPU that loads it until the process exits.  A call whose
 * rkv_hsa_workspace_size exceeds 4 MiB returns RKV_ERR_WORKSPACE and launches
 * nothing.  No call allocates.  The first call on each device looks up that
 * device's copy of the array (cudaGetSymbolAddress); make it before any
 * stream capture.  The address is remembered with the id of the CUDA context
 * it belongs to, so the first call after the device's context is reset
 * (cudaDeviceReset) looks it up again and is likewise a set-up call.  All
 * calls share the one array, so calls that overlap on the GPU (other streams,
 * other host threads) race: serialise them. */
int rkv_hsa_decode_noalloc(const void* Q, const void* K, const void* V, int dtype, int len_k,
                           int recent_window, int batch, long long q_item_stride,
                           long long kv_item_stride, const rkv_config* cfg, int head_begin,
                           int head_count, float* O, int* sel, int sel_stride, int* n_sel,
                           void* stream);

/* Status of rkv_hsa_decode_noalloc calls (no counterpart in the reference):
 * the no-allocation entry point has no workspace for rkv_workspace_status to
 * read, so this synchronises `stream`, reads the error word of the current
 * device's fixed scratch (RKV_ERR_DEVICE_TIMEOUT when a bounded in-kernel
 * wait of a call on that device ran out, with O and sel then incomplete),
 * clears it and returns it (RKV_OK otherwise).  Allocates nothing. */
int rkv_hsa_decode_noalloc_status(void* stream);

/* ---- KV-cache compaction ---------------------------------------------------
 * Applies stage 1's kept indices to the KV cache on the device: for every
 * item (layer or sequence) and KV head, row kept[i] of K (and of V) becomes
 * row i, for i < min(n_kept[item], out_len).  Replaces the reference
 * runner's removal of the evicted ranges from the model's KV cache
 * (runner.cpp:246-269, llama_memory_seq_rm per run of evicted positions).
 * K, V: [batch][num_heads_kv][len_k] rows of `dtype` (fp32, bf16 or q8_0
 * rows of head_dim values) at kv_item_stride bytes per item; V may be NULL
 * (then V_out must be NULL too).  kept, n_kept: device int arrays
 * [batch][kept_stride] and [batch], as rkv_evict writes them (ascending
 * indices; an index outside [0, len_k) is skipped).  Outputs: K_out, V_out
 * [batch][num_heads_kv][out_len] rows at out_item_stride bytes per item,
 * rows from n_kept on left as they are.  In place when K_out == K (and
 * V_out == V): then out_len must equal len_k and the strides must match, and
 * the kept lists must be strictly ascending (as rkv_evict writes them); K and
 * V must not overlap.  The order is not checked: in place, a list that is not
 * strictly ascending gives undefined rows (a row may be read after it was
 * overwritten), though every access stays inside the cache.  Out of place the
 * output must not overlap the input and any order works.  Asynchronous on
 * `stream`; allocates nothing. */
int rkv_compact_kv(const void* K, const void* V, int dtype, int head_dim, int num_heads_kv,
                   int len_k, int batch, long long kv_item_stride, const int* kept,
                   const int* n_kept, int kept_stride, void* K_out, void* V_out, int out_len,
                   long long out_item_stride, void* stream);

/* Stage 1 and the KV-cache compaction in one call: rkv_evict on Q and the
 * cache's own K rows, then rkv_compact_kv of K (and V) with the kept lists
 * just written, so evicted rows are never moved (the reference runner scores
 * and then removes the evicted ranges, runner.cpp:241-269).  The compaction
 * is launched as a programmatic dependent of the selection kernel: its grid
 * is scheduled while the selection still runs and waits in the kernel for
 * the kept lists.  Arguments as rkv_evict (K's item stride is kv_item_stride)
 * and rkv_compact_kv (V nullable; in place when K_out == K, which needs
 * out_len == len_k).  Asynchronous on `stream`; allocates nothing. */
int rkv_evict_compact(const void* Q, const void* K, const void* V, int dtype, int len_q, int len_k, int batch,
                      long long q_item_stride, long long kv_item_stride, const rkv_config* cfg,
                      int* kept, int kept_stride, int* n_kept, void* K_out, void* V_out, int out_len,
                      long long out_item_stride, void* workspace, size_t workspace_bytes, int engine,
                      void* stream);

/* ---- errors raised inside kernels ----------------------------------------
 * Kernels record a failed bounded wait in the workspace.  This synchronises
 * `stream`, returns RKV_OK or the recorded status, and clears it. */
int rkv_workspace_status(void* workspace, void* stream);

/* Diagnostic (no reference counterpart): launches one warp that waits on a
 * barrier nothing completes, through the same bounded wait the kernels use,
 * so the failure path can be checked without a GPU fault: the wait gives up
 * after about two seconds of device time and records RKV_ERR_DEVICE_TIMEOUT
 * in the workspace error word (clear on entry), which rkv_workspace_status
 * then returns; the CUDA context stays usable.  workspace: device memory,
 * 16-byte aligned, at least 16 bytes.  Asynchronous on `stream`. */
int rkv_selftest_wait_timeout(void* workspace, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RKV_H */
