/*
 * rkv_oracle.h -- CPU restatement of RocketKV's two kernels (TEST INFRASTRUCTURE).
 *
 * This library is the checker for the CUDA implementation.  Only the test
 * suite, the smoke check and the CPU-baseline leg of the benchmark load it;
 * the product library never links or calls it.
 *
 * Each function restates the algorithm of the reference file rocket.cpp
 * (Rishit2000/RocketKV-cpp) and cites the lines it follows.  It is pinned
 * against the reference itself: tests/test_oracle.py runs the reference
 * rocket.cpp (compiled from its own sources into oracle/_ref/) on the same
 * seeded inputs and against the known-answer values of test_rocket.cpp.
 *
 * Deliberate, documented differences from rocket.cpp:
 *   - stage 1 breaks score ties toward the lower token index (rocket.cpp:150-155
 *     uses std::nth_element with a score-only comparator, so its tie members
 *     are unspecified);
 *   - stage 2 lists the top-r query dimensions in ascending order (rocket.cpp
 *     sums over them in std::nth_element's output order), ties to the lower
 *     dimension; it forms each approximate page logit with 16 fused
 *     multiply-add chains (by 8-dimension group mod 8 and by dimension
 *     parity) combined in a fixed tree, uses rkvo_expf for the
 *     page softmax and sums that softmax in a fixed 256-way interleaved
 *     order -- the float operations the GPU selection performs, so its
 *     selected indices reproduce this oracle's bit for bit;
 *   - stage 2 optionally keeps a recent window of w tokens (w = 0 is the
 *     reference behaviour) and reports the selected token indices.
 */
#ifndef RKV_ORACLE_H
#define RKV_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int num_heads, num_heads_kv, dim_head;
    int window_size, kernel_size;
    int prompt_budget, topk_decode, chunk_size, r_dim;
    float compression_ratio;
} rkvo_config;

typedef struct {
    int token_budget, sequence_length, max_new_tokens;
    int capacity_budget, prompt_budget, chunk_size, r, k;
    float compression_ratio;
} rkvo_budget;

/* rocket.cpp:14-59 */
void rkvo_compute_params(int token_budget, int sequence_length, int max_new_tokens,
                         int head_dim, int window_size, rkvo_budget* out);

/* exp(x) by Cody-Waite reduction and a degree-7 Taylor polynomial; the same
 * sequence of IEEE operations as the GPU's stage-2 selection exp. */
float rkvo_expf(float x);

/* Stage 1 (rocket.cpp:61-169) with ties toward the lower index.
 * kept_out must hold max(len_k, prompt_budget, window) ints.  Returns the count.
 * total_out (nullable, len_k - obs_w floats) receives the cross-head pooled sum. */
int rkvo_prefill_eviction(const float* Q, const float* K, int len_q, int len_k,
                          const rkvo_config* cfg, int* kept_out, float* total_out);

/* Stage-1 pieces for head-sharded execution: per-head pooled scores for heads
 * [h0, h0+nh) into pooled_out[nh][nk]; and selection from all HK pooled rows. */
int rkvo_evict_pool_heads(const float* Q, const float* K, int len_q, int len_k,
                          const rkvo_config* cfg, int h0, int nh, float* pooled_out);
int rkvo_evict_select_pooled(const float* pooled, int len_q, int len_k,
                             const rkvo_config* cfg, int* kept_out);

/* Largest dim_head of the stage-2 restatement (and of the GPU kernels). */
#define RKVO_MAX_D 256

/* Stage 2 (rocket.cpp:171-382), canonical order, optional recent window.
 * O: [num_heads][dim_head] (zeroed first).  sel_out (nullable):
 * [num_heads_kv][sel_stride] ascending token indices; n_sel (nullable): per
 * KV head count.  kv_bytes: the element size of K on the GPU (2 for bf16, 4
 * for fp32), which fixes the page-logit summation order (16-byte chunks);
 * dim_head must be a multiple of 64 and at most RKVO_MAX_D.  Returns 0, or
 * -1 for an unsupported dim_head / kv_bytes. */
int rkvo_hsa_decode(const float* Q, const float* K, const float* V, int len_k,
                    int recent_window, const rkvo_config* cfg, float* O,
                    int* sel_out, int sel_stride, int* n_sel, int kv_bytes);

#ifdef __cplusplus
}
#endif
#endif
