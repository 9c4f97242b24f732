// ref_capi.cpp -- C entry points over the UNMODIFIED reference rocket.cpp
// (TEST INFRASTRUCTURE).  oracle/Makefile compiles this file together with
// the reference's own rocket.cpp, straight from the reference checkout, into
// oracle/_ref/.  The tests use it to pin the oracle restatement; the
// benchmark's CPU baseline times it.  The product library never loads it.
#include "rocket.h"   // the reference's header (rocket.h:1-49), found via -I<reference dir>

#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {
struct ref_cfg {  // field-for-field copy of the reference RocketConfig (rocket.h:18-34)
    int num_heads, num_heads_kv, dim_head;
    int window_size, kernel_size;
    int prompt_budget, topk_decode, chunk_size, r_dim;
    float compression_ratio;
};

RocketConfig to_cfg(const ref_cfg* c) {
    RocketConfig r{};
    r.num_heads = c->num_heads;
    r.num_heads_kv = c->num_heads_kv;
    r.dim_head = c->dim_head;
    r.window_size = c->window_size;
    r.kernel_size = c->kernel_size;
    r.prompt_budget = c->prompt_budget;
    r.topk_decode = c->topk_decode;
    r.chunk_size = c->chunk_size;
    r.r_dim = c->r_dim;
    r.compression_ratio = c->compression_ratio;
    return r;
}
}  // namespace

extern "C" {

// compute_rocket_params (rocket.h:36-41); out = 8 ints + 1 float in
// RocketBudgetParams field order.
void rkvref_compute_params(int token_budget, int seq_len, int max_new, int head_dim,
                           int window, void* out) {
    RocketBudgetParams p = compute_rocket_params(token_budget, seq_len, max_new, head_dim, window);
    std::memcpy(out, &p, sizeof(p));
}

int rkvref_sizeof_budget_params() { return (int)sizeof(RocketBudgetParams); }

// compute_prefill_eviction (rocket.h:43-46).  Returns the number of indices
// written to kept_out (which must hold max(len_k, prompt_budget) ints).
int rkvref_prefill_eviction(const float* Q, const float* K, int len_q, int len_k,
                            const void* cfg, int* kept_out) {
    std::vector<int> kept = compute_prefill_eviction(Q, K, len_q, len_k,
                                                     to_cfg(static_cast<const ref_cfg*>(cfg)));
    std::memcpy(kept_out, kept.data(), kept.size() * sizeof(int));
    return (int)kept.size();
}

// compute_hybrid_sparse_decode (rocket.h:48-50); O = [num_heads][dim_head].
int rkvref_hsa_decode(const float* Q, const float* K, const float* V, int len_k,
                      const void* cfg, float* O) {
    std::vector<float> out = compute_hybrid_sparse_decode(Q, K, V, len_k,
                                                          to_cfg(static_cast<const ref_cfg*>(cfg)));
    std::memcpy(O, out.data(), out.size() * sizeof(float));
    return (int)out.size();
}

// Threads the reference's own OpenMP loops use (1 in the as-shipped build).
int rkvref_max_threads() {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void rkvref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

}  // extern "C"
