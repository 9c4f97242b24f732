// rocket_cuda.cpp -- the rocket.h C++17 API (reference rocket.h:36-50)
// implemented over the C ABI of rkv.h.  Host code only: the work runs on the
// current CUDA device through the host-buffer entry points, which copy the
// caller's buffers in, launch the sm_100a kernels and copy the results back.
#include "rocket.h"

#include <stdexcept>
#include <string>

#include "rkv.h"

namespace {

rkv_config to_c(const RocketConfig& c) {
    rkv_config r;
    r.num_heads = c.num_heads;
    r.num_heads_kv = c.num_heads_kv;
    r.dim_head = c.dim_head;
    r.window_size = c.window_size;
    r.kernel_size = c.kernel_size;
    r.prompt_budget = c.prompt_budget;
    r.topk_decode = c.topk_decode;
    r.chunk_size = c.chunk_size;
    r.r_dim = c.r_dim;
    r.compression_ratio = c.compression_ratio;
    return r;
}

[[noreturn]] void raise(const char* what, int status) {
    const std::string msg = std::string(what) + ": " + rkv_status_string(status);
    if (status == RKV_ERR_INVALID_ARG) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

}  // namespace

// rocket.cpp:14-59
RocketBudgetParams compute_rocket_params(int token_budget, int sequence_length, int max_new_tokens,
                                         int head_dim, int window_size) {
    rkv_budget_params p;
    const int st = rkv_compute_params(token_budget, sequence_length, max_new_tokens, head_dim, window_size, &p);
    if (st != RKV_OK) raise("compute_rocket_params", st);
    RocketBudgetParams r;
    r.token_budget = p.token_budget;
    r.sequence_length = p.sequence_length;
    r.max_new_tokens = p.max_new_tokens;
    r.capacity_budget = p.capacity_budget;
    r.prompt_budget = p.prompt_budget;
    r.chunk_size = p.chunk_size;
    r.r = p.r;
    r.k = p.k;
    r.compression_ratio = p.compression_ratio;
    return r;
}

// rocket.cpp:61-169
std::vector<int> compute_prefill_eviction(const float* Q, const float* K, int len_q, int len_k,
                                          const RocketConfig& cfg) {
    const rkv_config c = to_c(cfg);
    const int cap = rkv_evict_max_kept(&c, len_q, len_k);
    if (cap < 0) raise("compute_prefill_eviction", -cap);
    std::vector<int> kept((size_t)cap);
    int n = 0;
    const int st = rkv_prefill_eviction_host(Q, K, len_q, len_k, &c, kept.data(), cap, &n);
    if (st != RKV_OK) raise("compute_prefill_eviction", st);
    kept.resize((size_t)n);
    return kept;
}

// rocket.cpp:171-382
std::vector<float> compute_hybrid_sparse_decode(const float* Q, const float* K, const float* V, int len_k,
                                                const RocketConfig& cfg) {
    const rkv_config c = to_c(cfg);
    if (c.num_heads < 0 || c.dim_head < 0) raise("compute_hybrid_sparse_decode", RKV_ERR_INVALID_ARG);
    std::vector<float> out((size_t)c.num_heads * (size_t)c.dim_head, 0.0f);
    const int st = rkv_hybrid_sparse_decode_host(Q, K, V, len_k, &c, out.data());
    if (st != RKV_OK) raise("compute_hybrid_sparse_decode", st);
    return out;
}
