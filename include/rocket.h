// rocket.h -- RocketKV's C++17 API, kept declaration-for-declaration equal to
// the reference header (Rishit2000/RocketKV-cpp rocket.h:1-49) so that callers
// such as the reference runner.cpp and test_rocket.cpp compile unchanged
// against this implementation.  Here the functions are served by the B200
// kernels of librkv_b200.so (through the C ABI in rkv.h) instead of the CPU
// loops of rocket.cpp.
//
// Behaviour differences from the reference, all on paths where the reference
// has no defined result:
//   - a CUDA failure or an unsupported shape throws std::runtime_error, and a
//     size that the reference cannot allocate (len_k < min(window_size, len_q))
//     throws std::invalid_argument;
//   - stage-1 score ties keep the lower token index.
#pragma once
#include <vector>

// Budget parameters derived from the user's token budget (rocket.h:4-15).
struct RocketBudgetParams {
    int token_budget;        // requested KV budget
    int sequence_length;     // prompt length N
    int max_new_tokens;      // expected generation length T
    int capacity_budget;     // KV capacity across prefill and decode
    int prompt_budget;       // tokens kept by stage-1 eviction
    int chunk_size;          // stage-2 page size
    int r;                   // stage-2 query dimensions kept
    int k;                   // stage-2 decode top-k
    float compression_ratio; // stage-2 compression ratio
};

// Configuration of both kernels (rocket.h:17-34).
struct RocketConfig {
    int num_heads;
    int num_heads_kv;
    int dim_head;

    int window_size = 32;    // observation window, always kept
    int kernel_size = 63;    // max-pooling width

    int prompt_budget;
    int topk_decode;
    int chunk_size;
    int r_dim;
    float compression_ratio;
};

RocketBudgetParams compute_rocket_params(
    int token_budget,
    int sequence_length,
    int max_new_tokens,
    int head_dim,
    int window_size = 32);

std::vector<int> compute_prefill_eviction(
    const float* Q, const float* K,
    int len_q, int len_k,
    const RocketConfig& cfg);

std::vector<float> compute_hybrid_sparse_decode(
    const float* Q, const float* K, const float* V,
    int len_k, const RocketConfig& cfg);
