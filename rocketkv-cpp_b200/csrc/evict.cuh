// evict.cuh -- stage-1 kernel arguments and launchers (see evict.cu).
#pragma once

#include "rkv_common.cuh"

namespace rkv {

struct EvictArgs {
    const uint8_t* Q;
    const uint8_t* K;
    int dtype;
    long long q_stride, k_stride;  // bytes between items
    int len_q, len_k, H, HK, G, D, obs_w, nk, R, ntiles;
    int q_head_rows;  // rows per query head in Q (len_q, or obs_w when compacted)
    int q_row0;       // first window row inside a head (len_q - obs_w, or 0)
    int k_head_rows;  // rows per KV head in K (len_k, or nk when compacted)
    int head_begin, head_count;
    float inv_sqrt_d;
    float* logits;      // [batch][head_count][R][nkp] logits of the CUDA-core engine; the per-tile tensor-core engine
                        // keeps head scores [batch][head_count][nk] here
    int nkp;            // nk rounded up to 4 (16-byte rows)
    float* hs;          // [batch][head_count][nk] head scores of the persistent tensor-core engines
    float2* tstats;     // [batch][head_count][R][ntiles]  (tile max, tile sum)
    float2* rstats;     // [batch][head_count][R]          (row max, 1/(sum+1e-9))
    unsigned* counters; // [batch][head_count]
    int* err;           // workspace error word (bounded in-kernel waits)
    unsigned* gbar;     // workspace word after it: the grid barrier of the one-launch tensor-core scorer
};

struct PoolArgs {
    const float* logits;  // logits [batch][head_count][R][nk], or head scores [batch][head_count][nk] (hs_direct)
    const float2* rstats;
    int R, nk, head_count, pad;
    int hs_direct;
    int pad_eff, log2w;   // filled by the launcher
    float* pooled;  // [batch][head_count][nk]
};

struct SelectArgs {
    const float* pooled;  // [batch][HK][nk], summed over heads in head order
    int HK, nk, obs_w, target_keep;
    uint32_t* keys;       // workspace [batch][nk]
    int* kept;
    int kept_stride;
    int* n_kept;
    int* err;             // workspace error word (the bounded grid barrier of the multi-CTA selection)
};

struct EvictShape {
    int G, obs_w, nk, R, ntiles, target_keep;
    bool keep_all;
    int nkp;
    size_t off_counters, off_rstats, off_tstats, off_logits, off_keys, off_pooled, off_hs, ws_bytes;
};

EvictShape evict_shape(const rkv_config& c, int len_q, int len_k, int batch, int head_count);
int evict_check_supported(const rkv_config& c, int dtype, const EvictShape& s);
int launch_evict_scores(const EvictArgs& a, int batch, cudaStream_t st);
// tcgen05 scoring (evict_mma.cu): statistics, then head scores for the pool kernel (hs_direct)
bool evict_mma_supported(const EvictArgs& a);
int launch_evict_mma(const EvictArgs& a, int batch, cudaStream_t st);
// row max and 1 / (sum + 1e-9) from the per-tile statistics (both tensor-core scorers)
int launch_evict_fold(const EvictArgs& a, int batch, cudaStream_t st);
// persistent warp-specialised tcgen05 scoring (evict_tc.cu): fp32, bf16, q8_0 (D = 128), G * obs_w <= 128
bool evict_tc_supported(const EvictArgs& a, int batch);
int launch_evict_tc(const EvictArgs& a, int batch, cudaStream_t st);
// q8_0 K and Q on kind::i8 tensor-core products (evict_q8.cu): D = 128, G * obs_w <= 128, 16-byte
// aligned K tiles; launch_evict_tc takes it for q8_0 wherever it applies
bool evict_q8_supported(const EvictArgs& a, int batch);
int launch_evict_q8(const EvictArgs& a, int batch, cudaStream_t st);
int launch_evict_pool(const PoolArgs& a, int batch, cudaStream_t st);
int launch_evict_select(const SelectArgs& a, int batch, cudaStream_t st);
int launch_evict_keep_all(int* kept, int kept_stride, int* n_kept, int len_k, int batch, cudaStream_t st);
// the bounded-wait diagnostic (rkv_selftest_wait_timeout)
int launch_wait_selftest(int* err, cudaStream_t st);

}  // namespace rkv
