// rkv_capi.cu -- the extern "C" entry points declared in include/rkv.h:
// argument validation, workspace planning, launches, and the host-buffer
// (rocket.h drop-in) paths with their per-thread device buffers.
#include <math.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "evict.cuh"
#include "hsa.cuh"

using namespace rkv;

namespace {

int check_cfg(const rkv_config* c) {
    if (!c) return RKV_ERR_INVALID_ARG;
    if (c->num_heads <= 0 || c->num_heads_kv <= 0 || c->dim_head <= 0) return RKV_ERR_INVALID_ARG;
    if (c->window_size < 0) return RKV_ERR_INVALID_ARG;
    return RKV_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per-thread, per-device resources of the host-buffer paths: one stream and
// one grow-only device buffer.  Released when the thread exits.
struct DevCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    void* buf = nullptr;
    size_t cap = 0;
    ~DevCtx() {
        if (buf) cudaFree(buf);
        if (stream) cudaStreamDestroy(stream);
    }
};

struct CtxList {
    std::vector<DevCtx*> v;
    ~CtxList() {
        for (DevCtx* c : v) delete c;
    }
};
thread_local CtxList t_ctx;

int get_ctx(size_t bytes, DevCtx** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return RKV_ERR_NO_DEVICE;
    DevCtx* ctx = nullptr;
    for (DevCtx* c : t_ctx.v)
        if (c->device == dev) ctx = c;
    if (!ctx) {
        ctx = new DevCtx();
        ctx->device = dev;
        if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
            delete ctx;
            return RKV_ERR_CUDA;
        }
        t_ctx.v.push_back(ctx);
    }
    if (ctx->cap < bytes) {
        if (ctx->buf) cudaFree(ctx->buf);
        ctx->buf = nullptr;
        ctx->cap = 0;
        if (cudaMalloc(&ctx->buf, bytes) != cudaSuccess) {
            cudaGetLastError();
            return RKV_ERR_CUDA;
        }
        ctx->cap = bytes;
    }
    *out = ctx;
    return RKV_OK;
}

struct Carve {  // bump allocator over one device buffer
    size_t off = 0;
    size_t take(size_t bytes) {
        const size_t o = off;
        off = align_up(off + (bytes ? bytes : 1), kWorkspaceAlign);
        return o;
    }
};

int finish_sync(cudaStream_t st, void* ws) {
    if (cudaStreamSynchronize(st) != cudaSuccess) return RKV_ERR_CUDA;
    if (ws) {
        int e = 0;
        if (cudaMemcpy(&e, ws, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return RKV_ERR_CUDA;
        if (e) return e;
    }
    return RKV_OK;
}

// Fills the stage-1 argument block for KV heads [head_begin, head_begin+head_count).
EvictArgs make_evict_args(const void* Q, const void* K, int dtype, int len_q, int len_k,
                          long long qs, long long ks, const rkv_config& c, const EvictShape& s,
                          int head_begin, int head_count, uint8_t* ws) {
    EvictArgs a{};
    a.Q = static_cast<const uint8_t*>(Q);
    a.K = static_cast<const uint8_t*>(K);
    a.dtype = dtype;
    a.q_stride = qs;
    a.k_stride = ks;
    a.len_q = len_q;
    a.len_k = len_k;
    a.H = c.num_heads;
    a.HK = c.num_heads_kv;
    a.G = s.G;
    a.D = c.dim_head;
    a.obs_w = s.obs_w;
    a.nk = s.nk;
    a.R = s.R;
    a.ntiles = s.ntiles;
    a.q_head_rows = len_q;
    a.q_row0 = len_q - s.obs_w;
    a.k_head_rows = len_k;
    a.head_begin = head_begin;
    a.head_count = head_count;
    a.inv_sqrt_d = 1.0f / sqrtf((float)c.dim_head);
    a.logits = reinterpret_cast<float*>(ws + s.off_logits);
    a.nkp = s.nkp;
    a.hs = reinterpret_cast<float*>(ws + s.off_hs);
    a.tstats = reinterpret_cast<float2*>(ws + s.off_tstats);
    a.rstats = reinterpret_cast<float2*>(ws + s.off_rstats);
    a.counters = reinterpret_cast<unsigned*>(ws + s.off_counters);
    a.err = reinterpret_cast<int*>(ws);
    a.gbar = reinterpret_cast<unsigned*>(ws + sizeof(int));
    return a;
}

int evict_run(const EvictArgs& a, const rkv_config& c, const EvictShape& s, int batch, uint8_t* ws,
              float* pooled_out, int* kept, int kept_stride, int* n_kept, int engine, cudaStream_t st) {
    if (cudaMemsetAsync(a.err, 0, sizeof(int) + sizeof(unsigned), st) != cudaSuccess) return RKV_ERR_CUDA;  // error word, grid barrier
    // engine chain: persistent tensor-core kernel, per-tile tensor-core kernel, CUDA cores
    bool tensor = false, persistent = false;
    int rc = RKV_OK;
    if ((engine == RKV_EVICT_AUTO || engine == RKV_EVICT_TENSOR) && evict_tc_supported(a, batch)) {
        rc = launch_evict_tc(a, batch, st);
        if (rc != RKV_OK && rc != RKV_ERR_UNSUPPORTED) return rc;
        tensor = persistent = rc == RKV_OK;
    }
    if (!tensor && engine != RKV_EVICT_SIMT && evict_mma_supported(a)) {
        if ((rc = launch_evict_mma(a, batch, st))) return rc;
        tensor = true;
    }
    if (!tensor) {
        if (engine == RKV_EVICT_TENSOR || engine == RKV_EVICT_TENSOR_TILES) return RKV_ERR_UNSUPPORTED;
        if ((rc = launch_evict_scores(a, batch, st))) return rc;
    }
    PoolArgs p{};
    p.hs_direct = tensor ? 1 : 0;
    p.logits = persistent ? a.hs : a.logits;
    p.rstats = a.rstats;
    p.R = s.R;
    p.nk = s.nk;
    p.head_count = a.head_count;
    p.pad = c.kernel_size / 2;
    p.pooled = pooled_out ? pooled_out : reinterpret_cast<float*>(ws + s.off_pooled);
    rc = launch_evict_pool(p, batch, st);
    if (rc || pooled_out) return rc;
    SelectArgs sa{};
    sa.pooled = p.pooled;
    sa.HK = c.num_heads_kv;
    sa.nk = s.nk;
    sa.obs_w = s.obs_w;
    sa.target_keep = s.target_keep;
    sa.keys = reinterpret_cast<uint32_t*>(ws + s.off_keys);
    sa.err = a.err;
    sa.kept = kept;
    sa.kept_stride = kept_stride;
    sa.n_kept = n_kept;
    return launch_evict_select(sa, batch, st);
}

int max_kept_of(const EvictShape& s, int len_k) {
    if (s.keep_all) return len_k;
    return s.target_keep + s.obs_w;
}

// stage 2 on device buffers; summary: page summaries (rkv_hsa_build_summary) or null
int hsa_decode_impl(const void* Q, const void* K, const void* V, const void* summary, int dtype, int len_k,
                    int recent_window, int batch, long long q_item_stride, long long kv_item_stride,
                    const rkv_config* cfg, int head_begin, int head_count, float* O, int* sel, int sel_stride,
                    int* n_sel, void* workspace, size_t workspace_bytes, void* stream);

}  // namespace

extern "C" {

int rkv_abi_version(void) { return RKV_ABI_VERSION; }

const char* rkv_status_string(int status) {
    switch (status) {
        case RKV_OK: return "ok";
        case RKV_ERR_INVALID_ARG: return "invalid argument";
        case RKV_ERR_UNSUPPORTED: return "unsupported configuration";
        case RKV_ERR_CUDA: return "CUDA runtime error";
        case RKV_ERR_WORKSPACE: return "workspace missing or too small";
        case RKV_ERR_DEVICE_TIMEOUT: return "bounded in-kernel wait timed out";
        case RKV_ERR_NO_DEVICE: return "no CUDA device";
        default: return "unknown status";
    }
}

void rkv_config_init(rkv_config* c) {
    if (!c) return;
    memset(c, 0, sizeof(*c));
    c->window_size = 32;
    c->kernel_size = 63;
}

// rocket.cpp:14-59, in float arithmetic as there.
int rkv_compute_params(int token_budget, int sequence_length, int max_new_tokens, int head_dim,
                       int window_size, rkv_budget_params* p) {
    if (!p) return RKV_ERR_INVALID_ARG;
    p->sequence_length = sequence_length;
    p->max_new_tokens = max_new_tokens;
    p->token_budget = sequence_length < token_budget ? sequence_length : token_budget;
    const float cr_initial = fmaxf(1.0f, (float)sequence_length / (float)p->token_budget);
    const float alpha = fminf(0.2f + log2f(cr_initial) * 0.06f, 0.8f);
    int capacity = (int)floorf((float)sequence_length / powf(cr_initial, alpha));
    const int floor_cap = 2 * max_new_tokens < sequence_length ? 2 * max_new_tokens : sequence_length;
    if (capacity < floor_cap) capacity = floor_cap;
    p->capacity_budget = capacity;
    int prompt = sequence_length - max_new_tokens < capacity - max_new_tokens ? sequence_length - max_new_tokens
                                                                              : capacity - max_new_tokens;
    if (prompt < window_size) prompt = window_size;
    p->prompt_budget = prompt;
    const int half = (int)roundf((float)p->token_budget / 2.0f);
    p->k = half < capacity ? half : capacity;
    const float cr2 = fmaxf(1.0f, (float)capacity / (float)p->token_budget);
    p->compression_ratio = cr2;
    const int c1 = (int)floorf(cr2), c2 = (int)ceilf(sqrtf(cr2));
    int chunk = c1 < c2 ? c1 : c2;
    if (chunk < 1) chunk = 1;
    p->chunk_size = chunk;
    int r = (int)roundf((float)head_dim * (float)chunk / cr2);
    if (r < 1) r = 1;
    p->r = r < head_dim ? r : head_dim;
    return RKV_OK;
}

// ---------------------------------------------------------------------------
// Stage 1
// ---------------------------------------------------------------------------
int rkv_evict_max_kept(const rkv_config* cfg, int len_q, int len_k) {
    if (check_cfg(cfg) || len_q < 0 || len_k < 0) return -RKV_ERR_INVALID_ARG;
    const EvictShape s = evict_shape(*cfg, len_q, len_k, 1, cfg->num_heads_kv);
    if (s.nk < 0 && !(len_k <= cfg->prompt_budget)) return -RKV_ERR_INVALID_ARG;
    const int n = max_kept_of(s, len_k);
    return n > 0 ? n : 1;
}

int rkv_evict_workspace_size(const rkv_config* cfg, int dtype, int len_q, int len_k, int batch,
                             size_t* bytes) {
    if (check_cfg(cfg) || !bytes || len_q < 0 || len_k < 0 || batch < 0) return RKV_ERR_INVALID_ARG;
    if (dtype < RKV_F32 || dtype > RKV_Q8_0) return RKV_ERR_INVALID_ARG;
    *bytes = evict_shape(*cfg, len_q, len_k, batch, cfg->num_heads_kv).ws_bytes;
    return RKV_OK;
}

static int evict_validate(const void* Q, const void* K, int dtype, int len_q, int len_k, int batch,
                          const rkv_config* cfg, const EvictShape& s) {
    if (check_cfg(cfg) || len_q < 0 || len_k < 0 || batch < 0) return RKV_ERR_INVALID_ARG;
    if (dtype < RKV_F32 || dtype > RKV_Q8_0) return RKV_ERR_INVALID_ARG;
    if (!s.keep_all && s.nk < 0) return RKV_ERR_INVALID_ARG;  // rocket.cpp:78 cannot size its buffer
    if (!s.keep_all && (!Q || !K)) return RKV_ERR_INVALID_ARG;
    return evict_check_supported(*cfg, dtype, s);
}

int rkv_evict(const void* Q, const void* K, int dtype, int len_q, int len_k, int batch,
              long long q_item_stride, long long k_item_stride, const rkv_config* cfg, int* kept,
              int kept_stride, int* n_kept, void* workspace, size_t workspace_bytes, int engine,
              void* stream) {
    if (engine < RKV_EVICT_AUTO || engine > RKV_EVICT_TENSOR_TILES) return RKV_ERR_INVALID_ARG;
    if (check_cfg(cfg)) return RKV_ERR_INVALID_ARG;
    const EvictShape s = evict_shape(*cfg, len_q, len_k, batch, cfg->num_heads_kv);
    int rc = evict_validate(Q, K, dtype, len_q, len_k, batch, cfg, s);
    if (rc) return rc;
    if (batch == 0) return RKV_OK;
    if (!kept || !n_kept || kept_stride < max_kept_of(s, len_k)) return RKV_ERR_INVALID_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (s.keep_all) return launch_evict_keep_all(kept, kept_stride, n_kept, len_k, batch, st);
    if (!workspace || workspace_bytes < s.ws_bytes || !aligned16(workspace)) return RKV_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const EvictArgs a = make_evict_args(Q, K, dtype, len_q, len_k, q_item_stride, k_item_stride, *cfg, s, 0,
                                        cfg->num_heads_kv, ws);
    return evict_run(a, *cfg, s, batch, ws, nullptr, kept, kept_stride, n_kept, engine, st);
}

int rkv_evict_pool_heads(const void* Q, const void* K, int dtype, int len_q, int len_k, int batch,
                         long long q_item_stride, long long k_item_stride, const rkv_config* cfg,
                         int head_begin, int head_count, float* pooled, void* workspace,
                         size_t workspace_bytes, int engine, void* stream) {
    if (engine < RKV_EVICT_AUTO || engine > RKV_EVICT_TENSOR_TILES) return RKV_ERR_INVALID_ARG;
    if (check_cfg(cfg)) return RKV_ERR_INVALID_ARG;
    if (head_begin < 0 || head_count < 0 || head_begin + head_count > cfg->num_heads_kv) return RKV_ERR_INVALID_ARG;
    EvictShape s = evict_shape(*cfg, len_q, len_k, batch, head_count);
    s.keep_all = false;  // the pooled rows are defined whenever nk >= 0
    int rc = evict_validate(Q, K, dtype, len_q, len_k, batch, cfg, s);
    if (rc) return rc;
    if (batch == 0 || head_count == 0 || s.nk == 0) return RKV_OK;
    if (!pooled) return RKV_ERR_INVALID_ARG;
    if (!workspace || workspace_bytes < s.ws_bytes || !aligned16(workspace)) return RKV_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const EvictArgs a = make_evict_args(Q, K, dtype, len_q, len_k, q_item_stride, k_item_stride, *cfg, s,
                                        head_begin, head_count, ws);
    return evict_run(a, *cfg, s, batch, ws, pooled, nullptr, 0, nullptr, engine, static_cast<cudaStream_t>(stream));
}

int rkv_evict_select_pooled(const float* pooled, int len_q, int len_k, int batch, const rkv_config* cfg,
                            int* kept, int kept_stride, int* n_kept, void* workspace, size_t workspace_bytes,
                            void* stream) {
    if (check_cfg(cfg) || len_q < 0 || len_k < 0 || batch < 0) return RKV_ERR_INVALID_ARG;
    const EvictShape s = evict_shape(*cfg, len_q, len_k, batch, cfg->num_heads_kv);
    if (!s.keep_all && s.nk < 0) return RKV_ERR_INVALID_ARG;
    if (batch == 0) return RKV_OK;
    if (!kept || !n_kept || kept_stride < max_kept_of(s, len_k)) return RKV_ERR_INVALID_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (s.keep_all) return launch_evict_keep_all(kept, kept_stride, n_kept, len_k, batch, st);
    if (!pooled) return RKV_ERR_INVALID_ARG;
    if (!workspace || workspace_bytes < s.ws_bytes || !aligned16(workspace)) return RKV_ERR_WORKSPACE;
    SelectArgs sa{};
    sa.pooled = pooled;
    sa.HK = cfg->num_heads_kv;
    sa.nk = s.nk;
    sa.obs_w = s.obs_w;
    sa.target_keep = s.target_keep;
    sa.keys = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + s.off_keys);
    sa.err = static_cast<int*>(workspace);
    if (cudaMemsetAsync(sa.err, 0, sizeof(int), st) != cudaSuccess) return RKV_ERR_CUDA;
    sa.kept = kept;
    sa.kept_stride = kept_stride;
    sa.n_kept = n_kept;
    return launch_evict_select(sa, batch, st);
}

int rkv_prefill_eviction_host(const float* Q, const float* K, int len_q, int len_k, const rkv_config* cfg,
                              int* kept_out, int kept_capacity, int* n_kept) {
    if (check_cfg(cfg) || !kept_out || !n_kept) return RKV_ERR_INVALID_ARG;
    const EvictShape s0 = evict_shape(*cfg, len_q, len_k, 1, cfg->num_heads_kv);
    int rc = evict_validate(Q, K, RKV_F32, len_q, len_k, 1, cfg, s0);
    if (rc) return rc;
    if (kept_capacity < max_kept_of(s0, len_k)) return RKV_ERR_INVALID_ARG;
    if (s0.keep_all) {  // rocket.cpp:67-71 and :134-138: every token is kept
        for (int i = 0; i < len_k; ++i) kept_out[i] = i;
        *n_kept = len_k;
        return RKV_OK;
    }
    // Only the window rows of Q (rocket.cpp:90) and the first nk rows of K
    // (rocket.cpp:97-99) are read, so only those cross PCIe.
    const int HKG = cfg->num_heads_kv * s0.G;
    const int D = cfg->dim_head;
    Carve cv;
    const size_t o_q = cv.take((size_t)HKG * s0.obs_w * D * 4);
    const size_t o_k = cv.take((size_t)cfg->num_heads_kv * s0.nk * D * 4);
    const size_t o_kept = cv.take((size_t)max_kept_of(s0, len_k) * 4);
    const size_t o_n = cv.take(4);
    const size_t o_ws = cv.take(s0.ws_bytes);
    DevCtx* ctx;
    if ((rc = get_ctx(cv.off, &ctx))) return rc;
    uint8_t* base = static_cast<uint8_t*>(ctx->buf);
    cudaStream_t st = ctx->stream;
    if (HKG > 0 && s0.obs_w > 0 &&
        cudaMemcpy2DAsync(base + o_q, (size_t)s0.obs_w * D * 4, Q + (size_t)(len_q - s0.obs_w) * D,
                          (size_t)len_q * D * 4, (size_t)s0.obs_w * D * 4, HKG, cudaMemcpyHostToDevice,
                          st) != cudaSuccess)
        return RKV_ERR_CUDA;
    if (s0.nk > 0 &&
        cudaMemcpy2DAsync(base + o_k, (size_t)s0.nk * D * 4, K, (size_t)len_k * D * 4, (size_t)s0.nk * D * 4,
                          cfg->num_heads_kv, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return RKV_ERR_CUDA;
    EvictArgs a = make_evict_args(base + o_q, base + o_k, RKV_F32, len_q, len_k, 0, 0, *cfg, s0, 0,
                                  cfg->num_heads_kv, base + o_ws);
    a.q_head_rows = s0.obs_w;
    a.q_row0 = 0;
    a.k_head_rows = s0.nk;
    int* dk = reinterpret_cast<int*>(base + o_kept);
    int* dn = reinterpret_cast<int*>(base + o_n);
    if ((rc = evict_run(a, *cfg, s0, 1, base + o_ws, nullptr, dk, max_kept_of(s0, len_k), dn, RKV_EVICT_AUTO, st)))
        return rc;
    const int nmax = max_kept_of(s0, len_k);
    if (cudaMemcpyAsync(kept_out, dk, (size_t)nmax * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(n_kept, dn, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return RKV_ERR_CUDA;
    return finish_sync(st, nullptr);
}

// ---------------------------------------------------------------------------
// Stage 2
// ---------------------------------------------------------------------------
int rkv_hsa_sel_capacity(const rkv_config* cfg, int len_k, int recent_window) {
    if (check_cfg(cfg)) return -RKV_ERR_INVALID_ARG;
    const int n = hsa_shape(*cfg, len_k, recent_window, 1, 1).sel_cap;
    return n > 0 ? n : 1;
}

int rkv_hsa_workspace_size(const rkv_config* cfg, int len_k, int recent_window, int batch, int head_count,
                           size_t* bytes) {
    if (check_cfg(cfg) || !bytes || batch < 0 || head_count < 0) return RKV_ERR_INVALID_ARG;
    *bytes = hsa_shape(*cfg, len_k, recent_window, batch, head_count).ws_bytes;
    return RKV_OK;
}

int rkv_hsa_decode(const void* Q, const void* K, const void* V, int dtype, int len_k, int recent_window,
                   int batch, long long q_item_stride, long long kv_item_stride, const rkv_config* cfg,
                   int head_begin, int head_count, float* O, int* sel, int sel_stride, int* n_sel,
                   void* workspace, size_t workspace_bytes, void* stream) {
    return hsa_decode_impl(Q, K, V, nullptr, dtype, len_k, recent_window, batch, q_item_stride, kv_item_stride, cfg,
                           head_begin, head_count, O, sel, sel_stride, n_sel, workspace, workspace_bytes, stream);
}

int rkv_hsa_summary_size(const rkv_config* cfg, int dtype, int len_k, int recent_window, int batch, size_t* bytes) {
    if (check_cfg(cfg) || !bytes || batch < 0 || len_k < 0) return RKV_ERR_INVALID_ARG;
    if (dtype != RKV_F32 && dtype != RKV_BF16) return dtype == RKV_Q8_0 ? RKV_ERR_UNSUPPORTED : RKV_ERR_INVALID_ARG;
    const int rc = hsa_check_supported(*cfg, dtype);
    if (rc) return rc;
    *bytes = (size_t)batch * (size_t)hsa_summary_shape(*cfg, dtype, len_k, recent_window).item_bytes;
    return RKV_OK;
}

int rkv_hsa_build_summary(const void* K, int dtype, int len_k, int recent_window, int batch,
                          long long kv_item_stride, const rkv_config* cfg, void* summary, void* stream) {
    if (check_cfg(cfg) || batch < 0 || len_k < 0) return RKV_ERR_INVALID_ARG;
    if (dtype != RKV_F32 && dtype != RKV_BF16) return dtype == RKV_Q8_0 ? RKV_ERR_UNSUPPORTED : RKV_ERR_INVALID_ARG;
    int rc = hsa_check_supported(*cfg, dtype);
    if (rc) return rc;
    if (batch == 0) return RKV_OK;
    if (!K || !summary || !aligned16(summary) || (kv_item_stride & 3) || (reinterpret_cast<uintptr_t>(K) & 3))
        return RKV_ERR_INVALID_ARG;
    const HsaSummaryShape sh = hsa_summary_shape(*cfg, dtype, len_k, recent_window);
    const long long rowb = (long long)cfg->dim_head * (dtype == RKV_F32 ? 4 : 2);
    if (batch > 1 && kv_item_stride < (long long)cfg->num_heads_kv * len_k * rowb) return RKV_ERR_INVALID_ARG;
    return launch_hsa_summary_build(static_cast<const uint8_t*>(K), dtype, cfg->dim_head, cfg->num_heads_kv, len_k,
                                    kv_item_stride, sh, static_cast<uint8_t*>(summary), batch,
                                    static_cast<cudaStream_t>(stream));
}

int rkv_hsa_decode_summary(const void* Q, const void* K, const void* V, const void* summary, int dtype,
                           int len_k, int recent_window, int batch, long long q_item_stride,
                           long long kv_item_stride, const rkv_config* cfg, int head_begin, int head_count,
                           float* O, int* sel, int sel_stride, int* n_sel, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (!summary || !aligned16(summary)) return RKV_ERR_INVALID_ARG;
    return hsa_decode_impl(Q, K, V, summary, dtype, len_k, recent_window, batch, q_item_stride, kv_item_stride, cfg,
                           head_begin, head_count, O, sel, sel_stride, n_sel, workspace, workspace_bytes, stream);
}

}  // extern "C"

namespace {

int hsa_decode_impl(const void* Q, const void* K, const void* V, const void* summary, int dtype, int len_k,
                    int recent_window, int batch, long long q_item_stride, long long kv_item_stride,
                    const rkv_config* cfg, int head_begin, int head_count, float* O, int* sel, int sel_stride,
                    int* n_sel, void* workspace, size_t workspace_bytes, void* stream) {
    if (check_cfg(cfg) || batch < 0 || len_k < 0) return RKV_ERR_INVALID_ARG;
    if (head_begin < 0 || head_count < 0 || head_begin + head_count > cfg->num_heads_kv) return RKV_ERR_INVALID_ARG;
    if (dtype != RKV_F32 && dtype != RKV_BF16) return dtype == RKV_Q8_0 ? RKV_ERR_UNSUPPORTED : RKV_ERR_INVALID_ARG;
    int rc = hsa_check_supported(*cfg, dtype);
    if (rc) return rc;
    if (batch == 0 || head_count == 0) return RKV_OK;
    const HsaShape s = hsa_shape(*cfg, len_k, recent_window, batch, head_count);
    if (!Q || !K || !V || !O) return RKV_ERR_INVALID_ARG;
    if (!aligned16(K) || !aligned16(V) || (kv_item_stride & 15) || (q_item_stride & 3)) return RKV_ERR_INVALID_ARG;
    if (sel && sel_stride < s.sel_cap) return RKV_ERR_INVALID_ARG;
    if (!workspace || workspace_bytes < s.ws_bytes || !aligned16(workspace)) return RKV_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(ws, 0, sizeof(int), st) != cudaSuccess) return RKV_ERR_CUDA;
    HsaArgs a{};
    a.Q = static_cast<const uint8_t*>(Q);
    a.K = static_cast<const uint8_t*>(K);
    a.V = static_cast<const uint8_t*>(V);
    a.q_stride = q_item_stride;
    a.kv_stride = kv_item_stride;
    a.len_k = len_k;
    a.H = cfg->num_heads;
    a.HK = cfg->num_heads_kv;
    a.G = s.G;
    a.D = cfg->dim_head;
    a.C = s.C;
    a.r = s.r;
    a.w = s.w;
    a.Lc = s.Lc;
    a.final_k = s.final_k;
    a.nchunks = s.nchunks;
    a.nch_pad = s.nch_pad;
    a.head_begin = head_begin;
    a.head_count = head_count;
    a.inv_sqrt_d = 1.0f / sqrtf((float)cfg->dim_head);
    a.O = O;
    if (sel) {
        a.sel = sel;
        a.sel_stride = sel_stride;
    } else {
        a.sel = reinterpret_cast<int*>(ws + s.off_sel);
        a.sel_stride = s.sel_cap > 0 ? s.sel_cap : 1;
    }
    a.n_sel = n_sel;
    a.wlogits = reinterpret_cast<float*>(ws + s.off_logits);
    a.wscore = reinterpret_cast<float*>(ws + s.off_scores);
    a.score_stride = s.sel_cap > 0 ? s.sel_cap : 1;
    a.err = reinterpret_cast<int*>(ws);
    if (summary) {
        const HsaSummaryShape sh = hsa_summary_shape(*cfg, dtype, len_k, recent_window);
        a.summary = static_cast<const uint8_t*>(summary);
        a.sum_stride = sh.item_bytes;
        a.sum_mask_off = sh.mask_off;
        a.npp = sh.npp;
    }
    return launch_hsa(a, dtype, batch, st);
}

}  // namespace

extern "C" {

int rkv_hsa_decode_host_ex(const void* Q, const void* K, const void* V, int dtype, int len_k, int recent_window,
                           int batch, long long q_item_stride, long long kv_item_stride, const rkv_config* cfg,
                           float* O, int* sel, int sel_stride, int* n_sel) {
    if (check_cfg(cfg) || batch < 0 || len_k < 0 || !O) return RKV_ERR_INVALID_ARG;
    if (batch == 0) return RKV_OK;
    if (!Q || !K || !V) return RKV_ERR_INVALID_ARG;
    const int HK = cfg->num_heads_kv;
    const HsaShape s = hsa_shape(*cfg, len_k, recent_window, batch, HK);
    if (sel && sel_stride < s.sel_cap) return RKV_ERR_INVALID_ARG;
    const size_t qbytes = (size_t)q_item_stride * (batch - 1) + (size_t)cfg->num_heads * cfg->dim_head * (dtype == RKV_F32 ? 4 : 2);
    const size_t kvbytes = (size_t)kv_item_stride * (batch - 1) + row_bytes(dtype, cfg->dim_head) * (size_t)HK * len_k;
    const size_t obytes = (size_t)batch * cfg->num_heads * cfg->dim_head * 4;
    const int sstride = s.sel_cap > 0 ? s.sel_cap : 1;
    // V in pinned host memory that the device can address (cudaHostAlloc, or
    // cudaHostRegister with mapping) is read in place by the attention kernel:
    // only the selected rows cross the bus.  Otherwise V is copied like K.
    const void* v_mapped = nullptr;
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, V) == cudaSuccess) {
        if (pa.type == cudaMemoryTypeHost && pa.devicePointer && aligned16(pa.devicePointer)) v_mapped = pa.devicePointer;
    } else {
        cudaGetLastError();
    }
    Carve cv;
    const size_t o_q = cv.take(qbytes), o_k = cv.take(kvbytes), o_v = cv.take(v_mapped ? 0 : kvbytes),
                 o_o = cv.take(obytes);
    const size_t o_sel = cv.take((size_t)batch * HK * sstride * 4), o_n = cv.take((size_t)batch * HK * 4);
    const size_t o_ws = cv.take(s.ws_bytes);
    DevCtx* ctx;
    int rc;
    if ((rc = get_ctx(cv.off, &ctx))) return rc;
    uint8_t* base = static_cast<uint8_t*>(ctx->buf);
    cudaStream_t st = ctx->stream;
    if (cudaMemcpyAsync(base + o_q, Q, qbytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(base + o_k, K, kvbytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        (!v_mapped && cudaMemcpyAsync(base + o_v, V, kvbytes, cudaMemcpyHostToDevice, st) != cudaSuccess) ||
        cudaMemsetAsync(base + o_o, 0, obytes, st) != cudaSuccess)
        return RKV_ERR_CUDA;
    const void* vd = v_mapped ? v_mapped : static_cast<const void*>(base + o_v);
    rc = rkv_hsa_decode(base + o_q, base + o_k, vd, dtype, len_k, recent_window, batch, q_item_stride,
                        kv_item_stride, cfg, 0, HK, reinterpret_cast<float*>(base + o_o),
                        reinterpret_cast<int*>(base + o_sel), sstride, reinterpret_cast<int*>(base + o_n),
                        base + o_ws, s.ws_bytes, st);
    if (rc) return rc;
    if (cudaMemcpyAsync(O, base + o_o, obytes, cudaMemcpyDeviceToHost, st) != cudaSuccess) return RKV_ERR_CUDA;
    if (n_sel && cudaMemcpyAsync(n_sel, base + o_n, (size_t)batch * HK * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return RKV_ERR_CUDA;
    if (sel && cudaMemcpy2DAsync(sel, (size_t)sel_stride * 4, base + o_sel, (size_t)sstride * 4,
                                 (size_t)s.sel_cap * 4, (size_t)batch * HK, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return RKV_ERR_CUDA;
    return finish_sync(st, base + o_ws);
}

int rkv_hybrid_sparse_decode_host(const float* Q, const float* K, const float* V, int len_k, const rkv_config* cfg,
                                  float* O) {
    if (check_cfg(cfg) || !O) return RKV_ERR_INVALID_ARG;
    const size_t HD = (size_t)cfg->num_heads * cfg->dim_head;
    if (len_k <= 0) {  // rocket.cpp:186
        memset(O, 0, HD * sizeof(float));
        return RKV_OK;
    }
    const long long kv_stride = (long long)cfg->num_heads_kv * len_k * cfg->dim_head * 4;
    return rkv_hsa_decode_host_ex(Q, K, V, RKV_F32, len_k, 0, 1, (long long)HD * 4, kv_stride, cfg, O, nullptr, 0,
                                  nullptr);
}

int rkv_workspace_status(void* workspace, void* stream) {
    if (!workspace) return RKV_ERR_INVALID_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(st) != cudaSuccess) return RKV_ERR_CUDA;
    int e = 0;
    if (cudaMemcpy(&e, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return RKV_ERR_CUDA;
    if (e && cudaMemset(workspace, 0, sizeof(int)) != cudaSuccess) return RKV_ERR_CUDA;
    return e;
}

int rkv_selftest_wait_timeout(void* workspace, void* stream) {
    if (!workspace || !aligned16(workspace)) return RKV_ERR_INVALID_ARG;
    return launch_wait_selftest(static_cast<int*>(workspace), static_cast<cudaStream_t>(stream));
}

}  // extern "C"
