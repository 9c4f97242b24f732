// compact.cu -- KV-cache compaction: the kept token rows of every (item, KV
// head) moved to the front of the cache, in order, on the device.  The
// device analogue of the reference runner's removal of every evicted range
// from the model's KV cache after stage 1 (runner.cpp:246-269, which builds a
// keep mask from compute_prefill_eviction's indices and calls
// llama_memory_seq_rm for each run of evicted positions).
//
// Rows are moved in 16-, 8-, 4- or 2-byte vectors (the widest that divides the
// row size and the alignment of the buffers), consecutive threads taking
// consecutive vectors of a row.  The kept list of an item is ascending, so
// destination row i never lies above its source row kept[i]; in place, one CTA
// per (item, KV head) walks its rows in chunks and reads every source row of a
// chunk before it writes any destination of it (later chunks' sources lie at
// or beyond their own destinations, above the chunk).  Out of place, the rows
// of an (item, KV head) are spread over several CTAs.
#include "rkv_common.cuh"

namespace rkv {
namespace {

constexpr int kCompactNT = 256;
constexpr int kCompactVPT = 4;  // vectors per thread per chunk

struct CompactArgs {
    const uint8_t* K;
    const uint8_t* V;
    uint8_t* Ko;
    uint8_t* Vo;
    const int* kept;
    const int* n_kept;
    int kept_stride, len_k, out_len, vpr;  // vpr: vectors per row
    long long rowb, in_item, out_item;     // bytes
};

template <typename VT>
__global__ void __launch_bounds__(kCompactNT) compact_kernel(const CompactArgs a) {
    // Launched as a programmatic dependent of stage 1's selection (rkv_evict_compact) the grid may start
    // while the selection still runs: this waits until it has completed and its kept lists are visible.
    // Launched normally there is nothing to wait for.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int hk = blockIdx.y, b = blockIdx.z;
    const int* kept = a.kept + (size_t)b * a.kept_stride;
    const int n = min(a.n_kept[b], a.out_len);
    const int chunk_rows = kCompactNT * kCompactVPT / a.vpr;  // >= 1 (vpr <= 1024)
    const long long nchunks = (n + chunk_rows - 1) / chunk_rows;
#pragma unroll 1
    for (int t = 0; t < 2; ++t) {  // K, then V
        const uint8_t* src = t == 0 ? a.K : a.V;
        uint8_t* dst = t == 0 ? a.Ko : a.Vo;
        if (!src) continue;
        src += (size_t)b * a.in_item + (size_t)hk * a.len_k * a.rowb;
        dst += (size_t)b * a.out_item + (size_t)hk * a.out_len * a.rowb;
        for (long long c = blockIdx.x; c < nchunks; c += gridDim.x) {
            const int r0 = (int)(c * chunk_rows);
            VT v[kCompactVPT];
            int row[kCompactVPT], vec[kCompactVPT];
#pragma unroll
            for (int u = 0; u < kCompactVPT; ++u) {
                const int g = threadIdx.x + u * kCompactNT;  // vector of the chunk
                row[u] = r0 + g / a.vpr;
                vec[u] = g % a.vpr;
                const int s = (g < chunk_rows * a.vpr && row[u] < n) ? kept[row[u]] : -1;
                if (s >= 0 && s < a.len_k) {
                    v[u] = reinterpret_cast<const VT*>(src + (size_t)s * a.rowb)[vec[u]];
                } else {
                    row[u] = -1;  // nothing to move (past the kept count, or an index outside the cache)
                }
            }
            __syncthreads();  // every source of the chunk read before any destination is written
#pragma unroll
            for (int u = 0; u < kCompactVPT; ++u)
                if (row[u] >= 0) reinterpret_cast<VT*>(dst + (size_t)row[u] * a.rowb)[vec[u]] = v[u];
            __syncthreads();
        }
    }
}

}  // namespace
}  // namespace rkv

using namespace rkv;

namespace {

// Validates, plans and launches one compaction; pdl: as a programmatic dependent launch of the previous
// kernel on the stream.
int compact_launch(const void* K, const void* V, int dtype, int head_dim, int num_heads_kv, int len_k, int batch,
                   long long kv_item_stride, const int* kept, const int* n_kept, int kept_stride, void* K_out,
                   void* V_out, int out_len, long long out_item_stride, bool pdl, cudaStream_t st) {
    if (dtype != RKV_F32 && dtype != RKV_BF16 && dtype != RKV_Q8_0) return RKV_ERR_INVALID_ARG;
    if (head_dim <= 0 || (dtype == RKV_Q8_0 && head_dim % 32 != 0)) return RKV_ERR_INVALID_ARG;
    if (num_heads_kv <= 0 || len_k < 0 || batch < 0 || out_len < 0 || kept_stride < 0) return RKV_ERR_INVALID_ARG;
    if (batch == 0 || num_heads_kv == 0) return RKV_OK;
    if (!K || !K_out || !kept || !n_kept || (V && !V_out) || (!V && V_out)) return RKV_ERR_INVALID_ARG;
    const long long rowb = (long long)row_bytes(dtype, head_dim);
    const long long in_need = (long long)num_heads_kv * len_k * rowb, out_need = (long long)num_heads_kv * out_len * rowb;
    if (batch > 1 && (kv_item_stride < in_need || out_item_stride < out_need)) return RKV_ERR_INVALID_ARG;
    const bool inplace = K_out == K || (V && V_out == V);
    if (inplace) {
        // one layout for source and destination, and no partial overlap between K and V
        if (K_out != K || V_out != V || out_len != len_k || (batch > 1 && out_item_stride != kv_item_stride))
            return RKV_ERR_INVALID_ARG;
    }
    // widest vector dividing the row size, the buffers' alignment and the item strides
    uintptr_t al = reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(K_out) | (uintptr_t)rowb;
    if (V) al |= reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(V_out);
    if (batch > 1) al |= (uintptr_t)kv_item_stride | (uintptr_t)out_item_stride;
    const int vb = (al & 15) == 0 ? 16 : (al & 7) == 0 ? 8 : (al & 3) == 0 ? 4 : (al & 1) == 0 ? 2 : 1;
    if (vb < 2) return RKV_ERR_INVALID_ARG;  // rows of whole 16-bit elements
    CompactArgs a{};
    a.K = static_cast<const uint8_t*>(K);
    a.V = static_cast<const uint8_t*>(V);
    a.Ko = static_cast<uint8_t*>(K_out);
    a.Vo = static_cast<uint8_t*>(V_out);
    a.kept = kept;
    a.n_kept = n_kept;
    a.kept_stride = kept_stride;
    a.len_k = len_k;
    a.out_len = out_len;
    a.rowb = rowb;
    a.vpr = (int)(rowb / vb);
    a.in_item = kv_item_stride;
    a.out_item = out_item_stride;
    if (a.vpr > kCompactNT * kCompactVPT) return RKV_ERR_UNSUPPORTED;
    // in place: one CTA per (item, KV head) walks its chunks in order; out of place: spread the chunks
    const int chunk_rows = kCompactNT * kCompactVPT / a.vpr;
    const int chunks = out_len > 0 ? (out_len + chunk_rows - 1) / chunk_rows : 1;
    const int split = inplace ? 1 : (chunks < 64 ? chunks : 64);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(split > 0 ? split : 1, num_heads_kv, batch);
    cfg.blockDim = dim3(kCompactNT);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e;
    switch (vb) {
        case 16: e = cudaLaunchKernelEx(&cfg, compact_kernel<uint4>, a); break;
        case 8: e = cudaLaunchKernelEx(&cfg, compact_kernel<uint2>, a); break;
        case 4: e = cudaLaunchKernelEx(&cfg, compact_kernel<uint32_t>, a); break;
        default: e = cudaLaunchKernelEx(&cfg, compact_kernel<uint16_t>, a); break;
    }
    if (e != cudaSuccess) (void)cudaGetLastError();
    return e == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

}  // namespace

extern "C" int rkv_compact_kv(const void* K, const void* V, int dtype, int head_dim, int num_heads_kv, int len_k,
                              int batch, long long kv_item_stride, const int* kept, const int* n_kept,
                              int kept_stride, void* K_out, void* V_out, int out_len, long long out_item_stride,
                              void* stream) {
    return compact_launch(K, V, dtype, head_dim, num_heads_kv, len_k, batch, kv_item_stride, kept, n_kept, kept_stride,
                          K_out, V_out, out_len, out_item_stride, false, static_cast<cudaStream_t>(stream));
}

extern "C" int rkv_evict_compact(const void* Q, const void* K, const void* V, int dtype, int len_q, int len_k,
                                 int batch, long long q_item_stride, long long kv_item_stride, const rkv_config* cfg,
                                 int* kept, int kept_stride, int* n_kept, void* K_out, void* V_out, int out_len,
                                 long long out_item_stride, void* workspace, size_t workspace_bytes, int engine,
                                 void* stream) {
    if (!cfg || dtype == RKV_F16) return RKV_ERR_INVALID_ARG;
    if (batch > 0 && (!K_out || (V && !V_out) || (!V && V_out))) return RKV_ERR_INVALID_ARG;
    int rc = rkv_evict(Q, K, dtype, len_q, len_k, batch, q_item_stride, kv_item_stride, cfg, kept, kept_stride, n_kept,
                       workspace, workspace_bytes, engine, stream);
    if (rc != RKV_OK || batch == 0) return rc;
    // the selection kernel is the last launch on the stream: the compaction starts behind it
    return compact_launch(K, V, dtype, cfg->dim_head, cfg->num_heads_kv, len_k, batch, kv_item_stride, kept, n_kept,
                          kept_stride, K_out, V_out, out_len, out_item_stride, true, static_cast<cudaStream_t>(stream));
}
