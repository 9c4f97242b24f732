// rkv_noalloc.cu -- stage-2 hybrid sparse decode for callers that cannot
// allocate device memory.
//
// rkv_hsa_decode needs a caller-allocated workspace.  Some callers have no
// way to provide one: an inference server or plugin host whose allocator
// owns the whole device heap and forbids raw cudaMalloc, or a hot loop that
// cannot accept cudaMalloc's implicit device synchronisation.  For them the
// scratch lives in a fixed array of device memory that the library itself
// declares, so a call allocates nothing.
#include <mutex>

#include "hsa.cuh"

namespace {

// Scratch of rkv_hsa_decode_noalloc.  Every GPU that loads this library holds
// these 4 MiB until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_hsa_noalloc_scratch[kNoAllocScratchBytes];

// In host code the array's name is only a stand-in; the device address of
// each GPU's copy comes from cudaGetSymbolAddress with that GPU current.
constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mutex;

int scratch_of_current_device(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return RKV_ERR_NO_DEVICE;
    if (dev < 0 || dev >= kMaxDevices) return RKV_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_hsa_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return RKV_ERR_CUDA;
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return RKV_OK;
}

}  // namespace

extern "C" int rkv_hsa_decode_noalloc(const void* Q, const void* K, const void* V, int dtype, int len_k,
                                      int recent_window, int batch, long long q_item_stride,
                                      long long kv_item_stride, const rkv_config* cfg, int head_begin,
                                      int head_count, float* O, int* sel, int sel_stride, int* n_sel,
                                      void* stream) {
    size_t need = 0;
    int rc = rkv_hsa_workspace_size(cfg, len_k, recent_window, batch, head_count, &need);
    if (rc != RKV_OK) return rc;
    if (need > kNoAllocScratchBytes) return RKV_ERR_WORKSPACE;  // batch too large for the fixed scratch
    void* ws = nullptr;
    if ((rc = scratch_of_current_device(&ws)) != RKV_OK) return rc;
    // rkv_hsa_decode clears the scratch's error word on `stream` before the
    // kernels run; everything else in the scratch is written before it is read.
    return rkv_hsa_decode(Q, K, V, dtype, len_k, recent_window, batch, q_item_stride, kv_item_stride, cfg,
                          head_begin, head_count, O, sel, sel_stride, n_sel, ws, kNoAllocScratchBytes, stream);
}
