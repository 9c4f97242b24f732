// rkv_noalloc.cu -- stage-2 hybrid sparse decode for callers that cannot
// allocate device memory.
//
// rkv_hsa_decode needs a caller-allocated workspace.  Some callers have no
// way to provide one: an inference server or plugin host whose allocator
// owns the whole device heap and forbids raw cudaMalloc, or a hot loop that
// cannot accept cudaMalloc's implicit device synchronisation.  For them the
// scratch lives in a fixed array of device memory that the library itself
// declares, so a call allocates nothing.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "hsa.cuh"

namespace {

// Scratch of rkv_hsa_decode_noalloc.  Every GPU that loads this library holds
// these 4 MiB until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_hsa_noalloc_scratch[kNoAllocScratchBytes];

// In host code the array's name is only a stand-in; the device address of
// each context's copy comes from cudaGetSymbolAddress with that context
// current.  The address is kept per device together with the unique id of the
// context it was looked up in (cuCtxGetId): a context created later on the
// same device (after cudaDeviceReset, or by another component resetting the
// primary context) has another id, and its copy of the array is looked up
// again instead of reusing an address from the destroyed context.
constexpr int kMaxDevices = 64;
struct ScratchSlot {
    unsigned long long ctx_id;
    void* addr;
};
ScratchSlot g_scratch[kMaxDevices];
std::mutex g_scratch_mutex;

PFN_cuCtxGetCurrent_v4000 g_get_current = nullptr;
PFN_cuCtxGetId_v12000 g_get_id = nullptr;

bool driver_entry_points() {
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    });
    return g_get_current && g_get_id;
}

// Unique id of the calling thread's current context; 0 when none is current yet.
int current_context_id(unsigned long long* id) {
    *id = 0;
    CUcontext c = nullptr;
    if (g_get_current(&c) != CUDA_SUCCESS) return RKV_ERR_CUDA;
    if (c && g_get_id(c, id) != CUDA_SUCCESS) return RKV_ERR_CUDA;
    return RKV_OK;
}

int scratch_of_current_device(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return RKV_ERR_NO_DEVICE;
    if (dev < 0 || dev >= kMaxDevices) return RKV_ERR_UNSUPPORTED;
    if (!driver_entry_points()) return RKV_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    unsigned long long id = 0;
    int rc = current_context_id(&id);
    if (rc != RKV_OK) return rc;
    ScratchSlot& s = g_scratch[dev];
    if (id == 0 || !s.addr || s.ctx_id != id) {
        // set-up, with this device current: the address of this context's copy
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_hsa_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return RKV_ERR_CUDA;
        }
        if ((rc = current_context_id(&id)) != RKV_OK) return rc;  // the lookup made the context current
        s.ctx_id = id;
        s.addr = p;
    }
    *out = s.addr;
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

// The kernels record a bounded in-kernel wait that ran out in the scratch's
// error word, as they do in a caller's workspace; this reads and clears the
// word of the current device's scratch after synchronising `stream`.
extern "C" int rkv_hsa_decode_noalloc_status(void* stream) {
    void* ws = nullptr;
    const int rc = scratch_of_current_device(&ws);
    if (rc != RKV_OK) return rc;
    return rkv_workspace_status(ws, stream);
}
