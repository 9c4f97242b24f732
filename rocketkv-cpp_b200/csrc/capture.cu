// capture.cu -- the capture side of stage 1 on the device: post-RoPE Q and K
// rows taken straight from the producing attention's buffers into the
// head-major layout the stage-1 kernels read.
//
// The reference runner intercepts the "Qcur-<layer>" / "Kcur-<layer>" ROPE
// tensors of the last layer in a ggml eval callback (runner.cpp:25-92): each
// micro-batch's tensor (ne = [dim_head, n_heads, n_tokens], F32, F16 or BF16)
// is copied to the host, converted to fp32 and scattered row by row into
// [n_heads][total_prompt_tokens][dim_head] at the micro-batch's token offset.
// Here the same scatter runs on the device with no host copy: one call per
// micro-batch and layer, rows read from the producer's buffer in place (any
// token and head stride) and converted exactly (fp16 and bf16 values are
// fp32 values; bf16 may also stay bf16).  Every layer can be captured into its
// own item, so stage 1 can score all layers in one batched call instead of
// only the last.
#include "rkv_common.cuh"

namespace rkv {
namespace {

struct CaptureArgs {
    const uint8_t* src;
    long long token_stride, head_stride;  // bytes
    int src_dtype, dst_dtype, n_tokens, n_heads, dim_head;
    int token_offset;               // global token index of the micro-batch's first row
    int dst_first, dst_tokens;      // dst rows hold tokens dst_first .. dst_first + dst_tokens - 1
    uint8_t* dst;                   // item base: [n_heads][dst_tokens][dim_head]
};

__device__ __forceinline__ float src_value(const uint8_t* row, int dtype, int d) {
    if (dtype == RKV_F32) return reinterpret_cast<const float*>(row)[d];
    const uint16_t b = reinterpret_cast<const uint16_t*>(row)[d];
    if (dtype == RKV_BF16) return __uint_as_float((uint32_t)b << 16);
    return __half2float(__ushort_as_half(b));  // fp16 -> fp32, exact
}

// One CTA per (token, group of heads); consecutive threads take consecutive
// elements of a row, so reads and writes are coalesced along dim_head.
__global__ void __launch_bounds__(256) capture_kernel(const CaptureArgs a) {
    const int t = blockIdx.x;
    const int dt = a.token_offset + t - a.dst_first;  // destination row
    if (dt < 0 || dt >= a.dst_tokens) return;          // uniform: a token outside the kept range
    const int per = a.n_heads * a.dim_head;
    for (int e = blockIdx.y * blockDim.x + threadIdx.x; e < per; e += gridDim.y * blockDim.x) {
        const int h = e / a.dim_head, d = e - h * a.dim_head;
        const uint8_t* row = a.src + (size_t)t * a.token_stride + (size_t)h * a.head_stride;
        const float v = src_value(row, a.src_dtype, d);
        const size_t o = ((size_t)h * a.dst_tokens + dt) * a.dim_head + d;
        if (a.dst_dtype == RKV_F32) {
            reinterpret_cast<float*>(a.dst)[o] = v;
        } else {  // bf16 source kept as bf16: the bits are copied
            reinterpret_cast<uint16_t*>(a.dst)[o] = (uint16_t)(__float_as_uint(v) >> 16);
        }
    }
}

}  // namespace
}  // namespace rkv

using namespace rkv;

extern "C" int rkv_capture_rows(const void* src, int src_dtype, int n_tokens, int n_heads, int dim_head,
                                long long token_stride, long long head_stride, int token_offset, void* dst,
                                int dst_dtype, int dst_first, int dst_tokens, long long dst_item_stride, int item,
                                void* stream) {
    if (n_tokens < 0 || n_heads <= 0 || dim_head <= 0 || dst_tokens < 0 || item < 0 || token_offset < 0)
        return RKV_ERR_INVALID_ARG;
    if (src_dtype != RKV_F32 && src_dtype != RKV_BF16 && src_dtype != RKV_F16) return RKV_ERR_INVALID_ARG;
    if (dst_dtype != RKV_F32 && dst_dtype != RKV_BF16) return RKV_ERR_UNSUPPORTED;
    if (dst_dtype == RKV_BF16 && src_dtype != RKV_BF16) return RKV_ERR_UNSUPPORTED;  // only exact conversions
    const int es = src_dtype == RKV_F32 ? 4 : 2;
    if (token_stride < (long long)es || head_stride < (long long)es) return RKV_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(src) % es) || (token_stride % es) || (head_stride % es)) return RKV_ERR_INVALID_ARG;
    if (n_tokens == 0 || dst_tokens == 0) return RKV_OK;
    if (!src || !dst) return RKV_ERR_INVALID_ARG;
    const size_t dst_bytes = (size_t)n_heads * dst_tokens * dim_head * (dst_dtype == RKV_F32 ? 4 : 2);
    if (item > 0 && dst_item_stride < (long long)dst_bytes) return RKV_ERR_INVALID_ARG;
    CaptureArgs a{};
    a.src = static_cast<const uint8_t*>(src);
    a.token_stride = token_stride;
    a.head_stride = head_stride;
    a.src_dtype = src_dtype;
    a.dst_dtype = dst_dtype;
    a.n_tokens = n_tokens;
    a.n_heads = n_heads;
    a.dim_head = dim_head;
    a.token_offset = token_offset;
    a.dst_first = dst_first;
    a.dst_tokens = dst_tokens;
    a.dst = static_cast<uint8_t*>(dst) + (size_t)item * dst_item_stride;
    const int per = n_heads * dim_head;
    int gy = (per + 255) / 256;
    if (gy > 64) gy = 64;
    capture_kernel<<<dim3(n_tokens, gy), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}
