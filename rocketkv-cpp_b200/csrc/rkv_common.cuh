// rkv_common.cuh -- shared device helpers for the RocketKV sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "rkv.h"

namespace rkv {

constexpr int kWorkspaceAlign = 256;
// First bytes of every workspace: the in-kernel error word.
constexpr size_t kWorkspaceHeader = 256;

// Clock-cycle budget of one bounded wait (about two seconds at 1.9 GHz).
constexpr long long kWaitCycles = 4000000000LL;

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// Element loads.  bf16 -> fp32 and fp16-scaled int8 -> fp32 are exact.
// ---------------------------------------------------------------------------
struct Q8Block {  // ggml block_q8_0 layout: fp16 scale, 32 int8 values (34 bytes)
    uint16_t d;
    int8_t qs[32];
};
static_assert(sizeof(Q8Block) == 34, "q8_0 block must be 34 bytes");

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

__device__ __forceinline__ float load_elem(const void* base, int dtype, size_t idx) {
    if (dtype == RKV_F32) return static_cast<const float*>(base)[idx];
    if (dtype == RKV_BF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(base)[idx]);
    const uint8_t* blk = static_cast<const uint8_t*>(base) + (idx / 32) * 34;
    const uint16_t sbits = static_cast<uint16_t>(blk[0]) | (static_cast<uint16_t>(blk[1]) << 8);
    const float s = __half2float(__ushort_as_half(sbits));
    return s * static_cast<float>(static_cast<int8_t>(blk[2 + idx % 32]));
}

// Bytes of one row of `dim` elements.
__host__ __device__ inline size_t row_bytes(int dtype, int dim) {
    return dtype == RKV_F32 ? (size_t)dim * 4 : dtype == RKV_BF16 ? (size_t)dim * 2 : (size_t)dim / 32 * 34;
}

// ---------------------------------------------------------------------------
// Deterministic exp for the stage-2 selection path, for x <= 0 (the softmax
// argument l - max) and NaN; the same IEEE operation sequence as the oracle's
// rkvo_expf.  Cody & Waite reduction x = n ln2 + r with n = round(x log2 e)
// taken by one fused multiply-add against 1.5 * 2^23 (round to nearest even,
// no double rounding), ln2 split into a short head and a tail, the degree-7
// Taylor polynomial (1/k!) by Horner with fused multiply-adds, then the exact
// two-step scaling p * 2^(n+64) * 2^-64 (one rounding, subnormals included).
// Branch-free.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float det_expf(float x) {
    const float log2e = __int_as_float(0x3fb8aa3b);
    const float ln2_hi = __int_as_float(0x3f317000);
    const float ln2_lo = __int_as_float(0x3805fdf4);
    const float magic = __int_as_float(0x4b400000);  // 1.5 * 2^23
    const float xc = fmaxf(x, -104.0f);
    const float t = __fmaf_rn(xc, log2e, magic);
    const float n = __fsub_rn(t, magic);
    float r = __fmaf_rn(-n, ln2_hi, xc);
    r = __fmaf_rn(-n, ln2_lo, r);
    float p = __int_as_float(0x39500d01);
    p = __fmaf_rn(p, r, __int_as_float(0x3ab60b61));
    p = __fmaf_rn(p, r, __int_as_float(0x3c088889));
    p = __fmaf_rn(p, r, __int_as_float(0x3d2aaaab));
    p = __fmaf_rn(p, r, __int_as_float(0x3e2aaaab));
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = __float_as_int(t) - 0x4b400000;  // n as an integer, -151 .. 0
    const float res = __fmul_rn(__fmul_rn(p, __int_as_float((ni + 64 + 127) << 23)), __int_as_float(0x1f800000));
    const float out = x < -103.97208404541015625f ? 0.0f : res;
    return x != x ? x : out;
}

// det_expf on two values at once with the packed fp32x2 operations of
// sm_100: the same operation sequence per lane, so each lane's result equals
// det_expf of it bit for bit (t - magic is exact; fma(-n, c, r) equals
// fma(n, -c, r)).
__device__ __forceinline__ float2 det_expf2(float2 x) {
    const float log2e = __int_as_float(0x3fb8aa3b);
    const float magic = __int_as_float(0x4b400000);
    const float2 xc = make_float2(fmaxf(x.x, -104.0f), fmaxf(x.y, -104.0f));
    const float2 t = __ffma2_rn(xc, make_float2(log2e, log2e), make_float2(magic, magic));
    const float2 n = __fadd2_rn(t, make_float2(-magic, -magic));
    const float nh = -__int_as_float(0x3f317000), nl = -__int_as_float(0x3805fdf4);
    float2 r = __ffma2_rn(n, make_float2(nh, nh), xc);
    r = __ffma2_rn(n, make_float2(nl, nl), r);
    float2 p = make_float2(__int_as_float(0x39500d01), __int_as_float(0x39500d01));
    p = __ffma2_rn(p, r, make_float2(__int_as_float(0x3ab60b61), __int_as_float(0x3ab60b61)));
    p = __ffma2_rn(p, r, make_float2(__int_as_float(0x3c088889), __int_as_float(0x3c088889)));
    p = __ffma2_rn(p, r, make_float2(__int_as_float(0x3d2aaaab), __int_as_float(0x3d2aaaab)));
    p = __ffma2_rn(p, r, make_float2(__int_as_float(0x3e2aaaab), __int_as_float(0x3e2aaaab)));
    p = __ffma2_rn(p, r, make_float2(0.5f, 0.5f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
    const int nx = __float_as_int(t.x) - 0x4b400000, ny = __float_as_int(t.y) - 0x4b400000;
    const float2 sc = make_float2(__int_as_float((nx + 64 + 127) << 23), __int_as_float((ny + 64 + 127) << 23));
    const float m64 = __int_as_float(0x1f800000);
    const float2 res = __fmul2_rn(__fmul2_rn(p, sc), make_float2(m64, m64));
    const float lim = -103.97208404541015625f;
    float2 out;
    out.x = x.x != x.x ? x.x : (x.x < lim ? 0.0f : res.x);
    out.y = x.y != x.y ? x.y : (x.y < lim ? 0.0f : res.y);
    return out;
}

// Order-preserving map float -> uint32 (larger float, larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, non-tensor) helpers.  No cluster multicast.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// One bulk global->shared copy; completion is signalled on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// As mbar_try_wait, but the thread may be suspended up to ~100 us waiting for
// the phase.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and records
// RKV_ERR_DEVICE_TIMEOUT in *err) if the clock budget runs out.  Waiting
// threads are suspended by try_wait's time hint, so they leave the issue
// slots to the warps that have work.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    // try_wait with a suspend-time hint parks the thread until the phase
    // completes (woken then, not after a sleep) or the hint runs out
    while (!mbar_try_wait_suspend(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicExch(err, (int)RKV_ERR_DEVICE_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Grid-wide barrier for cooperative launches (every CTA resident): arrive on
// the counter, then wait until it reaches `target` (k * gridDim.x for the
// k-th barrier of a launch; the counter starts at zero).  One thread per CTA
// calls it between __syncthreads.  Bounded: a timeout records
// RKV_ERR_DEVICE_TIMEOUT in *err and returns false.
__device__ __forceinline__ bool grid_sync_bounded(unsigned* cnt, unsigned target, int* err) {
    __threadfence();
    atomicAdd(cnt, 1u);
    const long long t0 = clock64();
    for (;;) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
        if (v >= target) break;
        if (clock64() - t0 > kWaitCycles) {
            atomicExch(err, (int)RKV_ERR_DEVICE_TIMEOUT);
            return false;
        }
        __nanosleep(100);
    }
    __threadfence();
    return true;
}

// ---------------------------------------------------------------------------
// Block-wide exclusive scan of one int per thread (blockDim.x threads,
// blockDim.x a multiple of 32, at most 1024).  `tmp` holds 33 ints.
// Returns the exclusive prefix; *total receives the block sum.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int block_exclusive_scan(int v, int* tmp, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) tmp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? tmp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nwarps) tmp[lane] = w;  // inclusive warp totals
        if (lane == nwarps - 1) tmp[32] = w;
    }
    __syncthreads();
    const int before = (warp > 0 ? tmp[warp - 1] : 0) + x - v;
    *total = tmp[32];
    __syncthreads();  // tmp reusable after return
    return before;
}

// Block-wide exclusive scan of two ints per thread at once (same contract as
// block_exclusive_scan; `tmp` holds 66 ints).  Returns the prefix of `a` and
// writes the prefix of `b` to *pb; the totals to *ta, *tb.
__device__ __forceinline__ int block_exclusive_scan2(int a, int b, int* tmp, int* pb, int* ta, int* tb) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    int x = a, y = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, x, o), v = __shfl_up_sync(0xffffffffu, y, o);
        if (lane >= o) {
            x += u;
            y += v;
        }
    }
    if (lane == 31) {
        tmp[warp] = x;
        tmp[33 + warp] = y;
    }
    __syncthreads();
    if (warp == 0) {
        int u = lane < nwarps ? tmp[lane] : 0, v = lane < nwarps ? tmp[33 + lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int uu = __shfl_up_sync(0xffffffffu, u, o), vv = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) {
                u += uu;
                v += vv;
            }
        }
        if (lane < nwarps) {
            tmp[lane] = u;
            tmp[33 + lane] = v;
        }
        if (lane == nwarps - 1) {
            tmp[32] = u;
            tmp[65] = v;
        }
    }
    __syncthreads();
    const int before_a = (warp > 0 ? tmp[warp - 1] : 0) + x - a;
    *pb = (warp > 0 ? tmp[33 + warp - 1] : 0) + y - b;
    *ta = tmp[32];
    *tb = tmp[65];
    __syncthreads();  // tmp reusable after return
    return before_a;
}

// Launch as a programmatic dependent of the kernel before it on the stream: the
// launch is processed while that kernel runs, and the kernel waits for its
// results with griddepcontrol.wait (a no-op in a kernel launched without the
// attribute).  After a non-kernel operation the stream orders as usual.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*f)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc{};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    lc.attrs = at;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, f, args...);
}

}  // namespace rkv
