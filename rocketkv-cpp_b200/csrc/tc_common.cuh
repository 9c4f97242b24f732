// tc_common.cuh -- tcgen05 (5th-generation tensor core), tensor-memory and
// tensor-TMA helpers for the sm_100a stage-1 scorers (PTX ISA 8.7).
// No cluster multicast anywhere.
#pragma once

#include "rkv_common.cuh"

namespace rkv {

constexpr int kMmaM = 128;  // MMA rows (tensor-memory lanes) of every stage-1 tile

// Shared-memory matrix descriptor, K-major, no swizzle.  lbo = bytes between
// the two 16-byte K units one MMA K step reads, sbo = bytes between 8-row
// groups; bits 46-47 = 1 (the sm_100 descriptor version).
__device__ __forceinline__ uint64_t mma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128
// bytes, 8-row groups 1024 bytes apart (sbo), the 16-byte chunk c of row r
// stored at chunk c ^ (r % 8) of the row, groups 1024-byte aligned.  The
// leading offset is unused for this layout (encoded as 1); layout type 2 in
// bits 61-63.  A K step inside the 128-byte row is taken by adding its byte
// offset to `addr`.
__device__ __forceinline__ uint64_t mma_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor: fp32 accumulator, K-major A and B, M = 128.
// fmt: 2 = TF32, 1 = BF16 (both operands).
__host__ __device__ constexpr uint32_t mma_idesc(uint32_t fmt, uint32_t n) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((n >> 3) << 17) | ((uint32_t)(kMmaM >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // one full warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // the allocating warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <bool TF32>
__device__ __forceinline__ void mma_issue(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (TF32)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc)
            : "memory");
}
// Arrives on `bar` once every MMA this thread issued before it has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// 32 consecutive accumulator columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive accumulator columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// x - (x with the low 13 mantissa bits cleared), exact: the part of an fp32
// value that a TF32 operand read of x drops (the tensor core reads the top
// 19 bits of a 32-bit operand).
__device__ __forceinline__ uint4 tf32_lo(const uint4& x) {
    return make_uint4(__float_as_uint(__fsub_rn(__uint_as_float(x.x), __uint_as_float(x.x & 0xFFFFE000u))),
                      __float_as_uint(__fsub_rn(__uint_as_float(x.y), __uint_as_float(x.y & 0xFFFFE000u))),
                      __float_as_uint(__fsub_rn(__uint_as_float(x.z), __uint_as_float(x.z & 0xFFFFE000u))),
                      __float_as_uint(__fsub_rn(__uint_as_float(x.w), __uint_as_float(x.w & 0xFFFFE000u))));
}

// 2^t on the MUFU (ex2.approx, results below the normal range flush to 0, -inf gives 0).
__device__ __forceinline__ float ex2_approx(float t) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(t));
    return y;
}

// Two int8 (the low and high byte of w) -> exact fp32, by placing each
// byte + 128 in the low mantissa bits of 2^23 and subtracting 2^23 + 128.
__device__ __forceinline__ float2 i8x2_to_f2(uint32_t w) {
    const uint32_t u = w ^ 0x8080u;
    const float2 f = make_float2(__uint_as_float(0x4B000000u | (u & 0xFFu)), __uint_as_float(0x4B000000u | ((u >> 8) & 0xFFu)));
    return __fadd2_rn(f, make_float2(-8388736.0f, -8388736.0f));
}

// 8-byte global load the compiler keeps where it is written (a prefetch into
// registers that must not sink to its first use).
__device__ __forceinline__ uint2 ldg_nc_v2_pinned(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// ---- issue by one elected lane of a converged warp --------------------------
// The whole warp runs the issuing loop (its operands stay warp-uniform) and
// elect.sync inside each statement picks the one lane that issues.
template <bool TF32>
__device__ __forceinline__ void mma_issue_w(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if (TF32)
        asm volatile(
            "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
            "l"(a), "l"(b), "r"(idesc), "r"(acc)
            : "memory");
}
__device__ __forceinline__ void mma_commit_w(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_w(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_w(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];\n\t}" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_4d_w(void* dst, const void* tmap, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5}], [%6];\n\t}" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

// One tiled 4-D tensor copy global -> shared (no multicast).
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

// hi: x with the low 13 mantissa bits cleared (the TF32 value); lo = x - hi (exact).
__device__ __forceinline__ void split_tf32(const uint4& x, uint4& hi, uint4& lo) {
    hi = make_uint4(x.x & 0xFFFFE000u, x.y & 0xFFFFE000u, x.z & 0xFFFFE000u, x.w & 0xFFFFE000u);
    lo = make_uint4(__float_as_uint(__fsub_rn(__uint_as_float(x.x), __uint_as_float(hi.x))),
                    __float_as_uint(__fsub_rn(__uint_as_float(x.y), __uint_as_float(hi.y))),
                    __float_as_uint(__fsub_rn(__uint_as_float(x.z), __uint_as_float(hi.z))),
                    __float_as_uint(__fsub_rn(__uint_as_float(x.w), __uint_as_float(hi.w))));
}

// One tiled 3-D tensor copy global -> shared (no multicast); completion is
// signalled on `bar`.  x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Named barrier over `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void group_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier that also returns whether `p` holds on every participating thread.
__device__ __forceinline__ bool group_all(int id, int nthreads, bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\t"
        "bar.red.and.pred b, %2, %3, a;\n\tselp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Bounded wait that also gives up when another role of the CTA has set
// *abort (it timed out first).  Returns false on either; a timeout records
// RKV_ERR_DEVICE_TIMEOUT in *err and sets *abort.  The waiting thread is
// suspended by try_wait's time hint (woken when the phase completes), so
// waiting warps leave the issue slots to the warps that work.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_suspend(bar, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            atomicExch(err, (int)RKV_ERR_DEVICE_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace rkv
