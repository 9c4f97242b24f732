// evict_tc.cu -- persistent, warp-specialised stage-1 scoring on the tcgen05
// tensor cores (sm_100a): the default engine for fp32, bf16 and q8_0 where
// the window rows fit in one MMA (G * obs_w <= 128) and the shared-memory
// plan fits.  evict_mma.cu keeps the non-persistent kernel for the rest.
//
// One CTA per SM walks a contiguous range of (item, KV head, 128-key tile)
// work units.  Per tile the contraction D[128 keys][N rows] = K_tile . Q^T
// (N = G * obs_w rounded up to 16) accumulates in tensor memory, alternating
// between two accumulators so the epilogue of a tile overlaps the MMAs of the
// next.  The reduction dimension is walked in "k-blocks" of 128 bytes of
// operand row (32 fp32 or 64 bf16 values; a q8_0 block of 32 values is one
// fp32 k-block after dequantisation).  Shared-memory operands use the
// K-major 128-byte-swizzle layout of tcgen05.
//
// fp32 (and dequantised q8_0) runs as three TF32 products per K step,
// hi.hi + hi.lo + lo.hi: the tensor core reads the top 19 bits of an fp32
// operand (hi), and lo = x - hi is exact, so the logits carry close to fp32
// accuracy.  bf16 runs one bf16 product (exact products, fp32 accumulation).
//
// Warp roles (448 threads):
//   warp 0      TMA producer (fp32, bf16): the window queries of each KV
//               head (one tensor copy per query head and k-block, into the
//               resident query block) and one copy per k-block of 128 key
//               rows into a ring of 16 KB stages;
//   warp 1      allocates tensor memory; issues the MMAs and the
//               tcgen05.commit arrivals that release stages and accumulators.
//               Warps 0 and 1 run their loops converged and one lane, picked
//               by elect.sync inside each issuing statement, issues: the
//               operands stay warp-uniform, which keeps the issue of a copy or
//               an MMA at a few cycles instead of ~100 (measured);
//   warps 2-5   operand converters: lo = x - hi of every fp32 k-block and
//               query block; q8_0 tiles loaded with coalesced 8-byte loads and
//               dequantised exactly to fp32 in shared memory (x and lo), the
//               q8_0 window queries likewise;
//   warps 6-13  epilogue, two warps per tensor-memory lane quarter (warp w
//               reads lanes 32 (w % 4) ..), each taking half of the window
//               rows.
//
// Two passes over the CTA's tiles (rocket.cpp:91-116): pass 0 writes the
// per-(row, tile) max and sum of exp(l - max) of l = (q . k) / sqrt(D); the
// epilogue then folds a head's tile statistics into the row max M_r and
// inv_r = 1 / (sum_r + 1e-9) (rocket.cpp:108-113), and pass 1 writes the head
// score of every key, sum_r exp(l - M_r) * inv_r, for the pooling kernel.
// Pass 1 has two forms.  While they fit in L2, pass 0 keeps every
// exp(l - quarter max) and pass 1 streams them once (one exp per (row, tile,
// quarter) rescales them).  For long prefixes, whose kept values would be
// written to and read back from HBM, pass 1 instead runs the copies and MMAs
// again over the tiles in reverse order (the first ones are still in L2) and
// forms each key's score from the logits in tensor memory.  Both passes run
// in one cooperative launch when every CTA can be resident: a bounded grid
// barrier between them holds only the epilogue (in the recompute form the
// copies and MMAs of pass 1 already run); otherwise one launch per pass.
// Every wait is bounded; a role that times out sets a CTA-wide abort flag so
// the others leave their loops; copies and MMAs in flight are waited for and
// the tensor memory is freed on every path.
#include "evict.cuh"
#include "tc_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <float.h>
#include <string.h>

#include <mutex>

namespace rkv {
namespace {

constexpr int kTcThreads = 448;
constexpr int kEpiThreads = 256;    // warps 6-13
constexpr int kStageB = 128 * 128;  // one operand stage: 128 rows x 128 bytes
constexpr int kMaxStages = 8;
constexpr int kLoStages = 2;
constexpr int kAccCols = 128;       // tensor-memory columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kTbStride = 36;       // floats per row of an epilogue warp's transpose buffer (16-byte rows, conflict-free)
constexpr int kBarConv = 1, kBarEpi = 2;
constexpr int kSmemMax = 227 * 1024;  // dynamic shared memory per CTA on sm_100
constexpr int kQ8Row = 136;           // bytes of one q8_0 row of 128 values
constexpr int kQ8Words = 128 * kQ8Row / 8 / 128;  // 8-byte words per converter thread of a q8_0 tile (17)

enum { KIND_F32 = 0, KIND_BF16 = 1, KIND_Q8 = 2 };

struct TcPlan {  // shared-memory offsets from the 1024-byte aligned base, and the work split
    int NP, nkb, rowb, S, q_atom, qbytes;
    int off_qhi, off_qlo, off_stg, off_epi, off_epi1, off_lo, off_raw, total;
    int nwork, nheads;  // work units (128-key tiles) and (item, KV head) pairs
    int p0, p1;         // the passes this launch runs: 0 = scores and statistics, 1 = head scores
    int rc;             // pass 1 recomputes the logits through the copy / MMA pipeline instead of reading
                        // the kept exp values (chosen when those would not fit in L2)
};

__host__ __device__ inline int align1k(int x) { return (x + 1023) & ~1023; }

inline TcPlan tc_plan(int kind, int R, int D) {
    TcPlan P{};
    P.NP = (R + 15) & ~15;
    P.rowb = D * (kind == KIND_BF16 ? 2 : 4);  // operand bytes per row (q8_0 as fp32)
    P.nkb = (P.rowb + 127) / 128;
    P.q_atom = P.NP * 128;
    P.qbytes = P.nkb * R * 128;  // the window rows' query copies (tensor copies count whole boxes)
    const bool tf32 = kind != KIND_BF16;
    int off = 1024;  // barriers, tensor-memory address, abort flag
    P.off_qhi = off;
    off += P.nkb * P.q_atom;
    P.off_qlo = off;
    if (tf32) off += P.nkb * P.q_atom;
    P.off_stg = off;
    if (kind == KIND_Q8) off += align1k(128 * kQ8Row);
    P.off_epi = off;  // pass 0: transpose buffers and quarter statistics
    off += align1k(8 * 16 * kTbStride * 4 + 4 * 128 * 8);
    P.off_epi1 = off;  // pass 1: row statistics, quarter weights, partial sums
    off += 8192;
    P.off_lo = off;
    if (tf32) off += kLoStages * kStageB;
    P.off_raw = off;
    const int room = kSmemMax - 1024 - off;  // 1 KB of slack aligns the base
    P.S = room / kStageB < kMaxStages ? room / kStageB : kMaxStages;
    P.total = off + P.S * kStageB;
    return P;
}

// mbarrier slots in the header
struct Bars {
    uint64_t *raw_full, *raw_empty, *lo_full, *lo_empty, *acc_full, *acc_empty, *q_full, *q_empty, *mma_done, *q_raw;
};
__device__ __forceinline__ Bars bars_of(uint8_t* sm) {
    uint64_t* b = reinterpret_cast<uint64_t*>(sm);
    return Bars{b, b + 8, b + 16, b + 20, b + 24, b + 26, b + 28, b + 29, b + 30, b + 31};
}

__device__ __forceinline__ void work_unit(const EvictArgs& a, int w, int& b, int& hc, int& tile) {
    tile = w % a.ntiles;
    const int t = w / a.ntiles;
    hc = t % a.head_count;
    b = t / a.head_count;
}

// 16-byte chunk c of row r of a 128-byte-swizzled operand block
__device__ __forceinline__ int sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// One q8_0 block (fp16 scale + 32 int8, as 17 16-bit words) -> 32 exact fp32
// values x, stored as row r of the swizzled blocks: x itself (the TF32 read
// takes its top bits) and lo = x - hi.
__device__ __forceinline__ void q8_block_store(const uint16_t (&wv)[17], uint8_t* hi, uint8_t* lo, int r) {
    const float s = __half2float(__ushort_as_half(wv[0]));
    const float2 s2 = make_float2(s, s);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float2 a = __fmul2_rn(s2, i8x2_to_f2(wv[1 + 2 * c]));  // fp16 x int8: exact in fp32
        const float2 b = __fmul2_rn(s2, i8x2_to_f2(wv[2 + 2 * c]));
        const float2 ah = make_float2(__uint_as_float(__float_as_uint(a.x) & 0xFFFFE000u),
                                      __uint_as_float(__float_as_uint(a.y) & 0xFFFFE000u));
        const float2 bh = make_float2(__uint_as_float(__float_as_uint(b.x) & 0xFFFFE000u),
                                      __uint_as_float(__float_as_uint(b.y) & 0xFFFFE000u));
        const float2 al = __fadd2_rn(a, make_float2(-ah.x, -ah.y)), bl = __fadd2_rn(b, make_float2(-bh.x, -bh.y));
        *reinterpret_cast<float4*>(hi + sw128(r, c)) = make_float4(a.x, a.y, b.x, b.y);
        *reinterpret_cast<float4*>(lo + sw128(r, c)) = make_float4(al.x, al.y, bl.x, bl.y);
    }
}

// Grid-wide barrier of the one-launch form (a cooperative launch: every CTA
// is resident).  Bounded; a timeout records RKV_ERR_DEVICE_TIMEOUT.
__device__ __forceinline__ bool grid_barrier(unsigned* cnt, unsigned n, int* err, volatile int* abort) {
    __threadfence();
    atomicAdd(cnt, 1u);
    const long long t0 = clock64();
    for (;;) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
        if (v >= n) break;
        if (*abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            atomicExch(err, (int)RKV_ERR_DEVICE_TIMEOUT);
            *abort = 1;
            return false;
        }
        __nanosleep(200);
    }
    __threadfence();
    return true;
}

// This CTA's work units [w0, w0 + nt).  With at least as many CTAs as
// (item, KV head) pairs every CTA takes tiles of one head only (the CTAs of a
// head split its tiles evenly), so the resident window queries are loaded once;
// else contiguous ranges.
__device__ __forceinline__ void cta_range(const TcPlan& P, int ntiles, int& w0, int& nt) {
    const int G = gridDim.x, c = blockIdx.x;
    if (P.nheads <= G) {
        const int base = G / P.nheads, extra = G % P.nheads;  // the first `extra` heads get base + 1 CTAs
        int h, j, m;
        if (c < extra * (base + 1)) {
            h = c / (base + 1), j = c % (base + 1), m = base + 1;
        } else {
            const int c2 = c - extra * (base + 1);
            h = extra + c2 / base, j = c2 % base, m = base;
        }
        const int t0 = (int)((long long)j * ntiles / m), t1 = (int)((long long)(j + 1) * ntiles / m);
        w0 = h * ntiles + t0;
        nt = t1 - t0;
    } else {
        w0 = (int)((long long)c * P.nwork / G);
        nt = (int)((long long)(c + 1) * P.nwork / G) - w0;
    }
}

template <int KIND>
__global__ void __launch_bounds__(kTcThreads, 1)
    evict_tc_kernel(const EvictArgs a, const TcPlan P, const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmq) {
    asm volatile("griddepcontrol.launch_dependents;");  // the pooling may be scheduled (it waits for this grid)
    constexpr bool TF32 = KIND != KIND_BF16;
    constexpr bool TMA = KIND != KIND_Q8;
    constexpr int EB = KIND == KIND_BF16 ? 2 : 4;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const Bars B = bars_of(sm);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 256);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + 260);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int w0, nt;
    cta_range(P, a.ntiles, w0, nt);
    // visits of the copy / convert / MMA pipeline: pass 0's tiles in order, then (recompute form) pass 1's
    // in reverse, so that pass 1 starts on the tiles pass 0 read last (still in L2)
    const int nv0 = P.p0 == 0 ? nt : 0, nv1 = (P.rc && P.p1 == 1) ? nt : 0, nv = nv0 + nv1;
    auto wof = [&](int v) { return w0 + (v < nv0 ? v : nt - 1 - (v - nv0)); };
    const int S = P.S;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&B.raw_full[i], 1);
            mbar_init(&B.raw_empty[i], 1);
        }
        for (int i = 0; i < kLoStages; ++i) {
            mbar_init(&B.lo_full[i], 128);
            mbar_init(&B.lo_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&B.acc_full[i], 1);
            mbar_init(&B.acc_empty[i], kEpiThreads);
        }
        mbar_init(B.q_full, 128);
        mbar_init(B.q_empty, 1);
        mbar_init(B.mma_done, 1);
        mbar_init(B.q_raw, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tslot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        // ---------------- TMA producer (the whole warp; one elected lane issues) ----------------
        if (TMA) {
            int issued = 0, qn = 0, prev = -1;
            bool ok = true;
            for (int i = 0; i < nv && ok; ++i) {
                int b, hc, tile;
                work_unit(a, wof(i), b, hc, tile);
                const int hk = a.head_begin + hc;
                const int head = wof(i) / a.ntiles;
                if (head != prev) {  // the window rows of this KV head's query group (rocket.cpp:85-90)
                    if (qn > 0 && !__all_sync(0xffffffffu, mbar_wait_or_abort(B.q_empty, (uint32_t)((qn - 1) & 1), a.err, abort_flag)))
                        break;
                    mbar_arrive_expect_tx_w(B.q_raw, (uint32_t)P.qbytes);
                    for (int g = 0; g < a.G; ++g)
                        for (int kb = 0; kb < P.nkb; ++kb)
                            tma_load_4d_w(sm + P.off_qhi + kb * P.q_atom + g * a.obs_w * 128, &tmq, kb * (128 / EB),
                                          a.q_row0, hk * a.G + g, b, B.q_raw);
                    ++qn;
                    prev = head;
                }
                const int y = hk * a.k_head_rows + tile * kMmaM;
                for (int kb = 0; kb < P.nkb; ++kb) {
                    const int g = i * P.nkb + kb, s = g % S;
                    if (g >= S && !__all_sync(0xffffffffu, mbar_wait_or_abort(&B.raw_empty[s], (uint32_t)(((g / S) + 1) & 1),
                                                                                a.err, abort_flag))) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx_w(&B.raw_full[s], kStageB);
                    tma_load_3d_w(sm + P.off_raw + s * kStageB, &tmk, kb * (128 / EB), y, b, &B.raw_full[s]);
                    ++issued;
                }
            }
            // every copy issued lands before the CTA can exit
            for (int g = issued > S ? issued - S : 0; g < issued; ++g)
                mbar_wait_bounded(&B.raw_full[g % S], (uint32_t)((g / S) & 1), a.err);
            if (qn > 0) mbar_wait_bounded(B.q_raw, (uint32_t)((qn - 1) & 1), a.err);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (the whole warp; one elected lane issues) ----------------
        {
            const uint32_t idesc = mma_idesc(TF32 ? 2u : 1u, (uint32_t)P.NP);
            int qn = 0, prev = -1;
            bool ok = true;
            for (int i = 0; i < nv && ok; ++i) {
                const int head = wof(i) / a.ntiles;
                if (head != prev) {
                    if (!__all_sync(0xffffffffu, mbar_wait_or_abort(B.q_full, (uint32_t)(qn & 1), a.err, abort_flag))) break;
                    ++qn;
                    prev = head;
                }
                const int ab = i & 1;
                if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait_or_abort(&B.acc_empty[ab], (uint32_t)(((i >> 1) + 1) & 1),
                                                                             a.err, abort_flag)))
                    break;
                tc_fence_after();
                const uint32_t dacc = tbase + (uint32_t)(ab * kAccCols);
                for (int kb = 0; kb < P.nkb; ++kb) {
                    const int g = i * P.nkb + kb, s = g % S, l = g % kLoStages;
                    const bool w = TF32 ? mbar_wait_or_abort(&B.lo_full[l], (uint32_t)((g / kLoStages) & 1), a.err, abort_flag)
                                        : mbar_wait_or_abort(&B.raw_full[s], (uint32_t)((g / S) & 1), a.err, abort_flag);
                    if (!__all_sync(0xffffffffu, w)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t kh = smem_u32(sm + P.off_raw + s * kStageB);
                    const uint32_t kl = smem_u32(sm + P.off_lo + l * kStageB);
                    const uint32_t qh = smem_u32(sm + P.off_qhi + kb * P.q_atom);
                    const uint32_t ql = smem_u32(sm + P.off_qlo + kb * P.q_atom);
                    const int rem = (P.rowb - kb * 128) / 32;
                    const int steps = rem < 4 ? rem : 4;
                    // a K step of 32 bytes adds 2 to the descriptors' start-address field
                    const uint64_t dKh = mma_desc_sw128(kh), dKl = mma_desc_sw128(kl);
                    const uint64_t dQh = mma_desc_sw128(qh), dQl = mma_desc_sw128(ql);
                    for (int st = 0; st < steps; ++st) {
                        const uint64_t o = (uint64_t)(2 * st);
                        mma_issue_w<TF32>(dacc, dKh + o, dQh + o, idesc, (kb | st) ? 1u : 0u);
                        if (TF32) {
                            mma_issue_w<TF32>(dacc, dKh + o, dQl + o, idesc, 1u);
                            mma_issue_w<TF32>(dacc, dKl + o, dQh + o, idesc, 1u);
                        }
                    }
                    mma_commit_w(&B.raw_empty[s]);
                    if (TF32) mma_commit_w(&B.lo_empty[l]);
                }
                if (!ok) break;
                mma_commit_w(&B.acc_full[ab]);
                if (i + 1 == nv || wof(i + 1) / a.ntiles != head) mma_commit_w(B.q_empty);
            }
            // every MMA issued completes before the tensor memory is freed
            mma_commit_w(B.mma_done);
            mbar_wait_bounded(B.mma_done, 0u, a.err);
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------- operand converters ----------------
        const int ct = tid - 64;
        int qn = 0, prev = -1;
        uint8_t* qhi = sm + P.off_qhi;
        uint8_t* qlo = sm + P.off_qlo;
        // the padding rows R .. NP-1 of the query blocks stay zero
        for (int p = ct; p < P.nkb * (P.NP - a.R) * 8; p += 128) {
            const int kb = p / ((P.NP - a.R) * 8), u = p % ((P.NP - a.R) * 8);
            const int off = kb * P.q_atom + a.R * 128 + u * 16;
            *reinterpret_cast<uint4*>(qhi + off) = make_uint4(0u, 0u, 0u, 0u);
            if (TF32) *reinterpret_cast<uint4*>(qlo + off) = make_uint4(0u, 0u, 0u, 0u);
        }
        uint2 pre[KIND == KIND_Q8 ? kQ8Words : 1];
        auto q8_fetch = [&](int i) {  // tile i of this CTA -> registers (coalesced 8-byte loads)
            if (KIND != KIND_Q8) return;
            int b, hc, tile;
            work_unit(a, wof(i), b, hc, tile);
            const int k0 = tile * kMmaM;
            const int nkeys = min(kMmaM, a.nk - k0);
            const uint2* src = reinterpret_cast<const uint2*>(a.K + (size_t)b * a.k_stride +
                                                              ((size_t)(a.head_begin + hc) * a.k_head_rows + k0) * kQ8Row);
            const int nw = nkeys * kQ8Row / 8;
#pragma unroll
            for (int j = 0; j < kQ8Words; ++j) {
                const int idx = ct + 128 * j;
                pre[j] = idx < nw ? ldg_nc_v2_pinned(src + idx) : make_uint2(0u, 0u);
            }
        };
        if (KIND == KIND_Q8 && nv > 0) q8_fetch(0);
        for (int i = 0; i < nv; ++i) {
            int b, hc, tile;
            work_unit(a, wof(i), b, hc, tile);
            const int head = wof(i) / a.ntiles;
            if (head != prev) {
                if (TMA) {
                    // the producer's query copies have landed: the low parts of fp32 rows
                    const bool ok = mbar_wait_or_abort(B.q_raw, (uint32_t)(qn & 1), a.err, abort_flag);
                    if (!group_all(kBarConv, 128, ok)) break;
                    if (TF32) {
                        const int per = a.R * 8;  // 16-byte units of the window rows in one query block
                        for (int p0 = 0; p0 < P.nkb * per; p0 += 8 * 128) {
                            uint4 x[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const int p = p0 + ct + 128 * j;
                                if (p < P.nkb * per)
                                    x[j] = *reinterpret_cast<const uint4*>(qhi + (p / per) * P.q_atom + (p % per) * 16);
                            }
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const int p = p0 + ct + 128 * j;
                                if (p < P.nkb * per)
                                    *reinterpret_cast<uint4*>(qlo + (p / per) * P.q_atom + (p % per) * 16) = tf32_lo(x[j]);
                            }
                        }
                    }
                } else {
                    const bool ok = qn == 0 || mbar_wait_or_abort(B.q_empty, (uint32_t)((qn - 1) & 1), a.err, abort_flag);
                    if (!group_all(kBarConv, 128, ok)) break;
                    // q8_0 window rows: every load of a round in flight first (rocket.cpp:85-90)
                    const int hk = a.head_begin + hc;
                    const uint8_t* Qb = a.Q + (size_t)b * a.q_stride;
                    const int npairs = a.R * P.nkb;
                    for (int p0 = 0; p0 < npairs; p0 += 3 * 128) {
                        uint16_t wv[3][17];
#pragma unroll
                        for (int j = 0; j < 3; ++j) {
                            const int p = p0 + ct + 128 * j;
                            if (p < npairs) {
                                const int r = p / P.nkb, kb = p % P.nkb;
                                const int h = hk * a.G + r / a.obs_w, pos = a.q_row0 + r % a.obs_w;
                                const uint16_t* src = reinterpret_cast<const uint16_t*>(
                                    Qb + ((size_t)h * a.q_head_rows + pos) * kQ8Row + kb * 34);
#pragma unroll
                                for (int t = 0; t < 17; ++t) wv[j][t] = __ldg(src + t);
                            }
                        }
#pragma unroll
                        for (int j = 0; j < 3; ++j) {
                            const int p = p0 + ct + 128 * j;
                            if (p < npairs) {
                                const int r = p / P.nkb, kb = p % P.nkb;
                                q8_block_store(wv[j], qhi + kb * P.q_atom, qlo + kb * P.q_atom, r);
                            }
                        }
                    }
                }
                fence_proxy_async();
                mbar_arrive1(B.q_full);
                ++qn;
                prev = head;
            }
            if (KIND == KIND_BF16) continue;
            if (KIND == KIND_Q8) {
                uint2* stg = reinterpret_cast<uint2*>(sm + P.off_stg);
#pragma unroll
                for (int j = 0; j < kQ8Words; ++j) stg[ct + 128 * j] = pre[j];
                group_sync(kBarConv, 128);
                if (i + 1 < nv) q8_fetch(i + 1);
            }
            bool ok = true;
            for (int kb = 0; kb < P.nkb; ++kb) {
                const int g = i * P.nkb + kb, s = g % S, l = g % kLoStages;
                uint8_t* raw = sm + P.off_raw + s * kStageB;
                uint8_t* lo = sm + P.off_lo + l * kStageB;
                bool w = true;
                if (KIND == KIND_F32)
                    w = mbar_wait_or_abort(&B.raw_full[s], (uint32_t)((g / S) & 1), a.err, abort_flag);
                else if (g >= S)
                    w = mbar_wait_or_abort(&B.raw_empty[s], (uint32_t)(((g / S) + 1) & 1), a.err, abort_flag);
                if (w && g >= kLoStages)
                    w = mbar_wait_or_abort(&B.lo_empty[l], (uint32_t)(((g / kLoStages) + 1) & 1), a.err, abort_flag);
                if (!group_all(kBarConv, 128, w)) {
                    ok = false;
                    break;
                }
                if (KIND == KIND_F32) {
                    // lo of the stage the producer landed (the swizzle is elementwise-neutral)
                    uint4 x[kStageB / 16 / 128];
#pragma unroll
                    for (int j = 0; j < kStageB / 16 / 128; ++j) x[j] = *reinterpret_cast<const uint4*>(raw + (ct + 128 * j) * 16);
#pragma unroll
                    for (int j = 0; j < kStageB / 16 / 128; ++j) *reinterpret_cast<uint4*>(lo + (ct + 128 * j) * 16) = tf32_lo(x[j]);
                } else {
                    // row ct, q8_0 block kb (one k-block of 32 fp32 values)
                    const uint16_t* h = reinterpret_cast<const uint16_t*>(sm + P.off_stg + ct * kQ8Row + kb * 34);
                    uint16_t wv[17];
#pragma unroll
                    for (int t = 0; t < 17; ++t) wv[t] = h[t];
                    q8_block_store(wv, raw, lo, ct);
                }
                fence_proxy_async();
                mbar_arrive1(&B.lo_full[l]);
            }
            if (!ok) break;
            if (KIND == KIND_Q8) group_sync(kBarConv, 128);  // the staging area is refilled next
        }
    } else {
        // ---------------- epilogue ----------------
        const int ep = warp - 6, et = tid - 192, q = warp & 3, kk = q * 32 + lane;
        const int hf = ep >> 2;  // which half of the window rows this warp takes
        const int nch = P.NP / 16, cmid = (nch + 1) / 2;
        const int c0 = hf ? cmid : 0, c1 = hf ? nch : cmid;
        float* tb = reinterpret_cast<float*>(sm + P.off_epi) + ep * 16 * kTbStride;
        float2* part = reinterpret_cast<float2*>(sm + P.off_epi + 8 * 16 * kTbStride * 4);  // [4][128]
        float* rsm = reinterpret_cast<float*>(sm + P.off_epi1);          // pass 1: row max M_r [128]
        float* rsi = reinterpret_cast<float*>(sm + P.off_epi1 + 512);    // pass 1: 1 / (row sum + 1e-9) [128]
        float* csm = reinterpret_cast<float*>(sm + P.off_epi1 + 1024);   // pass 1: [128][4] quarter weights
        float* red = reinterpret_cast<float*>(sm + P.off_epi1 + 3072);   // pass 1: [8][128] partial sums
        bool ok = true;
        // ---- pass 0: per-(row, tile) max and sum of exp(l - max) (rocket.cpp:91-107); unless pass 1
        // recomputes, every exp(l - quarter max) is kept (fp32, rows of nkp) with the quarter maxima
        for (int i = 0; i < nv0 && ok; ++i) {
            int b, hc, tile;
            work_unit(a, wof(i), b, hc, tile);
            const int k0 = tile * kMmaM, nkeys = min(kMmaM, a.nk - k0);
            const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
            const int ab = i & 1;
            const bool w = mbar_wait_or_abort(&B.acc_full[ab], (uint32_t)((i >> 1) & 1), a.err, abort_flag);
            if (!group_all(kBarEpi, kEpiThreads, w)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t trow = tbase + (uint32_t)(ab * kAccCols) + ((uint32_t)(q * 32) << 16);
            const int row = lane & 15, kh = lane >> 4;
            for (int c = c0; c < c1; ++c) {
                float v[16];
                tmem_ld16(trow + (uint32_t)(c * 16), v);
#pragma unroll
                for (int j = 0; j < 16; ++j) tb[j * kTbStride + lane] = kk < nkeys ? v[j] * a.inv_sqrt_d : -INFINITY;
                __syncwarp();
                // row c*16 + row, 16 of this warp's keys
                const float4* rv4 = reinterpret_cast<const float4*>(tb + row * kTbStride + kh * 16);
                float rv[16];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float4 f = rv4[t];
                    rv[4 * t] = f.x;
                    rv[4 * t + 1] = f.y;
                    rv[4 * t + 2] = f.z;
                    rv[4 * t + 3] = f.w;
                }
                float m = -FLT_MAX;  // rocket.cpp:93
#pragma unroll
                for (int t = 0; t < 16; ++t) m = fmaxf(m, rv[t]);
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
                float e[16];
                float s = 0.0f;
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const float2 x = mufu_expf2(__fadd2_rn(make_float2(rv[2 * t], rv[2 * t + 1]), make_float2(-m, -m)));
                    e[2 * t] = x.x;
                    e[2 * t + 1] = x.y;
                    s += x.x;
                    s += x.y;
                }
                s += __shfl_xor_sync(0xffffffffu, s, 16);
                const int r = c * 16 + row;
                if (kh == 0) {
                    part[q * 128 + r] = make_float2(m, s);
                    if (r < a.R && !P.rc) __stcg(a.qmax + ((row_base + r) * a.ntiles + tile) * 4 + q, m);
                }
                if (P.rc) {  // nothing kept: pass 1 recomputes
                    __syncwarp();  // the transpose buffer is rewritten next
                    continue;
                }
                // the exp values back through the transpose buffer, then one row per store
                // instruction: 32 consecutive keys, 128 contiguous bytes
                float4* eo = reinterpret_cast<float4*>(tb + row * kTbStride + kh * 16);
#pragma unroll
                for (int t = 0; t < 4; ++t) eo[t] = make_float4(e[4 * t], e[4 * t + 1], e[4 * t + 2], e[4 * t + 3]);
                __syncwarp();
                if (kk < nkeys) {
                    float* ecol = a.logits + (row_base + c * 16) * (size_t)a.nkp + k0 + kk;
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (c * 16 + j < a.R) __stcg(ecol + (size_t)j * a.nkp, tb[j * kTbStride + lane]);
                }
                __syncwarp();
            }
            tc_fence_before();
            mbar_arrive1(&B.acc_empty[ab]);
            group_sync(kBarEpi, kEpiThreads);
            if (et < a.R) {  // combine the four 32-key quarters of the tile
                float M = -FLT_MAX;
#pragma unroll
                for (int t = 0; t < 4; ++t) M = fmaxf(M, part[t * 128 + et].x);
                float Ssum = 0.0f;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float2 p = part[t * 128 + et];
                    Ssum += p.y * det_expf(p.x - M);
                }
                __stcg(a.tstats + (row_base + et) * a.ntiles + tile, make_float2(M, Ssum));
            }
            group_sync(kBarEpi, kEpiThreads);
        }
        // ---- the row fold (rocket.cpp:108-113): row max M_r over the tiles and
        // inv_r = 1 / (sum_t s_t exp(m_t - M_r) + 1e-9), one warp per row with every load in flight
        // first.  In one launch the rows of all heads are spread over all CTAs between two grid
        // barriers; a launch of pass 1 alone folds its own heads' rows.
        auto fold_row = [&](size_t x, float& M, float& inv) {  // x: row of the [item][head][R] statistics
            const float2* ts = a.tstats + x * a.ntiles;
            float2 v[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int ti = lane + 32 * t;
                v[t] = ti < a.ntiles ? __ldcg(ts + ti) : make_float2(-FLT_MAX, 0.0f);
            }
            M = -FLT_MAX;
#pragma unroll
            for (int t = 0; t < 4; ++t) M = fmaxf(M, v[t].x);
            for (int ti = lane + 128; ti < a.ntiles; ti += 32) M = fmaxf(M, __ldcg(ts + ti).x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float Ssum = 0.0f;
#pragma unroll
            for (int t = 0; t < 4; ++t) Ssum += v[t].y * expf(v[t].x - M);
            for (int ti = lane + 128; ti < a.ntiles; ti += 32) {
                const float2 w2 = __ldcg(ts + ti);
                Ssum += w2.y * expf(w2.x - M);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) Ssum += __shfl_xor_sync(0xffffffffu, Ssum, o);
            inv = 1.0f / (Ssum + 1e-9f);
        };
        const bool one_launch = P.p0 == 0 && P.p1 == 1;
        if (ok && one_launch) {
            // every CTA's statistics are written before any row folds them
            group_sync(kBarEpi, kEpiThreads);
            bool gb = true;
            if (et == 0) gb = grid_barrier(a.gbar, gridDim.x, a.err, abort_flag);
            ok = group_all(kBarEpi, kEpiThreads, gb);
            if (ok) {
                const size_t nrows = (size_t)P.nheads * a.R;
                for (size_t x = blockIdx.x + (size_t)gridDim.x * ep; x < nrows; x += (size_t)gridDim.x * 8) {
                    float M, inv;
                    fold_row(x, M, inv);
                    if (lane == 0) __stcg(a.rstats + x, make_float2(M, inv));
                }
                group_sync(kBarEpi, kEpiThreads);
                if (et == 0) gb = grid_barrier(a.gbar, 2u * gridDim.x, a.err, abort_flag);
                ok = group_all(kBarEpi, kEpiThreads, gb);
            }
        }
        int prev = -1;
        // ---- pass 1, recompute form: head scores sum_r exp(l - M_r) * inv_r (rocket.cpp:114-116) from
        // the logits in tensor memory.  A thread holds one key (its lane) and the rows of its chunks, so
        // the sum over the rows needs no transpose; the two warps of a lane quarter add their halves.
        for (int v = nv0; ok && v < nv; ++v) {
            int b, hc, tile;
            work_unit(a, wof(v), b, hc, tile);
            const int head = wof(v) / a.ntiles;
            const int k0 = tile * kMmaM, nkeys = min(kMmaM, a.nk - k0);
            const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
            if (head != prev) {
                group_sync(kBarEpi, kEpiThreads);  // the previous head's statistics are no longer read
                // padding rows (zero queries): M = FLT_MAX and inv = 0 make their terms exactly 0
                if (one_launch) {
                    for (int r = et; r < P.NP; r += kEpiThreads) {
                        const float2 x = r < a.R ? __ldcg(a.rstats + row_base + r) : make_float2(FLT_MAX, 0.0f);
                        rsm[r] = x.x;
                        rsi[r] = x.y;
                    }
                } else {
                    for (int r = ep; r < P.NP; r += 8) {
                        float M = FLT_MAX, inv = 0.0f;
                        if (r < a.R) fold_row(row_base + r, M, inv);
                        if (lane == 0) {
                            rsm[r] = M;
                            rsi[r] = r < a.R ? inv : 0.0f;
                        }
                    }
                }
                group_sync(kBarEpi, kEpiThreads);
                prev = head;
            }
            const int ab = v & 1;
            const bool w = mbar_wait_or_abort(&B.acc_full[ab], (uint32_t)((v >> 1) & 1), a.err, abort_flag);
            if (!group_all(kBarEpi, kEpiThreads, w)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t trow = tbase + (uint32_t)(ab * kAccCols) + ((uint32_t)(q * 32) << 16);
            float hsum = 0.0f;
            for (int c = c0; c < c1; ++c) {
                float x[16];
                tmem_ld16(trow + (uint32_t)(c * 16), x);
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    const int r = c * 16 + j;  // rows r, r + 1 (the padding rows have inv 0)
                    const float2 e = mufu_expf2(__fadd2_rn(__fmul2_rn(make_float2(x[j], x[j + 1]),
                                                                      make_float2(a.inv_sqrt_d, a.inv_sqrt_d)),
                                                           make_float2(-rsm[r], -rsm[r + 1])));
                    hsum = fmaf(e.x, rsi[r], hsum);
                    hsum = fmaf(e.y, rsi[r + 1], hsum);
                }
            }
            tc_fence_before();
            mbar_arrive1(&B.acc_empty[ab]);
            red[hf * 128 + kk] = hsum;
            group_sync(kBarEpi, kEpiThreads);
            if (et < 128 && et < nkeys) a.hs[((size_t)b * a.head_count + hc) * a.nk + k0 + et] = red[et] + red[128 + et];
            group_sync(kBarEpi, kEpiThreads);
        }
        // ---- pass 1: head scores sum_r exp(l - M_r) * inv_r (rocket.cpp:114-116) from the kept
        // exp(l - m_q): each term is e * (exp(m_q - M_r) * inv_r), one exp per (row, tile, quarter)
        const int kg = et & 31, rg = et >> 5;  // 4 keys (quarter kg / 8) x rows rg, rg + 8, ...
        for (int i = 0; ok && P.p1 == 1 && !P.rc && i < nt; ++i) {
            int b, hc, tile;
            work_unit(a, w0 + i, b, hc, tile);
            const int head = (w0 + i) / a.ntiles;
            const int k0 = tile * kMmaM, nkeys = min(kMmaM, a.nk - k0);
            const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
            if (head != prev) {
                if (one_launch) {
                    for (int r = et; r < P.NP; r += kEpiThreads) {
                        const float2 v = r < a.R ? __ldcg(a.rstats + row_base + r) : make_float2(-FLT_MAX, 0.0f);
                        rsm[r] = v.x;
                        rsi[r] = v.y;
                    }
                } else {
                    for (int r = ep; r < P.NP; r += 8) {
                        float M = -FLT_MAX, inv = 0.0f;
                        if (r < a.R) fold_row(row_base + r, M, inv);
                        if (lane == 0) {
                            rsm[r] = M;
                            rsi[r] = r < a.R ? inv : 0.0f;
                        }
                    }
                }
                group_sync(kBarEpi, kEpiThreads);
                prev = head;
            }
            // every load of the tile first: the quarter maxima and this thread's exp values
            const int kq = 4 * kg, qq = kg >> 3;
            float qm[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int x = et + kEpiThreads * j, r = x >> 2;
                qm[j] = (x < P.NP * 4 && r < a.R) ? __ldcg(a.qmax + ((row_base + r) * a.ntiles + tile) * 4 + (x & 3)) : -FLT_MAX;
            }
            float4 ev[16];
            const float* ebase = a.logits + row_base * (size_t)a.nkp + k0 + kq;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int r = rg + 8 * u;
                ev[u] = (r < a.R && kq < nkeys) ? __ldcg(reinterpret_cast<const float4*>(ebase + (size_t)r * a.nkp))
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            // weights of this tile: c[r][quarter] = exp(m_q - M_r) * inv_r (padding rows 0)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int x = et + kEpiThreads * j, r = x >> 2;
                if (x < P.NP * 4) csm[x] = r < a.R ? det_expf(qm[j] - rsm[r]) * rsi[r] : 0.0f;
            }
            group_sync(kBarEpi, kEpiThreads);
            float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int r = rg + 8 * u;
                const float cw = r < P.NP ? csm[r * 4 + qq] : 0.0f;
                acc0 = __ffma2_rn(make_float2(ev[u].x, ev[u].y), make_float2(cw, cw), acc0);
                acc1 = __ffma2_rn(make_float2(ev[u].z, ev[u].w), make_float2(cw, cw), acc1);
            }
            *reinterpret_cast<float4*>(red + rg * 128 + kq) = make_float4(acc0.x, acc0.y, acc1.x, acc1.y);
            group_sync(kBarEpi, kEpiThreads);
            if (et < 128 && et < nkeys) {
                float h = 0.0f;
#pragma unroll
                for (int g = 0; g < 8; ++g) h += red[g * 128 + et];
                a.hs[((size_t)b * a.head_count + hc) * a.nk + k0 + et] = h;
            }
            group_sync(kBarEpi, kEpiThreads);
        }
    }

    // ---- release the tensor memory on every path ----
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tbase, kTmemCols);
}

int kind_of(int dtype) { return dtype == RKV_F32 ? KIND_F32 : dtype == RKV_BF16 ? KIND_BF16 : KIND_Q8; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 0;
    return n;
}

// K as [batch][HK * k_head_rows][D] and Q as [batch][H][q_head_rows][D]; boxes
// of 128 bytes x 128 key rows and 128 bytes x obs_w query rows, 128-byte swizzle.
template <int KIND>
int encode_maps(const EvictArgs& a, int batch, CUtensorMap* tk, CUtensorMap* tq) {
    auto enc = encode_fn();
    if (!enc) return RKV_ERR_CUDA;
    const int eb = KIND == KIND_BF16 ? 2 : 4;
    const CUtensorMapDataType dt = KIND == KIND_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const cuuint64_t rowb = (cuuint64_t)a.D * eb;
    const cuuint64_t krows = (cuuint64_t)a.HK * a.k_head_rows;
    cuuint64_t kd[3] = {(cuuint64_t)a.D, krows, (cuuint64_t)batch};
    cuuint64_t ks[2] = {rowb, batch > 1 ? (cuuint64_t)a.k_stride : krows * rowb};
    cuuint32_t kbox[3] = {(cuuint32_t)(128 / eb), (cuuint32_t)kMmaM, 1u};
    cuuint32_t e3[3] = {1u, 1u, 1u};
    if (enc(tk, dt, 3, const_cast<uint8_t*>(a.K), kd, ks, kbox, e3, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return RKV_ERR_UNSUPPORTED;
    const cuuint64_t hb = (cuuint64_t)a.q_head_rows * rowb;
    cuuint64_t qd[4] = {(cuuint64_t)a.D, (cuuint64_t)a.q_head_rows, (cuuint64_t)a.H, (cuuint64_t)batch};
    cuuint64_t qs[3] = {rowb, hb, batch > 1 ? (cuuint64_t)a.q_stride : hb * a.H};
    cuuint32_t qbox[4] = {(cuuint32_t)(128 / eb), (cuuint32_t)a.obs_w, 1u, 1u};
    cuuint32_t e4[4] = {1u, 1u, 1u, 1u};
    if (enc(tq, dt, 4, const_cast<uint8_t*>(a.Q), qd, qs, qbox, e4, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return RKV_ERR_UNSUPPORTED;
    return RKV_OK;
}

template <int KIND>
int launch_kind(const EvictArgs& a, int batch, cudaStream_t st) {
    TcPlan P = tc_plan(KIND, a.R, a.D);
    P.nwork = batch * a.head_count * a.ntiles;
    P.nheads = batch * a.head_count;
    // keep pass 0's exp values for pass 1 while they fit in L2 with room to spare, else recompute
    // the logits in pass 1 (a second read of K, from HBM, costs less than writing and reading them)
    const double kept_bytes = (double)P.nheads * a.R * a.nkp * 4.0;
    P.rc = KIND != KIND_Q8 && kept_bytes > 48.0 * 1024 * 1024 ? 1 : 0;
    const int sms = sm_count();
    if (sms <= 0) return RKV_ERR_CUDA;
    const int grid = P.nwork < sms ? P.nwork : sms;
    CUtensorMap tk, tq;
    memset(&tk, 0, sizeof(tk));
    memset(&tq, 0, sizeof(tq));
    if (KIND != KIND_Q8) {
        const int rc = encode_maps<KIND>(a, batch, &tk, &tq);
        if (rc) return rc;
    }
    auto f = evict_tc_kernel<KIND>;
    const int smem = P.total + 1024;
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return RKV_ERR_CUDA;
    // both passes in one cooperative launch (one CTA per SM, all resident: the grid barrier between the
    // passes cannot wait on a CTA that has not started) ...
    P.p0 = 0;
    P.p1 = 1;
    void* args[] = {const_cast<EvictArgs*>(&a), &P, &tk, &tq};
    const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(f), dim3(grid), dim3(kTcThreads),
                                                      args, (size_t)smem, st);
    if (e == cudaSuccess) return RKV_OK;
    (void)cudaGetLastError();
    if (e != cudaErrorCooperativeLaunchTooLarge && e != cudaErrorNotSupported) return RKV_ERR_CUDA;
    // ... else one launch per pass
    for (int pass = 0; pass < 2; ++pass) {
        P.p0 = P.p1 = pass;
        f<<<grid, kTcThreads, smem, st>>>(a, P, tk, tq);
        if (cudaGetLastError() != cudaSuccess) return RKV_ERR_CUDA;
    }
    return RKV_OK;
}

}  // namespace

bool evict_tc_supported(const EvictArgs& a, int batch) {
    if (a.R <= 0 || a.R > 128 || a.ntiles <= 0 || batch <= 0) return false;
    if (a.dtype != RKV_F32 && a.dtype != RKV_BF16 && a.dtype != RKV_Q8_0) return false;
    const int kind = kind_of(a.dtype);
    if (tc_plan(kind, a.R, a.D).S < 2) return false;
    const uintptr_t qa = reinterpret_cast<uintptr_t>(a.Q), ka = reinterpret_cast<uintptr_t>(a.K);
    if (kind == KIND_Q8) {
        if (a.D != 128) return false;  // 136-byte rows: 8-byte aligned tiles
        if ((ka & 7) || (a.k_stride & 7) || (qa & 1) || (a.q_stride & 1)) return false;
        return true;
    }
    const long long rowb = (long long)a.D * (kind == KIND_BF16 ? 2 : 4);
    if (rowb % 32 != 0) return false;                  // whole MMA K steps
    if (a.obs_w % 8 != 0) return false;                // query copies land on 1024-byte swizzle groups
    if ((ka & 15) || (qa & 15)) return false;          // tensor-map base addresses
    if (batch > 1 && (a.k_stride <= 0 || (a.k_stride & 15) || a.q_stride <= 0 || (a.q_stride & 15))) return false;
    return true;
}

int launch_evict_tc(const EvictArgs& a, int batch, cudaStream_t st) {
    switch (kind_of(a.dtype)) {
        case KIND_F32: return launch_kind<KIND_F32>(a, batch, st);
        case KIND_BF16: return launch_kind<KIND_BF16>(a, batch, st);
        default: return evict_q8_supported(a, batch) ? launch_evict_q8(a, batch, st) : launch_kind<KIND_Q8>(a, batch, st);
    }
}

}  // namespace rkv
