// evict_tc.cu -- persistent, warp-specialised stage-1 scoring on the tcgen05
// tensor cores (sm_100a): the default engine for fp32, bf16 and q8_0 where
// the window rows fit in one MMA (G * obs_w <= 128) and the shared-memory
// plan fits.  evict_mma.cu keeps the non-persistent kernel for the rest.
//
// One CTA per SM walks a contiguous range of (item, KV head, 128-key tile)
// work units.  Per tile the contraction D[128 query rows][128 keys] =
// Q . K_tile^T accumulates in tensor memory (the window rows, G * obs_w of
// them, on the lanes; lanes past them are not used), cycling through four
// accumulators so the epilogue of a tile overlaps the MMAs of the next ones.  The
// reduction dimension is walked in "k-blocks" of 128 bytes of operand row (32
// fp32 or 64 bf16 values; a q8_0 block of 32 values is one fp32 k-block after
// dequantisation).  Shared-memory operands use the K-major 128-byte-swizzle
// layout of tcgen05.
//
// fp32 (and dequantised q8_0) runs as three TF32 products per K step,
// hi.hi + lo.hi + hi.lo: the tensor core reads the top 19 bits of an fp32
// operand (hi), and lo = x - hi is exact, so the logits carry close to fp32
// accuracy.  bf16 runs one bf16 product (exact products, fp32 accumulation).
//
// Warp roles (704 threads):
//   warp 0      TMA producer (fp32, bf16): the window queries of each KV
//               head (one tensor copy per query head and k-block, into the
//               resident query block) and one copy per k-block of 128 key
//               rows into a ring of 16 KB stages;
//   warp 1      allocates tensor memory; issues the MMAs and the
//               tcgen05.commit arrivals that release stages and accumulators
//               (bf16: warps 1 and 2, taking the tiles in turn).
//               Warps 0 and 1 run their loops converged and one lane, picked
//               by elect.sync inside each issuing statement, issues: the
//               operands stay warp-uniform, which keeps the issue of a copy or
//               an MMA at a few cycles instead of ~100 (measured);
//   warps 2-5   operand converters (3-5 for bf16, which only forwards the
//               window queries' arrival): lo = x - hi of every fp32 k-block and
//               query block; q8_0 tiles loaded with coalesced 8-byte loads and
//               dequantised exactly to fp32 in shared memory (x and lo), the
//               q8_0 window queries likewise;
//   warps 6-21  epilogue, four groups of four that take the tiles in turn (one
//               accumulator each); warp w reads lanes 32 (w % 4) .. 32 (w % 4)
//               + 31, so a thread holds one window row's 128 logits of a tile
//               (pass 0) or one key's logits of every window row (pass 1).
//
// Two passes over the CTA's tiles (rocket.cpp:91-116).  Pass 0: a thread
// forms its row's max and sum of exp(l - max) over the tile, l = (q . k) /
// sqrt(D), with no exchange between threads.  The epilogue then folds a
// head's tile statistics into the row max M_r and inv_r = 1 / (sum_r + 1e-9)
// (rocket.cpp:108-113).  Pass 1 runs the copies and MMAs again, over the tiles
// in reverse order (its first tiles are the ones pass 0 read last, still in
// L2), with the operands swapped so that the keys sit on the lanes (D[128
// keys][NP rows] = K_tile . Q^T), and writes the head score of every key,
// sum_r exp(l - M_r) * inv_r, for the pooling kernel: a thread adds its key's
// terms in row order, as the reference does.  Both passes run in one cooperative launch when every
// CTA can be resident: a bounded grid barrier between them holds only the
// epilogue while the copies and MMAs of pass 1 already run; otherwise one
// launch per pass.
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
#include <type_traits>

namespace rkv {
namespace {

constexpr int kTcThreads = 704;
constexpr int kAccs = 4;            // tensor-memory accumulators, one per epilogue group
constexpr int kEpiThreads = 128 * kAccs;  // warps 6-21
constexpr int kStageB = 128 * 128;  // one operand stage: 128 rows x 128 bytes
constexpr int kMaxStages = 8;
constexpr int kLoStages = 2;
constexpr int kAccCols = 128;       // tensor-memory columns per accumulator
constexpr int kTmemCols = kAccs * kAccCols;
constexpr int kBarConv = 1, kBarGrp = 2, kBarEpiAll = 2 + kAccs;  // named barriers: converters, epilogue groups, all epilogue warps
constexpr int kSmemMax = 227 * 1024;  // dynamic shared memory per CTA on sm_100
constexpr int kQ8Row = 136;           // bytes of one q8_0 row of 128 values
constexpr int kQ8Words = 128 * kQ8Row / 8 / 128;  // 8-byte words per converter thread of a q8_0 tile (17)

enum { KIND_F32 = 0, KIND_BF16 = 1, KIND_Q8 = 2 };

struct TcPlan {  // shared-memory offsets from the 1024-byte aligned base, and the work split
    int NP, nkb, rowb, S, q_atom, qbytes;
    int off_qhi, off_qlo, off_stg, off_epi, off_lo, off_raw, total;
    int nwork, nheads;  // work units (128-key tiles) and (item, KV head) pairs
    int aligned;        // split the tiles head by head (cta_range)
    int p0, p1;         // the passes this launch runs: 0 = scores and statistics, 1 = head scores
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
    // the MMA reads 128 query rows; rows NP .. 127 fall on what follows the query block (these bytes, the
    // low-part stages or the ring; their accumulator lanes are not used)
    P.off_epi = off;  // pass 1: per epilogue group, the window rows' (-M_r log2 e, inv_r) by row pairs
    off += kAccs * 128 * 8;
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
    return Bars{b, b + 8, b + 16, b + 20, b + 24, b + 24 + kAccs, b + 24 + 2 * kAccs, b + 25 + 2 * kAccs,
                b + 26 + 2 * kAccs, b + 27 + 2 * kAccs};
}

__device__ __forceinline__ void work_unit(const EvictArgs& a, int w, int& b, int& hc, int& tile) {
    tile = w % a.ntiles;
    const int t = w / a.ntiles;
    hc = t % a.head_count;
    b = t / a.head_count;
}

// exp(l - M) for two logits as 2^(x s2 - M log2 e), x the raw accumulator and s2 = log2(e) / sqrt(D): one
// fused multiply-add and the MUFU ex2 per value.  Its error is a few ulp of the exponent (t <= 0, relative
// error about |t| 2^-23) plus the rounding of M log2 e, a factor shared by every term of one (row, tile)
// sum or of one row's head-score terms; both lie far below the logits' own error (the fp32 accumulation of
// the dot product, and for fp32 operands the three TF32 products).  nm2 = -(M log2 e), kept finite so
// that an all -inf row gives 0, as exp(-inf - M) does.
__device__ __forceinline__ float neg_m2(float M) { return -fmaxf(M * 1.44269504088896341f, -FLT_MAX); }
__device__ __forceinline__ float2 exp2_pair(float x0, float x1, float s2, float2 nm2) {
    const float2 t = __ffma2_rn(make_float2(x0, x1), make_float2(s2, s2), nm2);
    return make_float2(ex2_approx(t.x), ex2_approx(t.y));
}

// The (sequence, KV head) of the work units a role walks through, with the division redone only when a
// unit leaves the current head's range of tiles: the per-visit loops of the copy and MMA roles are short
// serial chains, and an integer division by a runtime value is a long dependent sequence in them.
struct HeadCursor {
    int head = -1, lo = 0, hi = 0;
    __device__ __forceinline__ bool has(int w) const { return w >= lo && w < hi; }
    __device__ __forceinline__ void move(int w, int ntiles) {
        head = w / ntiles;
        lo = head * ntiles;
        hi = lo + ntiles;
    }
};

// Slot and phase parity of a ring of n stages, advanced one use at a time (slot = g % n, parity = (g / n) & 1)
struct StageRing {
    int s = 0;
    uint32_t ph = 0;
    __device__ __forceinline__ void next(int n) {
        if (++s == n) {
            s = 0;
            ph ^= 1u;
        }
    }
};

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

// This CTA's work units [w0, w0 + nt).  Head-aligned split (P.aligned, at least as many CTAs as
// (item, KV head) pairs): every CTA takes tiles of one head only (the CTAs of a head split its tiles
// evenly), so the resident window queries are loaded once; else the even split of all tiles into
// contiguous ranges, a CTA crossing at most a few head boundaries.
__device__ __forceinline__ void cta_range(const TcPlan& P, int ntiles, int& w0, int& nt) {
    const int G = gridDim.x, c = blockIdx.x;
    if (P.aligned) {
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
    // MMA issuers: bf16 needs no operand conversion, so warp 2 joins warp 1 and the two take the visits
    // in turn (one issuer's waits, fences and commits overlap the other's MMAs); fp32 and q8_0 keep all
    // four converter warps and one issuer
    constexpr int kIssuers = TF32 ? 1 : 2;
    constexpr int kConv = 128 - 32 * (kIssuers - 1);  // converter threads
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const Bars B = bars_of(sm);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 512);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + 516);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int w0, nt;
    cta_range(P, a.ntiles, w0, nt);
    // visits of the copy / convert / MMA pipeline: pass 0's tiles in order, then (recompute form) pass 1's
    // in reverse, so that pass 1 starts on the tiles pass 0 read last (still in L2)
    const int nv0 = P.p0 == 0 ? nt : 0, nv1 = P.p1 == 1 ? nt : 0, nv = nv0 + nv1;
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
        for (int i = 0; i < kAccs; ++i) {
            mbar_init(&B.acc_full[i], 1);
            mbar_init(&B.acc_empty[i], 128);  // the epilogue group of this accumulator
        }
        mbar_init(B.q_full, kConv);
        mbar_init(B.q_empty, kIssuers);
        mbar_init(B.mma_done, kIssuers);
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
            int issued = 0, qn = 0, b = 0, hk = 0;
            HeadCursor cur;
            StageRing rs;
            bool ok = true;
            for (int i = 0; i < nv && ok; ++i) {
                const int w = wof(i);
                if (!cur.has(w)) {  // the window rows of this KV head's query group (rocket.cpp:85-90)
                    cur.move(w, a.ntiles);
                    hk = a.head_begin + cur.head % a.head_count;
                    b = cur.head / a.head_count;
                    if (qn > 0 && !__all_sync(0xffffffffu, mbar_wait_or_abort(B.q_empty, (uint32_t)((qn - 1) & 1), a.err, abort_flag)))
                        break;
                    mbar_arrive_expect_tx_w(B.q_raw, (uint32_t)P.qbytes);
                    for (int g = 0; g < a.G; ++g)
                        for (int kb = 0; kb < P.nkb; ++kb)
                            tma_load_4d_w(sm + P.off_qhi + kb * P.q_atom + g * a.obs_w * 128, &tmq, kb * (128 / EB),
                                          a.q_row0, hk * a.G + g, b, B.q_raw);
                    ++qn;
                }
                const int y = hk * a.k_head_rows + (w - cur.lo) * kMmaM;
                for (int kb = 0; kb < P.nkb; ++kb) {
                    const int s = rs.s;
                    if (issued >= S &&
                        !__all_sync(0xffffffffu, mbar_wait_or_abort(&B.raw_empty[s], rs.ph ^ 1u, a.err, abort_flag))) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx_w(&B.raw_full[s], kStageB);
                    tma_load_3d_w(sm + P.off_raw + s * kStageB, &tmk, kb * (128 / EB), y, b, &B.raw_full[s]);
                    ++issued;
                    rs.next(S);
                }
            }
            // every copy issued lands before the CTA can exit
            for (int g = issued > S ? issued - S : 0; g < issued; ++g)
                mbar_wait_bounded(&B.raw_full[g % S], (uint32_t)((g / S) & 1), a.err);
            if (qn > 0) mbar_wait_bounded(B.q_raw, (uint32_t)((qn - 1) & 1), a.err);
        }
        __syncwarp();
    } else if (warp < 1 + kIssuers) {
        // ---------------- MMA issuers (whole warps; one elected lane issues) ----------------
        // Issuer j takes the visits i with i % kIssuers == j; every issuer walks all visits to follow the
        // stage ring and the KV heads (it waits for each head's window queries and releases them once
        // its own MMAs on the head are issued, so q_empty completes when every issuer has done so).
        {
            const int iss = warp - 1;
            // pass 0: D[128 query-row lanes][128 keys] = Q . K_tile^T; pass 1: D[128 key lanes][NP query rows] =
            // K_tile . Q^T (the same products with the operands swapped)
            const uint32_t idesc0 = mma_idesc(TF32 ? 2u : 1u, (uint32_t)kMmaM);
            const uint32_t idesc1 = mma_idesc(TF32 ? 2u : 1u, (uint32_t)P.NP);
            int qn = 0;
            HeadCursor cur;
            StageRing rs;
            bool ok = true;
            for (int i = 0; i < nv && ok; ++i) {
                const int w = wof(i);
                if (!cur.has(w)) {
                    if (!__all_sync(0xffffffffu, mbar_wait_or_abort(B.q_full, (uint32_t)(qn & 1), a.err, abort_flag))) break;
                    ++qn;
                    cur.move(w, a.ntiles);
                }
                if (i % kIssuers == iss) {
                    const int ab = i % kAccs;
                    if (i >= kAccs && !__all_sync(0xffffffffu, mbar_wait_or_abort(&B.acc_empty[ab], (uint32_t)(((i / kAccs) + 1) & 1),
                                                                                 a.err, abort_flag)))
                        break;
                    tc_fence_after();
                    const uint32_t dacc = tbase + (uint32_t)(ab * kAccCols);
                    for (int kb = 0; kb < P.nkb; ++kb) {
                        const int g = i * P.nkb + kb, s = rs.s, l = g % kLoStages;
                        const bool landed = TF32 ? mbar_wait_or_abort(&B.lo_full[l], (uint32_t)((g / kLoStages) & 1), a.err, abort_flag)
                                                 : mbar_wait_or_abort(&B.raw_full[s], rs.ph, a.err, abort_flag);
                        if (!__all_sync(0xffffffffu, landed)) {
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
                        const bool keys_on_lanes = i >= nv0;
                        const uint32_t idesc = keys_on_lanes ? idesc1 : idesc0;
                        auto mma = [&](uint64_t dq, uint64_t dk, uint32_t acc) {
                            mma_issue_w<TF32>(dacc, keys_on_lanes ? dk : dq, keys_on_lanes ? dq : dk, idesc, acc);
                        };
                        for (int st = 0; st < steps; ++st) {
                            const uint64_t o = (uint64_t)(2 * st);
                            mma(dQh + o, dKh + o, (kb | st) ? 1u : 0u);
                            if (TF32) {
                                mma(dQl + o, dKh + o, 1u);
                                mma(dQh + o, dKl + o, 1u);
                            }
                        }
                        mma_commit_w(&B.raw_empty[s]);
                        if (TF32) mma_commit_w(&B.lo_empty[l]);
                        rs.next(S);
                    }
                    if (!ok) break;
                    mma_commit_w(&B.acc_full[ab]);
                } else {
                    for (int kb = 0; kb < P.nkb; ++kb) rs.next(S);  // the other issuer's stages
                }
                if (i + 1 == nv || !cur.has(wof(i + 1))) mma_commit_w(B.q_empty);
            }
            // every MMA issued completes before the tensor memory is freed
            mma_commit_w(B.mma_done);
            mbar_wait_bounded(B.mma_done, 0u, a.err);
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------- operand converters ----------------
        const int ct = tid - 32 * (1 + kIssuers);
        int qn = 0, prev = -1;
        StageRing rs;
        uint8_t* qhi = sm + P.off_qhi;
        uint8_t* qlo = sm + P.off_qlo;
        // the padding rows R .. NP-1 of the query blocks stay zero
        for (int p = ct; p < P.nkb * (P.NP - a.R) * 8; p += kConv) {
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
                    if (!group_all(kBarConv, kConv, ok)) break;
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
                    if (!group_all(kBarConv, kConv, ok)) break;
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
                group_sync(kBarConv, kConv);
                if (i + 1 < nv) q8_fetch(i + 1);
            }
            bool ok = true;
            for (int kb = 0; kb < P.nkb; ++kb, rs.next(S)) {
                const int g = i * P.nkb + kb, s = rs.s, l = g % kLoStages;
                uint8_t* raw = sm + P.off_raw + s * kStageB;
                uint8_t* lo = sm + P.off_lo + l * kStageB;
                bool w = true;
                if (KIND == KIND_F32)
                    w = mbar_wait_or_abort(&B.raw_full[s], rs.ph, a.err, abort_flag);
                else if (g >= S)
                    w = mbar_wait_or_abort(&B.raw_empty[s], rs.ph ^ 1u, a.err, abort_flag);
                if (w && g >= kLoStages)
                    w = mbar_wait_or_abort(&B.lo_empty[l], (uint32_t)(((g / kLoStages) + 1) & 1), a.err, abort_flag);
                if (!group_all(kBarConv, kConv, w)) {
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
            if (KIND == KIND_Q8) group_sync(kBarConv, kConv);  // the staging area is refilled next
        }
    } else {
        // ---------------- epilogue ----------------
        // Four groups of four warps take the visits in turn (group g the ones on accumulator g); warp w of
        // a group reads tensor-memory lanes 32 (w % 4) .. 32 (w % 4) + 31.  Pass 0 has the window rows on
        // the lanes (a thread holds one row's logits of a tile), pass 1 the keys (one key's logits of
        // every row).
        const int ep = warp - 6, grp = ep >> 2, q = warp & 3;
        const int r = q * 32 + lane;  // this thread's lane: its window row in pass 0, its key in pass 1
        const bool row_ok = r < a.R;
        // rows of this warp in pass 0: all valid, none (padding), or some (a per-lane select)
        const int wmode = q * 32 + 32 <= a.R ? 0 : q * 32 >= a.R ? 1 : 2;
        const int gbar = kBarGrp + grp;
        const float s2 = a.inv_sqrt_d * 1.44269504088896341f;  // log2(e) / sqrt(D)
        const uint32_t tacc = tbase + (uint32_t)(grp * kAccCols) + ((uint32_t)(q * 32) << 16);
        bool ok = true;
        // ---- pass 0: per-(row, tile) max and sum of exp(l - max) (rocket.cpp:91-107)
        for (int v = grp; v < nv0 && ok; v += kAccs) {
            int b, hc, tile;
            work_unit(a, wof(v), b, hc, tile);
            const int k0 = tile * kMmaM, nkeys = min(kMmaM, a.nk - k0);
            const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
            const bool w = mbar_wait_or_abort(&B.acc_full[grp], (uint32_t)((v / kAccs) & 1), a.err, abort_flag);
            if (!group_all(gbar, 128, w)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // two sweeps over the row's 128 logits: the max, then the sum of exp(l - max).  The max is
            // taken over the accumulator and scaled once: rounding is monotonic and the scale positive, so
            // RN(max(x) / sqrt(D)) = max(RN(x / sqrt(D))).
            float M = -FLT_MAX, S = 0.0f;  // rocket.cpp:93
            if (wmode != 1) {
                auto sweeps = [&](auto full) {
                    float mx = -INFINITY;  // all -inf (or NaN): M = -FLT_MAX, as the running max from -FLT_MAX gives
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        float x[32];
                        tmem_ld32(tacc + (uint32_t)(c * 32), x);
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (decltype(full)::value || c * 32 + j < nkeys) mx = fmaxf(mx, x[j]);
                    }
                    M = fmaxf(mx * a.inv_sqrt_d, -FLT_MAX);
                    const float nm = neg_m2(M);
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        float x[32];
                        tmem_ld32(tacc + (uint32_t)(c * 32), x);
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            const float2 e = exp2_pair(x[j], x[j + 1], s2, make_float2(nm, nm));
                            if (decltype(full)::value || c * 32 + j < nkeys) S += e.x;
                            if (decltype(full)::value || c * 32 + j + 1 < nkeys) S += e.y;
                        }
                    }
                };
                if (nkeys == kMmaM)
                    sweeps(std::true_type{});
                else
                    sweeps(std::false_type{});
            }
            tc_fence_before();
            mbar_arrive1(&B.acc_empty[grp]);
            if (row_ok) __stcg(a.tstats + (row_base + r) * a.ntiles + tile, make_float2(M, S));
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
        if (one_launch) {
            // every CTA's statistics are written before any row folds them
            ok = group_all(kBarEpiAll, kEpiThreads, ok);
            bool gb = ok;
            if (ep == 0 && lane == 0 && ok) gb = grid_barrier(a.gbar, gridDim.x, a.err, abort_flag);
            ok = group_all(kBarEpiAll, kEpiThreads, gb);
            if (ok) {
                const size_t nrows = (size_t)P.nheads * a.R;
                for (size_t x = blockIdx.x + (size_t)gridDim.x * ep; x < nrows; x += (size_t)gridDim.x * (kEpiThreads / 32)) {
                    float M, inv;
                    fold_row(x, M, inv);
                    if (lane == 0) __stcg(a.rstats + x, make_float2(M, inv));
                }
                group_sync(kBarEpiAll, kEpiThreads);
                if (ep == 0 && lane == 0) gb = grid_barrier(a.gbar, 2u * gridDim.x, a.err, abort_flag);
                ok = group_all(kBarEpiAll, kEpiThreads, gb);
            }
        }
        // ---- pass 1: head scores sum_r exp(l - M_r) * inv_r (rocket.cpp:114-116), the logits computed
        // again with the keys on the tensor-memory lanes (D[128 keys][NP rows] = K_tile . Q^T): a thread
        // holds one key's logits of every window row and adds the terms in row order, as the reference
        // does, with no exchange between threads.  The rows' (-M_r log2 e, inv_r) sit in shared memory, one
        // copy per epilogue group, rewritten when the group's tiles move to another KV head, as one float4
        // per row pair (-M_2i log2 e, -M_2i+1 log2 e, inv_2i, inv_2i+1): each half is the paired operand
        // of one instruction.
        float* rst = reinterpret_cast<float*>(sm + P.off_epi) + grp * 256;
        auto put_row = [&](int row, float M, float inv) {
            rst[4 * (row >> 1) + (row & 1)] = neg_m2(M);
            rst[4 * (row >> 1) + 2 + (row & 1)] = inv;
        };
        const int nch = (a.R + 31) >> 5;  // 32-row chunks of the accumulator
        int prev = -1;
        for (int v = nv0 + (grp - nv0 % kAccs + kAccs) % kAccs; ok && v < nv; v += kAccs) {
            int b, hc, tile;
            work_unit(a, wof(v), b, hc, tile);
            const int head = wof(v) / a.ntiles;
            const int k0 = tile * kMmaM, nkeys = min(kMmaM, a.nk - k0);
            const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
            if (head != prev) {
                group_sync(gbar, 128);  // the group is done with the previous head's rows
                if (one_launch) {
                    if (r < a.R) {
                        const float2 x = __ldcg(a.rstats + row_base + r);
                        put_row(r, x.x, x.y);
                    }
                } else {
                    for (int rr = 0; rr < 32 && q * 32 + rr < a.R; ++rr) {  // warp-uniform bound
                        float M, inv;
                        fold_row(row_base + q * 32 + rr, M, inv);
                        if (lane == 0) put_row(q * 32 + rr, M, inv);
                    }
                }
                group_sync(gbar, 128);
                prev = head;
            }
            const bool w = mbar_wait_or_abort(&B.acc_full[grp], (uint32_t)((v / kAccs) & 1), a.err, abort_flag);
            if (!group_all(gbar, 128, w)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float hsum = 0.0f;
#pragma unroll 1
            for (int c = 0; c < nch; ++c) {
                float x[32];
                tmem_ld32(tacc + (uint32_t)(c * 32), x);
                if (c + 1 == nch) {  // every logit of the tile is in registers: the accumulator is free
                    tc_fence_before();
                    mbar_arrive1(&B.acc_empty[grp]);
                }
                const float4* rs4 = reinterpret_cast<const float4*>(rst + c * 64);
                auto terms = [&](auto full) {
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        if (!decltype(full)::value && c * 32 + j >= a.R) break;
                        const float4 st = rs4[j >> 1];  // (-M_r log2 e, -M_r+1 log2 e, inv_r, inv_r+1)
                        const float2 e = exp2_pair(x[j], x[j + 1], s2, make_float2(st.x, st.y));
                        const float2 t = __fmul2_rn(e, make_float2(st.z, st.w));
                        hsum = __fadd_rn(hsum, t.x);
                        if (!decltype(full)::value && c * 32 + j + 1 >= a.R) break;
                        hsum = __fadd_rn(hsum, t.y);
                    }
                };
                if (c * 32 + 32 <= a.R)
                    terms(std::true_type{});
                else
                    terms(std::false_type{});
            }
            if (r < nkeys) a.hs[((size_t)b * a.head_count + hc) * a.nk + k0 + r] = hsum;
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
    const int sms = sm_count();
    if (sms <= 0) return RKV_ERR_CUDA;
    const int grid = P.nwork < sms ? P.nwork : sms;
    // the head-aligned split unless it leaves some CTA more tiles than the even split would (64 heads of
    // 1024 tiles over 148 CTAs: 512 against 443)
    P.aligned = 0;
    if (P.nheads <= grid) {
        const int base = grid / P.nheads;
        P.aligned = (a.ntiles + base - 1) / base <= (P.nwork + grid - 1) / grid;
    }
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
