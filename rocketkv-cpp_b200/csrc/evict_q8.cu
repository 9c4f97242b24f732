// evict_q8.cu -- stage-1 scoring of q8_0 K and window queries on the tcgen05
// tensor cores with exact int8 products (kind::i8), persistent (sm_100a).
//
// A q8_0 row of 128 values is four blocks {fp16 d; int8 q[32]}.  The logit of
// window row r and key k (rocket.cpp:97-105, on the exactly dequantised
// values) is
//     l[r][k] = sum_b dq[r][b] * dk[k][b] * A_b[r][k] / sqrt(D),
//     A_b = sum over block b of qq * qk   (an exact int32 dot of 32 int8 pairs).
// Each A_b is one tcgen05.mma of kind::i8 (M = 128 keys, N = query rows,
// K = 32) into its own int32 tensor-memory accumulator.  Every accumulator is
// preset to the bit pattern of 1.5 * 2^23, so it holds 0x4B400000 + A_b and,
// read as a float, is exactly X_b = 1.5 * 2^23 + A_b (|A_b| <= 32*127*127 <
// 2^22).  One fused multiply-add with the key's block scale then gives the
// correctly rounded product without any conversion instruction:
//     fma(dk, X_b, -1.5 * 2^23 * dk) = round(dk * A_b)
// (the addend is exact: dk is an fp16 value, so 3 * 2^22 * dk has at most 13
// significant bits, and the fma rounds once).  The four block terms are then
// summed with the row's block scales, which carry 1/sqrt(D) * log2(e), so the
// logits come out in base-2 units and exp becomes the MUFU's ex2.
//
// Work split and passes follow the fp32/bf16 persistent scorer (evict_tc.cu):
// one CTA per SM walks a contiguous range of (item, KV head, 128-key tile)
// units twice.  Pass 0 writes per-(row, tile) softmax statistics (the row
// max over the tile and the sum of 2^(l - max)); after a bounded grid barrier
// the CTAs fold them into each row's max M_r and inv_r = 1 / (sum + 1e-9)
// (rocket.cpp:108-113); pass 1 recomputes the logits and writes the head
// score hs[k] = sum_r 2^(l[r][k] - M_r) * inv_r (rocket.cpp:114-116) for the
// pooling kernel.  Pass 1 visits the CTA's tiles in reverse order, so its
// first tiles are the ones pass 0 read last (still in L2).  The copies,
// repacking and MMAs of pass 1 run ahead while the epilogue waits at the grid
// barrier.  If the cooperative launch is refused, one launch per pass.
//
// Tensor memory: a ring of four slots, each holding the four block
// accumulators of one part of a tile (32 query rows: the MMA N), so the MMAs
// run up to three parts ahead of the epilogue and their latency is hidden.
//
// Warp roles (640 threads):
//   warp 0      producer: one bulk copy per tile visit of the tile's rows
//               (128 rows of 136 bytes, contiguous in K) into a raw ring;
//   warp 1      tensor memory and the MMAs (one elected lane issues);
//   warps 2-3   converters: each thread repacks two raw rows into the int8
//               operand (four 32-byte blocks in a 128-byte row, the K-major
//               128-byte-swizzle layout) and the key's block scales; at a new
//               KV head, the window query rows and their scales;
//   warps 4-19  epilogue, four warps per tensor-memory lane quarter, each
//               taking 8 of a part's 32 query rows (one 8-column chunk of
//               every block accumulator).
// Every wait is bounded; a role that times out sets a CTA-wide abort flag.
#include "evict.cuh"
#include "tc_common.cuh"

#include <float.h>

namespace rkv {
namespace {

constexpr int kQ8Threads = 640;
constexpr int kQ8Epi = 512;       // epilogue threads: four warps per tensor-memory lane quarter
constexpr int kEpiMembers = 4;     // epilogue warps per lane quarter, 8 of a part's 32 query rows each
constexpr int kQ8Conv = 64;  // converter threads (two warps, two rows each per tile)
constexpr int kQ8RowB = 136;                 // bytes of one q8_0 row of 128 values
constexpr int kQ8TileB = 128 * kQ8RowB;      // raw bytes of a full tile (17408, a multiple of 16)
constexpr int kOpB = 128 * 128;              // repacked int8 operand of a tile
constexpr int kOpStages = 2;
constexpr int kScStages = 4;                 // key-scale slots (the epilogue lags the MMAs)
constexpr int kMaxRaw = 8;
constexpr int kTmemColsQ8 = 512;
constexpr int kBarConvQ8 = 1, kBarEpiQ8 = 2;
constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

constexpr int kPartRows = 32;  // query rows of one MMA part (N)
constexpr int kSlots = 4;      // tensor-memory slots of 4 blocks x kPartRows columns

struct Q8Plan {
    int NP, NPT;  // query rows padded to a multiple of 32, and the parts of a tile (NP / 32)
    int SR;      // raw ring stages
    int off_raw, off_op, off_q, off_dq, off_dk, off_part, off_rtab, off_red, total;
    int nwork, nheads, p0, p1;
};

inline Q8Plan q8_plan(int R) {
    Q8Plan P{};
    P.NP = (R + 31) & ~31;
    P.NPT = P.NP / kPartRows;
    int off = 1024;  // barriers, tensor-memory slot, abort flag
    P.off_op = off;
    off += kOpStages * kOpB;
    P.off_q = off;
    off += 2 * P.NP * 128;  // query operand, double-buffered by KV head
    P.off_dq = off;
    off += 2 * (P.NP / 2) * 4 * 8;  // [2][NP/2 row pairs][4 blocks] float2
    P.off_dk = off;
    off += kScStages * 128 * 16;  // [slot][key][4 blocks] float
    P.off_part = off;
    off += 2 * 4 * 128 * 8;  // [tile parity][lane quarter][row] (max, sum)
    P.off_rtab = off;
    off += 64 * 16;  // pass 1: [row pair] (-M_r, -M_r+1, inv_r, inv_r+1)
    P.off_red = off;
    off += kEpiMembers * 128 * 4;  // pass 1: [member][key] partial head scores
    off = (off + 127) & ~127;
    P.off_raw = off;
    const int room = 227 * 1024 - 1024 - off;
    P.SR = room / kQ8TileB < kMaxRaw ? room / kQ8TileB : kMaxRaw;
    P.total = off + P.SR * kQ8TileB;
    return P;
}

struct Q8Bars {
    uint64_t *raw_full, *raw_empty, *op_full, *op_empty, *dk_full, *dk_empty, *acc_full, *acc_empty, *q_full,
        *q_empty_mma, *q_empty_epi, *mma_done;
};
__device__ __forceinline__ Q8Bars q8_bars(uint8_t* sm) {
    uint64_t* b = reinterpret_cast<uint64_t*>(sm);
    return Q8Bars{b, b + 8, b + 16, b + 18, b + 20, b + 24, b + 28, b + 32, b + 36, b + 38, b + 40, b + 42};
}

__device__ __forceinline__ void unit_of(const EvictArgs& a, int w, int& b, int& hc, int& tile) {
    tile = w % a.ntiles;
    const int t = w / a.ntiles;
    hc = t % a.head_count;
    b = t / a.head_count;
}

// This CTA's work units [w0, w0 + nt): with at least as many CTAs as
// (item, KV head) pairs the CTAs of a head split its tiles evenly; else
// contiguous ranges.
__device__ __forceinline__ void q8_range(const Q8Plan& P, int ntiles, int& w0, int& nt) {
    const int G = gridDim.x, c = blockIdx.x;
    if (P.nheads <= G) {
        const int base = G / P.nheads, extra = G % P.nheads;
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

__device__ __forceinline__ int sw128_off(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Half H of a raw q8_0 row (four {fp16 d; int8 q[32]} blocks, 136 bytes, 8-byte aligned; shared or global
// memory): blocks 2H and 2H + 1, bytes 68H .. 68H + 67, read as the 18 words from word 16H -> the two int8
// blocks at 16-byte chunks 4H .. 4H + 3 of operand row r (K-major, 128-byte swizzle), and their scales.
template <int H>
__device__ __forceinline__ void q8_half_repack(const uint8_t* raw_row, uint8_t* op, int r, float* d) {
    const uint2* src = reinterpret_cast<const uint2*>(raw_row) + 8 * H;
    uint32_t w[18];
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        const uint2 u = src[t];
        w[2 * t] = u.x;
        w[2 * t + 1] = u.y;
    }
    // in the half's words: block 2H starts two bytes into word H (its scale is the low half of word H),
    // block 2H + 1 at word H + 9 (its scale is the high half of word H + 8)
    uint32_t o[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        o[j] = __funnelshift_r(w[H + j], w[H + j + 1], 16);
        o[8 + j] = w[H + 9 + j];
    }
    d[0] = __half2float(__ushort_as_half((unsigned short)(w[H] & 0xFFFFu)));
    d[1] = __half2float(__ushort_as_half((unsigned short)(w[H + 8] >> 16)));
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(op + sw128_off(r, 4 * H + c)) = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_st8_magic(uint32_t taddr) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
                 "r"(kMagicBits)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float warp_max(float v) {
    float m;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(v));
    return m;
}

__device__ __forceinline__ void mma_i8_w(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, 1, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc)
        : "memory");
}

// Instruction descriptor, kind::i8: int32 accumulator, signed 8-bit A and B,
// both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((uint32_t)(kMmaM >> 4) << 24);
}

__device__ __forceinline__ bool grid_bar(unsigned* cnt, unsigned n, int* err, volatile int* abort) {
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

// The visits of one launch: v in [v0, v1) of the sequence (pass 0 over tiles
// 0 .. nt-1, then pass 1 over tiles nt-1 .. 0).
struct Visit {
    int v0, v1, nt, w0;
    __device__ __forceinline__ int pass(int v) const { return v >= nt ? 1 : 0; }
    __device__ __forceinline__ int unit(int v) const { return w0 + (v < nt ? v : 2 * nt - 1 - v); }
};

__global__ void __launch_bounds__(kQ8Threads, 1) evict_q8_kernel(const EvictArgs a, const Q8Plan P) {
    asm volatile("griddepcontrol.launch_dependents;");  // the pooling may be scheduled (it waits for this grid)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const Q8Bars B = q8_bars(sm);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 512);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + 516);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int w0, nt;
    q8_range(P, a.ntiles, w0, nt);
    Visit V{P.p0 == 0 ? 0 : nt, P.p1 == 1 ? 2 * nt : nt, nt, w0};
    const int SR = P.SR, NP = P.NP, NPT = P.NPT;
    auto head_of = [&](int v) { return V.unit(v) / a.ntiles; };

    if (tid == 0) {
        for (int i = 0; i < SR; ++i) {
            mbar_init(&B.raw_full[i], 1);
            mbar_init(&B.raw_empty[i], kQ8Conv / 32);  // one arrival per converter warp
        }
        for (int i = 0; i < kOpStages; ++i) {
            mbar_init(&B.op_full[i], kQ8Conv / 32);
            mbar_init(&B.op_empty[i], 1);
        }
        for (int i = 0; i < kScStages; ++i) {
            mbar_init(&B.dk_full[i], kQ8Conv / 32);
            mbar_init(&B.dk_empty[i], kQ8Epi / 32);
        }
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&B.acc_full[i], 1);
            mbar_init(&B.acc_empty[i], kQ8Epi / 32);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&B.q_full[i], kQ8Conv / 32);
            mbar_init(&B.q_empty_mma[i], 1);
            mbar_init(&B.q_empty_epi[i], kQ8Epi / 32);
        }
        mbar_init(B.mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tslot, kTmemColsQ8);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        // ---------------- producer: one bulk copy per tile visit ----------------
        int issued_lo = V.v0, issued_hi = V.v0;
        for (int v = V.v0; v < V.v1; ++v) {
            const int s = (v - V.v0) % SR, use = (v - V.v0) / SR;
            if (use > 0 && !__all_sync(0xffffffffu, mbar_wait_or_abort(&B.raw_empty[s], (uint32_t)((use + 1) & 1),
                                                                         a.err, abort_flag)))
                break;
            int b, hc, tile;
            unit_of(a, V.unit(v), b, hc, tile);
            const int k0 = tile * kMmaM, nkeys = min(kMmaM, a.nk - k0);
            // a tail of an odd number of rows also takes the first 8 bytes of the next row (a window row)
            const uint32_t bytes = (uint32_t)((nkeys * kQ8RowB + 15) & ~15);
            const uint8_t* src =
                a.K + (size_t)b * a.k_stride + ((size_t)(a.head_begin + hc) * a.k_head_rows + k0) * kQ8RowB;
            if (lane == 0) {
                mbar_arrive_expect_tx(&B.raw_full[s], bytes);
                bulk_load(sm + P.off_raw + (size_t)s * kQ8TileB, src, bytes, &B.raw_full[s]);
            }
            __syncwarp();
            issued_hi = v + 1;
        }
        // every copy issued lands before the CTA can exit
        if (lane == 0)
            for (int v = (issued_hi - issued_lo > SR ? issued_hi - SR : issued_lo); v < issued_hi; ++v)
                mbar_wait_bounded(&B.raw_full[(v - V.v0) % SR], (uint32_t)(((v - V.v0) / SR) & 1), a.err);
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        const uint32_t idesc = idesc_i8((uint32_t)kPartRows);
        int hv = -1, prev = -1;
        bool ok = true;
        for (int v = V.v0; v < V.v1 && ok; ++v) {
            const int x = v - V.v0;
            const int head = head_of(v);
            if (head != prev) {
                ++hv;
                prev = head;
                if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&B.q_full[hv & 1], (uint32_t)((hv >> 1) & 1), a.err,
                                                                abort_flag)))
                    break;
            }
            const int o = x % kOpStages;
            if (!__all_sync(0xffffffffu,
                            mbar_wait_or_abort(&B.op_full[o], (uint32_t)((x / kOpStages) & 1), a.err, abort_flag)))
                break;
            for (int pt = 0; pt < NPT; ++pt) {  // one part of 32 query rows per tensor-memory slot
                const int j = x * NPT + pt, slot = j % kSlots;
                if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&B.acc_empty[slot], (uint32_t)((j / kSlots) & 1),
                                                                a.err, abort_flag))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t dA = mma_desc_sw128(smem_u32(sm + P.off_op + o * kOpB));
                const uint64_t dB =
                    mma_desc_sw128(smem_u32(sm + P.off_q + (hv & 1) * NP * 128 + pt * kPartRows * 128));
#pragma unroll
                for (int blk = 0; blk < 4; ++blk)  // a 32-byte K step adds 2 to the start-address field
                    mma_i8_w(tbase + (uint32_t)(slot * 4 * kPartRows + blk * kPartRows), dA + 2 * blk, dB + 2 * blk,
                             idesc);
                mma_commit_w(&B.acc_full[slot]);
            }
            if (!ok) break;
            mma_commit_w(&B.op_empty[o]);
            if (v + 1 == V.v1 || head_of(v + 1) != head) mma_commit_w(&B.q_empty_mma[hv & 1]);
        }
        mma_commit_w(B.mma_done);
        mbar_wait_bounded(B.mma_done, 0u, a.err);
        __syncwarp();
    } else if (warp < 4) {
        // ---------------- converters ----------------
        const int ct = tid - 64;
        const float qscale = a.inv_sqrt_d * 1.4426950408889634f;  // 1/sqrt(D) * log2(e)
        int hv = -1, prev = -1;
        for (int v = V.v0; v < V.v1; ++v) {
            const int x = v - V.v0;
            int b, hc, tile;
            unit_of(a, V.unit(v), b, hc, tile);
            const int head = head_of(v);
            if (head != prev) {
                ++hv;
                prev = head;
                const int qb = hv & 1;
                bool w = true;
                if (hv >= 2) {
                    w = mbar_wait_or_abort(&B.q_empty_mma[qb], (uint32_t)(((hv >> 1) + 1) & 1), a.err, abort_flag);
                    if (w)
                        w = mbar_wait_or_abort(&B.q_empty_epi[qb], (uint32_t)(((hv >> 1) + 1) & 1), a.err, abort_flag);
                }
                if (!group_all(kBarConvQ8, kQ8Conv, w)) break;
                // window row ct of the KV head's query group (rocket.cpp:85-90)
                uint8_t* qop = sm + P.off_q + qb * NP * 128;
                float2* dqt = reinterpret_cast<float2*>(sm + P.off_dq) + qb * (NP / 2) * 4;
                for (int rr = ct; rr < NP; rr += kQ8Conv) {
                    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    if (rr < a.R) {
                        const int hk = a.head_begin + hc;
                        const int h = hk * a.G + rr / a.obs_w, pos = a.q_row0 + rr % a.obs_w;
                        const uint8_t* qrow = a.Q + (size_t)b * a.q_stride + ((size_t)h * a.q_head_rows + pos) * kQ8RowB;
                        q8_half_repack<0>(qrow, qop, rr, d);
                        q8_half_repack<1>(qrow, qop, rr, d + 2);
                    } else {
#pragma unroll
                        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(qop + sw128_off(rr, c)) = make_uint4(0u, 0u, 0u, 0u);
                    }
#pragma unroll
                    for (int t = 0; t < 4; ++t) reinterpret_cast<float*>(dqt + (rr >> 1) * 4 + t)[rr & 1] = d[t] * qscale;
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive1(&B.q_full[qb]);
            }
            // the tile's rows: raw ring -> int8 operand and key scales
            const int s = x % SR, o = x % kOpStages, ds = x % kScStages;
            bool w = mbar_wait_or_abort(&B.raw_full[s], (uint32_t)((x / SR) & 1), a.err, abort_flag);
            if (w && x >= kOpStages)
                w = mbar_wait_or_abort(&B.op_empty[o], (uint32_t)(((x / kOpStages) + 1) & 1), a.err, abort_flag);
            if (w && x >= kScStages)
                w = mbar_wait_or_abort(&B.dk_empty[ds], (uint32_t)(((x / kScStages) + 1) & 1), a.err, abort_flag);
            if (!group_all(kBarConvQ8, kQ8Conv, w)) break;
            const int nkeys = min(kMmaM, a.nk - tile * kMmaM);
#pragma unroll 1
            for (int rr = ct; rr < kMmaM; rr += kQ8Conv) {
                float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                uint8_t* orow = sm + P.off_op + o * kOpB;
                if (rr < nkeys) {
                    const uint8_t* raw_row = sm + P.off_raw + (size_t)s * kQ8TileB + rr * kQ8RowB;
                    q8_half_repack<0>(raw_row, orow, rr, d);
                    q8_half_repack<1>(raw_row, orow, rr, d + 2);
                } else {
#pragma unroll
                    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(orow + sw128_off(rr, c)) = make_uint4(0u, 0u, 0u, 0u);
                }
                *reinterpret_cast<float4*>(sm + P.off_dk + (size_t)(ds * 128 + rr) * 16) = make_float4(d[0], d[1], d[2], d[3]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive1(&B.raw_empty[s]);  // the raw rows are read
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive1(&B.op_full[o]);
                mbar_arrive1(&B.dk_full[ds]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int ep = warp - 4, et = tid - 128, q = warp & 3, mem = ep >> 2;
        const int kk = q * 32 + lane;
        const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
        float2* part = reinterpret_cast<float2*>(sm + P.off_part);  // [2][4][128]
        float4* rtab = reinterpret_cast<float4*>(sm + P.off_rtab);   // [64]
        float* red = reinterpret_cast<float*>(sm + P.off_red);       // [2][128]
        bool ok = true;
        int hv = -1, prev = -1, rt_head = -1;
        const bool one_launch = P.p0 == 0 && P.p1 == 1;

        auto fold_row = [&](size_t xr, float& M, float& inv) {  // one warp, row xr of [item][head][R]
            const float2* ts = a.tstats + xr * a.ntiles;
            M = -FLT_MAX;
            for (int ti = lane; ti < a.ntiles; ti += 32) M = fmaxf(M, __ldcg(ts + ti).x);
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
            float S = 0.0f;
            for (int ti = lane; ti < a.ntiles; ti += 32) {
                const float2 t2 = __ldcg(ts + ti);
                S += t2.y * exp2f(t2.x - M);
            }
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o2);
            inv = 1.0f / (S + 1e-9f);
        };

        // every slot starts free: its accumulators are preset
        for (int sl = 0; sl < kSlots; ++sl)
            for (int blk = 0; blk < 4; ++blk)
                tmem_st8_magic(tlane + (uint32_t)(sl * 4 * kPartRows + blk * kPartRows + mem * 8));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int sl = 0; sl < kSlots; ++sl) mbar_arrive1(&B.acc_empty[sl]);

        // one tile visit of the epilogue; false when a wait gave up
        auto visit = [&](int v) -> bool {
            const int x = v - V.v0, pass = V.pass(v);
            int b, hc, tile;
            unit_of(a, V.unit(v), b, hc, tile);
            const int head = head_of(v);
            const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
            const int k0 = tile * kMmaM, nkeys = min(kMmaM, a.nk - k0);
            if (head != prev) {
                ++hv;
                prev = head;
                const bool w = mbar_wait_or_abort(&B.q_full[hv & 1], (uint32_t)((hv >> 1) & 1), a.err, abort_flag);
                if (!group_all(kBarEpiQ8, kQ8Epi, w)) return false;
            }
            // pass 1 needs the head's row statistics (-M_r, inv_r), as row pairs; its first tile continues
            // pass 0's last head, so the table is keyed on the pass as well as the head
            if (pass == 1 && head != rt_head) {
                rt_head = head;
                {
                    if (one_launch) {
                        for (int p = et; p < NP / 2; p += kQ8Epi) {
                            const int r = 2 * p;
                            const float2 s0 = r < a.R ? __ldcg(a.rstats + row_base + r) : make_float2(0.0f, 0.0f);
                            const float2 s1 = r + 1 < a.R ? __ldcg(a.rstats + row_base + r + 1) : make_float2(0.0f, 0.0f);
                            rtab[p] = make_float4(-s0.x, -s1.x, s0.y, s1.y);
                        }
                    } else {
                        for (int r = ep; r < NP; r += kQ8Epi / 32) {
                            float M = 0.0f, inv = 0.0f;
                            if (r < a.R) fold_row(row_base + r, M, inv);
                            if (lane == 0) {
                                float* t4 = reinterpret_cast<float*>(rtab + (r >> 1));
                                t4[r & 1] = r < a.R ? -M : 0.0f;
                                t4[2 + (r & 1)] = r < a.R ? inv : 0.0f;
                            }
                        }
                    }
                    group_sync(kBarEpiQ8, kQ8Epi);
                }
            }
            const float2* dqt = reinterpret_cast<const float2*>(sm + P.off_dq) + (hv & 1) * (NP / 2) * 4;
            // this key's block scales and the exact addends -1.5 * 2^23 * dk
            const int ds = x % kScStages;
            // waits are warp-level here; a failed one skips the warp's work and the tile's barrier below
            // makes the exit decision uniform
            bool good = __all_sync(0xffffffffu, mbar_wait_or_abort(&B.dk_full[ds], (uint32_t)((x / kScStages) & 1),
                                                                    a.err, abort_flag));
            const float4 dk4 =
                good ? *reinterpret_cast<const float4*>(sm + P.off_dk + (size_t)(ds * 128 + kk) * 16) : make_float4(0, 0, 0, 0);
            __syncwarp();
            if (lane == 0 && good) mbar_arrive1(&B.dk_empty[ds]);
            // the key's block scales and the exact addends -1.5 * 2^23 * dk, as pairs for the paired fma
            const float2 dk2[4] = {make_float2(dk4.x, dk4.x), make_float2(dk4.y, dk4.y), make_float2(dk4.z, dk4.z),
                                   make_float2(dk4.w, dk4.w)};
            const float2 cdk2[4] = {make_float2(-kMagic * dk4.x, -kMagic * dk4.x), make_float2(-kMagic * dk4.y, -kMagic * dk4.y),
                                    make_float2(-kMagic * dk4.z, -kMagic * dk4.z), make_float2(-kMagic * dk4.w, -kMagic * dk4.w)};
            const bool kvalid = kk < nkeys, full = nkeys == kMmaM;  // full: every key of the tile is valid (uniform)
            float2 hsacc = make_float2(0.0f, 0.0f);
            // logits of rows r0 .. r0 + 7 (base-2 units) from one 8-column chunk of the four block
            // accumulators, then the pass's use of them
            auto chunk = [&](const uint32_t (&xv)[4][8], int r0) {
                float l[8];
                const float2* dq2 = dqt + (r0 >> 1) * 4;
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const float4 s01 = *reinterpret_cast<const float4*>(dq2 + p * 4);      // blocks 0, 1
                    const float4 s23 = *reinterpret_cast<const float4*>(dq2 + p * 4 + 2);  // blocks 2, 3
                    const float2 sq[4] = {make_float2(s01.x, s01.y), make_float2(s01.z, s01.w),
                                          make_float2(s23.x, s23.y), make_float2(s23.z, s23.w)};
                    float2 acc;
                    if (pass == 0) {
                        acc = make_float2(0.0f, 0.0f);
                    } else {
                        const float4 rt = rtab[r0 / 2 + p];
                        acc = make_float2(rt.x, rt.y);  // -M_r: the chain ends at l - M_r
                    }
#pragma unroll
                    for (int blk = 0; blk < 4; ++blk) {
                        const float2 X = make_float2(__uint_as_float(xv[blk][2 * p]), __uint_as_float(xv[blk][2 * p + 1]));
                        const float2 pb = __ffma2_rn(X, dk2[blk], cdk2[blk]);
                        acc = __ffma2_rn(sq[blk], pb, acc);
                    }
                    l[2 * p] = acc.x;
                    l[2 * p + 1] = acc.y;
                }
                if (pass == 0) {
                    // per-(row, lane quarter) max and sum of 2^(l - max) over this warp's 32 keys
                    float e[8], mq[8];
                    if (full) {
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            mq[t] = warp_max(l[t]);
                            e[t] = ex2_approx(l[t] - mq[t]);
                        }
                    } else {
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            const float lv = kvalid ? l[t] : -INFINITY;
                            mq[t] = warp_max(lv);
                            e[t] = kvalid ? ex2_approx(lv - mq[t]) : 0.0f;
                        }
                    }
                    // sums over the 32 lanes by recursive halving: lane L ends with row
                    // 4 ((L >> 4) & 1) + 2 ((L >> 3) & 1) + ((L >> 2) & 1)
                    const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float send = u16 ? e[t] : e[t + 4], keep = u16 ? e[t + 4] : e[t];
                        e[t] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                    }
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const float send = u8 ? e[t] : e[t + 2], keep = u8 ? e[t + 2] : e[t];
                        e[t] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                    }
                    {
                        const float send = u4 ? e[0] : e[1], keep = u4 ? e[1] : e[0];
                        e[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                    }
                    e[0] += __shfl_xor_sync(0xffffffffu, e[0], 2);
                    e[0] += __shfl_xor_sync(0xffffffffu, e[0], 1);
                    const int jr = (u16 ? 4 : 0) + (u8 ? 2 : 0) + (u4 ? 1 : 0);
                    float mine = mq[0];
#pragma unroll
                    for (int t = 1; t < 8; ++t)
                        if (t == jr) mine = mq[t];
                    const int r = r0 + jr;
                    if ((lane & 3) == 0 && r < a.R) part[((x & 1) * 4 + q) * 128 + r] = make_float2(mine, e[0]);
                } else if (kvalid) {
                    // head score terms 2^(l - M_r) * inv_r (rocket.cpp:114-116)
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const float4 rt = rtab[r0 / 2 + p];
                        const float2 ev = make_float2(ex2_approx(l[2 * p]), ex2_approx(l[2 * p + 1]));
                        hsacc = __ffma2_rn(ev, make_float2(rt.z, rt.w), hsacc);
                    }
                }
            };
            for (int pt = 0; pt < NPT && good; ++pt) {  // parts of 32 query rows, one per tensor-memory slot
                const int j = x * NPT + pt, slot = j % kSlots;
                good = __all_sync(0xffffffffu, mbar_wait_or_abort(&B.acc_full[slot], (uint32_t)((j / kSlots) & 1),
                                                                   a.err, abort_flag));
                if (!good) break;
                tc_fence_after();
                // this warp's 8 rows of the part: one 8-column chunk of each of the four blocks
                const uint32_t col = (uint32_t)(slot * 4 * kPartRows + mem * 8);
                uint32_t xa[4][8];
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) tmem_ld8(tlane + col + (uint32_t)(blk * kPartRows), xa[blk]);
                tmem_wait_ld();
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) tmem_st8_magic(tlane + col + (uint32_t)(blk * kPartRows));
                chunk(xa, pt * kPartRows + mem * 8);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive1(&B.acc_empty[slot]);
            }
            if (!group_all(kBarEpiQ8, kQ8Epi, good)) return false;
            if (pass == 0) {
                if (et < a.R) {  // combine the four lane quarters of the tile
                    const float2* pr = part + (x & 1) * 4 * 128 + et;
                    float M = -INFINITY;
#pragma unroll
                    for (int t = 0; t < 4; ++t) M = fmaxf(M, pr[t * 128].x);
                    float S = 0.0f;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float2 pq = pr[t * 128];
                        S += pq.x == -INFINITY ? 0.0f : pq.y * ex2_approx(pq.x - M);
                    }
                    __stcg(a.tstats + (row_base + et) * a.ntiles + tile, make_float2(M, S));
                }
            } else {
                red[mem * 128 + kk] = hsacc.x + hsacc.y;
                group_sync(kBarEpiQ8, kQ8Epi);
                if (et < 128 && et < nkeys)  // the members' partial sums, in member order
                    a.hs[((size_t)b * a.head_count + hc) * a.nk + k0 + et] = ((red[et] + red[128 + et]) + red[256 + et]) + red[384 + et];
                group_sync(kBarEpiQ8, kQ8Epi);
            }
            if (v + 1 == V.v1 || head_of(v + 1) != head) {
                __syncwarp();
                if (lane == 0) mbar_arrive1(&B.q_empty_epi[hv & 1]);
            }
            return true;
        };
        const int vmid = V.nt < V.v0 ? V.v0 : (V.nt > V.v1 ? V.v1 : V.nt);
        for (int v = V.v0; v < vmid && ok; ++v) ok = visit(v);
        if (ok && one_launch) {
            // ---- between the passes: the row fold over all CTAs (rocket.cpp:108-113); every CTA
            // takes both grid barriers, whatever its share of tiles ----
            group_sync(kBarEpiQ8, kQ8Epi);  // every statistic of this CTA is written
            bool gb = true;
            if (et == 0) gb = grid_bar(a.gbar, gridDim.x, a.err, abort_flag);
            ok = group_all(kBarEpiQ8, kQ8Epi, gb);
            if (ok) {
                const size_t nrows = (size_t)P.nheads * a.R;
                for (size_t xr = blockIdx.x + (size_t)gridDim.x * ep; xr < nrows; xr += (size_t)gridDim.x * (kQ8Epi / 32)) {
                    float M, inv;
                    fold_row(xr, M, inv);
                    if (lane == 0) __stcg(a.rstats + xr, make_float2(M, inv));
                }
                group_sync(kBarEpiQ8, kQ8Epi);
                if (et == 0) gb = grid_bar(a.gbar, 2u * gridDim.x, a.err, abort_flag);
                ok = group_all(kBarEpiQ8, kQ8Epi, gb);
            }
        }
        for (int v = vmid; v < V.v1 && ok; ++v) ok = visit(v);
    }

    // ---- release the tensor memory on every path ----
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tbase, kTmemColsQ8);
}

int q8_sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 0;
    return n;
}

}  // namespace

bool evict_q8_supported(const EvictArgs& a, int batch) {
    if (a.dtype != RKV_Q8_0 || a.D != 128 || a.R <= 0 || a.R > 128 || a.ntiles <= 0 || batch <= 0) return false;
    const uintptr_t ka = reinterpret_cast<uintptr_t>(a.K), qa = reinterpret_cast<uintptr_t>(a.Q);
    if ((ka & 15) || (qa & 7)) return false;                          // bulk copies; 8-byte query loads
    if (batch > 1 && ((a.k_stride & 15) || (a.q_stride & 7))) return false;
    if (a.k_head_rows & 1) return false;                              // every tile starts on 16 bytes
    if ((a.nk & 1) && a.k_head_rows <= a.nk) return false;            // an odd tail reads into the next row
    return q8_plan(a.R).SR >= 2;
}

int launch_evict_q8(const EvictArgs& a, int batch, cudaStream_t st) {
    Q8Plan P = q8_plan(a.R);
    P.nwork = batch * a.head_count * a.ntiles;
    P.nheads = batch * a.head_count;
    const int sms = q8_sm_count();
    if (sms <= 0) return RKV_ERR_CUDA;
    const int grid = P.nwork < sms ? P.nwork : sms;
    const int smem = P.total + 1024;
    if (cudaFuncSetAttribute(evict_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return RKV_ERR_CUDA;
    P.p0 = 0;
    P.p1 = 1;
    void* args[] = {const_cast<EvictArgs*>(&a), &P};
    const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(evict_q8_kernel), dim3(grid),
                                                      dim3(kQ8Threads), args, (size_t)smem, st);
    if (e == cudaSuccess) return RKV_OK;
    (void)cudaGetLastError();
    if (e != cudaErrorCooperativeLaunchTooLarge && e != cudaErrorNotSupported) return RKV_ERR_CUDA;
    for (int pass = 0; pass < 2; ++pass) {
        P.p0 = P.p1 = pass;
        evict_q8_kernel<<<grid, kQ8Threads, smem, st>>>(a, P);
        if (cudaGetLastError() != cudaSuccess) return RKV_ERR_CUDA;
    }
    return RKV_OK;
}

}  // namespace rkv
