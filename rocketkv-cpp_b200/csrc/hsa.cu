// hsa.cu -- stage-2 hybrid sparse decode on sm_100a (rocket.cpp:171-382).
//
// Three kernels per call; a unit is one (item, KV head):
//
// hsa_scan_kernel   grid (splits, KV heads, items)
//   0. query statistics of the GQA group: sum_h |q|, the sign of sum_h q, the
//      top-r dimensions (ties to the lower dimension, listed ascending) and the
//      per-head variance scale (rocket.cpp:197-250);
//   1. a producer warp streams the K rows of the CTA's page range through a
//      ring of 16 KB stages with 1-D bulk copies (cp.async.bulk, no multicast;
//      full/empty mbarriers; the first stages are issued before phase 0);
//      groups of consumer warps take the stages in turn.  Each page (C rows)
//      gets its sign-chosen max/min on the r dimensions and the approximate
//      logit per head (rocket.cpp:252-289), four lanes per page: the sign
//      choice and the top-r selection are masks on packed bf16 pairs (one
//      max.bf16x2 per pair and row), the multiply-adds are paired fp32 FMAs
//      with one chain per 16-byte chunk, and an IEEE division applies the
//      scale.  Logits go to the workspace.  Large batches use one CTA per
//      unit; small ones split a unit's pages over several CTAs so the grid
//      still covers the GPU.
//
// hsa_select_kernel one 128-thread CTA per unit
//   2. per-head page softmax with the deterministic exp and a fixed 256-way
//      summation order, the group sum, a weighted radix select of the top
//      final_k tokens by (score desc, index asc) and a stable compaction to
//      ascending order (rocket.cpp:291-340), then the recent window; the
//      logits are staged in shared memory by one bulk copy;
//
// hsa_attn_kernel   grid (KV heads, items)
//   3. exact attention over the selected rows (rocket.cpp:342-378): the
//      selected K rows and then V rows are gathered with 16-byte read-only
//      loads, several tokens in flight per thread; scores (eight lanes per
//      token, q in registers, paired FMAs), per-head softmax statistics, then
//      p * v with one thread per 16-byte V vector.  Selected indices and
//      scores stay in shared memory when they fit.
//
// Phases 0-2 repeat the oracle's float operations one for one, so the selected
// indices equal the oracle's bit for bit; O is tolerance-checked.
#include "hsa.cuh"

#include <float.h>

namespace rkv {
namespace {

constexpr int kNT = 256;
constexpr int kStageBytes = 16384;
constexpr int kMaxScanStages = 8;  // scan ring stages at most (barrier slots)
constexpr int kTailSmemMax = 96 * 1024;  // attention: indices + scores kept in shared memory up to this
constexpr int kSelSmemMax = 24 * 1024;   // selection: page logits staged in shared memory up to this

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<uint16_t>(uint16_t v) { return bf16_bits_to_f32(v); }

template <typename T>
__device__ __forceinline__ void vec_to_f(const uint4& v, float* out);
template <>
__device__ __forceinline__ void vec_to_f<float>(const uint4& v, float* out) {
    out[0] = __uint_as_float(v.x);
    out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z);
    out[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void vec_to_f<uint16_t>(const uint4& v, float* out) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

// A plain (coherent) 16-byte global load: V may be pinned host memory that
// the host path maps into the device's address space.
__device__ __forceinline__ uint4 ld_global_v4(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// (d.x, d.y) += (a.x * b.x, a.y * b.y), each lane one fused multiply-add
// rounded once (the paired fp32 FMA of sm_100).
__device__ __forceinline__ void ffma2(float2& d, const float2 a, const float2 b) { d = __ffma2_rn(a, b, d); }

// ===========================================================================
// Scan kernel: phases 0 and 1
// ===========================================================================
// A page is handled by a quad of four lanes.  A K row is a sequence of 16-byte
// chunks (8 bf16 or 4 fp32 dimensions); lane j of the quad owns the chunks
// j + 4 i (i < NSL, its slots).  Per chunk and head the lane runs a paired
// fused multiply-add chain -- one lane of the pair over the chunk's even
// dimensions, one over its odd ones, ascending -- and the chunk value is
// even + odd; the lane adds its slot values pairwise ((s0+s1)+(s2+s3)...),
// and the quad adds its lanes as (l0 + l2) + (l1 + l3).  Odd quads visit
// their slots in the order i ^ 1, so the two quads that share a shared-memory
// wavefront read opposite halves of the banks; every chunk has its own chain
// and the slot tree adds pairs (i, i ^ 1) first, so the order of visits
// changes no result.  The oracle's chunk_dot restates this order.
//
// Per chunk the shared table `tab` holds, in 16-byte units:
//   q   per head the chunk's s q values (s = -1 where sum_h q < 0; zero on
//       dimensions outside the top r);
//   xm  per dimension the sign bit that turns a K value x into s x, so the
//       page maximum of s x is s times the sign-chosen max / min;
//   sm  all ones on the top-r dimensions, zero elsewhere;
// with an odd unit stride so eight consecutive chunks fall in distinct banks.

constexpr int kScanConsumers = 256;                    // eight consumer warps
constexpr int kScanThreads = kScanConsumers + 32;      // and one producer warp

// Named barrier 1 over the consumer warps (the producer warp is not in it).
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kScanConsumers) : "memory");
}
__device__ __forceinline__ bool consumer_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kScanConsumers)
        : "memory");
    return r != 0;
}

// Per-word operations on one 16-byte chunk of K (four 32-bit words).
template <typename T>
struct Chunk;
template <>
struct Chunk<uint16_t> {  // a word holds a bf16 dimension pair
    static constexpr int NPC = 4;  // dimension pairs per chunk
    static __device__ __forceinline__ uint32_t wmax(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));  // NaN-ignoring, exact
        return d;
    }
    static __device__ __forceinline__ float2 pair(const uint4& m, int k) {
        const uint32_t w = k == 0 ? m.x : k == 1 ? m.y : k == 2 ? m.z : m.w;
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
};
template <>
struct Chunk<float> {  // a word holds one fp32 dimension
    static constexpr int NPC = 2;
    static __device__ __forceinline__ uint32_t wmax(uint32_t a, uint32_t b) {
        return __float_as_uint(fmaxf(__uint_as_float(a), __uint_as_float(b)));
    }
    static __device__ __forceinline__ float2 pair(const uint4& m, int k) {
        return k == 0 ? make_float2(__uint_as_float(m.x), __uint_as_float(m.y))
                      : make_float2(__uint_as_float(m.z), __uint_as_float(m.w));
    }
};

__device__ __forceinline__ uint4 flip4(const uint4& x, const uint4& xm, const uint4& sm) {
    return make_uint4((x.x ^ xm.x) & sm.x, (x.y ^ xm.y) & sm.y, (x.z ^ xm.z) & sm.z, (x.w ^ xm.w) & sm.w);
}
template <typename T>
__device__ __forceinline__ uint4 max4(const uint4& a, const uint4& b) {
    return make_uint4(Chunk<T>::wmax(a.x, b.x), Chunk<T>::wmax(a.y, b.y), Chunk<T>::wmax(a.z, b.z),
                      Chunk<T>::wmax(a.w, b.w));
}

// The reference's sign-chosen page extremum starts from -FLT_MAX / +FLT_MAX
// and skips NaN (rocket.cpp:261-278); in the flipped domain that is a clamp.
// It only changes a representative that is -inf or NaN, and such a
// representative on a selected dimension makes the page's sum non-finite
// (inf and NaN propagate through the chains; 0 * inf is NaN), so pages are
// first summed unclamped and a warp whose sums are not all finite recomputes
// its pages with the clamp (CLAMP) -- the same result either way.
__device__ __forceinline__ float2 clamp_rep(float2 m) {
    return make_float2(fmaxf(m.x, -FLT_MAX), fmaxf(m.y, -FLT_MAX));
}

// This lane's value of one page per head.  MODE 0: the page is two rows of the
// stage; MODE 1: prow >= 1 rows; MODE 2: the representatives are in pst (a
// page longer than a stage).  Slot i reads chunk bytes at (i even ? rA : rB)
// + 64 i, its table at (i even ? tA : tB) + 4 i QS, its representatives at
// (i even ? pA : pB) + 4 i CD.
template <typename T, int D, int MAXG, int MODE, bool CLAMP>
__device__ __forceinline__ void lane_page(const uint8_t* rA, const uint8_t* rB, int prow, const uint4* tA,
                                          const uint4* tB, const float* pA, const float* pB, float (&lv)[MAXG]) {
    constexpr int ES = (int)sizeof(T), RB = D * ES;
    constexpr int CD = 16 / ES, NSL = D / CD / 4, NPC = Chunk<T>::NPC;
    constexpr int QU = (CD / 4) * MAXG, QS = (QU + 2) | 1;
    float sv[NSL][MAXG];
#pragma unroll
    for (int i = 0; i < NSL; ++i) {
        const uint4* tq = ((i & 1) ? tB : tA) + 4 * i * QS;
        float2 P[NPC];
        if constexpr (MODE == 2) {
            const float* pp = ((i & 1) ? pB : pA) + 4 * i * CD;
#pragma unroll
            for (int k = 0; k < NPC; ++k) P[k] = *reinterpret_cast<const float2*>(pp + 2 * k);
        } else {
            const uint4 xm = tq[QU], sm = tq[QU + 1];
            const uint8_t* rp = ((i & 1) ? rB : rA) + 64 * i;
            uint4 m = flip4(*reinterpret_cast<const uint4*>(rp), xm, sm);
            if constexpr (MODE == 0) {
                m = max4<T>(m, flip4(*reinterpret_cast<const uint4*>(rp + RB), xm, sm));
            } else {
                for (int rr = 1; rr < prow; ++rr)
                    m = max4<T>(m, flip4(*reinterpret_cast<const uint4*>(rp + rr * RB), xm, sm));
            }
#pragma unroll
            for (int k = 0; k < NPC; ++k) P[k] = CLAMP ? clamp_rep(Chunk<T>::pair(m, k)) : Chunk<T>::pair(m, k);
        }
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
            const float4* qh = reinterpret_cast<const float4*>(tq + h * (CD / 4));
            float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int u = 0; u < CD / 4; ++u) {
                const float4 qq = qh[u];
                ffma2(acc, make_float2(qq.x, qq.y), P[2 * u]);
                ffma2(acc, make_float2(qq.z, qq.w), P[2 * u + 1]);
            }
            sv[i][h] = __fadd_rn(acc.x, acc.y);
        }
    }
#pragma unroll
    for (int w = 1; w < NSL; w *= 2)
#pragma unroll
        for (int i = 0; i < NSL; i += 2 * w)
#pragma unroll
            for (int h = 0; h < MAXG; ++h) sv[i][h] = __fadd_rn(sv[i][h], sv[i + w][h]);
#pragma unroll
    for (int h = 0; h < MAXG; ++h) lv[h] = sv[0][h];
}

// (l0 + l2) + (l1 + l3) over the quad; every lane of the quad gets the sums.
template <int MAXG>
__device__ __forceinline__ void quad_sum(float (&v)[MAXG]) {
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
        v[h] = __fadd_rn(v[h], __shfl_xor_sync(0xffffffffu, v[h], 2));
        v[h] = __fadd_rn(v[h], __shfl_xor_sync(0xffffffffu, v[h], 1));
    }
}

template <typename T, int D, int MAXG>
__global__ void __launch_bounds__(kScanThreads, 2) hsa_scan_kernel(const HsaArgs a) {
    asm volatile("griddepcontrol.launch_dependents;");  // the selection may be scheduled (it waits for this grid)
    constexpr int ES = (int)sizeof(T);
    constexpr int RB = D * ES;           // bytes per K row
    constexpr int CD = 16 / ES;          // dimensions per 16-byte chunk
    constexpr int NCH = D / CD;          // chunks per row
    constexpr int QU = (CD / 4) * MAXG;  // q units per chunk
    constexpr int QS = (QU + 2) | 1;     // table units per chunk (odd)
    constexpr int PST = D + 4;           // carry-mode row stride of pst (floats)

    extern __shared__ __align__(128) uint8_t ring[];
    const int NS = a.nstage;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)NS * kStageBytes);
    uint64_t* empty = full + kMaxScanStages;
    float* pst = reinterpret_cast<float*>(ring + (size_t)NS * kStageBytes + 16 * kMaxScanStages);  // carry: [2][PST]

    __shared__ __align__(16) float qf[MAXG * D];
    __shared__ __align__(16) uint4 tab[NCH * QS];
    __shared__ float sabs[D], qsum[D];
    __shared__ int Rl[D];
    __shared__ unsigned char dsel[D];
    __shared__ float sumall[MAXG], cscale[MAXG];
    __shared__ int scan_tmp[33];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, hc = blockIdx.y, b = blockIdx.z, hk = a.head_begin + hc;
    const int G = a.G;
    const int p_beg = split * a.pages_per_split;
    const int p_end = min(a.nchunks, p_beg + a.pages_per_split);
    if (p_beg >= p_end) return;  // uniform
    const uint8_t* Qg = a.Q + (size_t)b * a.q_stride + (size_t)hk * G * D * sizeof(T);
    const uint8_t* Ku = a.K + (size_t)b * a.kv_stride + (size_t)hk * a.len_k * RB;
    float* wl = a.wlogits + ((size_t)b * a.head_count + hc) * (size_t)G * a.nch_pad;
    const int SR = a.stage_rows;
    const int row_beg = p_beg * a.C, row_end = min(p_end * a.C, a.Lc);
    const int nst = (row_end - row_beg + SR - 1) / SR;
    const bool producer = tid == kScanConsumers;
    auto issue = [&](int s, int slot) {  // the producer lane
        const int t0 = row_beg + s * SR;
        const uint32_t bytes = (uint32_t)(min(SR, row_end - t0) * RB);
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_load(ring + (size_t)slot * kStageBytes, Ku + (size_t)t0 * RB, bytes, &full[slot]);
    };

    if (producer) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], a.wg);  // one arrival per consumer warp of the stage's group
        }
        fence_mbar_init();
        // the first stages stream in while phase 0 runs
        for (int s = 0; s < NS && s < nst; ++s) issue(s, s);
    }
    for (int e = tid; e < G * D; e += kScanThreads) qf[e] = to_f<T>(reinterpret_cast<const T*>(Qg)[e]);
    __syncthreads();

    // ---- phase 0: group query statistics (rocket.cpp:197-250) --------------
    if (tid < D) {
        float sa = 0.0f, sv = 0.0f;
        for (int h = 0; h < G; ++h) {
            const float qv = qf[h * D + tid];
            sa = __fadd_rn(sa, fabsf(qv));
            sv = __fadd_rn(sv, qv);
        }
        sabs[tid] = sa;
        qsum[tid] = sv;
    }
    if (lane == 0 && warp < G) {  // sequential over d, as rocket.cpp:210 accumulates
        const float4* q4 = reinterpret_cast<const float4*>(qf + warp * D);
        float s = 0.0f;
#pragma unroll 8
        for (int v = 0; v < D / 4; ++v) {
            const float4 x = q4[v];
            s = __fadd_rn(s, fabsf(x.x));
            s = __fadd_rn(s, fabsf(x.y));
            s = __fadd_rn(s, fabsf(x.z));
            s = __fadd_rn(s, fabsf(x.w));
        }
        sumall[warp] = s;
    }
    __syncthreads();
    int flag = 0;
    if (tid < D) {
        int rank = 0;
        const float me = sabs[tid];
#pragma unroll 8
        for (int e = 0; e < D; ++e) {
            const float o = sabs[e];
            rank += (o > me || (o == me && e < tid)) ? 1 : 0;
        }
        flag = (a.r >= D || rank < a.r) ? 1 : 0;
    }
    int nr;
    const int pos = block_exclusive_scan(flag, scan_tmp, &nr);
    if (flag) Rl[pos] = tid;
    if (tid < D) dsel[tid] = (unsigned char)flag;
    __syncthreads();
    if (tid < G) {
        float sk;
        if (a.r >= D) {
            sk = sumall[tid];
        } else {
            sk = 0.0f;
            for (int i = 0; i < nr; ++i) sk = __fadd_rn(sk, fabsf(qf[tid * D + Rl[i]]));
        }
        cscale[tid] = __fsqrt_rn(__fmul_rn((float)D, __fdiv_rn(sk, __fadd_rn(sumall[tid], 1e-9f))));
    }
    // the chunk table, one dimension pair per thread (rocket.cpp:263: sign >= 0 takes the max)
    for (int p = tid; p < D / 2; p += kScanThreads) {
        const int d0 = 2 * p, d1 = d0 + 1, c = d0 / CD, e0 = d0 % CD;
        const bool s0 = !(qsum[d0] >= 0.0f), s1 = !(qsum[d1] >= 0.0f);
        const bool n0 = dsel[d0] != 0, n1 = dsel[d1] != 0;
        uint32_t* xw = reinterpret_cast<uint32_t*>(&tab[c * QS + QU]);
        uint32_t* sw = reinterpret_cast<uint32_t*>(&tab[c * QS + QU + 1]);
        if (ES == 2) {
            xw[e0 / 2] = (s0 ? 0x8000u : 0u) | (s1 ? 0x80000000u : 0u);
            sw[e0 / 2] = (n0 ? 0xffffu : 0u) | (n1 ? 0xffff0000u : 0u);
        } else {
            xw[e0] = s0 ? 0x80000000u : 0u;
            xw[e0 + 1] = s1 ? 0x80000000u : 0u;
            sw[e0] = n0 ? 0xffffffffu : 0u;
            sw[e0 + 1] = n1 ? 0xffffffffu : 0u;
        }
        float* qa = reinterpret_cast<float*>(&tab[c * QS]);
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
            float v0 = 0.0f, v1 = 0.0f;
            if (h < G) {
                const float q0 = qf[h * D + d0], q1 = qf[h * D + d1];
                v0 = n0 ? (s0 ? -q0 : q0) : 0.0f;
                v1 = n1 ? (s1 ? -q1 : q1) : 0.0f;
            }
            qa[h * CD + e0] = v0;
            qa[h * CD + e0 + 1] = v1;
        }
    }
    __syncthreads();

    // ---- phase 1: stream K, page representatives, approximate logits ------
    if (warp == kScanConsumers / 32) {
        // producer: refill a slot once its consumer warps released it
        if (lane == 0) {
            int slot = 0, ph = 0;  // slot of stage s, parity of its previous use
            for (int s = NS; s < nst; ++s) {
                if (!mbar_wait_bounded(&empty[slot], (uint32_t)ph, a.err)) break;
                fence_proxy_async();
                issue(s, slot);
                if (++slot == NS) {
                    slot = 0;
                    ph ^= 1;
                }
            }
        }
        return;
    }
    const int WG = a.wg, NGRP = a.ngrp, PPS = a.pps;
    if (warp >= WG * NGRP) return;  // idle consumer warp (no barrier counts it)
    const int g = warp / WG, wi = warp - g * WG;
    const int j = lane & 3, qd = lane >> 2, qpar = qd & 1;
    const int quad = wi * 8 + qd;  // page within the stage
    // slot i of this lane reads chunk j + 4 (i ^ qpar)
    const int offA = 16 * (j + 4 * qpar), offB = 16 * (j - 4 * qpar);
    const uint4* tA = tab + (j + 4 * qpar) * QS;
    const uint4* tB = tab + (j - 4 * qpar) * QS;
    // lane j divides heads j, j + 4, ...
    float my_scale[(MAXG + 3) / 4];
#pragma unroll
    for (int u = 0; u < (MAXG + 3) / 4; ++u) my_scale[u] = (j + 4 * u < G) ? cscale[j + 4 * u] : 1.0f;

    if (!a.carry_mode) {
        int slot = g, ph = 0;
        for (int s = g; s < nst; s += NGRP) {
            const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)ph, a.err);
            if (!__all_sync(0xffffffffu, ok)) break;  // the producer's wait then runs out too
            const int c_lo = p_beg + s * PPS;
            const int npg = min(PPS, p_end - c_lo);
            const int t0 = row_beg + s * SR;
            const uint8_t* st = ring + (size_t)slot * kStageBytes;
            float v[MAXG];
#pragma unroll
            for (int h = 0; h < MAXG; ++h) v[h] = 0.0f;
            const int r0 = quad * a.C;
            const int prow = min(a.C, row_end - t0 - r0);
            const uint8_t* rbase = st + (size_t)r0 * RB;
            if (quad < npg) {
                if (prow == 2)
                    lane_page<T, D, MAXG, 0, false>(rbase + offA, rbase + offB, 2, tA, tB, nullptr, nullptr, v);
                else
                    lane_page<T, D, MAXG, 1, false>(rbase + offA, rbase + offB, prow, tA, tB, nullptr, nullptr, v);
            }
            quad_sum<MAXG>(v);
            bool finite = true;
#pragma unroll
            for (int h = 0; h < MAXG; ++h) finite = finite && fabsf(v[h]) <= FLT_MAX;
            if (!__all_sync(0xffffffffu, finite)) {
                // a non-finite representative somewhere in the warp's pages: redo them clamped
#pragma unroll
                for (int h = 0; h < MAXG; ++h) v[h] = 0.0f;
                if (quad < npg)
                    lane_page<T, D, MAXG, 1, true>(rbase + offA, rbase + offB, prow, tA, tB, nullptr, nullptr, v);
                quad_sum<MAXG>(v);
            }
            if (quad < npg) {
#pragma unroll
                for (int u = 0; u < (MAXG + 3) / 4; ++u) {
                    const int h = j + 4 * u;
                    float mine = 0.0f;
#pragma unroll
                    for (int hh = 0; hh < MAXG; ++hh)
                        if (hh == h) mine = v[hh];
                    if (h < G) wl[(size_t)h * a.nch_pad + c_lo + quad] = __fdiv_rn(mine, my_scale[u]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            slot += NGRP;
            if (slot >= NS) {
                slot -= NS;
                ph ^= 1;
            }
        }
    } else {
        // a page spans several stages: all consumer warps take every stage;
        // threads tid < D keep the running maximum of s x on dimension tid
        const bool c_sg = tid < D && !(qsum[tid] >= 0.0f), c_en = tid < D && dsel[tid] != 0;
        float carry = __int_as_float(0x7fffffff);  // NaN: nothing seen yet
        int slot = 0, ph = 0;
        for (int s = 0; s < nst; ++s) {
            const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)ph, a.err);
            // uniform decision: the loop below meets named barriers
            if (consumer_any(!ok)) break;
            const int t0 = row_beg + s * SR, nrows = min(SR, row_end - t0);
            const uint8_t* st = ring + (size_t)slot * kStageBytes;
            const int c_lo = t0 / a.C;
            const int c_hi = (t0 + nrows == row_end) ? p_end : (t0 + nrows) / a.C;
            if (tid < D) {
                for (int rr = 0; rr < nrows; ++rr) {
                    const int t = t0 + rr;
                    float x = to_f<T>(*reinterpret_cast<const T*>(st + (size_t)rr * RB + (size_t)tid * ES));
                    x = c_en ? (c_sg ? -x : x) : 0.0f;
                    carry = fmaxf(carry, x);
                    if ((t + 1) % a.C == 0 || t == row_end - 1) {
                        pst[(t / a.C - c_lo) * PST + tid] = fmaxf(carry, -FLT_MAX);
                        carry = __int_as_float(0x7fffffff);
                    }
                }
            }
            consumer_sync();
            if (warp == 0) {
                float v[MAXG];
#pragma unroll
                for (int h = 0; h < MAXG; ++h) v[h] = 0.0f;
                const int npg = c_hi - c_lo;  // at most two pages end in a stage
                if (quad < npg) {
                    const float* pp = pst + quad * PST;
                    lane_page<T, D, MAXG, 2, true>(nullptr, nullptr, 0, tA, tB, pp + (j + 4 * qpar) * CD,
                                                   pp + (j - 4 * qpar) * CD, v);
                }
                quad_sum<MAXG>(v);
                if (quad < npg) {
#pragma unroll
                    for (int u = 0; u < (MAXG + 3) / 4; ++u) {
                        const int h = j + 4 * u;
                        float mine = 0.0f;
#pragma unroll
                        for (int hh = 0; hh < MAXG; ++hh)
                            if (hh == h) mine = v[hh];
                        if (h < G) wl[(size_t)h * a.nch_pad + c_lo + quad] = __fdiv_rn(mine, my_scale[u]);
                    }
                }
            }
            consumer_sync();  // pst reuse
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == NS) {
                slot = 0;
                ph ^= 1;
            }
        }
    }
}

// ===========================================================================
// Select kernel: phase 2, one 128-thread CTA per unit
// ===========================================================================
// The unit's page logits are staged in shared memory by one bulk copy (SMEM;
// otherwise they are used in place in the workspace).  Per-head page softmax
// (rocket.cpp:291-309) with the deterministic exp and the 256-way summation
// order (thread t holds partials t and t + 128, partial j summing pages j,
// j + 256, ... ascending; then the halving tree), the group sum
// (rocket.cpp:311-323), a 4 x 8-bit radix select of the final_k-th token by
// (score desc, index asc) with pages weighted by their token count, and a
// stable compaction in ascending token order (rocket.cpp:325-340); then the
// recent window.  Small CTAs with little shared memory, so several units
// proceed side by side per SM.
constexpr int kSelThreads = 128;

template <int MAXG, bool SMEM>
__global__ void __launch_bounds__(kSelThreads, 8) hsa_select_kernel(const HsaArgs a) {
    // launched as a programmatic dependent of the scan: its page logits are complete and visible after this
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");  // the attention may be scheduled (it waits for this grid)
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t* lbar = reinterpret_cast<uint64_t*>(sm);
    float* r0 = reinterpret_cast<float*>(sm + 128);  // staged logits [G][NP]

    __shared__ float part[MAXG][kSelThreads];
    __shared__ float red_[MAXG][kSelThreads / 32];
    __shared__ float hmax[MAXG], hinv[MAXG];
    __shared__ int hist[256], scan_tmp[66];
    __shared__ int s_kk;
    __shared__ uint32_t s_prefix;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t unit = blockIdx.x;
    const int G = a.G, nch = a.nchunks, NP = a.nch_pad, C = a.C, Lc = a.Lc;
    int* sel = a.sel + unit * a.sel_stride;
    int nfirst;
    if (nch > 0) {
        float* wg = a.wlogits + unit * (size_t)G * NP;
        float* wl = SMEM ? r0 : wg;  // [G][NP]
        if (SMEM && tid == 0) {
            mbar_init(lbar, 1);
            fence_mbar_init();
            // the unit's logits are one contiguous, 16-byte aligned block
            const uint32_t bytes = (uint32_t)((size_t)G * NP * sizeof(float));
            mbar_arrive_expect_tx(lbar, bytes);
            bulk_load(r0, wg, bytes, lbar);
        }
        for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
        __syncthreads();
        const bool ok = SMEM ? mbar_wait_bounded(lbar, 0, a.err) : true;
        if (__syncthreads_or(!ok)) return;  // uniform: nobody passes an incomplete copy

        // per-head maximum (rocket.cpp:294: starts at -FLT_MAX)
        float m[MAXG];
#pragma unroll
        for (int h = 0; h < MAXG; ++h) m[h] = -FLT_MAX;
        for (int c = tid; c < nch; c += kSelThreads)
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
                if (h < G) m[h] = fmaxf(m[h], wl[(size_t)h * NP + c]);
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
            float v = m[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) red_[h][warp] = v;
        }
        __syncthreads();
        if (tid < G) {
            float v = -FLT_MAX;
            for (int wi = 0; wi < kSelThreads / 32; ++wi) v = fmaxf(v, red_[tid][wi]);
            hmax[tid] = v;
        }
        __syncthreads();
        // p = exp(l - max) over the logits; partials t and t + 128
        float P0[MAXG], P1[MAXG];
#pragma unroll
        for (int h = 0; h < MAXG; ++h) P0[h] = P1[h] = 0.0f;
        // the two pages c and c + 128 of a thread through the paired exp (each lane's result is det_expf's)
        for (int base = 0; base < nch; base += 256) {
            const int c0 = base + tid, c1 = c0 + kSelThreads;
            const bool v0 = c0 < nch, v1 = c1 < nch;
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
                if (h < G) {
                    float* row = wl + (size_t)h * NP;
                    const float x0 = v0 ? __fsub_rn(row[c0], hmax[h]) : 0.0f;
                    const float x1 = v1 ? __fsub_rn(row[c1], hmax[h]) : 0.0f;
                    const float2 e = det_expf2(make_float2(x0, x1));
                    if (v0) {
                        row[c0] = e.x;
                        P0[h] = __fadd_rn(P0[h], e.x);
                    }
                    if (v1) {
                        row[c1] = e.y;
                        P1[h] = __fadd_rn(P1[h], e.y);
                    }
                }
        }
        // halving tree: s = 128 in the thread, 64 and 32 in shared memory, 16 ... 1 in warp 0
#pragma unroll
        for (int h = 0; h < MAXG; ++h) part[h][tid] = __fadd_rn(P0[h], P1[h]);
        __syncthreads();
        if (tid < 64)
#pragma unroll
            for (int h = 0; h < MAXG; ++h) part[h][tid] = __fadd_rn(part[h][tid], part[h][tid + 64]);
        __syncthreads();
        if (warp == 0) {
#pragma unroll
            for (int h = 0; h < MAXG; ++h) {
                float v = __fadd_rn(part[h][lane], part[h][lane + 32]);
#pragma unroll
                for (int s = 16; s > 0; s >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, s));
                if (lane == 0 && h < G) hinv[h] = __fdiv_rn(1.0f, __fadd_rn(v, 1e-9f));
            }
        }
        __syncthreads();
        // group score per page as an order-preserving key, over head 0's row
        uint32_t* keys = reinterpret_cast<uint32_t*>(wl);
        for (int c = tid; c < nch; c += kSelThreads) {
            float g = 0.0f;
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
                if (h < G) g = __fadd_rn(g, __fmul_rn(wl[(size_t)h * NP + c], hinv[h]));
            keys[c] = float_key(g);
        }
        if (tid == 0) {
            s_prefix = 0u;
            s_kk = a.final_k;
        }
        __syncthreads();
        // 4 x 8-bit radix select of the final_k-th token.  Warp 0 scans the
        // 256 bins from the top digit down and clears them: two barriers a pass.
        uint32_t mask = 0u;
        for (int shift = 24; shift >= 0; shift -= 8) {
            const uint32_t prefix = s_prefix;
            for (int c = tid; c < nch; c += kSelThreads) {
                const uint32_t k = keys[c];
                if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], min(C, Lc - c * C));
            }
            __syncthreads();
            if (warp == 0) {
                int cnt[8], local = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    cnt[j] = hist[255 - 8 * lane - j];
                    local += cnt[j];
                }
                int incl = local;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                const int before = incl - local;
                const int kk = s_kk;
                __syncwarp();
                if (before < kk && before + local >= kk) {
                    int run = before;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (run + cnt[j] >= kk) {
                            s_kk = kk - run;
                            s_prefix = prefix | ((uint32_t)(255 - 8 * lane - j) << shift);
                            break;
                        }
                        run += cnt[j];
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) hist[255 - 8 * lane - j] = 0;
            }
            mask |= 255u << shift;
            __syncthreads();
        }
        const uint32_t thr = s_prefix;
        const int need = s_kk;
        // stable compaction: thread t owns the contiguous page range [c_beg, c_end);
        // threshold ties are taken in token order until `need` is met, so the
        // output position is (weight above the threshold before the range) +
        // min(tie weight before the range, need): one scan of both weights
        const int per = (nch + kSelThreads - 1) / kSelThreads;
        const int c_beg = min(nch, tid * per), c_end = min(nch, c_beg + per);
        int gtw = 0, eqw = 0;
        for (int c = c_beg; c < c_end; ++c) {
            const uint32_t k = keys[c];
            const int wt = min(C, Lc - c * C);
            if (k > thr) gtw += wt;
            else if (k == thr) eqw += wt;
        }
        int eq_rank, tot_gt, tot_eq;
        const int gt_before = block_exclusive_scan2(gtw, eqw, scan_tmp, &eq_rank, &tot_gt, &tot_eq);
        int pos = gt_before + min(eq_rank, need);
        for (int c = c_beg; c < c_end; ++c) {
            const uint32_t k = keys[c];
            const int wt = min(C, Lc - c * C);
            int take = 0;
            if (k > thr) {
                take = wt;
            } else if (k == thr) {
                take = max(0, min(wt, need - eq_rank));
                eq_rank += wt;
            }
            for (int j = 0; j < take; ++j) sel[pos + j] = c * C + j;
            pos += take;
        }
        nfirst = a.final_k;
    } else {
        // no scoring needed: every eligible token (final_k >= Lc) or none
        nfirst = a.final_k > 0 ? Lc : 0;
        for (int t = tid; t < nfirst; t += kSelThreads) sel[t] = t;
    }
    for (int t = tid; t < a.w; t += kSelThreads) sel[nfirst + t] = Lc + t;
    if (tid == 0 && a.n_sel) a.n_sel[unit] = nfirst + a.w;
}

// ===========================================================================
// Attention kernel: phase 3
// ===========================================================================
// Exact attention over the unit's selected rows (rocket.cpp:342-378).
// Gathers are direct 16-byte read-only loads, several tokens in flight per
// thread.  Pass A: eight lanes per token form q.k for every head (paired
// FMAs, q held in registers); pass B: per-head max, p = exp(s - max) and
// sum(p); pass C: each thread owns one 16-byte vector of the V row and
// accumulates p * v per head; the token groups are merged in shared memory.
// SMEM: the selected indices and scores live in shared memory (the common
// case); otherwise in the workspace.
template <typename T, int D, int MAXG, bool SMEM>
__global__ void __launch_bounds__(kNT, 3) hsa_attn_kernel(const HsaArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    float* red = reinterpret_cast<float*>(sm);  // merge buffer [NGC][MAXG][D]
    int* sel_s = reinterpret_cast<int*>(sm + a.tail_r0_bytes);
    float* sc_s = reinterpret_cast<float*>(sm + a.tail_r0_bytes + (size_t)a.score_stride * 4);

    __shared__ __align__(16) float qf[MAXG * D];
    __shared__ float part_[MAXG][kNT / 32];
    __shared__ float hmax[MAXG], hinv[MAXG];

    constexpr size_t RB = (size_t)D * sizeof(T);
    constexpr int EPV = 16 / (int)sizeof(T);  // elements per 16-byte vector
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hc = blockIdx.x, b = blockIdx.y, hk = a.head_begin + hc;
    const int G = a.G;
    const size_t unit = (size_t)b * a.head_count + hc;
    const uint8_t* Qg = a.Q + (size_t)b * a.q_stride + (size_t)hk * G * D * sizeof(T);
    const uint8_t* Ku = a.K + (size_t)b * a.kv_stride + (size_t)hk * a.len_k * RB;
    const uint8_t* Vu = a.V + (size_t)b * a.kv_stride + (size_t)hk * a.len_k * RB;
    const int* sel_g = a.sel + unit * a.sel_stride;
    const int nfirst = a.nchunks > 0 ? a.final_k : (a.final_k > 0 ? a.Lc : 0);
    const int n = nfirst + a.w;
    const int* sel = SMEM ? sel_s : sel_g;
    float* sc = SMEM ? sc_s : a.wscore + unit * (size_t)G * a.score_stride;  // [G][score_stride]

    for (int e = tid; e < G * D; e += kNT) qf[e] = to_f<T>(reinterpret_cast<const T*>(Qg)[e]);
    // launched as a programmatic dependent of the selection: its lists are complete and visible after this
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (SMEM)
        for (int i = tid; i < n; i += kNT) sel_s[i] = sel_g[i];
    __syncthreads();

    constexpr int CPR = (int)RB / 16;  // 16-byte vectors per row
    constexpr int NPART = 8;           // pass-A lanes per token
    constexpr int CPP = CPR / NPART;   // vectors per lane
    constexpr int TPR = kNT / NPART;   // tokens per pass-A round
    constexpr int UA = CPP >= 4 ? 1 : 4 / CPP;
    constexpr int NGC = kNT / CPR;     // pass-C token groups
    constexpr int UC = 4;
    constexpr bool QREG = CPP * EPV * MAXG <= 48;  // the lane's q values fit in registers
    static_assert(CPP >= 1 && NGC >= 1, "row layout");
    // ---- pass A: scores ----
    {
        const int lp = tid % NPART, tok = tid / NPART;
        float2 qr[QREG ? CPP * EPV / 2 : 1][MAXG];
        if constexpr (QREG) {
#pragma unroll
            for (int c = 0; c < CPP; ++c)
#pragma unroll
                for (int e2 = 0; e2 < EPV / 2; ++e2)
#pragma unroll
                    for (int h = 0; h < MAXG; ++h)
                        qr[c * (EPV / 2) + e2][h] =
                            h < G ? *reinterpret_cast<const float2*>(qf + h * D + (lp + c * NPART) * EPV + 2 * e2)
                                  : make_float2(0.0f, 0.0f);
        }
        for (int j0 = 0; j0 < n; j0 += TPR * UA) {  // uniform trip count
            uint4 kw[UA][CPP];
#pragma unroll
            for (int u = 0; u < UA; ++u) {
                const int j = j0 + u * TPR + tok;
                if (j < n) {
                    const uint4* kr = reinterpret_cast<const uint4*>(Ku + (size_t)sel[j] * RB);
#pragma unroll
                    for (int c = 0; c < CPP; ++c) kw[u][c] = __ldg(kr + lp + c * NPART);
                }
            }
#pragma unroll
            for (int u = 0; u < UA; ++u) {
                const int j = j0 + u * TPR + tok;
                float2 acc[MAXG];
#pragma unroll
                for (int h = 0; h < MAXG; ++h) acc[h] = make_float2(0.0f, 0.0f);
                if (j < n) {
#pragma unroll
                    for (int c = 0; c < CPP; ++c) {
                        float kf[EPV];
                        vec_to_f<T>(kw[u][c], kf);
#pragma unroll
                        for (int e2 = 0; e2 < EPV / 2; ++e2) {
                            const float2 kv = make_float2(kf[2 * e2], kf[2 * e2 + 1]);
#pragma unroll
                            for (int h = 0; h < MAXG; ++h) {
                                if constexpr (QREG) {
                                    ffma2(acc[h], qr[c * (EPV / 2) + e2][h], kv);
                                } else if (h < G) {
                                    const float2 q = *reinterpret_cast<const float2*>(
                                        qf + h * D + (lp + c * NPART) * EPV + 2 * e2);
                                    ffma2(acc[h], q, kv);
                                }
                            }
                        }
                    }
                }
                float dot[MAXG], mine = 0.0f;
#pragma unroll
                for (int h = 0; h < MAXG; ++h) {
                    dot[h] = acc[h].x + acc[h].y;
                    dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], 4);
                    dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], 2);
                    dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], 1);
                    if (h == lp) mine = dot[h];
                }
                if (j < n && lp < G) sc[(size_t)lp * a.score_stride + j] = mine * a.inv_sqrt_d;
            }
        }
    }
    __syncthreads();
    // ---- pass B: softmax statistics over the n scores per head ----
    {
        float m[MAXG];
#pragma unroll
        for (int h = 0; h < MAXG; ++h) m[h] = -FLT_MAX;  // rocket.cpp:350: all -inf gives exp(-inf) = 0
        for (int i = tid; i < n; i += kNT)
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
                if (h < G) m[h] = fmaxf(m[h], sc[(size_t)h * a.score_stride + i]);
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
            float v = m[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) part_[h][warp] = v;
        }
        __syncthreads();
        if (tid < G) {
            float v = -FLT_MAX;
            for (int wi = 0; wi < kNT / 32; ++wi) v = fmaxf(v, part_[tid][wi]);
            hmax[tid] = v;
        }
        __syncthreads();
        float ssum[MAXG];
#pragma unroll
        for (int h = 0; h < MAXG; ++h) ssum[h] = 0.0f;
        for (int i = tid; i < n; i += kNT)
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
                if (h < G) {
                    const float p = __expf(sc[(size_t)h * a.score_stride + i] - hmax[h]);
                    sc[(size_t)h * a.score_stride + i] = p;
                    ssum[h] += p;
                }
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
            float v = ssum[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) part_[h][warp] = v;
        }
        __syncthreads();
        if (tid < G) {
            float v = 0.0f;
            for (int wi = 0; wi < kNT / 32; ++wi) v += part_[tid][wi];
            hinv[tid] = 1.0f / (v + 1e-9f);  // rocket.cpp:367
        }
        __syncthreads();
    }
    // ---- pass C: p * v ----
    const int vi = tid % CPR, cg = tid / CPR;
    float acc[MAXG][EPV];
#pragma unroll
    for (int h = 0; h < MAXG; ++h)
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[h][e] = 0.0f;
    for (int j0 = cg; j0 < n; j0 += NGC * UC) {
        uint4 vw[UC];
#pragma unroll
        for (int u = 0; u < UC; ++u) {
            const int j = j0 + u * NGC;
            if (j < n) vw[u] = ld_global_v4(reinterpret_cast<const uint4*>(Vu + (size_t)sel[j] * RB) + vi);
        }
#pragma unroll
        for (int u = 0; u < UC; ++u) {
            const int j = j0 + u * NGC;
            if (j < n) {
                float vf[EPV];
                vec_to_f<T>(vw[u], vf);
#pragma unroll
                for (int h = 0; h < MAXG; ++h) {
                    if (h < G) {
                        const float p = sc[(size_t)h * a.score_stride + j];
#pragma unroll
                        for (int e = 0; e < EPV; ++e) acc[h][e] = fmaf(p, vf[e], acc[h][e]);
                    }
                }
            }
        }
    }
    // merge the NGC token groups
#pragma unroll
    for (int h = 0; h < MAXG; ++h)
        if (h < G)
#pragma unroll
            for (int e = 0; e < EPV; ++e) red[((size_t)cg * MAXG + h) * D + vi * EPV + e] = acc[h][e];
    __syncthreads();
    float* Ob = a.O + (size_t)b * a.H * D + (size_t)hk * G * D;
    for (int e = tid; e < G * D; e += kNT) {
        const int h = e / D, d = e - h * D;
        float o = 0.0f;
        for (int g = 0; g < NGC; ++g) o += red[((size_t)g * MAXG + h) * D + d];
        Ob[h * D + d] = n > 0 ? o * hinv[h] : 0.0f;
    }
}

// ===========================================================================
// Page summaries (persistent cache state: per-page max and min of K)
// ===========================================================================
// For every (item, KV head), dimension d and page p (rows p C .. min(p C + C,
// Lc) - 1 of the compressed cache), the summary holds the NaN-ignoring max of
// x and of -x over the page's rows, in the K element type, laid out
// [2][D][npp] with the pages of a dimension contiguous.  These are exactly the
// values hsa_scan_kernel forms in its sign-flipped domain (max.bf16x2 / fmaxf
// over the rows, the first row first), so a scan that reads them for the
// selected dimensions -- max x where sum_h q >= 0, max -x elsewhere -- repeats
// the same float operations and selects the same tokens.

constexpr int kSumBuildNT = 256;

// Zeroes every item's non-finite masks ([KV head][D / 32] words after its extrema); one CTA per item.
__global__ void hsa_summary_mask_clear(uint8_t* summary, long long sum_stride, long long mask_off, int words) {
    uint32_t* m = reinterpret_cast<uint32_t*>(summary + (size_t)blockIdx.x * sum_stride + mask_off);
    for (int x = threadIdx.x; x < words; x += blockDim.x) m[x] = 0u;
}

// The extrema of one page (rows p C .. min(p C + C, Lc) - 1) over two 16-byte
// chunks of the row: NaN-ignoring max of x and of -x, word by word, the first
// row first -- the scan's operations in its sign-flipped domain.
template <typename T, int RB>
__device__ __forceinline__ void page_extrema(const uint8_t* Kh, int p, int C, int Lc, int ch, uint4 (&m)[2],
                                             uint4 (&n)[2]) {
    constexpr uint32_t FLIP = sizeof(T) == 2 ? 0x80008000u : 0x80000000u;
    const uint4 fl = make_uint4(FLIP, FLIP, FLIP, FLIP);
    const int r0 = p * C, r1 = min(r0 + C, Lc);
    const uint4* row = reinterpret_cast<const uint4*>(Kh + (size_t)r0 * RB) + ch;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        m[u] = __ldg(row + u);
        n[u] = make_uint4(m[u].x ^ fl.x, m[u].y ^ fl.y, m[u].z ^ fl.z, m[u].w ^ fl.w);
    }
    for (int r = r0 + 1; r < r1; ++r) {
        row += RB / 16;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const uint4 v = __ldg(row + u);
            m[u] = max4<T>(m[u], v);
            n[u] = max4<T>(n[u], make_uint4(v.x ^ fl.x, v.y ^ fl.y, v.z ^ fl.z, v.w ^ fl.w));
        }
    }
}

// Non-finite flags (-inf or NaN: the scan clamps such a representative at -FLT_MAX) of the dimensions of
// one 32-bit word of the extrema, as bits at the dimensions' positions modulo 32.
template <typename T>
__device__ __forceinline__ uint32_t nonfinite_bits(uint32_t m, uint32_t n, int d0) {
    uint32_t bits = 0u;
    if (sizeof(T) == 2) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const uint32_t x = (m >> (16 * hf)) & 0xffffu, y = (n >> (16 * hf)) & 0xffffu;
            if ((x & 0x7fffu) > 0x7f80u || x == 0xff80u || (y & 0x7fffu) > 0x7f80u || y == 0xff80u)
                bits |= 1u << ((d0 + hf) & 31);
        }
    } else if ((m & 0x7fffffffu) > 0x7f800000u || m == 0xff800000u || (n & 0x7fffffffu) > 0x7f800000u ||
               n == 0xff800000u) {
        bits = 1u << (d0 & 31);
    }
    return bits;
}

// One warp per 64 pages of an (item, KV head): lane l takes pages 2l and
// 2l + 1 of the warp's group and reads their rows 32 bytes at a time (whole
// sectors), and per dimension stores the two pages' extrema as one 4-byte
// (bf16) or 8-byte (fp32) word, so a warp writes 128 or 256 contiguous bytes
// of a dimension's row per store.  No shared-memory transpose.  Pages from
// nchunks to npp (the row padding) are written as zeros.
constexpr int kBuildPagesPerWarp = 64;

template <typename T, int D>
__global__ void __launch_bounds__(kSumBuildNT, sizeof(T) == 2 ? 4 : 3) hsa_summary_build_kernel(const uint8_t* K, long long kv_stride,
                                                                         int len_k, int C, int Lc, int nchunks,
                                                                         int npp, uint8_t* summary,
                                                                         long long sum_stride, long long mask_off) {
    constexpr int ES = (int)sizeof(T), RB = D * ES, NCH = RB / 16;  // 16-byte chunks per row
    constexpr int WPC = 4;                                          // 32-bit words per chunk
    constexpr int DPW = 4 / ES;                                     // dimensions per word
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hk = blockIdx.y, b = blockIdx.z;
    const int g0 = (blockIdx.x * (kSumBuildNT / 32) + warp) * kBuildPagesPerWarp;
    if (g0 >= npp) return;  // warp-uniform
    const int pa = g0 + 2 * lane, pb = pa + 1;  // npp is a multiple of 8: pa < npp implies pb < npp
    const uint8_t* Kh = K + (size_t)b * kv_stride + (size_t)hk * len_k * RB;
    T* Sm = reinterpret_cast<T*>(summary + (size_t)b * sum_stride + (size_t)hk * 2 * D * npp * ES);  // [2][D][npp]
    const bool va = pa < nchunks, vb = pb < nchunks, wr = pa < npp;
    uint32_t* mask = reinterpret_cast<uint32_t*>(summary + (size_t)b * sum_stride + mask_off) + hk * (D / 32);
#pragma unroll 1
    for (int ch = 0; ch < NCH; ch += 2) {
        uint32_t nf = 0u;  // non-finite flags of this chunk pair's dimensions (they share one mask word)
        uint4 ma[2] = {}, na[2] = {}, mb[2] = {}, nb[2] = {};
        if (va) page_extrema<T, RB>(Kh, pa, C, Lc, ch, ma, na);
        if (vb) page_extrema<T, RB>(Kh, pb, C, Lc, ch, mb, nb);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
#pragma unroll
            for (int w = 0; w < WPC; ++w) {
                const uint32_t am = w == 0 ? ma[u].x : w == 1 ? ma[u].y : w == 2 ? ma[u].z : ma[u].w;
                const uint32_t an = w == 0 ? na[u].x : w == 1 ? na[u].y : w == 2 ? na[u].z : na[u].w;
                const uint32_t bm = w == 0 ? mb[u].x : w == 1 ? mb[u].y : w == 2 ? mb[u].z : mb[u].w;
                const uint32_t bn = w == 0 ? nb[u].x : w == 1 ? nb[u].y : w == 2 ? nb[u].z : nb[u].w;
                const int d0 = ((ch + u) * WPC + w) * DPW;  // first dimension of the word
                if (va) nf |= nonfinite_bits<T>(am, an, d0);
                if (vb) nf |= nonfinite_bits<T>(bm, bn, d0);
                if (!wr) continue;
                if (ES == 2) {
                    *reinterpret_cast<uint32_t*>(Sm + (size_t)d0 * npp + pa) = __byte_perm(am, bm, 0x5410);
                    *reinterpret_cast<uint32_t*>(Sm + (size_t)(d0 + 1) * npp + pa) = __byte_perm(am, bm, 0x7632);
                    *reinterpret_cast<uint32_t*>(Sm + (size_t)(D + d0) * npp + pa) = __byte_perm(an, bn, 0x5410);
                    *reinterpret_cast<uint32_t*>(Sm + (size_t)(D + d0 + 1) * npp + pa) = __byte_perm(an, bn, 0x7632);
                } else {
                    *reinterpret_cast<uint2*>(Sm + (size_t)d0 * npp + pa) = make_uint2(am, bm);
                    *reinterpret_cast<uint2*>(Sm + (size_t)(D + d0) * npp + pa) = make_uint2(an, bn);
                }
            }
        }
        // a chunk pair's 16 (bf16) or 8 (fp32) dimensions lie in one 32-dimension mask word
        const uint32_t m = __reduce_or_sync(0xffffffffu, nf);
        if (lane == 0 && m) atomicOr(mask + (ch * WPC * DPW) / 32, m);
    }
}

// Long pages (four rows or more): one thread per (page, 32-bit word of the
// row) reads the page's rows word by word, so consecutive threads read
// consecutive words of a row (coalesced along the row), and the extrema pass
// through a [2][D][TP] tile in shared memory to leave as 16-byte runs of a
// dimension's pages.  Same values as hsa_summary_build_kernel.
// bf16 rows of 128 values, pages of one or two rows (the headline layout).  A warp takes 16 pages: it reads
// one page per load instruction (lanes 0-15 the 16 chunks of the first row, lanes 16-31 those of the
// second), so K is read once in whole lines; one shuffle gives each lane both rows' chunk, and lanes 0-15
// form the max of x, lanes 16-31 the max of -x of the same eight dimensions (max(first row, second row), as
// page_extrema).  The warp's extrema pass through its own shared-memory tile, [page pair][summary row],
// written as 32-byte vectors, and leave as one 32-byte run of pages per summary row and pair of lanes, so
// every output sector is written whole by one instruction.  Pages from nchunks to npp are written as zeros.
constexpr int kTilePages = 16;
__global__ void __launch_bounds__(kSumBuildNT, 3) hsa_summary_build_tile_kernel(const uint8_t* K, long long kv_stride,
                                                                              int len_k, int C, int Lc, int nchunks,
                                                                              int npp, uint8_t* summary,
                                                                              long long sum_stride, long long mask_off) {
    constexpr int D = 128, RB = D * 2, NR = 2 * D;  // summary rows of an (item, KV head): max x, then max -x
    extern __shared__ __align__(16) uint32_t tsm[];  // [warp][page pair][NR] words
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hk = blockIdx.y, b = blockIdx.z;
    const int p0 = (blockIdx.x * (kSumBuildNT / 32) + warp) * kTilePages;
    if (p0 >= npp) return;  // warp-uniform
    const int np = min(kTilePages, npp - p0);  // 16, or 8 at the end (npp is a multiple of 8)
    const int sg = lane >> 4, c = lane & 15;   // sign (0: max x, 1: max -x) and chunk: dimensions 8c .. 8c + 7
    uint32_t* wt = tsm + warp * (kTilePages / 2) * NR;
    const uint8_t* Kh = K + (size_t)b * kv_stride + (size_t)hk * len_k * RB + c * 16;
    const uint32_t fl = sg ? 0x80008000u : 0u;
    uint32_t nf = 0u;  // non-finite flags of the lane's eight dimensions
#pragma unroll 1
    for (int hb = 0; hb < np / 8; ++hb) {  // eight pages at a time
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int p = p0 + 8 * hb + j;
            v[j] = make_uint4(0u, 0u, 0u, 0u);
            if (p < nchunks) {
                const int r0 = p * C, r = r0 + sg < min(r0 + C, Lc) ? r0 + sg : r0;  // a one-row page repeats it
                v[j] = __ldg(reinterpret_cast<const uint4*>(Kh + (size_t)r * RB));
            }
        }
        uint32_t acc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t o[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const uint32_t q = __shfl_xor_sync(0xffffffffu, o[w], 16);
                const uint32_t r0w = sg ? q : o[w], r1w = sg ? o[w] : q;  // the first row first
                acc[j][w] = Chunk<uint16_t>::wmax(r0w ^ fl, r1w ^ fl);
            }
            if (p0 + 8 * hb + j < nchunks) {
#pragma unroll
                for (int w = 0; w < 4; ++w)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const uint32_t x = (acc[j][w] >> (16 * hf)) & 0xffffu;
                        if ((x & 0x7fffu) > 0x7f80u || x == 0xff80u) nf |= 1u << (2 * w + hf);
                    }
            } else {
#pragma unroll
                for (int w = 0; w < 4; ++w) acc[j][w] = 0u;  // padding pages
            }
        }
        // page pair m (pages 2m, 2m + 1 of the tile): the words of dimensions 8c .. 8c + 7, two vectors
#pragma unroll
        for (int mm = 0; mm < 4; ++mm) {
            uint32_t wd[8];
#pragma unroll
            for (int d = 0; d < 8; ++d)
                wd[d] = __byte_perm(acc[2 * mm][d >> 1], acc[2 * mm + 1][d >> 1], (d & 1) ? 0x7632u : 0x5410u);
            uint32_t* dst = wt + (4 * hb + mm) * NR + sg * D + 8 * c;
            *reinterpret_cast<uint4*>(dst) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
            *reinterpret_cast<uint4*>(dst + 4) = make_uint4(wd[4], wd[5], wd[6], wd[7]);
        }
    }
    __syncwarp();
    uint16_t* Sb = reinterpret_cast<uint16_t*>(summary + (size_t)b * sum_stride + (size_t)hk * NR * npp * 2);  // [NR][npp]
    if (np == kTilePages) {  // two lanes per summary row, 16 bytes each: 32 bytes of pages
#pragma unroll 4
        for (int r0 = 0; r0 < NR; r0 += 16) {
            const int row = r0 + (lane >> 1), h = lane & 1;
            const uint4 o = make_uint4(wt[(4 * h) * NR + row], wt[(4 * h + 1) * NR + row], wt[(4 * h + 2) * NR + row],
                                       wt[(4 * h + 3) * NR + row]);
            *reinterpret_cast<uint4*>(Sb + (size_t)row * npp + p0 + 8 * h) = o;
        }
    } else {  // the last eight pages: one lane per row
#pragma unroll 4
        for (int r0 = 0; r0 < NR; r0 += 32) {
            const int row = r0 + lane;
            const uint4 o = make_uint4(wt[row], wt[NR + row], wt[2 * NR + row], wt[3 * NR + row]);
            *reinterpret_cast<uint4*>(Sb + (size_t)row * npp + p0) = o;
        }
    }
    // flags: lanes c and c + 16 cover the same dimensions; mask word c / 4, bits 8 (c % 4) ..
    uint32_t* mask = reinterpret_cast<uint32_t*>(summary + (size_t)b * sum_stride + mask_off) + hk * (D / 32);
#pragma unroll
    for (int mw = 0; mw < D / 32; ++mw) {
        const uint32_t m = __reduce_or_sync(0xffffffffu, (c >> 2) == mw ? nf << (8 * (c & 3)) : 0u);
        if (lane == 0 && m) atomicOr(mask + mw, m);
    }
}

template <typename T, int D>
__global__ void __launch_bounds__(kSumBuildNT) hsa_summary_build_rows_kernel(const uint8_t* K, long long kv_stride,
                                                                         int len_k, int C, int Lc, int nchunks,
                                                                         int npp, int TP, uint8_t* summary,
                                                                         long long sum_stride, long long mask_off) {
    constexpr int ES = (int)sizeof(T), RB = D * ES, W = RB / 4;  // 32-bit words per row
    constexpr uint32_t FLIP = ES == 2 ? 0x80008000u : 0x80000000u;
    extern __shared__ __align__(16) uint8_t smraw[];
    __shared__ uint32_t nfm[D / 32];        // dimensions with an extremum of -inf or NaN on this tile
    T* tile = reinterpret_cast<T*>(smraw);  // [2][D][TP]
    const int pt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
    if (threadIdx.x < D / 32) nfm[threadIdx.x] = 0u;
    __syncthreads();
    const int p0 = pt * TP;
    const uint8_t* Kh = K + (size_t)b * kv_stride + (size_t)hk * len_k * RB;
    for (int x = threadIdx.x; x < TP * W; x += kSumBuildNT) {
        const int p = x / W, wd = x % W, page = p0 + p;
        uint32_t m = 0u, n = 0u;
        if (page < nchunks) {
            const int r0 = page * C, r1 = min(r0 + C, Lc);
            const uint32_t v0 = *reinterpret_cast<const uint32_t*>(Kh + (size_t)r0 * RB + 4 * wd);
            m = v0;
            n = v0 ^ FLIP;
            for (int r = r0 + 1; r < r1; ++r) {
                const uint32_t v = *reinterpret_cast<const uint32_t*>(Kh + (size_t)r * RB + 4 * wd);
                m = Chunk<T>::wmax(m, v);
                n = Chunk<T>::wmax(n, v ^ FLIP);
            }
        }
        if (page < nchunks) {  // -inf or NaN: the scan clamps such a representative at -FLT_MAX
            uint32_t bits = 0u;
            if (ES == 2) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const uint32_t x = (m >> (16 * hf)) & 0xffffu, y = (n >> (16 * hf)) & 0xffffu;
                    if ((x & 0x7fffu) > 0x7f80u || x == 0xff80u || (y & 0x7fffu) > 0x7f80u || y == 0xff80u)
                        bits |= 1u << ((2 * wd + hf) & 31);
                }
            } else if ((m & 0x7fffffffu) > 0x7f800000u || m == 0xff800000u || (n & 0x7fffffffu) > 0x7f800000u ||
                       n == 0xff800000u) {
                bits = 1u << (wd & 31);
            }
            if (bits) atomicOr(&nfm[(ES == 2 ? 2 * wd : wd) >> 5], bits);
        }
        if (ES == 2) {
            tile[(0 * D + 2 * wd) * TP + p] = (T)(m & 0xffffu);
            tile[(0 * D + 2 * wd + 1) * TP + p] = (T)(m >> 16);
            tile[(1 * D + 2 * wd) * TP + p] = (T)(n & 0xffffu);
            tile[(1 * D + 2 * wd + 1) * TP + p] = (T)(n >> 16);
        } else {
            reinterpret_cast<uint32_t*>(tile)[(0 * D + wd) * TP + p] = m;
            reinterpret_cast<uint32_t*>(tile)[(1 * D + wd) * TP + p] = n;
        }
    }
    __syncthreads();
    if (threadIdx.x < D / 32 && nfm[threadIdx.x])
        atomicOr(reinterpret_cast<uint32_t*>(summary + (size_t)b * sum_stride + mask_off) + hk * (D / 32) + threadIdx.x,
                 nfm[threadIdx.x]);
    // rows of TP pages out, 16 bytes at a time (npp and TP are multiples of 8 pages)
    const int np = min(TP, npp - p0);
    const int vpr = np * ES / 16;
    uint8_t* Sb = summary + (size_t)b * sum_stride + (size_t)hk * 2 * D * npp * ES;
    for (int x = threadIdx.x; x < 2 * D * vpr; x += kSumBuildNT) {
        const int row = x / vpr, v = x % vpr;
        *reinterpret_cast<uint4*>(Sb + ((size_t)row * npp + p0) * ES + 16 * v) =
            *reinterpret_cast<const uint4*>(smraw + ((size_t)row * TP) * ES + 16 * v);
    }
}


// Phases 0 and 1 from the page summaries.  A tile is TP pages, a column of
// 32 PPL pages per warp: lane l scores PPL consecutive pages.  Every
// dimension has a fixed place ("position") in the order the sums take them:
// for the quad lanes j = 0, 2, 1, 3 of the stateless scan, their chunks
// j, j + 4, ..., and per chunk the even and then the odd dimensions.  The
// position table in shared memory holds, per position, the byte offset of the
// dimension's row in the tile and s q per head; the code walks the positions
// as straight-line code (no lists, no loop-carried state), and the entry read
// is the same on every lane of the warp (a broadcast).  Only the selected
// dimensions' rows are loaded, one bulk copy each, in position order, in two
// halves (the positions of quad lanes 0, 2 and of 1, 3), each on its own
// mbarrier with bounded waits: one half of the next tile is in flight while
// the other half of this one is scored; several CTAs per SM overlap as well.
// An unselected position has q = +0 and reads a zero row, so it adds
// fma(+0, +0, acc) = acc exactly (a chain that starts at +0 never reaches -0).
// Per page and head the sum is therefore hsa_scan_kernel's: per 16-byte chunk
// an even and an odd fused multiply-add chain over the selected dimensions,
// chunk value even + odd; the chunks j, j + 4, ... of quad lane j added
// pairwise as a balanced tree (kept here as a binary-counter stack), and the
// four lane totals as (l0 + l2) + (l1 + l3); then the IEEE division by the
// head's scale.  The representatives are clamped at -FLT_MAX, which is the
// scan's result on every page (the clamp only changes a representative that
// makes a page's sum non-finite, where the scan recomputes clamped).
constexpr int kSumScanNT = 128;
constexpr int kSumScanWarps = kSumScanNT / 32;
constexpr int kSumScanCtas = 3;  // CTAs per SM the tile size is chosen for

__host__ __device__ constexpr int sumscan_ppl(int maxg, int es, int d) { return maxg <= 4 && es * d <= 512 ? 4 : 2; }
template <int B>
struct VecBytes;
template <>
struct VecBytes<4> { using type = uint32_t; };
template <>
struct VecBytes<8> { using type = uint2; };
template <>
struct VecBytes<16> { using type = uint4; };

// dimension at position p, and position of dimension d (CD dimensions per 16-byte chunk, NSL chunks per quad
// lane): p = ((jj NSL + i) 2 + parity) CD / 2 + u for the dimension (j + 4 i) CD + 2 u + parity, jj the rank
// of quad lane j in the order 0, 2, 1, 3 (an involution: rank and lane map the same way)
template <int CD, int NSL>
__device__ __forceinline__ int sumscan_dim(int p) {
    const int u = p % (CD / 2), par = (p / (CD / 2)) & 1, i = (p / CD) % NSL, jj = p / (CD * NSL);
    const int j = jj == 1 ? 2 : jj == 2 ? 1 : jj;
    return (j + 4 * i) * CD + 2 * u + par;
}
template <int CD, int NSL>
__device__ __forceinline__ int sumscan_pos(int d) {
    const int c = d / CD, x = d % CD, j = c & 3, i = c >> 2;
    const int jj = j == 1 ? 2 : j == 2 ? 1 : j;
    return ((jj * NSL + i) * 2 + (x & 1)) * (CD / 2) + (x >> 1);
}

// One half of a tile for one warp (the positions of quad lanes 0, 2 for HALF 0, of 1, 3 for HALF 1): the
// lane's PPL pages over the half's positions; A = l0 + l2, B = l1 + l3.  CLAMP: representatives clamped at
// -FLT_MAX (needed only where a selected dimension has an extremum of -inf or NaN somewhere in the unit).
template <typename T, int D, int MAXG, bool CLAMP, int HALF>
__device__ __forceinline__ void sumscan_score_half(const float4* qtab, const uint8_t* col,
                                                   float2 (&A)[MAXG][sumscan_ppl(MAXG, (int)sizeof(T), D) / 2],
                                                   float2 (&B)[MAXG][sumscan_ppl(MAXG, (int)sizeof(T), D) / 2]) {
    constexpr int ES = (int)sizeof(T);
    constexpr int CD = 16 / ES, NCH = D / CD, NSL = NCH / 4, HCD = CD / 2;
    constexpr int TOP = NSL >= 16 ? 4 : NSL >= 8 ? 3 : NSL >= 4 ? 2 : 1;  // log2(NSL)
    constexpr int PPL = sumscan_ppl(MAXG, ES, D), PV = PPL / 2;
    constexpr int NQ = (MAXG + 1 + 3) / 4;  // float4s per position
    using RowV = typename VecBytes<ES * PPL>::type;
#pragma unroll
    for (int jh = 0; jh < 2; ++jh) {
        const int jj = 2 * HALF + jh;
        float2 stk[TOP][MAXG][PV];
        float2 cur[MAXG][PV];
#pragma unroll
        for (int i = 0; i < NSL; ++i) {
            float2 acc[2][MAXG][PV];
#pragma unroll
            for (int par = 0; par < 2; ++par) {
#pragma unroll
                for (int u = 0; u < HCD; ++u) {
                    const int p = ((jj * NSL + i) * 2 + par) * HCD + u;
                    float qh[4 * NQ];
#pragma unroll
                    for (int k = 0; k < NQ; ++k) {
                        const float4 e = qtab[p * NQ + k];
                        qh[4 * k] = e.x;
                        qh[4 * k + 1] = e.y;
                        qh[4 * k + 2] = e.z;
                        qh[4 * k + 3] = e.w;
                    }
                    const RowV X = *reinterpret_cast<const RowV*>(col + __float_as_int(qh[0]));
                    const uint32_t* wv = reinterpret_cast<const uint32_t*>(&X);
                    float2 P[PV];
#pragma unroll
                    for (int v = 0; v < PV; ++v) {
                        if (ES == 2)
                            P[v] = make_float2(__uint_as_float(wv[v] << 16), __uint_as_float(wv[v] & 0xffff0000u));
                        else
                            P[v] = make_float2(__uint_as_float(wv[2 * v]), __uint_as_float(wv[2 * v + 1]));
                        if (CLAMP) P[v] = make_float2(fmaxf(P[v].x, -FLT_MAX), fmaxf(P[v].y, -FLT_MAX));
                    }
#pragma unroll
                    for (int h = 0; h < MAXG; ++h)
#pragma unroll
                        for (int v = 0; v < PV; ++v)
                            acc[par][h][v] = __ffma2_rn(make_float2(qh[1 + h], qh[1 + h]), P[v],
                                                        u == 0 ? make_float2(0.0f, 0.0f) : acc[par][h][v]);
                }
            }
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
#pragma unroll
                for (int v = 0; v < PV; ++v) cur[h][v] = __fadd2_rn(acc[0][h][v], acc[1][h][v]);
            // balanced pairwise tree over the slots: merge while the low bits of i are ones
#pragma unroll
            for (int l = 0; l < TOP; ++l)
                if (((i + 1) & ((2 << l) - 1)) == 0)
#pragma unroll
                    for (int h = 0; h < MAXG; ++h)
#pragma unroll
                        for (int v = 0; v < PV; ++v) cur[h][v] = __fadd2_rn(stk[l][h][v], cur[h][v]);
            // then keep it at the level of its trailing ones (the last slot leaves the total in cur)
#pragma unroll
            for (int l = 0; l < TOP; ++l)
                if (((i + 1) & ((2 << l) - 1)) == (1 << l))
#pragma unroll
                    for (int h = 0; h < MAXG; ++h)
#pragma unroll
                        for (int v = 0; v < PV; ++v) stk[l][h][v] = cur[h][v];
        }
#pragma unroll
        for (int h = 0; h < MAXG; ++h)
#pragma unroll
            for (int v = 0; v < PV; ++v) {
                if (jj == 0) A[h][v] = cur[h][v];
                if (jj == 1) A[h][v] = __fadd2_rn(A[h][v], cur[h][v]);
                if (jj == 2) B[h][v] = cur[h][v];
                if (jj == 3) B[h][v] = __fadd2_rn(B[h][v], cur[h][v]);
            }
    }
}

template <typename T, int D, int MAXG>
__global__ void __launch_bounds__(kSumScanNT, kSumScanCtas) hsa_sumscan_kernel(const HsaArgs a) {
    asm volatile("griddepcontrol.launch_dependents;");  // the selection may be scheduled (it waits for this grid)
    constexpr int ES = (int)sizeof(T);
    constexpr int CD = 16 / ES, NCH = D / CD, NSL = NCH / 4;
    constexpr int TOP = NSL >= 16 ? 4 : NSL >= 8 ? 3 : NSL >= 4 ? 2 : 1;  // log2(NSL)
    static_assert((1 << TOP) == NSL, "slots per quad lane: a power of two from 2 to 16");
    constexpr int PPL = sumscan_ppl(MAXG, ES, D), PV = PPL / 2;  // pages per lane, page pairs per lane
    constexpr int COLP = 32 * PPL;                         // pages per column: a warp's share of a tile
    constexpr int NQ = (MAXG + 1 + 3) / 4;                 // float4s per position
    constexpr int NPW = D / 32;                            // 32-position words
    constexpr int DPT = (D + kSumScanNT - 1) / kSumScanNT;  // dimensions per thread in phase 0
    static_assert(NPW % 2 == 0 && NPW <= 32, "D from 64 to 1024");
    extern __shared__ __align__(128) uint8_t sbuf[];  // [nr][TP] extrema in position order, then a zero row
    __shared__ __align__(16) float4 qtab[D * NQ];     // per position: row offset, s q per head (sum |q| first)
    __shared__ uint32_t selw[NPW], negw[NPW];         // selected dimensions, sign-flipped dimensions
    __shared__ float cscale[MAXG];
    __shared__ uint64_t full[2];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, hc = blockIdx.y, b = blockIdx.z, hk = a.head_begin + hc;
    const int G = a.G;
    const int p_beg = split * a.pages_per_split;
    const int p_end = min(a.nchunks, p_beg + a.pages_per_split);
    if (p_beg >= p_end) return;  // uniform
    const T* Qg = reinterpret_cast<const T*>(a.Q + (size_t)b * a.q_stride + (size_t)hk * G * D * sizeof(T));
    float* wl = a.wlogits + ((size_t)b * a.head_count + hc) * (size_t)G * a.nch_pad;
    const uint8_t* summ = a.summary + (size_t)b * a.sum_stride;
    const uint32_t nfw = tid < NPW ? reinterpret_cast<const uint32_t*>(summ + a.sum_mask_off)[hk * NPW + tid] : 0u;
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    // ---- phase 0: group query statistics (rocket.cpp:197-250), as hsa_scan_kernel ----
    float* sabs = reinterpret_cast<float*>(qtab);  // sum over the heads of |q| per dimension (dead after the rank)
    float qv[DPT][MAXG];
    bool negd[DPT];
#pragma unroll
    for (int k = 0; k < DPT; ++k) {
        const int d = tid + k * kSumScanNT;
        float sa = 0.0f, sv = 0.0f;
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
            qv[k][h] = 0.0f;
            if (h < G && d < D) {
                const float q = to_f<T>(Qg[h * D + d]);
                qv[k][h] = q;
                sa = __fadd_rn(sa, fabsf(q));
                sv = __fadd_rn(sv, q);
            }
        }
        if (d < D) sabs[d] = sa;
        negd[k] = !(sv >= 0.0f);  // rocket.cpp:263: sign >= 0 takes the max
    }
    __syncthreads();
    // top r by (sum |q| desc, dimension asc)
#pragma unroll
    for (int k = 0; k < DPT; ++k) {
        const int d = tid + k * kSumScanNT;
        bool s = false;
        if (d < D) {
            int rank = 0;
            const float me = sabs[d];
#pragma unroll 8
            for (int e = 0; e < D; ++e) {
                const float o = sabs[e];
                rank += (o > me || (o == me && e < d)) ? 1 : 0;
            }
            s = a.r >= D || rank < a.r;
        }
        const uint32_t bs = __ballot_sync(0xffffffffu, s), bn = __ballot_sync(0xffffffffu, negd[k] && d < D);
        if (lane == 0 && warp + k * kSumScanWarps < NPW) {
            selw[warp + k * kSumScanWarps] = bs;
            negw[warp + k * kSumScanWarps] = bn;
        }
    }
    __syncthreads();  // masks ready; sabs dead
    // every warp: which positions are selected, and the running counts, so a selected position's row
    // (its entry) is known everywhere without another barrier
    uint32_t pb[NPW];
    int pbase[NPW + 1];
    pbase[0] = 0;
#pragma unroll
    for (int k = 0; k < NPW; ++k) {
        const int d = sumscan_dim<CD, NSL>(32 * k + lane);
        pb[k] = __ballot_sync(0xffffffffu, (selw[d >> 5] >> (d & 31)) & 1u);
        pbase[k + 1] = pbase[k] + __popc(pb[k]);
    }
    const int nr = pbase[NPW], eh = pbase[NPW / 2];  // selected rows; rows of the first half
    const int TP = a.stage_rows;
    const int rowb = TP * ES;
    const uint8_t* Sb = summ + (size_t)hk * 2 * D * a.npp * ES;
    const int ntile = (p_end - p_beg + TP - 1) / TP;
    auto issue = [&](int t, int half) {  // warp 0: the copies of one half of tile t
        const int tp0 = p_beg + t * TP;
        const int np = min(TP, a.npp - tp0);  // whole 8-page groups: bytes a multiple of 16
        if (lane == 0) mbar_arrive_expect_tx(&full[half], (uint32_t)((size_t)(half ? nr - eh : eh) * np * ES));
        __syncwarp();
#pragma unroll
        for (int k = half * (NPW / 2); k < (half + 1) * (NPW / 2); ++k) {
            if ((pb[k] >> lane) & 1u) {
                const int d = sumscan_dim<CD, NSL>(32 * k + lane);
                const int e = pbase[k] + __popc(pb[k] & ((1u << lane) - 1u));
                const int row = (int)((negw[d >> 5] >> (d & 31)) & 1u) * D + d;
                bulk_load(sbuf + (size_t)e * rowb, Sb + ((size_t)row * a.npp + tp0) * ES, (uint32_t)(np * ES),
                          &full[half]);
            }
        }
    };
    if (warp == 0) {
        issue(0, 0);
        issue(0, 1);
    }
    // the position table: this thread's dimensions
#pragma unroll
    for (int k = 0; k < DPT; ++k) {
        const int d = tid + k * kSumScanNT;
        if (d < D) {
            const int p = sumscan_pos<CD, NSL>(d), w = p >> 5, l = p & 31;
            uint32_t bw = 0;
            int base = 0;
#pragma unroll
            for (int x = 0; x < NPW; ++x)
                if (x == w) {
                    bw = pb[x];
                    base = pbase[x];
                }
            const bool s = (bw >> l) & 1u;
            const int off = (s ? base + __popc(bw & ((1u << l) - 1u)) : nr) * rowb;
            float e[4 * NQ];
            e[0] = __int_as_float(off);
#pragma unroll
            for (int h = 0; h < 4 * NQ - 1; ++h) {
                const float q = (s && h < MAXG) ? qv[k][h] : 0.0f;
                e[1 + h] = negd[k] ? -q : q;
            }
            if (!s) {
#pragma unroll
                for (int h = 1; h < 4 * NQ; ++h) e[h] = 0.0f;  // +0: adds exactly nothing
            }
#pragma unroll
            for (int x = 0; x < NQ; ++x) qtab[p * NQ + x] = make_float4(e[4 * x], e[4 * x + 1], e[4 * x + 2], e[4 * x + 3]);
        }
    }
    // per-head scales (rocket.cpp:240-250): sum over all dimensions and over the selected ones, ascending
    if (warp == (kSumScanWarps > 1 ? 1 : 0) && lane < G) {
        const T* qh = Qg + lane * D;
        float s_all = 0.0f, s_sel = 0.0f;
#pragma unroll
        for (int x = 0; x < NPW; ++x) {
            const uint32_t m = selw[x];
#pragma unroll
            for (int y = 0; y < 32; ++y) {
                const float q = fabsf(to_f<T>(qh[32 * x + y]));
                s_all = __fadd_rn(s_all, q);
                if ((m >> y) & 1u) s_sel = __fadd_rn(s_sel, q);
            }
        }
        const float sk = a.r >= D ? s_all : s_sel;
        cscale[lane] = __fsqrt_rn(__fmul_rn((float)D, __fdiv_rn(sk, __fadd_rn(s_all, 1e-9f))));
    }
    // the zero row the unselected positions read
    for (int x = tid; x < rowb / 16; x += kSumScanNT)
        *reinterpret_cast<uint4*>(sbuf + (size_t)nr * rowb + 16 * x) = make_uint4(0u, 0u, 0u, 0u);
    // a selected dimension with an extremum of -inf or NaN somewhere in the unit: clamp
    const bool need_clamp = __syncthreads_or(tid < NPW && (nfw & selw[tid]) != 0u) != 0;

    // ---- phase 1: page logits from the summaries ----
    const int wp0 = warp * COLP, lp = wp0 + lane * PPL;  // the warp's and the lane's first page in a tile
    float rscale[MAXG];
#pragma unroll
    for (int h = 0; h < MAXG; ++h) rscale[h] = h < G ? cscale[h] : 1.0f;
    for (int t = 0; t < ntile; ++t) {
        const int tp0 = p_beg + t * TP;
        const bool active = wp0 < TP && tp0 + wp0 < p_end;  // warp-uniform: warps past the tile or the unit skip
        const uint8_t* col = sbuf + (size_t)lp * ES;
        float2 A[MAXG][PV], B[MAXG][PV];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const bool ok = mbar_wait_bounded(&full[half], (uint32_t)(t & 1), a.err);
            if (!__syncthreads_and(ok)) {  // timed out: the copies in flight land before the exit
                if (tid == 0) {
                    mbar_wait_bounded(&full[half], (uint32_t)(t & 1), a.err);
                    if (half == 0) mbar_wait_bounded(&full[1], (uint32_t)(t & 1), a.err);
                    if (half == 1 && t + 1 < ntile) mbar_wait_bounded(&full[0], (uint32_t)((t + 1) & 1), a.err);
                }
                return;
            }
            if (active) {
                if (half == 0) {
                    if (need_clamp)
                        sumscan_score_half<T, D, MAXG, true, 0>(qtab, col, A, B);
                    else
                        sumscan_score_half<T, D, MAXG, false, 0>(qtab, col, A, B);
                } else {
                    if (need_clamp)
                        sumscan_score_half<T, D, MAXG, true, 1>(qtab, col, A, B);
                    else
                        sumscan_score_half<T, D, MAXG, false, 1>(qtab, col, A, B);
                }
            }
            __syncthreads();  // the half's rows are free for the next tile
            if (warp == 0 && t + 1 < ntile) issue(t + 1, half);
        }
        if (active) {
            const int pa = tp0 + lp;
#pragma unroll
            for (int h = 0; h < MAXG; ++h) {
                if (h >= G) break;  // uniform
                float o[PPL];
#pragma unroll
                for (int v = 0; v < PV; ++v) {
                    const float2 s = __fadd2_rn(A[h][v], B[h][v]);
                    o[2 * v] = __fdiv_rn(s.x, rscale[h]);
                    o[2 * v + 1] = __fdiv_rn(s.y, rscale[h]);
                }
                float* dst = wl + (size_t)h * a.nch_pad + pa;
                if (pa + PPL <= p_end) {
                    if (PPL == 4)
                        *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
                    else
                        *reinterpret_cast<float2*>(dst) = make_float2(o[0], o[1]);
                } else {
#pragma unroll
                    for (int pg = 0; pg < PPL; ++pg)
                        if (pa + pg < p_end) dst[pg] = o[pg];
                }
            }
        }
    }
}

int num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        n = 148;
    return n;
}

template <typename T, int D, int MAXG>
int launch_t(HsaArgs a, int batch, cudaStream_t st) {
    if (a.nchunks > 0 && a.summary) {
        // page logits from the summaries.  Tile: whole columns of 32 PPL pages (a warp each), as many as
        // kSumScanCtas CTAs per SM hold for the r selected rows and the zero row
        constexpr int PPL = sumscan_ppl(MAXG, (int)sizeof(T), D), COLP = 32 * PPL;
        auto fs = hsa_sumscan_kernel<T, D, MAXG>;
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, fs) != cudaSuccess) return RKV_ERR_CUDA;
        int dev = 0, sm_smem = 0, reserved = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess)
            return RKV_ERR_CUDA;
        const long long per_cta = (long long)sm_smem / kSumScanCtas - reserved - (long long)fa.sharedSizeBytes;
        const int nr = a.r < D ? a.r : D;
        const size_t run_b = (size_t)(nr + 1) * sizeof(T);  // bytes per tile page
        int tp = per_cta > 0 ? (int)((size_t)per_cta / run_b) / COLP * COLP : 0;
        if (tp > kSumScanWarps * COLP) tp = kSumScanWarps * COLP;
        if (tp < COLP) tp = COLP;
        a.stage_rows = tp;
        // enough CTAs to cover the GPU
        const long long units = (long long)batch * a.head_count;
        const long long want = (long long)kSumScanCtas * num_sms();
        int splits = units >= want ? 1 : (int)((want + units - 1) / units);
        const int max_splits = (a.nchunks + tp - 1) / tp;
        if (splits > max_splits) splits = max_splits;
        if (splits < 1) splits = 1;
        a.pages_per_split = ((a.nchunks + splits - 1) / splits + tp - 1) / tp * tp;  // whole tiles
        a.splits = (a.nchunks + a.pages_per_split - 1) / a.pages_per_split;
        const size_t smem = run_b * tp;
        if (cudaFuncSetAttribute(fs, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return RKV_ERR_CUDA;
        if (cudaFuncSetAttribute(fs, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
            return RKV_ERR_CUDA;
        fs<<<dim3(a.splits, a.head_count, batch), kSumScanNT, smem, st>>>(a);
        if (cudaGetLastError() != cudaSuccess) return RKV_ERR_CUDA;
    } else if (a.nchunks > 0) {
        auto fs = hsa_scan_kernel<T, D, MAXG>;
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, fs) != cudaSuccess) return RKV_ERR_CUDA;
        const int sr_max = kStageBytes / (int)(D * sizeof(T));
        if (a.C <= sr_max) {
            // pages per stage: a power of two times 8 (a warp's eight quads), at most 64
            a.carry_mode = 0;
            int pps = sr_max / a.C;
            if (pps >= 8) {
                int p2 = 1;
                while (p2 * 2 <= (pps < 64 ? pps : 64) / 8) p2 *= 2;
                pps = 8 * p2;
            }
            a.pps = pps;
            a.stage_rows = pps * a.C;
            a.wg = (pps + 7) / 8;
        } else {
            a.carry_mode = 1;
            a.stage_rows = sr_max;
            a.pps = 0;
            a.wg = kScanConsumers / 32;
        }
        // ring depth for two CTAs per SM (113 KB of shared memory each, static part included)
        const size_t extra = 16 * kMaxScanStages + (a.carry_mode ? (size_t)2 * (D + 4) * 4 : 0);
        const size_t budget = 113 * 1024, fixed = fa.sharedSizeBytes + extra;
        int ns = fixed < budget ? (int)((budget - fixed) / kStageBytes) : 0;
        if (ns > 6) ns = 6;
        if (ns < 3) ns = 3;
        a.nstage = ns;
        a.ngrp = a.carry_mode ? 1 : (kScanConsumers / 32) / a.wg;
        if (a.ngrp > ns - 1) a.ngrp = ns - 1;
        // Group g takes stages g, g + ngrp, ... in ring slot s % ns.  With ngrp dividing ns every
        // slot belongs to one group, which uses it in order; otherwise a group could wait on a slot
        // two phases ahead of its last completed phase, which a parity wait cannot tell from the
        // previous phase (it would pass before the copy lands).
        while (ns % a.ngrp != 0) --a.ngrp;
        // enough scan CTAs to cover the GPU; every split keeps at least 4 stages of pages
        const long long units = (long long)batch * a.head_count;
        const long long want = 2LL * num_sms();
        int splits = units >= want ? 1 : (int)((want + units - 1) / units);
        const int min_pages = a.carry_mode ? 1 : 4 * a.pps;
        const int max_splits = (a.nchunks + min_pages - 1) / min_pages;
        if (splits > max_splits) splits = max_splits;
        if (splits < 1) splits = 1;
        a.pages_per_split = (a.nchunks + splits - 1) / splits;
        a.splits = (a.nchunks + a.pages_per_split - 1) / a.pages_per_split;
        const size_t smem_s = (size_t)ns * kStageBytes + extra;
        if (cudaFuncSetAttribute(fs, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_s) != cudaSuccess)
            return RKV_ERR_CUDA;
        fs<<<dim3(a.splits, a.head_count, batch), kScanThreads, smem_s, st>>>(a);
        if (cudaGetLastError() != cudaSuccess) return RKV_ERR_CUDA;
    }
    // phase 2: one CTA per unit; the logits are staged when they fit
    const int units = batch * a.head_count;
    const size_t lg = (size_t)a.G * a.nch_pad * sizeof(float);
    const bool sel_smem = a.nchunks > 0 && lg <= (size_t)kSelSmemMax;
    const size_t smem_sel = sel_smem ? 128 + lg : 0;
    auto fsel = sel_smem ? hsa_select_kernel<MAXG, true> : hsa_select_kernel<MAXG, false>;
    if (cudaFuncSetAttribute(fsel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_sel) != cudaSuccess)
        return RKV_ERR_CUDA;
    // the selection and the attention are programmatic dependent launches: each is scheduled while its
    // predecessor's last wave runs and waits in the kernel for that grid's results
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(units);
    lc.blockDim = dim3(kSelThreads);
    lc.dynamicSmemBytes = smem_sel;
    lc.stream = st;
    lc.attrs = pdl;
    lc.numAttrs = 1;
    if (cudaLaunchKernelEx(&lc, fsel, a) != cudaSuccess) {
        (void)cudaGetLastError();
        return RKV_ERR_CUDA;
    }
    // phase 3 shared memory: [merge buffer][indices][scores]
    constexpr int NGC = kNT / (int)(D * sizeof(T) / 16);
    const size_t merge = (size_t)NGC * MAXG * D * sizeof(float);
    const size_t lists = (size_t)a.score_stride * 4 * (1 + a.G);
    const bool smem_path = lists <= (size_t)kTailSmemMax;
    a.tail_r0_bytes = (int)align_up(merge, 16);
    const size_t smem_t = (size_t)a.tail_r0_bytes + (smem_path ? lists : 0);
    auto ft = smem_path ? hsa_attn_kernel<T, D, MAXG, true> : hsa_attn_kernel<T, D, MAXG, false>;
    if (cudaFuncSetAttribute(ft, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_t) != cudaSuccess)
        return RKV_ERR_CUDA;
    lc.gridDim = dim3(a.head_count, batch);
    lc.blockDim = dim3(kNT);
    lc.dynamicSmemBytes = smem_t;
    if (cudaLaunchKernelEx(&lc, ft, a) != cudaSuccess) {
        (void)cudaGetLastError();
        return RKV_ERR_CUDA;
    }
    return RKV_OK;
}

template <typename T, int D>
int launch_d(const HsaArgs& a, int batch, cudaStream_t st) {
    switch (a.G) {
        case 1: return launch_t<T, D, 1>(a, batch, st);
        case 2: return launch_t<T, D, 2>(a, batch, st);
        case 3: return launch_t<T, D, 3>(a, batch, st);
        case 4: return launch_t<T, D, 4>(a, batch, st);
        default: return launch_t<T, D, 8>(a, batch, st);
    }
}

template <typename T>
int launch_dt(const HsaArgs& a, int batch, cudaStream_t st) {
    switch (a.D) {
        case 64: return launch_d<T, 64>(a, batch, st);
        case 128: return launch_d<T, 128>(a, batch, st);
        case 256: return launch_d<T, 256>(a, batch, st);
        default: return RKV_ERR_UNSUPPORTED;
    }
}

}  // namespace

HsaShape hsa_shape(const rkv_config& c, int len_k, int recent_window, int batch, int head_count) {
    HsaShape s{};
    s.G = c.num_heads / c.num_heads_kv;
    if (s.G < 1) s.G = 1;
    // rocket.cpp:177-183 (fallbacks used when chunk_size / r_dim are 0)
    if (c.chunk_size > 0) {
        s.C = c.chunk_size;
    } else {
        const int a = (int)floorf(c.compression_ratio), b = (int)ceilf(sqrtf(c.compression_ratio));
        s.C = a < b ? a : b;
        if (s.C < 1) s.C = 1;
    }
    if (c.r_dim > 0) {
        s.r = c.r_dim;
    } else {
        int r = (int)roundf((float)c.dim_head * (float)s.C / c.compression_ratio);
        if (r < 1) r = 1;
        s.r = r < c.dim_head ? r : c.dim_head;
    }
    if (s.r > c.dim_head) s.r = c.dim_head;
    int w = recent_window < 0 ? 0 : recent_window;
    if (len_k < 0) len_k = 0;
    s.w = w < len_k ? w : len_k;
    s.Lc = len_k - s.w;
    s.final_k = c.topk_decode < s.Lc ? c.topk_decode : s.Lc;
    s.nchunks = (s.final_k > 0 && s.final_k < s.Lc) ? (s.Lc + s.C - 1) / s.C : 0;
    s.sel_cap = (s.final_k > 0 ? s.final_k : 0) + s.w;
    size_t off = kWorkspaceHeader;
    s.nch_pad = (s.nchunks + 3) / 4 * 4;  // 16-byte rows, so a unit's logits are one aligned block
    s.off_logits = off;
    off = align_up(off + (size_t)batch * head_count * s.G * (size_t)s.nch_pad * sizeof(float), kWorkspaceAlign);
    s.off_sel = off;
    off = align_up(off + (size_t)batch * head_count * (size_t)(s.sel_cap > 0 ? s.sel_cap : 1) * sizeof(int),
                   kWorkspaceAlign);
    s.off_scores = off;
    off = align_up(off + (size_t)batch * head_count * s.G * (size_t)(s.sel_cap > 0 ? s.sel_cap : 1) * sizeof(float),
                   kWorkspaceAlign);
    s.ws_bytes = off;
    return s;
}

HsaSummaryShape hsa_summary_shape(const rkv_config& c, int dtype, int len_k, int recent_window) {
    const HsaShape h = hsa_shape(c, len_k, recent_window, 1, c.num_heads_kv);
    HsaSummaryShape s{};
    s.C = h.C;
    s.Lc = h.Lc;
    s.nchunks = h.Lc > 0 ? (h.Lc + h.C - 1) / h.C : 0;  // every page, whether or not a call scores them
    s.npp = (s.nchunks + 7) / 8 * 8;
    s.mask_off = (long long)c.num_heads_kv * 2 * c.dim_head * s.npp * (dtype == RKV_F32 ? 4 : 2);
    s.item_bytes = s.mask_off + ((long long)c.num_heads_kv * (c.dim_head / 8) + 15) / 16 * 16;
    return s;
}

template <typename T, int D>
static int build_t(const uint8_t* K, int HK, int len_k, long long kv_stride, const HsaSummaryShape& s,
                   uint8_t* summary, int batch, cudaStream_t st) {
    hsa_summary_mask_clear<<<batch, 128, 0, st>>>(summary, s.item_bytes, s.mask_off, HK * (D / 32));
    constexpr int pages_per_cta = (kSumBuildNT / 32) * kBuildPagesPerWarp;
    dim3 grid((s.npp + pages_per_cta - 1) / pages_per_cta, HK, batch);
    if (sizeof(T) == 2 && D == 128 && s.C <= 2) {  // bf16 pages of one or two rows: a page per load instruction
        constexpr int pages_per_cta = (kSumBuildNT / 32) * kTilePages;
        const size_t smem = (size_t)(kSumBuildNT / 32) * (kTilePages / 2) * 2 * D * sizeof(uint32_t);
        auto f = hsa_summary_build_tile_kernel;
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return RKV_ERR_CUDA;
        f<<<dim3((s.npp + pages_per_cta - 1) / pages_per_cta, HK, batch), kSumBuildNT, smem, st>>>(
            K, kv_stride, len_k, s.C, s.Lc, s.nchunks, s.npp, summary, s.item_bytes, s.mask_off);
    } else if (s.C >= 4) {  // long pages: coalesced row reads, extrema transposed through shared memory
        const int rowb = D * (int)sizeof(T);
        int TP = 16384 / rowb;
        if (TP > 64) TP = 64;
        if (TP < 8) TP = 8;
        const size_t smem = (size_t)2 * D * TP * sizeof(T);
        auto f = hsa_summary_build_rows_kernel<T, D>;
        if (smem > 48 * 1024 && cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return RKV_ERR_CUDA;
        f<<<dim3((s.npp + TP - 1) / TP, HK, batch), kSumBuildNT, smem, st>>>(K, kv_stride, len_k, s.C, s.Lc, s.nchunks,
                                                                             s.npp, TP, summary, s.item_bytes, s.mask_off);
    } else {
        hsa_summary_build_kernel<T, D><<<grid, kSumBuildNT, 0, st>>>(K, kv_stride, len_k, s.C, s.Lc, s.nchunks, s.npp,
                                                                     summary, s.item_bytes, s.mask_off);
    }
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

int launch_hsa_summary_build(const uint8_t* K, int dtype, int D, int HK, int len_k, long long kv_stride,
                             const HsaSummaryShape& s, uint8_t* summary, int batch, cudaStream_t st) {
    if (batch <= 0 || s.nchunks <= 0) return RKV_OK;
    const bool f32 = dtype == RKV_F32;
    switch (D) {
        case 64: return f32 ? build_t<float, 64>(K, HK, len_k, kv_stride, s, summary, batch, st)
                            : build_t<uint16_t, 64>(K, HK, len_k, kv_stride, s, summary, batch, st);
        case 128: return f32 ? build_t<float, 128>(K, HK, len_k, kv_stride, s, summary, batch, st)
                             : build_t<uint16_t, 128>(K, HK, len_k, kv_stride, s, summary, batch, st);
        case 256: return f32 ? build_t<float, 256>(K, HK, len_k, kv_stride, s, summary, batch, st)
                             : build_t<uint16_t, 256>(K, HK, len_k, kv_stride, s, summary, batch, st);
        default: return RKV_ERR_UNSUPPORTED;
    }
}

int hsa_check_supported(const rkv_config& c, int dtype) {
    if (dtype != RKV_F32 && dtype != RKV_BF16) return RKV_ERR_UNSUPPORTED;
    if (c.dim_head != 64 && c.dim_head != 128 && c.dim_head != 256) return RKV_ERR_UNSUPPORTED;
    if (c.num_heads / c.num_heads_kv > 8) return RKV_ERR_UNSUPPORTED;
    return RKV_OK;
}

int launch_hsa(HsaArgs a, int dtype, int batch, cudaStream_t st) {
    if (batch <= 0 || a.head_count <= 0) return RKV_OK;
    return dtype == RKV_F32 ? launch_dt<float>(a, batch, st) : launch_dt<uint16_t>(a, batch, st);
}

}  // namespace rkv
