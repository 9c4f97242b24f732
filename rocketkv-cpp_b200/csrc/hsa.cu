// hsa.cu -- stage-2 hybrid sparse decode on sm_100a (rocket.cpp:171-382).
//
// One CTA per (item, KV head) unit, three phases:
//   0. query statistics of the GQA group: sum_h |q|, sign of sum_h q, the
//      top-r dimensions (ties to the lower dimension, listed ascending) and
//      the per-head variance scale (rocket.cpp:197-250);
//   1. the K rows of the scored range stream through a 3-stage ring of 16 KB
//      bulk copies (cp.async.bulk, full/empty mbarriers, no multicast; thread
//      0 refills a slot once every warp has released it).  Each page (chunk
//      of C rows) gets its sign-chosen max/min on the r dimensions and the
//      approximate logit per head (rocket.cpp:252-289): eight lanes per page,
//      lane j runs a fused multiply-add chain over the selected-dimension list
//      entries j, j+8, ..., and a fixed butterfly adds the eight.  The logits
//      go to the workspace;
//   2. per-head softmax over pages with the deterministic exp and a fixed
//      256-way summation order, the group sum, and a weighted radix select of
//      the top final_k tokens by (score desc, index asc) with stable
//      compaction to ascending order (rocket.cpp:291-340), then the recent
//      window.  Phases 0-2 repeat the oracle's float operations one for one,
//      so the selected indices match it bit for bit;
//   3. exact attention over the selected rows: the K/V rows are gathered into
//      the same ring by per-row bulk copies, a lane group per token reads
//      them, online softmax per head, and a cross-group merge in shared
//      memory (rocket.cpp:342-378).
#include "hsa.cuh"

#include <float.h>

namespace rkv {
namespace {

constexpr int kNT = 256;
constexpr int kStageBytes = 16384;
constexpr int kNStage = 3;

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

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// q values of one selected dimension for the group's heads, then the
// dimension index with the sign of sum_h q in bit 31 (set = negative).
template <int MAXG>
struct QPack {
    static constexpr int kWords = (MAXG + 1 + 3) / 4 * 4;
};

template <typename T, int D, int MAXG>
__global__ void __launch_bounds__(kNT, (MAXG <= 3 ? 3 : 2)) hsa_kernel(const HsaArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t* ring = sm;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + a.off_bar);
    uint64_t* empty = full + kNStage;
    float* pst = reinterpret_cast<float*>(sm + a.off_pst);  // carry mode only: [2][D + 1]

    constexpr int QW = QPack<MAXG>::kWords;
    __shared__ float qf[MAXG * D];
    __shared__ __align__(16) float qpk[D * QW];
    __shared__ float sabs[D], qsum[D];
    __shared__ int Rl[D], flag[D];
    __shared__ float part[MAXG][kNT];
    __shared__ float sumall[MAXG], cscale[MAXG], hmax[MAXG], hinv[MAXG];
    __shared__ int hist[256], scan_tmp[33];
    __shared__ int s_nr, s_abort, s_kk;
    __shared__ uint32_t s_prefix;

    constexpr size_t RB = (size_t)D * sizeof(T);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hc = blockIdx.x, b = blockIdx.y, hk = a.head_begin + hc;
    const int G = a.G;
    const uint8_t* Qg = a.Q + (size_t)b * a.q_stride + (size_t)hk * G * D * sizeof(T);
    const uint8_t* Ku = a.K + (size_t)b * a.kv_stride + (size_t)hk * a.len_k * RB;
    const uint8_t* Vu = a.V + (size_t)b * a.kv_stride + (size_t)hk * a.len_k * RB;
    int* sel = a.sel + ((size_t)b * a.head_count + hc) * a.sel_stride;
    const int nch = a.nchunks;
    float* wl = a.wlogits + ((size_t)b * a.head_count + hc) * (size_t)G * nch;

    uint64_t* full3 = empty + kNStage;   // phase-3 ring barriers
    uint64_t* empty3 = full3 + kNStage;
    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kNStage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNT / 32);
            mbar_init(&full3[s], 1);
            mbar_init(&empty3[s], kNT / 32);
        }
        fence_mbar_init();
    }
    for (int e = tid; e < G * D; e += kNT) qf[e] = to_f<T>(reinterpret_cast<const T*>(Qg)[e]);
    __syncthreads();

    int nfirst;  // selected tokens from the scored range
    if (nch > 0) {
        // ---- phase 0: group query statistics (rocket.cpp:197-250) ----------
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
        if (tid < G) {
            float s = 0.0f;
            for (int d = 0; d < D; ++d) s = __fadd_rn(s, fabsf(qf[tid * D + d]));
            sumall[tid] = s;
        }
        __syncthreads();
        if (tid < D) {
            int rank = 0;
            const float me = sabs[tid];
            for (int e = 0; e < D; ++e) {
                const float o = sabs[e];
                rank += (o > me || (o == me && e < tid)) ? 1 : 0;
            }
            flag[tid] = (a.r >= D || rank < a.r) ? 1 : 0;
        }
        __syncthreads();
        if (tid == 0) {
            int nr = 0;
            for (int d = 0; d < D; ++d)
                if (flag[d]) Rl[nr++] = d;
            s_nr = nr;
        }
        __syncthreads();
        const int nr = s_nr;
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
        for (int i = tid; i < nr; i += kNT) {
            const int d = Rl[i];
#pragma unroll
            for (int h = 0; h < MAXG; ++h) qpk[i * QW + h] = h < G ? qf[h * D + d] : 0.0f;
            qpk[i * QW + QW - 1] = __int_as_float(d | (qsum[d] >= 0.0f ? 0 : (int)0x80000000));
        }

        // ---- phase 1: stream K, page representatives, approximate logits --
        const int SR = a.stage_rows;
        const int nst = (a.Lc + SR - 1) / SR;
        __syncthreads();  // qpk, cscale ready
        if (tid == 0) {
            for (int s = 0; s < kNStage && s < nst; ++s) {
                const int t0 = s * SR;
                const uint32_t bytes = (uint32_t)(min(SR, a.Lc - t0) * RB);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_load(ring + (size_t)s * kStageBytes, Ku + (size_t)t0 * RB, bytes, &full[s]);
            }
        }
        float carry = -INFINITY;  // carry mode: running signed max of dimension list entry `tid`
        bool timed_out = false;
        for (int s = 0; s < nst; ++s) {
            const int slot = s % kNStage;
            const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)((s / kNStage) & 1), a.err);
            // A failed wait is uniform across the block (nobody passes an incomplete
            // phase); carry mode also decides it with a block vote, as its loop syncs.
            if (a.carry_mode ? __syncthreads_or(!ok) : !ok) {
                timed_out = true;
                break;
            }
            const int t0 = s * SR, nrows = min(SR, a.Lc - t0);
            const T* st = reinterpret_cast<const T*>(ring + (size_t)slot * kStageBytes);
            const int c_lo = t0 / a.C;
            const int c_hi = (t0 + nrows == a.Lc) ? nch : (t0 + nrows) / a.C;
            const int ntask = (c_hi - c_lo) * 8;
            if (a.carry_mode) {
                if (tid < nr) {
                    const int w = __float_as_int(qpk[tid * QW + QW - 1]);
                    const int d = w & 0x7fffffff;
                    const bool neg = w < 0;
                    for (int rr = 0; rr < nrows; ++rr) {
                        const int t = t0 + rr;
                        const float x = to_f<T>(st[rr * D + d]);
                        carry = fmaxf(carry, neg ? -x : x);
                        if ((t + 1) % a.C == 0 || t == a.Lc - 1) {
                            pst[(t / a.C - c_lo) * (D + 1) + tid] = neg ? -carry : carry;
                            carry = -INFINITY;
                        }
                    }
                }
                __syncthreads();
            }
            // tasks (page, slice): slice s8 sums list entries i = s8, s8+8, ...
            for (int base = warp * 32; base < ntask; base += kNT) {
                const int task = base + lane;
                const int cl = task >> 3, s8 = task & 7;
                float acc[MAXG];
#pragma unroll
                for (int h = 0; h < MAXG; ++h) acc[h] = 0.0f;
                if (task < ntask) {
                    const int r0 = cl * a.C, r1 = min(r0 + a.C, nrows);
                    for (int i = s8; i < nr; i += 8) {
                        const float* qp = qpk + i * QW;
                        float P;
                        if (!a.carry_mode) {
                            const int w = __float_as_int(qp[QW - 1]);
                            const int d = w & 0x7fffffff;
                            const bool neg = w < 0;
                            float m = -INFINITY;
                            for (int rr = r0; rr < r1; ++rr) {
                                const float x = to_f<T>(st[rr * D + d]);
                                m = fmaxf(m, neg ? -x : x);
                            }
                            P = neg ? -m : m;
                        } else {
                            P = pst[cl * (D + 1) + i];
                        }
#pragma unroll
                        for (int h = 0; h < MAXG; ++h) acc[h] = __fmaf_rn(qp[h], P, acc[h]);
                    }
                }
#pragma unroll
                for (int h = 0; h < MAXG; ++h) {
                    acc[h] = __fadd_rn(acc[h], __shfl_xor_sync(0xffffffffu, acc[h], 4));
                    acc[h] = __fadd_rn(acc[h], __shfl_xor_sync(0xffffffffu, acc[h], 2));
                    acc[h] = __fadd_rn(acc[h], __shfl_xor_sync(0xffffffffu, acc[h], 1));
                }
                if (task < ntask && s8 == 0) {
#pragma unroll
                    for (int h = 0; h < MAXG; ++h)
                        if (h < G) wl[(size_t)h * nch + c_lo + cl] = __fdiv_rn(acc[h], cscale[h]);
                }
            }
            if (a.carry_mode) __syncthreads();  // pst reuse
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            // producer: refill the slot of the previous stage once every warp released it
            if (tid == 0 && s >= 1 && s - 1 + kNStage < nst) {
                const int sp = s - 1, ps = sp % kNStage;
                if (mbar_wait_bounded(&empty[ps], (uint32_t)((sp / kNStage) & 1), a.err)) {
                    fence_proxy_async();
                    const int s2 = sp + kNStage, t2 = s2 * SR;
                    const uint32_t bytes = (uint32_t)(min(SR, a.Lc - t2) * RB);
                    mbar_arrive_expect_tx(&full[ps], bytes);
                    bulk_load(ring + (size_t)ps * kStageBytes, Ku + (size_t)t2 * RB, bytes, &full[ps]);
                } else {
                    // no refill: the consumers' wait on this slot then runs out as well
                    timed_out = true;
                }
            }
        }
        if (timed_out) s_abort = 1;
        __syncthreads();
        if (s_abort) return;

        // ---- phase 2: page softmax per head, group sum, weighted top-k ----
        float m[MAXG];
#pragma unroll
        for (int h = 0; h < MAXG; ++h) m[h] = -INFINITY;
        for (int c = tid; c < nch; c += kNT)
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
                if (h < G) m[h] = fmaxf(m[h], wl[(size_t)h * nch + c]);
#pragma unroll
        for (int h = 0; h < MAXG; ++h) {
            float v = m[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) part[h][warp] = v;
        }
        __syncthreads();
        if (tid < G) {
            float v = -INFINITY;
            for (int wi = 0; wi < kNT / 32; ++wi) v = fmaxf(v, part[tid][wi]);
            hmax[tid] = v;
        }
        __syncthreads();
        float ps[MAXG];
#pragma unroll
        for (int h = 0; h < MAXG; ++h) ps[h] = 0.0f;
        for (int c = tid; c < nch; c += kNT)
#pragma unroll
            for (int h = 0; h < MAXG; ++h)
                if (h < G) {
                    const float e = det_expf(__fsub_rn(wl[(size_t)h * nch + c], hmax[h]));
                    wl[(size_t)h * nch + c] = e;
                    ps[h] = __fadd_rn(ps[h], e);
                }
#pragma unroll
        for (int h = 0; h < MAXG; ++h) part[h][tid] = ps[h];
        __syncthreads();
        // halving tree part[j] += part[j + s], s = 128 ... 1: the first three
        // steps cross warps (shared memory), the last five run in warp 0.
        for (int s = kNT / 2; s >= 32; s >>= 1) {
            if (tid < s)
#pragma unroll
                for (int h = 0; h < MAXG; ++h) part[h][tid] = __fadd_rn(part[h][tid], part[h][tid + s]);
            __syncthreads();
        }
        if (warp == 0) {
#pragma unroll
            for (int h = 0; h < MAXG; ++h) {
                float v = part[h][lane];
#pragma unroll
                for (int s = 16; s > 0; s >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, s));
                if (lane == 0 && h < G) hinv[h] = __fdiv_rn(1.0f, __fadd_rn(v, 1e-9f));
            }
        }
        __syncthreads();
        uint32_t* keys = reinterpret_cast<uint32_t*>(wl);
        for (int c = tid; c < nch; c += kNT) {
            float g = 0.0f;
            for (int h = 0; h < G; ++h) g = __fadd_rn(g, __fmul_rn(wl[(size_t)h * nch + c], hinv[h]));
            keys[c] = float_key(g);
        }
        if (tid == 0) {
            s_prefix = 0u;
            s_kk = a.final_k;
        }
        __syncthreads();
        uint32_t mask = 0u;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = tid; i < 256; i += kNT) hist[i] = 0;
            __syncthreads();
            const uint32_t prefix = s_prefix;
            for (int c = tid; c < nch; c += kNT) {
                const uint32_t k = keys[c];
                if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], min(a.C, a.Lc - c * a.C));
            }
            __syncthreads();
            // token counts from the top digit down; the digit where the running count reaches kk
            const int kk = s_kk;
            const int v = hist[255 - tid];
            int tot;
            const int before = block_exclusive_scan(v, scan_tmp, &tot);
            if (before < kk && before + v >= kk) {
                s_kk = kk - before;
                s_prefix = prefix | ((uint32_t)(255 - tid) << shift);
            }
            mask |= 255u << shift;
            __syncthreads();
        }
        const uint32_t thr = s_prefix;
        const int need = s_kk;
        // Stable compaction: thread tid owns the contiguous page range
        // [c_beg, c_end); two block scans give its threshold-tie rank and its
        // output position, so the selection lands in ascending token order.
        const int per = (nch + kNT - 1) / kNT;
        const int c_beg = min(nch, tid * per), c_end = min(nch, c_beg + per);
        int eqw = 0;
        for (int c = c_beg; c < c_end; ++c)
            if (keys[c] == thr) eqw += min(a.C, a.Lc - c * a.C);
        int tot;
        int eq_rank = block_exclusive_scan(eqw, scan_tmp, &tot);
        int takes = 0;
        for (int c = c_beg, eb = eq_rank; c < c_end; ++c) {
            const uint32_t k = keys[c];
            const int wt = min(a.C, a.Lc - c * a.C);
            if (k > thr) takes += wt;
            else if (k == thr) { takes += max(0, min(wt, need - eb)); eb += wt; }
        }
        int pos = block_exclusive_scan(takes, scan_tmp, &tot);
        for (int c = c_beg; c < c_end; ++c) {
            const uint32_t k = keys[c];
            const int wt = min(a.C, a.Lc - c * a.C);
            int take = 0;
            if (k > thr) take = wt;
            else if (k == thr) { take = max(0, min(wt, need - eq_rank)); eq_rank += wt; }
            for (int j = 0; j < take; ++j) sel[pos + j] = c * a.C + j;
            pos += take;
        }
        nfirst = a.final_k;
    } else {
        // No scoring needed: every eligible token (final_k >= Lc) or none.
        nfirst = a.final_k > 0 ? a.Lc : 0;
        for (int t = tid; t < nfirst; t += kNT) sel[t] = t;
    }
    for (int t = tid; t < a.w; t += kNT) sel[nfirst + t] = a.Lc + t;
    const int n = nfirst + a.w;
    if (tid == 0 && a.n_sel) a.n_sel[(size_t)b * a.head_count + hc] = n;
    __syncthreads();

    // ---- phase 3: exact attention over the selected rows -------------------
    // The selected K and V rows are gathered into the ring by bulk copies
    // (one per row, issued by the lanes of warp 0), TS tokens per 16 KB stage:
    // K rows first, then V rows.  A lane group of LPT lanes handles a token:
    // 16-byte shared-memory reads, the q.k dot per head reduced across the
    // group, and an online softmax per head.
    constexpr int TS = kStageBytes / (2 * (int)RB);
    constexpr int EPV = 16 / (int)sizeof(T);
    constexpr int NV = D / EPV;
    constexpr int LPT = NV < 32 ? NV : 32;
    constexpr int VPL = NV / LPT;
    constexpr int EPL = VPL * EPV;
    constexpr int TPW = 32 / LPT;
    constexpr int NGROUPS = (kNT / 32) * TPW;
    const int gl = lane % LPT;
    const int grp = warp * TPW + lane / LPT;
    const int nst3 = (n + TS - 1) / TS;

    auto issue3 = [&](int s) {  // called by all lanes of warp 0
        const int slot = s % kNStage;
        const int j0 = s * TS, nt = min(TS, n - j0);
        if (lane == 0) mbar_arrive_expect_tx(&full3[slot], (uint32_t)(2 * nt * RB));
        __syncwarp();
        uint8_t* dst = ring + (size_t)slot * kStageBytes;
        for (int j = lane; j < nt; j += 32) {
            const int t = sel[j0 + j];
            bulk_load(dst + (size_t)j * RB, Ku + (size_t)t * RB, (uint32_t)RB, &full3[slot]);
            bulk_load(dst + (size_t)(TS + j) * RB, Vu + (size_t)t * RB, (uint32_t)RB, &full3[slot]);
        }
    };
    if (warp == 0) {
        fence_proxy_async();
        for (int s = 0; s < kNStage && s < nst3; ++s) issue3(s);
    }

    float qr[MAXG][EPL];
#pragma unroll
    for (int h = 0; h < MAXG; ++h)
#pragma unroll
        for (int v = 0; v < VPL; ++v)
#pragma unroll
            for (int e = 0; e < EPV; ++e)
                qr[h][v * EPV + e] = (h < G) ? qf[h * D + (gl + v * LPT) * EPV + e] : 0.0f;
    float mrun[MAXG], lrun[MAXG], acc[MAXG][EPL];
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
        mrun[h] = -INFINITY;
        lrun[h] = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[h][e] = 0.0f;
    }
    bool ok3 = true;
    for (int s = 0; s < nst3; ++s) {
        const int slot = s % kNStage;
        if (!mbar_wait_bounded(&full3[slot], (uint32_t)((s / kNStage) & 1), a.err)) {
            ok3 = false;
            break;
        }
        const int nt = min(TS, n - s * TS);
        const uint8_t* kst = ring + (size_t)slot * kStageBytes;
        const uint8_t* vst = kst + (size_t)TS * RB;
        for (int jb = warp * TPW; jb < nt; jb += NGROUPS) {
            const int j = jb + lane / LPT;
            const bool okj = j < nt;
            float kf[EPL], vf[EPL];
#pragma unroll
            for (int v = 0; v < VPL; ++v) {
                if (okj) {
                    const uint4 kw = *reinterpret_cast<const uint4*>(kst + (size_t)j * RB + (size_t)(gl + v * LPT) * 16);
                    const uint4 vw = *reinterpret_cast<const uint4*>(vst + (size_t)j * RB + (size_t)(gl + v * LPT) * 16);
                    vec_to_f<T>(kw, kf + v * EPV);
                    vec_to_f<T>(vw, vf + v * EPV);
                } else {
#pragma unroll
                    for (int e = 0; e < EPV; ++e) {
                        kf[v * EPV + e] = 0.0f;
                        vf[v * EPV + e] = 0.0f;
                    }
                }
            }
            float sc[MAXG];
#pragma unroll
            for (int h = 0; h < MAXG; ++h) {
                float t = 0.0f;
#pragma unroll
                for (int e = 0; e < EPL; ++e) t = fmaf(qr[h][e], kf[e], t);
                sc[h] = t;
            }
#pragma unroll
            for (int o = LPT / 2; o > 0; o >>= 1)
#pragma unroll
                for (int h = 0; h < MAXG; ++h) sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], o);
            if (okj) {
#pragma unroll
                for (int h = 0; h < MAXG; ++h) {
                    if (h < G) {
                        const float x = sc[h] * a.inv_sqrt_d;
                        const float mn = fmaxf(mrun[h], x);
                        const float corr = __expf(mrun[h] - mn);
                        const float p = __expf(x - mn);
                        lrun[h] = fmaf(lrun[h], corr, p);
#pragma unroll
                        for (int e = 0; e < EPL; ++e) acc[h][e] = fmaf(p, vf[e], acc[h][e] * corr);
                        mrun[h] = mn;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty3[slot]);
        if (warp == 0 && s >= 1 && s - 1 + kNStage < nst3) {
            const int sp = s - 1;
            if (mbar_wait_bounded(&empty3[sp % kNStage], (uint32_t)((sp / kNStage) & 1), a.err)) {
                fence_proxy_async();
                issue3(sp + kNStage);
            } else {
                ok3 = false;  // the consumers' wait on the unfilled slot runs out as well
            }
        }
    }
    if (!ok3) s_abort = 1;
    __syncthreads();
    if (s_abort) return;
    float* comb = reinterpret_cast<float*>(ring);  // [NGROUPS][MAXG][D + 2]
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
        if (h < G) {
            float* cg = comb + ((size_t)grp * MAXG + h) * (D + 2);
#pragma unroll
            for (int v = 0; v < VPL; ++v)
#pragma unroll
                for (int e = 0; e < EPV; ++e) cg[(gl + v * LPT) * EPV + e] = acc[h][v * EPV + e];
            if (gl == 0) {
                cg[D] = mrun[h];
                cg[D + 1] = lrun[h];
            }
        }
    }
    __syncthreads();
    float* Ob = a.O + (size_t)b * a.H * D + (size_t)hk * G * D;
    for (int e = tid; e < G * D; e += kNT) {
        const int h = e / D, d = e - h * D;
        float M = -INFINITY;
        for (int g = 0; g < NGROUPS; ++g) M = fmaxf(M, comb[((size_t)g * MAXG + h) * (D + 2) + D]);
        float L = 0.0f, o = 0.0f;
        if (M != -INFINITY) {
            for (int g = 0; g < NGROUPS; ++g) {
                const float* cg = comb + ((size_t)g * MAXG + h) * (D + 2);
                const float mg = cg[D];
                if (mg == -INFINITY) continue;
                const float f = __expf(mg - M);
                L = fmaf(cg[D + 1], f, L);
                o = fmaf(cg[d], f, o);
            }
        }
        Ob[h * D + d] = L > 0.0f ? o / L : 0.0f;
    }
}

template <typename T, int D, int MAXG>
int launch_t(HsaArgs a, int batch, cudaStream_t st) {
    constexpr int EPV = 16 / (int)sizeof(T);
    constexpr int NV = D / EPV;
    constexpr int LPT = NV < 32 ? NV : 32;
    constexpr int NGROUPS = (kNT / 32) * (32 / LPT);
    const int sr_max = kStageBytes / (int)(D * sizeof(T));
    if (a.C <= sr_max) {
        a.carry_mode = 0;
        a.stage_rows = a.C * (sr_max / a.C);
        a.chunks_per_stage = a.stage_rows / a.C;
    } else {
        a.carry_mode = 1;
        a.stage_rows = sr_max;
        a.chunks_per_stage = 2;
    }
    const size_t ring = (size_t)kNStage * kStageBytes;
    const size_t comb = (size_t)NGROUPS * MAXG * (D + 2) * sizeof(float);
    const size_t region0 = align_up(ring > comb ? ring : comb, 128);
    a.off_bar = (int)region0;
    a.off_pst = (int)(region0 + 128);
    a.smem_bytes = (int)(a.off_pst + (a.carry_mode ? (size_t)2 * (D + 1) * sizeof(float) : 0));
    auto fn = hsa_kernel<T, D, MAXG>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, a.smem_bytes) != cudaSuccess)
        return RKV_ERR_CUDA;
    dim3 grid(a.head_count, batch);
    fn<<<grid, kNT, a.smem_bytes, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
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
    s.off_logits = off;
    off = align_up(off + (size_t)batch * head_count * s.G * (size_t)s.nchunks * sizeof(float), kWorkspaceAlign);
    s.off_sel = off;
    off = align_up(off + (size_t)batch * head_count * (size_t)(s.sel_cap > 0 ? s.sel_cap : 1) * sizeof(int),
                   kWorkspaceAlign);
    s.ws_bytes = off;
    return s;
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
