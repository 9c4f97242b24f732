// evict.cu -- stage-1 prefill eviction on sm_100a (rocket.cpp:61-169).
//
// Three kernels per call, each batched over items (layers / sequences):
//   evict_logits_kernel  grid (key tiles, KV heads, items)
//       logits l[r][k] = (q_r . k_k) / sqrt(D) for the R = G * obs_w window
//       rows of the KV head's query group (rocket.cpp:97-105), stored to the
//       workspace, plus per-(row, tile) max and sum of exp(l - max).  The last
//       CTA of a head folds the tile statistics into the row max M_r and
//       1 / (sum_r + 1e-9) (rocket.cpp:108-113).
//   evict_pool_kernel    grid (position tiles, KV heads, items)
//       head score hs[k] = sum_r exp(l[r][k] - M_r) * inv_r in row order
//       (rocket.cpp:114-116; the tensor-core engine of evict_mma.cu computes
//       it there and this kernel reads it), then max-pool over [k - pad, k + pad] clipped
//       to the sequence (rocket.cpp:120-129) by a doubling sparse table in
//       shared memory; one pooled row per KV head.
//   evict_select_kernel  grid (items)
//       sum of the pooled rows over KV heads in head order (rocket.cpp:142-148),
//       top target_keep by (score desc, index asc) via a 4 x 8-bit radix
//       select on order-preserving float keys, stable compaction into
//       ascending order, then the observation window (rocket.cpp:150-166).
#include "evict.cuh"

#include <float.h>

namespace rkv {
namespace {

constexpr int kNT = 256;      // threads of the scoring CTAs
constexpr int kKT = 128;      // keys per logits tile
constexpr int kRC = 32;       // query rows per pass (8 warps x 4 rows)
constexpr int kPoolKT = 256;  // positions per pooling CTA
constexpr int kSelNT = 1024;  // threads of the selection CTA

__global__ void __launch_bounds__(kNT) evict_logits_kernel(EvictArgs a) {
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ __align__(16) float sm[];
    const int DP = a.D + 4;
    float* Ks = sm;              // [kKT][DP]
    float* Qs = sm + kKT * DP;   // [kRC][DP]
    __shared__ int s_last;

    const int tile = blockIdx.x, hc = blockIdx.y, b = blockIdx.z;
    const int hk = a.head_begin + hc;
    const int k0 = tile * kKT;
    const int nkeys = min(kKT, a.nk - k0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint8_t* Kb = a.K + (size_t)b * a.k_stride;
    const uint8_t* Qb = a.Q + (size_t)b * a.q_stride;

    // K tile -> fp32 shared memory (exact conversion for bf16 and q8_0).
    const size_t krow0 = (size_t)hk * a.k_head_rows + k0;
    for (int e = tid; e < kKT * a.D; e += kNT) {
        const int kr = e / a.D, d = e - kr * a.D;
        float v = 0.0f;
        if (kr < nkeys) v = load_elem(Kb, a.dtype, (krow0 + kr) * a.D + d);
        Ks[kr * DP + d] = v;
    }

    const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
    for (int rc0 = 0; rc0 < a.R; rc0 += kRC) {
        __syncthreads();
        for (int e = tid; e < kRC * a.D; e += kNT) {
            const int rr = e / a.D, d = e - rr * a.D;
            const int r = rc0 + rr;
            float v = 0.0f;
            if (r < a.R) {
                const int h = hk * a.G + r / a.obs_w;
                const int pos = a.q_row0 + r % a.obs_w;
                v = load_elem(Qb, a.dtype, ((size_t)h * a.q_head_rows + pos) * a.D + d);
            }
            Qs[rr * DP + d] = v;
        }
        __syncthreads();

        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
        const float* qw = Qs + (warp * 4) * DP;
#pragma unroll 2
        for (int d = 0; d < a.D; d += 4) {
            float4 kv[4], qv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(Ks + (lane + 32 * j) * DP + d);
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(qw + i * DP + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float t = acc[i][j];
                    t = fmaf(qv[i].x, kv[j].x, t);
                    t = fmaf(qv[i].y, kv[j].y, t);
                    t = fmaf(qv[i].z, kv[j].z, t);
                    t = fmaf(qv[i].w, kv[j].w, t);
                    acc[i][j] = t;
                }
        }

#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = rc0 + warp * 4 + i;
            if (r >= a.R) break;  // warp-uniform
            float l[4];
            float m = -FLT_MAX;  // rocket.cpp:93 starts the row max here
            float* lrow = a.logits + (row_base + r) * (size_t)a.nk + k0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int key = lane + 32 * j;
                l[j] = acc[i][j] * a.inv_sqrt_d;
                if (key < nkeys) {
                    lrow[key] = l[j];
                    m = fmaxf(m, l[j]);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (lane + 32 * j < nkeys) s += expf(l[j] - m);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) a.tstats[(row_base + r) * a.ntiles + tile] = make_float2(m, s);
        }
    }

    // The last CTA of this (item, head) folds the tile statistics.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&a.counters[(size_t)b * a.head_count + hc], 1u);
        s_last = (prev == (unsigned)a.ntiles - 1u);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int r = tid; r < a.R; r += kNT) {
        const float2* ts = a.tstats + (row_base + r) * a.ntiles;
        float M = -FLT_MAX;
        for (int t = 0; t < a.ntiles; ++t) M = fmaxf(M, __ldcg(&ts[t].x));
        float S = 0.0f;
        for (int t = 0; t < a.ntiles; ++t) {
            const float2 v = __ldcg(ts + t);
            S += v.y * expf(v.x - M);
        }
        a.rstats[row_base + r] = make_float2(M, 1.0f / (S + 1e-9f));
    }
    if (tid == 0) a.counters[(size_t)b * a.head_count + hc] = 0u;
}

// One CTA per (position tile, KV head, item): head scores for the tile plus
// its +-pad halo, then the clipped window max.  The cross-head sum happens in
// the select kernel, in head order.
__global__ void __launch_bounds__(kNT) evict_pool_kernel(PoolArgs a) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a dependent of the scorer
    asm volatile("griddepcontrol.launch_dependents;");  // the selection may be scheduled (it waits)
    extern __shared__ __align__(16) float sm[];
    const int pe = a.pad_eff;
    const int NA = kPoolKT + 2 * pe;
    float* bufA = sm;
    float* bufB = sm + NA;
    float2* rs = reinterpret_cast<float2*>(sm + 2 * NA);  // [R]
    const int tid = threadIdx.x, hc = blockIdx.y, b = blockIdx.z;
    const int k0 = blockIdx.x * kPoolKT;
    const int x0 = k0 - pe;
    const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;
    float* out = a.pooled + ((size_t)b * a.head_count + hc) * a.nk;

    if (a.pad < 0) {
        // Empty pooling window: every pooled score stays -FLT_MAX (rocket.cpp:122).
        for (int i = tid; i < kPoolKT; i += kNT)
            if (k0 + i < a.nk) out[k0 + i] = -FLT_MAX;
        return;
    }
    if (!a.hs_direct)
        for (int r = tid; r < a.R; r += kNT) rs[r] = a.rstats[row_base + r];
    __syncthreads();
    for (int x = tid; x < NA; x += kNT) {
        const int p = x0 + x;
        float v = -FLT_MAX;  // rocket.cpp:122: NaN never wins the pool
        if (p >= 0 && p < a.nk) {
            if (a.hs_direct) {
                v = __ldg(a.logits + ((size_t)b * a.head_count + hc) * a.nk + p);
            } else {
                const float* lp = a.logits + row_base * (size_t)a.nk + p;
                float hs = 0.0f;
#pragma unroll 8
                for (int r = 0; r < a.R; ++r) {
                    const float e = expf(__ldg(lp + (size_t)r * a.nk) - rs[r].x);
                    hs = __fadd_rn(hs, __fmul_rn(e, rs[r].y));
                }
                v = hs;
            }
        }
        bufA[x] = v;
    }
    __syncthreads();
    // Doubling: after step m, buf[x] = max(A[x .. x + 2^(m+1) - 1]).
    float* src = bufA;
    float* dst = bufB;
    for (int m = 0; m < a.log2w; ++m) {
        const int len = 1 << m;
        const int lim = NA - 2 * len + 1;
        for (int x = tid; x < lim; x += kNT) dst[x] = fmaxf(src[x], src[x + len]);
        __syncthreads();
        float* t = src;
        src = dst;
        dst = t;
    }
    const int off2 = 2 * pe - (1 << a.log2w) + 1;
    for (int i = tid; i < kPoolKT; i += kNT)
        if (k0 + i < a.nk) out[k0 + i] = fmaxf(src[i], src[i + off2]);
}

__global__ void __launch_bounds__(kSelNT) evict_select_kernel(SelectArgs a) {
    asm volatile("griddepcontrol.launch_dependents;");  // a dependent compaction may start (it waits)
    __shared__ int hist[256];
    __shared__ int scan_tmp[66];
    __shared__ uint32_t s_prefix, s_lo[32], s_hi[32];
    __shared__ int s_kk;
    const int tid = threadIdx.x, b = blockIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t* keys = a.keys + (size_t)b * a.nk;
    int* kept = a.kept + (size_t)b * a.kept_stride;

    // total = sum of the HK pooled rows in head order (rocket.cpp:143-146), as order-preserving keys
    uint32_t kmin = 0xffffffffu, kmax = 0u;
    for (int i = tid; i < a.nk; i += kSelNT) {
        float v = 0.0f;
        for (int h = 0; h < a.HK; ++h) v = __fadd_rn(v, a.pooled[((size_t)b * a.HK + h) * a.nk + i]);
        const uint32_t k = float_key(v);
        keys[i] = k;
        kmin = min(kmin, k);
        kmax = max(kmax, k);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    if (lane == 0) {
        s_lo[warp] = kmin;
        s_hi[warp] = kmax;
    }
    __syncthreads();
    kmin = s_lo[lane];
    kmax = s_hi[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    // radix select of the target_keep-th largest key in digits of up to 8 bits, starting below the
    // bits every key shares (as in evict_select_reg_kernel)
    const uint32_t diff = kmin ^ kmax;
    int rem = diff ? 32 - __clz(diff) : 0;
    uint32_t mask = rem == 32 ? 0u : ~((1u << rem) - 1u);
    if (tid == 0) {
        s_prefix = kmax & mask;
        s_kk = a.target_keep;
    }
    __syncthreads();
    while (rem > 0 && a.target_keep > 0) {
        const int w = rem < 8 ? rem : 8, shift = rem - w, nb = 1 << w;
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        for (int i = tid; i < a.nk; i += kSelNT) {
            const uint32_t k = keys[i];
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & (uint32_t)(nb - 1)], 1);
        }
        __syncthreads();
        if (warp == 0) {
            int c[8], sum = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int idx = 8 * lane + t;
                c[t] = idx < nb ? hist[nb - 1 - idx] : 0;
                sum += c[t];
            }
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            int before = incl - sum;
            const int kk = s_kk;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (c[t] > 0 && before < kk && before + c[t] >= kk) {
                    s_kk = kk - before;
                    s_prefix = prefix | ((uint32_t)(nb - 1 - (8 * lane + t)) << shift);
                }
                before += c[t];
            }
        }
        mask |= (uint32_t)(nb - 1) << shift;
        rem = shift;
        __syncthreads();
    }
    const uint32_t T = a.target_keep > 0 ? s_prefix : 0xffffffffu;
    const int need = a.target_keep > 0 ? s_kk : 0;  // threshold-key members kept, lowest index first

    // stable compaction: each thread a contiguous chunk, one dual block scan
    const int C = (a.nk + kSelNT - 1) / kSelNT;
    const int i0 = tid * C, i1 = min(i0 + C, a.nk);
    int gt = 0, eq = 0;
    for (int i = i0; i < i1; ++i) {
        const uint32_t k = keys[i];
        gt += k > T ? 1 : 0;
        eq += k == T ? 1 : 0;
    }
    int gt_before, eq_tot, gt_tot;
    const int eq_before = block_exclusive_scan2(eq, gt, scan_tmp, &gt_before, &eq_tot, &gt_tot);
    if (a.target_keep > 0) {
        int pos = gt_before + min(eq_before, need), e = eq_before;
        for (int i = i0; i < i1; ++i) {
            const uint32_t k = keys[i];
            if (k > T) {
                kept[pos++] = i;
            } else if (k == T) {
                if (e < need) kept[pos++] = i;
                ++e;
            }
        }
    }
    for (int t = tid; t < a.obs_w; t += kSelNT) kept[a.target_keep + t] = a.nk + t;
    if (tid == 0) a.n_kept[b] = a.target_keep + a.obs_w;
}

// The same selection with every key in registers (up to kSelPer consecutive
// keys per thread, nk <= 16384): the head-order sum, a radix select in
// digits of up to 8 bits that starts below the bits every key shares (the
// common prefix of the block's min and max key: the pooled sums share their
// sign and top exponent bits, which would put every key of a first 8-bit
// digit into one or two bins), one warp scanning the bins, and one dual
// block scan for the stable compaction (position of a kept key = keys above
// the threshold before it + min(threshold keys before it, the number of
// threshold keys kept)).
constexpr int kSelPer = 16;
__global__ void __launch_bounds__(kSelNT) evict_select_reg_kernel(SelectArgs a) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a dependent of the pooling
    asm volatile("griddepcontrol.launch_dependents;");  // a dependent compaction may start (it waits)
    __shared__ int hist[256];
    __shared__ int scan_tmp[66];
    __shared__ uint32_t s_prefix, s_lo[32], s_hi[32];
    __shared__ int s_kk;
    const int tid = threadIdx.x, b = blockIdx.x, lane = tid & 31, warp = tid >> 5;
    int* kept = a.kept + (size_t)b * a.kept_stride;
    int C = (a.nk + kSelNT - 1) / kSelNT;
    const bool vec = (a.nk & 3) == 0;
    if (vec) C = (C + 3) & ~3;  // whole 16-byte groups per thread
    const int i0 = tid * C;
    // total = sum of the HK pooled rows in head order (rocket.cpp:143-146)
    float v[kSelPer];
#pragma unroll
    for (int j = 0; j < kSelPer; ++j) v[j] = 0.0f;
    if (vec) {
        for (int h0 = 0; h0 < a.HK; h0 += 2) {  // two heads' loads in flight at once
            float4 x[2][kSelPer / 4];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float4* row = reinterpret_cast<const float4*>(a.pooled + ((size_t)b * a.HK + h0 + u) * a.nk + i0);
#pragma unroll
                for (int g = 0; g < kSelPer / 4; ++g)
                    x[u][g] = (h0 + u < a.HK && 4 * g < C && i0 + 4 * g < a.nk) ? __ldg(row + g) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                if (h0 + u >= a.HK) break;
#pragma unroll
                for (int g = 0; g < kSelPer / 4; ++g) {
                    v[4 * g] = __fadd_rn(v[4 * g], x[u][g].x);
                    v[4 * g + 1] = __fadd_rn(v[4 * g + 1], x[u][g].y);
                    v[4 * g + 2] = __fadd_rn(v[4 * g + 2], x[u][g].z);
                    v[4 * g + 3] = __fadd_rn(v[4 * g + 3], x[u][g].w);
                }
            }
        }
    } else {
        for (int h = 0; h < a.HK; ++h) {
            const float* row = a.pooled + ((size_t)b * a.HK + h) * a.nk + i0;
            float x[kSelPer];
#pragma unroll
            for (int j = 0; j < kSelPer; ++j) x[j] = (j < C && i0 + j < a.nk) ? __ldg(row + j) : 0.0f;
#pragma unroll
            for (int j = 0; j < kSelPer; ++j) v[j] = __fadd_rn(v[j], x[j]);
        }
    }
    uint32_t key[kSelPer];
    uint32_t valid = 0u, kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
    for (int j = 0; j < kSelPer; ++j) {
        key[j] = float_key(v[j]);
        if (j < C && i0 + j < a.nk) {
            valid |= 1u << j;
            kmin = min(kmin, key[j]);
            kmax = max(kmax, key[j]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    if (lane == 0) {
        s_lo[warp] = kmin;
        s_hi[warp] = kmax;
    }
    __syncthreads();
    kmin = s_lo[lane];
    kmax = s_hi[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    // bits below the common prefix of every key
    const uint32_t diff = kmin ^ kmax;
    int rem = diff ? 32 - __clz(diff) : 0;
    uint32_t mask = rem == 32 ? 0u : ~((1u << rem) - 1u);
    if (tid == 0) {
        s_prefix = kmax & mask;
        s_kk = a.target_keep;
    }
    __syncthreads();
    // radix select of the target_keep-th largest key, digits of up to 8 bits from the top
    while (rem > 0 && a.target_keep > 0) {
        const int w = rem < 8 ? rem : 8, shift = rem - w, nb = 1 << w;
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix;
#pragma unroll
        for (int j = 0; j < kSelPer; ++j)
            if (((valid >> j) & 1u) && (key[j] & mask) == prefix) atomicAdd(&hist[(key[j] >> shift) & (uint32_t)(nb - 1)], 1);
        __syncthreads();
        if (warp == 0) {  // the digit where the count from the top reaches kk; lane L: digits nb-1-8L ..
            int c[8], sum = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int idx = 8 * lane + t;
                c[t] = idx < nb ? hist[nb - 1 - idx] : 0;
                sum += c[t];
            }
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            int before = incl - sum;
            const int kk = s_kk;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (c[t] > 0 && before < kk && before + c[t] >= kk) {
                    s_kk = kk - before;
                    s_prefix = prefix | ((uint32_t)(nb - 1 - (8 * lane + t)) << shift);
                }
                before += c[t];
            }
        }
        mask |= (uint32_t)(nb - 1) << shift;
        rem = shift;
        __syncthreads();
    }
    const uint32_t T = a.target_keep > 0 ? s_prefix : 0xffffffffu;
    const int need = a.target_keep > 0 ? s_kk : 0;  // threshold-key members kept, lowest index first
    int gt = 0, eq = 0;
#pragma unroll
    for (int j = 0; j < kSelPer; ++j)
        if ((valid >> j) & 1u) {
            gt += key[j] > T ? 1 : 0;
            eq += key[j] == T ? 1 : 0;
        }
    int gt_before, eq_tot, gt_tot;
    const int eq_before = block_exclusive_scan2(eq, gt, scan_tmp, &gt_before, &eq_tot, &gt_tot);
    if (a.target_keep > 0) {
        int pos = gt_before + min(eq_before, need), e = eq_before;
#pragma unroll
        for (int j = 0; j < kSelPer; ++j) {
            if (!((valid >> j) & 1u)) continue;
            if (key[j] > T) {
                kept[pos++] = i0 + j;
            } else if (key[j] == T) {
                if (e < need) kept[pos++] = i0 + j;
                ++e;
            }
        }
    }
    for (int t = tid; t < a.obs_w; t += kSelNT) kept[a.target_keep + t] = a.nk + t;
    if (tid == 0) a.n_kept[b] = a.target_keep + a.obs_w;
}

// The selection of long prefixes over several CTAs per item (one cooperative
// launch, every CTA resident): each CTA holds a contiguous chunk of up to
// kCoopNT * kSelPer keys in registers; the key range (min, max), the radix
// histograms and the per-CTA counts are merged in the workspace, and every
// CTA of an item takes the same digit decision from the merged histogram
// after a bounded grid barrier.  Workspace words (zeroed before the launch):
// [0] the barrier counter, then per item ~min and max, 4 x 256 histogram
// bins, and per CTA the (above, equal) threshold counts.
constexpr int kCoopNT = 512;
struct SelCoop {
    unsigned* bar;
    unsigned* mm;  // [item][2]: ~min, max (atomicMax of both)
    int* hist;     // [item][4][256]
    int* cnt;      // [item][P][2]
    int P, chunk;
};

__global__ void __launch_bounds__(kCoopNT) evict_select_coop_kernel(SelectArgs a, SelCoop c) {
    asm volatile("griddepcontrol.launch_dependents;");  // a dependent compaction may start (it waits)
    __shared__ int hist[256];
    __shared__ int scan_tmp[66];
    __shared__ uint32_t s_lo[16], s_hi[16], s_prefix;
    __shared__ int s_kk, s_ok, s_pre[2];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = blockIdx.x / c.P, p = blockIdx.x % c.P;
    const int base = p * c.chunk, end = min(base + c.chunk, a.nk);
    const int C = (c.chunk + kCoopNT - 1) / kCoopNT;  // <= kSelPer
    const int i0 = base + tid * C;
    unsigned nbar = 0;
    auto gsync = [&]() -> bool {  // grid barrier; false once any CTA's wait has run out
        __syncthreads();
        if (tid == 0) s_ok = grid_sync_bounded(c.bar, (++nbar) * gridDim.x, a.err) ? 1 : 0;
        else ++nbar;
        __syncthreads();
        return s_ok != 0;
    };
    // total = sum of the HK pooled rows in head order (rocket.cpp:143-146)
    float v[kSelPer];
#pragma unroll
    for (int j = 0; j < kSelPer; ++j) v[j] = 0.0f;
    for (int h = 0; h < a.HK; ++h) {
        const float* row = a.pooled + ((size_t)b * a.HK + h) * a.nk + i0;
        float x[kSelPer];
#pragma unroll
        for (int j = 0; j < kSelPer; ++j) x[j] = (j < C && i0 + j < end) ? __ldg(row + j) : 0.0f;
#pragma unroll
        for (int j = 0; j < kSelPer; ++j) v[j] = __fadd_rn(v[j], x[j]);
    }
    uint32_t key[kSelPer], valid = 0u, kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
    for (int j = 0; j < kSelPer; ++j) {
        key[j] = float_key(v[j]);
        if (j < C && i0 + j < end) {
            valid |= 1u << j;
            kmin = min(kmin, key[j]);
            kmax = max(kmax, key[j]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    if (lane == 0) {
        s_lo[warp] = kmin;
        s_hi[warp] = kmax;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kCoopNT / 32; ++w) {
            kmin = min(kmin, s_lo[w]);
            kmax = max(kmax, s_hi[w]);
        }
        atomicMax(&c.mm[2 * b], ~kmin);
        atomicMax(&c.mm[2 * b + 1], kmax);
    }
    if (!gsync()) return;
    kmin = ~__ldcg(&c.mm[2 * b]);
    kmax = __ldcg(&c.mm[2 * b + 1]);
    const uint32_t diff = kmin ^ kmax;
    int rem = diff ? 32 - __clz(diff) : 0;
    uint32_t mask = rem == 32 ? 0u : ~((1u << rem) - 1u);
    uint32_t prefix = kmax & mask;
    int kk = a.target_keep;
    // every CTA of the grid takes the same four barrier rounds, whatever its item needs
    for (int ps = 0; ps < 4; ++ps) {
        const bool active = rem > 0 && a.target_keep > 0;  // uniform over the item's CTAs
        const int w = rem < 8 ? rem : 8, shift = active ? rem - w : 0, nb = 1 << w;
        int* gh = c.hist + ((size_t)b * 4 + ps) * 256;
        if (active) {
            if (tid < 256) hist[tid] = 0;
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kSelPer; ++j)
                if (((valid >> j) & 1u) && (key[j] & mask) == prefix)
                    atomicAdd(&hist[(key[j] >> shift) & (uint32_t)(nb - 1)], 1);
            __syncthreads();
            if (tid < nb && hist[tid]) atomicAdd(&gh[tid], hist[tid]);
        }
        if (!gsync()) return;
        if (!active) continue;
        if (warp == 0) {  // the same decision in every CTA of the item, from the merged histogram
            int cc[8], sum = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int idx = 8 * lane + t;
                cc[t] = idx < nb ? __ldcg(&gh[nb - 1 - idx]) : 0;
                sum += cc[t];
            }
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            int before = incl - sum;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (cc[t] > 0 && before < kk && before + cc[t] >= kk) {
                    s_kk = kk - before;
                    s_prefix = prefix | ((uint32_t)(nb - 1 - (8 * lane + t)) << shift);
                }
                before += cc[t];
            }
        }
        __syncthreads();
        prefix = s_prefix;
        kk = s_kk;
        mask |= (uint32_t)(nb - 1) << shift;
        rem = shift;
    }
    const uint32_t T = a.target_keep > 0 ? prefix : 0xffffffffu;
    const int need = a.target_keep > 0 ? kk : 0;  // threshold-key members kept, lowest index first
    int gt = 0, eq = 0;
#pragma unroll
    for (int j = 0; j < kSelPer; ++j)
        if ((valid >> j) & 1u) {
            gt += key[j] > T ? 1 : 0;
            eq += key[j] == T ? 1 : 0;
        }
    int gt_before, eq_tot, gt_tot;
    const int eq_before = block_exclusive_scan2(eq, gt, scan_tmp, &gt_before, &eq_tot, &gt_tot);
    if (tid == 0) {
        c.cnt[((size_t)b * c.P + p) * 2] = gt_tot;
        c.cnt[((size_t)b * c.P + p) * 2 + 1] = eq_tot;
    }
    if (!gsync()) return;
    if (tid == 0) {  // the counts of the item's CTAs before this one
        int g0 = 0, e0 = 0;
        for (int q = 0; q < p; ++q) {
            g0 += __ldcg(&c.cnt[((size_t)b * c.P + q) * 2]);
            e0 += __ldcg(&c.cnt[((size_t)b * c.P + q) * 2 + 1]);
        }
        s_pre[0] = g0;
        s_pre[1] = e0;
    }
    __syncthreads();
    int* kept = a.kept + (size_t)b * a.kept_stride;
    if (a.target_keep > 0) {
        const int eb = s_pre[1] + eq_before;
        int pos = s_pre[0] + gt_before + min(eb, need), e = eb;
#pragma unroll
        for (int j = 0; j < kSelPer; ++j) {
            if (!((valid >> j) & 1u)) continue;
            if (key[j] > T) {
                kept[pos++] = i0 + j;
            } else if (key[j] == T) {
                if (e < need) kept[pos++] = i0 + j;
                ++e;
            }
        }
    }
    if (p == 0) {
        for (int t = tid; t < a.obs_w; t += kCoopNT) kept[a.target_keep + t] = a.nk + t;
        if (tid == 0) a.n_kept[b] = a.target_keep + a.obs_w;
    }
}

__global__ void evict_keep_all_kernel(int* kept, int kept_stride, int* n_kept, int len_k) {
    asm volatile("griddepcontrol.launch_dependents;");  // a dependent compaction may start (it waits)
    const int b = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < len_k; i += gridDim.x * blockDim.x)
        kept[(size_t)b * kept_stride + i] = i;
    if (blockIdx.x == 0 && threadIdx.x == 0) n_kept[b] = len_k;
}

// One warp waits on a barrier that nothing arrives at; the bounded wait runs
// out and records RKV_ERR_DEVICE_TIMEOUT (the diagnostic of the failure path).
__global__ void wait_selftest_kernel(int* err) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    mbar_wait_bounded(&bar, 0, err);
}

int floor_log2(int x) {
    int j = 0;
    while ((2 << j) <= x) ++j;
    return j;
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
EvictShape evict_shape(const rkv_config& c, int len_q, int len_k, int batch, int head_count) {
    EvictShape s{};
    s.G = c.num_heads / c.num_heads_kv;
    s.obs_w = len_q < c.window_size ? len_q : c.window_size;
    s.nk = len_k - s.obs_w;
    s.R = s.G * s.obs_w;
    s.ntiles = s.nk > 0 ? (s.nk + kKT - 1) / kKT : 0;
    s.target_keep = c.prompt_budget - s.obs_w > 0 ? c.prompt_budget - s.obs_w : 0;
    s.keep_all = (len_k <= c.prompt_budget) || (s.target_keep >= s.nk);
    const size_t B = (size_t)batch, HC = (size_t)head_count, R = (size_t)s.R;
    const size_t nk = s.nk > 0 ? (size_t)s.nk : 0;
    size_t off = kWorkspaceHeader;
    s.off_counters = off; off = align_up(off + B * HC * sizeof(unsigned), kWorkspaceAlign);
    s.off_rstats = off;   off = align_up(off + B * HC * R * sizeof(float2), kWorkspaceAlign);
    s.off_tstats = off;   off = align_up(off + B * HC * R * s.ntiles * sizeof(float2), kWorkspaceAlign);
    s.nkp = (int)((nk + 3) & ~(size_t)3);
    s.off_logits = off;   off = align_up(off + B * HC * R * (size_t)s.nkp * sizeof(float), kWorkspaceAlign);
    s.off_keys = off;     off = align_up(off + B * nk * sizeof(uint32_t), kWorkspaceAlign);
    s.off_pooled = off;   off = align_up(off + B * (size_t)c.num_heads_kv * nk * sizeof(float), kWorkspaceAlign);
    s.off_hs = off;       off = align_up(off + B * HC * nk * sizeof(float), kWorkspaceAlign);
    s.ws_bytes = off;
    return s;
}

static size_t logits_smem(int D) { return (size_t)(kKT + kRC) * (D + 4) * sizeof(float); }

static int pool_smem(int pad_eff, int R, size_t* bytes) {
    *bytes = (size_t)2 * (kPoolKT + 2 * (size_t)pad_eff) * sizeof(float) + (size_t)R * sizeof(float2);
    return *bytes <= (size_t)200 * 1024 ? RKV_OK : RKV_ERR_UNSUPPORTED;
}

int evict_check_supported(const rkv_config& c, int dtype, const EvictShape& s) {
    if (c.dim_head % 4 != 0 || c.dim_head > 256) return RKV_ERR_UNSUPPORTED;
    if (dtype == RKV_Q8_0 && c.dim_head % 32 != 0) return RKV_ERR_INVALID_ARG;
    if (!s.keep_all && c.kernel_size / 2 >= 0) {
        const int pe = (c.kernel_size / 2 < s.nk - 1) ? c.kernel_size / 2 : s.nk - 1;
        size_t b;
        if (pool_smem(pe, s.R, &b) != RKV_OK) return RKV_ERR_UNSUPPORTED;
    }
    return RKV_OK;
}

static int set_smem_attr(const void* fn, size_t bytes) {
    if (bytes <= 48 * 1024) return RKV_OK;
    return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess
               ? RKV_OK
               : RKV_ERR_CUDA;
}

int launch_evict_scores(const EvictArgs& a, int batch, cudaStream_t st) {
    if (a.R > 0 && a.ntiles > 0) {
        const size_t smem = logits_smem(a.D);
        if (set_smem_attr((const void*)evict_logits_kernel, smem) != RKV_OK) return RKV_ERR_CUDA;
        if (cudaMemsetAsync(a.counters, 0, (size_t)batch * a.head_count * sizeof(unsigned), st) != cudaSuccess)
            return RKV_ERR_CUDA;
        dim3 grid(a.ntiles, a.head_count, batch);
        evict_logits_kernel<<<grid, kNT, smem, st>>>(a);
        if (cudaGetLastError() != cudaSuccess) return RKV_ERR_CUDA;
    }
    return RKV_OK;
}

int launch_evict_pool(const PoolArgs& in, int batch, cudaStream_t st) {
    PoolArgs a = in;
    if (a.nk <= 0) return RKV_OK;
    a.pad_eff = a.pad < 0 ? 0 : (a.pad < a.nk - 1 ? a.pad : a.nk - 1);
    a.log2w = floor_log2(2 * a.pad_eff + 1);
    size_t smem;
    if (pool_smem(a.pad_eff, a.R, &smem) != RKV_OK) return RKV_ERR_UNSUPPORTED;
    if (set_smem_attr((const void*)evict_pool_kernel, smem) != RKV_OK) return RKV_ERR_CUDA;
    dim3 grid((a.nk + kPoolKT - 1) / kPoolKT, a.head_count, batch);
    if (launch_pdl(evict_pool_kernel, grid, dim3(kNT), smem, st, a) != cudaSuccess) {
        (void)cudaGetLastError();
        return RKV_ERR_CUDA;
    }
    return RKV_OK;
}

int launch_evict_select(const SelectArgs& a, int batch, cudaStream_t st) {
    if (a.nk <= kSelNT * kSelPer) {
        if (launch_pdl(evict_select_reg_kernel, dim3(batch), dim3(kSelNT), 0, st, a) != cudaSuccess) {
            (void)cudaGetLastError();
            return RKV_ERR_CUDA;
        }
        return RKV_OK;
    }
    // long prefixes: several CTAs per item in one cooperative launch, bookkeeping in the keys region
    SelCoop c{};
    c.chunk = kCoopNT * kSelPer;
    c.P = (a.nk + c.chunk - 1) / c.chunk;
    const size_t words = 1 + 2 * (size_t)batch + 1024 * (size_t)batch + 2 * (size_t)c.P * batch;
    if (a.err && words <= (size_t)batch * a.nk) {
        c.bar = a.keys;
        c.mm = a.keys + 1;
        c.hist = reinterpret_cast<int*>(a.keys + 1 + 2 * (size_t)batch);
        c.cnt = c.hist + 1024 * (size_t)batch;
        if (cudaMemsetAsync(a.keys, 0, words * sizeof(uint32_t), st) != cudaSuccess) return RKV_ERR_CUDA;
        SelectArgs aa = a;
        void* args[] = {&aa, &c};
        const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(evict_select_coop_kernel),
                                                          dim3(batch * c.P), dim3(kCoopNT), args, 0, st);
        if (e == cudaSuccess) return RKV_OK;
        (void)cudaGetLastError();
        if (e != cudaErrorCooperativeLaunchTooLarge && e != cudaErrorNotSupported) return RKV_ERR_CUDA;
    }
    evict_select_kernel<<<batch, kSelNT, 0, st>>>(a);  // one CTA per item
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

int launch_wait_selftest(int* err, cudaStream_t st) {
    if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return RKV_ERR_CUDA;
    wait_selftest_kernel<<<1, 32, 0, st>>>(err);
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

int launch_evict_keep_all(int* kept, int kept_stride, int* n_kept, int len_k, int batch, cudaStream_t st) {
    const int blocks = len_k > 0 ? (len_k + 255) / 256 : 1;
    dim3 grid(blocks < 1024 ? blocks : 1024, batch);
    evict_keep_all_kernel<<<grid, 256, 0, st>>>(kept, kept_stride, n_kept, len_k);
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

}  // namespace rkv
