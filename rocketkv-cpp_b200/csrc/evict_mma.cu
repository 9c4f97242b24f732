// evict_mma.cu -- stage-1 scoring on the tcgen05 tensor cores (sm_100a).
//
// The window rows of a KV head's query group against 128 keys per CTA form
// one MMA tile: D[128 keys][N rows] = K_tile[128][D] . Q_rows[N][D]^T, with
// N = G * obs_w rounded up to 16 and the accumulator in tensor memory.
// fp32 inputs run as three TF32 products per K step (hi.hi + hi.lo + lo.hi,
// where hi keeps the top 10 mantissa bits of x and lo = x - hi exactly), so
// the logits carry close to fp32 accuracy; bf16 inputs run one bf16 product
// (exact products, fp32 accumulation).
//
// Operands are staged by the threads in shared memory in the K-major,
// no-swizzle layout of tcgen05 (8-row core matrices of 16-byte rows; the
// 16-byte K unit u of row r at u * rows * 16 + r * 16), one 64-byte slice of
// every row at a time, double-buffered, the next slice loaded into registers
// meanwhile; one thread issues the MMAs and a
// tcgen05.commit to an mbarrier releases each buffer.  Every wait is bounded;
// tensor memory is freed on every path.
//
// Three launches per call (rocket.cpp:97-116):
//   MODE 0  per (row, tile) max and sum of exp(l - max) of the logits
//           l = (q . k) / sqrt(D);
//   evict_fold_kernel folds those into the row max M_r and 1 / (sum_r + 1e-9);
//   MODE 1  computes the logits again and the head score of every key,
//           hs[k] = sum_r exp(l[r][k] - M_r) * inv_r in row order, written
//           for the pooling kernel (the logits are never stored).
#include "evict.cuh"
#include "tc_common.cuh"

#include <float.h>

namespace rkv {
namespace {

constexpr int kMT = 128;       // keys per tile: the MMA's M
constexpr int kMmaNT = 128;    // threads: warp w reads tensor-memory lanes 32w .. 32w+31
constexpr int kSliceB = 64;    // bytes of every row staged per slice (four 16-byte K units, two MMA K steps)
constexpr int kTB = 129;       // row stride (floats) of the statistics transpose buffer

struct MmaLayout {  // shared-memory offsets, the same on host and device
    int NP, slices, upr, kb, qb, buf, bars, epi, total;
};
__host__ __device__ inline MmaLayout mma_layout(int R, int D, int es, int mode) {
    MmaLayout L{};
    L.NP = (R + 15) & ~15;
    const int rowb = D * es;
    L.upr = rowb / 16;                       // 16-byte units per row
    L.slices = (rowb + kSliceB - 1) / kSliceB;
    const int split = es == 4 ? 2 : 1;
    L.kb = kMT * kSliceB;                    // one K operand slice
    L.qb = L.NP * kSliceB;                   // one Q operand slice
    L.buf = split * (L.kb + L.qb);
    L.bars = 0;                              // two mbarriers + the tensor-memory address
    L.epi = 128 + 2 * L.buf;
    const int epi_bytes = mode == 0 ? 32 * kTB * 4 : L.NP * 8;
    L.total = L.epi + epi_bytes;
    return L;
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kMmaNT) evict_mma_kernel(const EvictArgs a) {
    asm volatile("griddepcontrol.launch_dependents;");
    constexpr int ES = (int)sizeof(T);
    constexpr bool TF32 = ES == 4;
    extern __shared__ __align__(128) uint8_t sm[];
    const MmaLayout L = mma_layout(a.R, a.D, ES, MODE);
    uint64_t* done = reinterpret_cast<uint64_t*>(sm);  // [2]: MMAs of buffer 0 / 1 complete
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 16);

    const int tile = blockIdx.x, hc = blockIdx.y, b = blockIdx.z;
    const int hk = a.head_begin + hc;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int k0 = tile * kMT;
    const int nkeys = min(kMT, a.nk - k0);
    const int NP = L.NP;
    const uint32_t tcols = NP <= 32 ? 32u : NP <= 64 ? 64u : NP <= 128 ? 128u : 256u;
    const size_t row_base = ((size_t)b * a.head_count + hc) * a.R;

    if (tid == 0) {
        mbar_init(&done[0], 1);
        mbar_init(&done[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, tcols);
    if (MODE == 1) {
        float2* rs = reinterpret_cast<float2*>(sm + L.epi);
        for (int r = tid; r < NP; r += kMmaNT) rs[r] = r < a.R ? a.rstats[row_base + r] : make_float2(0.0f, 0.0f);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    // ---- operand slices and MMAs ----
    const uint8_t* Kb = a.K + (size_t)b * a.k_stride;
    const uint8_t* Qb = a.Q + (size_t)b * a.q_stride;
    const size_t rowb = (size_t)a.D * ES;
    const uint8_t* krow = Kb + ((size_t)hk * a.k_head_rows + k0 + tid) * rowb;  // this thread's key row
    const uint32_t idesc = mma_idesc(TF32 ? 2u : 1u, (uint32_t)NP);
    constexpr int UPS = kSliceB / 16;  // 16-byte units per row and slice
    // this thread's Q rows: r = tid and r = tid + 128 (zero beyond R)
    const uint8_t* qrow[2] = {nullptr, nullptr};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int r = tid + i * kMmaNT;
        if (r < a.R) {
            const int h = hk * a.G + r / a.obs_w;
            const int pos = a.q_row0 + r % a.obs_w;
            qrow[i] = Qb + ((size_t)h * a.q_head_rows + pos) * rowb;
        }
    }
    // the next slice's global data is loaded into registers while the current one is stored and multiplied
    uint4 kx[UPS], qx[2][UPS];
    auto fetch = [&](int s) {
        const int u0 = s * UPS, nu = min(UPS, L.upr - u0);
#pragma unroll
        for (int u = 0; u < UPS; ++u) {
            kx[u] = make_uint4(0u, 0u, 0u, 0u);
            if (u < nu && tid < nkeys) kx[u] = __ldg(reinterpret_cast<const uint4*>(krow) + u0 + u);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                qx[i][u] = make_uint4(0u, 0u, 0u, 0u);
                if (u < nu && qrow[i]) qx[i][u] = __ldg(reinterpret_cast<const uint4*>(qrow[i]) + u0 + u);
            }
        }
    };
    bool ok = true;
    fetch(0);
    for (int s = 0; s < L.slices && ok; ++s) {
        const int bi = s & 1;
        uint8_t* buf = sm + 128 + bi * L.buf;
        uint8_t* khi = buf;
        uint8_t* klo = buf + L.kb;
        uint8_t* qhi = buf + (TF32 ? 2 : 1) * L.kb;
        uint8_t* qlo = qhi + L.qb;
        if (s >= 2) {  // the MMAs of slice s - 2 read this buffer
            const bool w = mbar_wait_bounded(&done[bi], (uint32_t)(((s - 2) >> 1) & 1), a.err);
            if (__syncthreads_or(!w)) {
                ok = false;
                break;
            }
        }
        const int nu = min(UPS, L.upr - s * UPS);  // units in this slice (even)
#pragma unroll
        for (int u = 0; u < UPS; ++u) {
            if (u >= nu) break;
            if (TF32) {
                uint4 h, l;
                split_tf32(kx[u], h, l);
                *reinterpret_cast<uint4*>(khi + u * (kMT * 16) + tid * 16) = h;
                *reinterpret_cast<uint4*>(klo + u * (kMT * 16) + tid * 16) = l;
            } else {
                *reinterpret_cast<uint4*>(khi + u * (kMT * 16) + tid * 16) = kx[u];
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int r = tid + i * kMmaNT;
                if (r >= NP) break;
                if (TF32) {
                    uint4 h, l;
                    split_tf32(qx[i][u], h, l);
                    *reinterpret_cast<uint4*>(qhi + u * (NP * 16) + r * 16) = h;
                    *reinterpret_cast<uint4*>(qlo + u * (NP * 16) + r * 16) = l;
                } else {
                    *reinterpret_cast<uint4*>(qhi + u * (NP * 16) + r * 16) = qx[i][u];
                }
            }
        }
        if (s + 1 < L.slices) fetch(s + 1);
        fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t kh = smem_u32(khi), kl = smem_u32(klo), qh = smem_u32(qhi), ql = smem_u32(qlo);
            const uint32_t lboK = kMT * 16, lboQ = (uint32_t)NP * 16;
            for (int st = 0; st < nu / 2; ++st) {  // one MMA K step = two 16-byte units
                const uint64_t aH = mma_desc(kh + 2 * st * lboK, lboK, 128);
                const uint64_t bH = mma_desc(qh + 2 * st * lboQ, lboQ, 128);
                mma_issue<TF32>(tbase, aH, bH, idesc, (s | st) ? 1u : 0u);
                if (TF32) {
                    const uint64_t aL = mma_desc(kl + 2 * st * lboK, lboK, 128);
                    const uint64_t bL = mma_desc(ql + 2 * st * lboQ, lboQ, 128);
                    mma_issue<TF32>(tbase, aH, bL, idesc, 1u);
                    mma_issue<TF32>(tbase, aL, bH, idesc, 1u);
                }
            }
            mma_commit(&done[bi]);
        }
    }
    if (ok) {  // the last commit covers every MMA issued before it
        const int sl = L.slices - 1;
        const bool w = mbar_wait_bounded(&done[sl & 1], (uint32_t)((sl >> 1) & 1), a.err);
        ok = !__syncthreads_or(!w);
    }
    tc_fence_after();

    // ---- epilogue: lane = key, columns = window rows ----
    if (ok) {
        const int kk = warp * 32 + lane;  // key within the tile
        const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);
        if (MODE == 0) {
            float* tb = reinterpret_cast<float*>(sm + L.epi);  // [32 rows][kTB]
            for (int j0 = 0; j0 < NP; j0 += 32) {
                float v[32];
                tmem_ld32(trow + (uint32_t)j0, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) tb[j * kTB + kk] = kk < nkeys ? v[j] * a.inv_sqrt_d : -INFINITY;
                __syncthreads();
                // thread t: row j = t / 4, keys (t % 4) * 32 .. + 31; four lanes combine
                const int j = tid >> 2, q4 = tid & 3;
                const float* rowv = tb + j * kTB + q4 * 32;
                float m = -FLT_MAX;  // rocket.cpp:93
#pragma unroll 8
                for (int i = 0; i < 32; ++i) m = fmaxf(m, rowv[i]);
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
                float sum = 0.0f;
#pragma unroll 8
                for (int i = 0; i < 32; ++i) sum += expf(rowv[i] - m);
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                const int r = j0 + j;
                if (q4 == 0 && r < a.R) a.tstats[(row_base + r) * a.ntiles + tile] = make_float2(m, sum);
                __syncthreads();
            }
        } else {
            const float2* rs = reinterpret_cast<const float2*>(sm + L.epi);
            float hs = 0.0f;
            for (int j0 = 0; j0 < NP; j0 += 32) {
                float v[32];
                tmem_ld32(trow + (uint32_t)j0, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int r = j0 + j;
                    if (r < a.R) {
                        const float e = expf(v[j] * a.inv_sqrt_d - rs[r].x);
                        hs = __fadd_rn(hs, __fmul_rn(e, rs[r].y));
                    }
                }
            }
            if (kk < nkeys) a.logits[((size_t)b * a.head_count + hc) * a.nk + k0 + kk] = hs;
        }
    }
    // ---- release the tensor memory on every path ----
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tbase, tcols);
    if (!ok) return;

}

// Row max M_r and 1 / (sum_r + 1e-9) from the tile statistics
// (rocket.cpp:108-113), one warp per (item, head, row): max over the tiles,
// then sum_t s_t * exp(m_t - M_r).
constexpr int kFoldRows = 8;  // rows (warps) per CTA
__global__ void __launch_bounds__(kFoldRows * 32) evict_fold_kernel(const EvictArgs a) {
    asm volatile("griddepcontrol.launch_dependents;");
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * kFoldRows + (threadIdx.x >> 5), hc = blockIdx.y, b = blockIdx.z;
    if (r >= a.R) return;  // warp-uniform
    const size_t row = ((size_t)b * a.head_count + hc) * a.R + r;
    const float2* ts = a.tstats + row * a.ntiles;
    float M = -FLT_MAX;
    for (int t = lane; t < a.ntiles; t += 32) M = fmaxf(M, ts[t].x);
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
    float S = 0.0f;
    for (int t = lane; t < a.ntiles; t += 32) {
        const float2 v = ts[t];
        S += v.y * expf(v.x - M);
    }
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) S += __shfl_xor_sync(0xffffffffu, S, x);
    if (lane == 0) a.rstats[row] = make_float2(M, 1.0f / (S + 1e-9f));
}

template <typename T>
int launch_t(const EvictArgs& a, int batch, cudaStream_t st) {
    const MmaLayout L0 = mma_layout(a.R, a.D, (int)sizeof(T), 0);
    const MmaLayout L1 = mma_layout(a.R, a.D, (int)sizeof(T), 1);
    // Resident CTAs share the SM's 512 tensor-memory columns: size the shared
    // memory so at most 512 / tcols of them fit (228 KB per SM, 1 KB reserved per CTA).
    const int tcols = L0.NP <= 32 ? 32 : L0.NP <= 64 ? 64 : L0.NP <= 128 ? 128 : 256;
    const int maxc = 512 / tcols;
    const size_t floor = (size_t)(228 * 1024) / (size_t)(maxc + 1) - 1024 + 256;
    const size_t s0 = (size_t)L0.total > floor ? (size_t)L0.total : floor;
    const size_t s1 = (size_t)L1.total > floor ? (size_t)L1.total : floor;
    auto f0 = evict_mma_kernel<T, 0>;
    auto f1 = evict_mma_kernel<T, 1>;
    if (cudaFuncSetAttribute(f0, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s0) != cudaSuccess ||
        cudaFuncSetAttribute(f1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s1) != cudaSuccess)
        return RKV_ERR_CUDA;
    dim3 grid(a.ntiles, a.head_count, batch);
    f0<<<grid, kMmaNT, s0, st>>>(a);
    if (cudaGetLastError() != cudaSuccess) return RKV_ERR_CUDA;
    if (launch_evict_fold(a, batch, st) != RKV_OK) return RKV_ERR_CUDA;
    f1<<<grid, kMmaNT, s1, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

}  // namespace

int launch_evict_fold(const EvictArgs& a, int batch, cudaStream_t st) {
    evict_fold_kernel<<<dim3((a.R + kFoldRows - 1) / kFoldRows, a.head_count, batch), kFoldRows * 32, 0, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

bool evict_mma_supported(const EvictArgs& a) {
    if (a.dtype != RKV_F32 && a.dtype != RKV_BF16) return false;
    const int es = a.dtype == RKV_F32 ? 4 : 2;
    const long long rowb = (long long)a.D * es;
    if (rowb % 32 != 0 || a.D > 256) return false;        // whole MMA K steps (32 bytes each)
    if (a.R <= 0 || a.R > 256 || a.ntiles <= 0) return false;
    if ((reinterpret_cast<uintptr_t>(a.Q) | reinterpret_cast<uintptr_t>(a.K)) & 15) return false;
    if ((a.q_stride | a.k_stride) & 15) return false;      // 16-byte row loads
    return true;
}

int launch_evict_mma(const EvictArgs& a, int batch, cudaStream_t st) {
    return a.dtype == RKV_F32 ? launch_t<float>(a, batch, st) : launch_t<uint16_t>(a, batch, st);
}

}  // namespace rkv
