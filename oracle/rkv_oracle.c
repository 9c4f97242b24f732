/*
 * rkv_oracle.c -- CPU restatement of RocketKV stage 1 and stage 2 (TEST
 * INFRASTRUCTURE; see rkv_oracle.h).  Built with -ffp-contract=off so every
 * float operation below is one IEEE-rounded operation, in the order written.
 *
 * Reference: Rishit2000/RocketKV-cpp, rocket.cpp and rocket.h.
 */
#include "rkv_oracle.h"

#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* ------------------------------------------------------------------------ */
/* Budget derivation: rocket.cpp:14-59 (all arithmetic in float, as there). */
/* ------------------------------------------------------------------------ */
void rkvo_compute_params(int token_budget, int sequence_length, int max_new_tokens,
                         int head_dim, int window_size, rkvo_budget* p) {
    p->sequence_length = sequence_length;                          /* :22 */
    p->max_new_tokens = max_new_tokens;                            /* :23 */
    p->token_budget = imin(sequence_length, token_budget);         /* :24 */
    float cr_initial = fmaxf(1.0f, (float)sequence_length / (float)p->token_budget); /* :27 */
    float alpha = fminf(0.2f + log2f(cr_initial) * 0.06f, 0.8f);   /* :30 */
    int capacity = (int)floorf((float)sequence_length / powf(cr_initial, alpha)); /* :33 */
    capacity = imax(capacity, imin(2 * max_new_tokens, sequence_length));          /* :34 */
    p->capacity_budget = capacity;
    int prompt = imin(sequence_length - max_new_tokens, capacity - max_new_tokens); /* :38 */
    prompt = imax(window_size, prompt);                            /* :39 */
    p->prompt_budget = prompt;
    p->k = imin((int)roundf((float)p->token_budget / 2.0f), capacity);             /* :43 */
    float cr2 = fmaxf(1.0f, (float)capacity / (float)p->token_budget);             /* :46 */
    p->compression_ratio = cr2;
    int chunk = imin((int)floorf(cr2), (int)ceilf(sqrtf(cr2)));    /* :50-51 */
    chunk = imax(1, chunk);
    p->chunk_size = chunk;
    p->r = imin(head_dim, imax(1, (int)roundf((float)head_dim * (float)chunk / cr2))); /* :55 */
}

/* ------------------------------------------------------------------------ */
/* exp for the stage-2 selection path, x <= 0 (the softmax argument l - max).  */
/* Method: Cody & Waite argument reduction x = n*ln2 + r, |r| <= ln2/2, with  */
/* n rounded by one fused multiply-add against 1.5*2^23, ln2 split into a     */
/* 12-bit-short head and a tail, then the degree-7 Taylor polynomial of e^r   */
/* (coefficients 1/k!) in Horner form with fused multiply-adds, then an exact */
/* two-step scaling by 2^n.  Every step is a correctly rounded IEEE operation,*/
/* so the CUDA copy of this routine returns the same bits.  Accuracy is       */
/* checked against double-precision exp in the tests.                         */
/* ------------------------------------------------------------------------ */
static float f_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }

float rkvo_expf(float x) {
    if (x != x) return x;
    if (x > 0.0f) return expf(x);  /* outside the selection's domain (x = l - max <= 0) */
    const float log2e = f_from_bits(0x3fb8aa3bu);   /* 1/ln2 rounded to float   */
    const float ln2_hi = f_from_bits(0x3f317000u);  /* ln2, low 12 bits cleared */
    const float ln2_lo = f_from_bits(0x3805fdf4u);  /* ln2 - ln2_hi, rounded    */
    const float magic = f_from_bits(0x4b400000u);   /* 1.5 * 2^23               */
    const float xc = x < -104.0f ? -104.0f : x;
    /* n = round-to-nearest-even(x * log2e): one fused multiply-add against 1.5*2^23 */
    const float t = fmaf(xc, log2e, magic);
    const float n = t - magic;
    float r = fmaf(-n, ln2_hi, xc);
    r = fmaf(-n, ln2_lo, r);
    float p = f_from_bits(0x39500d01u);             /* 1/7! */
    p = fmaf(p, r, f_from_bits(0x3ab60b61u));       /* 1/6! */
    p = fmaf(p, r, f_from_bits(0x3c088889u));       /* 1/5! */
    p = fmaf(p, r, f_from_bits(0x3d2aaaabu));       /* 1/4! */
    p = fmaf(p, r, f_from_bits(0x3e2aaaabu));       /* 1/3! */
    p = fmaf(p, r, 0.5f);                           /* 1/2! */
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    uint32_t tb;
    memcpy(&tb, &t, 4);
    const int ni = (int)tb - 0x4b400000;            /* n as an integer, -151 .. 0 */
    /* exact two-step scaling: p * 2^(n+64) is exact, * 2^-64 rounds once (subnormals too) */
    const float res = (p * f_from_bits((uint32_t)(ni + 64 + 127) << 23)) * f_from_bits(0x1f800000u);
    return x < -103.97208404541015625f ? 0.0f : res;
}

/* ------------------------------------------------------------------------ */
/* Stage 1 (rocket.cpp:61-169).                                              */
/* ------------------------------------------------------------------------ */

/* Scores and pools KV heads [h0, h0+nh): rocket.cpp:73-130. */
int rkvo_evict_pool_heads(const float* Q, const float* K, int len_q, int len_k,
                          const rkvo_config* cfg, int h0, int nh, float* pooled_out) {
    const int D = cfg->dim_head;
    const int obs_w = imin(cfg->window_size, len_q);               /* :73 */
    const int nk = len_k - obs_w;                                  /* :74 */
    const int G = cfg->num_heads / cfg->num_heads_kv;              /* :75 */
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);               /* :76 */
    const int pad = cfg->kernel_size / 2;                          /* :79 */
    if (nk < 0) return -1;
    float* head_scores = (float*)malloc(sizeof(float) * (size_t)(nk > 0 ? nk : 1));
    float* logits = (float*)malloc(sizeof(float) * (size_t)(nk > 0 ? nk : 1));
    for (int hi = 0; hi < nh; ++hi) {
        const int h_kv = h0 + hi;
        for (int k = 0; k < nk; ++k) head_scores[k] = 0.0f;
        for (int h_rel = 0; h_rel < G; ++h_rel) {                  /* :86 */
            const int h = h_kv * G + h_rel;
            for (int w = 0; w < obs_w; ++w) {                      /* :89 */
                const int q_pos = len_q - obs_w + w;
                const float* q = Q + ((size_t)h * len_q + q_pos) * D;
                float max_logit = -FLT_MAX;
                for (int k = 0; k < nk; ++k) {                     /* :97-105 */
                    const float* kp = K + ((size_t)h_kv * len_k + k) * D;
                    float dot = 0.0f;
                    for (int d = 0; d < D; ++d) dot += q[d] * kp[d];
                    logits[k] = dot * inv_sqrt_d;
                    if (logits[k] > max_logit) max_logit = logits[k];
                }
                float sum_exp = 0.0f;                              /* :108-112 */
                for (int k = 0; k < nk; ++k) {
                    logits[k] = expf(logits[k] - max_logit);
                    sum_exp += logits[k];
                }
                const float inv_sum = 1.0f / (sum_exp + 1e-9f);    /* :113 */
                for (int k = 0; k < nk; ++k) head_scores[k] += logits[k] * inv_sum; /* :114-116 */
            }
        }
        float* pooled = pooled_out + (size_t)hi * (size_t)nk;      /* :120-129 */
        for (int i = 0; i < nk; ++i) {
            float mv = -FLT_MAX;
            const int s = imax(0, i - pad), e = imin(nk - 1, i + pad);
            for (int j = s; j <= e; ++j)
                if (head_scores[j] > mv) mv = head_scores[j];
            pooled[i] = mv;
        }
    }
    free(head_scores);
    free(logits);
    return 0;
}

typedef struct { float score; int idx; } scored_t;

/* Order: score descending, index ascending (the tie rule of rocket.cpp:327-333,
 * applied here to stage 1 as well). */
static int cmp_desc_lowidx(const void* a, const void* b) {
    const scored_t* x = (const scored_t*)a;
    const scored_t* y = (const scored_t*)b;
    if (x->score != y->score) return x->score > y->score ? -1 : 1;
    return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

static int cmp_int(const void* a, const void* b) {
    int x = *(const int*)a, y = *(const int*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

static int iota_out(int* out, int n) {
    for (int i = 0; i < n; ++i) out[i] = i;
    return n;
}

/* Cross-head sum and top-k: rocket.cpp:132-168. */
int rkvo_evict_select_pooled(const float* pooled, int len_q, int len_k,
                             const rkvo_config* cfg, int* kept_out) {
    if (len_k <= cfg->prompt_budget) return iota_out(kept_out, len_k);     /* :66-71 */
    const int obs_w = imin(cfg->window_size, len_q);
    const int nk = len_k - obs_w;
    if (nk < 0) return -1;
    const int target_keep = imax(0, cfg->prompt_budget - obs_w);           /* :133 */
    if (target_keep >= nk) return iota_out(kept_out, len_k);               /* :134-138 */
    scored_t* ti = (scored_t*)malloc(sizeof(scored_t) * (size_t)nk);
    for (int i = 0; i < nk; ++i) {                                          /* :142-148 */
        float total = 0.0f;
        for (int h = 0; h < cfg->num_heads_kv; ++h) total += pooled[(size_t)h * nk + i];
        ti[i].score = total;
        ti[i].idx = i;
    }
    qsort(ti, (size_t)nk, sizeof(scored_t), cmp_desc_lowidx);              /* :150-155, ties -> lower index */
    int n = 0;
    for (int i = 0; i < target_keep; ++i) kept_out[n++] = ti[i].idx;       /* :160-162 */
    for (int i = nk; i < len_k; ++i) kept_out[n++] = i;                    /* :163-165 */
    qsort(kept_out, (size_t)n, sizeof(int), cmp_int);                      /* :166 */
    free(ti);
    return n;
}

int rkvo_prefill_eviction(const float* Q, const float* K, int len_q, int len_k,
                          const rkvo_config* cfg, int* kept_out, float* total_out) {
    if (len_k <= cfg->prompt_budget) return iota_out(kept_out, len_k);
    const int obs_w = imin(cfg->window_size, len_q);
    const int nk = len_k - obs_w;
    if (nk < 0) return -1;
    const int HK = cfg->num_heads_kv;
    float* pooled = (float*)malloc(sizeof(float) * (size_t)HK * (size_t)(nk > 0 ? nk : 1));
    rkvo_evict_pool_heads(Q, K, len_q, len_k, cfg, 0, HK, pooled);
    if (total_out) {
        for (int i = 0; i < nk; ++i) {
            float t = 0.0f;
            for (int h = 0; h < HK; ++h) t += pooled[(size_t)h * nk + i];
            total_out[i] = t;
        }
    }
    int n = rkvo_evict_select_pooled(pooled, len_q, len_k, cfg, kept_out);
    free(pooled);
    return n;
}

/* ------------------------------------------------------------------------ */
/* Stage 2 (rocket.cpp:171-382).                                             */
/* ------------------------------------------------------------------------ */

/* Sum of n values in the fixed order the GPU block uses: 256 interleaved
 * partial sums (partial j holds elements j, j+256, ... in ascending order),
 * then a halving tree (partial[j] += partial[j+s], s = 128, 64, ..., 1). */
static float canonical_sum256(const float* v, int n) {
    float part[256];
    for (int j = 0; j < 256; ++j) {
        float s = 0.0f;
        for (int c = j; c < n; c += 256) s += v[c];
        part[j] = s;
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int j = 0; j < s; ++j) part[j] = part[j] + part[j + s];
    return part[0];
}

/* Approximate page logit numerator sum_i q[R[i]] * P[i] (rocket.cpp:281-286),
 * in the fixed order the GPU uses.  The D dimensions form chunks of cd (16
 * bytes of K: 8 two-byte or 4 four-byte elements); "lane" j = 0..3 owns the
 * chunks c = j + 4 i, i = 0 .. D / cd / 4 - 1.  Per chunk: one fused
 * multiply-add chain over its selected even dimensions and one over its
 * selected odd dimensions, ascending, value = even + odd.  The lane adds its
 * chunk values pairwise (s0+s1, s2+s3, ..., then pairs of those, ...), and the
 * four lanes are added as (l0 + l2) + (l1 + l3). */
static float chunk_dot(const float* q, const int* R, const float* P, int nr, int D, int cd) {
    float pd[RKVO_MAX_D];
    unsigned char on[RKVO_MAX_D];
    for (int d = 0; d < D; ++d) on[d] = 0;
    for (int i = 0; i < nr; ++i) { on[R[i]] = 1; pd[R[i]] = P[i]; }
    const int nsl = D / cd / 4;
    float l[4];
    for (int j = 0; j < 4; ++j) {
        float sv[RKVO_MAX_D / 16];
        for (int i = 0; i < nsl; ++i) {
            const int c = j + 4 * i;
            float ev = 0.0f, od = 0.0f;
            for (int e = 0; e < cd; e += 2) {
                const int d = c * cd + e;
                if (on[d]) ev = fmaf(q[d], pd[d], ev);
                if (on[d + 1]) od = fmaf(q[d + 1], pd[d + 1], od);
            }
            sv[i] = ev + od;
        }
        for (int w = 1; w < nsl; w *= 2)
            for (int i = 0; i < nsl; i += 2 * w) sv[i] = sv[i] + sv[i + w];
        l[j] = sv[0];
    }
    return (l[0] + l[2]) + (l[1] + l[3]);
}

int rkvo_hsa_decode(const float* Q, const float* K, const float* V, int len_k,
                    int recent_window, const rkvo_config* cfg, float* O,
                    int* sel_out, int sel_stride, int* n_sel, int kv_bytes) {
    const int H = cfg->num_heads, HK = cfg->num_heads_kv, D = cfg->dim_head;
    const int G = imax(1, H / HK);                                          /* :175 */
    const int C = (cfg->chunk_size > 0) ? cfg->chunk_size                   /* :177-178 */
        : imax(1, imin((int)floorf(cfg->compression_ratio), (int)ceilf(sqrtf(cfg->compression_ratio))));
    int r = (cfg->r_dim > 0) ? cfg->r_dim                                   /* :181-183 */
        : imin(D, imax(1, (int)roundf((float)D * (float)C / cfg->compression_ratio)));
    r = imin(r, D);
    const int w = imax(0, imin(recent_window, len_k));
    const int Lc = len_k - w;                 /* tokens eligible for the top-k */
    const int final_k = imin(cfg->topk_decode, Lc);                         /* :184 */
    if (D <= 0 || D > RKVO_MAX_D || D % 64 != 0 || (kv_bytes != 2 && kv_bytes != 4)) return -1;
    memset(O, 0, sizeof(float) * (size_t)H * D);                            /* :185 */
    if (n_sel) for (int h = 0; h < HK; ++h) n_sel[h] = 0;
    if (len_k <= 0) return 0;                                               /* :186 */
    if (final_k <= 0 && w == 0) return 0;
    const int nchunks = final_k > 0 ? (Lc + C - 1) / C : 0;                 /* :180 */
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);                        /* :188 */

    float* sabs = (float*)malloc(sizeof(float) * D);
    float* qsum = (float*)malloc(sizeof(float) * D);
    float* sum_all = (float*)malloc(sizeof(float) * G);
    float* sum_kept = (float*)malloc(sizeof(float) * G);
    float* cscale = (float*)malloc(sizeof(float) * G);
    int* R = (int*)malloc(sizeof(int) * D);
    float* P = (float*)malloc(sizeof(float) * D);
    float* logit = (float*)malloc(sizeof(float) * (size_t)G * (nchunks > 0 ? nchunks : 1));
    float* gp = (float*)malloc(sizeof(float) * (nchunks > 0 ? nchunks : 1));
    scored_t* order = (scored_t*)malloc(sizeof(scored_t) * (nchunks > 0 ? nchunks : 1));
    unsigned char* take = (unsigned char*)malloc((size_t)(len_k > 0 ? len_k : 1));
    int* sel = (int*)malloc(sizeof(int) * (size_t)len_k);
    float* es = (float*)malloc(sizeof(float) * (size_t)len_k);

    for (int h_kv = 0; h_kv < HK; ++h_kv) {                                 /* :191 */
        const float* kb = K + (size_t)h_kv * len_k * D;
        const float* vb = V + (size_t)h_kv * len_k * D;
        const float* qg = Q + (size_t)h_kv * G * D;
        float* og = O + (size_t)h_kv * G * D;
        int ns = 0;
        memset(take, 0, (size_t)len_k);

        if (final_k > 0) {
            for (int h = 0; h < G; ++h) sum_all[h] = 0.0f;                  /* :197-214 */
            for (int d = 0; d < D; ++d) {
                float sa = 0.0f, sv = 0.0f;
                for (int h = 0; h < G; ++h) {
                    const float qv = qg[h * D + d];
                    const float av = fabsf(qv);
                    sa += av;
                    sv += qv;
                    sum_all[h] += av;
                }
                sabs[d] = sa;
                qsum[d] = sv;
            }
            /* top-r dimensions (:222-244), listed in ascending order */
            int nr = 0;
            for (int d = 0; d < D; ++d) {
                int rank = 0;
                for (int e = 0; e < D; ++e)
                    if (sabs[e] > sabs[d] || (sabs[e] == sabs[d] && e < d)) ++rank;
                if (r >= D || rank < r) R[nr++] = d;
            }
            for (int h = 0; h < G; ++h) {
                if (r >= D) { sum_kept[h] = sum_all[h]; continue; }         /* :230 */
                float s = 0.0f;
                for (int i = 0; i < nr; ++i) s += fabsf(qg[h * D + R[i]]);  /* :239-242 */
                sum_kept[h] = s;
            }
            for (int h = 0; h < G; ++h)                                     /* :246-250 */
                cscale[h] = sqrtf((float)D * (sum_kept[h] / (sum_all[h] + 1e-9f)));

            /* chunk representatives and approximate logits (:252-289) */
            for (int c = 0; c < nchunks; ++c) {
                const int t0 = c * C, t1 = imin(t0 + C, Lc);
                for (int i = 0; i < nr; ++i) {
                    const int d = R[i];
                    if (qsum[d] >= 0.0f) {                                  /* sign >= 0 */
                        float mv = -FLT_MAX;
                        for (int t = t0; t < t1; ++t) if (kb[(size_t)t * D + d] > mv) mv = kb[(size_t)t * D + d];
                        P[i] = mv;
                    } else {
                        float mv = FLT_MAX;
                        for (int t = t0; t < t1; ++t) if (kb[(size_t)t * D + d] < mv) mv = kb[(size_t)t * D + d];
                        P[i] = mv;
                    }
                }
                for (int h = 0; h < G; ++h)
                    logit[(size_t)h * nchunks + c] = chunk_dot(qg + (size_t)h * D, R, P, nr, D, 16 / kv_bytes) / cscale[h];
            }
            /* per-head softmax over chunks (:291-309), then the group sum (:311-323) */
            for (int c = 0; c < nchunks; ++c) gp[c] = 0.0f;
            for (int h = 0; h < G; ++h) {
                float* lh = logit + (size_t)h * nchunks;
                float mx = -FLT_MAX;
                for (int c = 0; c < nchunks; ++c) if (lh[c] > mx) mx = lh[c];
                for (int c = 0; c < nchunks; ++c) lh[c] = rkvo_expf(lh[c] - mx);
                const float inv = 1.0f / (canonical_sum256(lh, nchunks) + 1e-9f);
                for (int c = 0; c < nchunks; ++c) lh[c] = lh[c] * inv;
            }
            for (int c = 0; c < nchunks; ++c) {
                float g = 0.0f;
                for (int h = 0; h < G; ++h) g += logit[(size_t)h * nchunks + c];
                gp[c] = g;
                order[c].score = g;
                order[c].idx = c;
            }
            /* token top-k: score descending, index ascending (:325-340) */
            qsort(order, (size_t)nchunks, sizeof(scored_t), cmp_desc_lowidx);
            int need = final_k;
            for (int i = 0; i < nchunks && need > 0; ++i) {
                const int t0 = order[i].idx * C, t1 = imin(t0 + C, Lc);
                for (int t = t0; t < t1 && need > 0; ++t) { take[t] = 1; --need; }
            }
        }
        for (int t = Lc; t < len_k; ++t) take[t] = 1;                       /* recent window */
        for (int t = 0; t < len_k; ++t) if (take[t]) sel[ns++] = t;         /* :340, sorted */
        if (sel_out) memcpy(sel_out + (size_t)h_kv * sel_stride, sel, sizeof(int) * (size_t)ns);
        if (n_sel) n_sel[h_kv] = ns;

        /* exact attention over the selected tokens (:342-378) */
        for (int h = 0; h < G; ++h) {
            const float* qh = qg + (size_t)h * D;
            float* oh = og + (size_t)h * D;
            for (int d = 0; d < D; ++d) oh[d] = 0.0f;
            float mx = -FLT_MAX;
            for (int i = 0; i < ns; ++i) {
                const float* kt = kb + (size_t)sel[i] * D;
                float dot = 0.0f;
                for (int d = 0; d < D; ++d) dot += qh[d] * kt[d];
                es[i] = dot * inv_sqrt_d;
                if (es[i] > mx) mx = es[i];
            }
            float se = 0.0f;
            for (int i = 0; i < ns; ++i) { es[i] = expf(es[i] - mx); se += es[i]; }
            const float inv = 1.0f / (se + 1e-9f);
            for (int i = 0; i < ns; ++i) {
                const float pr = es[i] * inv;
                const float* vt = vb + (size_t)sel[i] * D;
                for (int d = 0; d < D; ++d) oh[d] += pr * vt[d];
            }
        }
    }
    free(sabs); free(qsum); free(sum_all); free(sum_kept); free(cscale); free(R); free(P);
    free(logit); free(gp); free(order); free(take); free(sel); free(es);
    return 0;
}
