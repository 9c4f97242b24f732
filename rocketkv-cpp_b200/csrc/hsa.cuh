// hsa.cuh -- stage-2 hybrid sparse decode arguments and launcher (see hsa.cu).
#pragma once

#include "rkv_common.cuh"

namespace rkv {

struct HsaArgs {
    const uint8_t* Q;
    const uint8_t* K;
    const uint8_t* V;
    long long q_stride, kv_stride;  // bytes between items
    int len_k, H, HK, G, D;
    int C;          // chunk (page) size
    int r;          // query dimensions kept
    int w;          // recent window (tokens always attended)
    int Lc;         // len_k - w: tokens eligible for the top-k
    int final_k;    // min(topk, Lc)
    int nchunks;    // ceil(Lc / C) when the page scoring runs, else 0
    int head_begin, head_count;
    int sel_stride;
    float inv_sqrt_d;
    float* O;        // [batch][H][D]
    int* sel;        // [batch][head_count][sel_stride]
    int* n_sel;      // nullable [batch][head_count]
    float* wlogits;  // workspace [batch][head_count][G][nchunks]
    float* wscore;   // workspace [batch][head_count][G][score_stride]: attention scores / p
    int score_stride;
    int* err;        // workspace error word
    // launch plan, filled by the launcher
    int splits;           // scan CTAs per unit
    int pages_per_split;  // pages each scan CTA covers
    int stage_rows;       // rows per scan stage
    int carry_mode;       // a page spans more than one scan stage
    int pps;              // pages per scan stage (not carry mode)
    int wg;               // consumer warps per stage (a group)
    int ngrp;             // groups, taking stages in turn
    int nstage;           // scan ring stages
    int tail_r0_bytes;    // attention-kernel shared memory for the merge buffer
    int nch_pad;          // row stride of the page logits (nchunks rounded up to 4)
    // page summaries (nullable): per (item, KV head) [2][D][npp] values of the K type, the
    // NaN-ignoring max over a page's rows of x and of -x; the scan then reads these instead of K
    const uint8_t* summary;
    long long sum_stride;  // bytes between items
    long long sum_mask_off;  // bytes from an item's summaries to its non-finite masks
    int npp;               // pages per summary row (nchunks rounded up to 8)
};

// Page-summary geometry for (cfg, len_k, recent_window): pages per row and bytes per item.
struct HsaSummaryShape {
    int C, Lc, nchunks, npp;
    long long mask_off;    // bytes from an item's start to its masks: [KV head][D / 32] words, after the extrema
    long long item_bytes;  // extrema [KV head][2][D][npp], then the masks (16-byte multiple)
};
HsaSummaryShape hsa_summary_shape(const rkv_config& c, int dtype, int len_k, int recent_window);
int launch_hsa_summary_build(const uint8_t* K, int dtype, int D, int HK, int len_k, long long kv_stride,
                             const HsaSummaryShape& s, uint8_t* summary, int batch, cudaStream_t st);

struct HsaShape {
    int G, C, r, w, Lc, final_k, nchunks, nch_pad, sel_cap;
    size_t off_logits, off_sel, off_scores, ws_bytes;
};

HsaShape hsa_shape(const rkv_config& c, int len_k, int recent_window, int batch, int head_count);
int hsa_check_supported(const rkv_config& c, int dtype);
int launch_hsa(HsaArgs a, int dtype, int batch, cudaStream_t st);

}  // namespace rkv
