// ovf_gemv.cuh — the quantized decode GEMV (launch parameters and host API).
//
// One kernel streams Q4_K (144 B), Q6_K (210 B) and Q8_0 (int8 + fp32 scale)
// weight rows from HBM with 1-D bulk copies (the TMA engine) into a ring of
// shared-memory stages, contracts them with a Q8_K / Q8_0 activation held in
// shared memory using dp4a, and sums each row's super-block terms in
// ascending order so the result is bit-identical to the reference's
// sequential fp32 accumulation.  Fused prologues (RMSNorm + activation
// quantization) and epilogues (bias, residual add, SiLU*up, logits+argmax)
// remove the separate elementwise launches of a decode step.
#pragma once

#include "ovf_common.cuh"

namespace ovf {

enum ActMode : int {
    ACT_PREQ_Q8K = 0,  // Q8_K activation given in global memory (ProjectPreQuantized)
    ACT_F32 = 1,       // fp32 x, quantized inside every CTA (ProjectParallel)
    ACT_F32_RMSNORM = 2,  // fp32 x -> (x * norm_scale) * gamma -> quantized
};

enum EpiMode : int {
    EPI_STORE = 0,          // out[row] = bias + sum
    EPI_RESIDUAL = 1,       // out[row] = resid[row] + (bias + sum)
    EPI_SILU_PAIR = 2,      // seg0 = gate, seg1 = up: out[row] = silu(gate)*up
    EPI_LOGITS_ARGMAX = 3,  // out[row] = sum; greedy argmax tracked in DevStep
    // tensor-parallel epilogues: results go to the exchange buffer of every
    // rank (tp_dst[w], w < tp_world) instead of out
    EPI_GROUPS_TP = 4,      // Q8_0 groups (heads): dst[(tp_index0 + group) * tp_rows + row] = group sum
    EPI_TERMS_TP = 5,       // every block's term: dst[(tp_index0 + block) * tp_rows + row]
    EPI_LOGITS_TP = 6,      // dst[tp_index0 + row] = sum; the rank's argmax key goes to tp_keys[w][tp_rank]
    EPI_ROWS_TP = 7,        // dst[tp_index0 * tp_rows + row] = bias + sum (an expert's output for every rank)
};

// Device-resident per-session step state (greedy loop without host syncs).
struct DevStep {
    unsigned long long argmax_key;  // (orderable logit << 32) | ~index
    int done_ctas;                  // last-CTA ticket of the logits kernel
    int token;                      // token fed to the next step
    int cur_pos;                    // position being decoded
    int next_pos;                   // position of the next token
    int n_generated;
    int pad[3];
};

// Bit pattern of "not written yet" in a residual output whose RMSNorm is
// formed on the fly (a NaN payload that no arithmetic on finite values
// produces).
static constexpr uint32_t kNormSentinel = 0x7FBADBADu;

struct GemvSeg {
    const uint8_t *w;    // K-quant blocks, or Q8_0 int8 quants
    const float *ws;     // Q8_0 fp32 scales [rows x K/32]
    const float *bias;   // optional
    float *out;
    int type;
    int rows;
    int groups;          // row tiles in this segment
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg;
    int K;
    int rows_per_group;  // T: rows per tile (T/2 gate + T/2 up rows in pair mode)
    int stages;
    int q8_group;        // Q8_0 blocks per summation group (== K/32 when ungrouped)
    int act_mode;
    int epi;
    int pair;            // EPI_SILU_PAIR: seg0 = gate, seg1 = up, same row groups
    int total_groups;    // row tiles over all segments
    const float *x;
    const float *gamma;
    float eps;
    const int8_t *aq;    // ACT_PREQ_Q8K
    const float *as;
    const int16_t *ab;
    int8_t *aq_out;      // optional copy of the quantized activation (CTA 0)
    float *as_out;
    int16_t *ab_out;
    const float *norm_scale;  // ACT_F32_RMSNORM: RMSNorm scale of x, computed by its producer
    const float *resid;
    float *norm_out;     // EPI_RESIDUAL: also produce the RMSNorm scale of the output (eps); the
                         // output must hold kNormSentinel when the launch starts
    float *fill_sentinel;  // optional: buffer to fill with kNormSentinel (for a later launch)
    int fill_n;
    DevStep *step;       // EPI_LOGITS_ARGMAX
    int *tokens_out;     // EPI_LOGITS_ARGMAX: generated token log (optional)
    const int *expert_sel;  // routed expert: segment weights are offset by expert_sel[expert_slot] * stride
    int expert_slot;        // (read after griddepcontrol.wait; no weight is staged before it)
    float *tp_dst[8];       // EPI_*_TP: every rank's exchange buffer (peer pointers)
    unsigned long long *tp_keys[8];  // EPI_LOGITS_TP: every rank's argmax key table
    int tp_world, tp_rank, tp_index0, tp_rows;
    int64_t expert_wstride;  // bytes between experts' quants
    int64_t expert_sstride;  // bytes between experts' Q8_0 scales
    int expert_mod, expert_rank;  // expert parallel (mod > 1): run only if expert % mod == rank, as local
                                  // expert expert / mod; other ranks' CTAs leave at once
    L2Prefetch pf;       // weights of a later launch to pull into L2 once this one's are issued
    TraceSlot *trace;    // OVF_TRACE timeline slot, or null
};

struct GemvPlan {
    int rows_per_tile, stages, warps, grid;
    size_t smem;
};

// Host launcher.  Validates the shape combination, plans tiles/stages from
// the device's SM count and shared memory, and launches with PDL.
ovf_status gemv_launch(GemvParams p, cudaStream_t stream, bool pdl, GemvPlan *plan_out = nullptr);

int block_bytes(int type);  // bytes per 256 (K-quant) or per 32 (Q8_0: 32 + 4)

}  // namespace ovf
