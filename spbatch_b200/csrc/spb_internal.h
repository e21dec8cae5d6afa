// Internal launch interface between the C ABI (api.cu), the reference-API
// shims (dropin.cu) and the kernels.
#pragma once

#include "spb_common.cuh"

namespace spb {

// union.cu
// Optional work folded into the union launch so the layer needs no extra
// launches: zero the fp32 output the down projection accumulates into, zero
// the cross-CTA tile counters/flags, and write the fp16 copy of x (rows padded
// with zeros to Np) that the tensor-core path reads.
struct PrepJobs {
    float *zero_out = nullptr;
    int64_t zero_n = 0;
    uint32_t *zero_u32 = nullptr;
    int64_t zero_u32_n = 0;
    const float *x = nullptr;
    __half *x16 = nullptr;
    int B = 0, Np = 0, d = 0;
};
int launch_union_bits(const float *idx, int B, int f, int G, uint32_t *tok_bits, uint32_t *seg_bits,
                      const PrepJobs &jobs, cudaStream_t st);
// union words from per-token bits [B][W] (segments of G tokens)
int launch_union_from_bits(const uint32_t *tok_in, int B, int f, int G, uint32_t *seg_bits, const PrepJobs &jobs,
                           cudaStream_t st);
int launch_compact(const uint32_t *seg_bits, int S, int f, int32_t *merge_idx, int32_t *act_cum, int32_t *counts,
                   cudaStream_t st);

// gemv.cu -- CUDA-core gather GEMV path
struct FusedGemvArgs {
    const void *wg, *wu, *wd;  // [f][d] rows, format wtype
    int wtype;
    const float *x;             // [B][d]
    int B, d, f;
    const uint32_t *seg_bits;   // [W] batch union
    const uint32_t *tok_bits;   // [B][W]
    const __half *bias_g, *bias_u;  // [f] fp16 gate / up biases, or null
    int act, per_token;
    __half *h;                  // [f][B] compacted
    int32_t *merge;             // [f] out: union ids
    int32_t *count;             // [1] out: U
    float *out;                 // [B][d], pre-zeroed
    uint32_t *err;              // [1] sticky device error code
};
int launch_fused_gemv(const FusedGemvArgs &a, cudaStream_t st);

// stream_ffn.cu -- single-launch streaming path (B <= 4): union, gather and
// down projection in one kernel
struct StreamFfnArgs {
    const void *wg, *wu, *wd;  // [f][d] rows, format wtype
    int wtype;
    const float *x;            // [B][d]
    const float *idx;          // [B][f] labels, active if > 0 (or null with tok_in)
    const uint32_t *tok_in;    // [B][W] per-token activity bits, or null
    const __half *bias_g, *bias_u;  // [f] fp16 gate / up biases, or null
    int B, d, f, act, per_token;
    int32_t *merge_out;        // [f] optional: ascending union ids
    int32_t *count_out;        // [1] optional: union size
    float *out;                // [B][d]
    uint32_t *err;             // [1] sticky device error code
    uint32_t *seg_bits;              // [W] workspace: union words
    uint32_t *tok_bits;              // [B][W] workspace: token words
    unsigned long long *grid_bar;    // workspace: grid-barrier arrival counter
    unsigned long long *launch_ctr;  // workspace: monotonic CTA ticket counter
    unsigned long long *zero_flag;   // workspace: launch number + 1 once `out` is zeroed
};
bool stream_ffn_supported(int wtype, int B, int d);
// drop-in up projection on the bulk-copy streaming design (fp16, d <= 4096)
bool dropin_up_stream_supported(int B, int d, int G);
int launch_dropin_up_stream(const __half *wg, const __half *wu, const float *x, float *gate_dst, float *up_dst,
                            const int32_t *merge_idx, const int32_t *act_cum, int B, int d, int f, int G,
                            uint32_t *err, cudaStream_t st);
int launch_stream_ffn(const StreamFfnArgs &a, cudaStream_t st);

// Drop-in (segment) variants, reference layout: compacted fp32 [B][f] with
// slot r of token t holding neuron merge_idx[(t/G)*f + r].
int launch_dropin_up(const __half *wg, const __half *wu, const float *x, float *gate_dst, float *up_dst,
                     const int32_t *merge_idx, const int32_t *act_cum, int B, int d, int f, int G, cudaStream_t st);
int launch_dropin_down(const __half *wd, const float *h, float *out, const int32_t *merge_idx,
                       const int32_t *act_cum, int B, int d, int f, int G, cudaStream_t st);

// tc_ffn.cu -- tcgen05 tensor-core path (one launch after the union)
struct TcLaunch {
    const void *wg, *wu, *wd;
    int wtype;                // SPB_W_F16 / SPB_W_Q8_0 / SPB_W_Q4_0 (row layout of wg, wu, wd)
    bool allow_dense;         // whole row ranges may stream (no compacted ids requested)
    const float *labels;      // [B][f] fp32 labels, or null when tok_in is given
    const uint32_t *tok_in;   // [B][W] per-token activity bits, or null
    const float *x;           // [B][d]
    __half *x16;              // [Np][d] workspace
    __half *h16;              // [Np][fpad] workspace
    uint32_t *seg_bits, *tok_bits;
    uint32_t *tc_bits;        // [W] union words by atomic OR, zero on entry (the launch re-zeroes them)
    float *out;
    int32_t *merge_out, *count_out;
    float *xchg;              // [grid][Np][64] partner-exchange slots
    uint32_t *ready;          // [grid / 2] per-cluster counters
    unsigned int *gbar;       // [3] per-launch counters, zero when first used
    const __half *bias_g, *bias_u;  // [f] fp16 gate / up biases, or null
    uint32_t *err;
    int B, Np, d, f, fpad, act, per_token, grid;
};
int launch_ffn_tc(const TcLaunch &L, cudaStream_t st);

// Test hooks: settable only in libraries built with SPB_DEBUG_HOOKS (through
// spb_debug_config); all zero in the product library.
struct DebugHooks {
    uint64_t timeout_ns = 0;  // bounded-wait limit of the tensor path (0: 2 s)
    int inject = 0;           // 1: the tensor path's rank-1 CTAs never signal their results
    int nkb = 0;              // tensor path: force K blocks per gate/up stage
    int stages = 0;           // tensor path: cap the ring depth
    uint32_t hint_acc = 0;    // tensor path: suspend hint of the epilogue's accumulator waits (ns)
    uint32_t hint = 0;        // tensor path: suspend hint of the ring waits (ns)
    int split_stages = 0;     // tensor path: split gate/up stages over two ring units
    int launch_flags = 0;     // tensor path, measurement only: 1 = no cooperative attribute, 2 = no
                              // programmatic dependent launch
    int dense_permille = 0;   // tensor path: union share of f (per mille) from which whole row ranges
                              // stream (0 default, above 1000 never)
};
const DebugHooks &debug_hooks();

// predict.cu -- low-rank activity predictor
// predictor scratch inside the caller's workspace
// Batches above this size take the predictor's tensor-core route (fp16 GEMMs
// with fp32 accumulation); up to it the CUDA-core kernels with one fixed
// summation order (logits and sets bit-exact against the oracle).
constexpr int kPredExactMaxBatch = 16;

struct PredScratch {
    uint32_t *hist;      // [B][2048] logit histograms (top 11 key bits)
    uint2 *cand;         // [B][f] (key, id) candidates of the threshold bin
    uint32_t *cand_cnt;  // [B]
    int2 *sel;           // [B] threshold bin, keys still needed from it
    uint32_t *bits;      // [B][W] set words when the caller wants labels only
    __half *x16;         // [B][d] fp16 activations (tensor-core route, B > kPredExactMaxBatch)
};
int launch_predict(const __half *p1, const __half *p2, const float *x, int B, int d, int D, int f, int k,
                   float threshold, float *labels, uint32_t *bits, int32_t *idx, int32_t *counts, float *logits,
                   __half *hidden, const PredScratch &scratch, cudaStream_t st);

}  // namespace spb
