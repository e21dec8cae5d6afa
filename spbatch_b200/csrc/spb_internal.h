// Internal launch interface between the C ABI (api.cu), the reference-API
// shims (dropin.cu) and the kernels.
#pragma once

#include "spb_common.cuh"

namespace spb {

// union.cu
int launch_union_bits(const float *idx, int B, int f, int G, uint32_t *tok_bits, uint32_t *seg_bits,
                      float *zero_out, int64_t zero_n, cudaStream_t st);
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
    int act, per_token;
    __half *h;                  // [f][B] compacted
    int32_t *merge;             // [f] out: union ids
    int32_t *count;             // [1] out: U
    float *out;                 // [B][d], pre-zeroed
};
int launch_fused_gemv(const FusedGemvArgs &a, cudaStream_t st);

// Drop-in (segment) variants, reference layout: compacted fp32 [B][f] with
// slot r of token t holding neuron merge_idx[(t/G)*f + r].
int launch_dropin_up(const __half *wg, const __half *wu, const float *x, float *gate_dst, float *up_dst,
                     const int32_t *merge_idx, const int32_t *act_cum, int B, int d, int f, int G, cudaStream_t st);
int launch_dropin_down(const __half *wd, const float *h, float *out, const int32_t *merge_idx,
                       const int32_t *act_cum, int B, int d, int f, int G, cudaStream_t st);

}  // namespace spb
