// Device helpers shared by the predictor kernels (predict.cu) and the
// streaming FFN kernel's predictor-fused mode (stream_ffn.cu): the
// fixed-order dot products that keep the predicted sets bit-exact against
// the CPU oracle, and the order key of the logit histogram.
#pragma once

#include "spb_common.cuh"

namespace spb {

constexpr int kHistBins = 2048;  // logit histogram: the top 11 bits of the order key

// Mixed-precision FMA (sm_100): fp16 operands, fp32 addend and result, one
// rounding -- the value fmaf((float)a, (float)b, c) gives, without the two
// conversions.  fma2_lohi adds the low pair, then the high pair.
__device__ __forceinline__ float fma2_lohi(uint32_t a, uint32_t b, float c) {
    asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %1;\n\t"
        "mov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
        : "+f"(c)
        : "r"(a), "r"(b));
    return c;
}

// Fixed-order dot of one fp16 row (n values, n % 256 == 0) with nt vectors
// held in shared memory as fp32 (stride n); result broadcast to all lanes.
template <int NT, int kBatch = 8>  // kBatch: 16-byte loads in flight per lane (the FMA order is unchanged)
__device__ __forceinline__ void fixed_dot(const __half *__restrict__ row, const __half *__restrict__ vs, int n,
                                          int nt, float (&acc)[NT]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    const int nch = n / 8;
    for (int c0 = lane; c0 < nch; c0 += 32 * kBatch) {
        uint4 wv[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int c = c0 + u * 32;
            wv[u] = c < nch ? ld_stream_v4(row + (int64_t)c * 8) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int c = c0 + u * 32;
            if (c >= nch) break;
            const uint32_t *pw = reinterpret_cast<const uint32_t *>(&wv[u]);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < nt) {
                    // the staged vector holds fp16 values (exact: x and hidden
                    // are fp16-rounded): one conflict-free 16-byte load per
                    // chunk; elements in order, fp16 x fp16 + fp32
                    const uint4 hv = *reinterpret_cast<const uint4 *>(vs + (int64_t)t * n + c * 8);
                    const uint32_t *ph = reinterpret_cast<const uint32_t *>(&hv);
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[t] = fma2_lohi(pw[q], ph[q], acc[t]);
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
    }
}

// Order-preserving map of an fp32 logit to an unsigned key.
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Fixed-order dot of R shared-memory rows (rows, rows + n, ...) with one
// shared-memory vector: the order of fixed_dot per row (lane l takes the
// 8-element chunks l, l + 32, ... in turn, elements in order, then the xor
// butterfly), the rows' FMA chains interleaved.
template <int R>
__device__ __forceinline__ void fixed_dot_smem_rows(const __half *rows, const __half *v, int n, float (&acc)[R]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    const int nch = n / 8;
    for (int c = lane; c < nch; c += 32) {
        const uint4 hv = *reinterpret_cast<const uint4 *>(v + c * 8);
        const uint32_t *ph = reinterpret_cast<const uint32_t *>(&hv);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(rows + (size_t)r * n + c * 8);
            const uint32_t *pw = reinterpret_cast<const uint32_t *>(&wv);
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[r] = fma2_lohi(pw[q], ph[q], acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
}

}  // namespace spb
