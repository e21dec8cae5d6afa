// Weight-row formats and the in-register dequantisation shared by the
// gather kernels and spb_dequantize_rows.
#pragma once

#include "spb_common.cuh"

namespace spb {

template <int WT>
__host__ __device__ constexpr int64_t row_bytes_of(int d) {
    return WT == SPB_W_F16 ? (int64_t)d * 2 : (WT == SPB_W_Q8_0 ? (int64_t)d + d / 16 : (int64_t)d / 2 + d / 16);
}

// Eight consecutive dequantised weights starting at element e (e % 8 == 0).
template <int WT>
__device__ __forceinline__ void fetch8(const uint8_t *__restrict__ row, int d, int e, float (&w)[8]) {
    if (WT == SPB_W_F16) {
        const uint4 v = ld_stream_v4(row + (int64_t)e * 2);
        const uint32_t *pv = reinterpret_cast<const uint32_t *>(&v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f2 = h2f2(pv[q]);
            w[2 * q] = f2.x;
            w[2 * q + 1] = f2.y;
        }
    } else if (WT == SPB_W_Q8_0) {
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(row + e));
        const float sc = __half2float(__ldg(reinterpret_cast<const __half *>(row + d) + e / 32));
        const int8_t *q = reinterpret_cast<const int8_t *>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (float)q[i] * sc;
    } else {
        const int b = e >> 5, o = e & 31;
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(row + b * 16 + (o & 15)));
        const float sc = __half2float(__ldg(reinterpret_cast<const __half *>(row + d / 2) + b));
        const uint8_t *q = reinterpret_cast<const uint8_t *>(&v);
        const int sh = o < 16 ? 0 : 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (float)((int)((q[i] >> sh) & 15) - 8) * sc;
    }
}

// Eight consecutive dequantised weights of chunk c (elements 8c..8c+7) of a
// row staged in shared memory; the same arithmetic as fetch8.
template <int WT>
__device__ __forceinline__ void deq8_smem(const uint8_t *row, int d, int c, float (&w)[8]) {
    if (WT == SPB_W_F16) {
        const uint4 v = *reinterpret_cast<const uint4 *>(row + (int64_t)c * 16);
        const uint32_t *pv = reinterpret_cast<const uint32_t *>(&v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f2 = h2f2(pv[q]);
            w[2 * q] = f2.x;
            w[2 * q + 1] = f2.y;
        }
    } else if (WT == SPB_W_Q8_0) {
        const uint2 v = *reinterpret_cast<const uint2 *>(row + c * 8);
        const float sc = __half2float(reinterpret_cast<const __half *>(row + d)[c >> 2]);
        const int8_t *q = reinterpret_cast<const int8_t *>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (float)q[i] * sc;
    } else {
        const int b = c >> 2, o = (c & 3) * 8;
        const uint2 v = *reinterpret_cast<const uint2 *>(row + b * 16 + (o & 15));
        const float sc = __half2float(reinterpret_cast<const __half *>(row + d / 2)[b]);
        const uint8_t *q = reinterpret_cast<const uint8_t *>(&v);
        const int sh = o < 16 ? 0 : 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (float)((int)((q[i] >> sh) & 15) - 8) * sc;
    }
}

}  // namespace spb
