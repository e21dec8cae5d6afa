// ggml Q8_0 / Q4_0 weight preparation (host) and a device dequantisation
// entry point that runs the gather kernels' own in-register decoding.
//
// Block formats as named by the benchmark definition (ggml; not vendored by
// the reference, whose only block-format fact is the half-block nibble
// placement of cuda/kernel.cu:348,354-355):
//   Q8_0: 32-element blocks, scale = absmax / 127 (fp16), q = round(x / scale)
//   Q4_0: 32-element blocks, m = element of largest magnitude (sign kept),
//         scale = m / -8 (fp16), q = min(15, (int)(x / scale + 8.5)); byte j of
//         the block holds element j (low nibble) and j + 16 (high nibble)
// Row layout ("split"): all quant bytes of the row, then its fp16 scales, so
// every row starts 16-byte aligned when d % 256 == 0.
#include <cmath>
#include <cstring>

#include "spb_internal.h"
#include "spb_quant.cuh"

namespace spb {

__global__ void dequant_rows_kernel(const uint8_t *__restrict__ q, int wtype, int rows, int d, float *__restrict__ out) {
    const int64_t n8 = (int64_t)rows * (d / 8);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / (d / 8)), e = (int)(i % (d / 8)) * 8;
        float w[8];
        if (wtype == SPB_W_Q8_0) fetch8<SPB_W_Q8_0>(q + r * row_bytes_of<SPB_W_Q8_0>(d), d, e, w);
        else if (wtype == SPB_W_Q4_0) fetch8<SPB_W_Q4_0>(q + r * row_bytes_of<SPB_W_Q4_0>(d), d, e, w);
        else fetch8<SPB_W_F16>(q + r * row_bytes_of<SPB_W_F16>(d), d, e, w);
#pragma unroll
        for (int k = 0; k < 8; ++k) out[(int64_t)r * d + e + k] = w[k];
    }
}

static void quantize_block_q8(const float *x, int8_t *q, __half *s) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
    const float dd = amax / 127.0f;
    const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
    for (int i = 0; i < 32; ++i) q[i] = (int8_t)std::lround(x[i] * id);
    *s = __float2half_rn(dd);
}

static void quantize_block_q4(const float *x, uint8_t *q, __half *s) {
    float amax = 0.0f, m = 0.0f;
    for (int i = 0; i < 32; ++i)
        if (std::fabs(x[i]) > amax) {
            amax = std::fabs(x[i]);
            m = x[i];
        }
    const float dd = m / -8.0f;
    const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
    for (int j = 0; j < 16; ++j) {
        int q0 = (int)(x[j] * id + 8.5f), q1 = (int)(x[j + 16] * id + 8.5f);
        q0 = q0 > 15 ? 15 : q0;
        q1 = q1 > 15 ? 15 : q1;
        q[j] = (uint8_t)(q0 | (q1 << 4));
    }
    *s = __float2half_rn(dd);
}

}  // namespace spb

extern "C" {

int64_t spb_weight_row_bytes(int wtype, int d) {
    using namespace spb;
    if (d <= 0 || d % 32) return -1;
    switch (wtype) {
        case SPB_W_F16: return row_bytes_of<SPB_W_F16>(d);
        case SPB_W_Q8_0: return row_bytes_of<SPB_W_Q8_0>(d);
        case SPB_W_Q4_0: return row_bytes_of<SPB_W_Q4_0>(d);
        default: return -1;
    }
}

int spb_quantize(const float *w, int rows, int d, int wtype, uint8_t *out) {
    using namespace spb;
    if (!w || !out || rows <= 0 || d <= 0 || d % 32) return fail(SPB_ERR_INVALID, "spb_quantize: bad arguments");
    if (wtype != SPB_W_Q8_0 && wtype != SPB_W_Q4_0) return fail(SPB_ERR_INVALID, "spb_quantize: Q8_0 or Q4_0 only");
    const int64_t rb = spb_weight_row_bytes(wtype, d);
    const int64_t qb = wtype == SPB_W_Q8_0 ? d : d / 2;
    for (int r = 0; r < rows; ++r) {
        const float *x = w + (int64_t)r * d;
        uint8_t *row = out + r * rb;
        __half *sc = reinterpret_cast<__half *>(row + qb);
        for (int b = 0; b < d / 32; ++b) {
            if (wtype == SPB_W_Q8_0)
                quantize_block_q8(x + b * 32, reinterpret_cast<int8_t *>(row) + b * 32, sc + b);
            else
                quantize_block_q4(x + b * 32, row + b * 16, sc + b);
        }
    }
    return SPB_OK;
}

int spb_dequantize_rows(const void *q, int wtype, int rows, int d, float *out, void *stream) {
    using namespace spb;
    if (!q || !out || rows <= 0 || d <= 0 || d % 256) return fail(SPB_ERR_INVALID, "spb_dequantize_rows: bad arguments");
    if (wtype != SPB_W_F16 && wtype != SPB_W_Q8_0 && wtype != SPB_W_Q4_0)
        return fail(SPB_ERR_INVALID, "spb_dequantize_rows: unknown weight type");
    dequant_rows_kernel<<<2 * num_sms(), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t *>(q), wtype, rows, d, out);
    SPB_LAUNCH_CHECK("dequant_rows_kernel");
    return SPB_OK;
}

}  // extern "C"
