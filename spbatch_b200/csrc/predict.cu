// DejaVu-style low-rank activity predictor (BASELINE north_star (1); the
// reference defines it only as PyTorch training code,
// DejaVu_predictor/main_mlp.py:137-141 and trainer_mlp.py:35-37):
//
//   hidden[t][r] = fp16( ReLU( sum_k P1[r][k] * fp16(x[t][k]) ) )   P1: [D][d]
//   logit[t][j]  =            sum_r P2[j][r] * hidden[t][r]          P2: [f][D]
//   active       = top-k of logit[t][:] (ties -> lower neuron id), or
//                  logit >= threshold (sigmoid(logit) >= 0.5 <=> logit >= 0)
//
// Index sets must be bit-exact against the CPU oracle, so every dot product
// uses one fixed fp32 order that the oracle restates: lane l of a warp
// accumulates the 8-element chunks l, l+32, l+64, ... in order with fused
// multiply-adds, then the warp adds lanes pairwise with xor-shuffles
// (offsets 16, 8, 4, 2, 1).  Floating-point addition is commutative, so
// every lane of the butterfly ends with the same value.
//
// Launches: hidden GEMV, logit GEMV (both CUDA cores, weights stream once per
// token group), per-token exact radix select that writes the reference's
// label format ([B][f] fp32, 1 = active) and the ascending index list.
#include "spb_internal.h"
#include "spb_scan.cuh"

namespace spb {

constexpr int kPredThreads = 256;
constexpr int kPredWarps = kPredThreads / 32;
constexpr int kPredTokens = 8;  // tokens per CTA (activations staged in shared memory)

// Fixed-order dot of one fp16 row (n values, n % 256 == 0) with nt vectors
// held in shared memory as fp32 (stride n); result broadcast to all lanes.
template <int NT>
__device__ __forceinline__ void fixed_dot(const __half *__restrict__ row, const float *__restrict__ vs, int n,
                                          int nt, float (&acc)[NT]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    for (int c = lane; c < n / 8; c += 32) {
        const uint4 wv = ld_stream_v4(row + (int64_t)c * 8);
        const uint32_t *pw = reinterpret_cast<const uint32_t *>(&wv);
        float w[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f2 = h2f2(pw[q]);
            w[2 * q] = f2.x;
            w[2 * q + 1] = f2.y;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < nt) {
                const float *v = vs + (int64_t)t * n + c * 8;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[t] = fmaf(w[e], v[e], acc[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
    }
}

// hidden[t][r], grid (ceil(D / rows), ceil(B / kPredTokens)).
__global__ void __launch_bounds__(kPredThreads)
pred_hidden_kernel(const __half *__restrict__ p1, const float *__restrict__ x, __half *__restrict__ hidden, int B,
                   int d, int D, int rows_per_cta) {
    extern __shared__ __align__(16) float xs[];  // [kPredTokens][d]
    const int t0 = blockIdx.y * kPredTokens, nt = min(kPredTokens, B - t0);
    for (int i = threadIdx.x; i < nt * d; i += blockDim.x)
        xs[i] = __half2float(__float2half_rn(x[(int64_t)t0 * d + i]));
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r1 = min(D, (int)(blockIdx.x + 1) * rows_per_cta);
    for (int r = blockIdx.x * rows_per_cta + warp; r < r1; r += kPredWarps) {
        float acc[kPredTokens];
        fixed_dot<kPredTokens>(p1 + (int64_t)r * d, xs, d, nt, acc);
        if (lane == 0)
            for (int t = 0; t < nt; ++t) hidden[(int64_t)(t0 + t) * D + r] = __float2half_rn(fmaxf(acc[t], 0.0f));
    }
}

// logit[t][j], grid (ceil(f / rows), ceil(B / kPredTokens)).
__global__ void __launch_bounds__(kPredThreads)
pred_logit_kernel(const __half *__restrict__ p2, const __half *__restrict__ hidden, float *__restrict__ logits, int B,
                  int D, int f, int rows_per_cta) {
    extern __shared__ __align__(16) float hs[];  // [kPredTokens][D]
    const int t0 = blockIdx.y * kPredTokens, nt = min(kPredTokens, B - t0);
    for (int i = threadIdx.x; i < nt * D; i += blockDim.x) hs[i] = __half2float(hidden[(int64_t)t0 * D + i]);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j1 = min(f, (int)(blockIdx.x + 1) * rows_per_cta);
    for (int j = blockIdx.x * rows_per_cta + warp; j < j1; j += kPredWarps) {
        float acc[kPredTokens];
        fixed_dot<kPredTokens>(p2 + (int64_t)j * D, hs, D, nt, acc);
        if (lane == 0)
            for (int t = 0; t < nt; ++t) logits[(int64_t)(t0 + t) * f + j] = acc[t];
    }
}

// Order-preserving map of an fp32 logit to an unsigned key.
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kSelThreads = 1024;

// One CTA per token.  k > 0: exact top-k (ties broken toward lower ids);
// k == 0: logit >= threshold.  Writes labels [B][f] (1.0 / 0.0), the ascending
// active list idx[t][0..count) (capacity `cap` per token) and counts[t].
__global__ void __launch_bounds__(kSelThreads)
pred_select_kernel(const float *__restrict__ logits, int f, int k, float threshold, float *__restrict__ labels,
                   int32_t *__restrict__ idx, int cap, int32_t *__restrict__ counts) {
    extern __shared__ uint32_t keys[];  // [f]
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sel_prefix, sel_mask;
    __shared__ int need;
    __shared__ int warp_tot[33];
    const int t = blockIdx.x;
    const float *lg = logits + (int64_t)t * f;
    for (int j = threadIdx.x; j < f; j += blockDim.x) keys[j] = order_key(lg[j]);
    uint32_t thr_key = 0;
    int take_eq = 0;  // how many keys equal to thr_key are active (lowest ids first)
    if (k > 0 && k < f) {
        if (threadIdx.x == 0) {
            sel_prefix = 0u;
            sel_mask = 0u;
            need = k;
        }
        __syncthreads();
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
            __syncthreads();
            const uint32_t pfx = sel_prefix, msk = sel_mask;
            for (int j = threadIdx.x; j < f; j += blockDim.x) {
                const uint32_t key = keys[j];
                if ((key & msk) == pfx) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                int rem = need;
                int b = 255;
                for (; b > 0; --b) {
                    if ((int)hist[b] >= rem) break;
                    rem -= (int)hist[b];
                }
                sel_prefix = pfx | ((uint32_t)b << shift);
                sel_mask = msk | (255u << shift);
                need = rem;
            }
            __syncthreads();
        }
        thr_key = sel_prefix;
        take_eq = need;
    }
    __syncthreads();
    // active flags in index order, then an ordered scan for the list positions
    int carry = 0, eq_seen = 0;
    for (int base = 0; base < f; base += blockDim.x) {
        const int j = base + threadIdx.x;
        const uint32_t key = j < f ? keys[j] : 0u;
        int is_eq = (k > 0 && k < f && j < f && key == thr_key) ? 1 : 0;
        // rank of this key among equal keys (by index) = eq_seen + exclusive scan
        int eq_incl = warp_incl_scan(is_eq);
        if ((threadIdx.x & 31) == 31) warp_tot[threadIdx.x >> 5] = eq_incl;
        __syncthreads();
        if (threadIdx.x < 32) {
            const int v = threadIdx.x < (int)(blockDim.x >> 5) ? warp_tot[threadIdx.x] : 0;
            const int vi = warp_incl_scan(v);
            warp_tot[threadIdx.x] = vi - v;
            if (threadIdx.x == 31) warp_tot[32] = vi;
        }
        __syncthreads();
        const int eq_rank = eq_seen + warp_tot[threadIdx.x >> 5] + eq_incl - is_eq;
        const int eq_total = warp_tot[32];
        __syncthreads();
        bool active = false;
        if (j < f) {
            if (k >= f) active = true;
            else if (k > 0) active = key > thr_key || (is_eq && eq_rank < take_eq);
            else active = lg[j] >= threshold;  // float compare: -0.0 >= 0.0 holds
            labels[(int64_t)t * f + j] = active ? 1.0f : 0.0f;
        }
        int a = active ? 1 : 0;
        int a_incl = warp_incl_scan(a);
        if ((threadIdx.x & 31) == 31) warp_tot[threadIdx.x >> 5] = a_incl;
        __syncthreads();
        if (threadIdx.x < 32) {
            const int v = threadIdx.x < (int)(blockDim.x >> 5) ? warp_tot[threadIdx.x] : 0;
            const int vi = warp_incl_scan(v);
            warp_tot[threadIdx.x] = vi - v;
            if (threadIdx.x == 31) warp_tot[32] = vi;
        }
        __syncthreads();
        const int pos = carry + warp_tot[threadIdx.x >> 5] + a_incl - a;
        if (active && idx && pos < cap) idx[(int64_t)t * cap + pos] = j;
        carry += warp_tot[32];
        eq_seen += eq_total;
        __syncthreads();
    }
    if (threadIdx.x == 0 && counts) counts[t] = carry;
}

int launch_predict(const __half *p1, const __half *p2, const float *x, int B, int d, int D, int f, int k,
                   float threshold, float *labels, int32_t *idx, int32_t *counts, float *logits, __half *hidden,
                   cudaStream_t st) {
    const int sms = num_sms();
    const int ty = (B + kPredTokens - 1) / kPredTokens;
    {
        const int ctas = max(1, (2 * sms + ty - 1) / ty);
        const int rows = (D + ctas - 1) / ctas;
        const size_t smem = sizeof(float) * kPredTokens * d;
        if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: d too large");
        if (int rc = ensure_smem((const void *)pred_hidden_kernel, smem)) return rc;
        pred_hidden_kernel<<<dim3((D + rows - 1) / rows, ty), kPredThreads, smem, st>>>(p1, x, hidden, B, d, D, rows);
        SPB_LAUNCH_CHECK("pred_hidden_kernel");
    }
    {
        const int ctas = max(1, (4 * sms + ty - 1) / ty);
        const int rows = (f + ctas - 1) / ctas;
        const size_t smem = sizeof(float) * kPredTokens * D;
        if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: D too large");
        if (int rc = ensure_smem((const void *)pred_logit_kernel, smem)) return rc;
        pred_logit_kernel<<<dim3((f + rows - 1) / rows, ty), kPredThreads, smem, st>>>(p2, hidden, logits, B, D, f,
                                                                                       rows);
        SPB_LAUNCH_CHECK("pred_logit_kernel");
    }
    {
        const size_t smem = sizeof(uint32_t) * f;
        if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: f too large");
        if (int rc = ensure_smem((const void *)pred_select_kernel, smem)) return rc;
        const int cap = k > 0 ? k : f;
        pred_select_kernel<<<B, kSelThreads, smem, st>>>(logits, f, k, threshold, labels, idx, cap, counts);
        SPB_LAUNCH_CHECK("pred_select_kernel");
    }
    return SPB_OK;
}

}  // namespace spb
