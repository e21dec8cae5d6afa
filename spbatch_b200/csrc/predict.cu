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

#include <algorithm>

namespace spb {

constexpr int kPredThreads = 256;
constexpr int kPredWarps = kPredThreads / 32;
constexpr int kPredTokens = 8;  // tokens per CTA (activations staged in shared memory)

// Fixed-order dot of one fp16 row (n values, n % 256 == 0) with nt vectors
// held in shared memory as fp32 (stride n); result broadcast to all lanes.
template <int NT>
__device__ __forceinline__ void fixed_dot(const __half *__restrict__ row, const __half *__restrict__ vs, int n,
                                          int nt, float (&acc)[NT]) {
    const int lane = threadIdx.x & 31;
    constexpr int kBatch = 8;  // 16-byte loads in flight per lane (the FMA order is unchanged)
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
                    // the staged vector holds fp16 values (exact: x and hidden
                    // are fp16-rounded): one conflict-free 16-byte load per
                    // chunk, converted exactly; same FMA order
                    const uint4 hv = *reinterpret_cast<const uint4 *>(vs + (int64_t)t * n + c * 8);
                    const uint32_t *ph = reinterpret_cast<const uint32_t *>(&hv);
                    float ve[8];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float2 f2 = h2f2(ph[q]);
                        ve[2 * q] = f2.x;
                        ve[2 * q + 1] = f2.y;
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[t] = fmaf(w[e], ve[e], acc[t]);
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

// hidden[t][r], grid (ceil(D / rows), ceil(B / kPredTokens)).
__global__ void __launch_bounds__(kPredThreads)
pred_hidden_kernel(const __half *__restrict__ p1, const float *__restrict__ x, __half *__restrict__ hidden, int B,
                   int d, int D, int rows_per_cta) {
    extern __shared__ __align__(16) __half xs[];  // [kPredTokens][d], fp16-rounded x
    const int t0 = blockIdx.y * kPredTokens, nt = min(kPredTokens, B - t0);
    {  // float4 loads, several in flight per thread (d % 256 == 0)
        const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)t0 * d);
        const int n4 = nt * d / 4;
        for (int base = threadIdx.x; base < n4; base += 4 * blockDim.x) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * blockDim.x;
                v[u] = i < n4 ? __ldg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * blockDim.x;
                if (i < n4) {
                    const __half2 h0 = __floats2half2_rn(v[u].x, v[u].y), h1 = __floats2half2_rn(v[u].z, v[u].w);
                    uint2 pk;
                    pk.x = *reinterpret_cast<const uint32_t *>(&h0);
                    pk.y = *reinterpret_cast<const uint32_t *>(&h1);
                    reinterpret_cast<uint2 *>(xs)[i] = pk;
                }
            }
        }
    }
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
    extern __shared__ __align__(16) __half hs[];  // [kPredTokens][D]
    const int t0 = blockIdx.y * kPredTokens, nt = min(kPredTokens, B - t0);
    {  // 8 fp16 values per 16-byte load (D % 256 == 0)
        const uint4 *src = reinterpret_cast<const uint4 *>(hidden + (int64_t)t0 * D);
        const int n8 = nt * D / 8;
        for (int i = threadIdx.x; i < n8; i += blockDim.x) reinterpret_cast<uint4 *>(hs)[i] = __ldg(src + i);
    }
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
constexpr int kSelWarps = kSelThreads / 32;

// Exclusive block scan of one int per thread (kSelThreads threads); *total
// receives the block sum.  Two __syncthreads.
__device__ __forceinline__ int sel_block_scan(int v, int *warp_tot, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int incl = warp_incl_scan(v);
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < kSelWarps ? warp_tot[lane] : 0;
        const int wi = warp_incl_scan(w);
        warp_tot[lane] = wi - w;
        if (lane == 31) warp_tot[32] = wi;
    }
    __syncthreads();
    *total = warp_tot[32];
    return warp_tot[warp] + incl - v;
}

// One CTA per token.  k > 0: exact top-k (ties broken toward lower ids);
// k == 0: logit >= threshold.  Writes labels [B][f] (1.0 / 0.0), the ascending
// active list idx[t][0..count) (capacity `cap` per token) and counts[t].
// The threshold key is found by an 8-bit radix select (4 passes, bins
// searched by one warp with a suffix scan); then each thread owns a
// contiguous run of indices, so two block scans place the equal keys (lowest
// ids first) and the active ids in index order.
__global__ void __launch_bounds__(kSelThreads)
pred_select_kernel(const float *__restrict__ logits, int f, int k, float threshold, float *__restrict__ labels,
                   uint32_t *__restrict__ bits, int32_t *__restrict__ idx, int cap, int32_t *__restrict__ counts) {
    extern __shared__ uint32_t keys[];  // [f], then [kSelWarps][256] per-warp histograms
    uint32_t *whist = keys + ((f + 3) & ~3);
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sel_prefix, sel_mask;
    __shared__ int need;
    __shared__ int warp_tot[33];
    const int t = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *lg = logits + (int64_t)t * f;
    if ((f & 3) == 0) {  // float4 loads, four in flight per thread
        const float4 *src = reinterpret_cast<const float4 *>(lg);
        const int n4 = f >> 2;
        for (int base = threadIdx.x; base < n4; base += 4 * blockDim.x) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * blockDim.x;
                v[u] = i < n4 ? __ldg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * blockDim.x;
                if (i < n4)
                    reinterpret_cast<uint4 *>(keys)[i] =
                        make_uint4(order_key(v[u].x), order_key(v[u].y), order_key(v[u].z), order_key(v[u].w));
            }
        }
    } else {
        for (int j = threadIdx.x; j < f; j += blockDim.x) keys[j] = order_key(lg[j]);
    }
    const bool topk = k > 0 && k < f;
    if (threadIdx.x == 0) {
        sel_prefix = 0u;
        sel_mask = 0u;
        need = k;
    }
    __syncthreads();
    if (topk) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            // per-warp histograms: logits crowd into a few bins, so a shared
            // histogram would serialise the whole block on those counters
            for (int i = threadIdx.x; i < kSelWarps * 256; i += blockDim.x) whist[i] = 0u;
            __syncthreads();
            const uint32_t pfx = sel_prefix, msk = sel_mask;
            uint32_t *wh = whist + warp * 256;
            for (int j = threadIdx.x; j < f; j += blockDim.x) {
                const uint32_t key = keys[j];
                if ((key & msk) == pfx) atomicAdd(&wh[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (threadIdx.x < 256) {
                uint32_t sum = 0;
                for (int w = 0; w < kSelWarps; ++w) sum += whist[w * 256 + threadIdx.x];
                hist[threadIdx.x] = sum;
            }
            __syncthreads();
            if (warp == 0) {
                // lane l holds bins 255-8l .. 248-8l (descending); the answer is
                // the highest bin b with (count of bins > b) < need <= (count of bins >= b)
                uint32_t c[8], sum = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    c[q] = hist[255 - 8 * lane - q];
                    sum += c[q];
                }
                uint32_t incl = sum;  // inclusive scan over lanes (descending bins)
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += n;
                }
                const int rem = need;
                uint32_t before = incl - sum;  // keys in higher bins than this lane's
                int found = -1, rem_out = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (found < 0 && (int)(before + c[q]) >= rem) {
                        found = 255 - 8 * lane - q;
                        rem_out = rem - (int)before;
                    }
                    before += c[q];
                }
                const uint32_t ball = __ballot_sync(0xffffffffu, found >= 0);
                const int src = ball ? __ffs(ball) - 1 : 31;
                const int b = __shfl_sync(0xffffffffu, found >= 0 ? found : 0, src);
                const int r = __shfl_sync(0xffffffffu, rem_out, src);
                if (lane == 0) {
                    sel_prefix = pfx | ((uint32_t)b << shift);
                    sel_mask = msk | (255u << shift);
                    need = r;
                }
            }
            __syncthreads();
        }
    }
    const uint32_t thr_key = sel_prefix;
    const int take_eq = need;  // how many keys equal to thr_key are active (lowest ids first)
    // contiguous index run of this thread, whole 32-neuron words so that the
    // thread writes its bit words alone
    const int per = 32 * ((f + 32 * kSelThreads - 1) / (32 * kSelThreads));
    const int j0 = min(f, (int)threadIdx.x * per), j1 = min(f, j0 + per);
    int n_eq = 0;
    if (topk)
        for (int j = j0; j < j1; ++j) n_eq += keys[j] == thr_key;
    int tot;
    int eq_rank = sel_block_scan(n_eq, warp_tot, &tot);  // equal keys before this run
    int n_act = 0;
    for (int j = j0; j < j1; ++j) {
        bool active;
        if (k >= f) active = true;
        else if (k > 0) active = keys[j] > thr_key || (keys[j] == thr_key && eq_rank++ < take_eq);
        else active = lg[j] >= threshold;  // float compare: -0.0 >= 0.0 holds
        n_act += active;
    }
    __syncthreads();
    int pos = sel_block_scan(n_act, warp_tot, &tot);
    eq_rank -= n_eq;  // replay the same decisions, now writing
    const int W = (f + 31) / 32;
    uint32_t word = 0;
    for (int j = j0; j < j1; ++j) {
        bool active;
        if (k >= f) active = true;
        else if (k > 0) active = keys[j] > thr_key || (keys[j] == thr_key && eq_rank++ < take_eq);
        else active = lg[j] >= threshold;
        if (labels) labels[(int64_t)t * f + j] = active ? 1.0f : 0.0f;
        word |= (active ? 1u : 0u) << (j & 31);
        if (bits && ((j & 31) == 31 || j == j1 - 1)) {
            bits[(int64_t)t * W + (j >> 5)] = word;
            word = 0;
        }
        if (active) {
            if (idx && pos < cap) idx[(int64_t)t * cap + pos] = j;
            ++pos;
        }
    }
    if (threadIdx.x == 0 && counts) counts[t] = tot;
}

int launch_predict(const __half *p1, const __half *p2, const float *x, int B, int d, int D, int f, int k,
                   float threshold, float *labels, uint32_t *bits, int32_t *idx, int32_t *counts, float *logits,
                   __half *hidden, cudaStream_t st) {
    const int sms = num_sms();
    const int ty = (B + kPredTokens - 1) / kPredTokens;
    {
        // one row per warp when that fills the GPU: every row's loads are in
        // flight at once (each warp's 8 KB row is the fixed-order dot unit)
        const int ctas = max(1, (2 * sms + ty - 1) / ty);
        const int rows = std::min((D + ctas - 1) / ctas, kPredWarps);
        const size_t smem = sizeof(__half) * kPredTokens * d;
        if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: d too large");
        if (int rc = ensure_smem((const void *)pred_hidden_kernel, smem)) return rc;
        pred_hidden_kernel<<<dim3((D + rows - 1) / rows, ty), kPredThreads, smem, st>>>(p1, x, hidden, B, d, D, rows);
        SPB_LAUNCH_CHECK("pred_hidden_kernel");
    }
    {
        // at most four rows per warp: rows of D = 1024 are only 2 KB, so a
        // warp walking many of them in turn is latency-bound; more CTAs keep
        // more rows in flight (each CTA re-stages 8 x D fp16 from L2)
        const int ctas = max(1, (4 * sms + ty - 1) / ty);
        const int rows = std::min((f + ctas - 1) / ctas, 4 * kPredWarps);
        const size_t smem = sizeof(__half) * kPredTokens * D;
        if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: D too large");
        if (int rc = ensure_smem((const void *)pred_logit_kernel, smem)) return rc;
        pred_logit_kernel<<<dim3((f + rows - 1) / rows, ty), kPredThreads, smem, st>>>(p2, hidden, logits, B, D, f,
                                                                                       rows);
        SPB_LAUNCH_CHECK("pred_logit_kernel");
    }
    {
        const size_t smem = sizeof(uint32_t) * (((f + 3) & ~3) + kSelWarps * 256);
        if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: f too large");
        if (int rc = ensure_smem((const void *)pred_select_kernel, smem)) return rc;
        const int cap = k > 0 ? k : f;
        pred_select_kernel<<<B, kSelThreads, smem, st>>>(logits, f, k, threshold, labels, bits, idx, cap, counts);
        SPB_LAUNCH_CHECK("pred_select_kernel");
    }
    return SPB_OK;
}

}  // namespace spb
