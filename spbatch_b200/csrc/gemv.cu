// CUDA-core gather GEMV path (small batches).
//
// gate/up: one warp per active neuron.  Each lane streams 16-byte chunks of
// the neuron's W_gate and W_up rows (ld.global.nc, no L1 allocation), FMAs
// them in fp32 against the fp16-rounded activations held in shared memory,
// and the warp reduces with xor-shuffles.  The fused epilogue applies
// ReLU(gate)*up (or the dReLU variant), the per-token mask, rounds h to fp16
// and stores it compacted.  This replaces mm_up + relu_and_mul_f32 +
// convert_fp32_to_fp16 of the reference (cuda/kernel.cu:595-704, 522-529,
// 321-356) for B <= 4, where tensor-core tiles would be mostly padding.
//
// down: CTAs tile (2048-column slice of d) x (slice of the active list); each
// thread owns 8 output columns and streams the 16-byte chunk of every active
// W_down row (stored [f][d], so the d x f "column gather" is a row gather)
// into 8*NT fp32 accumulators, then adds its partial sums into the
// pre-zeroed output with vector atomics.  This replaces mm_down
// (cuda/kernel.cu:706-816), whose 16 CTAs per 8 tokens cannot fill 148 SMs.
//
// Work is split by position in the compacted list, so every CTA gets the same
// number of rows whatever the union size; the union size never reaches the
// host.
#include "spb_internal.h"
#include "spb_scan.cuh"
#include "spb_quant.cuh"

namespace spb {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvUnroll = 4;  // 16-byte chunks in flight per row per lane

// Accumulates NT dot products of the fp16 row `w` (d values) with xs[t][0..d)
// into acc[t] (per-lane partial sums; caller reduces across the warp).
template <int NT>
__device__ __forceinline__ void row_dot2(const __half *__restrict__ rg, const __half *__restrict__ ru,
                                         const float *__restrict__ xs, int d, float (&ag)[NT], float (&au)[NT]) {
    const int lane = threadIdx.x & 31;
    const int nch = d >> 3;
    for (int c0 = 0; c0 < nch; c0 += 32 * kGemvUnroll) {
        uint4 vg[kGemvUnroll], vu[kGemvUnroll];
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            const int c = c0 + u * 32 + lane;
            if (c < nch) {
                vg[u] = ld_stream_v4(rg + (int64_t)c * 8);
                if (ru) vu[u] = ld_stream_v4(ru + (int64_t)c * 8);
            }
        }
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            const int c = c0 + u * 32 + lane;
            if (c < nch) {
                float wg[8], wu[8];
                const uint32_t *pg = reinterpret_cast<const uint32_t *>(&vg[u]);
                const uint32_t *pu = reinterpret_cast<const uint32_t *>(&vu[u]);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float2 a = h2f2(pg[q]);
                    wg[2 * q] = a.x;
                    wg[2 * q + 1] = a.y;
                    if (ru) {
                        float2 b = h2f2(pu[q]);
                        wu[2 * q] = b.x;
                        wu[2 * q + 1] = b.y;
                    }
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const float4 *xp = reinterpret_cast<const float4 *>(xs + (int64_t)t * d + c * 8);
                    const float4 x0 = xp[0], x1 = xp[1];
                    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) ag[t] = fmaf(wg[k], xv[k], ag[t]);
                    if (ru) {
#pragma unroll
                        for (int k = 0; k < 8; ++k) au[t] = fmaf(wu[k], xv[k], au[t]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        ag[t] = warp_sum(ag[t]);
        if (ru) au[t] = warp_sum(au[t]);
    }
}

// Loads tokens [t0, t0 + NT) of x (rows of d fp32) into shared memory rounded
// to fp16 (the reference converts x to fp16 before its products,
// cuda/kernel.cu:978); tokens >= B are zero.  float4 loads, eight in flight
// per thread (d % 4 == 0: rows stay 16-byte aligned).
template <int NT>
__device__ __forceinline__ void load_x_rounded(const float *__restrict__ x, int B, int t0, int d, float *xs) {
    const int d4 = d >> 2, n4 = NT * d4;
    constexpr int kInFlight = 8;
    for (int base = threadIdx.x; base < n4; base += kInFlight * blockDim.x) {
        float4 v[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int i = base + u * blockDim.x;
            const int t = i / d4;
            v[u] = (i < n4 && t0 + t < B)
                       ? __ldg(reinterpret_cast<const float4 *>(x + (int64_t)(t0 + t) * d) + (i - t * d4))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int i = base + u * blockDim.x;
            if (i < n4) {
                const float4 r = make_float4(__half2float(__float2half_rn(v[u].x)), __half2float(__float2half_rn(v[u].y)),
                                             __half2float(__float2half_rn(v[u].z)), __half2float(__float2half_rn(v[u].w)));
                reinterpret_cast<float4 *>(xs)[i] = r;
            }
        }
    }
}

__device__ __forceinline__ float apply_act(float g, float u, int act) {
    g = fmaxf(g, 0.0f);
    return act == SPB_ACT_RELU_RELU_MUL ? g * fmaxf(u, 0.0f) : g * u;
}

// ---- fused path -----------------------------------------------------------
//
// Weight formats (one row per neuron, rows 16-byte aligned):
//   SPB_W_F16   d fp16 values
//   SPB_W_Q8_0  d int8 quants, then d/32 fp16 block scales; w = q * scale
//   SPB_W_Q4_0  d/2 bytes (block b: byte j holds element j in its low nibble
//               and element j + 16 in its high nibble), then d/32 fp16 scales;
//               w = (nibble - 8) * scale
// Dequantisation happens in registers: (float)q * (float)scale, the same
// single fp32 rounding the oracle performs, so dequantised values are
// identical.

// NT dot products of the gate and up rows with the activations in shared
// memory (xs[t][0..d)); per-lane partial sums reduced across the warp.
template <int NT, int WT>
__device__ __forceinline__ void row_dot2_q(const uint8_t *__restrict__ rg, const uint8_t *__restrict__ ru,
                                           const float *__restrict__ xs, int d, int nt, float (&ag)[NT],
                                           float (&au)[NT]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < NT; ++t) ag[t] = au[t] = 0.0f;
    for (int c = lane; c < d / 8; c += 32) {
        float wg[8], wu[8];
        fetch8<WT>(rg, d, c * 8, wg);
        fetch8<WT>(ru, d, c * 8, wu);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < nt) {
                const float4 *xp = reinterpret_cast<const float4 *>(xs + (int64_t)t * d + c * 8);
                const float4 x0 = xp[0], x1 = xp[1];
                const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    ag[t] = fmaf(wg[k], xv[k], ag[t]);
                    au[t] = fmaf(wu[k], xv[k], au[t]);
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        ag[t] = warp_sum(ag[t]);
        au[t] = warp_sum(au[t]);
    }
}

// Tokens are processed in groups of NT (the activations of a group sit in
// shared memory); weights are re-read per group, mostly from L2.
template <int NT, int WT>
__global__ void __launch_bounds__(kGemvThreads) fused_gateup_gemv_kernel(FusedGemvArgs a) {
    extern __shared__ __align__(16) float smem[];
    const int W = words_of(a.f);
    float *xs = smem;
    int *prefix = reinterpret_cast<int *>(xs + NT * a.d);
    int *wtot = prefix + W + 1;
    int *nid = wtot + 64;

    scan_popc(a.seg_bits, W, prefix, wtot);
    const int U = prefix[W];
    const int p0 = (int)((int64_t)U * blockIdx.x / gridDim.x);
    const int p1 = (int)((int64_t)U * (blockIdx.x + 1) / gridDim.x);
    extract_positions(a.seg_bits, prefix, W, p0, p1, nid);
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x == 0) *a.count = U;
    for (int i = threadIdx.x; i < p1 - p0; i += blockDim.x) a.merge[p0 + i] = nid[i];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rb = row_bytes_of<WT>(a.d);
    const uint8_t *wg = static_cast<const uint8_t *>(a.wg);
    const uint8_t *wu = static_cast<const uint8_t *>(a.wu);
    for (int t0 = 0; t0 < a.B; t0 += NT) {
        const int nt = min(NT, a.B - t0);
        __syncthreads();
        load_x_rounded<NT>(a.x, a.B, t0, a.d, xs);
        __syncthreads();
        for (int i = warp; i < p1 - p0; i += kGemvWarps) {
            const int j = nid[i];
            float ag[NT], au[NT];
            row_dot2_q<NT, WT>(wg + j * rb, wu + j * rb, xs, a.d, nt, ag, au);
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t < nt) {
                        // sparse bias add (cuda/kernel.cu:818-830): fp16 bias
                        // of the neuron added to the fp32 product
                        float gv = ag[t], uv = au[t];
                        if (a.bias_g) gv += __half2float(a.bias_g[j]);
                        if (a.bias_u) uv += __half2float(a.bias_u[j]);
                        float hv = apply_act(gv, uv, a.act);
                        if (a.per_token) {
                            const uint32_t word = a.tok_bits[(int64_t)(t0 + t) * W + (j >> 5)];
                            if (!((word >> (j & 31)) & 1u)) hv = 0.0f;
                        }
                        a.h[(int64_t)(p0 + i) * a.B + t0 + t] = __float2half_rn(hv);
                    }
                }
            }
        }
    }
}

constexpr int kDownCols = kGemvThreads * 8;  // output columns per CTA
constexpr int kDownUnroll = 8;               // rows in flight per thread

template <int NT, int WT>
__global__ void __launch_bounds__(kGemvThreads) fused_down_gemv_kernel(FusedGemvArgs a, int cap) {
    extern __shared__ __align__(16) float smem[];
    int *nid = reinterpret_cast<int *>(smem);             // [cap]
    float *hs = smem + cap;                               // [cap][NT]
    const int U = *a.count;
    const int p0 = (int)((int64_t)U * blockIdx.y / gridDim.y);
    const int p1 = (int)((int64_t)U * (blockIdx.y + 1) / gridDim.y);
    const int n = p1 - p0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) nid[i] = a.merge[p0 + i];
    const int m = blockIdx.x * kDownCols + threadIdx.x * 8;
    const int64_t rb = row_bytes_of<WT>(a.d);
    const uint8_t *wd = static_cast<const uint8_t *>(a.wd);
    for (int t0 = 0; t0 < a.B; t0 += NT) {
        const int nt = min(NT, a.B - t0);
        __syncthreads();
        for (int i = threadIdx.x; i < n * NT; i += blockDim.x) {
            const int p = i / NT, t = i - p * NT;
            hs[i] = t < nt ? __half2float(a.h[(int64_t)(p0 + p) * a.B + t0 + t]) : 0.0f;
        }
        __syncthreads();
        if (m >= a.d || n == 0) continue;
        float acc[NT][8];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[t][k] = 0.0f;
        for (int p = 0; p < n; p += kDownUnroll) {
            float w[kDownUnroll][8];
#pragma unroll
            for (int u = 0; u < kDownUnroll; ++u)
                if (p + u < n) fetch8<WT>(wd + nid[p + u] * rb, a.d, m, w[u]);
#pragma unroll
            for (int u = 0; u < kDownUnroll; ++u) {
                if (p + u < n) {
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const float hv = hs[(p + u) * NT + t];
#pragma unroll
                        for (int k = 0; k < 8; ++k) acc[t][k] = fmaf(w[u][k], hv, acc[t][k]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < nt) {
                float4 *o = reinterpret_cast<float4 *>(a.out + (int64_t)(t0 + t) * a.d + m);
                atomicAdd(o, make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]));
                atomicAdd(o + 1, make_float4(acc[t][4], acc[t][5], acc[t][6], acc[t][7]));
            }
        }
    }
}

template <int NT, int WT>
static int launch_fused_gemv_nt(const FusedGemvArgs &a, cudaStream_t st) {
    const int sms = num_sms();
    const int W = words_of(a.f);
    // gate/up: a fixed grid, each CTA takes an equal share of the union.
    int grid = 2 * sms;
    const int cap_g = a.f / grid + 2;
    size_t smem_g = sizeof(float) * NT * a.d + sizeof(int) * (W + 1 + 64 + cap_g);
    if (smem_g > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "gemv: d too large for shared-memory staging");
    auto kg = fused_gateup_gemv_kernel<NT, WT>;
    if (int rc_ = ensure_smem((const void *)kg, smem_g)) return rc_;
    kg<<<grid, kGemvThreads, smem_g, st>>>(a);
    SPB_LAUNCH_CHECK("fused_gateup_gemv_kernel");

    const int slices = (a.d + kDownCols - 1) / kDownCols;
    const int chunks = (2 * sms + slices - 1) / slices;
    const int cap_d = a.f / chunks + 2;
    size_t smem_d = (sizeof(float) * NT + sizeof(int)) * cap_d;
    auto kd = fused_down_gemv_kernel<NT, WT>;
    if (int rc_ = ensure_smem((const void *)kd, smem_d)) return rc_;
    kd<<<dim3(slices, chunks), kGemvThreads, smem_d, st>>>(a, cap_d);
    SPB_LAUNCH_CHECK("fused_down_gemv_kernel");
    return SPB_OK;
}

template <int WT>
static int launch_fused_gemv_wt(const FusedGemvArgs &a, cudaStream_t st) {
    if (a.B <= 1) return launch_fused_gemv_nt<1, WT>(a, st);
    if (a.B <= 2) return launch_fused_gemv_nt<2, WT>(a, st);
    return launch_fused_gemv_nt<4, WT>(a, st);
}

int launch_fused_gemv(const FusedGemvArgs &a, cudaStream_t st) {
    switch (a.wtype) {
        case SPB_W_F16: return launch_fused_gemv_wt<SPB_W_F16>(a, st);
        case SPB_W_Q8_0: return launch_fused_gemv_wt<SPB_W_Q8_0>(a, st);
        case SPB_W_Q4_0: return launch_fused_gemv_wt<SPB_W_Q4_0>(a, st);
        default: return fail(SPB_ERR_INVALID, "gemv: unknown weight type");
    }
}

// ---- drop-in (segment) path -------------------------------------------------

constexpr int kSegTokens = 8;

// grid (C, S): CTA (c, s) computes compacted slots [c*n/C, (c+1)*n/C) of
// segment s for its (up to) 8 tokens.  gate_dst / up_dst are [B][f] fp32.
__global__ void __launch_bounds__(kGemvThreads)
dropin_up_kernel(const __half *__restrict__ wg, const __half *__restrict__ wu, const float *__restrict__ x,
                 float *__restrict__ gate_dst, float *__restrict__ up_dst, const int32_t *__restrict__ merge_idx,
                 const int32_t *__restrict__ act_cum, int B, int d, int f, int G) {
    extern __shared__ __align__(16) float xs[];
    const int s = blockIdx.y;
    const int t0 = s * G;
    const int n = act_cum[s] - (s > 0 ? act_cum[s - 1] : 0);
    const int p0 = (int)((int64_t)n * blockIdx.x / gridDim.x);
    const int p1 = (int)((int64_t)n * (blockIdx.x + 1) / gridDim.x);
    const int tend = min(B, t0 + G);
    load_x_rounded<kSegTokens>(x, tend, t0, d, xs);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t *mi = merge_idx + (int64_t)s * f;
    for (int r = p0 + warp; r < p1; r += kGemvWarps) {
        const int j = mi[r];
        float ag[kSegTokens], au[kSegTokens];
#pragma unroll
        for (int t = 0; t < kSegTokens; ++t) ag[t] = au[t] = 0.0f;
        row_dot2<kSegTokens>(wg + (int64_t)j * d, wu ? wu + (int64_t)j * d : nullptr, xs, d, ag, au);
        if (lane == 0) {
#pragma unroll
            for (int t = 0; t < kSegTokens; ++t) {
                if (t0 + t < tend) {
                    gate_dst[(int64_t)(t0 + t) * f + r] = ag[t];
                    if (wu) up_dst[(int64_t)(t0 + t) * f + r] = au[t];
                }
            }
        }
    }
}

// grid (slices, C, S).  h is compacted fp32 [B][f] (rounded to fp16 here,
// cuda/kernel.cu:1019); out [B][d] must be zero on entry.
__global__ void __launch_bounds__(kGemvThreads)
dropin_down_kernel(const __half *__restrict__ wd, const float *__restrict__ h, float *__restrict__ out,
                   const int32_t *__restrict__ merge_idx, const int32_t *__restrict__ act_cum, int B, int d, int f,
                   int G, int cap) {
    extern __shared__ __align__(16) float smem[];
    float *hs = smem;                                            // [cap][8]
    int *nid = reinterpret_cast<int *>(hs + cap * kSegTokens);  // [cap]
    const int s = blockIdx.z;
    const int t0 = s * G, tend = min(B, t0 + G);
    const int ns = act_cum[s] - (s > 0 ? act_cum[s - 1] : 0);
    const int p0 = (int)((int64_t)ns * blockIdx.y / gridDim.y);
    const int p1 = (int)((int64_t)ns * (blockIdx.y + 1) / gridDim.y);
    const int n = p1 - p0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) nid[i] = merge_idx[(int64_t)s * f + p0 + i];
    for (int i = threadIdx.x; i < n * kSegTokens; i += blockDim.x) {
        const int p = i / kSegTokens, t = i - p * kSegTokens;
        hs[i] = t0 + t < tend ? __half2float(__float2half_rn(h[(int64_t)(t0 + t) * f + p0 + p])) : 0.0f;
    }
    __syncthreads();
    const int m = blockIdx.x * kDownCols + threadIdx.x * 8;
    if (m >= d || n == 0) return;
    float acc[kSegTokens][8];
#pragma unroll
    for (int t = 0; t < kSegTokens; ++t)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[t][k] = 0.0f;
    for (int p = 0; p < n; p += kDownUnroll) {
        uint4 v[kDownUnroll];
#pragma unroll
        for (int u = 0; u < kDownUnroll; ++u)
            if (p + u < n) v[u] = ld_stream_v4(wd + (int64_t)nid[p + u] * d + m);
#pragma unroll
        for (int u = 0; u < kDownUnroll; ++u) {
            if (p + u < n) {
                const uint32_t *pv = reinterpret_cast<const uint32_t *>(&v[u]);
                float w[8];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float2 f2 = h2f2(pv[q]);
                    w[2 * q] = f2.x;
                    w[2 * q + 1] = f2.y;
                }
#pragma unroll
                for (int t = 0; t < kSegTokens; ++t) {
                    const float hv = hs[(p + u) * kSegTokens + t];
#pragma unroll
                    for (int k = 0; k < 8; ++k) acc[t][k] = fmaf(w[k], hv, acc[t][k]);
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kSegTokens; ++t) {
        if (t0 + t < tend) {
            float4 *o = reinterpret_cast<float4 *>(out + (int64_t)(t0 + t) * d + m);
            atomicAdd(o, make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]));
            atomicAdd(o + 1, make_float4(acc[t][4], acc[t][5], acc[t][6], acc[t][7]));
        }
    }
}

int launch_dropin_up(const __half *wg, const __half *wu, const float *x, float *gate_dst, float *up_dst,
                     const int32_t *merge_idx, const int32_t *act_cum, int B, int d, int f, int G, cudaStream_t st) {
    if (G > kSegTokens) return fail(SPB_ERR_UNSUPPORTED, "drop-in path uses segments of at most 8 tokens");
    const int S = (B + G - 1) / G;
    const int C = max(1, (2 * num_sms() + S - 1) / S);
    size_t smem = sizeof(float) * kSegTokens * d;
    if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "drop-in up: d too large");
    if (int rc_ = ensure_smem((const void *)dropin_up_kernel, smem)) return rc_;
    dropin_up_kernel<<<dim3(C, S), kGemvThreads, smem, st>>>(wg, wu, x, gate_dst, up_dst, merge_idx, act_cum, B, d,
                                                             f, G);
    SPB_LAUNCH_CHECK("dropin_up_kernel");
    return SPB_OK;
}

int launch_dropin_down(const __half *wd, const float *h, float *out, const int32_t *merge_idx,
                       const int32_t *act_cum, int B, int d, int f, int G, cudaStream_t st) {
    if (G > kSegTokens) return fail(SPB_ERR_UNSUPPORTED, "drop-in path uses segments of at most 8 tokens");
    const int S = (B + G - 1) / G;
    SPB_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)B * d, st));
    const int slices = (d + kDownCols - 1) / kDownCols;
    // enough position chunks to fill the GPU, and at least f / 4096 so the
    // per-CTA staging (cap rows of h and ids) stays within shared memory
    const int C = max(max(1, (2 * num_sms() + slices * S - 1) / (slices * S)), f / 4096 + 1);
    const int cap = f / C + 2;
    size_t smem = (sizeof(float) * kSegTokens + sizeof(int)) * cap;
    if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "drop-in down: f too large");
    if (int rc_ = ensure_smem((const void *)dropin_down_kernel, smem)) return rc_;
    dropin_down_kernel<<<dim3(slices, C, S), kGemvThreads, smem, st>>>(wd, h, out, merge_idx, act_cum, B, d, f, G,
                                                                       cap);
    SPB_LAUNCH_CHECK("dropin_down_kernel");
    return SPB_OK;
}

}  // namespace spb
