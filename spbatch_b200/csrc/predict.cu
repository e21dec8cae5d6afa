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
//
// Batches above kPredExactMaxBatch would re-stream the weights once per
// 8-token group on CUDA cores; they take the tensor cores instead: x is
// rounded to fp16, hidden = fp16(ReLU(x P1^T)) and logits = hidden P2^T are
// two cuBLASLt GEMMs (fp16 operands, fp32 accumulation, the ReLU and the fp16
// rounding in the first GEMM's epilogue), a histogram pass bins the logits,
// and the same selects run.  The tensor cores' summation order is not the
// oracle's: logits agree to fp32 rounding, and the sets are the exact top-k
// of these logits (they can differ from the oracle's where two logits lie
// within that rounding of the k-th).
#include "spb_internal.h"
#include "spb_scan.cuh"
#include "tc_ptx.cuh"

#include <cublasLt.h>

#include <algorithm>
#include <mutex>
#include <vector>

namespace spb {

using namespace ptx;

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

constexpr int kPredThreads = 256;
constexpr int kPredWarps = kPredThreads / 32;
// Tokens per CTA (their activations staged in shared memory) are a template
// parameter: one at B = 1 (fewest registers), eight otherwise.

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

constexpr int kHistBins = 2048;  // logit histogram: the top 11 bits of the order key

// Programmatic dependent launch: each predictor kernel is launched while the
// previous one drains, waits for its results (griddepcontrol.wait) before
// reading them, and lets its own successor launch early.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const char *what,
                      Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, what);
    return SPB_OK;
}

// hidden[t][r], grid (ceil(D / rows), ceil(B / NT)); the first CTA column
// also zeroes the tokens' logit histograms.  KB: loads in flight per lane
// (16 holds a whole 8 KB row at d = 4096).
template <int NT, int KB>
__global__ void __launch_bounds__(kPredThreads)
pred_hidden_kernel(const __half *__restrict__ p1, const float *__restrict__ x, __half *__restrict__ hidden, int B,
                   int d, int D, int rows_per_cta, uint32_t *__restrict__ hist, uint32_t *__restrict__ cand_cnt) {
    extern __shared__ __align__(16) __half xs[];  // [NT][d], fp16-rounded x
    pdl_enter();
    const int t0 = blockIdx.y * NT, nt = min(NT, B - t0);
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
    if (hist && blockIdx.x == 0) {
        for (int i = threadIdx.x; i < nt * kHistBins; i += blockDim.x) hist[(int64_t)t0 * kHistBins + i] = 0u;
        if (cand_cnt && threadIdx.x < nt) cand_cnt[t0 + threadIdx.x] = 0u;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r1 = min(D, (int)(blockIdx.x + 1) * rows_per_cta);
    for (int r = blockIdx.x * rows_per_cta + warp; r < r1; r += kPredWarps) {
        float acc[NT];
        fixed_dot<NT, KB>(p1 + (int64_t)r * d, xs, d, nt, acc);
        if (lane == 0)
            for (int t = 0; t < nt; ++t) hidden[(int64_t)(t0 + t) * D + r] = __float2half_rn(fmaxf(acc[t], 0.0f));
    }
}

// Order-preserving map of an fp32 logit to an unsigned key.
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// logit[t][j], grid (ceil(f / rows), ceil(B / NT)).  With `hist` (top-k
// selection) it also counts each logit in its token's histogram of the top
// 11 bits of the order key, so the select skips a full pass.
template <int NT>
__global__ void __launch_bounds__(kPredThreads)
pred_logit_kernel(const __half *__restrict__ p2, const __half *__restrict__ hidden, float *__restrict__ logits, int B,
                  int D, int f, int rows_per_cta, uint32_t *__restrict__ hist) {
    extern __shared__ __align__(16) __half hs[];  // [NT][D]
    pdl_enter();
    const int t0 = blockIdx.y * NT, nt = min(NT, B - t0);
    {  // 8 fp16 values per 16-byte load (D % 256 == 0)
        const uint4 *src = reinterpret_cast<const uint4 *>(hidden + (int64_t)t0 * D);
        const int n8 = nt * D / 8;
        for (int i = threadIdx.x; i < n8; i += blockDim.x) reinterpret_cast<uint4 *>(hs)[i] = __ldg(src + i);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j1 = min(f, (int)(blockIdx.x + 1) * rows_per_cta);
    for (int j = blockIdx.x * rows_per_cta + warp; j < j1; j += kPredWarps) {
        float acc[NT];
        fixed_dot<NT, 8>(p2 + (int64_t)j * D, hs, D, nt, acc);
        if (lane < nt) {  // lane t records token t (every lane holds every sum)
            float v = acc[0];
#pragma unroll
            for (int t = 1; t < NT; ++t)
                if (lane == t) v = acc[t];
            logits[(int64_t)(t0 + lane) * f + j] = v;
            if (hist) atomicAdd(hist + (int64_t)(t0 + lane) * kHistBins + (order_key(v) >> 21), 1u);
        }
    }
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

// Radix narrowing over src[0..n): for each 8-bit digit at shift0, then
// (13 -> 5 -> 0 or 24 -> 16 -> 8 -> 0), the keys matching (*prefix, *mask)
// are counted per digit and the digit holding the *need-th largest key is
// appended; on return *prefix is that key and *need the number of keys equal
// to it that belong to the top set.  Whole block (kSelThreads threads).
__device__ void radix_narrow(const uint32_t *src, int n, int shift0, uint32_t *whist, uint32_t *bins,
                             uint32_t *sel_prefix, uint32_t *sel_mask, int *need) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int shift = shift0; shift >= 0; shift = shift == 13 ? 5 : (shift == 5 ? 0 : shift - 8)) {
        // per-warp histograms: logits crowd into a few bins, so a shared
        // histogram would serialise the whole block on those counters
        for (int i = threadIdx.x; i < kSelWarps * 256; i += blockDim.x) whist[i] = 0u;
        __syncthreads();
        const uint32_t pfx = *sel_prefix, msk = *sel_mask;
        uint32_t *wh = whist + warp * 256;
        for (int j = threadIdx.x; j < n; j += blockDim.x) {
            const uint32_t key = src[j];
            if ((key & msk) == pfx) atomicAdd(&wh[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 256) {
            uint32_t sum = 0;
            for (int w = 0; w < kSelWarps; ++w) sum += whist[w * 256 + threadIdx.x];
            bins[threadIdx.x] = sum;
        }
        __syncthreads();
        if (warp == 0) {
            // lane l holds bins 255-8l .. 248-8l (descending); the answer is
            // the highest bin b with (count of bins > b) < need <= (count of bins >= b)
            uint32_t c[8], sum = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                c[q] = bins[255 - 8 * lane - q];
                sum += c[q];
            }
            uint32_t incl = sum;  // inclusive scan over lanes (descending bins)
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t nn = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += nn;
            }
            const int rem = *need;
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
            const int srcl = ball ? __ffs(ball) - 1 : 31;
            const int b = __shfl_sync(0xffffffffu, found >= 0 ? found : 0, srcl);
            const int r = __shfl_sync(0xffffffffu, rem_out, srcl);
            if (lane == 0) {
                *sel_prefix = pfx | ((uint32_t)b << shift);
                *sel_mask = msk | (255u << shift);
                *need = r;
            }
        }
        __syncthreads();
    }
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
                   uint32_t *__restrict__ bits, int32_t *__restrict__ idx, int cap, int32_t *__restrict__ counts,
                   const uint32_t *__restrict__ hist) {
    // [f] keys (raw fp32 bits in threshold mode), [W] active bits, [kSelWarps][256]
    // per-warp histograms, [f] candidate keys (top-k with the logit histogram)
    extern __shared__ uint32_t keys[];
    const int W = (f + 31) / 32;
    uint32_t *sbits = keys + ((f + 3) & ~3);
    uint32_t *whist = sbits + ((W + 3) & ~3);
    uint32_t *cand = whist + kSelWarps * 256;
    const bool raw = k == 0;  // threshold mode compares the fp32 logits themselves
    pdl_enter();
    __shared__ uint32_t bins[256];
    __shared__ uint32_t sel_prefix, sel_mask;
    __shared__ int need;
    __shared__ int warp_tot[33];
    const int t = blockIdx.x;
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
                        raw ? make_uint4(__float_as_uint(v[u].x), __float_as_uint(v[u].y), __float_as_uint(v[u].z),
                                         __float_as_uint(v[u].w))
                            : make_uint4(order_key(v[u].x), order_key(v[u].y), order_key(v[u].z), order_key(v[u].w));
            }
        }
    } else {
        for (int j = threadIdx.x; j < f; j += blockDim.x) keys[j] = raw ? __float_as_uint(lg[j]) : order_key(lg[j]);
    }
    for (int w = threadIdx.x; w < W; w += blockDim.x) sbits[w] = 0u;
    const bool topk = k > 0 && k < f;
    if (threadIdx.x == 0) {
        sel_prefix = 0u;
        sel_mask = 0u;
        need = k;
    }
    __syncthreads();
    // Radix passes over `src[0..n)`: 8-bit digits at `shift`, narrowing
    // (sel_prefix, sel_mask, need) to the key of the k-th largest element.
    int n_src = f;
    const uint32_t *src = keys;
    int shift0 = 24;
    if (topk && hist) {
        // The logit launch counted every key's top 11 bits: the bin holding
        // the k-th largest key and the count above it come from one scan of
        // the 2048 bins (thread i: bins 2047 - 2i and 2046 - 2i, descending).
        const uint32_t *h = hist + (int64_t)t * kHistBins;
        const uint32_t ha = h[kHistBins - 1 - 2 * threadIdx.x], hb = h[kHistBins - 2 - 2 * threadIdx.x];
        int tot0;
        const int above = sel_block_scan((int)(ha + hb), warp_tot, &tot0);
        if (above < k && k <= above + (int)(ha + hb)) {
            const bool in_a = above + (int)ha >= k;
            const uint32_t bin = in_a ? kHistBins - 1 - 2 * threadIdx.x : kHistBins - 2 - 2 * threadIdx.x;
            sel_prefix = bin << 21;
            sel_mask = 0xFFE00000u;
            need = k - (in_a ? above : above + (int)ha);
        }
        __syncthreads();
        // Only the keys in that bin still compete: gather them (ascending
        // index order) and finish the select on them alone.
        const uint32_t pfx = sel_prefix;
        const int per = (f + kSelThreads - 1) / kSelThreads;
        const int j0 = min(f, (int)threadIdx.x * per), j1 = min(f, j0 + per);
        int nc = 0;
        for (int j = j0; j < j1; ++j) nc += (keys[j] & 0xFFE00000u) == pfx;
        int ncand;
        int pos = sel_block_scan(nc, warp_tot, &ncand);
        for (int j = j0; j < j1; ++j)
            if ((keys[j] & 0xFFE00000u) == pfx) cand[pos++] = keys[j];
        __syncthreads();
        n_src = ncand;
        src = cand;
        shift0 = 13;  // digits of bits 20..13, 12..5, then 7..0 (bits 7..5 already fixed)
    }
    if (topk) radix_narrow(src, n_src, shift0, whist, bins, &sel_prefix, &sel_mask, &need);
    const uint32_t thr_key = sel_prefix;
    const int take_eq = need;  // how many keys equal to thr_key are active (lowest ids first)
    // contiguous index run of this thread
    const int per = (f + kSelThreads - 1) / kSelThreads;
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
        else active = __uint_as_float(keys[j]) >= threshold;  // float compare: -0.0 >= 0.0 holds
        n_act += active;
    }
    __syncthreads();
    int pos = sel_block_scan(n_act, warp_tot, &tot);
    eq_rank -= n_eq;  // replay the same decisions, now writing
    uint32_t word = 0;
    for (int j = j0; j < j1; ++j) {
        bool active;
        if (k >= f) active = true;
        else if (k > 0) active = keys[j] > thr_key || (keys[j] == thr_key && eq_rank++ < take_eq);
        else active = __uint_as_float(keys[j]) >= threshold;
        if (labels) labels[(int64_t)t * f + j] = active ? 1.0f : 0.0f;
        word |= (active ? 1u : 0u) << (j & 31);
        if ((j & 31) == 31 || j == j1 - 1) {  // runs are not word-aligned: merge in shared memory
            if (word) atomicOr(&sbits[j >> 5], word);
            word = 0;
        }
        if (active) {
            if (idx && pos < cap) idx[(int64_t)t * cap + pos] = j;
            ++pos;
        }
    }
    if (bits) {
        __syncthreads();
        for (int w = threadIdx.x; w < W; w += blockDim.x) bits[(int64_t)t * W + w] = sbits[w];
    }
    if (threadIdx.x == 0 && counts) counts[t] = tot;
}


// ---- grid-wide top-k for set outputs (bits / labels, no index list) --------
// Pass A, grid (ceil(f / 256), B): every CTA finds the token's threshold bin
// from the logit histogram, writes its 256 neurons' words (active iff the
// key's top 11 bits are above that bin) and appends the bin's candidates.
// Pass B, one CTA per token: exact selection among the candidates (radix
// narrowing on the low 21 bits, equal keys taken lowest id first), whose
// winners are ORed into the words.  The same set as pred_select_kernel.
constexpr int kGsThreads = 256;

__global__ void __launch_bounds__(kGsThreads)
pred_gsel_a_kernel(const float *__restrict__ logits, int f, int k, const uint32_t *__restrict__ hist,
                   uint32_t *__restrict__ bits, float *__restrict__ labels, uint2 *__restrict__ cand,
                   uint32_t *__restrict__ cand_cnt, int2 *__restrict__ sel) {
    __shared__ int warp_tot[kGsThreads / 32 + 1];
    __shared__ uint32_t s_bin;
    __shared__ int s_need;
    pdl_enter();
    const int t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int W = (f + 31) / 32;
    // thread i holds bins 2047 - 8i .. 2040 - 8i (descending)
    const uint32_t *h = hist + (int64_t)t * kHistBins;
    uint32_t c[8], sum = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        c[q] = h[kHistBins - 1 - 8 * tid - q];
        sum += c[q];
    }
    const int incl = warp_incl_scan((int)sum);
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int v = lane < kGsThreads / 32 ? warp_tot[lane] : 0;
        const int vi = warp_incl_scan(v);
        if (lane < kGsThreads / 32) warp_tot[lane] = vi - v;
    }
    __syncthreads();
    int before = warp_tot[warp] + incl - (int)sum;  // keys in bins above this thread's
    if (before < k && k <= before + (int)sum) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (before < k && k <= before + (int)c[q]) {
                s_bin = kHistBins - 1 - 8 * tid - q;
                s_need = k - before;
            }
            before += c[q];
        }
    }
    __syncthreads();
    const uint32_t bin = s_bin;
    const int j = blockIdx.x * kGsThreads + tid;
    const uint32_t key = j < f ? order_key(logits[(int64_t)t * f + j]) : 0u;
    const bool active = j < f && (key >> 21) > bin;
    const bool is_cand = j < f && (key >> 21) == bin;
    const uint32_t word = __ballot_sync(0xffffffffu, active);
    if (lane == 0 && j < f) bits[(int64_t)t * W + (j >> 5)] = word;
    if (labels && j < f) labels[(int64_t)t * f + j] = active ? 1.0f : 0.0f;
    const uint32_t cb = __ballot_sync(0xffffffffu, is_cand);
    if (cb) {
        uint32_t base = 0;
        if (lane == 0) base = atomicAdd(cand_cnt + t, (uint32_t)__popc(cb));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (is_cand) cand[(int64_t)t * f + base + __popc(cb & ((1u << lane) - 1u))] = make_uint2(key, (uint32_t)j);
    }
    if (blockIdx.x == 0 && tid == 0) sel[t] = make_int2((int)bin, s_need);
}

__global__ void __launch_bounds__(kSelThreads)
pred_gsel_b_kernel(int f, int k, uint32_t *__restrict__ bits, float *__restrict__ labels,
                   const uint2 *__restrict__ cand, uint32_t *__restrict__ cand_cnt, const int2 *__restrict__ sel,
                   int32_t *__restrict__ counts) {
    extern __shared__ uint32_t ckeys[];  // [n] candidate keys, then [kSelWarps][256] histograms
    __shared__ uint32_t bins[256];
    __shared__ uint32_t sel_prefix, sel_mask;
    __shared__ int need;
    pdl_enter();
    const int t = blockIdx.x;
    const int W = (f + 31) / 32;
    const int n = (int)cand_cnt[t];
    uint32_t *whist = ckeys + ((n + 3) & ~3);
    const uint2 *ct = cand + (int64_t)t * f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ckeys[i] = ct[i].x;
    if (threadIdx.x == 0) {
        sel_prefix = (uint32_t)sel[t].x << 21;
        sel_mask = 0xFFE00000u;
        need = sel[t].y;
    }
    __syncthreads();
    radix_narrow(ckeys, n, 13, whist, bins, &sel_prefix, &sel_mask, &need);
    const uint32_t thr = sel_prefix;
    const int take_eq = need;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint2 cj = ct[i];
        bool on = cj.x > thr;
        if (cj.x == thr) {  // equal keys: the take_eq lowest ids (candidates arrive in any order)
            int rank = 0;
            for (int q = 0; q < n; ++q) {
                const uint2 o = ct[q];
                rank += o.x == thr && o.y < cj.y;
            }
            on = rank < take_eq;
        }
        if (on) {
            atomicOr(bits + (int64_t)t * W + (cj.y >> 5), 1u << (cj.y & 31));
            if (labels) labels[(int64_t)t * f + cj.y] = 1.0f;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        cand_cnt[t] = 0u;  // ready for the next call
        if (counts) counts[t] = k;
    }
}

// ---- one-launch predictor for one token (top-k into set words) ------------
//
// At B = 1 the four-launch chain above spends most of its time in launch
// ramps and in the two select launches.  This kernel does the whole
// predictor in one cooperative launch of one CTA per SM:
//   A. Warps kPfHidW.. copy the CTA's contiguous slice of P2 rows [j0, j1)
//      into shared memory with 16-byte cp.async (P2 is not written by the
//      previous kernel, so the copies start before the dependency wait).
//   B. Warps 0..kPfHidW-1 stage x as fp16 and compute the CTA's share of
//      hidden = fp16(ReLU(P1 x)) (warp per row, the chain's fixed-order dot),
//      zero the histogram and set words, then meet the grid at a barrier.
//   C. Logits of the slice from shared memory with the same fixed order
//      (bit-identical to pred_logit_kernel), kept as order keys and written
//      out; the keys are binned in shared memory and the non-zero bins added
//      to the global 11-bit histogram.
//   D. Grid barrier; every CTA reads the histogram and all logits (L2) in one
//      round trip, finds the threshold bin and how many keys it still needs
//      from it, compacts that bin's candidates in id order (block scan), and
//      decides its own rows: above the bin, or in it with rank < need (rank =
//      candidates with a larger key, or an equal key and a lower id) -- the
//      exact top-k with ties to the lower id.
// Grid barriers use a monotonic counter in this module's device memory:
// every CTA arrives at both barriers of every launch, so arrival counts stay
// multiples of the grid, and launches of this full-device grid do not overlap.
constexpr int kPfThreads = 512;
constexpr int kPfWarps = kPfThreads / 32;
constexpr int kPfHidW = 8;  // warps computing hidden rows; the others copy the P2 slice
constexpr uint64_t kPfTimeoutNs = 2000000000ull;
__device__ unsigned long long g_pf_arrivals;

__device__ __forceinline__ void pf_block_sync(int nthreads) {
    if (nthreads == (int)blockDim.x) __syncthreads();
    else asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Grid barrier for the first nthreads threads (whole warps) of every CTA
// (cooperative launch: every CTA is resident).  Bounded: a barrier that
// never completes sets *fail and the launch finishes.
__device__ __forceinline__ void pf_grid_sync(int *fail, int nthreads) {
    pf_block_sync(nthreads);
    if (threadIdx.x == 0) {
        unsigned long long ticket;
        __threadfence();
        asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(ticket) : "l"(&g_pf_arrivals) : "memory");
        const unsigned long long target = (ticket / gridDim.x + 1) * gridDim.x;
        const uint64_t t0 = globaltimer();
        for (;;) {
            unsigned long long v;
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(&g_pf_arrivals) : "memory");
            if (v >= target) break;
            if (globaltimer() - t0 > kPfTimeoutNs) {
                *fail = 1;
                break;
            }
            __nanosleep(64);
        }
    }
    pf_block_sync(nthreads);
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

// Shared memory: xs [d] | hs [D] | keys [rows] | shist [2048] |
// P2 slice [rows][D] (reused in D: candidates [f], logits [f]).
template <int KB>
__global__ void __launch_bounds__(kPfThreads, 1)
pred_fused_kernel(const __half *__restrict__ p1, const __half *__restrict__ p2, const float *__restrict__ x, int d,
                  int D, int f, int k, int rows, __half *__restrict__ hidden, float *__restrict__ logits,
                  uint32_t *__restrict__ hist, uint32_t *__restrict__ bits, float *__restrict__ labels,
                  int32_t *__restrict__ counts) {
    extern __shared__ __align__(16) uint8_t pf_smem[];
    __half *xs = reinterpret_cast<__half *>(pf_smem);
    __half *hs = xs + d;
    uint32_t *keys = reinterpret_cast<uint32_t *>(hs + D);
    uint32_t *shist = keys + ((rows + 3) & ~3);
    __half *p2s = reinterpret_cast<__half *>(shist + kHistBins);
    uint2 *cand = reinterpret_cast<uint2 *>(p2s);     // [f] candidates (phase D)
    float *lgs = reinterpret_cast<float *>(cand + f);  // [f] logits (phase D)
    __shared__ int s_fail, s_nc, s_need;
    __shared__ uint32_t s_bin;
    __shared__ int warp_tot[kPfWarps + 1];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, W = (f + 31) / 32;
    const int j0 = min(f, (int)blockIdx.x * rows), nrow = min(f, j0 + rows) - j0;
    constexpr int kHidT = kPfHidW * 32;
    if (tid == 0) s_fail = 0;
    // ---- A / B ----
    if (warp >= kPfHidW) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(p2s);
        const char *src = reinterpret_cast<const char *>(p2 + (size_t)j0 * D);
        const int n16 = nrow * D / 8;  // 16-byte pieces of the slice
        for (int i = tid - kHidT; i < n16; i += kPfThreads - kHidT) cp_async16_full(dst + i * 16, src + (size_t)i * 16);
        cp_async_commit();
        asm volatile("griddepcontrol.wait;" ::: "memory");
        cp_async_wait_all();
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int i = tid; i < d / 4; i += kHidT) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
            const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
            uint2 pk;
            pk.x = *reinterpret_cast<const uint32_t *>(&h0);
            pk.y = *reinterpret_cast<const uint32_t *>(&h1);
            reinterpret_cast<uint2 *>(xs)[i] = pk;
        }
        for (int i = blockIdx.x * kHidT + tid; i < kHistBins; i += G * kHidT) hist[i] = 0u;
        for (int i = blockIdx.x * kHidT + tid; i < W; i += G * kHidT) bits[i] = 0u;
        pf_block_sync(kHidT);
        const int hr = (D + G - 1) / G;
        for (int r = blockIdx.x * hr + warp; r < min(D, (int)(blockIdx.x + 1) * hr); r += kPfHidW) {
            float acc[1];
            fixed_dot<1, KB>(p1 + (int64_t)r * d, xs, d, 1, acc);
            if (lane == 0) hidden[r] = __float2half_rn(fmaxf(acc[0], 0.0f));
        }
        pf_grid_sync(&s_fail, kHidT);
        for (int i = tid; i < D / 8; i += kHidT)
            reinterpret_cast<uint4 *>(hs)[i] = __ldcg(reinterpret_cast<const uint4 *>(hidden) + i);
    }
    __syncthreads();
    // ---- C. logits of the slice, four rows per warp at a time ----
    {
        constexpr int R = 4;
        const int nfull = nrow / R * R;
        for (int r = warp * R; r < nfull; r += kPfWarps * R) {
            float acc[R];
            fixed_dot_smem_rows<R>(p2s + (size_t)r * D, hs, D, acc);
            if (lane < R) {
                float v = acc[0];
#pragma unroll
                for (int q = 1; q < R; ++q)
                    if (lane == q) v = acc[q];
                logits[j0 + r + lane] = v;
                keys[r + lane] = order_key(v);
            }
        }
        for (int r = nfull + warp; r < nrow; r += kPfWarps) {
            float acc[1];
            fixed_dot_smem_rows<1>(p2s + (size_t)r * D, hs, D, acc);
            if (lane == 0) {
                logits[j0 + r] = acc[0];
                keys[r] = order_key(acc[0]);
            }
        }
    }
    for (int i = tid; i < kHistBins; i += kPfThreads) shist[i] = 0u;
    __syncthreads();
    for (int r = tid; r < nrow; r += kPfThreads) atomicAdd(&shist[keys[r] >> 21], 1u);
    __syncthreads();
    for (int i = tid; i < kHistBins; i += kPfThreads)
        if (shist[i]) atomicAdd(hist + i, shist[i]);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    pf_grid_sync(&s_fail, kPfThreads);
    // ---- D. the exact top-k, each CTA deciding its own rows ----
    // One round trip: the histogram (thread i: bins 2047 - 4i .. 2044 - 4i,
    // descending) and all logits (L2) into shared memory.
    uint32_t c4[4], sum = 0;
    {
        constexpr int U = 8;
        const bool vec = (f & 3) == 0;
        const int n4 = vec ? f >> 2 : 0;
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = tid + u * kPfThreads;
            v[u] = i < n4 ? __ldcg(reinterpret_cast<const float4 *>(logits) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) c4[q] = __ldcg(hist + kHistBins - 1 - 4 * tid - q);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = tid + u * kPfThreads;
            if (i < n4) reinterpret_cast<float4 *>(lgs)[i] = v[u];
        }
        for (int i = tid + U * kPfThreads; i < n4; i += kPfThreads)
            reinterpret_cast<float4 *>(lgs)[i] = __ldcg(reinterpret_cast<const float4 *>(logits) + i);
        if (!vec)
            for (int j = tid; j < f; j += kPfThreads) lgs[j] = __ldcg(logits + j);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) sum += c4[q];
    const int incl = warp_incl_scan((int)sum);
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int v = lane < kPfWarps ? warp_tot[lane] : 0;
        const int vi = warp_incl_scan(v);
        if (lane < kPfWarps) warp_tot[lane] = vi - v;
    }
    __syncthreads();
    int before = warp_tot[warp] + incl - (int)sum;  // keys in bins above this thread's
    if (before < k && k <= before + (int)sum) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (before < k && k <= before + (int)c4[q]) {
                s_bin = kHistBins - 1 - 4 * tid - q;
                s_need = k - before;
            }
            before += c4[q];
        }
    }
    __syncthreads();
    const uint32_t bin = s_bin;
    // candidates (keys in the threshold bin) compacted in id order: each
    // thread counts its contiguous run, one block scan places them
    const int per = (f + kPfThreads - 1) / kPfThreads;
    const int ja = min(f, tid * per), jb = min(f, ja + per);
    int mine = 0;
    for (int j = ja; j < jb; ++j) mine += (order_key(lgs[j]) >> 21) == bin;
    const int mi = warp_incl_scan(mine);
    if (lane == 31) warp_tot[warp] = mi;
    __syncthreads();
    if (warp == 0) {
        const int v = lane < kPfWarps ? warp_tot[lane] : 0;
        const int vi = warp_incl_scan(v);
        if (lane < kPfWarps) warp_tot[lane] = vi - v;
        if (lane == kPfWarps - 1) s_nc = vi;
    }
    __syncthreads();
    {
        int pos = warp_tot[warp] + mi - mine;
        for (int j = ja; j < jb; ++j) {
            const uint32_t key = order_key(lgs[j]);
            if ((key >> 21) == bin) cand[pos++] = make_uint2(key, (uint32_t)j);
        }
    }
    __syncthreads();
    const int nc = s_nc, need = s_need;
    // own rows, a warp per 32 rows: above the bin, or ranked among the
    // candidates (rank = larger keys, or equal keys with lower ids)
    for (int r0 = warp * 32; r0 < nrow; r0 += kPfWarps * 32) {
        const int r = r0 + lane;
        const uint32_t key = r < nrow ? keys[r] : 0u;
        const uint32_t j = (uint32_t)(j0 + r);
        bool on = r < nrow && (key >> 21) > bin;
        uint32_t inbin = __ballot_sync(0xffffffffu, r < nrow && (key >> 21) == bin);
        while (inbin) {  // the warp ranks each in-bin row together
            const int src = __ffs(inbin) - 1;
            inbin &= inbin - 1;
            const uint32_t kk = __shfl_sync(0xffffffffu, key, src);
            const uint32_t jj = __shfl_sync(0xffffffffu, j, src);
            int rank = 0;
            for (int q = lane; q < nc; q += 32) {
                const uint2 o = cand[q];
                rank += o.x > kk || (o.x == kk && o.y < jj);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
            if (lane == src) on = rank < need;
        }
        if (on) atomicOr(bits + (j >> 5), 1u << (j & 31));
        if (labels && r < nrow) labels[j] = on ? 1.0f : 0.0f;
    }
    if (counts && blockIdx.x == 0 && tid == 0) counts[0] = s_fail ? -1 : k;
}

// Tensor-core route: x -> fp16 (and the histograms / candidate counters zeroed).
__global__ void __launch_bounds__(256)
pred_prep_kernel(const float *__restrict__ x, __half *__restrict__ x16, int64_t n, uint32_t *__restrict__ hist,
                 int B, uint32_t *__restrict__ cand_cnt) {
    pdl_enter();
    const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, gs = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = gt; i < n / 4; i += gs) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t *>(&h0);
        pk.y = *reinterpret_cast<const uint32_t *>(&h1);
        reinterpret_cast<uint2 *>(x16)[i] = pk;
    }
    if (hist)
        for (int64_t i = gt; i < (int64_t)B * kHistBins; i += gs) hist[i] = 0u;
    if (cand_cnt)
        for (int64_t i = gt; i < B; i += gs) cand_cnt[i] = 0u;
}

// Per-token histograms of the logits' top 11 key bits (tensor-core route),
// grid (ceil(f / 4096), B): a shared histogram per CTA, flushed once.
__global__ void __launch_bounds__(256)
pred_hist_kernel(const float *__restrict__ logits, int f, uint32_t *__restrict__ hist) {
    __shared__ uint32_t bins[kHistBins];
    pdl_enter();
    const int t = blockIdx.y;
    for (int i = threadIdx.x; i < kHistBins; i += blockDim.x) bins[i] = 0u;
    __syncthreads();
    const int j1 = min(f, (int)(blockIdx.x + 1) * 4096);
    for (int j = blockIdx.x * 4096 + threadIdx.x; j < j1; j += blockDim.x)
        atomicAdd(&bins[order_key(__ldg(logits + (int64_t)t * f + j)) >> 21], 1u);
    __syncthreads();
    for (int i = threadIdx.x; i < kHistBins; i += blockDim.x)
        if (bins[i]) atomicAdd(hist + (int64_t)t * kHistBins + i, bins[i]);
}

namespace {

cublasLtHandle_t lt_handle() {
    static std::mutex mu;
    static std::vector<cublasLtHandle_t> handles;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if ((int)handles.size() <= dev) handles.resize(dev + 1, nullptr);
    if (!handles[dev] && cublasLtCreate(&handles[dev]) != CUBLAS_STATUS_SUCCESS) handles[dev] = nullptr;
    return handles[dev];
}

// C[n][m] (row-major, m contiguous) = op(A[m][K] row-major) . B[n][K]^T in
// column-major terms: C (m x n, ld m) = A^T (A stored K x m, ld K) . B (K x n, ld K).
// fp16 A and B, fp32 accumulation; C fp16 with ReLU, or fp32.
int lt_gemm(const __half *a, const __half *b, void *c, int m, int n, int K, bool relu_fp16, cudaStream_t st) {
    cublasLtHandle_t h = lt_handle();
    if (!h) return fail(SPB_ERR_CUDA, "spb_predict: cublasLtCreate failed");
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
    int rc = SPB_OK;
    const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
    const cublasLtEpilogue_t epi = relu_fp16 ? CUBLASLT_EPILOGUE_RELU : CUBLASLT_EPILOGUE_DEFAULT;
    const cudaDataType_t ct = relu_fp16 ? CUDA_R_16F : CUDA_R_32F;
    const float alpha = 1.0f, beta = 0.0f;
    if (cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA)) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB)) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_EPILOGUE, &epi, sizeof(epi)) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&la, CUDA_R_16F, K, m, K) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&lb, CUDA_R_16F, K, n, K) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&lc, ct, m, n, m) != CUBLAS_STATUS_SUCCESS) {
        rc = fail(SPB_ERR_CUDA, "spb_predict: cublasLt descriptors");
    } else if (cublasLtMatmul(h, op, &alpha, a, la, b, lb, &beta, c, lc, c, lc, nullptr, nullptr, 0, st) !=
               CUBLAS_STATUS_SUCCESS) {
        rc = fail(SPB_ERR_CUDA, "spb_predict: cublasLtMatmul failed");
    }
    if (lc) cublasLtMatrixLayoutDestroy(lc);
    if (lb) cublasLtMatrixLayoutDestroy(lb);
    if (la) cublasLtMatrixLayoutDestroy(la);
    if (op) cublasLtMatmulDescDestroy(op);
    return rc;
}

}  // namespace

int launch_predict(const __half *p1, const __half *p2, const float *x, int B, int d, int D, int f, int k,
                   float threshold, float *labels, uint32_t *bits, int32_t *idx, int32_t *counts, float *logits,
                   __half *hidden, const PredScratch &sc, cudaStream_t st) {
    // logit histograms only serve the top-k selection
    uint32_t *hist = (k > 0 && k < f) ? sc.hist : nullptr;
    // sets without an index list: the grid-wide select
    const bool grid_sel = hist && !idx;
    const int sms = num_sms();
    if (grid_sel && B == 1 && d % 256 == 0) {
        // one launch: P2 slices resident in shared memory, select in the tail
        const int G = sms;
        const int rows = (f + G - 1) / G;
        const size_t slice = std::max(sizeof(__half) * (size_t)rows * D, (sizeof(uint2) + sizeof(float)) * (size_t)f);
        const size_t smem =
            sizeof(__half) * (size_t)(d + D) + sizeof(uint32_t) * ((size_t)((rows + 3) & ~3) + kHistBins) + slice;
        if (smem <= 220 * 1024) {
            auto kern = d / 8 >= 32 * 16 ? pred_fused_kernel<16> : pred_fused_kernel<8>;
            if (int rc = ensure_smem((const void *)kern, smem)) return rc;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(G);
            cfg.blockDim = dim3(kPfThreads);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = st;
            cudaLaunchAttribute attr[2];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            // the grid barriers need every CTA resident
            attr[1].id = cudaLaunchAttributeCooperative;
            attr[1].val.cooperative = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 2;
            uint32_t *wb = bits ? bits : sc.bits;
            const cudaError_t e =
                cudaLaunchKernelEx(&cfg, kern, p1, p2, x, d, D, f, k, rows, hidden, logits, hist, wb, labels, counts);
            if (e != cudaSuccess) return cuda_fail(e, "pred_fused_kernel");
            return SPB_OK;
        }
    }
    if (B > kPredExactMaxBatch) {
        // tensor-core route: x16, two GEMMs, histograms
        const int64_t n = (int64_t)B * d;
        if (int rc = launch_pdl(pred_prep_kernel, dim3(std::max(1, std::min(2 * sms, (int)((n / 4 + 255) / 256)))),
                                dim3(256), 0, st, "pred_prep_kernel", x, sc.x16, n, hist, B,
                                grid_sel ? sc.cand_cnt : nullptr))
            return rc;
        if (int rc = lt_gemm(p1, sc.x16, hidden, D, B, d, true, st)) return rc;
        if (int rc = lt_gemm(p2, hidden, logits, f, B, D, false, st)) return rc;
        if (hist)
            if (int rc = launch_pdl(pred_hist_kernel, dim3((f + 4095) / 4096, B), dim3(256), 0, st,
                                    "pred_hist_kernel", (const float *)logits, f, hist))
                return rc;
    } else {
        {
            // 8 tokens beyond B = 1: wider groups make the CUDA-core loop
            // shared-memory and FMA bound (measured slower at B = 32 / 64)
            const int NTH = B == 1 ? 1 : 8;
            const int ty = (B + NTH - 1) / NTH;
            // one row per warp when that fills the GPU: every row's loads are in
            // flight at once (each warp's 8 KB row is the fixed-order dot unit)
            const int ctas = max(1, (2 * sms + ty - 1) / ty);
            const int rows = std::min((D + ctas - 1) / ctas, kPredWarps);
            const size_t smem = sizeof(__half) * NTH * d;
            if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: d too large");
            const bool kb16 = d / 8 >= 32 * 16;
            auto kern = NTH == 1 ? (kb16 ? pred_hidden_kernel<1, 16> : pred_hidden_kernel<1, 8>)
                      : NTH == 8 ? (kb16 ? pred_hidden_kernel<8, 16> : pred_hidden_kernel<8, 8>)
                                 : (kb16 ? pred_hidden_kernel<8, 16> : pred_hidden_kernel<8, 8>);
            if (int rc = ensure_smem((const void *)kern, smem)) return rc;
            if (int rc = launch_pdl(kern, dim3((D + rows - 1) / rows, ty), dim3(kPredThreads), smem, st,
                                    "pred_hidden_kernel", p1, x, hidden, B, d, D, rows, hist,
                                    grid_sel ? sc.cand_cnt : nullptr))
                return rc;
        }
        {
            // at most four rows per warp: rows of D = 1024 are only 2 KB, so a
            // warp walking many of them in turn is latency-bound; more CTAs keep
            // more rows in flight (each CTA re-stages NT x D fp16 from L2)
            const int NTL = B == 1 ? 1 : 8;
            const int ty = (B + NTL - 1) / NTL;
            const int ctas = max(1, (4 * sms + ty - 1) / ty);
            const int rows = std::min((f + ctas - 1) / ctas, 4 * kPredWarps);
            const size_t smem = sizeof(__half) * NTL * D;
            if (smem > 200 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: D too large");
            auto kern = NTL == 1 ? pred_logit_kernel<1> : pred_logit_kernel<8>;
            if (int rc = ensure_smem((const void *)kern, smem)) return rc;
            if (int rc = launch_pdl(kern, dim3((f + rows - 1) / rows, ty), dim3(kPredThreads), smem, st,
                                    "pred_logit_kernel", p2, hidden, logits, B, D, f, rows, hist))
                return rc;
        }
    }
    if (grid_sel) {
        uint32_t *wb = bits ? bits : sc.bits;
        if (int rc = launch_pdl(pred_gsel_a_kernel, dim3((f + kGsThreads - 1) / kGsThreads, B), dim3(kGsThreads), 0,
                                st, "pred_gsel_a_kernel", logits, f, k, hist, wb, labels, sc.cand, sc.cand_cnt,
                                sc.sel))
            return rc;
        // candidates of the threshold bin: at most f per token
        const size_t smem = sizeof(uint32_t) * (((f + 3) & ~3) + kSelWarps * 256);
        if (smem > 227 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: f too large");
        if (int rc = ensure_smem((const void *)pred_gsel_b_kernel, smem)) return rc;
        if (int rc = launch_pdl(pred_gsel_b_kernel, dim3(B), dim3(kSelThreads), smem, st, "pred_gsel_b_kernel", f, k,
                                wb, labels, sc.cand, sc.cand_cnt, sc.sel, counts))
            return rc;
        return SPB_OK;
    }
    {
        // the candidate buffer doubles the key storage; without room for it
        // the select runs its four passes over all keys
        const size_t wpad = ((f + 31) / 32 + 3) & ~3;
        size_t smem = sizeof(uint32_t) * (2 * ((f + 3) & ~3) + wpad + kSelWarps * 256);
        if (smem > 227 * 1024) {
            hist = nullptr;
            smem = sizeof(uint32_t) * (((f + 3) & ~3) + wpad + kSelWarps * 256);
        }
        if (smem > 227 * 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_predict: f too large");
        if (int rc = ensure_smem((const void *)pred_select_kernel, smem)) return rc;
        const int cap = k > 0 ? k : f;
        if (int rc = launch_pdl(pred_select_kernel, dim3(B), dim3(kSelThreads), smem, st, "pred_select_kernel",
                                logits, f, k, threshold, labels, bits, idx, cap, counts, hist))
            return rc;
    }
    return SPB_OK;
}

}  // namespace spb
