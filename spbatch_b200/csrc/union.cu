// Union / compaction of per-token active-neuron sets.
//
// Replaces the reference's four-launch get_idx_cuda sequence
// (merge_batch_sparsity_kernel -> cub::DeviceScan::InclusiveSum ->
// move_activation -> generate_indices_kernel + cudaStreamSynchronize,
// cuda/kernel.cu:540-593, 877-937) with two launches and no host sync:
//
//   union_bits_kernel  one warp per 32-neuron word: ballot over every token's
//                      label (coalesced 128-byte loads), writes per-token and
//                      per-segment bit words; also zero-fills the FFN output
//                      the down projection accumulates into.
//   compact_kernel     one CTA per segment: block scan of word popcounts and
//                      ascending emission of neuron ids, plus the cumulative
//                      counts the reference's act_neurons_device holds.
//
// The fused FFN path skips compact_kernel: its CTAs rebuild the slice of the
// index list they own from the segment bits (spb_scan.cuh).
#include <mutex>
#include <string>
#include <vector>

#include "spb_internal.h"
#include "spb_scan.cuh"

namespace spb {

constexpr int kUnionWarps = 8;

__global__ void __launch_bounds__(kUnionWarps * 32)
union_bits_kernel(const float *__restrict__ idx, int B, int f, int W, int G, uint32_t *__restrict__ tok_bits,
                  uint32_t *__restrict__ seg_bits, PrepJobs jobs) {
    // Launched with programmatic dependent launch: the CTAs may be resident
    // before the previous kernel on the stream finishes, and wait here until
    // its results are visible.  The dependent launch (the FFN kernel) may
    // then start its prologue; it waits for this grid's results before
    // reading them.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int w = blockIdx.x * kUnionWarps + (threadIdx.x >> 5);
    if (w < W) {
        const int j = w * 32 + lane;
        const bool in = j < f;
        uint32_t seg = 0;
        int t = 0;
        constexpr int U = 32;  // all of a 32-token batch's labels in flight at once
        for (; t + U <= B; t += U) {
            float v[U];
#pragma unroll
            for (int i = 0; i < U; ++i) v[i] = in ? __ldg(idx + (int64_t)(t + i) * f + j) : 0.0f;
#pragma unroll
            for (int i = 0; i < U; ++i) {
                uint32_t b = __ballot_sync(0xffffffffu, v[i] > 0.0f);
                if (tok_bits && lane == 0) tok_bits[(int64_t)(t + i) * W + w] = b;
                seg |= b;
                if ((t + i) % G == G - 1 || t + i == B - 1) {
                    if (lane == 0) seg_bits[(int64_t)((t + i) / G) * W + w] = seg;
                    seg = 0;
                }
            }
        }
        for (; t < B; ++t) {
            float v = in ? __ldg(idx + (int64_t)t * f + j) : 0.0f;
            uint32_t b = __ballot_sync(0xffffffffu, v > 0.0f);
            if (tok_bits && lane == 0) tok_bits[(int64_t)t * W + w] = b;
            seg |= b;
            if (t % G == G - 1 || t == B - 1) {
                if (lane == 0) seg_bits[(int64_t)(t / G) * W + w] = seg;
                seg = 0;
            }
        }
    }
    const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (jobs.zero_out) {
        const int64_t n4 = jobs.zero_n / 4;
        for (int64_t i = gtid; i < n4; i += stride)
            reinterpret_cast<float4 *>(jobs.zero_out)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t i = n4 * 4 + gtid; i < jobs.zero_n; i += stride) jobs.zero_out[i] = 0.0f;
    }
    if (jobs.zero_u32)
        for (int64_t i = gtid; i < jobs.zero_u32_n; i += stride) jobs.zero_u32[i] = 0u;
    if (jobs.x16) {
        // fp16 copy of x, rows padded with zeros to Np (the MMA N extent)
        const int64_t n2 = (int64_t)jobs.Np * jobs.d / 2;
        for (int64_t i = gtid; i < n2; i += stride) {
            const int64_t e = 2 * i;
            const int t = (int)(e / jobs.d);
            float2 v = t < jobs.B ? *reinterpret_cast<const float2 *>(jobs.x + e) : make_float2(0.f, 0.f);
            reinterpret_cast<__half2 *>(jobs.x16)[i] = __floats2half2_rn(v.x, v.y);
        }
    }
}

// Union words from per-token bits: word w of segment s is the OR of the
// tokens' words; also runs the same prep jobs as union_bits_kernel.
__global__ void __launch_bounds__(kUnionWarps * 32)
union_from_bits_kernel(const uint32_t *__restrict__ tok_in, int B, int f, int W, int G,
                       uint32_t *__restrict__ seg_bits, PrepJobs jobs) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int S = (B + G - 1) / G;
    for (int64_t i = gtid; i < (int64_t)S * W; i += stride) {
        const int s = (int)(i / W), w = (int)(i % W);
        uint32_t u = 0;
        for (int t = s * G; t < min(B, (s + 1) * G); ++t) u |= __ldg(tok_in + (int64_t)t * W + w);
        if (w == W - 1 && (f & 31)) u &= (1u << (f & 31)) - 1u;
        seg_bits[i] = u;
    }
    if (jobs.zero_out) {
        const int64_t n4 = jobs.zero_n / 4;
        for (int64_t i = gtid; i < n4; i += stride)
            reinterpret_cast<float4 *>(jobs.zero_out)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t i = n4 * 4 + gtid; i < jobs.zero_n; i += stride) jobs.zero_out[i] = 0.0f;
    }
}

constexpr int kCompactThreads = 1024;

// CTA s compacts segment s.  act_cum[s] = number of active neurons in
// segments 0..s (inclusive), the reference's cumulative convention
// (cuda/kernel.cu:590-593).
__global__ void __launch_bounds__(kCompactThreads)
compact_kernel(const uint32_t *__restrict__ seg_bits, int W, int f, int32_t *__restrict__ merge_idx,
               int32_t *__restrict__ act_cum, int32_t *__restrict__ counts) {
    __shared__ int warp_tot[33];
    __shared__ int prefix[kCompactThreads + 1];
    __shared__ int before;
    const int s = blockIdx.x;
    // Active neurons of all earlier segments.
    int acc = 0;
    for (int64_t i = threadIdx.x; i < (int64_t)s * W; i += blockDim.x) acc += __popc(seg_bits[i]);
    acc = __reduce_add_sync(0xffffffffu, acc);
    if (threadIdx.x == 0) before = 0;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) atomicAdd(&before, acc);

    const uint32_t *bits = seg_bits + (int64_t)s * W;
    int32_t *out = merge_idx + (int64_t)s * f;
    int carry = 0;
    for (int base = 0; base < W; base += kCompactThreads) {
        const int n = min(kCompactThreads, W - base);
        scan_popc(bits + base, n, prefix, warp_tot);
        const int w = base + threadIdx.x;
        if (threadIdx.x < n) {
            uint32_t word = bits[w];
            int p = carry + prefix[threadIdx.x];
            while (word) {
                int b = __ffs(word) - 1;
                word &= word - 1;
                out[p++] = w * 32 + b;
            }
        }
        carry += prefix[n];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        if (counts) counts[s] = carry;
        if (act_cum) act_cum[s] = before + carry;
    }
}

int launch_union_bits(const float *idx, int B, int f, int G, uint32_t *tok_bits, uint32_t *seg_bits,
                      const PrepJobs &jobs, cudaStream_t st) {
    const int W = words_of(f);
    int grid = (W + kUnionWarps - 1) / kUnionWarps;
    if (jobs.x16 || jobs.zero_out) grid = max(grid, num_sms());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kUnionWarps * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SPB_CUDA_TRY(cudaLaunchKernelEx(&cfg, union_bits_kernel, idx, B, f, W, G, tok_bits, seg_bits, jobs));
    return SPB_OK;
}

int launch_union_from_bits(const uint32_t *tok_in, int B, int f, int G, uint32_t *seg_bits, const PrepJobs &jobs,
                           cudaStream_t st) {
    const int W = words_of(f);
    const int S = (B + G - 1) / G;
    int grid = (S * W + 255) / 256;
    if (jobs.zero_out) grid = max(grid, num_sms());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(max(1, grid));
    cfg.blockDim = dim3(kUnionWarps * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SPB_CUDA_TRY(cudaLaunchKernelEx(&cfg, union_from_bits_kernel, tok_in, B, f, W, G, seg_bits, jobs));
    return SPB_OK;
}

int launch_compact(const uint32_t *seg_bits, int S, int f, int32_t *merge_idx, int32_t *act_cum, int32_t *counts,
                   cudaStream_t st) {
    compact_kernel<<<S, kCompactThreads, 0, st>>>(seg_bits, words_of(f), f, merge_idx, act_cum, counts);
    SPB_LAUNCH_CHECK("compact_kernel");
    return SPB_OK;
}

}  // namespace spb

// ---------------------------------------------------------------------------
// Allocation-free union entry point.
//
// Some callers cannot allocate device memory at the point where they need
// the union: code running inside a framework whose allocator owns the whole
// device, plug-ins that are handed only input and output buffers, and
// real-time paths that may not call cudaMalloc (it can synchronise the
// device).  spb_union_static serves them with the same kernels as spb_union,
// but its scratch -- the per-segment union bit words and the per-segment
// counts -- lives in the fixed device array below instead of a caller
// workspace.  The array is part of the library image: every GPU that loads
// the library holds it (256 KB) until the process exits.
namespace spb {
namespace {

constexpr int kUnionStaticWords = 1 << 16;  // 65536 u32 words = 256 KB

static __device__ __align__(256) uint32_t g_union_static_scratch[kUnionStaticWords];

// Device address of the array on the current device; looked up once per
// device (host code must not use the symbol itself as a device pointer).
int static_scratch_address(uint32_t **out) {
    static std::mutex mu;
    static std::vector<uint32_t *> addr;
    int dev = 0;
    SPB_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if ((int)addr.size() <= dev) addr.resize(dev + 1, nullptr);
    if (!addr[dev]) {
        void *p = nullptr;
        SPB_CUDA_TRY(cudaGetSymbolAddress(&p, g_union_static_scratch));
        addr[dev] = static_cast<uint32_t *>(p);
    }
    *out = addr[dev];
    return SPB_OK;
}

}  // namespace
}  // namespace spb

extern "C" int spb_union_static(const float *idx, int B, int f, int group, int32_t *merge_idx, int32_t *act_cum,
                                uint32_t *tok_bits, void *stream) {
    using namespace spb;
    if (!idx || !merge_idx || !act_cum) return fail(SPB_ERR_INVALID, "spb_union_static: null pointer");
    if (B <= 0 || f <= 0 || group < 0) return fail(SPB_ERR_INVALID, "spb_union_static: bad shape");
    const int G = group == 0 ? B : group;
    const int S = (B + G - 1) / G;
    const int W = words_of(f);
    // scratch: S*W union words, then S+1 counts (each region 64-word aligned)
    const int64_t words_bits = ((int64_t)S * W + 63) / 64 * 64;
    const int64_t need = words_bits + S + 1;
    if (need > kUnionStaticWords)
        return fail(SPB_ERR_UNSUPPORTED, "spb_union_static: segments x words (" + std::to_string(need) +
                                             " words of scratch) exceed the fixed 65536-word scratch array; "
                                             "use spb_union with a workspace");
    uint32_t *scratch = nullptr;
    if (int rc = static_scratch_address(&scratch)) return rc;
    uint32_t *seg_bits = scratch;
    int32_t *counts = reinterpret_cast<int32_t *>(scratch + words_bits);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Every segment word and count is rewritten by these launches, so nothing
    // left in the array by an earlier call is read.
    int rc = launch_union_bits(idx, B, f, G, tok_bits, seg_bits, PrepJobs{}, st);
    if (rc) return rc;
    return launch_compact(seg_bits, S, f, merge_idx, act_cum, counts, st);
}

