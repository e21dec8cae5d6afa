// Streaming single-launch FFN for small batches (B <= 4) on CUDA cores.
//
// One launch (one CTA per SM) does the whole layer -- batch union, gathered
// gate/up, ReLU*up, gathered down -- replacing get_idx_cuda + mm_up +
// relu_and_mul + convert_fp32_to_fp16 + mm_down (cuda/kernel.cu:566-816,
// 522-529, 321-356).
//
// Union.  Every CTA reads the B <= 4 label rows (f fp32 each, active if > 0)
// through L2 and builds the union words in shared memory itself, so no
// grid-wide step is needed (measured faster than sharing the words through a
// grid barrier: 7B, B = 2: 20.5 against 21.1 us).  The grid-barrier path,
// where each CTA scans its share of the 32-neuron words, publishes them and
// reads all words back, remains for larger token counts.  CTA 0
// zeroes `out` and publishes the launch number (taken from per-CTA tickets of
// a monotonic counter); the other CTAs check it only before their final
// reductions.
//
// Rows.  Every CTA rebuilds the ascending union list from the words (one
// block scan) and takes an equal contiguous share of it, so no CTA holds more
// than one neuron above the average.  For each of its neurons j one producer
// thread copies the three weight rows -- W_gate[j], W_up[j] and W_down[j],
// each contiguous because W_down is stored [f][d] -- into a ring of
// shared-memory stages with 1-D bulk copies (cp.async.bulk, completion
// counted as transaction bytes on an mbarrier).  With up to 8 stages of 24 KB
// (d = 4096, fp16) in flight per SM the HBM pipe stays full without register
// staging.  Launched with programmatic dependent launch (the prologue
// overlaps the previous kernel's tail).
//
// The 16 consumer warps split the hidden dimension: thread `tid` owns the
// 8-element chunks tid, tid + 512, ... of every row and keeps the
// fp16-rounded activations of those chunks in registers.  For fp16 weights
// the products use the sm_100 mixed-precision FMA (fp16 operands, fp32
// accumulator: the value fmaf((float)w, (float)x, acc) gives, without the
// conversions).  Per group of neurons the partial gate/up sums are
// reduce-scattered across each warp, summed over the warps in a fixed order
// through shared memory (one barrier per group), turned into
// h = fp16(ReLU(gate) * up) (or the dReLU form) with the per-token mask, and
// h * W_down[j] is accumulated into per-thread output registers.  At the end
// each thread adds its output chunk into `out` with vector fp32 reductions.
//
// Weight formats: fp16, Q8_0 and Q4_0 rows (spb_quant.cuh); quantised rows are
// dequantised from shared memory in registers with the oracle's arithmetic.
// Every wait is bounded (2 s of %globaltimer); on timeout the kernel records
// an error code in the workspace and finishes without waiting again.  After
// such an error the workspace must be zeroed before it is used again.
#include "spb_internal.h"
#include "spb_quant.cuh"
#include "spb_scan.cuh"
#include "tc_ptx.cuh"

namespace spb {

using namespace ptx;

namespace {

constexpr int kSfConsumers = 512;  // 16 consumer warps
constexpr int kSfWarps = kSfConsumers / 32;
constexpr int kSfThreads = kSfConsumers + 32;  // + producer warp
constexpr int kSfMaxStages = 16;
constexpr uint64_t kSfTimeoutNs = 2000000000ull;
constexpr size_t kSfSmemLimit = 227 * 1024;

enum : uint32_t { kErrSfFull = 11, kErrSfEmpty = 12, kErrSfZero = 13, kErrSfGrid = 14 };

struct SfCtl {
    uint64_t full[kSfMaxStages];
    uint64_t empty[kSfMaxStages];
    unsigned long long launch;
    volatile int abort;
    int U;
};

struct SfArgs {
    const uint8_t *wg, *wu, *wd;  // [f] rows of rb bytes
    const float *x;               // [B][d]
    const float *idx;             // [B][f] labels, or null with tok_in
    const uint32_t *tok_in;       // [B][W] per-token activity bits, or null
    const __half *bias_g, *bias_u;  // [f] fp16 gate / up biases, or null
    float *out;                   // [B][d]
    int32_t *merge;               // [f] or null
    int32_t *count;               // [1] or null
    uint32_t *err;
    uint32_t *seg_bits;              // [W] workspace (several-token union)
    uint32_t *tok_bits;              // [B][W] workspace
    unsigned long long *grid_bar;    // monotonic grid-barrier arrival counter
    unsigned long long *launch_ctr;  // monotonic CTA ticket counter
    unsigned long long *zero_flag;   // launch number + 1 once `out` is zeroed
    unsigned long long *trace;     // [grid][kSfTraceSlots] stamps, or null
    int B, d, f, W, act, per_token, stages, cap, local_union;
    int rb;           // row bytes (multiple of 16)
    int stage_bytes;  // 3 * rb
    int off_bits, off_nid, off_mask, off_red, off_stage;
};

// Stamps written when tracing is enabled (spb_trace_enable): 0 start,
// 1 union words ready, 2 first copy issued, 3 first stage consumed,
// 4 last copy issued, 5 consumers done, 7 end; 8 neurons of this CTA.
constexpr int kSfTraceSlots = 16;

__device__ __forceinline__ void bulk_copy(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool sf_wait(uint64_t *bar, uint32_t parity, SfCtl *ctl, uint32_t *err, uint32_t code) {
    if (mbar_test(bar, parity)) return true;
    if (ctl->abort) return false;
    const uint64_t t0 = globaltimer();
    while (!mbar_test(bar, parity)) {
        if (ctl->abort) return false;
        if (globaltimer() - t0 > kSfTimeoutNs) {
            atomicCAS(err, 0u, code);
            ctl->abort = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Grid-wide barrier over a monotonic 64-bit arrival counter (used by
// cooperative launches only, so every CTA is resident).  Arrival k of all
// launches belongs to the barrier ending at the next multiple of the grid
// size.
__device__ __forceinline__ unsigned long long grid_arrive(unsigned long long *ctr) {
    unsigned long long ticket;
    // release: the CTA's earlier writes (visible to thread 0 through the
    // preceding __syncthreads) are ordered before the arrival
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(ticket) : "l"(ctr) : "memory");
    return (ticket / gridDim.x + 1) * gridDim.x;
}

__device__ __forceinline__ void grid_wait(const unsigned long long *ctr, unsigned long long target, SfCtl *ctl,
                                          uint32_t *err) {
    if (ld_acquire_u64(ctr) >= target) return;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_u64(ctr) < target) {
        if (globaltimer() - t0 > kSfTimeoutNs) {
            atomicCAS(err, 0u, kErrSfGrid);
            ctl->abort = 1;
            return;
        }
        __nanosleep(32);
    }
}

// Mixed-precision FMA (sm_100): fp16 operands, exact product, fp32 addend and
// result -- the same value as fmaf((float)a, (float)b, c).
__device__ __forceinline__ float fma_f16(unsigned short a, unsigned short b, float c) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
    return d;
}
__device__ __forceinline__ unsigned short lo16(uint32_t v) { return (unsigned short)(v & 0xffffu); }
__device__ __forceinline__ unsigned short hi16(uint32_t v) { return (unsigned short)(v >> 16); }

// acc + sum_e w[e] * x[e] over 8 packed fp16 values.
__device__ __forceinline__ float dot8_f16(const uint4 &w, const uint32_t (&x)[4], float acc) {
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        acc = fma_f16(lo16(wv[q]), lo16(x[q]), acc);
        acc = fma_f16(hi16(wv[q]), hi16(x[q]), acc);
    }
    return acc;
}

template <int N>
struct Log2 {
    static constexpr int value = 1 + Log2<N / 2>::value;
};
template <>
struct Log2<1> {
    static constexpr int value = 0;
};

// Warp reduce-scatter of N values per lane: each halving step exchanges half
// of the remaining values with the lane O apart and keeps the other half; once
// one value is left, a butterfly over the remaining offsets completes it.
// Lane l ends with the warp sum of value l >> (5 - log2 N): N - 1 shuffles
// plus the butterfly, against 5 N for one butterfly per value.
template <int N, int O>
struct ReduceScatter {
    static __device__ __forceinline__ float run(float *cur, int lane) {
        constexpr int H = N / 2;
        const bool upper = (lane & O) != 0;
#pragma unroll
        for (int i = 0; i < H; ++i) {
            const float send = upper ? cur[i] : cur[i + H];
            const float keep = upper ? cur[i + H] : cur[i];
            cur[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
        }
        return ReduceScatter<H, O / 2>::run(cur, lane);
    }
};
template <int O>
struct ReduceScatter<1, O> {
    static __device__ __forceinline__ float run(float *cur, int) {
        float v = cur[0];
#pragma unroll
        for (int o = O; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        return v;
    }
};

__device__ __forceinline__ float sf_act(float g, float u, int act) {
    g = fmaxf(g, 0.0f);
    return act == SPB_ACT_RELU_RELU_MUL ? g * fmaxf(u, 0.0f) : g * u;
}

// NT: tokens (B <= NT), CPT: 8-element chunks per consumer thread
// (ceil(d / 4096)).
template <int NT, int WT, int CPT>
__global__ void __launch_bounds__(kSfThreads, 1) stream_ffn_kernel(const SfArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    SfCtl *ctl = reinterpret_cast<SfCtl *>(smem);
    int *nid = reinterpret_cast<int *>(smem + a.off_nid);
    uint8_t *mask = smem + a.off_mask;
    float *red = reinterpret_cast<float *>(smem + a.off_red);  // [2][kSfWarps][V]
    uint8_t *stage = smem + a.off_stage;
    // neurons per reduction barrier (fewer where registers are short)
    constexpr int G = (CPT == 1 && NT <= 2) ? 4 : 2;
    constexpr int V = 2 * G * NT;  // values reduced per group (8, 16 or 32)
    constexpr int kSh = 5 - Log2<V>::value;
    constexpr bool kF16 = WT == SPB_W_F16;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = a.stages;
    const int d8 = a.d >> 3;
    unsigned long long *tr = a.trace ? a.trace + (size_t)blockIdx.x * kSfTraceSlots : nullptr;
    if (tr && tid == 0) tr[0] = globaltimer();

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], kSfWarps);
        }
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // With a programmatic dependent launch the previous kernel may still be
    // finishing: wait for it before touching global memory.
    grid_dependency_wait();

    // Activations: loads issued now, converted once the union is known.
    float xraw[CPT][NT][8];
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
        const int c = tid + k * kSfConsumers;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
            if (warp < kSfWarps && c < d8 && t < a.B) {
                const float4 *xp = reinterpret_cast<const float4 *>(a.x + (int64_t)t * a.d + c * 8);
                v0 = __ldg(xp);
                v1 = __ldg(xp + 1);
            }
            xraw[k][t][0] = v0.x, xraw[k][t][1] = v0.y, xraw[k][t][2] = v0.z, xraw[k][t][3] = v0.w;
            xraw[k][t][4] = v1.x, xraw[k][t][5] = v1.y, xraw[k][t][6] = v1.z, xraw[k][t][7] = v1.w;
        }
    }

    // ---- launch number; CTA 0 zeroes `out` ----
    // Every CTA takes a ticket from a monotonic counter; launches are stream
    // ordered (a dependent launch waits above for its predecessor), so all
    // tickets of one launch precede the next launch's and ticket / grid is
    // the launch number.  CTA 0 zeroes `out` and then publishes launch + 1;
    // the other CTAs check the flag only before their final reductions.
    if (tid == 0) ctl->launch = atomicAdd(a.launch_ctr, 1ull) / gridDim.x;
    if (blockIdx.x == 0) {
        const int n4 = a.B * a.d / 4;
        for (int q = tid; q < n4; q += kSfThreads)
            reinterpret_cast<float4 *>(a.out)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // ---- the batch union: union words [W] and token words [NT][W] ----
    uint32_t *ubits = reinterpret_cast<uint32_t *>(smem + a.off_bits);
    uint32_t *tbits = ubits + a.W;
    if (a.tok_in) {
        // Per-token bits from the caller: every CTA reads the B x W words
        // (1.4 KB per token at f = 11008) through L2 -- no grid-wide step.
        for (int w = tid; w < a.W; w += kSfThreads) {
            const uint32_t last = (w == a.W - 1 && (a.f & 31)) ? (1u << (a.f & 31)) - 1u : ~0u;
            uint32_t un = 0;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const uint32_t bt = t < a.B ? (__ldg(a.tok_in + (int64_t)t * a.W + w) & last) : 0u;
                if (t < a.B) tbits[t * a.W + w] = bt;
                un |= bt;
            }
            ubits[w] = un;
        }
    } else if (a.local_union) {
        // Up to four tokens: every CTA reads the whole label rows (f fp32, active if
        // > 0) through L2 and builds the words itself -- no grid-wide step.
        if ((a.f & 3) == 0 && (reinterpret_cast<uintptr_t>(a.idx) & 15u) == 0) {
            // float4 loads: lane l of a warp covers neurons 4(q0 + l) .. +3; eight
            // lanes' nibbles form one 32-neuron word.
            constexpr int UR = NT == 1 ? 8 : (NT == 2 ? 4 : 2);  // rows of 544 float4 in flight
            const int nq = a.f >> 2;
            for (int base = 0; base < nq; base += UR * kSfThreads) {
                float4 v[UR][NT];
    #pragma unroll
                for (int u = 0; u < UR; ++u) {
                    const int q = base + u * kSfThreads + warp * 32 + lane;
    #pragma unroll
                    for (int t = 0; t < NT; ++t)
                        v[u][t] = (q < nq && t < a.B) ? __ldg(reinterpret_cast<const float4 *>(a.idx + (int64_t)t * a.f) + q)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                }
    #pragma unroll
                for (int u = 0; u < UR; ++u) {
                    const int q = base + u * kSfThreads + warp * 32 + lane;
                    uint32_t un = 0;
    #pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        uint32_t nib = (v[u][t].x > 0.f ? 1u : 0u) | (v[u][t].y > 0.f ? 2u : 0u) |
                                       (v[u][t].z > 0.f ? 4u : 0u) | (v[u][t].w > 0.f ? 8u : 0u);
                        nib <<= 4 * (lane & 7);
                        nib |= __shfl_xor_sync(0xffffffffu, nib, 1);
                        nib |= __shfl_xor_sync(0xffffffffu, nib, 2);
                        nib |= __shfl_xor_sync(0xffffffffu, nib, 4);
                        un |= nib;
                        if ((lane & 7) == 0 && q < nq && t < a.B) tbits[t * a.W + (q >> 3)] = nib;
                    }
                    if ((lane & 7) == 0 && q < nq) ubits[q >> 3] = un;
                }
            }
        } else {
            for (int w = warp; w < a.W; w += kSfThreads / 32) {
                const int j = w * 32 + lane;
                float lab[NT];
    #pragma unroll
                for (int t = 0; t < NT; ++t) lab[t] = (j < a.f && t < a.B) ? __ldg(a.idx + (int64_t)t * a.f + j) : 0.0f;
                uint32_t un = 0;
    #pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const uint32_t bt = __ballot_sync(0xffffffffu, lab[t] > 0.0f);
                    un |= bt;
                    if (lane == 0 && t < a.B) tbits[t * a.W + w] = bt;
                }
                if (lane == 0) ubits[w] = un;
            }
        }
    } else {
        // Several tokens: each CTA scans its share of the words and publishes
        // them; after a grid barrier (the launch is cooperative) every CTA
        // reads all words back.  Reading all B label rows in every CTA would
        // cost B x f x 4 bytes of L2 traffic per SM.
        const int w0 = (int)((int64_t)a.W * blockIdx.x / gridDim.x);
        const int w1 = (int)((int64_t)a.W * (blockIdx.x + 1) / gridDim.x);
        for (int w = w0 + warp; w < w1; w += kSfThreads / 32) {
            const int j = w * 32 + lane;
            float lab[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) lab[t] = (j < a.f && t < a.B) ? __ldg(a.idx + (int64_t)t * a.f + j) : 0.0f;
            uint32_t un = 0;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const uint32_t bt = __ballot_sync(0xffffffffu, lab[t] > 0.0f);
                un |= bt;
                if (lane == 0 && t < a.B) a.tok_bits[(int64_t)t * a.W + w] = bt;
            }
            if (lane == 0) a.seg_bits[w] = un;
        }
        __syncthreads();
        if (tid == 0) grid_wait(a.grid_bar, grid_arrive(a.grid_bar), ctl, a.err);
        __syncthreads();
        for (int w = tid; w < a.W; w += kSfThreads) {
            ubits[w] = __ldcg(a.seg_bits + w);
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (t < a.B) tbits[t * a.W + w] = __ldcg(a.tok_bits + (int64_t)t * a.W + w);
        }
    }
    __syncthreads();
    if (blockIdx.x == 0 && tid == 0) {
        __threadfence();
        st_release_u64(a.zero_flag, ctl->launch + 1);
    }
    if (tr && tid == 0) tr[1] = globaltimer();

    // ---- phase 2: this CTA's share of the ascending union list ----
    // One pass: each thread loads KW consecutive union words and their token
    // words, the block scans the popcounts, and each thread emits the ids
    // (and token masks) of its words that fall in [p0, p1).
    {
        constexpr int KW = 2;  // words per thread: W <= 1088 (f <= 34816)
        int *wsum = reinterpret_cast<int *>(smem + a.off_red);  // [kSfThreads / 32 + 1]
        uint32_t wb[KW], tb[KW][NT];
        int c = 0;
#pragma unroll
        for (int k = 0; k < KW; ++k) {
            const int w = tid * KW + k;
            wb[k] = w < a.W ? ubits[w] : 0u;
#pragma unroll
            for (int t = 0; t < NT; ++t)
                tb[k][t] = (a.per_token && t < a.B && w < a.W) ? tbits[t * a.W + w] : 0xffffffffu;
            c += __popc(wb[k]);
        }
        const int incl = warp_incl_scan(c);
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const int v = lane < kSfThreads / 32 ? wsum[lane] : 0;
            const int vi = warp_incl_scan(v);
            if (lane < kSfThreads / 32) wsum[lane] = vi - v;
            if (lane == 31) wsum[kSfThreads / 32] = vi;
        }
        __syncthreads();
        const int U = wsum[kSfThreads / 32];
        const int p0 = (int)((int64_t)U * blockIdx.x / gridDim.x);
        const int p1 = (int)((int64_t)U * (blockIdx.x + 1) / gridDim.x);
        int pos = wsum[warp] + incl - c;
        if (pos < p1 && pos + c > p0) {
#pragma unroll
            for (int k = 0; k < KW; ++k) {
                uint32_t word = wb[k];
                while (word) {
                    const int b = __ffs(word) - 1;
                    word &= word - 1;
                    if (pos >= p0 && pos < p1) {
                        const int j = (tid * KW + k) * 32 + b;
                        uint32_t m = 0;
#pragma unroll
                        for (int t = 0; t < NT; ++t) m |= ((tb[k][t] >> b) & 1u) << t;
                        nid[pos - p0] = j;
                        mask[pos - p0] = (uint8_t)m;
                        if (a.merge) a.merge[pos] = j;
                    }
                    ++pos;
                }
            }
        }
        if (tid == 0) ctl->U = p1 - p0;
        if (a.count && blockIdx.x == 0 && tid == 0) *a.count = U;
        __syncthreads();
    }
    const int n = ctl->U;
    if (tr && tid == 0) tr[8] = (unsigned long long)n;

    if (warp == kSfWarps) {
        // ---- producer ----
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;  // parity of the empty phase to wait for on wrap
            for (int i = 0; i < n; ++i) {
                if (i >= S && !sf_wait(&ctl->empty[s], ph ^ 1u, ctl, a.err, kErrSfEmpty)) break;
                const int64_t off = (int64_t)nid[i] * a.rb;
                uint8_t *dst = stage + (size_t)s * a.stage_bytes;
                mbar_arrive_expect_tx(&ctl->full[s], (uint32_t)a.stage_bytes);
                bulk_copy(smem_u32(dst), a.wg + off, a.rb, &ctl->full[s]);
                bulk_copy(smem_u32(dst + a.rb), a.wu + off, a.rb, &ctl->full[s]);
                bulk_copy(smem_u32(dst + 2 * a.rb), a.wd + off, a.rb, &ctl->full[s]);
                if (tr && i == 0) tr[2] = globaltimer();
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            if (tr) tr[4] = globaltimer();
        }
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        // The consumers wait for every issued stage before they finish, so no
        // copy is in flight into this CTA's shared memory when it exits.
    } else {
        // ---- consumers ----
        // Activations of the owned chunks, rounded to fp16 as the reference
        // does before its products (cuda/kernel.cu:978).  fp16 weights: packed
        // fp16 pairs for the mixed-precision FMA; quantised weights: fp32.
        uint32_t xh[CPT][NT][4];
        float xf[kF16 ? 1 : CPT][kF16 ? 1 : NT][8];
#pragma unroll
        for (int k = 0; k < CPT; ++k)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if constexpr (kF16) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const __half2 p = __floats2half2_rn(xraw[k][t][2 * q], xraw[k][t][2 * q + 1]);
                        xh[k][t][q] = *reinterpret_cast<const uint32_t *>(&p);
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) xf[k][t][e] = __half2float(__float2half_rn(xraw[k][t][e]));
                }
            }
        float acc[CPT][NT][8];
#pragma unroll
        for (int k = 0; k < CPT; ++k)
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[k][t][e] = 0.0f;

        int s_next = 0;
        uint32_t ph_next = 0;  // parity of the full phase of stage s_next
        bool failed = false;
        for (int i0 = 0, grp = 0; i0 < n; i0 += G, ++grp) {
            int st[G];
            uint32_t hmask = 0;  // bit g*NT + t: h of (neuron i0+g, token t) is kept
            float part[V];
#pragma unroll
            for (int v = 0; v < V; ++v) part[v] = 0.0f;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                st[g] = s_next;
                const int i = i0 + g;
                if (i < n) {
                    const int s = s_next;
                    if (!failed && !sf_wait(&ctl->full[s], ph_next, ctl, a.err, kErrSfFull)) failed = true;
                    if (++s_next == S) {
                        s_next = 0;
                        ph_next ^= 1u;
                    }
                    if (tr && tid == 0 && i == 0) tr[3] = globaltimer();
                    const uint32_t m = mask[i];
                    hmask |= (m & ((1u << NT) - 1u) & ((1u << a.B) - 1u)) << (g * NT);
                    const uint8_t *row = stage + (size_t)s * a.stage_bytes;
#pragma unroll
                    for (int k = 0; k < CPT; ++k) {
                        const int c = tid + k * kSfConsumers;
                        if (c >= d8) continue;
                        if constexpr (kF16) {
                            const uint4 vg = *reinterpret_cast<const uint4 *>(row + (size_t)c * 16);
                            const uint4 vu = *reinterpret_cast<const uint4 *>(row + a.rb + (size_t)c * 16);
#pragma unroll
                            for (int t = 0; t < NT; ++t) {
                                part[g * NT + t] = dot8_f16(vg, xh[k][t], part[g * NT + t]);
                                part[(G + g) * NT + t] = dot8_f16(vu, xh[k][t], part[(G + g) * NT + t]);
                            }
                        } else {
                            float wg[8], wu[8];
                            deq8_smem<WT>(row, a.d, c, wg);
                            deq8_smem<WT>(row + a.rb, a.d, c, wu);
#pragma unroll
                            for (int t = 0; t < NT; ++t) {
                                float sg = part[g * NT + t], su = part[(G + g) * NT + t];
#pragma unroll
                                for (int e = 0; e < 8; ++e) {
                                    sg = fmaf(wg[e], xf[k][t][e], sg);
                                    su = fmaf(wu[e], xf[k][t][e], su);
                                }
                                part[g * NT + t] = sg;
                                part[(G + g) * NT + t] = su;
                            }
                        }
                    }
                }
            }
            // Reduce-scatter across the warp: lane l ends with the warp's sum of
            // value l >> kSh (lanes sharing a value hold the same sum).
            const float mine = ReduceScatter<V, 16>::run(part, lane);
            float *rbuf = red + (size_t)(grp & 1) * kSfWarps * V;
            if ((lane & ((1 << kSh) - 1)) == 0) rbuf[warp * V + (lane >> kSh)] = mine;
            named_bar(1, kSfConsumers);
            // lane v < V sums value v over the warps in a fixed order (every
            // warp computes the same sums, which saves a second barrier)
            float tot = 0.0f;
            if (lane < V) {
#pragma unroll
                for (int w = 0; w < kSfWarps; ++w) tot += rbuf[w * V + lane];
            }
            // lanes v < G*NT hold gate sums; the matching up sum is in lane v + G*NT
            const float up = __shfl_sync(0xffffffffu, tot, (lane + G * NT) & 31);
            uint32_t hbits = 0;  // fp16 h of (neuron lane / NT, token lane % NT)
            if (lane < G * NT && ((hmask >> lane) & 1u)) {
                float gs = tot, us = up;
                if (a.bias_g || a.bias_u) {  // sparse bias add (cuda/kernel.cu:818-830)
                    const int jn = nid[i0 + lane / NT];
                    if (a.bias_g) gs += __half2float(a.bias_g[jn]);
                    if (a.bias_u) us += __half2float(a.bias_u[jn]);
                }
                hbits = __half_as_ushort(__float2half_rn(sf_act(gs, us, a.act)));
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                uint32_t h[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) h[t] = __shfl_sync(0xffffffffu, hbits, g * NT + t);
                if (i0 + g < n) {
                    const uint8_t *row = stage + (size_t)st[g] * a.stage_bytes + 2 * (size_t)a.rb;
#pragma unroll
                    for (int k = 0; k < CPT; ++k) {
                        const int c = tid + k * kSfConsumers;
                        if (c >= d8) continue;
                        if constexpr (kF16) {
                            const uint4 vd = *reinterpret_cast<const uint4 *>(row + (size_t)c * 16);
                            const uint32_t wv[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
                            for (int t = 0; t < NT; ++t) {
                                const unsigned short ht = (unsigned short)h[t];
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    acc[k][t][2 * q] = fma_f16(lo16(wv[q]), ht, acc[k][t][2 * q]);
                                    acc[k][t][2 * q + 1] = fma_f16(hi16(wv[q]), ht, acc[k][t][2 * q + 1]);
                                }
                            }
                        } else {
                            float wd[8];
                            deq8_smem<WT>(row, a.d, c, wd);
#pragma unroll
                            for (int t = 0; t < NT; ++t) {
                                const float hf = __half2float(__ushort_as_half((unsigned short)h[t]));
#pragma unroll
                                for (int e = 0; e < 8; ++e) acc[k][t][e] = fmaf(hf, wd[e], acc[k][t][e]);
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ctl->empty[st[g]]);
                }
            }
        }
        if (tr && tid == 0) tr[5] = globaltimer();

        // `out` must have been zeroed by CTA 0 (long done in practice).
        if (ld_acquire_u64(a.zero_flag) < ctl->launch + 1) {
            const uint64_t t0 = globaltimer();
            while (ld_acquire_u64(a.zero_flag) < ctl->launch + 1) {
                if (ctl->abort || globaltimer() - t0 > kSfTimeoutNs) {
                    atomicCAS(a.err, 0u, kErrSfZero);
                    ctl->abort = 1;
                    break;
                }
                __nanosleep(128);
            }
        }
        if (!ctl->abort) {
#pragma unroll
            for (int k = 0; k < CPT; ++k) {
                const int c = tid + k * kSfConsumers;
                if (c >= d8) continue;
                // Every CTA adds into the same [B][d] addresses at about the
                // same time: CTA b starts at token b mod NT, so concurrent
                // CTAs spread over the tokens' rows (one static order per
                // rotation, so the registers stay statically indexed).
                const int rot = (int)(blockIdx.x & (NT - 1));
#pragma unroll
                for (int r = 0; r < NT; ++r) {
                    if (rot != r) continue;
#pragma unroll
                    for (int q = 0; q < NT; ++q) {
                        const int t = (q + r) % NT;
                        if (t < a.B) {
                            float4 *o = reinterpret_cast<float4 *>(a.out + (int64_t)t * a.d + c * 8);
                            atomicAdd(o, make_float4(acc[k][t][0], acc[k][t][1], acc[k][t][2], acc[k][t][3]));
                            atomicAdd(o + 1, make_float4(acc[k][t][4], acc[k][t][5], acc[k][t][6], acc[k][t][7]));
                        }
                    }
                }
            }
        }
    }
    if (tr) {
        __syncthreads();
        if (tid == 0) tr[7] = globaltimer();
    }
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int NT, int WT, int CPT>
int launch_sf(const StreamFfnArgs &fa, cudaStream_t st) {
    SfArgs a{};
    const int64_t rb = row_bytes_of<WT>(fa.d);
    const int grid = num_sms();
    a.wg = static_cast<const uint8_t *>(fa.wg);
    a.wu = static_cast<const uint8_t *>(fa.wu);
    a.wd = static_cast<const uint8_t *>(fa.wd);
    a.x = fa.x;
    a.idx = fa.idx;
    a.tok_in = fa.tok_in;
    a.bias_g = fa.bias_g;
    a.bias_u = fa.bias_u;
    a.out = fa.out;
    a.merge = fa.merge_out;
    a.count = fa.count_out;
    a.err = fa.err;
    a.seg_bits = fa.seg_bits;
    a.tok_bits = fa.tok_bits;
    a.grid_bar = fa.grid_bar;
    a.local_union = fa.B <= 4 || fa.tok_in != nullptr;
    a.launch_ctr = fa.launch_ctr;
    a.zero_flag = fa.zero_flag;
    a.B = fa.B;
    a.d = fa.d;
    a.f = fa.f;
    a.W = words_of(fa.f);
    a.act = fa.act;
    a.per_token = fa.per_token;
    a.rb = (int)rb;
    a.stage_bytes = (int)(3 * rb);
    a.cap = fa.f / grid + 2;
    size_t off = align_up(sizeof(SfCtl), 16);
    a.off_nid = (int)off;
    off = align_up(off + sizeof(int) * a.cap, 16);
    a.off_mask = (int)off;
    off = align_up(off + a.cap, 16);
    a.off_red = (int)off;
    off = align_up(off + sizeof(float) * 2 * kSfWarps * 32, 1024);
    a.off_stage = (int)off;
    int S = (int)((kSfSmemLimit - off) / (size_t)a.stage_bytes);
    if (S > kSfMaxStages) S = kSfMaxStages;
    if (S < 2) return fail(SPB_ERR_UNSUPPORTED, "stream ffn: rows too long for shared-memory staging");
    a.stages = S;
    size_t smem = off + (size_t)S * a.stage_bytes;
    // the union words live in the stage ring before the first copy
    a.off_bits = a.off_stage;
    const size_t need_bits = a.off_stage + sizeof(uint32_t) * (size_t)a.W * (1 + NT);
    if (need_bits > smem) smem = need_bits;
    if (smem > kSfSmemLimit) return fail(SPB_ERR_UNSUPPORTED, "stream ffn: shared memory");
    a.trace = static_cast<unsigned long long *>(trace_buffer((size_t)grid * kSfTraceSlots));
    auto kern = stream_ffn_kernel<NT, WT, CPT>;
    if (int rc = ensure_smem((const void *)kern, smem)) return rc;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kSfThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    // programmatic dependent launch: the launch overlaps the previous
    // kernel's tail; the kernel waits for it before touching global memory.
    // Cooperative: CTAs wait for CTA 0's zeroed output (and, with several
    // labelled tokens, for the grid barrier), so all of them must be resident.
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    SPB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
    return SPB_OK;
}

template <int WT>
int launch_sf_wt(const StreamFfnArgs &fa, cudaStream_t st) {
    const int cpt = (fa.d / 8 + kSfConsumers - 1) / kSfConsumers;
    if (cpt == 1) {
        if (fa.B <= 1) return launch_sf<1, WT, 1>(fa, st);
        if (fa.B <= 2) return launch_sf<2, WT, 1>(fa, st);
        return launch_sf<4, WT, 1>(fa, st);
    }
    if (fa.B <= 1) return launch_sf<1, WT, 2>(fa, st);
    return launch_sf<2, WT, 2>(fa, st);
}


// ---- drop-in up projection (group-union semantics) --------------------------
//
// up_mul_mat_cuda_sparse / gate_and_up_mul_mat_cuda_sparse (cuda/kernel.cu:
// 595-704, 971-1010) compute, for each group of G <= 8 tokens, the products of
// the group's compacted neuron list with the group's tokens, written
// compacted: dst[t][r] = W[merge_idx[g][r]] . fp16(x[t]).  Here the CTAs are
// split evenly over the groups and each takes an equal share of its group's
// list, so the group's activations stay in registers (fp16 pairs) for the
// whole launch.  Rows stream through the same bulk-copy ring as the fused
// kernel; per group of 4 (up) or 2 (gate + up) neurons the 32 partial sums
// are reduce-scattered across the warp, summed over the warps in fixed order
// and written by warp 0.
struct DropUpArgs {
    const uint8_t *wg, *wu;     // [f][d] fp16 rows (wu null: up only)
    const float *x;             // [B][d]
    float *gdst, *udst;         // [B][f] compacted
    const int32_t *merge_idx;   // [S][f]
    const int32_t *act_cum;     // [S] cumulative counts
    int B, d, f, G, S, stages, cap, rb, stage_bytes;
    int off_nid, off_red, off_stage;
    uint32_t *err;
};

template <int NMAT>
__global__ void __launch_bounds__(kSfThreads, 1) dropin_up_stream_kernel(const DropUpArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    SfCtl *ctl = reinterpret_cast<SfCtl *>(smem);
    int *nid = reinterpret_cast<int *>(smem + a.off_nid);
    float *red = reinterpret_cast<float *>(smem + a.off_red);  // [2][kSfWarps][32]
    uint8_t *stage = smem + a.off_stage;
    constexpr int NT = 8;                 // tokens per group (G <= 8)
    constexpr int GN = NMAT == 1 ? 4 : 2;  // neurons per reduction barrier
    constexpr int V = GN * NT * NMAT;      // = 32 values per group of neurons
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = a.stages;

    // this CTA's group and share of the group's list
    const int per = gridDim.x / a.S;  // CTAs per group (the host keeps grid >= S)
    const int sg = blockIdx.x / per, local = blockIdx.x - sg * per;
    if (sg >= a.S) return;
    const int n_s = a.act_cum[sg] - (sg > 0 ? a.act_cum[sg - 1] : 0);
    const int p0 = (int)((int64_t)n_s * local / per), p1 = (int)((int64_t)n_s * (local + 1) / per);
    const int n = p1 - p0;
    const int t0 = sg * a.G, tend = min(a.B, t0 + a.G);

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], kSfWarps);
        }
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = tid; i < n; i += kSfThreads) nid[i] = a.merge_idx[(int64_t)sg * a.f + p0 + i];
    __syncthreads();

    if (warp == kSfWarps) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int i = 0; i < n; ++i) {
                if (i >= S && !sf_wait(&ctl->empty[s], ph ^ 1u, ctl, a.err, kErrSfEmpty)) break;
                const int64_t off = (int64_t)nid[i] * a.rb;
                uint8_t *dst = stage + (size_t)s * a.stage_bytes;
                mbar_arrive_expect_tx(&ctl->full[s], (uint32_t)a.stage_bytes);
                bulk_copy(smem_u32(dst), a.wg + off, a.rb, &ctl->full[s]);
                if (NMAT == 2) bulk_copy(smem_u32(dst + a.rb), a.wu + off, a.rb, &ctl->full[s]);
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        return;
    }

    // consumers: this thread's 8-element chunk of d for the group's tokens
    const int c = tid;  // d <= 4096: one chunk per thread
    uint32_t xh[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
        if (c < (a.d >> 3) && t0 + t < tend) {
            const float4 *xp = reinterpret_cast<const float4 *>(a.x + (int64_t)(t0 + t) * a.d + c * 8);
            v0 = __ldg(xp);
            v1 = __ldg(xp + 1);
        }
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const __half2 p = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
            xh[t][q] = *reinterpret_cast<const uint32_t *>(&p);
        }
    }
    const bool own = c < (a.d >> 3);
    int s_next = 0;
    uint32_t ph_next = 0;
    bool failed = false;
    for (int i0 = 0, grp = 0; i0 < n; i0 += GN, ++grp) {
        int st[GN];
        float part[V];
#pragma unroll
        for (int v = 0; v < V; ++v) part[v] = 0.0f;
#pragma unroll
        for (int g = 0; g < GN; ++g) {
            st[g] = s_next;
            if (i0 + g < n) {
                const int s = s_next;
                if (!failed && !sf_wait(&ctl->full[s], ph_next, ctl, a.err, kErrSfFull)) failed = true;
                if (++s_next == S) {
                    s_next = 0;
                    ph_next ^= 1u;
                }
                if (own) {
                    const uint8_t *row = stage + (size_t)s * a.stage_bytes;
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        const uint4 w = *reinterpret_cast<const uint4 *>(row + m * a.rb + (size_t)c * 16);
#pragma unroll
                        for (int t = 0; t < NT; ++t)
                            part[(m * GN + g) * NT + t] = dot8_f16(w, xh[t], part[(m * GN + g) * NT + t]);
                    }
                }
            }
        }
        const float mine = ReduceScatter<V, 16>::run(part, lane);  // lane l: value l
        float *rbuf = red + (size_t)(grp & 1) * kSfWarps * V;
        rbuf[warp * V + lane] = mine;
        named_bar(1, kSfConsumers);
        // the rows of this group are no longer needed
#pragma unroll
        for (int g = 0; g < GN; ++g)
            if (i0 + g < n && lane == 0) mbar_arrive(&ctl->empty[st[g]]);
        if (warp == 0) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kSfWarps; ++w) tot += rbuf[w * V + lane];
            const int m = lane / (GN * NT), g = (lane / NT) % GN, t = lane % NT;
            if (i0 + g < n && t0 + t < tend) {
                float *dst = m ? a.udst : a.gdst;
                dst[(int64_t)(t0 + t) * a.f + p0 + i0 + g] = tot;
            }
        }
    }
}

template <int NMAT>
int launch_dropin_up_stream_t(const DropUpArgs &in, cudaStream_t st) {
    DropUpArgs a = in;
    const int grid = num_sms();
    const int per = grid / a.S;
    a.cap = a.f / per + 2;
    a.rb = a.d * 2;
    a.stage_bytes = NMAT * a.rb;
    size_t off = align_up(sizeof(SfCtl), 16);
    a.off_nid = (int)off;
    off = align_up(off + sizeof(int) * a.cap, 16);
    a.off_red = (int)off;
    off = align_up(off + sizeof(float) * 2 * kSfWarps * 32, 1024);
    a.off_stage = (int)off;
    int S = (int)((kSfSmemLimit - off) / (size_t)a.stage_bytes);
    if (S > kSfMaxStages) S = kSfMaxStages;
    if (S < 2) return fail(SPB_ERR_UNSUPPORTED, "drop-in up: rows too long for shared-memory staging");
    a.stages = S;
    const size_t smem = off + (size_t)S * a.stage_bytes;
    auto kern = dropin_up_stream_kernel<NMAT>;
    if (int rc = ensure_smem((const void *)kern, smem)) return rc;
    kern<<<per * a.S, kSfThreads, smem, st>>>(a);
    SPB_LAUNCH_CHECK("dropin_up_stream_kernel");
    return SPB_OK;
}

}  // namespace

bool stream_ffn_supported(int wtype, int B, int d) {
    if (B < 1 || B > 4 || d % 64 != 0) return false;
    const int cpt = (d / 8 + kSfConsumers - 1) / kSfConsumers;
    if (cpt > 2 || (cpt == 2 && B > 2)) return false;
    const int64_t rb = wtype == SPB_W_F16    ? row_bytes_of<SPB_W_F16>(d)
                       : wtype == SPB_W_Q8_0 ? row_bytes_of<SPB_W_Q8_0>(d)
                                             : row_bytes_of<SPB_W_Q4_0>(d);
    return rb % 16 == 0;
}

bool dropin_up_stream_supported(int B, int d, int G) {
    const int S = (B + G - 1) / G;
    return G >= 1 && G <= 8 && d % 64 == 0 && d <= 4096 && S <= num_sms();
}

int launch_dropin_up_stream(const __half *wg, const __half *wu, const float *x, float *gate_dst, float *up_dst,
                            const int32_t *merge_idx, const int32_t *act_cum, int B, int d, int f, int G,
                            uint32_t *err, cudaStream_t st) {
    DropUpArgs a{};
    a.wg = reinterpret_cast<const uint8_t *>(wg);
    a.wu = reinterpret_cast<const uint8_t *>(wu);
    a.x = x;
    a.gdst = gate_dst;
    a.udst = up_dst;
    a.merge_idx = merge_idx;
    a.act_cum = act_cum;
    a.B = B;
    a.d = d;
    a.f = f;
    a.G = G;
    a.S = (B + G - 1) / G;
    a.err = err;
    return wu ? launch_dropin_up_stream_t<2>(a, st) : launch_dropin_up_stream_t<1>(a, st);
}

int launch_stream_ffn(const StreamFfnArgs &a, cudaStream_t st) {
    switch (a.wtype) {
        case SPB_W_F16: return launch_sf_wt<SPB_W_F16>(a, st);
        case SPB_W_Q8_0: return launch_sf_wt<SPB_W_Q8_0>(a, st);
        case SPB_W_Q4_0: return launch_sf_wt<SPB_W_Q4_0>(a, st);
        default: return fail(SPB_ERR_INVALID, "stream ffn: unknown weight type");
    }
}

}  // namespace spb
