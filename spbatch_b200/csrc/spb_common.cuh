// Shared device/host helpers of the B200 sparse-FFN library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "spb.h"

namespace spb {

constexpr int kWarp = 32;
constexpr int kNumSMs = 148;  // B200; the launch code queries the real count

// ---- host-side error plumbing -------------------------------------------
void set_error(const std::string &msg);
int fail(int status, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);
int num_sms();
// Raises a kernel's dynamic shared-memory limit once per (device, kernel)
// and only when a larger size is requested, so calls made while a stream is
// being captured into a CUDA graph do not repeat the attribute update.
int ensure_smem(const void *kernel, size_t bytes);
// Device buffer for per-CTA phase timestamps when tracing is enabled on the
// current device and large enough for `slots` u64 entries; otherwise null.
void *trace_buffer(size_t slots);

#define SPB_CUDA_TRY(call)                                       \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return ::spb::cuda_fail(e_, #call); \
    } while (0)

#define SPB_LAUNCH_CHECK(what)                                     \
    do {                                                           \
        cudaError_t e_ = cudaGetLastError();                       \
        if (e_ != cudaSuccess) return ::spb::cuda_fail(e_, what);  \
    } while (0)

// ---- workspace layout ---------------------------------------------------
// All regions are 256-byte aligned slices of one caller-owned buffer.  The
// first 4 bytes hold a sticky device error code (0 = none) that kernels set
// instead of trapping when a bounded wait runs out; nothing clears it but the
// caller.
constexpr int kMaxTcGrid = 160;  // upper bound on the tensor-path grid (148 SMs on B200)

struct Workspace {
    uint32_t *err;         // [1] sticky device error code
    unsigned long long *launch_ctr;  // [1] streaming kernel: monotonic CTA ticket counter
    unsigned long long *grid_bar;    // [1] streaming kernel: grid-barrier arrival counter
    unsigned long long *zero_flag;   // [1] streaming kernel: launch number + 1 once `out` is zeroed
    uint32_t *tok_bits;    // [B][W] per-token activity bits
    uint32_t *seg_bits;    // [S][W] per-segment union bits
    uint32_t *tc_bits;     // [W] tensor path: batch union accumulated by atomic OR (zero between launches)
    int32_t *merge_idx;    // [S][f] compacted ascending neuron ids
    int32_t *counts;       // [S + 1] per-segment counts (+1 spare)
    __half *h;             // [f][B] fp16 intermediate of the CUDA-core path
    __half *x16;           // [Np][d] fp16 activations of the tensor path
    unsigned int *gbar;    // [3] tensor path: per-launch counters (barrier arrivals, prepared CTAs, finished CTAs)
    uint32_t *ready;       // [kMaxTcGrid / 2] tensor path: per-cluster h-publication counters (zeroed per launch)
    __half *h16;           // [Np][fpad] tensor path: fp16 h, K-major per token
    float *xchg;           // [kMaxTcGrid][Np][64] tensor path: per-CTA gate/up exchange slots
    int Np, fpad;
    size_t bytes;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ inline int words_of(int f) { return (f + 31) / 32; }

// MMA N extent for a batch of B tokens: a multiple of 16 in [16, 256].
inline int padded_batch(int B) { return B <= 16 ? 16 : ((B + 15) / 16) * 16; }

// Lays the workspace out over `base` (nullptr: only compute the size).
inline Workspace carve_workspace(void *base, int B, int d, int f, int group) {
    int S = group <= 0 ? 1 : (B + group - 1) / group;
    int W = words_of(f);
    Workspace w{};
    w.Np = B <= 256 ? padded_batch(B) : 0;
    size_t off = 0;
    auto take = [&](size_t n) {
        size_t o = off;
        off += align256(n);
        return base ? (void *)((char *)base + o) : nullptr;
    };
    w.fpad = (f + 63) / 64 * 64;
    uint32_t *sync = (uint32_t *)take(sizeof(uint32_t) * (64 + kMaxTcGrid / 2));
    w.err = sync;
    w.launch_ctr = sync ? reinterpret_cast<unsigned long long *>(sync + 16) : nullptr;
    w.zero_flag = sync ? reinterpret_cast<unsigned long long *>(sync + 24) : nullptr;
    w.grid_bar = sync ? reinterpret_cast<unsigned long long *>(sync + 32) : nullptr;
    w.ready = sync ? sync + 64 : nullptr;
    w.gbar = sync ? sync + 40 : nullptr;
    w.tok_bits = (uint32_t *)take(sizeof(uint32_t) * (size_t)B * W);
    w.seg_bits = (uint32_t *)take(sizeof(uint32_t) * (size_t)S * W);
    w.tc_bits = (uint32_t *)take(sizeof(uint32_t) * (size_t)W);
    w.merge_idx = (int32_t *)take(sizeof(int32_t) * (size_t)S * f);
    w.counts = (int32_t *)take(sizeof(int32_t) * (size_t)(S + 1));
    w.h = (__half *)take(sizeof(__half) * (size_t)f * B);
    if (d > 0 && w.Np > 0) {
        w.x16 = (__half *)take(sizeof(__half) * (size_t)w.Np * d);
        w.h16 = (__half *)take(sizeof(__half) * (size_t)w.Np * w.fpad);
        w.xchg = (float *)take(sizeof(float) * (size_t)kMaxTcGrid * w.Np * 64);
    }
    w.bytes = off;
    return w;
}

// ---- device helpers -----------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float2 h2f2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace spb
