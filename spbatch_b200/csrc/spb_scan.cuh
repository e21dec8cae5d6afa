// Block-level scan and bit-compaction helpers shared by the union kernel and
// the FFN kernels (which rebuild their slice of the index list from the
// union bitmask instead of waiting for a separate compaction launch).
#pragma once

#include "spb_common.cuh"

namespace spb {

// Inclusive warp scan.
__device__ __forceinline__ int warp_incl_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Exclusive scan over popc(bits[w]) for w < W, written to prefix[0..W]
// (prefix[W] = total).  `warp_tot` is scratch of >= 32 ints.  All threads of
// the block must call it; blockDim.x must be a multiple of 32.  Ends with a
// __syncthreads(), so prefix[] is readable on return.
__device__ __forceinline__ void scan_popc(const uint32_t *__restrict__ bits, int W, int *prefix,
                                          int *warp_tot) {
    const int nthreads = blockDim.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = nthreads >> 5;
    int carry = 0;
    for (int base = 0; base < W; base += nthreads) {
        int w = base + threadIdx.x;
        int c = w < W ? __popc(bits[w]) : 0;
        int incl = warp_incl_scan(c);
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int t = lane < nwarps ? warp_tot[lane] : 0;
            int ti = warp_incl_scan(t);
            if (lane < nwarps) warp_tot[lane] = ti - t;  // exclusive warp offsets
            if (lane == 31) warp_tot[32] = ti;            // chunk total (lanes >= nwarps add 0)
        }
        __syncthreads();
        if (w < W) prefix[w] = carry + warp_tot[warp] + incl - c;
        carry += warp_tot[32];
        __syncthreads();
    }
    if (threadIdx.x == 0) prefix[W] = carry;
    __syncthreads();
}

// For positions [p0, p1) of the ascending list of set bits, writes the bit
// indices (neuron ids) to out[p - p0].  prefix[] is the exclusive popcount
// scan from scan_popc.  Caller synchronises afterwards.
__device__ __forceinline__ void extract_positions(const uint32_t *__restrict__ bits, const int *prefix, int W,
                                                  int p0, int p1, int *out) {
    for (int w = threadIdx.x; w < W; w += blockDim.x) {
        int e = prefix[w], n = prefix[w + 1];
        if (n <= p0 || e >= p1) continue;
        uint32_t word = bits[w];
        int p = e;
        while (word) {
            int b = __ffs(word) - 1;
            word &= word - 1;
            if (p >= p0 && p < p1) out[p - p0] = w * 32 + b;
            ++p;
        }
    }
}

}  // namespace spb
