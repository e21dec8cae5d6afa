// One-shot all-reduce of the sharded layer's [B][d] fp32 partial outputs over
// NVLink peer memory (the exchange step of neuron sharding; the reference is
// single-GPU, and the library's first version called NCCL here).
//
// Every rank has receive slots [2][world][stride] that the other ranks have
// mapped (CUDA IPC).  One launch per layer, epoch e (kept in the rank's sync
// region, advanced by the kernel itself, so graph replays stay in step):
//   1. push: each CTA stores its slice of this rank's partial into slot
//      (e & 1, rank) of every peer -- posted NVLink stores, no round trips;
//   2. the CTA fences at system scope and counts itself done; the last CTA
//      stores e into slot `rank` of every peer's `in` flags (release);
//   3. every CTA waits until its own `in` flags all reach e (acquire) and
//      sums its slice over the ranks in rank order from local memory (its own
//      partial, the peers' slots), the same order on every rank, so all ranks
//      end with identical bits.
// A peer reuses a slot parity two calls later, and it can start that call
// only after this rank has raised its flag for the call in between, which it
// does once this call's kernel is done: one barrier per call suffices.
// Every wait is bounded (2 s of %globaltimer): on timeout the kernel records
// code 1 in the error word and finishes.  No TMA and no multicast: ordinary
// stores to peer addresses.
#include "spb_internal.h"
#include "tc_ptx.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstring>

namespace spb {

using namespace ptx;

namespace {

constexpr int kMaxRanks = 8;
constexpr int kArThreads = 512;
constexpr uint64_t kArTimeoutNs = 2000000000ull;

// Sync region of one rank (uint32 words): [0] epoch, [1] CTAs done,
// [16, 16 + kMaxRanks) `in` flags.
constexpr int kSyncEpoch = 0, kSyncDone = 1, kSyncIn = 16, kSyncWords = 64;

struct ArArgs {
    const float *partial;         // this rank's partial (local)
    float *recv[kMaxRanks];       // every rank's receive slots, as this GPU addresses them
    uint32_t *sync[kMaxRanks];    // every rank's sync region, as this GPU addresses them
    float *out;
    int64_t n4, stride;           // float4 count; slot stride in floats
    int world, rank;
    uint32_t *err;
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kArThreads) allreduce_peer_kernel(const ArArgs a) {
    __shared__ uint32_t s_epoch;
    __shared__ int s_last;
    uint32_t *mine = a.sync[a.rank];
    if (threadIdx.x == 0) s_epoch = mine[kSyncEpoch] + 1u;
    __syncthreads();
    const uint32_t e = s_epoch;
    const int64_t slot = ((int64_t)(e & 1u) * a.world + a.rank) * a.stride;
    const int64_t i0 = (int64_t)blockIdx.x * kArThreads + threadIdx.x, step = (int64_t)gridDim.x * kArThreads;
    // 1. push this rank's partial to every peer
    for (int64_t i = i0; i < a.n4; i += step) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.partial) + i);
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
            if (r < a.world && r != a.rank) reinterpret_cast<float4 *>(a.recv[r] + slot)[i] = v;
    }
    // 2. the last CTA (every CTA's stores fenced before it counted) signals
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(mine + kSyncDone, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last && threadIdx.x == 0) {
        __threadfence_system();
        mine[kSyncDone] = 0u;
        mine[kSyncEpoch] = e;  // every CTA has read the old epoch
        for (int r = 0; r < a.world; ++r) st_release_sys(a.sync[r] + kSyncIn + a.rank, e);
    }
    // 3. wait for every rank's push, then sum in rank order
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer();
        for (int r = 0; r < a.world; ++r)
            while ((int32_t)(ld_acquire_sys(mine + kSyncIn + r) - e) < 0)
                if (globaltimer() - t0 > kArTimeoutNs) {
                    atomicCAS(a.err, 0u, 1u);
                    break;
                }
    }
    __syncthreads();
    const float *own = a.recv[a.rank] + (int64_t)(e & 1u) * a.world * a.stride;
    for (int64_t i = i0; i < a.n4; i += step) {
        float4 v[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
            if (r < a.world)
                v[r] = r == a.rank ? __ldcg(reinterpret_cast<const float4 *>(a.partial) + i)
                                   : __ldcg(reinterpret_cast<const float4 *>(own + r * a.stride) + i);
        float4 s = v[0];
#pragma unroll
        for (int r = 1; r < kMaxRanks; ++r)
            if (r < a.world) {
                s.x += v[r].x;
                s.y += v[r].y;
                s.z += v[r].z;
                s.w += v[r].w;
            }
        reinterpret_cast<float4 *>(a.out)[i] = s;
    }
}

// The allocation holding a device pointer (driver API, looked up through the
// runtime so the library needs no link-time libcuda).
using AddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
int allocation_base(const void *p, CUdeviceptr *base) {
    static AddressRangeFn fn = nullptr;
    if (!fn) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        SPB_CUDA_TRY(cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q));
        if (!f || q != cudaDriverEntryPointSuccess) return fail(SPB_ERR_CUDA, "cuMemGetAddressRange unavailable");
        fn = reinterpret_cast<AddressRangeFn>(f);
    }
    size_t size = 0;
    if (fn(base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS)
        return fail(SPB_ERR_INVALID, "peer memory: not a device allocation");
    return SPB_OK;
}

struct PeerHandle {
    cudaIpcMemHandle_t h;
    uint64_t offset;  // of the exported pointer within its allocation
};

}  // namespace

}  // namespace spb

using namespace spb;

extern "C" {

size_t spb_peer_handle_bytes(void) { return sizeof(PeerHandle); }

size_t spb_peer_sync_bytes(void) { return sizeof(uint32_t) * kSyncWords; }

int spb_peer_export(const void *dev_ptr, void *handle_out) {
    if (!dev_ptr || !handle_out) return fail(SPB_ERR_INVALID, "spb_peer_export: null pointer");
    CUdeviceptr base = 0;
    if (int rc = allocation_base(dev_ptr, &base)) return rc;
    PeerHandle ph{};
    SPB_CUDA_TRY(cudaIpcGetMemHandle(&ph.h, reinterpret_cast<void *>(base)));
    ph.offset = reinterpret_cast<uint64_t>(dev_ptr) - (uint64_t)base;
    std::memcpy(handle_out, &ph, sizeof(ph));
    return SPB_OK;
}

int spb_peer_import(const void *handle, void **dev_ptr_out) {
    if (!handle || !dev_ptr_out) return fail(SPB_ERR_INVALID, "spb_peer_import: null pointer");
    PeerHandle ph;
    std::memcpy(&ph, handle, sizeof(ph));
    void *base = nullptr;
    SPB_CUDA_TRY(cudaIpcOpenMemHandle(&base, ph.h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr_out = static_cast<char *>(base) + ph.offset;
    return SPB_OK;
}

int spb_peer_close(void *dev_ptr) {
    if (!dev_ptr) return SPB_OK;
    CUdeviceptr base = 0;
    if (int rc = allocation_base(dev_ptr, &base)) return rc;
    SPB_CUDA_TRY(cudaIpcCloseMemHandle(reinterpret_cast<void *>(base)));
    return SPB_OK;
}

int spb_allreduce_peer(const float *partial, float *const *recv, uint32_t *const *syncs, int world, int rank,
                       int64_t stride, float *out, int64_t n, uint32_t *err, void *stream) {
    if (!partial || !recv || !syncs || !out || !err) return fail(SPB_ERR_INVALID, "spb_allreduce_peer: null pointer");
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail(SPB_ERR_INVALID, "spb_allreduce_peer: world must be 1..8 and rank in range");
    if (n < 0 || n % 4 || stride % 4 || n > stride)
        return fail(SPB_ERR_INVALID, "spb_allreduce_peer: n and stride must be multiples of 4, n <= stride");
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    ArArgs a{};
    for (int r = 0; r < world; ++r) {
        if (!recv[r] || !syncs[r] || !al(recv[r]))
            return fail(SPB_ERR_INVALID, "spb_allreduce_peer: slots must be non-null and 16-byte aligned");
        a.recv[r] = recv[r];
        a.sync[r] = syncs[r];
    }
    if (!al(partial) || !al(out)) return fail(SPB_ERR_INVALID, "spb_allreduce_peer: partial and out must be 16-byte aligned");
    a.partial = partial;
    a.out = out;
    a.n4 = n / 4;
    a.stride = stride;
    a.world = world;
    a.rank = rank;
    a.err = err;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), (a.n4 + kArThreads - 1) / kArThreads));
    allreduce_peer_kernel<<<grid, kArThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    SPB_CUDA_TRY(cudaGetLastError());
    return SPB_OK;
}

}  // extern "C"
