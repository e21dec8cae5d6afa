// Tensor-core sparse FFN layer (tcgen05 / TMEM), one persistent launch.
//
// Replaces the reference's mm_up (x2) + relu_and_mul + mm_down sequence
// (cuda/kernel.cu:595-816, 971-1048; mma.sync m16n8k16 with ldmatrix) for
// batches whose union forms real MMA tiles.  Everything after the union
// launch happens in ffn_tc_kernel, one CTA per SM:
//
//  gate/up units   a 128-neuron tile of the batch union (positions
//                  [128 i, 128 i + 128) of the ascending index list) times a
//                  K-slice of d.  Each ring stage holds one K group: the
//                  gathered W_gate and W_up rows for nkb 64-wide K blocks (a
//                  contiguous 128*nkb-byte run per row) plus one copy of the
//                  matching fp16 activations, shared by both matrices.  The
//                  gathered rows arrive by cp.async (a warp copies whole row
//                  runs per instruction), the activations by 2D TMA tiles,
//                  all in the 128-byte-swizzled K-major layout the MMA reads.
//                  A stage's barrier completes on the producers' cp.async
//                  arrivals plus the TMA transaction bytes, so no producer
//                  waits on its own copies.  The copy rate of the four
//                  producer warps follows the bytes in flight, so the stage
//                  size is chosen to keep the most weight bytes in flight in
//                  the ring (three or more stages).  Per stage one thread issues
//                  tcgen05.mma.kind::f16 M=128 x N=Np x K=16 into two TMEM
//                  accumulators.  When several CTAs split a tile's K range,
//                  each writes its fp32 partials and the last to arrive
//                  (atomic per-tile counter) reduces them in fixed order.  The
//                  epilogue applies ReLU(gate)*up (or dReLU) and the per-token
//                  mask, rounds h to fp16 (cuda/kernel.cu:1019) into a K-major
//                  buffer and publishes a per-tile ready flag.
//  down unit       a 256-column slice of the output times a chunk of the
//                  union: W_down rows (stored [f][d], so each row contributes
//                  a contiguous 512-byte run) are the MN-major A operand, h the
//                  K-major B operand; out^T[2 x 128 x Np] accumulates in TMEM
//                  and is added into the pre-zeroed output with fp32
//                  reductions.  The W_down rows of a stage are copied as soon
//                  as its ring slot is free -- they overlap the tail of the
//                  gate/up phase -- and only the stage's h tile waits for the
//                  ready flags of the gate/up tiles it reads.
//
// Warp roles (544 threads): warps 0-3 epilogue (TMEM lanes 0-127), warps 4-15
// producers (cp.async + TMA), warp 16 TMEM allocator + MMA issuer.  Waiting
// threads sleep on the mbarrier (try_wait with a suspend hint) instead of
// spinning, which would steal shared-memory bandwidth from the producers.
// Every wait is bounded (2 s of %globaltimer); on timeout the kernel records an
// error code in the workspace and unwinds instead of hanging.
#include "spb_internal.h"
#include "spb_scan.cuh"
#include "tc_ptx.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace spb {

using namespace ptx;

// Warp roles: 0-3 epilogue, 4-15 producers, 16 MMA.  The cp.async rate of a
// warp is bounded by the copies it can keep in flight, so the copy rate of
// the CTA grows with the number of producer warps (4 warps: ~30 GB/s per SM
// on a 512-byte row gather, 8 warps: ~50 GB/s in isolation).
constexpr int kProducerWarps = 12;
constexpr int kProducerWarp0 = 4;
constexpr int kMmaWarp = kProducerWarp0 + kProducerWarps;
constexpr int kTcThreads = (kMmaWarp + 1) * 32;
constexpr int kTileM = 128;          // neurons per gate/up tile, rows per MMA
constexpr int kDnCols = 256;         // output columns per down item (two M=128 tiles)
constexpr uint32_t kATile = 16384;   // 128 rows x 128 bytes (one 64-wide K block)
constexpr int kMaxStages = 8;
constexpr int kMaxGuUnits = 4;       // gate/up units per CTA the shared id table holds
constexpr uint64_t kTimeoutNs = 2000000000ull;

enum : uint32_t { kErrTimeoutFull = 1, kErrTimeoutEmpty = 2, kErrTimeoutAcc = 3, kErrTimeoutFlag = 4 };

struct TcCtl {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t acc_full;
    uint64_t acc_empty;
    uint32_t tmem_base;
    volatile int abort;
    int is_last;
    int pad;
};

// How the layer is cut into units; every thread derives the same plan from U.
struct Plan {
    int U, T, Sk, ngu, KG, MT, KC, ndn;
};

struct TcArgs {
    const __half *wg, *wu, *wd;  // [f][d]
    __half *h16;                 // [Np][fpad]
    const uint32_t *seg_bits;    // [W]
    const uint32_t *tok_bits;    // [B][W]
    float *out;                  // [B][d], zero on entry
    int32_t *merge_out;          // [f]
    int32_t *count_out;          // [1]
    float *partial;              // [grid][2][Np][128]
    uint32_t *tile_cnt;          // [Tmax], zero on entry
    uint32_t *tile_ready;        // [Tmax], zero on entry
    uint32_t *err;
    unsigned long long *trace;   // stamps, or null
    int B, Np, d, f, fpad, W, act, per_token;
    int P;                       // ring stages
    int nkb;                     // 64-wide K blocks per gate/up stage (row run = 128 * nkb bytes)
    int ns;                      // neurons per down stage (64 or 128)
    int debug;                   // profiling knobs (SPB_TC_DEBUG): 1 no MMAs, 2 no weight copies
    int force_sk;                // profiling knob (SPB_TC_SK): K-split per tile, 0 = automatic
    uint32_t stage_bytes;
};

// TMA descriptors of the activations and of h (box 64 x Np, 128-byte swizzle).
struct TcMaps {
    CUtensorMap x, h;
};

// Phase stamps written when tracing is enabled (spb_trace_enable).
enum TraceSlot {
    kTrStart = 0,        // after the dependency wait
    kTrScanned = 1,      // union scanned, ids emitted
    kTrGuIssued = 2,     // producers: last gate/up stage issued
    kTrGuMmaDone = 3,    // MMA: last gate/up stage issued + committed
    kTrGuAcc = 4,        // epilogue: gate/up accumulators ready
    kTrGuPublished = 5,  // epilogue: h written / partial handed off
    kTrFirstFlag = 6,    // producers: h tiles of the first down stage available
    kTrDnIssued = 7,     // producers: last down stage issued
    kTrDnAcc = 8,        // epilogue: last down accumulator ready
    kTrEnd = 9,          // before TMEM release
    kTrBits = 10,        // union words copied to shared memory
    kTrScan = 11,        // scan done
    kTrGuIds = 12,       // gate/up tile ids emitted
    kTrDnIds = 13,       // down chunk ids emitted
};
constexpr int kTraceSlots = 16;
// Per-stage stamps of CTA 0: [stage][4] = producer past its empty wait,
// producer done issuing, (unused), MMA thread sees the stage full.
constexpr int kStageTraceBase = 160 * kTraceSlots;
constexpr int kStageTraceMax = 256;

__device__ __forceinline__ void stamp(const TcArgs &a, int slot) {
    if (a.trace) a.trace[(size_t)blockIdx.x * kTraceSlots + slot] = globaltimer();
}

__device__ __forceinline__ void stage_stamp(const TcArgs &a, int stage, int what) {
    if (a.trace && blockIdx.x == 0 && stage < kStageTraceMax)
        a.trace[kStageTraceBase + stage * 4 + what] = globaltimer();
}

__device__ __forceinline__ Plan make_plan(int U, int d, int nkb, int grid, int force_sk) {
    Plan p;
    p.U = U;
    p.T = (U + kTileM - 1) / kTileM;
    p.KG = d / (64 * nkb);
    p.Sk = p.T ? max(1, min(min(8, p.KG), grid / p.T)) : 1;
    if (force_sk > 0 && p.T) p.Sk = max(1, min(min(force_sk, p.KG), kMaxGuUnits * grid / p.T));
    p.ngu = p.T * p.Sk;
    p.MT = d / kDnCols;
    p.KC = p.T ? max(1, min(p.T, grid / p.MT)) : 0;
    p.ndn = p.MT * p.KC;
    return p;
}

struct Unit {
    int kind;              // 0 gate/up, 1 down, -1 none
    int tile, kg0, kg1;    // gate/up: tile and K-group range
    int mt, P0, P1;        // down: 256-column slice and union positions [P0, P1)
    int stages;
};

__device__ __forceinline__ int num_gu_units(const Plan &p, int c, int grid) {
    return p.ngu > c ? (p.ngu - c + grid - 1) / grid : 0;
}

// The u-th unit of CTA c: gate/up items c, c+grid, ... then its down item
// (there is at most one: ndn <= grid).
__device__ __forceinline__ Unit unit_of(const Plan &p, int c, int grid, int u, int ns) {
    Unit x{};
    x.kind = -1;
    const int n_gu = num_gu_units(p, c, grid);
    if (u < n_gu) {
        const int g = c + u * grid;
        const int ks = g % p.Sk;
        x.kind = 0;
        x.tile = g / p.Sk;
        x.kg0 = ks * p.KG / p.Sk;
        x.kg1 = (ks + 1) * p.KG / p.Sk;
        x.stages = x.kg1 - x.kg0;  // one K group (gate + up rows) per stage
        return x;
    }
    if (u == n_gu && c < p.ndn) {
        const int kc = c / p.MT;
        x.kind = 1;
        x.mt = c % p.MT;
        x.P0 = (p.T * kc / p.KC) * kTileM;
        x.P1 = min(p.U, (p.T * (kc + 1) / p.KC) * kTileM);
        x.stages = x.P1 > x.P0 ? (x.P1 - x.P0 + ns - 1) / ns : 0;
    }
    return x;
}

// Writes the neuron ids of union positions [P0, P1) to out[p - P0] (the whole
// block cooperates, one 32-neuron word per thread); out[i] for
// P1 - P0 <= i < n is set to `fill`.
__device__ __forceinline__ void emit_ids(const uint32_t *bits, const int *prefix, int W, int P0, int P1, int n,
                                         int fill, int *out) {
    for (int i = max(P1 - P0, 0) + (int)threadIdx.x; i < n; i += blockDim.x) out[i] = fill;
    for (int w = threadIdx.x; w < W; w += blockDim.x) {
        int p = prefix[w];
        if (prefix[w + 1] <= P0 || p >= P1) continue;
        uint32_t word = bits[w];
        while (word) {
            const int b = __ffs(word) - 1;
            word &= word - 1;
            if (p >= P0 && p < P1) out[p - P0] = w * 32 + b;
            ++p;
        }
    }
}

__device__ __forceinline__ void raise_error(uint32_t *err, TcCtl *ctl, uint32_t code) {
    atomicCAS(err, 0u, code);
    ctl->abort = 1;
}

// Bounded mbarrier wait; false on timeout or abort.  `hint_ns` is how long a
// waiting thread may sleep between checks (it wakes on completion).
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, TcCtl *ctl, uint32_t *err, uint32_t code,
                                         uint32_t hint_ns) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_test_sleep(bar, parity, hint_ns)) {
        if (ctl->abort) return false;
        if (globaltimer() - t0 > kTimeoutNs) {
            raise_error(err, ctl, code);
            return false;
        }
    }
    return true;
}

// Bounded wait for a gate/up tile's ready flag.
__device__ __forceinline__ bool wait_flag(const uint32_t *flag, TcCtl *ctl, uint32_t *err) {
    if (ld_acquire_u32(flag) != 0) return true;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_u32(flag) == 0) {
        if (ctl->abort) return false;
        if (globaltimer() - t0 > kTimeoutNs) {
            raise_error(err, ctl, kErrTimeoutFlag);
            return false;
        }
        __nanosleep(256);
    }
    return true;
}

__device__ __forceinline__ float act_h(float g, float u, int act) {
    g = fmaxf(g, 0.0f);
    return act == SPB_ACT_RELU_RELU_MUL ? g * fmaxf(u, 0.0f) : g * u;
}

__global__ void __launch_bounds__(kTcThreads, 1)
ffn_tc_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int P = a.P, W = a.W, Np = a.Np, nkb = a.nkb, ns = a.ns;
    uint8_t *ring = smem;
    TcCtl *ctl = reinterpret_cast<TcCtl *>(ring + (size_t)P * a.stage_bytes);
    // prologue-only tables live in the ring, which no copy touches before the
    // ids are emitted
    int *prefix = reinterpret_cast<int *>(ring);               // [W + 1]
    int *wtot = prefix + W + 1;                                // [64]
    uint32_t *bits = reinterpret_cast<uint32_t *>(wtot + 64);  // [W]
    int *gu_ids = reinterpret_cast<int *>(ctl + 1);            // [kMaxGuUnits][128]
    int *dn_ids = gu_ids + kMaxGuUnits * kTileM;               // [max_chunk]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t ncols = Np * 2 <= 32 ? 32 : (Np * 2 <= 64 ? 64 : (Np * 2 <= 128 ? 128 : (Np * 2 <= 256 ? 256 : 512)));

    if (tid == 0) {
        for (int i = 0; i < P; ++i) {
            mbar_init(&ctl->full[i], kProducerWarps * 32 + 1);  // producer cp.async arrivals + 1 TMA expect_tx arrival
            mbar_init(&ctl->empty[i], 1);
        }
        mbar_init(&ctl->acc_full, 1);
        mbar_init(&ctl->acc_empty, 128);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) tmem_alloc(&ctl->tmem_base, ncols);

    // Inputs written by the union launch become visible here.
    grid_dependency_wait();
    if (tid == 0) stamp(a, kTrStart);
    for (int w = tid; w < W; w += kTcThreads) bits[w] = a.seg_bits[w];
    __syncthreads();
    if (tid == 0) stamp(a, kTrBits);
    scan_popc(bits, W, prefix, wtot);  // ends with __syncthreads
    if (tid == 0) stamp(a, kTrScan);
    const int grid = gridDim.x, c = blockIdx.x;
    const Plan pl = make_plan(prefix[W], a.d, nkb, grid, a.force_sk);
    if (c == 0 && tid == 0) *a.count_out = pl.U;
    const int n_gu = min(num_gu_units(pl, c, grid), kMaxGuUnits);
    const int nunits = n_gu + (c < pl.ndn ? 1 : 0);
    // neuron ids of this CTA's tiles and down chunk; a.f (out of range) marks
    // padding rows, which are zero-filled
    for (int u = 0; u < n_gu; ++u) {
        const Unit un = unit_of(pl, c, grid, u, ns);
        emit_ids(bits, prefix, W, un.tile * kTileM, min(pl.U, un.tile * kTileM + kTileM), kTileM, a.f,
                 gu_ids + u * kTileM);
    }
    if (tid == 0) stamp(a, kTrGuIds);
    const Unit dn = unit_of(pl, c, grid, n_gu, ns);
    if (dn.kind == 1) emit_ids(bits, prefix, W, dn.P0, dn.P1, dn.stages * ns, a.f, dn_ids);
    if (tid == 0) stamp(a, kTrDnIds);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    if (tid == 0) stamp(a, kTrScanned);

    if (warp >= kProducerWarp0 && warp < kProducerWarp0 + kProducerWarps) {
        // ------------------------------------------------------------ producers
        const int pt = tid - kProducerWarp0 * 32, pw = pt >> 5;
        const bool leader = pt == 0;
        const bool copy_w = !(a.debug & 2);
        int s = 0;
        for (int u = 0; u < nunits; ++u) {
            const Unit un = unit_of(pl, c, grid, u, ns);
            bool ok = true;
            int flag_next = un.kind == 1 ? un.P0 / kTileM : 0;  // first gate/up tile not yet seen ready
            // CTAs sharing a K range start at different K groups: rows are 8 KB
            // apart, so CTAs stepping through the same column window in lock
            // step would all hit the same few DRAM channels.
            const int nk = un.kind == 0 ? un.kg1 - un.kg0 : 1;  // K groups of the unit
            const int rot = un.kind == 0 && nk > 0 ? (un.tile % nk) : 0;
            for (int st = 0; st < un.stages; ++st, ++s) {
                const int slot = s % P, round = s / P;
                ok = round == 0 || wait_bar(&ctl->empty[slot], (round - 1) & 1, ctl, a.err, kErrTimeoutEmpty, 1000);
                if (!ok) break;
                uint64_t *bar = &ctl->full[slot];
                const uint32_t sbase = smem_u32(ring + (size_t)slot * a.stage_bytes);
                if (leader) stage_stamp(a, s, 0);
                if (un.kind == 0) {
                    // one K group: gate and up rows (nkb x 128 B each) + the activations
                    const int kbase = (un.kg0 + (st + rot) % nk) * 64 * nkb;
                    if (leader) {  // activations: nkb TMA tiles of 64 columns x Np rows
                        mbar_arrive_expect_tx(bar, (uint32_t)nkb * Np * 128);
                        for (int kbl = 0; kbl < nkb; ++kbl)
                            tma_load_2d(sbase + 2 * nkb * kATile + kbl * Np * 128, &maps.x, bar, kbase + kbl * 64, 0);
                    }
                    // weights: 128 rows x (nkb x 128 B) per matrix; each warp
                    // instruction copies whole row runs
                    const int cpr = nkb * 8;    // 16-byte chunks per row run
                    const int rpw = 32 / cpr;   // rows per warp instruction
                    const int ch = lane & (cpr - 1), kbl = ch >> 3, cc = ch & 7;
                    if (copy_w) {
#pragma unroll
                        for (int m = 0; m < 2; ++m) {
                            const __half *wl = (m ? a.wu : a.wg) + kbase + ch * 8;
                            const uint32_t dl = sbase + (m * nkb + kbl) * kATile + (uint32_t)cc * 16;
                            for (int r = pw * rpw + lane / cpr; r < 128; r += kProducerWarps * rpw) {
                                const int j = gu_ids[u * kTileM + r];
                                // padding rows past the union copy row 0: the epilogue
                                // zeroes h for them, so their products are never used
                                cp_async16_full((dl + r * 128) ^ ((uint32_t)(r & 7) << 4),
                                                wl + (int64_t)(j < a.f ? j : 0) * a.d);
                            }
                        }
                    }
                } else {
                    const int p0s = un.P0 + st * ns;
                    // W_down rows as the MN-major operand: ns neurons x 256
                    // columns (32 chunks), one row per warp.  They do not depend
                    // on the gate/up phase, so they are copied at once; only h
                    // waits for its tiles below.
                    const int m0 = un.mt * kDnCols;
                    const uint32_t lbo = (uint32_t)(ns / 8) * 1024;
                    const int mb = lane >> 3, cc = lane & 7;
                    if (copy_w) {
                        for (int kk = pw; kk < ns; kk += kProducerWarps) {
                            const int j = dn_ids[(p0s - un.P0) + kk];
                            const int kg = kk >> 3, kr = kk & 7;
                            cp_async16(sbase + mb * lbo + kg * 1024 + kr * 128 + ((cc ^ kr) << 4),
                                       a.wd + (int64_t)(j < a.f ? j : 0) * a.d + m0 + lane * 8, j < a.f ? 16u : 0u);
                        }
                    }
                    if (leader) {
                        // h of this stage's neurons: wait for the gate/up tiles
                        // that hold them (published by other CTAs), then TMA
                        // ns/64 tiles of 64 neurons x Np tokens.
                        const int t1 = (min(p0s + ns, un.P1) - 1) / kTileM;
                        for (; flag_next <= t1 && ok; ++flag_next) ok = wait_flag(a.tile_ready + flag_next, ctl, a.err);
                        if (st == 0) stamp(a, kTrFirstFlag);
                        // the h stores were made through the generic proxy;
                        // the TMA below reads through the async proxy
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        mbar_arrive_expect_tx(bar, (uint32_t)(ns / 64) * Np * 128);
                        for (int kbl = 0; kbl < ns / 64; ++kbl)
                            tma_load_2d(sbase + (uint32_t)ns * 512 + kbl * Np * 128, &maps.h, bar, p0s + kbl * 64, 0);
                    }
                }
                cp_async_mbar_arrive(bar);
                if (leader) stage_stamp(a, s, 1);
            }
            if (!ok) break;
            if (leader) stamp(a, un.kind == 0 ? kTrGuIssued : kTrDnIssued);
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_gu = idesc_f16_f32(kTileM, Np, false, false);
            const uint32_t id_dn = idesc_f16_f32(kTileM, Np, true, false);
            const uint32_t lbo = (uint32_t)(ns / 8) * 1024;
            const bool do_mma = !(a.debug & 1);
            int s = 0;
            for (int u = 0; u < nunits && !ctl->abort; ++u) {
                const Unit un = unit_of(pl, c, grid, u, ns);
                if (u > 0 && !wait_bar(&ctl->acc_empty, (u - 1) & 1, ctl, a.err, kErrTimeoutAcc, 2000)) break;
                tc_fence_after();
                bool ok = true;
                for (int st = 0; st < un.stages; ++st, ++s) {
                    const int slot = s % P, round = s / P;
                    if (!wait_bar(&ctl->full[slot], round & 1, ctl, a.err, kErrTimeoutFull, 1000)) {
                        ok = false;
                        break;
                    }
                    stage_stamp(a, s, 3);
                    // the producers' cp.async data were written through the
                    // generic proxy; make them visible to the MMA's async proxy
                    fence_proxy_async_smem();
                    tc_fence_after();
                    const uint32_t sbase = smem_u32(ring + (size_t)slot * a.stage_bytes);
                    if (do_mma && un.kind == 0) {
                        // gate rows -> TMEM columns [0, Np), up rows -> [Np, 2 Np)
                        const uint32_t xoff = 2 * nkb * kATile;
                        for (int kbl = 0; kbl < nkb; ++kbl) {
#pragma unroll
                            for (int k4 = 0; k4 < 4; ++k4) {
                                const uint64_t bd = desc_sw128(sbase + xoff + kbl * Np * 128 + k4 * 32, 16, 1024);
                                const uint32_t acc = (st > 0 || kbl > 0 || k4 > 0) ? 1u : 0u;
#pragma unroll
                                for (int m = 0; m < 2; ++m) {
                                    const uint64_t ad = desc_sw128(sbase + (m * nkb + kbl) * kATile + k4 * 32, 16, 1024);
                                    mma_f16(tmem + m * Np, ad, bd, id_gu, acc);
                                }
                            }
                        }
                    } else if (do_mma) {
                        const uint32_t hoff = (uint32_t)ns * 512;
                        for (int kbl = 0; kbl < ns / 64; ++kbl) {
#pragma unroll
                            for (int k4 = 0; k4 < 4; ++k4) {
                                const uint64_t bd = desc_sw128(sbase + hoff + kbl * Np * 128 + k4 * 32, 16, 1024);
                                const uint32_t acc = (st > 0 || kbl > 0 || k4 > 0) ? 1u : 0u;
#pragma unroll
                                for (int mt2 = 0; mt2 < 2; ++mt2) {
                                    const uint64_t ad =
                                        desc_sw128(sbase + mt2 * 2 * lbo + (kbl * 8 + k4 * 2) * 1024, lbo, 1024);
                                    mma_f16(tmem + mt2 * Np, ad, bd, id_dn, acc);
                                }
                            }
                        }
                    }
                    mma_commit(&ctl->empty[slot]);
                }
                if (!ok) break;
                mma_commit(&ctl->acc_full);
                if (un.kind == 0) stamp(a, kTrGuMmaDone);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int e = tid;  // TMEM lane == tile row
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        for (int u = 0; u < nunits; ++u) {
            const Unit un = unit_of(pl, c, grid, u, ns);
            const bool ok = wait_bar(&ctl->acc_full, u & 1, ctl, a.err, kErrTimeoutAcc, 20000);
            if (!named_bar_and(2, 128, ok)) break;
            tc_fence_after();
            if (e == 0) stamp(a, un.kind == 0 ? kTrGuAcc : kTrDnAcc);
            if (un.kind == 0) {
                const int pos = un.tile * kTileM + e;
                const bool valid = pos < pl.U;
                const int j = valid ? gu_ids[u * kTileM + e] : 0;
                const bool direct = pl.Sk == 1;
                const uint32_t *mrow = a.tok_bits + (j >> 5);
                float *part = a.partial + (size_t)(c + u * grid) * 2 * Np * kTileM;  // gate/up item index
                for (int c0 = 0; c0 < Np; c0 += 16) {
                    float gv[16], uv[16];
                    tmem_ld16(trow + c0, gv);
                    tmem_ld16(trow + Np + c0, uv);
                    if (direct) {
                        uint32_t mw[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            mw[i] = (a.per_token && valid && c0 + i < a.B) ? __ldg(mrow + (int64_t)(c0 + i) * W) : ~0u;
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int t = c0 + i;
                            float hv = 0.0f;
                            if (valid && t < a.B && ((mw[i] >> (j & 31)) & 1u)) hv = act_h(gv[i], uv[i], a.act);
                            a.h16[(int64_t)t * a.fpad + pos] = __float2half_rn(hv);
                        }
                    } else {
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            part[(size_t)(c0 + i) * kTileM + e] = gv[i];
                            part[(size_t)(Np + c0 + i) * kTileM + e] = uv[i];
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&ctl->acc_empty);
                bool writer = direct;
                if (!direct) {
                    __threadfence();
                    named_bar(2, 128);
                    if (e == 0) ctl->is_last = atomicAdd(&a.tile_cnt[un.tile], 1u) == (uint32_t)(pl.Sk - 1);
                    named_bar(2, 128);
                    writer = ctl->is_last != 0;
                    if (writer) {
                        __threadfence();
                        for (int c0 = 0; c0 < Np; c0 += 16) {
                            float g[16], uu[16];
                            uint32_t mw[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                g[i] = uu[i] = 0.0f;
                                mw[i] = (a.per_token && valid && c0 + i < a.B) ? __ldg(mrow + (int64_t)(c0 + i) * W)
                                                                              : ~0u;
                            }
                            for (int ks = 0; ks < pl.Sk; ++ks) {  // fixed order: deterministic sums
                                const float *pp = a.partial + (size_t)(un.tile * pl.Sk + ks) * 2 * Np * kTileM;
                                float pg[16], pu[16];
#pragma unroll
                                for (int i = 0; i < 16; ++i) {
                                    pg[i] = __ldcg(pp + (size_t)(c0 + i) * kTileM + e);
                                    pu[i] = __ldcg(pp + (size_t)(Np + c0 + i) * kTileM + e);
                                }
#pragma unroll
                                for (int i = 0; i < 16; ++i) {
                                    g[i] += pg[i];
                                    uu[i] += pu[i];
                                }
                            }
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const int t = c0 + i;
                                float hv = 0.0f;
                                if (valid && t < a.B && ((mw[i] >> (j & 31)) & 1u)) hv = act_h(g[i], uu[i], a.act);
                                a.h16[(int64_t)t * a.fpad + pos] = __float2half_rn(hv);
                            }
                        }
                    }
                }
                if (writer) {
                    if (valid) a.merge_out[pos] = j;
                    __threadfence();
                    named_bar(2, 128);
                    if (e == 0) st_release_u32(a.tile_ready + un.tile, 1u);
                }
                if (e == 0) stamp(a, kTrGuPublished);
            } else {
#pragma unroll
                for (int mt2 = 0; mt2 < 2; ++mt2) {
                    const int m = un.mt * kDnCols + mt2 * kTileM + e;
                    for (int c0 = 0; c0 < Np; c0 += 16) {
                        float v[16];
                        tmem_ld16(trow + mt2 * Np + c0, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (c0 + i < a.B) atomicAdd(a.out + (int64_t)(c0 + i) * a.d + m, v[i]);
                    }
                }
                tc_fence_before();
                mbar_arrive(&ctl->acc_empty);
            }
        }
    }

    __syncthreads();
    if (tid == 0) stamp(a, kTrEnd);
    if (warp == kMmaWarp) {
        if (ctl->abort) __nanosleep(100000);  // let in-flight MMAs and copies drain before freeing TMEM
        tc_fence_after();
        tmem_dealloc(tmem, ncols);
    }
}

// ---------------------------------------------------------------------------------
// Tensor maps are encoded on the host once per (device, address, shape) and cached.
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct MapKey {
    int dev;
    const void *ptr;
    uint64_t cols, rows;
    uint32_t box_rows;
    bool operator==(const MapKey &o) const {
        return dev == o.dev && ptr == o.ptr && cols == o.cols && rows == o.rows && box_rows == o.box_rows;
    }
};

// fp16 matrix [rows][cols] (row-major), box of 64 columns x box_rows rows,
// 128-byte swizzle, out-of-range elements read as zero.
int tensor_map(const void *ptr, uint64_t cols, uint64_t rows, uint32_t box_rows, CUtensorMap *out) {
    static std::mutex mu;
    static std::vector<std::pair<MapKey, CUtensorMap>> cache;
    static EncodeTiledFn encode = nullptr;
    int dev = 0;
    SPB_CUDA_TRY(cudaGetDevice(&dev));
    const MapKey key{dev, ptr, cols, rows, box_rows};
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : cache)
        if (e.first == key) {
            *out = e.second;
            return SPB_OK;
        }
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        SPB_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess) return fail(SPB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    memset(&m, 0, sizeof(m));
    const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    if (cache.size() > 4096) cache.clear();
    cache.push_back({key, m});
    *out = m;
    return SPB_OK;
}

}  // namespace

// Stage geometry: K blocks per gate/up stage, neurons per down stage and ring
// depth; both kinds of stage share the ring slots.
struct Geometry {
    int nkb, ns, P;
    uint32_t stage_bytes;
    size_t smem;
};

static Geometry pick_geometry(int Np, int W, int max_chunk, int d) {
    const size_t fixed = sizeof(TcCtl) + sizeof(int) * (kMaxGuUnits * kTileM + max_chunk) + 1024 + 64;
    const size_t prologue = sizeof(int) * (W + 1 + 64) + sizeof(uint32_t) * W;  // in the ring
    const size_t budget = 227 * 1024;
    const char *env = getenv("SPB_TC_NKB");
    const int forced = env ? atoi(env) : 0;
    // The producer warps' copy rate follows the weight bytes in flight: maximise (P - 1) x the smaller of the gate/up and down
    // stages' weight bytes; prefer longer row runs on ties.
    Geometry best{0, 0, 0, 0, 0};
    size_t best_score = 0;
    for (int nkb = 4; nkb >= 1; --nkb) {
        if (forced && nkb != forced) continue;
        if ((d / 64) % nkb) continue;
        for (int ns = 128; ns >= 64; ns -= 64) {
            const uint32_t gu = (uint32_t)nkb * (2 * kATile + (uint32_t)Np * 128);
            const uint32_t dn = (uint32_t)ns * 512 + (uint32_t)(ns / 64) * Np * 128;
            const uint32_t stage = ((gu > dn ? gu : dn) + 1023) & ~1023u;
            if (fixed + 2 * (size_t)stage > budget || 2 * (size_t)stage < prologue) continue;
            const int P = (int)std::min<size_t>((budget - fixed) / stage, kMaxStages);
            const size_t w_gu = (size_t)nkb * 2 * kATile, w_dn = (size_t)ns * 512;
            // rank: the longer row run, then the weight bytes in flight
            const size_t score = ((size_t)nkb << 40) + (size_t)(P - 1) * std::min(w_gu, w_dn);
            if (score > best_score) {
                best_score = score;
                best = Geometry{nkb, ns, P, stage, fixed + (size_t)P * stage};
            }
        }
    }
    return best;
}

int launch_ffn_tc(const TcLaunch &L, cudaStream_t st) {
    const int Np = L.Np;
    if (Np < 16 || Np > 256 || Np % 16) return fail(SPB_ERR_UNSUPPORTED, "tensor path: batch must be 1..256");
    if (L.d % kDnCols) return fail(SPB_ERR_INVALID, "tensor path: d must be a multiple of 256");
    TcArgs a{};
    a.wg = static_cast<const __half *>(L.wg);
    a.wu = static_cast<const __half *>(L.wu);
    a.wd = static_cast<const __half *>(L.wd);
    a.h16 = L.h16;
    a.seg_bits = L.seg_bits;
    a.tok_bits = L.tok_bits;
    a.out = L.out;
    a.merge_out = L.merge_out;
    a.count_out = L.count_out;
    a.partial = L.partial;
    a.tile_cnt = L.tile_cnt;
    a.tile_ready = L.tile_ready;
    a.err = L.err;
    a.trace = static_cast<unsigned long long *>(trace_buffer((size_t)kStageTraceBase + kStageTraceMax * 4));
    a.B = L.B;
    a.Np = Np;
    a.d = L.d;
    a.f = L.f;
    a.fpad = L.fpad;
    a.W = words_of(L.f);
    a.act = L.act;
    a.per_token = L.per_token;
    a.debug = getenv("SPB_TC_DEBUG") ? atoi(getenv("SPB_TC_DEBUG")) : 0;
    a.force_sk = getenv("SPB_TC_SK") ? atoi(getenv("SPB_TC_SK")) : 0;
    // Longest down chunk: ceil(T / KC) tiles with KC = min(T, grid / MT).
    const int Tmax = (L.f + kTileM - 1) / kTileM;
    const int MT = L.d / kDnCols;
    const int KCmin = std::max(1, std::min(Tmax, L.grid / MT));
    const int max_chunk = ((Tmax + KCmin - 1) / KCmin + 1) * kTileM;
    if ((Tmax + L.grid - 1) / L.grid > kMaxGuUnits) return fail(SPB_ERR_UNSUPPORTED, "tensor path: f too large");
    const Geometry g = pick_geometry(Np, a.W, max_chunk, L.d);
    if (g.P < 2) return fail(SPB_ERR_UNSUPPORTED, "tensor path: shared memory too small for two stages");
    a.P = g.P;
    a.nkb = g.nkb;
    a.ns = g.ns;
    a.stage_bytes = g.stage_bytes;

    TcMaps maps;
    int rc;
    if ((rc = tensor_map(L.x16, L.d, Np, Np, &maps.x))) return rc;
    if ((rc = tensor_map(L.h16, L.fpad, Np, Np, &maps.h))) return rc;
    if ((rc = ensure_smem((const void *)ffn_tc_kernel, g.smem))) return rc;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(L.grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SPB_CUDA_TRY(cudaLaunchKernelEx(&cfg, ffn_tc_kernel, maps, a));
    return SPB_OK;
}

}  // namespace spb
