// Tensor-core sparse FFN layer (tcgen05 / TMEM), one persistent launch.
//
// Replaces the reference's mm_up (x2) + relu_and_mul + mm_down sequence
// (cuda/kernel.cu:595-816, 971-1048; mma.sync m16n8k16 with ldmatrix) for
// batches whose union forms real MMA tiles.  Everything after the union
// launch happens in ffn_tc_kernel, one CTA per SM:
//
//  gate/up units   a 128-neuron tile of the batch union (positions
//                  [128 i, 128 i + 128) of the ascending index list) times a
//                  K-slice of d.  Each ring stage holds one matrix's gathered
//                  rows for nkb 64-wide K blocks (a contiguous 128*nkb-byte run
//                  per row: DRAM efficiency of a row gather grows with the run
//                  length) plus the matching fp16 activations, copied with
//                  cp.async into the 128-byte-swizzled K-major layout.  Gate
//                  and up stages alternate; one thread issues
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
//                  reductions.  The W_down copies do not depend on h, so they
//                  are issued before the h tile's ready flag is checked.
//
// Warp roles (288 threads): warps 0-3 epilogue (TMEM lanes 0-127), warps 4-7
// cp.async producers, warp 8 TMEM allocator + MMA issuer.  Every wait is
// bounded (2 s of %globaltimer); on timeout the kernel records an error code in
// the workspace and unwinds instead of hanging.
#include "spb_internal.h"
#include "spb_scan.cuh"
#include "tc_ptx.cuh"

#include <algorithm>
#include <cstdlib>

namespace spb {

using namespace ptx;

constexpr int kTcThreads = 288;
constexpr int kTileM = 128;          // neurons per gate/up tile, rows per MMA
constexpr int kDnCols = 256;         // output columns per down item (two M=128 tiles)
constexpr uint32_t kATile = 16384;   // 128 rows x 128 bytes (one 64-wide K block)
constexpr int kMaxStages = 8;
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
    const __half *x16;           // [Np][d]
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
    unsigned long long *trace;   // [grid][kTraceSlots] %globaltimer stamps, or null
    int B, Np, d, f, fpad, W, act, per_token;
    int P;                       // ring stages
    int nkb;                     // 64-wide K blocks per gate/up stage (row run = 128 * nkb bytes)
    int ns;                      // neurons per down stage (64 or 128)
    int max_chunk;               // capacity of the shared down-unit id list
    uint32_t stage_bytes;
};

// Phase stamps written when tracing is enabled (spb_trace_enable).
enum TraceSlot {
    kTrStart = 0,        // after the dependency wait
    kTrScanned = 1,      // union scanned, plan known
    kTrGuIssued = 2,     // producers: last gate/up stage issued
    kTrGuMmaDone = 3,    // MMA: last gate/up stage issued + committed
    kTrGuAcc = 4,        // epilogue: gate/up accumulators ready
    kTrGuPublished = 5,  // epilogue: h written / partial handed off
    kTrFirstFlag = 6,    // producers: first down-chunk h tile available
    kTrDnIssued = 7,     // producers: last down stage issued
    kTrDnAcc = 8,        // epilogue: last down accumulator ready
    kTrEnd = 9,          // before TMEM release
};
constexpr int kTraceSlots = 16;

__device__ __forceinline__ void stamp(const TcArgs &a, int slot) {
    if (a.trace) a.trace[(size_t)blockIdx.x * kTraceSlots + slot] = globaltimer();
}

__device__ __forceinline__ Plan make_plan(int U, int d, int nkb, int grid) {
    Plan p;
    p.U = U;
    p.T = (U + kTileM - 1) / kTileM;
    p.KG = d / (64 * nkb);
    p.Sk = p.T ? max(1, min(min(8, p.KG), grid / p.T)) : 1;
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

// The u-th unit of CTA c: gate/up items c, c+grid, ... then its down item
// (there is at most one: ndn <= grid).
__device__ __forceinline__ Unit unit_of(const Plan &p, int c, int grid, int u, int ns) {
    Unit x{};
    x.kind = -1;
    const int n_gu = p.ngu > c ? (p.ngu - c + grid - 1) / grid : 0;
    if (u < n_gu) {
        const int g = c + u * grid;
        const int ks = g % p.Sk;
        x.kind = 0;
        x.tile = g / p.Sk;
        x.kg0 = ks * p.KG / p.Sk;
        x.kg1 = (ks + 1) * p.KG / p.Sk;
        x.stages = 2 * (x.kg1 - x.kg0);  // gate and up stages alternate
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

__device__ __forceinline__ int num_units(const Plan &p, int c, int grid) {
    const int a = p.ngu > c ? (p.ngu - c + grid - 1) / grid : 0;
    return a + (c < p.ndn ? 1 : 0);
}

// Neuron id at position pos of the ascending union list; bits and their
// exclusive popcount scan are in shared memory.
__device__ __forceinline__ int id_at(const uint32_t *bits, const int *prefix, int W, int pos) {
    int lo = 0, hi = W - 1;  // last word with prefix[w] <= pos
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= pos) lo = mid; else hi = mid - 1;
    }
    return lo * 32 + (int)__fns(bits[lo], 0, pos - prefix[lo] + 1);
}

__device__ __forceinline__ void raise_error(uint32_t *err, TcCtl *ctl, uint32_t code) {
    atomicCAS(err, 0u, code);
    ctl->abort = 1;
}

// Bounded mbarrier wait; false on timeout or abort.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, TcCtl *ctl, uint32_t *err, uint32_t code) {
    for (int i = 0; i < 4096; ++i)
        if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_test(bar, parity)) {
        if (ctl->abort) return false;
        if (globaltimer() - t0 > kTimeoutNs) {
            raise_error(err, ctl, code);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ float act_h(float g, float u, int act) {
    g = fmaxf(g, 0.0f);
    return act == SPB_ACT_RELU_RELU_MUL ? g * fmaxf(u, 0.0f) : g * u;
}

__global__ void __launch_bounds__(kTcThreads, 1) ffn_tc_kernel(const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int P = a.P, W = a.W, Np = a.Np, nkb = a.nkb, ns = a.ns;
    uint8_t *ring = smem;
    TcCtl *ctl = reinterpret_cast<TcCtl *>(ring + (size_t)P * a.stage_bytes);
    int *prefix = reinterpret_cast<int *>(ctl + 1);    // [W + 1]
    int *wtot = prefix + W + 1;                         // [64]
    uint32_t *bits = reinterpret_cast<uint32_t *>(wtot + 64);  // [W]
    uint16_t *dn_ids = reinterpret_cast<uint16_t *>(bits + W);  // [max_chunk]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t ncols = Np * 2 <= 32 ? 32 : (Np * 2 <= 64 ? 64 : (Np * 2 <= 128 ? 128 : (Np * 2 <= 256 ? 256 : 512)));

    if (tid == 0) {
        for (int i = 0; i < P; ++i) {
            mbar_init(&ctl->full[i], 128);
            mbar_init(&ctl->empty[i], 1);
        }
        mbar_init(&ctl->acc_full, 1);
        mbar_init(&ctl->acc_empty, 128);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 8) tmem_alloc(&ctl->tmem_base, ncols);

    // Inputs written by the union launch become visible here.
    grid_dependency_wait();
    if (tid == 0) stamp(a, kTrStart);
    for (int w = tid; w < W; w += kTcThreads) bits[w] = a.seg_bits[w];
    __syncthreads();
    scan_popc(bits, W, prefix, wtot);  // ends with __syncthreads
    const int grid = gridDim.x, c = blockIdx.x;
    const Plan pl = make_plan(prefix[W], a.d, nkb, grid);
    if (c == 0 && tid == 0) *a.count_out = pl.U;
    const int nunits = num_units(pl, c, grid);
    // ids of this CTA's down chunk, shared by its producers
    const Unit dn = unit_of(pl, c, grid, nunits - 1, ns);
    if (dn.kind == 1) {
        const int n = dn.stages * ns;
        for (int i = dn.P1 - dn.P0 + tid; i < n; i += kTcThreads) dn_ids[i] = 0xFFFF;
        for (int w = tid; w < W; w += kTcThreads) {  // word-parallel emission of [P0, P1)
            int p = prefix[w];
            if (prefix[w + 1] <= dn.P0 || p >= dn.P1) continue;
            uint32_t word = bits[w];
            while (word) {
                const int b = __ffs(word) - 1;
                word &= word - 1;
                if (p >= dn.P0 && p < dn.P1) dn_ids[p - dn.P0] = (uint16_t)(w * 32 + b);
                ++p;
            }
        }
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    if (tid == 0) stamp(a, kTrScanned);

    if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------ producers
        const int pt = tid - 128;
        const int lag = P - 1;
        const int cpr = nkb * 8;  // 16-byte chunks per row per gate/up stage
        int s = 0;                // stages committed
        int arrived = 0;          // stages whose full barrier this thread has arrived on
        int known_ready = -1;     // highest tile index whose ready flag this thread has seen
        // Arrive on every committed stage.  Must run before any wait on another
        // tile's ready flag: the stages still held back by the lag may be the
        // ones this CTA's own gate/up epilogue (and so some flag) depends on.
        auto flush = [&]() {
            cp_async_wait(0);
            fence_proxy_async_smem();
            for (; arrived < s; ++arrived) mbar_arrive(&ctl->full[arrived % P]);
        };
        for (int u = 0; u < nunits && !ctl->abort; ++u) {
            const Unit un = unit_of(pl, c, grid, u, ns);
            // gate/up: this thread copies chunk (pt % cpr) of rows i * (128 / cpr) + pt / cpr
            int rid[32];
            if (un.kind == 0) {
                const int rstep = 128 / cpr;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if (i < cpr) {
                        const int pos = un.tile * kTileM + i * rstep + pt / cpr;
                        rid[i] = pos < pl.U ? id_at(bits, prefix, W, pos) : -1;
                    }
                }
            }
            for (int st = 0; st < un.stages; ++st, ++s) {
                const int slot = s % P, round = s / P;
                if (round > 0 && !wait_bar(&ctl->empty[slot], (round - 1) & 1, ctl, a.err, kErrTimeoutEmpty)) break;
                const uint32_t sbase = smem_u32(ring + (size_t)slot * a.stage_bytes);
                if (un.kind == 0) {
                    const int kg = un.kg0 + (st >> 1);
                    const __half *w = (st & 1) ? a.wu : a.wg;
                    const int kbase = kg * 64 * nkb;
                    const int ch = pt % cpr, kbl = ch >> 3, cc = ch & 7;
                    const int rstep = 128 / cpr;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if (i < cpr) {
                            const int r = i * rstep + pt / cpr;
                            const int j = rid[i];
                            cp_async16(sbase + kbl * kATile + r * 128 + ((cc ^ (r & 7)) << 4),
                                       w + (int64_t)(j < 0 ? 0 : j) * a.d + kbase + ch * 8, j < 0 ? 0u : 16u);
                        }
                    }
                    const uint32_t xoff = nkb * kATile;
                    for (int q = pt; q < Np * cpr; q += 128) {
                        const int r = q / cpr, xc = q % cpr;
                        cp_async16(sbase + xoff + (xc >> 3) * (Np * 128) + r * 128 + (((xc & 7) ^ (r & 7)) << 4),
                                   a.x16 + (int64_t)r * a.d + kbase + xc * 8, 16u);
                    }
                } else {
                    const int p0s = un.P0 + st * ns;
                    const int m0 = un.mt * kDnCols;
                    const uint32_t lbo = (uint32_t)(ns / 8) * 1024;
                    // W_down rows, MN-major: ns neurons x 32 chunks (256 columns); lane = chunk
                    const int ch = pt & 31, mt2 = ch >> 4, mh = (ch >> 3) & 1, cc = ch & 7;
                    for (int kk = pt >> 5; kk < ns; kk += 4) {
                        const uint16_t id = dn_ids[p0s - un.P0 + kk];
                        const int kg = kk >> 3, kr = kk & 7;
                        const uint32_t dst = mt2 * 2 * lbo + mh * lbo + kg * 1024 + kr * 128 + ((cc ^ kr) << 4);
                        cp_async16(sbase + dst, a.wd + (int64_t)(id == 0xFFFF ? 0 : id) * a.d + m0 + ch * 8,
                                   id == 0xFFFF ? 0u : 16u);
                    }
                    // h of these neurons: wait for their gate/up tile to be published
                    const int tile = p0s / kTileM;
                    if (tile > known_ready) {
                        const uint32_t *flag = a.tile_ready + tile;
                        bool ok = ld_acquire_u32(flag) != 0;
                        if (!ok) {
                            cp_async_commit();  // the W_down copies above, as their own group
                            flush();
                            const uint64_t t0 = globaltimer();
                            while (!(ok = ld_acquire_u32(flag) != 0)) {
                                if (ctl->abort) break;
                                if (globaltimer() - t0 > kTimeoutNs) {
                                    raise_error(a.err, ctl, kErrTimeoutFlag);
                                    break;
                                }
                                __nanosleep(128);
                            }
                        }
                        if (!ok) break;
                        known_ready = tile;
                        if (pt == 0 && st == 0) stamp(a, kTrFirstFlag);
                    }
                    const uint32_t hoff = (uint32_t)ns * 512;
                    const int hcpr = ns / 8;
                    for (int q = pt; q < Np * hcpr; q += 128) {
                        const int t = q / hcpr, hc = q % hcpr;
                        cp_async16(sbase + hoff + (hc >> 3) * (Np * 128) + t * 128 + (((hc & 7) ^ (t & 7)) << 4),
                                   a.h16 + (int64_t)t * a.fpad + p0s + hc * 8, 16u);
                    }
                }
                cp_async_commit();
                // keep `lag` stages of copies in flight; a stage's groups
                // complete in order, so once at most `lag` groups are pending
                // the oldest unarrived stage has landed
                if (s + 1 - arrived > lag) {
                    cp_async_wait(lag);
                    fence_proxy_async_smem();
                    mbar_arrive(&ctl->full[arrived % P]);
                    ++arrived;
                }
            }
            if (pt == 0) stamp(a, un.kind == 0 ? kTrGuIssued : kTrDnIssued);
            if (ctl->abort) break;
        }
        flush();  // release the stages still in flight
    } else if (warp == 8) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_gu = idesc_f16_f32(kTileM, Np, false, false);
            const uint32_t id_dn = idesc_f16_f32(kTileM, Np, true, false);
            const uint32_t lbo = (uint32_t)(ns / 8) * 1024;
            int s = 0;
            for (int u = 0; u < nunits && !ctl->abort; ++u) {
                const Unit un = unit_of(pl, c, grid, u, ns);
                if (u > 0 && !wait_bar(&ctl->acc_empty, (u - 1) & 1, ctl, a.err, kErrTimeoutAcc)) break;
                tc_fence_after();
                bool ok = true;
                for (int st = 0; st < un.stages; ++st, ++s) {
                    const int slot = s % P, round = s / P;
                    if (!wait_bar(&ctl->full[slot], round & 1, ctl, a.err, kErrTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sbase = smem_u32(ring + (size_t)slot * a.stage_bytes);
                    if (un.kind == 0) {
                        const uint32_t dcol = tmem + (st & 1) * Np;  // gate or up accumulator
                        const uint32_t xoff = nkb * kATile;
                        for (int kbl = 0; kbl < nkb; ++kbl) {
#pragma unroll
                            for (int k4 = 0; k4 < 4; ++k4) {
                                const uint64_t ad = desc_sw128(sbase + kbl * kATile + k4 * 32, 16, 1024);
                                const uint64_t bd = desc_sw128(sbase + xoff + kbl * Np * 128 + k4 * 32, 16, 1024);
                                mma_f16(dcol, ad, bd, id_gu, (st > 1 || kbl > 0 || k4 > 0) ? 1u : 0u);
                            }
                        }
                    } else {
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
            const bool ok = wait_bar(&ctl->acc_full, u & 1, ctl, a.err, kErrTimeoutAcc);
            if (!named_bar_and(2, 128, ok)) break;
            tc_fence_after();
            if (e == 0) stamp(a, un.kind == 0 ? kTrGuAcc : kTrDnAcc);
            if (un.kind == 0) {
                const int pos = un.tile * kTileM + e;
                const bool valid = pos < pl.U;
                const int j = valid ? id_at(bits, prefix, W, pos) : 0;
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
    if (warp == 8) {
        if (ctl->abort) __nanosleep(100000);  // let in-flight MMAs drain before freeing TMEM
        tc_fence_after();
        tmem_dealloc(tmem, ncols);
    }
}

// ---------------------------------------------------------------------------------
// Stage geometry: the largest row run (K blocks per gate/up stage) that still
// leaves two ring stages; the down stage uses the same slot.
struct Geometry {
    int nkb, ns, P;
    uint32_t stage_bytes;
    size_t smem;
};

static Geometry pick_geometry(int Np, int W, int max_chunk, int d) {
    const size_t fixed = sizeof(TcCtl) + sizeof(int) * (W + 1 + 64) + sizeof(uint32_t) * W +
                         sizeof(uint16_t) * max_chunk + 1024 + 64;
    const size_t budget = 227 * 1024;
    const char *env = getenv("SPB_TC_NKB");
    const int forced = env ? atoi(env) : 0;
    const char *envp = getenv("SPB_TC_MINP");
    const int want_p = envp ? atoi(envp) : 4;
    Geometry best{0, 0, 0, 0, 0};
    // Longest row run (nkb) that keeps at least want_p ring stages: the ring is
    // what keeps enough bytes in flight per SM; fall back to any P >= 2.
    for (int pass = 0; pass < 2 && best.P == 0; ++pass) {
        for (int nkb = 4; nkb >= 1; --nkb) {
            if (forced && nkb != forced) continue;
            if ((d / 64) % nkb) continue;
            const uint32_t gu = (uint32_t)nkb * (kATile + (uint32_t)Np * 128);
            int ns = 128;
            if ((uint32_t)ns * 512 + 2u * Np * 128 > gu) ns = 64;
            const uint32_t dn = (uint32_t)ns * 512 + (uint32_t)(ns / 64) * Np * 128;
            const uint32_t stage = ((gu > dn ? gu : dn) + 1023) & ~1023u;
            const int P = (int)std::min<size_t>((budget - fixed) / stage, kMaxStages);
            if (P >= (pass == 0 ? want_p : 2)) {
                best = Geometry{nkb, ns, P, stage, fixed + (size_t)P * stage};
                break;
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
    a.x16 = L.x16;
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
    a.trace = static_cast<unsigned long long *>(trace_buffer((size_t)L.grid * kTraceSlots));
    a.B = L.B;
    a.Np = Np;
    a.d = L.d;
    a.f = L.f;
    a.fpad = L.fpad;
    a.W = words_of(L.f);
    a.act = L.act;
    a.per_token = L.per_token;
    // Longest down chunk: ceil(T / KC) tiles with KC = min(T, grid / MT).
    const int Tmax = (L.f + kTileM - 1) / kTileM;
    const int MT = L.d / kDnCols;
    const int KCmin = std::max(1, std::min(Tmax, L.grid / MT));
    a.max_chunk = ((Tmax + KCmin - 1) / KCmin + 1) * kTileM;
    const Geometry g = pick_geometry(Np, a.W, a.max_chunk, L.d);
    if (g.P < 2) return fail(SPB_ERR_UNSUPPORTED, "tensor path: shared memory too small for two stages");
    if ((L.d / 64) % g.nkb) return fail(SPB_ERR_INVALID, "tensor path: d does not split into stage K blocks");
    a.P = g.P;
    a.nkb = g.nkb;
    a.ns = g.ns;
    a.stage_bytes = g.stage_bytes;
    if (int rc = ensure_smem((const void *)ffn_tc_kernel, g.smem)) return rc;

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
    SPB_CUDA_TRY(cudaLaunchKernelEx(&cfg, ffn_tc_kernel, a));
    return SPB_OK;
}

}  // namespace spb
