// Tensor-core sparse FFN layer (tcgen05 / TMEM), one persistent launch.
//
// Replaces the reference's mm_up (x2) + relu_and_mul + mm_down sequence
// (cuda/kernel.cu:595-816, 971-1048; mma.sync m16n8k16 with ldmatrix) for
// batches whose union forms real MMA tiles.  Everything after the union
// launch happens in ffn_tc_kernel, one CTA per SM:
//
//  gate/up units   a 128-neuron tile of the batch union (positions
//                  [128 i, 128 i + 128) of the ascending index list) times a
//                  K-slice of d.  Gathered W_gate / W_up rows and the fp16
//                  activations stream through a cp.async ring in 128-byte
//                  swizzled layout; one thread issues
//                  tcgen05.mma.kind::f16 M=128 x N=Np x K=16 into two TMEM
//                  accumulators (gate, up).  When several CTAs split a tile's
//                  K range, each writes its fp32 partials and the last to
//                  arrive (atomic per-tile counter) reduces them in fixed order.
//                  The epilogue applies ReLU(gate)*up (or dReLU) and the
//                  per-token mask, rounds h to fp16 (cuda/kernel.cu:1019) into
//                  a K-major buffer and publishes a per-tile ready flag.
//  down units      a 128-column slice of the output times a chunk of the
//                  union: W_down rows (stored [f][d]) are gathered as an
//                  MN-major operand, h as K-major; out^T[128 x Np] accumulates
//                  in TMEM and is added into the pre-zeroed output with
//                  fp32 reductions.  The W_down tiles do not depend on h, so
//                  they stream in before the h tile's ready flag is seen.
//
// Warp roles (288 threads): warps 0-3 epilogue (TMEM lanes 0-127), warps 4-7
// cp.async producers, warp 8 TMEM allocator + MMA issuer.  Every wait is
// bounded (2 s of %globaltimer); on timeout the kernel records an error code in
// the workspace and unwinds instead of hanging.
#include "spb_internal.h"
#include "spb_scan.cuh"
#include "tc_ptx.cuh"

namespace spb {

using namespace ptx;

constexpr int kTcThreads = 288;
constexpr int kTileM = 128;          // neurons per gate/up tile, output columns per down tile
constexpr int kKB = 64;              // K elements per 128-byte swizzle row
constexpr uint32_t kATile = 16384;   // 128 rows x 128 bytes
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

struct Plan {
    int U, T, Sk, ngu, KB, MT, KC, ndn;
};

__device__ __forceinline__ Plan make_plan(int U, int d, int grid) {
    Plan p;
    p.U = U;
    p.T = (U + kTileM - 1) / kTileM;
    p.KB = d / kKB;
    p.Sk = p.T ? max(1, min(min(8, p.KB), grid / p.T)) : 1;
    p.ngu = p.T * p.Sk;
    p.MT = d / kTileM;
    p.KC = p.T ? max(1, min(p.T, grid / p.MT)) : 0;
    p.ndn = p.MT * p.KC;
    return p;
}

struct Unit {
    int kind;  // 0 gate/up, 1 down, -1 none
    int tile, ks, kb0, kb1;          // gate/up
    int mt, P0, P1;                  // down
    int stages;
};

// The u-th unit of CTA c: gate/up items c, c+grid, ... then down items.
__device__ __forceinline__ Unit unit_of(const Plan &p, int c, int grid, int u) {
    Unit x{};
    x.kind = -1;
    const int n_gu = p.ngu > c ? (p.ngu - c + grid - 1) / grid : 0;
    if (u < n_gu) {
        const int g = c + u * grid;
        x.kind = 0;
        x.tile = g / p.Sk;
        x.ks = g % p.Sk;
        x.kb0 = x.ks * p.KB / p.Sk;
        x.kb1 = (x.ks + 1) * p.KB / p.Sk;
        x.stages = x.kb1 - x.kb0;
        return x;
    }
    u -= n_gu;
    const int i = c + u * grid;
    if (i < p.ndn) {
        const int kc = i / p.MT;
        x.kind = 1;
        x.mt = i % p.MT;
        x.P0 = (p.T * kc / p.KC) * kTileM;
        x.P1 = min(p.U, (p.T * (kc + 1) / p.KC) * kTileM);
        x.stages = x.P1 > x.P0 ? (x.P1 - x.P0 + kKB - 1) / kKB : 0;
    }
    return x;
}

__device__ __forceinline__ int num_units(const Plan &p, int c, int grid) {
    const int a = p.ngu > c ? (p.ngu - c + grid - 1) / grid : 0;
    const int b = p.ndn > c ? (p.ndn - c + grid - 1) / grid : 0;
    return a + b;
}

// Neuron id at position pos of the ascending union list (prefix = exclusive
// popcount scan of the union words, in shared memory).
__device__ __forceinline__ int id_at(const uint32_t *__restrict__ bits, const int *prefix, int W, int pos) {
    int lo = 0, hi = W - 1;  // last word with prefix[w] <= pos
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= pos) lo = mid; else hi = mid - 1;
    }
    const uint32_t word = bits[lo];
    const int b = (int)__fns(word, 0, pos - prefix[lo] + 1);
    return lo * 32 + b;
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
    int B, Np, d, f, fpad, W, act, per_token, P;
    uint32_t stage_bytes;
};

__global__ void __launch_bounds__(kTcThreads, 1) ffn_tc_kernel(const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int P = a.P;
    uint8_t *ring = smem;
    TcCtl *ctl = reinterpret_cast<TcCtl *>(ring + (size_t)P * a.stage_bytes);
    int *prefix = reinterpret_cast<int *>(ctl + 1);
    int *wtot = prefix + a.W + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int Np = a.Np;
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
    scan_popc(a.seg_bits, a.W, prefix, wtot);  // ends with __syncthreads
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    const int grid = gridDim.x, c = blockIdx.x;
    const Plan pl = make_plan(prefix[a.W], a.d, grid);
    if (c == 0 && tid == 0) *a.count_out = pl.U;
    const int nunits = num_units(pl, c, grid);

    if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------ producers
        const int pt = tid - 128;
        const int lag = P - 1;
        int s = 0;        // stages committed
        int arrived = 0;  // stages whose full barrier this thread has arrived on
        // Arrive on every committed stage.  Must run before any wait on another
        // tile's ready flag: the stages still held back by the lag may be the
        // ones this CTA's own gate/up epilogue (and so some flag) depends on.
        auto flush = [&]() {
            cp_async_wait(0);
            fence_proxy_async_smem();
            for (; arrived < s; ++arrived) mbar_arrive(&ctl->full[arrived % P]);
        };
        for (int u = 0; u < nunits && !ctl->abort; ++u) {
            const Unit un = unit_of(pl, c, grid, u);
            // gate/up rows this thread copies: r = 16 i + pt / 8 (same every stage)
            int rid[8];
            if (un.kind == 0) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int pos = un.tile * kTileM + i * 16 + (pt >> 3);
                    rid[i] = pos < pl.U ? id_at(a.seg_bits, prefix, a.W, pos) : -1;
                }
            }
            for (int st = 0; st < un.stages; ++st, ++s) {
                const int slot = s % P, round = s / P;
                if (round > 0 && !wait_bar(&ctl->empty[slot], (round - 1) & 1, ctl, a.err, kErrTimeoutEmpty)) break;
                uint8_t *stage = ring + (size_t)slot * a.stage_bytes;
                const uint32_t sbase = smem_u32(stage);
                if (un.kind == 0) {
                    const int kb = un.kb0 + st;
                    // A_gate, A_up: 128 rows x 8 chunks each; 8 lanes per row
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int q = i * 128 + pt, r = q >> 3, ch = q & 7;
                        const int j = rid[i];
                        const int64_t off = (int64_t)(j < 0 ? 0 : j) * a.d + kb * kKB + ch * 8;
                        const uint32_t dst = r * 128 + ((ch ^ (r & 7)) << 4);
                        const uint32_t nb = j < 0 ? 0u : 16u;
                        cp_async16(sbase + dst, a.wg + off, nb);
                        cp_async16(sbase + kATile + dst, a.wu + off, nb);
                    }
                    // activations: Np rows x 8 chunks
                    for (int q = pt; q < Np * 8; q += 128) {
                        const int r = q >> 3, ch = q & 7;
                        cp_async16(sbase + 2 * kATile + r * 128 + ((ch ^ (r & 7)) << 4),
                                   a.x16 + (int64_t)r * a.d + kb * kKB + ch * 8, 16u);
                    }
                } else {
                    const int p0s = un.P0 + st * kKB;
                    const int m0 = un.mt * kTileM;
                    // W_down rows, MN-major: 64 neurons x 16 chunks of 8 columns
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int q = i * 128 + pt, kk = q >> 4, ch = q & 15;
                        const int j = p0s + kk < un.P1 ? id_at(a.seg_bits, prefix, a.W, p0s + kk) : -1;
                        const int kg = kk >> 3, kr = kk & 7, mh = ch >> 3, cc = ch & 7;
                        const uint32_t dst = mh * 8192 + kg * 1024 + kr * 128 + ((cc ^ kr) << 4);
                        cp_async16(sbase + dst, a.wd + (int64_t)(j < 0 ? 0 : j) * a.d + m0 + ch * 8, j < 0 ? 0u : 16u);
                    }
                    // h of this 64-neuron chunk: wait for its gate/up tile
                    const uint32_t *flag = a.tile_ready + (p0s / kTileM);
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
                    for (int q = pt; q < Np * 8; q += 128) {
                        const int t = q >> 3, ch = q & 7;
                        cp_async16(sbase + kATile + t * 128 + ((ch ^ (t & 7)) << 4),
                                   a.h16 + (int64_t)t * a.fpad + p0s + ch * 8, 16u);
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
            if (ctl->abort) break;
        }
        flush();  // release the stages still in flight
    } else if (warp == 8) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_gu = idesc_f16_f32(kTileM, Np, false, false);
            const uint32_t id_dn = idesc_f16_f32(kTileM, Np, true, false);
            int s = 0;
            for (int u = 0; u < nunits && !ctl->abort; ++u) {
                const Unit un = unit_of(pl, c, grid, u);
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
#pragma unroll
                        for (int k4 = 0; k4 < 4; ++k4) {
                            const uint64_t bd = desc_sw128(sbase + 2 * kATile + k4 * 32, 16, 1024);
                            const uint32_t acc = (st > 0 || k4 > 0) ? 1u : 0u;
                            mma_f16(tmem, desc_sw128(sbase + k4 * 32, 16, 1024), bd, id_gu, acc);
                            mma_f16(tmem + Np, desc_sw128(sbase + kATile + k4 * 32, 16, 1024), bd, id_gu, acc);
                        }
                    } else {
#pragma unroll
                        for (int k4 = 0; k4 < 4; ++k4) {
                            const uint64_t ad = desc_sw128(sbase + k4 * 2048, 8192, 1024);
                            const uint64_t bd = desc_sw128(sbase + kATile + k4 * 32, 16, 1024);
                            mma_f16(tmem, ad, bd, id_dn, (st > 0 || k4 > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit(&ctl->empty[slot]);
                }
                if (!ok) break;
                mma_commit(&ctl->acc_full);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int e = tid;  // TMEM lane == tile row
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        for (int u = 0; u < nunits; ++u) {
            const Unit un = unit_of(pl, c, grid, u);
            const bool ok = wait_bar(&ctl->acc_full, u & 1, ctl, a.err, kErrTimeoutAcc);
            if (!named_bar_and(2, 128, ok)) break;
            tc_fence_after();
            if (un.kind == 0) {
                const int pos = un.tile * kTileM + e;
                const bool valid = pos < pl.U;
                const int j = valid ? id_at(a.seg_bits, prefix, a.W, pos) : 0;
                const bool direct = pl.Sk == 1;
                float *part = a.partial + (size_t)(c + (u * grid)) * 2 * Np * kTileM;  // gate/up item index
                for (int c0 = 0; c0 < Np; c0 += 16) {
                    float gv[16], uv[16];
                    tmem_ld16(trow + c0, gv);
                    tmem_ld16(trow + Np + c0, uv);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int t = c0 + i;
                        if (direct) {
                            float hv = 0.0f;
                            if (valid && t < a.B) {
                                const float g = fmaxf(gv[i], 0.0f);
                                hv = a.act == SPB_ACT_RELU_RELU_MUL ? g * fmaxf(uv[i], 0.0f) : g * uv[i];
                                if (a.per_token && !((a.tok_bits[(int64_t)t * a.W + (j >> 5)] >> (j & 31)) & 1u))
                                    hv = 0.0f;
                            }
                            a.h16[(int64_t)t * a.fpad + pos] = __float2half_rn(hv);
                        } else {
                            part[(size_t)t * kTileM + e] = gv[i];
                            part[(size_t)(Np + t) * kTileM + e] = uv[i];
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
                        for (int t = 0; t < Np; ++t) {
                            float g = 0.0f, uu = 0.0f;
                            for (int ks = 0; ks < pl.Sk; ++ks) {
                                const float *pp = a.partial + (size_t)(un.tile * pl.Sk + ks) * 2 * Np * kTileM;
                                g += __ldcg(pp + (size_t)t * kTileM + e);
                                uu += __ldcg(pp + (size_t)(Np + t) * kTileM + e);
                            }
                            float hv = 0.0f;
                            if (valid && t < a.B) {
                                g = fmaxf(g, 0.0f);
                                hv = a.act == SPB_ACT_RELU_RELU_MUL ? g * fmaxf(uu, 0.0f) : g * uu;
                                if (a.per_token && !((a.tok_bits[(int64_t)t * a.W + (j >> 5)] >> (j & 31)) & 1u))
                                    hv = 0.0f;
                            }
                            a.h16[(int64_t)t * a.fpad + pos] = __float2half_rn(hv);
                        }
                    }
                }
                if (writer) {
                    if (valid) a.merge_out[pos] = j;
                    __threadfence();
                    named_bar(2, 128);
                    if (e == 0) st_release_u32(a.tile_ready + un.tile, 1u);
                }
            } else {
                const int m = un.mt * kTileM + e;
                for (int c0 = 0; c0 < Np; c0 += 16) {
                    float v[16];
                    tmem_ld16(trow + c0, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int t = c0 + i;
                        if (t < a.B) atomicAdd(a.out + (int64_t)t * a.d + m, v[i]);
                    }
                }
                tc_fence_before();
                mbar_arrive(&ctl->acc_empty);
            }
        }
    }

    __syncthreads();
    if (warp == 8) {
        if (ctl->abort) __nanosleep(100000);  // let in-flight MMAs drain before freeing TMEM
        tc_fence_after();
        tmem_dealloc(tmem, ncols);
    }
}

// ---------------------------------------------------------------------------------
int tc_stage_bytes(int Np) { return (int)(2 * kATile + (uint32_t)Np * 128); }

int launch_ffn_tc(const TcLaunch &L, cudaStream_t st) {
    const int Np = L.Np;
    if (Np < 16 || Np > 256 || Np % 16) return fail(SPB_ERR_UNSUPPORTED, "tensor path: batch must be 1..256");
    if (L.d % kTileM) return fail(SPB_ERR_INVALID, "tensor path: d must be a multiple of 128");
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
    a.B = L.B;
    a.Np = Np;
    a.d = L.d;
    a.f = L.f;
    a.fpad = L.fpad;
    a.W = words_of(L.f);
    a.act = L.act;
    a.per_token = L.per_token;
    a.stage_bytes = (uint32_t)tc_stage_bytes(Np);
    const size_t fixed = sizeof(TcCtl) + sizeof(int) * (a.W + 1 + 64) + 1024;
    const size_t budget = 227 * 1024;
    int P = (int)((budget - fixed) / a.stage_bytes);
    P = min(P, kMaxStages);
    if (P < 2) return fail(SPB_ERR_UNSUPPORTED, "tensor path: shared memory too small for two stages");
    a.P = P;
    const size_t smem = fixed + (size_t)P * a.stage_bytes;
    if (int rc = ensure_smem((const void *)ffn_tc_kernel, smem)) return rc;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(L.grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
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
