// Tensor-core sparse FFN layer (tcgen05 / TMEM), one launch after the union.
//
// Replaces the reference's mm_up (x2) + relu_and_mul + mm_down sequence
// (cuda/kernel.cu:595-816, 971-1048; mma.sync m16n8k16 with ldmatrix) for
// batches whose union forms real MMA tiles.
//
// The launch is cooperative (every CTA is resident, one per SM) and grouped
// in clusters of two CTAs.  Each CTA runs two phases.
//
//   gate/up   Cluster c owns the contiguous union positions [U c / C,
//             U (c+1) / C) (C clusters), so every cluster gathers the same
//             number of rows to within one, and walks them in tiles of at
//             most 128 neurons.  CTA rank 0 multiplies the tile's gathered
//             W_gate rows with the batch, CTA rank 1 the W_up rows
//             (tcgen05.mma.kind::f16, M = 128 rows, N = Np tokens, K = d,
//             fp32 accumulator in TMEM).  Each ring stage holds nkb 64-wide K
//             blocks of the rows (cp.async, a 128 * nkb-byte run per row;
//             quantised rows are expanded to fp16 by the producers) and the
//             activation tile (TMA), both in the 128-byte-swizzled K-major
//             layout the MMA reads.  The pair then trades halves: a
//             CTA writes its results for the partner's 64 rows to its
//             workspace slot and signals the partner's mbarrier (release at
//             cluster scope); with the partner's half it forms h = act(gate,
//             up) * mask for its own 64 rows, rounds it to fp16
//             (cuda/kernel.cu:1019) and stores it K-major ([token][position])
//             in the workspace.  A per-cluster counter published with release
//             semantics tells the down phase which positions are ready.
//   down      Unit (m, k): output columns [256 m, 256 m + 256) times union
//             chunk k (64-aligned positions [Q_k, Q_k+1), about U / KC of
//             them).  W_down rows (stored [f][d]: a contiguous 512-byte run
//             per row) are the MN-major A operand, copied by cp.async as soon
//             as a ring slot is free -- they overlap the end of the gate/up
//             phase; the h tile (TMA) waits for the counters of the clusters
//             that produced it.  out^T[256 x Np] accumulates over the whole
//             chunk in TMEM and is added to the pre-zeroed output with 16-byte
//             fp32 reductions, so every output element receives KC
//             contributions.
//
// Warp roles (544 threads): warps 0-3 epilogue (TMEM lanes 0-127), warps 4-15
// producers, warp 16 TMEM allocation and MMA issue.  Every wait is bounded
// (2 s of %globaltimer); when one runs out the kernel records a code in the
// workspace's error word, stops issuing work, waits for its own copies (the
// cp.async groups and the TMA barriers) and its MMAs (the last commit) to
// land, frees its TMEM and returns.
#include "spb_internal.h"
#include "spb_scan.cuh"
#include "tc_ptx.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace spb {

using namespace ptx;

constexpr int kEpiWarps = 4;
constexpr int kProducerWarp0 = kEpiWarps;
constexpr int kProducerWarps = 12;
constexpr int kProducerThreads = kProducerWarps * 32;
constexpr int kMmaWarp = kProducerWarp0 + kProducerWarps;
constexpr int kTmaWarp = kMmaWarp + 1;
constexpr int kTcThreads = (kTmaWarp + 1) * 32;
constexpr int kTcWarps = kTcThreads / 32;
constexpr int kTileM = 128;          // neurons per gate/up tile (MMA M)
constexpr int kDnRows = 64;          // union positions per down stage
constexpr int kBoxRows = 32;         // rows per weight TMA box when whole row ranges stream
constexpr int kDenseMinPermille = 900;  // union share of f from which whole row ranges may stream
constexpr int kSlice = 256;          // output columns per down unit (two M = 128 MMAs)
constexpr uint32_t kATile = 16384;   // 128 rows x 128 bytes (one 64-wide K block)
constexpr uint32_t kDnLbo = (kDnRows / 8) * 1024;  // byte distance between 64-column blocks of a down stage
constexpr uint32_t kDnWBytes = 4 * kDnLbo;         // 64 rows x 256 columns fp16
constexpr int kMaxUnits = 16;         // ring units (a gate/up stage takes one or two, a down stage one)
constexpr int kMaxBufs = 16;
constexpr uint32_t kTmemCols = 512;
constexpr int kEpiBar = 1;           // named barrier of the epilogue warps
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;

enum : uint32_t {
    kErrTimeoutFull = 1,   // MMA issuer: a stage's copies never landed
    kErrTimeoutEmpty = 2,  // producer: a stage was never released by the MMAs
    kErrTimeoutAcc = 3,    // accumulator hand-off between MMA issuer and epilogue
    kErrTimeoutXchg = 4,   // the partner CTA's gate/up results never arrived
    kErrTimeoutFlag = 5,   // down phase: a cluster never published its h
    kErrTimeoutGrid = 6,   // the grid barrier after the union never completed
    kErrLaunchShape = 7,   // launched without 2-CTA clusters or with an odd grid
};

constexpr int kMaxStagingSlots = 7;
// Quantised weights: the first kQCopyThreads producer threads copy raw blocks
// into the staging slots, the others expand landed slots into the ring.
constexpr int kQCopyThreads = 128;
constexpr int kQExpThreads = kProducerThreads - kQCopyThreads;

struct TcCtl {
    // one of each per ring unit; every occupancy of a unit completes one
    // phase of all three (units past a stage's first arm with no bytes)
    uint64_t full[kMaxUnits];    // producers' cp.async arrivals
    uint64_t tma[kMaxUnits];     // TMA bytes of the stage's activation / h tile
    uint64_t empty[kMaxUnits];   // MMA commit: the unit may be overwritten
    uint64_t acc_full[kMaxBufs];
    uint64_t acc_empty[kMaxBufs];
    uint64_t xchg_full;   // partner: its results for this CTA's rows are in its slot
    uint64_t xchg_free;   // partner: it has read this CTA's slot
    uint64_t ids_ready;   // epilogue: the down unit's ids are emitted
    uint64_t stg_full[kMaxStagingSlots];   // quantised: a staging slot's raw blocks have landed
    uint64_t stg_empty[kMaxStagingSlots];  // quantised: a staging slot has been expanded
    uint32_t tmem_base;
    int last;             // this CTA finished last: it resets the launch's counters
    volatile int abort;
};

struct TcArgs {
    const __half *wg, *wu, *wd;  // [f][d] rows (fp16), or quantised rows of rowb bytes (wtype)
    int wtype;                   // SPB_W_F16 / SPB_W_Q8_0 / SPB_W_Q4_0
    int64_t rowb;                // bytes per stored weight row
    int nstg;                    // quantised weights: staging slots (stages staged ahead of the ring)
    uint32_t stg_bytes;          // bytes of one staging slot (all producers' tasks of one stage)
    int stg_tasks;               // task capacity of a slot (quant bytes first, then 4-byte scale pairs)
    int dense_min;               // fp16: a union of at least this many neurons streams whole row ranges
                                 // (every neuron a position, 2-D TMA boxes) instead of gathering rows
    const float *labels;         // [B][f] fp32 labels (> 0 active), or null with tok_in
    const uint32_t *tok_in;      // [B][W] per-token activity bits given by the caller, or null
    const float *x;              // [B][d] fp32 activations
    __half *x16;                 // [Np][d] fp16 activations (rows >= B zero), written in phase 0
    __half *h16;                 // [Np][fpad] h, K-major per token
    uint32_t *seg_bits;          // [W] (unused: the union travels in tc_bits)
    uint32_t *tc_bits;           // [W] batch union, OR-accumulated in phase 0; zero on entry, re-zeroed by
                                 // the launch's last CTA
    const __half *bias_g, *bias_u;  // [f] fp16 gate / up biases, or null
    unsigned int *gbar;          // [3] per-launch counters: grid-barrier arrivals, CTAs whose share of
                                 // the activations / zeroed output is written, CTAs done (zero on entry;
                                 // the last CTA to finish resets them and the cluster counters)
    float *out;                  // [B][d], zero on entry
    int32_t *merge_out;          // [f]
    int32_t *count_out;          // [1]
    float *xchg;                 // [grid][Np][64] per-CTA exchange slots
    uint32_t *ready;             // [grid / 2] per-cluster published-half-tile counters, zero on entry
    uint32_t *err;
    unsigned long long *trace;   // phase stamps, or null
    int B, Np, d, f, W, fpad, act, per_token;
    int nu;                      // ring units
    int gw;                      // units per gate/up stage (1 or 2; nu is even when 2)
    int nkb;                     // 64-wide K blocks per gate/up stage
    int nbuf;                    // TMEM accumulator buffers of 2 Np columns
    int KC;                      // union chunks of the down phase
    int max_gu, max_dn;          // capacities of the id tables
    int xdsm;                    // 1: the pair exchanges through distributed shared memory
    uint32_t unit_bytes;
    uint64_t timeout_ns;
    uint32_t hint_acc, hint;     // suspend-time hints of the accumulator / ring waits (ns)
    int inject;                  // test hook: 1 = CTA rank 1 never signals its results; profiling only
                                 // (quantised producers): 8 = no expansion, 16 = no copies;
                                 // profiling only: 2 = no output reductions, 4 = no W_down copies
};

// TMA descriptors of the activations and of h (box 64 x Np, 128-byte swizzle).
struct TcMaps {
    CUtensorMap x, h;
    CUtensorMap wg, wu;  // [f][d] rows, box 64 x kBoxRows (dense streaming)
    CUtensorMap wd;      // [f][d] rows, box 64 x kDnRows (dense streaming)
};

// Phase stamps written when tracing is enabled (spb_trace_enable).
enum TraceSlot {
    kTrStart = 0,       // after the dependency wait
    kTrScanned = 1,     // union scanned, ids emitted
    kTrGuIssued = 2,    // producers: all gate/up stages issued
    kTrGuMmaDone = 3,   // MMA: last gate/up tile committed
    kTrGuAcc = 4,       // epilogue: first tile's accumulator ready
    kTrXchg = 5,        // epilogue: partner's half arrived (first tile)
    kTrHDone = 6,       // epilogue: last tile's h published
    kTrFirstFlag = 7,   // producers: h of the first down stage available
    kTrDnIssued = 8,    // producers: all stages issued
    kTrDnAcc = 9,       // epilogue: down accumulator ready
    kTrEnd = 10,        // before TMEM release
    kTrPhase0 = 11,     // phase-0 work done, before the grid barrier
    kTrBarrier = 12,    // past the grid barrier
    kTrScan = 13,       // union scanned
    kTrEmitGu = 14,     // gate/up ids emitted (thread 0's share)
    kTrEmitDn = 15,     // down ids emitted (thread 0's share)
};
constexpr int kTraceSlots = 16;
// Per-unit stamps of CTA 0: [unit][4] = MMA issuer: first stage full,
// committed; epilogue: accumulator seen, released.
constexpr int kUnitTraceBase = 160 * kTraceSlots;
constexpr int kUnitTraceMax = 128;
// Per-stage stamps of CTA 0: [stage][4] = leader past the empty wait, leader
// done issuing, MMA issuer saw the stage complete.
constexpr int kStageTraceBase = kUnitTraceBase + kUnitTraceMax * 4;
constexpr int kStageTraceMax = 256;

__device__ __forceinline__ void stage_stamp(const TcArgs &a, int stage, int what) {
    if (a.trace && blockIdx.x == 0 && stage < kStageTraceMax) a.trace[kStageTraceBase + stage * 4 + what] = globaltimer();
}

__device__ __forceinline__ void stamp(const TcArgs &a, int slot) {
    if (a.trace) a.trace[(size_t)blockIdx.x * kTraceSlots + slot] = globaltimer();
}

__device__ __forceinline__ void unit_stamp(const TcArgs &a, int unit, int what) {
    if (a.trace && blockIdx.x == 0 && unit < kUnitTraceMax) a.trace[kUnitTraceBase + unit * 4 + what] = globaltimer();
}

__device__ __forceinline__ void raise_error(uint32_t *err, TcCtl *ctl, uint32_t code) {
    atomicCAS(err, 0u, code);
    ctl->abort = 1;
}

// Bounded mbarrier wait; false on timeout or abort.  `hint_ns` is how long a
// waiting thread may sleep between checks (it wakes on completion).
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, TcCtl *ctl, const TcArgs &a, uint32_t code,
                                         uint32_t hint_ns) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_test_sleep(bar, parity, hint_ns)) {
        if (ctl->abort) return false;
        if (globaltimer() - t0 > a.timeout_ns) {
            raise_error(a.err, ctl, code);
            return false;
        }
    }
    return true;
}

// The same for barriers the partner CTA arrives on (acquire at cluster scope).
__device__ __forceinline__ bool wait_bar_cluster(uint64_t *bar, uint32_t parity, TcCtl *ctl, const TcArgs &a,
                                                 uint32_t code) {
    const uint64_t t0 = globaltimer();
    while (!mbar_test_cluster(bar, parity, 2000)) {
        if (ctl->abort) return false;
        if (globaltimer() - t0 > a.timeout_ns) {
            raise_error(a.err, ctl, code);
            return false;
        }
    }
    return true;
}

// Bounded wait until a cluster's counter reaches `target` (acquire, GPU scope).
__device__ __forceinline__ bool wait_count(const uint32_t *cnt, uint32_t target, TcCtl *ctl, const TcArgs &a) {
    if (ld_acquire_u32(cnt) >= target) return true;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_u32(cnt) < target) {
        if (ctl->abort) return false;
        if (globaltimer() - t0 > a.timeout_ns) {
            raise_error(a.err, ctl, kErrTimeoutFlag);
            return false;
        }
        __nanosleep(128);
    }
    return true;
}

// The ring: stages occupy consecutive units in round robin; unit-step t
// (the t-th unit occupied in this launch) is unit t % NU and completes phase
// t / NU of that unit's barriers.
__device__ __forceinline__ bool ring_wait_empty(int t, int NU, TcCtl *ctl, const TcArgs &a) {
    return t < NU || wait_bar(&ctl->empty[t % NU], (uint32_t)(t / NU - 1) & 1u, ctl, a, kErrTimeoutEmpty, a.hint);
}

__device__ __forceinline__ float act_h(float g, float u, int act) {
    g = fmaxf(g, 0.0f);
    return act == SPB_ACT_RELU_RELU_MUL ? g * fmaxf(u, 0.0f) : g * u;
}

// First union position of cluster c of C (U positions in all; U <= 32768 and
// C <= 80, so the product fits 32 bits).
__device__ __forceinline__ int cluster_start(int U, int c, int C) { return (int)((uint32_t)(U * c) / (uint32_t)C); }

// Rows [r0, r1) of tile i when a cluster's n positions are cut into nt
// near-equal tiles of at most 128.
__device__ __forceinline__ void tile_rows(int n, int nt, int i, int &r0, int &r1) {
    r0 = (int)((uint32_t)(n * i) / (uint32_t)nt);
    r1 = (int)((uint32_t)(n * (i + 1)) / (uint32_t)nt);
}

__device__ __forceinline__ int tiles_of(int n) { return (n + kTileM - 1) / kTileM; }

// First position of cluster c's gate/up share.  Gathered rows: the union
// positions split evenly.  Whole row ranges (dense): positions are neuron
// ids, split in whole kBoxRows-row boxes (nb = f / kBoxRows rounded up).
__device__ __forceinline__ int span_start(bool dense, int Uv, int c, int C) {
    if (!dense) return cluster_start(Uv, c, C);
    const int nb = (Uv + kBoxRows - 1) / kBoxRows;
    return min(Uv, kBoxRows * (int)((uint32_t)(nb * c) / (uint32_t)C));
}

// Tile i of nt over a share of n positions: near-equal splits, in whole boxes
// when the rows stream as boxes.
__device__ __forceinline__ void tile_span(bool dense, int n, int nt, int i, int &r0, int &r1) {
    if (!dense) {
        tile_rows(n, nt, i, r0, r1);
        return;
    }
    const int nb = (n + kBoxRows - 1) / kBoxRows;
    r0 = min(n, kBoxRows * (int)((uint32_t)(nb * i) / (uint32_t)nt));
    r1 = min(n, kBoxRows * (int)((uint32_t)(nb * (i + 1)) / (uint32_t)nt));
}

// Union chunk k of KC for the down phase: 64-aligned start, so the h tiles'
// TMA coordinates are 16-byte aligned.
__device__ __forceinline__ int chunk_start(int U, int k, int KC) {
    if (k >= KC) return U;
    return min(U, (int)(((uint32_t)(U * k) / (uint32_t)KC + 63u) & ~63u));
}

// The word holding union position p (0 <= p < U): the largest w with
// prefix[w] <= p.
__device__ __forceinline__ int word_of(const int *prefix, int W, int p) {
    int lo = 0, hi = W - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= p) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// For positions [p0, p1) of the ascending union, writes the neuron ids to
// out[p - p0] (16-bit: f <= 32768).  Warps `warp0 + i * nwarps` take one
// 32-neuron word each, every lane placing its own bit by its rank in the
// word; only the words that hold the range are visited.
__device__ __forceinline__ void emit_ids16(const uint32_t *bits, const int *prefix, int W, int p0, int p1,
                                           uint16_t *out, int warp0, int nwarps) {
    if (p1 <= p0) return;
    const int lane = threadIdx.x & 31;
    const int w0 = word_of(prefix, W, p0), w1 = word_of(prefix, W, p1 - 1);
    for (int w = w0 + warp0; w <= w1; w += nwarps) {
        const uint32_t word = bits[w];
        if ((word >> lane) & 1u) {
            const int p = prefix[w] + __popc(word & ((1u << lane) - 1u));
            if (p >= p0 && p < p1) out[p - p0] = (uint16_t)(w * 32 + lane);
        }
    }
}

// ---------------------------------------------------------------------------------
// Quantised weights (ggml Q8_0 / Q4_0 blocks of 32 along d, in the "split" row
// layout: the row's quant bytes, then its fp16 scales).  The MMA still reads
// fp16 operands, so the producers expand the gathered blocks in shared memory.
// The producer warps split in two.  Copying threads issue, per stage, the raw
// bytes and scale pair of every task (one 32-element block of one row) with
// cp.async into a staging slot and arrive on the slot's barrier when their
// copies land (cp.async.mbarrier.arrive); they run up to nstg stages ahead.
// Expanding threads wait for a slot, write the 32 fp16 values of each task
// into the stage's swizzled operand tile, arrive on the stage's `full`
// barrier and free the slot.  Copy latency thus overlaps the expansion of
// earlier stages, and the quant bytes in flight do not depend on the (four
// times larger) fp16 tiles.  Values: q * scale computed in fp32 and rounded to fp16 once --
// the product of an 8-bit integer and an fp16 scale is exact in fp32, so this
// is the oracle's dequantised value (spbo_dequantize) rounded to the operand
// type.
struct QStage {
    int t;                   // unit-step of the stage in the ring
    int kind;                // 0 gate/up (tile rows x nkb K blocks), 1 down (positions x 256 columns)
    int rows;                // gate/up: tile rows; down: valid positions (the rest up to 16 are zero)
    int st;                  // gate/up: K step within the tile
    const uint16_t *ids;     // neuron ids of the stage's rows
};

constexpr int kMaxStaging = 7;  // cp.async.wait_group takes immediates 0..7

struct QuantProducer {
    TcCtl *ctl;
    uint8_t *ring, *stg;
    int pt, NU, nkb;
    const __half *wm;                // this CTA's gate/up matrix (raw rows): W_gate on rank 0, W_up on rank 1
    int rot, KG, m;
    int n, ntile;                    // this CTA's gate/up positions and tiles
    const uint16_t *gu_ids, *dn_ids;
    int Q0, Q1;                      // the down unit's positions

    // The stage at unit-step t: gate/up stages first (tile t / KG, K step
    // t % KG), then the down stages.
    __device__ __forceinline__ QStage stage(int t) const {
        const int ngu = ntile * KG;
        if (t < ngu) {
            const int i = t / KG;
            int r0, r1;
            tile_rows(n, ntile, i, r0, r1);
            return QStage{t, 0, r1 - r0, t - i * KG, gu_ids + r0};
        }
        const int p0 = Q0 + (t - ngu) * kDnRows;
        return QStage{t, 1, min(kDnRows, Q1 - p0), 0, dn_ids + (p0 - Q0)};
    }

    // tasks of a stage: gate/up rows x 2 nkb blocks, down positions x 8 blocks
    __device__ __forceinline__ int tasks_of(const TcArgs &a, const QStage &q) const {
        return q.kind == 0 ? q.rows * 2 * nkb : q.rows * 8;
    }
    // Task i: its MMA row r (gate/up: the tile row; down: the position),
    // block blk within the stage, global block index gb along d.
    __device__ __forceinline__ void task_of(const TcArgs &a, const QStage &q, int i, int &r, int &blk, int &gb) const {
        if (q.kind == 0) {
            const int lb = 2 * nkb;
            r = i / lb;
            blk = i - r * lb;
            gb = ((q.st + rot) % KG) * lb + blk;
        } else {
            r = i >> 3;
            blk = i & 7;
            gb = m * 8 + blk;
        }
    }
    __device__ __forceinline__ void task_src(const TcArgs &a, const QStage &q, int i, const uint8_t *&row, int &gb, int &r,
                                             int &blk) const {
        task_of(a, q, i, r, blk, gb);
        if (q.kind == 0) {
            row = reinterpret_cast<const uint8_t *>(wm) + (int64_t)q.ids[r] * a.rowb;
        } else {
            row = reinterpret_cast<const uint8_t *>(a.wd) + (int64_t)q.ids[r] * a.rowb;
        }
    }

    __device__ __forceinline__ void issue(const TcArgs &a, const QStage &q, int slot, int lt, int nthr) const {
        const uint32_t sq = smem_u32(stg + (size_t)slot * a.stg_bytes);
        const uint32_t ss = sq + (uint32_t)a.stg_tasks * (a.wtype == SPB_W_Q8_0 ? 32u : 16u);
        const int nt = (a.inject & 16) ? 0 : tasks_of(a, q);
        const int sco = a.wtype == SPB_W_Q8_0 ? a.d : a.d / 2;  // scales after the quant bytes
        for (int i = lt; i < nt; i += nthr) {
            const uint8_t *row;
            int gb, r, blk;
            task_src(a, q, i, row, gb, r, blk);
            if (a.wtype == SPB_W_Q8_0) {
                cp_async16_full(sq + i * 32, row + gb * 32);
                cp_async16_full(sq + i * 32 + 16, row + gb * 32 + 16);
            } else {
                cp_async16_full(sq + i * 16, row + gb * 16);
            }
            cp_async4(ss + i * 4, row + sco + (gb & ~1) * 2);
        }
        // the slot's barrier completes once every copying thread's copies landed
        cp_async_mbar_arrive(&ctl->stg_full[slot]);
    }

    // The oldest staged stage has landed (this thread's part): expand it into
    // its ring unit once the MMAs have released the unit.
    __device__ __forceinline__ bool finish(const TcArgs &a, const QStage &q, int slot, int lt, int nthr) const {
        if (lt == 0) stage_stamp(a, q.t, 3);
        if (!ring_wait_empty(q.t, NU, ctl, a)) return false;
        if (lt == 0) stage_stamp(a, q.t, 0);
        const uint8_t *sq = stg + (size_t)slot * a.stg_bytes;
        const uint8_t *ss = sq + (size_t)a.stg_tasks * (a.wtype == SPB_W_Q8_0 ? 32 : 16);
        const uint32_t ubase = smem_u32(ring + (size_t)(q.t % NU) * a.unit_bytes);
        const int nt = (a.inject & 8) ? 0 : tasks_of(a, q);
        for (int i = lt; i < nt; i += nthr) {
            int r, blk, gb;
            task_of(a, q, i, r, blk, gb);
            // the block's scale in both halves of a half2
            const uint32_t sp = *reinterpret_cast<const uint32_t *>(ss + i * 4);
            const uint32_t sc2 = __byte_perm(sp, 0, (gb & 1) ? 0x3232 : 0x1010);
            uint32_t raw[8];
            if (a.wtype == SPB_W_Q8_0) {
                const uint4 v0 = *reinterpret_cast<const uint4 *>(sq + i * 32);
                const uint4 v1 = *reinterpret_cast<const uint4 *>(sq + i * 32 + 16);
                raw[0] = v0.x; raw[1] = v0.y; raw[2] = v0.z; raw[3] = v0.w;
                raw[4] = v1.x; raw[5] = v1.y; raw[6] = v1.z; raw[7] = v1.w;
            } else {
                const uint4 v = *reinterpret_cast<const uint4 *>(sq + i * 16);
                raw[0] = v.x; raw[1] = v.y; raw[2] = v.z; raw[3] = v.w;
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                // Elements 8c .. 8c + 7 of the block as four half2 pairs.  An
                // integer u < 1024 placed in the mantissa of 1024.0 (0x6400)
                // is the fp16 value 1024 + u exactly; subtracting the offset
                // gives q (Q8_0: u = q + 128) or q - 8 (Q4_0: u = nibble)
                // exactly, and one fp16 multiply by the scale rounds the exact
                // product once -- the fp32 product rounded to fp16.
                uint32_t wd[2];
                uint32_t off;
                if (a.wtype == SPB_W_Q8_0) {
                    wd[0] = raw[2 * c] ^ 0x80808080u;
                    wd[1] = raw[2 * c + 1] ^ 0x80808080u;
                    off = 0x64806480u;  // 1152.0 in both halves
                } else {
                    // element j (< 16) is the low nibble of byte j, element j + 16 its high nibble
                    const int sh = c < 2 ? 0 : 4;
                    wd[0] = (raw[(c & 1) * 2] >> sh) & 0x0f0f0f0fu;
                    wd[1] = (raw[(c & 1) * 2 + 1] >> sh) & 0x0f0f0f0fu;
                    off = 0x64086408u;  // 1032.0 in both halves
                }
                uint32_t h[4];
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint32_t u = __byte_perm(wd[p >> 1], 0x64646464u, (p & 1) ? 0x4342 : 0x4140);
                    __half2 v = __hsub2(*reinterpret_cast<const __half2 *>(&u),
                                        *reinterpret_cast<const __half2 *>(&off));
                    v = __hmul2(v, *reinterpret_cast<const __half2 *>(&sc2));
                    h[p] = *reinterpret_cast<uint32_t *>(&v);
                }
                const uint4 o = make_uint4(h[0], h[1], h[2], h[3]);
                uint32_t dst;
                if (q.kind == 0) {
                    const int cc = (blk & 1) * 4 + c;
                    dst = ubase + (blk >> 1) * kATile + r * 128 + ((cc ^ (r & 7)) << 4);
                } else {
                    const int c8 = (blk & 1) * 4 + c, kr = r & 7;
                    dst = ubase + (blk >> 1) * kDnLbo + (r >> 3) * 1024 + kr * 128 + ((c8 ^ kr) << 4);
                }
                st_shared_v4(dst, o);
            }
        }
        if (q.kind == 1) {
            // positions past the chunk, up to the next multiple of 16: zero rows
            const int nr16 = (q.rows + 15) & ~15;
            for (int i = q.rows * 32 + lt; i < nr16 * 32; i += nthr) {
                const int r = i >> 5, c = i & 31, mb = c >> 3, c8 = c & 7, kr = r & 7;
                st_shared_v4(ubase + mb * kDnLbo + (r >> 3) * 1024 + kr * 128 + ((c8 ^ kr) << 4),
                             make_uint4(0u, 0u, 0u, 0u));
            }
        }
        // (the MMA issuer fences its view of these generic-proxy writes
        // against the async proxy once the stage's barrier completes)
        mbar_arrive(&ctl->full[q.t % NU]);
        mbar_arrive(&ctl->stg_empty[slot]);  // the copying threads may refill the slot
        if (lt == 0) stage_stamp(a, q.t, 1);
        return true;
    }

};

// kQuant: the producers expand quantised rows (a separate instantiation, so
// the fp16 kernel carries none of that code).
template <bool kQuant>
__global__ void __launch_bounds__(kTcThreads, 1)
ffn_tc_kernel(const __grid_constant__ TcMaps maps, const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NU = a.nu, GW = a.gw, W = a.W, Np = a.Np, nkb = a.nkb, nbuf = a.nbuf;
    uint8_t *ring = smem;
    // quantised weights: staging slots for the raw blocks, after the ring
    uint8_t *stg = ring + (size_t)NU * a.unit_bytes;
    TcCtl *ctl = reinterpret_cast<TcCtl *>(stg + (size_t)a.nstg * a.stg_bytes);
    uint32_t *tokmask = reinterpret_cast<uint32_t *>(ctl + 1);  // [8][128] per tile row: its tokens' bits
    uint16_t *gu_ids = reinterpret_cast<uint16_t *>(tokmask + 8 * kTileM);  // [max_gu]
    uint16_t *dn_ids = gu_ids + a.max_gu;                                    // [max_dn]
    // [Np][64] fp32: the partner's results for this CTA's rows, when they
    // travel through distributed shared memory (a.xdsm)
    float *xrecv = reinterpret_cast<float *>(reinterpret_cast<uintptr_t>(dn_ids + a.max_dn + 3) & ~uintptr_t(15));
    // union tables: the down ids are emitted from them while the gate/up
    // stages stream
    int *prefix = reinterpret_cast<int *>(xrecv + (a.xdsm ? 64 * Np : 0));  // [W + 1]
    int *wtot = prefix + W + 1;                                              // [64]
    uint32_t *bits = reinterpret_cast<uint32_t *>(wtot + 64);                // [W]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // The pairing, the exchange through the partner's shared memory and the
    // grid-wide counters assume 2-CTA clusters over an even grid; a launch
    // that arrives in any other shape (a tool that replays it without its
    // cluster attribute) records an error and touches nothing else.
    if (cluster_nctarank() != 2u || (gridDim.x & 1u)) {
        if (tid == 0) atomicCAS(a.err, 0u, (uint32_t)kErrLaunchShape);
        return;
    }
    const uint32_t rank = cluster_ctarank(), peer = rank ^ 1u;
    const int clu = blockIdx.x >> 1, nclu = gridDim.x >> 1;

    if (tid == 0) {
        for (int i = 0; i < NU; ++i) {
            mbar_init(&ctl->full[i], kQuant ? kQExpThreads : kProducerThreads);
            mbar_init(&ctl->tma[i], 1);
            mbar_init(&ctl->empty[i], 1);
        }
        for (int i = 0; i < nbuf; ++i) {
            mbar_init(&ctl->acc_full[i], 1);
            mbar_init(&ctl->acc_empty[i], kEpiWarps * 32);
        }
        mbar_init(&ctl->xchg_full, kEpiWarps * 32);
        mbar_init(&ctl->xchg_free, kEpiWarps * 32);
        mbar_init(&ctl->ids_ready, kEpiWarps * 32);
        if (kQuant)
            for (int i = 0; i < a.nstg; ++i) {
                mbar_init(&ctl->stg_full[i], kQCopyThreads);
                mbar_init(&ctl->stg_empty[i], kQExpThreads);
            }
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) tmem_alloc(&ctl->tmem_base, kTmemCols);
    // the partner may arrive on this CTA's barriers only once they exist
    cluster_sync_all();

    // Whatever the previous kernel on the stream wrote (these inputs, this
    // workspace) becomes visible here.
    grid_dependency_wait();
    if (tid == 0) stamp(a, kTrStart);
    // ---- phase 0.  Labels: every CTA computes a share of the union words,
    // the fp16 activations and the zeroed output, then one grid barrier.
    // Bits (tok_in): every CTA ORs the caller's per-token words itself (B x W
    // words through L2) and needs no grid-wide step; its share of the
    // activations and of the zeroed output is published on a counter that
    // only the activation loads and the first output reduction wait for.
    const bool bits_in = a.tok_in != nullptr;
    if (bits_in) {
        for (int w = tid; w < W; w += kTcThreads) {
            uint32_t u = 0;
            const uint32_t *col = a.tok_in + w;
#pragma unroll 8
            for (int t = 0; t < a.B; ++t) u |= __ldg(col + (int64_t)t * W);
            if (w == W - 1 && (a.f & 31)) u &= (1u << (a.f & 31)) - 1u;
            bits[w] = u;
        }
        const int64_t gt = (int64_t)blockIdx.x * kTcThreads + tid, gs = (int64_t)gridDim.x * kTcThreads;
        const int64_t n2 = (int64_t)Np * a.d / 2;
        for (int64_t i = gt; i < n2; i += gs) {
            const int t = (int)((2 * i) / a.d);
            const float2 v = t < a.B ? *reinterpret_cast<const float2 *>(a.x + 2 * i) : make_float2(0.f, 0.f);
            reinterpret_cast<__half2 *>(a.x16)[i] = __floats2half2_rn(v.x, v.y);
        }
        const int64_t n4 = (int64_t)a.B * a.d / 4;
        for (int64_t i = gt; i < n4; i += gs) reinterpret_cast<float4 *>(a.out)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            red_add_release_u32(a.gbar + 1, 1u);
        }
    } else {
        const int64_t gt = (int64_t)blockIdx.x * kTcThreads + tid, gs = (int64_t)gridDim.x * kTcThreads;
        const int64_t n2 = (int64_t)Np * a.d / 2;
        // the first two activation pairs of this thread are loaded before the
        // label reads, so both wait on memory together
        float2 xv0 = make_float2(0.f, 0.f), xv1 = make_float2(0.f, 0.f);
        if (gt < n2 && (int)((2 * gt) / a.d) < a.B) xv0 = *reinterpret_cast<const float2 *>(a.x + 2 * gt);
        if (gt + gs < n2 && (int)((2 * (gt + gs)) / a.d) < a.B) xv1 = *reinterpret_cast<const float2 *>(a.x + 2 * (gt + gs));
        // Items (word w, 8-token group c), item i handled by warp i of the
        // grid's warps taken CTA-major, so every warp of every SM keeps label
        // loads in flight (one 128-byte row segment per token); the groups'
        // ballots meet in tc_bits by atomic OR.
        const int TC = (a.B + 7) >> 3;
        const int gwarps = gridDim.x * kTcWarps, items = W * TC;
        for (int it = warp * gridDim.x + blockIdx.x; it < items; it += gwarps) {
            const int w = it / TC, t0 = (it - w * TC) * 8;
            const int j = w * 32 + lane;
            const bool in = j < a.f;
            float v[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) v[q] = (in && t0 + q < a.B) ? __ldg(a.labels + (int64_t)(t0 + q) * a.f + j) : 0.0f;
            bool any = false;
#pragma unroll
            for (int q = 0; q < 8; ++q) any |= v[q] > 0.0f;
            const uint32_t seg = __ballot_sync(0xffffffffu, any);
            if (lane == 0 && seg) atomicOr(a.tc_bits + w, seg);
        }
        if (gt < n2) reinterpret_cast<__half2 *>(a.x16)[gt] = __floats2half2_rn(xv0.x, xv0.y);
        if (gt + gs < n2) reinterpret_cast<__half2 *>(a.x16)[gt + gs] = __floats2half2_rn(xv1.x, xv1.y);
        for (int64_t i = gt + 2 * gs; i < n2; i += gs) {
            const int t = (int)((2 * i) / a.d);
            const float2 v = t < a.B ? *reinterpret_cast<const float2 *>(a.x + 2 * i) : make_float2(0.f, 0.f);
            reinterpret_cast<__half2 *>(a.x16)[i] = __floats2half2_rn(v.x, v.y);
        }
        const int64_t n4 = (int64_t)a.B * a.d / 4;
        for (int64_t i = gt; i < n4; i += gs) reinterpret_cast<float4 *>(a.out)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tid == 0) stamp(a, kTrPhase0);
        // grid barrier on gbar[0] (arrivals)
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            red_add_release_u32(a.gbar, 1u);
            const uint64_t t0 = globaltimer();
            while (ld_acquire_u32(a.gbar) < gridDim.x) {
                if (globaltimer() - t0 > a.timeout_ns) {
                    raise_error(a.err, ctl, kErrTimeoutGrid);
                    break;
                }
                __nanosleep(32);
            }
        }
        __syncthreads();
        if (tid == 0) stamp(a, kTrBarrier);
        for (int w = tid; w < W; w += kTcThreads) bits[w] = __ldcg(a.tc_bits + w);
    }
    __syncthreads();
    scan_popc(bits, W, prefix, wtot);  // ends with __syncthreads
    if (tid == 0) stamp(a, kTrScan);
    const int U = prefix[W];
    // A union covering most of the neurons streams whole row ranges: every
    // neuron is a position (Uv = f), rows arrive as 2-D TMA boxes at the
    // copy engine's rate, and the inactive neurons' h is zero by the mask.
    // ...when it also needs no more tiles per cluster than the gathered union
    // (the row-range shares are whole kBoxRows boxes): at 7B B = 32 (U/f =
    // 0.85) the gather fits one 128-row tile per cluster and whole ranges
    // two (87 against 69 us); at 13B B = 64 (U/f = 0.93) both need two and
    // whole ranges win (112.6 against 122.7 us).
    const bool dense = !kQuant && U >= a.dense_min &&
                       tiles_of(kBoxRows * ((a.W * 32 / kBoxRows + nclu - 1) / nclu)) <= tiles_of((U + nclu - 1) / nclu);
    const int Uv = dense ? a.f : U;
    // gate/up work of this cluster
    const int P0 = span_start(dense, Uv, clu, nclu);
    const int n = span_start(dense, Uv, clu + 1, nclu) - P0;
    const int ntile = tiles_of(n);
    // down unit of this CTA: 256-column slice m of union chunk k
    const int MT = a.d / kSlice;
    const int unit = blockIdx.x;
    const bool has_dn = unit < MT * a.KC;
    const int m = unit % MT, k = unit / MT;
    const int Q0 = has_dn ? chunk_start(Uv, k, a.KC) : 0;
    const int Q1 = has_dn ? chunk_start(Uv, k + 1, a.KC) : 0;
    const int ndn = (Q1 - Q0 + kDnRows - 1) / kDnRows;  // down stages
    if (blockIdx.x == 0 && tid == 0) *a.count_out = U;
    if (!dense) emit_ids16(bits, prefix, W, P0, P0 + n, gu_ids, warp, kTcWarps);
    if (tid == 0) stamp(a, kTrEmitGu);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    if (tid == 0) stamp(a, kTrScanned);
    // The next launch on the stream may be scheduled now; it waits for this
    // grid to finish before it touches anything.
    if (tid == 0) grid_launch_dependents();

    const int KG = a.d / (64 * nkb);

    if (kQuant && warp >= kProducerWarp0 && warp < kMmaWarp) {
        // ------------------------------------------------- producers (quantised)
        const int pt = tid - kProducerWarp0 * 32;
        const QuantProducer qp{ctl, ring, stg, pt, NU, nkb, rank ? a.wu : a.wg, (KG ? clu % KG : 0), KG, m, n, ntile,
                               gu_ids, dn_ids, Q0, Q1};
        bool ok = !ctl->abort;
        const int ngu = ntile * KG, total = ngu + ndn, S = a.nstg;
        if (pt < kQCopyThreads) {
            // copying threads: stage t's raw blocks into slot t % S once the
            // expansion of stage t - S has emptied it; they run up to S
            // stages ahead of the expansion
            for (int t = 0; t < total && ok; ++t) {
                // the down stages' ids come from the epilogue warps
                if (t == ngu) ok = wait_bar(&ctl->ids_ready, 0, ctl, a, kErrTimeoutAcc, a.hint);
                if (ok && t >= S)
                    ok = wait_bar(&ctl->stg_empty[t % S], (uint32_t)(t / S - 1) & 1u, ctl, a, kErrTimeoutFull, a.hint);
                if (ok) qp.issue(a, qp.stage(t), t % S, pt, kQCopyThreads);
            }
            // Every copy this thread issued lands before the CTA can exit.
            cp_async_wait_all();
        } else {
            // expanding threads: each landed slot into its ring unit
            const int lt = pt - kQCopyThreads;
            for (int t = 0; t < total && ok; ++t) {
                ok = wait_bar(&ctl->stg_full[t % S], (uint32_t)(t / S) & 1u, ctl, a, kErrTimeoutFull, a.hint);
                if (ok) ok = qp.finish(a, qp.stage(t), t % S, lt, kQExpThreads);
            }
        }
    } else if (warp >= kProducerWarp0 && warp < kMmaWarp && !dense) {
        // ------------------------------------------------------------ producers
        // (idle when whole row ranges stream: the TMA warp moves the rows)
        const int pt = tid - kProducerWarp0 * 32, pw = pt >> 5;
        const bool leader = pt == 0;  // stamps only
        const __half *wm = rank ? a.wu : a.wg;
        const int rot = KG ? clu % KG : 0;  // spreads the clusters' column windows over DRAM
        const int cpr = nkb * 8;            // 16-byte chunks per row run
        const int rpw = 32 / cpr;           // rows per warp instruction
        const int ch = lane & (cpr - 1), kbl = ch >> 3, cc = ch & 7;
        bool ok = !ctl->abort;
        int s = 0, t = 0;  // stage index (for stamps), unit-step
        for (int i = 0; i < ntile && ok; ++i) {
            int r0, r1;
            tile_rows(n, ntile, i, r0, r1);
            const int rows = r1 - r0;
            const uint16_t *tids = gu_ids + r0;
            for (int st = 0; st < KG; ++st, ++s, t += GW) {
                // the second unit of a two-unit stage is released by the
                // same commit as the first
                if (!(ok = ring_wait_empty(t, NU, ctl, a))) break;
                const uint32_t sbase = smem_u32(ring + (size_t)(t % NU) * a.unit_bytes);
                const int kbase = ((st + rot) % KG) * 64 * nkb;
                if (leader) stage_stamp(a, s, 0);
                // weight rows: rows x (nkb x 128 B); rows past the tile are not
                // copied (their MMA rows are never read)
                const uint32_t dl = sbase + kbl * kATile + (uint32_t)cc * 16;
                const __half *src = wm + kbase + ch * 8;
                for (int r = pw * rpw + lane / cpr; r < rows; r += kProducerWarps * rpw)
                    cp_async16_full((dl + r * 128) ^ ((uint32_t)(r & 7) << 4), src + (int64_t)tids[r] * a.d);
                cp_async_mbar_arrive(&ctl->full[t % NU]);
                if (GW == 2) cp_async_mbar_arrive(&ctl->full[(t + 1) % NU]);
                if (leader) stage_stamp(a, s, 1);
            }
        }
        if (leader) stamp(a, kTrGuIssued);
        // Down stages: W_down rows (64 positions x 256 columns, MN-major:
        // 64-column blocks kDnLbo apart, 8-row K groups 1024 B apart; rows past
        // the chunk up to the next multiple of 16 zero-filled) are copied at
        // once; the TMA warp adds the h tile once its producers published it.
        const int mb = lane >> 3, c8 = lane & 7;
        const int cbase = m * kSlice;
        if (ok && ndn > 0) ok = wait_bar(&ctl->ids_ready, 0, ctl, a, kErrTimeoutAcc, a.hint);
        for (int st = 0; st < ndn && ok; ++st, ++s, ++t) {
            if (!(ok = ring_wait_empty(t, NU, ctl, a))) break;
            const uint32_t sbase = smem_u32(ring + (size_t)(t % NU) * a.unit_bytes);
            const int p0 = Q0 + st * kDnRows;
            const int nr = min(kDnRows, Q1 - p0), nr16 = (nr + 15) & ~15;
            if (leader) stage_stamp(a, s, 0);
            for (int kk = pw; kk < (a.inject == 4 ? 0 : nr16); kk += kProducerWarps) {
                const bool valid = kk < nr;
                const int j = valid ? dn_ids[p0 - Q0 + kk] : 0;
                const int kg = kk >> 3, kr = kk & 7;
                cp_async16(sbase + mb * kDnLbo + kg * 1024 + kr * 128 + ((c8 ^ kr) << 4),
                           a.wd + (int64_t)j * a.d + cbase + lane * 8, valid ? 16u : 0u);
            }
            if (leader) stage_stamp(a, s, 1);
            cp_async_mbar_arrive(&ctl->full[t % NU]);
        }
        if (leader) stamp(a, kTrDnIssued);
        // Every copy this thread issued lands before the CTA can exit.
        cp_async_wait_all();
    } else if (warp == kTmaWarp) {
        // ------------------------------------------------------------ TMA issue
        // One thread streams the activation tiles of the gate/up stages and
        // the h tiles of the down stages into the ring, each on its slot's
        // transaction barrier.
        if (lane == 0) {
            int t = 0;  // unit-step
            // x16 was written by generic stores in phase 0 (by every CTA when
            // the sets came as bits); TMA reads through the async proxy
            bool ok = !ctl->abort;
            if (bits_in && ok) ok = wait_count(a.gbar + 1, gridDim.x, ctl, a);
            asm volatile("fence.proxy.async.global;" ::: "memory");
            const int rot = KG ? clu % KG : 0;
            const CUtensorMap *wmap = rank ? &maps.wu : &maps.wg;
            for (int i = 0; i < ntile && ok; ++i) {
                int r0 = 0, r1 = 0;
                if (dense) tile_span(true, n, ntile, i, r0, r1);
                // whole row ranges: the tile's rows as kBoxRows-row boxes per K block
                const int nbx = dense ? (r1 - r0 + kBoxRows - 1) / kBoxRows : 0;
                for (int st = 0; st < KG; ++st, t += GW) {
                    if (!(ok = ring_wait_empty(t, NU, ctl, a))) break;
                    const uint32_t sbase = smem_u32(ring + (size_t)(t % NU) * a.unit_bytes);
                    const int kbase = ((st + rot) % KG) * 64 * nkb;
                    uint64_t *bar = &ctl->tma[t % NU];
                    mbar_arrive_expect_tx(bar, (uint32_t)nkb * (Np + nbx * kBoxRows) * 128);
                    if (GW == 2) mbar_arrive(&ctl->tma[(t + 1) % NU]);
                    for (int kb = 0; kb < nkb; ++kb) {
                        tma_load_2d(sbase + nkb * kATile + kb * Np * 128, &maps.x, bar, kbase + kb * 64, 0);
                        for (int bx = 0; bx < nbx; ++bx)
                            tma_load_2d(sbase + kb * kATile + bx * kBoxRows * 128, wmap, bar, kbase + kb * 64,
                                        P0 + r0 + bx * kBoxRows);
                    }
                }
            }
            // clusters [.., cl_ok) are known to have published all their h
            int cl_ok = 0;
            while (cl_ok + 1 < nclu && span_start(dense, Uv, cl_ok + 1, nclu) <= Q0) ++cl_ok;
            for (int st = 0; st < ndn && ok; ++st, ++t) {
                if (!(ok = ring_wait_empty(t, NU, ctl, a))) break;
                const int p0 = Q0 + st * kDnRows;
                const int nr16 = (min(kDnRows, Q1 - p0) + 15) & ~15;
                // h of positions [p0, p0 + nr16): wait for every cluster that
                // owns one of them and has not been confirmed yet
                const int last = min(p0 + nr16, Uv) - 1;
                bool fresh = false;
                while (ok && cl_ok < nclu && span_start(dense, Uv, cl_ok, nclu) <= last) {
                    const int cn = span_start(dense, Uv, cl_ok + 1, nclu) - span_start(dense, Uv, cl_ok, nclu);
                    ok = wait_count(a.ready + cl_ok, 2u * (uint32_t)tiles_of(cn), ctl, a);
                    fresh = true;
                    ++cl_ok;
                }
                if (!ok) break;
                if (st == 0) stamp(a, kTrFirstFlag);
                // h was stored through the generic proxy; TMA reads through
                // the async proxy
                if (fresh) asm volatile("fence.proxy.async.global;" ::: "memory");
                const uint32_t sbase = smem_u32(ring + (size_t)(t % NU) * a.unit_bytes);
                mbar_arrive_expect_tx(&ctl->tma[t % NU], (uint32_t)Np * 128 + (dense ? kDnWBytes : 0u));
                tma_load_2d(sbase + kDnWBytes, &maps.h, &ctl->tma[t % NU], p0, 0);
                // whole row ranges: the 64 W_down rows as four 64-column boxes
                // (rows past f read as zero)
                if (dense)
                    for (int mb = 0; mb < 4; ++mb)
                        tma_load_2d(sbase + mb * kDnLbo, &maps.wd, &ctl->tma[t % NU], m * kSlice + mb * 64, p0);
            }
            // Every TMA this thread issued lands before the CTA can exit: the
            // last NU unit-steps it armed each complete their phase.
            const uint64_t t0 = globaltimer();
            for (int q = t - 1; q >= 0 && q >= t - NU; --q)
                while (!mbar_test_sleep(&ctl->tma[q % NU], (uint32_t)(q / NU) & 1u, 1000) &&
                       globaltimer() - t0 < a.timeout_ns) {
                }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_gu = idesc_f16_f32(kTileM, Np, false, false);
            const uint32_t id_dn = idesc_f16_f32(kTileM, Np, true, false);
            uint64_t *last_bar = nullptr;  // barrier of the most recent commit, for the drain
            uint32_t last_par = 0;
            bool ok = !ctl->abort;
            int s = 0, ub = 0;
            auto acquire_buf = [&](int &buf) -> bool {
                buf = ub % nbuf;
                const int rnd = ub / nbuf;
                if (rnd > 0 && !wait_bar(&ctl->acc_empty[buf], (rnd - 1) & 1, ctl, a, kErrTimeoutAcc, a.hint))
                    return false;
                tc_fence_after();
                return true;
            };
            int t = 0;  // unit-step
            // (whole row ranges: the TMA barrier alone covers the stage)
            auto wait_unit = [&](int q) -> bool {
                const uint32_t par = (uint32_t)(q / NU) & 1u;
                return (dense || wait_bar(&ctl->full[q % NU], par, ctl, a, kErrTimeoutFull, a.hint)) &&
                       wait_bar(&ctl->tma[q % NU], par, ctl, a, kErrTimeoutFull, a.hint);
            };
            // A two-unit stage is complete when its first unit is: the
            // producers' arrivals there cover every copy of the stage and the
            // TMA bytes are counted there; the second unit's barriers only
            // keep their phase count in step.
            auto wait_stage = [&](int) -> bool {
                if (!wait_unit(t)) return false;
                stage_stamp(a, s, 2);
                // the producers' cp.async data were written through the
                // generic proxy; make them visible to the MMA's async proxy
                fence_proxy_async_smem();
                tc_fence_after();
                return true;
            };
            auto commit_acc = [&](int buf) {
                unit_stamp(a, ub, 1);
                mma_commit(&ctl->acc_full[buf]);
                last_bar = &ctl->acc_full[buf];
                last_par = (uint32_t)(ub / nbuf) & 1u;
                ++ub;
            };
            for (int i = 0; i < ntile && ok; ++i) {
                int buf;
                if (!(ok = acquire_buf(buf))) break;
                const uint32_t dgu = tmem + (uint32_t)(buf * 2 * Np);
                for (int st = 0; st < KG; ++st, ++s, t += GW) {
                    if (!(ok = wait_stage(GW))) break;
                    if (st == 0) unit_stamp(a, ub, 0);
                    const uint32_t sbase = smem_u32(ring + (size_t)(t % NU) * a.unit_bytes);
                    const uint32_t xoff = sbase + (uint32_t)nkb * kATile;
                    for (int kb = 0; kb < nkb; ++kb) {
#pragma unroll
                        for (int k4 = 0; k4 < 4; ++k4) {
                            const uint64_t ad = desc_sw128(sbase + kb * kATile + k4 * 32, 16, 1024);
                            const uint64_t bd = desc_sw128(xoff + kb * Np * 128 + k4 * 32, 16, 1024);
                            mma_f16(dgu, ad, bd, id_gu, (st > 0 || kb > 0 || k4 > 0) ? 1u : 0u);
                        }
                    }
                    if (GW == 2) mma_commit(&ctl->empty[(t + 1) % NU]);
                    mma_commit(&ctl->empty[t % NU]);
                    last_bar = &ctl->empty[t % NU];
                    last_par = (uint32_t)(t / NU) & 1u;
                }
                if (!ok) break;
                commit_acc(buf);
            }
            if (ok && ndn > 0) {
                int buf;
                if ((ok = acquire_buf(buf))) {
                    const uint32_t ddn = tmem + (uint32_t)(buf * 2 * Np);
                    for (int st = 0; st < ndn; ++st, ++s, ++t) {
                        if (!(ok = wait_stage(1))) break;
                        if (st == 0) unit_stamp(a, ub, 0);
                        const uint32_t sbase = smem_u32(ring + (size_t)(t % NU) * a.unit_bytes);
                        const int nk = (min(kDnRows, Q1 - Q0 - st * kDnRows) + 15) >> 4;  // K steps of 16 positions
                        for (int ks = 0; ks < nk; ++ks) {
                            const uint64_t bd = desc_sw128(sbase + kDnWBytes + ks * 32, 16, 1024);
#pragma unroll
                            for (int mt = 0; mt < 2; ++mt) {
                                const uint64_t ad = desc_sw128(sbase + mt * 2 * kDnLbo + ks * 2 * 1024, kDnLbo, 1024);
                                mma_f16(ddn + mt * Np, ad, bd, id_dn, (st > 0 || ks > 0) ? 1u : 0u);
                            }
                        }
                        mma_commit(&ctl->empty[t % NU]);
                        last_bar = &ctl->empty[t % NU];
                        last_par = (uint32_t)(t / NU) & 1u;
                    }
                    if (ok) commit_acc(buf);
                }
            }
            // MMAs may still be reading shared memory or writing TMEM (after
            // an abort): wait for the last commit, which covers every earlier
            // tcgen05 operation, before the CTA releases either.
            if (last_bar) {
                const uint64_t t0 = globaltimer();
                while (!mbar_test_sleep(last_bar, last_par, 1000) && globaltimer() - t0 < a.timeout_ns) {
                }
            }
        }
        __syncwarp();
    } else if (warp < kEpiWarps) {
        // ------------------------------------------------------------ epilogue
        const int e = tid;  // TMEM lane == tile row (gate/up) or output column (down)
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        const uint32_t peer_full = mapa_shared(smem_u32(&ctl->xchg_full), peer);
        const uint32_t peer_free = mapa_shared(smem_u32(&ctl->xchg_free), peer);
        // slots hold 64 rows: the half of the tile the partner finishes
        float *myslot = a.xchg + (size_t)blockIdx.x * Np * 64;
        const float *peerslot = a.xchg + (size_t)(blockIdx.x ^ 1) * Np * 64;
        const uint32_t peer_recv = mapa_shared(smem_u32(xrecv), peer);
        const bool signal = !(a.inject == 1 && rank == 1);
        const bool mine_half = (e >> 6) == (int)rank;  // rows this CTA finishes (warp-uniform)
        // the down unit's ids, while the gate/up stages stream
        if (!dense) emit_ids16(bits, prefix, W, Q0, Q1, dn_ids, warp, kEpiWarps);
        if (e == 0) stamp(a, kTrEmitDn);
        mbar_arrive(&ctl->ids_ready);
        int ub = 0;
        bool ok = named_bar_and(kEpiBar, 128, !ctl->abort);
        for (int i = 0; i < ntile && ok; ++i) {
            int r0, r1;
            tile_span(dense, n, ntile, i, r0, r1);
            const int rows = r1 - r0;
            const bool valid = e < rows;
            const int j = valid ? (dense ? P0 + r0 + e : gu_ids[r0 + e]) : 0;
            // While the gate/up MMAs run: this row's per-token activity bits
            // (bit t of word t/32), so forming h reads no global memory.
            if (mine_half) {
                for (int t0 = 0; t0 < Np; t0 += 32) {
                    uint32_t word = 0;
                    if (!a.per_token) {
                        // union semantics: every union neuron for every token
                        // (whole row ranges also hold neurons outside it)
                        word = (!dense || (valid && ((bits[j >> 5] >> (j & 31)) & 1u))) ? ~0u : 0u;
                    } else if (valid && a.tok_in) {
                        const uint32_t *mcol = a.tok_in + (j >> 5);
#pragma unroll 8
                        for (int q = 0; q < 32; ++q)
                            if (t0 + q < a.B) word |= ((__ldg(mcol + (int64_t)(t0 + q) * W) >> (j & 31)) & 1u) << q;
                    } else if (valid) {
                        const float *lcol = a.labels + j;
#pragma unroll 8
                        for (int q = 0; q < 32; ++q)
                            if (t0 + q < a.B) word |= (__ldg(lcol + (int64_t)(t0 + q) * a.f) > 0.0f ? 1u : 0u) << q;
                    }
                    tokmask[(t0 >> 5) * kTileM + e] = word;
                }
            }
            const int buf = ub % nbuf;
            ok = wait_bar(&ctl->acc_full[buf], (uint32_t)(ub / nbuf) & 1u, ctl, a, kErrTimeoutAcc, a.hint_acc);
            if (!(ok = named_bar_and(kEpiBar, 128, ok))) break;
            tc_fence_after();
            if (e == 0) unit_stamp(a, ub, 2);
            if (i == 0 && e == 0) stamp(a, kTrGuAcc);
            const uint32_t acc = trow + (uint32_t)(buf * 2 * Np);
            // 1. results for the partner's rows to this CTA's slot, once the
            //    partner has read the previous tile's
            if (i > 0) ok = wait_bar_cluster(&ctl->xchg_free, (uint32_t)(i - 1) & 1u, ctl, a, kErrTimeoutXchg);
            if (!(ok = named_bar_and(kEpiBar, 128, ok))) break;
            if (!mine_half) {
                for (int c0 = 0; c0 < Np; c0 += 16) {
                    float v[16];
                    tmem_ld16(acc + c0, v);
                    tmem_ld_wait();
                    if (a.xdsm) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) st_shared_cluster_f32(peer_recv + ((c0 + q) * 64 + (e & 63)) * 4, v[q]);
                    } else {
#pragma unroll
                        for (int q = 0; q < 16; ++q) __stcg(myslot + (size_t)(c0 + q) * 64 + (e & 63), v[q]);
                    }
                }
            }
            if (signal) mbar_arrive_remote(peer_full);
            // 2. the partner's results for this CTA's rows
            ok = wait_bar_cluster(&ctl->xchg_full, (uint32_t)i & 1u, ctl, a, kErrTimeoutXchg);
            if (!(ok = named_bar_and(kEpiBar, 128, ok))) break;
            if (i == 0 && e == 0) stamp(a, kTrXchg);
            // 3. h = act(gate, up) * mask for this CTA's rows -> fp16 h16[t][pos]
            const int pos = P0 + r0 + e;
            if (mine_half) {
                __half *hcol = a.h16 + pos;
                const float bgj = (a.bias_g && valid) ? __half2float(a.bias_g[j]) : 0.0f;
                const float buj = (a.bias_u && valid) ? __half2float(a.bias_u[j]) : 0.0f;
                for (int c0 = 0; c0 < Np; c0 += 16) {
                    float mine[16];
                    tmem_ld16(acc + c0, mine);
                    float other[16];
                    if (a.xdsm) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) other[q] = xrecv[(c0 + q) * 64 + (e & 63)];
                    } else {
#pragma unroll
                        for (int q = 0; q < 16; ++q) other[q] = __ldcg(peerslot + (size_t)(c0 + q) * 64 + (e & 63));
                    }
                    const uint32_t mw = tokmask[(c0 >> 5) * kTileM + e] >> (c0 & 31);
                    tmem_ld_wait();
                    if (valid) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const int t = c0 + q;
                            // sparse bias add (cuda/kernel.cu:818-830) before the activation
                            const float g = (rank ? other[q] : mine[q]) + bgj;
                            const float u = (rank ? mine[q] : other[q]) + buj;
                            float hv = 0.0f;
                            if (t < a.B && ((mw >> q) & 1u)) hv = act_h(g, u, a.act);
                            hcol[(int64_t)t * a.fpad] = __float2half_rn(hv);
                        }
                    }
                }
                if (valid && !dense) a.merge_out[pos] = j;
            }
            mbar_arrive_remote(peer_free);  // the partner's slot has been read
            tc_fence_before();
            mbar_arrive(&ctl->acc_empty[buf]);
            // positions [Uv, Uv rounded up to 64) of h are read by the last
            // down stage: the cluster holding position U - 1 zeroes them
            if (i == ntile - 1 && P0 + n == Uv && rank == 0) {
                const int tail = ((Uv + 63) & ~63) - Uv;
                for (int q = e; q < tail * Np; q += 128)
                    a.h16[(int64_t)(q / tail) * a.fpad + Uv + q % tail] = __float2half_rn(0.0f);
            }
            // publish: h rows of this tile (and the zero tail) visible GPU-wide
            // before the cluster's counter moves
            __threadfence();
            named_bar(kEpiBar, 128);
            if (e == 0) {
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.ready + clu) : "memory");
                unit_stamp(a, ub, 3);
            }
            ++ub;
        }
        if (e == 0) stamp(a, kTrHDone);
        if (ok && ndn > 0) {
            // 4. the down unit: out[t][256 m + col] += acc (once every CTA's
            // share of `out` is zeroed)
            const int buf = ub % nbuf;
            ok = wait_bar(&ctl->acc_full[buf], (uint32_t)(ub / nbuf) & 1u, ctl, a, kErrTimeoutAcc, a.hint_acc);
            if (ok && bits_in) ok = wait_count(a.gbar + 1, gridDim.x, ctl, a);
            if ((ok = named_bar_and(kEpiBar, 128, ok))) {
                tc_fence_after();
                if (e == 0) {
                    unit_stamp(a, ub, 2);
                    stamp(a, kTrDnAcc);
                }
                const uint32_t dacc = trow + (uint32_t)(buf * 2 * Np);
#pragma unroll 1
                for (int mt = 0; mt < 2; ++mt) {
                    // lane 4q + r adds columns [4q, 4q + 4) of its quad for
                    // token c0 + 4g + r: one 16-byte reduction instead of four
                    float *oquad = a.out + m * kSlice + mt * kTileM + (e & ~3);
                    for (int c0 = 0; c0 < Np && c0 < a.B; c0 += 16) {
                        float v[16];
                        tmem_ld16(dacc + mt * Np + c0, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int g = 0; g < 4; ++g) {
                            quad_transpose(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
                            const int t = c0 + 4 * g + (e & 3);
                            if (t < a.B && a.inject != 2)
                                red_add_v4(oquad + (int64_t)t * a.d, v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&ctl->acc_empty[buf]);
                if (e == 0) unit_stamp(a, ub, 3);
            }
        }
    }

    __syncthreads();
    if (tid == 0) stamp(a, kTrEnd);
    // The last CTA to finish resets the per-launch counters: every other CTA
    // has passed all its waits on them.
    if (tid == 0) {
        __threadfence();
        ctl->last = atomicAdd(a.gbar + 2, 1u) == gridDim.x - 1;
        if (ctl->last) {
            for (int c = 0; c < nclu; ++c) a.ready[c] = 0u;
            a.gbar[0] = 0u;
            a.gbar[1] = 0u;
            a.gbar[2] = 0u;
        }
    }
    __syncthreads();
    if (ctl->last && !bits_in)
        for (int w = tid; w < W; w += kTcThreads) a.tc_bits[w] = 0u;
    // The partner may still signal this CTA's barriers until it is done.
    cluster_sync_all();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
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
    CUtensorMap mp;
    memset(&mp, 0, sizeof(mp));
    const CUresult r = encode(&mp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    if (cache.size() > 4096) cache.clear();
    cache.push_back({key, mp});
    *out = mp;
    return SPB_OK;
}

}  // namespace

// Ring geometry: K blocks per gate/up stage, unit size and unit count.  A
// down stage (64 W_down rows x 256 columns + the h tile) fills one unit; a
// gate/up stage (nkb K blocks of 128 rows + the activation tile) one or two.
struct Geometry {
    int nkb, nu, gw;
    uint32_t unit_bytes;
    size_t smem;
};

// Pairs exchange their gate/up halves through distributed shared memory up
// to this batch width (an [Np][64] fp32 receive buffer), through L2 above it.
constexpr int kXdsmMaxNp = 64;

static size_t fixed_smem(int Np, int W, int max_gu, int max_dn) {
    return sizeof(TcCtl) + sizeof(uint32_t) * 8 * kTileM + sizeof(uint16_t) * (size_t)(max_gu + max_dn) + 16 +
           (Np <= kXdsmMaxNp ? sizeof(float) * 64 * (size_t)Np : 0) + sizeof(int) * (size_t)(2 * W + 65) + 1024 + 64;
}

static Geometry pick_geometry(int Np, int W, int max_gu, int max_dn, int d, int force_nkb, int force_units,
                              bool no_split) {
    const size_t fixed = fixed_smem(Np, W, max_gu, max_dn);
    const size_t budget = 227 * 1024;
    const uint32_t dn = (kDnWBytes + (uint32_t)Np * 128 + 1023) & ~1023u;
    // The copy rate follows the weight bytes in flight and the contiguous run
    // per row (128 * nkb bytes): score the smaller of the gate/up and down
    // weight bytes in flight, weighted towards longer runs.
    Geometry best{0, 0, 0, 0, 0};
    size_t best_score = 0;
    for (int nkb = 4; nkb >= 1; nkb >>= 1) {
        if (force_nkb && nkb != force_nkb) continue;
        if ((d / 64) % nkb) continue;
        const uint32_t gu = ((uint32_t)nkb * (kATile + (uint32_t)Np * 128) + 1023) & ~1023u;
        // When two down stages fit in one gate/up stage, the ring counts
        // half-stage units: a gate/up stage takes two, a down stage one, so
        // twice as many down stages are in flight (and prefetched while the
        // gate/up phase ends).
        const bool halves = !no_split && 2 * dn <= gu;
        const uint32_t unit = halves ? gu / 2 : (gu > dn ? gu : dn);
        const int gw = halves ? 2 : 1;
        if (budget < fixed + 2u * gw * unit) continue;
        int nu = (int)std::min<size_t>((budget - fixed) / unit, kMaxUnits);
        if (force_units) nu = std::min(nu, force_units);
        if (gw == 2) nu &= ~1;
        if (nu < 2 * gw) continue;
        const size_t in_gu = (size_t)(nu / gw - 1) * nkb * kATile, in_dn = (size_t)(nu - 1) * kDnWBytes;
        const size_t score = std::min(in_gu, in_dn) * (size_t)(nkb * nkb);
        if (score > best_score) {
            best_score = score;
            best = Geometry{nkb, nu, gw, unit, fixed + (size_t)nu * unit};
        }
    }
    return best;
}

// Quantised weights: ring units hold the expanded fp16 stages (whole-stage
// units) and the staging slots hold the raw blocks of nstg stages.
struct QGeometry {
    Geometry g;
    int nstg, tasks;
    uint32_t slot;
};

static QGeometry pick_geometry_quant(int Np, int W, int max_gu, int max_dn, int d, int wtype, int force_nkb) {
    const size_t fixed = fixed_smem(Np, W, max_gu, max_dn);
    const size_t budget = 227 * 1024;
    const uint32_t qb = wtype == SPB_W_Q8_0 ? 32u : 16u;
    const uint32_t dn = (kDnWBytes + (uint32_t)Np * 128 + 1023) & ~1023u;
    QGeometry best{};
    size_t best_score = 0;
    for (int nkb = 4; nkb >= 1; nkb >>= 1) {
        if (force_nkb && nkb != force_nkb) continue;
        if ((d / 64) % nkb) continue;
        const uint32_t gu = ((uint32_t)nkb * (kATile + (uint32_t)Np * 128) + 1023) & ~1023u;
        const uint32_t unit = gu > dn ? gu : dn;
        const int tasks = std::max(kTileM * 2 * nkb, kDnRows * 8);
        const uint32_t slot = ((uint32_t)tasks * (qb + 4) + 127) & ~127u;
        for (int nu = 2; nu <= kMaxUnits; ++nu) {
            if (fixed + (size_t)nu * unit + 2u * slot > budget) break;
            const int nstg = (int)std::min<size_t>((budget - fixed - (size_t)nu * unit) / slot, kMaxStaging);
            // Every stage costs a round trip through the ring (the activation
            // tile's TMA, the expansion, the MMA's release), so the widest
            // stages win; then the stages staged ahead, then a third unit.
            const size_t score = (size_t)nkb * 1000000 + (size_t)nstg * 10 + (nu >= 3 ? 1 : 0);
            if (score > best_score) {
                best_score = score;
                best = QGeometry{Geometry{nkb, nu, 1, unit, fixed + (size_t)nu * unit + (size_t)nstg * slot}, nstg,
                                 tasks, slot};
            }
        }
    }
    return best;
}

// Clusters of two that can be resident at once with `smem` bytes per CTA
// (cached per device and size).
static int max_clusters(const void *kernel, size_t smem, int sms) {
    struct Entry {
        int dev;
        const void *kernel;
        size_t smem;
        int n;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return sms / 2;
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : cache)
        if (e.dev == dev && e.kernel == kernel && e.smem == smem) return e.n;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sms / 2;
    }
    n = std::min(n, sms / 2);
    cache.push_back(Entry{dev, kernel, smem, n});
    return n;
}

int launch_ffn_tc(const TcLaunch &L, cudaStream_t st) {
    const int Np = L.Np;
    if (Np < 16 || Np > 256 || Np % 16) return fail(SPB_ERR_UNSUPPORTED, "tensor path: batch must be 1..256");
    if (L.d % kSlice) return fail(SPB_ERR_INVALID, "tensor path: d must be a multiple of 256");
    const DebugHooks &dbg = debug_hooks();
    TcArgs a{};
    a.wg = static_cast<const __half *>(L.wg);
    a.wu = static_cast<const __half *>(L.wu);
    a.wd = static_cast<const __half *>(L.wd);
    a.wtype = L.wtype;
    a.rowb = L.wtype == SPB_W_F16 ? (int64_t)L.d * 2
                                  : (L.wtype == SPB_W_Q8_0 ? (int64_t)L.d + L.d / 16 : (int64_t)L.d / 2 + L.d / 16);
    a.labels = L.labels;
    a.tok_in = L.tok_in;
    a.x = L.x;
    a.x16 = L.x16;
    a.gbar = L.gbar;
    a.bias_g = L.bias_g;
    a.bias_u = L.bias_u;
    a.h16 = L.h16;
    a.seg_bits = L.seg_bits;
    a.tc_bits = L.tc_bits;
    a.out = L.out;
    a.merge_out = L.merge_out;
    a.count_out = L.count_out;
    a.xchg = L.xchg;
    a.ready = L.ready;
    a.err = L.err;
    a.trace = static_cast<unsigned long long *>(trace_buffer((size_t)kStageTraceBase + kStageTraceMax * 4));
    a.B = L.B;
    a.Np = Np;
    a.d = L.d;
    a.f = L.f;
    a.W = words_of(L.f);
    a.fpad = L.fpad;
    a.act = L.act;
    a.per_token = L.per_token;
    a.timeout_ns = dbg.timeout_ns ? dbg.timeout_ns : kDefaultTimeoutNs;
    a.hint_acc = dbg.hint_acc ? dbg.hint_acc : 20000;
    a.hint = dbg.hint ? dbg.hint : 1000;
    a.inject = dbg.inject;
    a.nbuf = std::min<int>(kMaxBufs, (int)kTmemCols / (2 * Np));
    a.xdsm = Np <= kXdsmMaxNp ? 1 : 0;

    const int sms = std::min(L.grid, kMaxTcGrid);
    const void *kernel = L.wtype == SPB_W_F16 ? (const void *)ffn_tc_kernel<false> : (const void *)ffn_tc_kernel<true>;
    const int MT = L.d / kSlice;
    // size the id tables for the most clusters this device can hold, then
    // check the launch against the real count
    int nclu = sms / 2;
    Geometry g{};
    int rc;
    for (int pass = 0; pass < 2; ++pass) {
        a.KC = std::max(1, (2 * nclu) / MT);
        a.max_gu = (L.f + nclu - 1) / nclu + 1;
        a.max_dn = (L.f + a.KC - 1) / a.KC + 128;
        if (L.wtype == SPB_W_F16) {
            g = pick_geometry(Np, a.W, a.max_gu, a.max_dn, L.d, dbg.nkb, dbg.stages, dbg.split_stages != 0);
            a.nstg = 0;
            a.stg_bytes = 0;
            a.stg_tasks = 0;
        } else {
            const QGeometry q = pick_geometry_quant(Np, a.W, a.max_gu, a.max_dn, L.d, L.wtype, dbg.nkb);
            g = q.g;
            a.nstg = q.nstg;
            a.stg_bytes = q.slot;
            a.stg_tasks = q.tasks;
            if (g.nu >= 2 && q.nstg < 2) g.nu = 0;
        }
        if (g.nu < 2) return fail(SPB_ERR_UNSUPPORTED, "tensor path: shared memory too small for two stages");
        if ((rc = ensure_smem(kernel, g.smem))) return rc;
        const int fit = max_clusters(kernel, g.smem, sms);
        if (fit >= nclu) break;
        nclu = std::max(1, fit);
    }
    a.nu = g.nu;
    a.gw = g.gw;
    a.nkb = g.nkb;
    a.unit_bytes = g.unit_bytes;

    TcMaps maps;
    if ((rc = tensor_map(L.x16, L.d, Np, Np, &maps.x))) return rc;
    if ((rc = tensor_map(L.h16, L.fpad, Np, Np, &maps.h))) return rc;
    // Whole row ranges stream when the union covers nearly all neurons (fp16
    // rows; not when the compacted ids are asked for).  Measured on B200 (7B):
    // at U/f = 0.85 (B = 32) streaming whole ranges took 87 us against 69 us
    // gathering -- the kBoxRows-aligned shares leave clusters with a 96- and
    // a 64-row tile, twice the ring stages -- while at U/f = 0.99 (B = 64) it
    // took 95.9 us against 99.9 us.
    a.dense_min = INT32_MAX;
    if (L.wtype == SPB_W_F16 && L.allow_dense) {
        const int permille = dbg.dense_permille ? dbg.dense_permille : kDenseMinPermille;
        if (permille <= 1000) {
            a.dense_min = (int)(((int64_t)L.f * permille + 999) / 1000);
            if ((rc = tensor_map(L.wg, L.d, L.f, kBoxRows, &maps.wg))) return rc;
            if ((rc = tensor_map(L.wu, L.d, L.f, kBoxRows, &maps.wu))) return rc;
            if ((rc = tensor_map(L.wd, L.d, L.f, kDnRows, &maps.wd))) return rc;
        }
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * nclu);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[3];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // CTAs of the down phase wait for h that CTAs of other clusters publish:
    // the cooperative launch guarantees every CTA is resident at once (the
    // launch fails instead if the grid cannot be)
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    attr[2].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[2].val.programmaticStreamSerializationAllowed = 1;
    // measurement hook (debug library only): drop attributes to see their cost
    int na = 0;
    cudaLaunchAttribute use[3];
    for (int i = 0; i < 3; ++i) {
        if (i == 1 && (dbg.launch_flags & 1)) continue;
        if (i == 2 && (dbg.launch_flags & 2)) continue;
        use[na++] = attr[i];
    }
    cfg.attrs = use;
    cfg.numAttrs = na;
    if (L.wtype == SPB_W_F16)
        SPB_CUDA_TRY(cudaLaunchKernelEx(&cfg, ffn_tc_kernel<false>, maps, a));
    else
        SPB_CUDA_TRY(cudaLaunchKernelEx(&cfg, ffn_tc_kernel<true>, maps, a));
    return SPB_OK;
}

}  // namespace spb
