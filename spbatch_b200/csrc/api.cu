// C ABI (include/spb.h): argument checking, workspace carving and launch
// sequencing.  No entry point synchronises the host or allocates memory.
#include <cstdio>
#include <mutex>
#include <vector>

#include "spb_internal.h"
#ifdef SPB_DEBUG_HOOKS
#include "spb_debug.h"
#endif

namespace spb {

static thread_local std::string g_last_error;

void set_error(const std::string &msg) { g_last_error = msg; }

int fail(int status, const std::string &msg) {
    g_last_error = msg;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    return SPB_ERR_CUDA;
}

int num_sms() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return kNumSMs;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = kNumSMs;
        cache[dev] = n;
    }
    return cache[dev];
}

int ensure_smem(const void *kernel, size_t bytes) {
    static std::mutex mu;
    static std::vector<std::pair<std::pair<int, const void *>, size_t>> done;
    int dev = 0;
    SPB_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : done) {
        if (e.first.first == dev && e.first.second == kernel) {
            if (e.second >= bytes) return SPB_OK;
            SPB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
            e.second = bytes;
            return SPB_OK;
        }
    }
    if (bytes > 48 * 1024)
        SPB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    done.push_back({{dev, kernel}, bytes < 48 * 1024 ? 48 * 1024 : bytes});
    return SPB_OK;
}

constexpr int kGemvMaxBatch = 4;

static std::mutex g_trace_mu;
static void *g_trace_buf = nullptr;
static size_t g_trace_slots = 0;

void *trace_buffer(size_t slots) {
    std::lock_guard<std::mutex> lk(g_trace_mu);
    return g_trace_buf && slots <= g_trace_slots ? g_trace_buf : nullptr;
}

static DebugHooks g_debug;

const DebugHooks &debug_hooks() { return g_debug; }

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace spb

using namespace spb;

extern "C" {

const char *spb_last_error(void) { return g_last_error.c_str(); }

int spb_version(void) { return 1; }

size_t spb_ffn_workspace_bytes(int B, int d, int f, int group) {
    if (B <= 0 || d <= 0 || f <= 0) return 0;
    return carve_workspace(nullptr, B, d, f, group).bytes;
}

int spb_union(const float *idx, int B, int f, int group, int32_t *merge_idx, int32_t *act_cum, uint32_t *tok_bits,
              void *workspace, size_t workspace_bytes, void *stream) {
    if (!idx || !merge_idx || !act_cum) return fail(SPB_ERR_INVALID, "spb_union: null pointer");
    if (B <= 0 || f <= 0 || group < 0) return fail(SPB_ERR_INVALID, "spb_union: bad shape");
    const int G = group == 0 ? B : group;
    const int S = (B + G - 1) / G;
    Workspace ws = carve_workspace(workspace, B, 0, f, group);
    if (!workspace || workspace_bytes < ws.bytes) return fail(SPB_ERR_WORKSPACE, "spb_union: workspace too small");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = launch_union_bits(idx, B, f, G, tok_bits, ws.seg_bits, PrepJobs{}, st);
    if (rc) return rc;
    return launch_compact(ws.seg_bits, S, f, merge_idx, act_cum, ws.counts, st);
}

}  // extern "C"

// The layer with the active sets either as fp32 labels (idx) or as per-token
// bit words (tok_in); exactly one of the two is given.
static int ffn_impl(const void *w_gate, const void *w_up, const void *w_down, int wtype, const float *x,
                    const float *idx, const uint32_t *tok_in, const void *bias_gate, const void *bias_up, int B,
                    int d, int f, int act, int per_token_mask, int path, float *out, int32_t *merge_idx_out,
                    int32_t *count_out, void *workspace, size_t workspace_bytes, void *stream) {
    const __half *bg = static_cast<const __half *>(bias_gate), *bu = static_cast<const __half *>(bias_up);
    if (!w_gate || !w_up || !w_down || !x || (!idx && !tok_in) || !out)
        return fail(SPB_ERR_INVALID, "spb_ffn_forward: null pointer");
    if (B <= 0 || d <= 0 || f <= 0) return fail(SPB_ERR_INVALID, "spb_ffn_forward: bad shape");
    if (d % 64 != 0) return fail(SPB_ERR_INVALID, "spb_ffn_forward: d must be a multiple of 64");
    if (B > 256) return fail(SPB_ERR_UNSUPPORTED, "spb_ffn_forward: B > 256");
    if (wtype != SPB_W_F16 && wtype != SPB_W_Q8_0 && wtype != SPB_W_Q4_0)
        return fail(SPB_ERR_INVALID, "spb_ffn_forward: unknown weight type");
    if (act != SPB_ACT_RELU_MUL && act != SPB_ACT_RELU_RELU_MUL)
        return fail(SPB_ERR_INVALID, "spb_ffn_forward: unknown activation");
    if (!aligned16(w_gate) || !aligned16(w_up) || !aligned16(w_down) || !aligned16(x) || !aligned16(out))
        return fail(SPB_ERR_INVALID, "spb_ffn_forward: weights, x and out must be 16-byte aligned");
    if (words_of(f) > 1024) return fail(SPB_ERR_UNSUPPORTED, "spb_ffn_forward: f > 32768");
    Workspace ws = carve_workspace(workspace, B, d, f, 0);
    if (!workspace || workspace_bytes < ws.bytes)
        return fail(SPB_ERR_WORKSPACE, "spb_ffn_forward: workspace too small");
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // Batches of up to four tokens stream on the CUDA cores; larger ones take
    // the tensor-core path (fp16 or quantised rows, d a multiple of 256).
    if (path == SPB_PATH_AUTO) path = (B <= kGemvMaxBatch || d % 256 != 0) ? SPB_PATH_GEMV : SPB_PATH_TENSOR;
    int32_t *merge = merge_idx_out ? merge_idx_out : ws.merge_idx;
    int32_t *count = count_out ? count_out : ws.counts;

    if (path == SPB_PATH_TENSOR) {
        if (B > 256) return fail(SPB_ERR_UNSUPPORTED, "spb_ffn_forward: tensor path serves B <= 256");
        if (d % 256 != 0) return fail(SPB_ERR_INVALID, "spb_ffn_forward: tensor path needs d % 256 == 0");
        // one cooperative launch: union, fp16 activations and the zeroed
        // output are its first phase
        TcLaunch L{};
        L.wg = w_gate;
        L.wu = w_up;
        L.wd = w_down;
        L.wtype = wtype;
        L.allow_dense = merge_idx_out == nullptr;
        L.labels = idx;
        L.tok_in = tok_in;
        L.bias_g = bg;
        L.bias_u = bu;
        L.x = x;
        L.gbar = ws.gbar;
        L.x16 = ws.x16;
        L.h16 = ws.h16;
        L.ready = ws.ready;
        L.fpad = ws.fpad;
        L.seg_bits = ws.seg_bits;
        L.tc_bits = ws.tc_bits;
        L.tok_bits = ws.tok_bits;
        L.out = out;
        L.merge_out = merge;
        L.count_out = count;
        L.xchg = ws.xchg;
        L.err = ws.err;
        L.B = B;
        L.Np = ws.Np;
        L.d = d;
        L.f = f;
        L.act = act;
        L.per_token = per_token_mask;
        L.grid = num_sms() < kMaxTcGrid ? num_sms() : kMaxTcGrid;
        return launch_ffn_tc(L, st);
    }
    if (path != SPB_PATH_GEMV) return fail(SPB_ERR_INVALID, "spb_ffn_forward: unknown path");

    if (stream_ffn_supported(wtype, B, d)) {
        StreamFfnArgs sa{};
        sa.wg = w_gate;
        sa.wu = w_up;
        sa.wd = w_down;
        sa.wtype = wtype;
        sa.x = x;
        sa.idx = idx;
        sa.tok_in = tok_in;
        sa.bias_g = bg;
        sa.bias_u = bu;
        sa.B = B;
        sa.d = d;
        sa.f = f;
        sa.act = act;
        sa.per_token = per_token_mask;
        sa.merge_out = merge_idx_out;
        sa.count_out = count_out;
        sa.out = out;
        sa.err = ws.err;
        sa.seg_bits = ws.seg_bits;
        sa.tok_bits = ws.tok_bits;
        sa.grid_bar = ws.grid_bar;
        sa.launch_ctr = ws.launch_ctr;
        sa.zero_flag = ws.zero_flag;
        return launch_stream_ffn(sa, st);
    }
    // With the per-token mask and no index outputs, token t's output depends
    // only on its own active set, so a batch the streaming kernel cannot hold
    // (quantised weights with B > 4, d > 4096 with B > 2) runs as consecutive
    // streaming launches over token groups it can hold: each group reads
    // its own union, at the streaming kernel's rate.
    int chunk = 4;
    while (chunk > 1 && !stream_ffn_supported(wtype, chunk, d)) chunk /= 2;
    if (per_token_mask && !merge_idx_out && !count_out && stream_ffn_supported(wtype, chunk, d)) {
        for (int t0 = 0; t0 < B; t0 += chunk) {
            StreamFfnArgs sa{};
            sa.wg = w_gate;
            sa.wu = w_up;
            sa.wd = w_down;
            sa.wtype = wtype;
            sa.x = x + (int64_t)t0 * d;
            sa.idx = idx ? idx + (int64_t)t0 * f : nullptr;
            sa.tok_in = tok_in ? tok_in + (int64_t)t0 * words_of(f) : nullptr;
            sa.bias_g = bg;
            sa.bias_u = bu;
            sa.B = B - t0 < chunk ? B - t0 : chunk;
            sa.d = d;
            sa.f = f;
            sa.act = act;
            sa.per_token = 1;
            sa.out = out + (int64_t)t0 * d;
            sa.err = ws.err;
            sa.seg_bits = ws.seg_bits;
            sa.tok_bits = ws.tok_bits;
            sa.grid_bar = ws.grid_bar;
            sa.launch_ctr = ws.launch_ctr;
            sa.zero_flag = ws.zero_flag;
            if (int rc = launch_stream_ffn(sa, st)) return rc;
        }
        return SPB_OK;
    }
    PrepJobs jobs;
    jobs.zero_out = out;
    jobs.zero_n = (int64_t)B * d;
    int rc = tok_in ? launch_union_from_bits(tok_in, B, f, B, ws.seg_bits, jobs, st)
                    : launch_union_bits(idx, B, f, B, ws.tok_bits, ws.seg_bits, jobs, st);
    if (rc) return rc;
    FusedGemvArgs a{};
    a.wg = w_gate;
    a.wu = w_up;
    a.wd = w_down;
    a.wtype = wtype;
    a.x = x;
    a.B = B;
    a.d = d;
    a.f = f;
    a.seg_bits = ws.seg_bits;
    a.tok_bits = tok_in ? tok_in : ws.tok_bits;
    a.bias_g = bg;
    a.bias_u = bu;
    a.act = act;
    a.per_token = per_token_mask;
    a.h = ws.h;
    a.merge = merge;
    a.count = count;
    a.out = out;
    a.err = ws.err;
    return launch_fused_gemv(a, st);
}

extern "C" {

int spb_ffn_forward(const void *w_gate, const void *w_up, const void *w_down, int wtype, const float *x,
                    const float *idx, int B, int d, int f, int act, int per_token_mask, int path, float *out,
                    int32_t *merge_idx_out, int32_t *count_out, void *workspace, size_t workspace_bytes,
                    void *stream) {
    if (!idx) return fail(SPB_ERR_INVALID, "spb_ffn_forward: null pointer");
    return ffn_impl(w_gate, w_up, w_down, wtype, x, idx, nullptr, nullptr, nullptr, B, d, f, act, per_token_mask,
                    path, out, merge_idx_out, count_out, workspace, workspace_bytes, stream);
}

int spb_ffn_forward_bits(const void *w_gate, const void *w_up, const void *w_down, int wtype, const float *x,
                         const uint32_t *tok_bits, int B, int d, int f, int act, int per_token_mask, int path,
                         float *out, int32_t *merge_idx_out, int32_t *count_out, void *workspace,
                         size_t workspace_bytes, void *stream) {
    if (!tok_bits) return fail(SPB_ERR_INVALID, "spb_ffn_forward_bits: null pointer");
    return ffn_impl(w_gate, w_up, w_down, wtype, x, nullptr, tok_bits, nullptr, nullptr, B, d, f, act,
                    per_token_mask, path, out, merge_idx_out, count_out, workspace, workspace_bytes, stream);
}

int spb_ffn_forward_bias(const void *w_gate, const void *w_up, const void *w_down, int wtype, const float *x,
                         const float *idx, const uint32_t *tok_bits, const void *bias_gate, const void *bias_up, int B,
                         int d, int f, int act, int per_token_mask, int path, float *out, int32_t *merge_idx_out,
                         int32_t *count_out, void *workspace, size_t workspace_bytes, void *stream) {
    if ((idx == nullptr) == (tok_bits == nullptr))
        return fail(SPB_ERR_INVALID, "spb_ffn_forward_bias: give exactly one of idx and tok_bits");
    if ((bias_gate && ((uintptr_t)bias_gate & 1)) || (bias_up && ((uintptr_t)bias_up & 1)))
        return fail(SPB_ERR_INVALID, "spb_ffn_forward_bias: biases must be 2-byte aligned fp16");
    return ffn_impl(w_gate, w_up, w_down, wtype, x, idx, tok_bits, bias_gate, bias_up, B, d, f, act, per_token_mask,
                    path, out, merge_idx_out, count_out, workspace, workspace_bytes, stream);
}

// Predictor workspace: fp16 hidden [B][D], fp32 logits [B][f], then the
// select's scratch (PredScratch).
static size_t predict_layout(int B, int d, int D, int f, char *base, __half **hidden, float **logits,
                             PredScratch *sc) {
    size_t off = 0;
    auto take = [&](size_t n) {
        char *p = base ? base + off : nullptr;
        off += align256(n);
        return p;
    };
    char *h = take(sizeof(__half) * (size_t)B * D);
    char *l = take(sizeof(float) * (size_t)B * f);
    char *hi = take(sizeof(uint32_t) * 2048 * (size_t)B);
    char *ca = take(sizeof(uint2) * (size_t)B * f);
    char *cc = take(sizeof(uint32_t) * (size_t)B);
    char *se = take(sizeof(int2) * (size_t)B);
    char *bi = take(sizeof(uint32_t) * (size_t)B * words_of(f));
    char *xh = B > kPredExactMaxBatch ? take(sizeof(__half) * (size_t)B * d) : nullptr;
    if (base) {
        sc->x16 = reinterpret_cast<__half *>(xh);
        *hidden = reinterpret_cast<__half *>(h);
        *logits = reinterpret_cast<float *>(l);
        sc->hist = reinterpret_cast<uint32_t *>(hi);
        sc->cand = reinterpret_cast<uint2 *>(ca);
        sc->cand_cnt = reinterpret_cast<uint32_t *>(cc);
        sc->sel = reinterpret_cast<int2 *>(se);
        sc->bits = reinterpret_cast<uint32_t *>(bi);
    }
    return off;
}

static size_t spb_predict_workspace_bytes_d(int B, int d, int D, int f) {
    if (B <= 0 || d <= 0 || D <= 0 || f <= 0) return 0;
    return predict_layout(B, d, D, f, nullptr, nullptr, nullptr, nullptr);
}

size_t spb_predict_workspace_bytes(int B, int D, int f) {
    // d is not known here: room for the largest activations the tensor-core
    // route stages (d up to 16384); spb_predict checks the actual need
    return spb_predict_workspace_bytes_d(B, 16384, D, f);
}

int spb_predict(const void *p1, const void *p2, const float *x, int B, int d, int D, int f, int k, float threshold,
                float *labels_out, uint32_t *bits_out, int32_t *idx_out, int32_t *count_out, float *logits_out,
                void *workspace, size_t workspace_bytes, void *stream) {
    if (!p1 || !p2 || !x || (!labels_out && !bits_out)) return fail(SPB_ERR_INVALID, "spb_predict: null pointer");
    if (B <= 0 || d <= 0 || D <= 0 || f <= 0 || k < 0) return fail(SPB_ERR_INVALID, "spb_predict: bad shape");
    if (d % 256 || D % 256) return fail(SPB_ERR_INVALID, "spb_predict: d and D must be multiples of 256");
    if (!aligned16(p1) || !aligned16(p2)) return fail(SPB_ERR_INVALID, "spb_predict: weights must be 16-byte aligned");
    const size_t need = spb_predict_workspace_bytes_d(B, d, D, f);
    if (!workspace || workspace_bytes < need) return fail(SPB_ERR_WORKSPACE, "spb_predict: workspace too small");
    __half *hidden = nullptr;
    float *logits = nullptr;
    PredScratch sc{};
    predict_layout(B, d, D, f, static_cast<char *>(workspace), &hidden, &logits, &sc);
    if (logits_out) logits = logits_out;
    return launch_predict(static_cast<const __half *>(p1), static_cast<const __half *>(p2), x, B, d, D, f, k,
                          threshold, labels_out, bits_out, idx_out, count_out, logits, hidden, sc,
                          static_cast<cudaStream_t>(stream));
}

int spb_trace_enable(void *device_buffer, size_t slots) {
    std::lock_guard<std::mutex> lk(g_trace_mu);
    g_trace_buf = device_buffer;
    g_trace_slots = device_buffer ? slots : 0;
    return SPB_OK;
}

#ifdef SPB_DEBUG_HOOKS
int spb_debug_config(int key, long long value) {
    switch (key) {
        case SPB_DEBUG_TIMEOUT_NS: g_debug.timeout_ns = value > 0 ? (uint64_t)value : 0; return SPB_OK;
        case SPB_DEBUG_INJECT: g_debug.inject = (int)value; return SPB_OK;
        case SPB_DEBUG_TC_NKB: g_debug.nkb = (int)value; return SPB_OK;
        case SPB_DEBUG_TC_STAGES: g_debug.stages = (int)value; return SPB_OK;
        case SPB_DEBUG_TC_HINT_ACC: g_debug.hint_acc = (uint32_t)value; return SPB_OK;
        case SPB_DEBUG_TC_HINT: g_debug.hint = (uint32_t)value; return SPB_OK;
        case SPB_DEBUG_TC_SPLIT_STAGES: g_debug.split_stages = (int)value; return SPB_OK;
        case SPB_DEBUG_TC_LAUNCH_FLAGS: g_debug.launch_flags = (int)value; return SPB_OK;
        case SPB_DEBUG_TC_DENSE_PERMILLE: g_debug.dense_permille = (int)value; return SPB_OK;
        default: return fail(SPB_ERR_INVALID, "spb_debug_config: unknown key");
    }
}
#endif

int spb_ffn_launches(int B, int d, int wtype, int path) {
    if (B <= 0 || d <= 0) return 0;
    if (path == SPB_PATH_AUTO) path = (B <= kGemvMaxBatch || d % 256 != 0) ? SPB_PATH_GEMV : SPB_PATH_TENSOR;
    if (path == SPB_PATH_TENSOR) return 1;  // one cooperative tensor-core launch
    if (stream_ffn_supported(wtype, B, d)) return 1;
    int chunk = 4;  // the token-group split spb_ffn_forward makes
    while (chunk > 1 && !stream_ffn_supported(wtype, chunk, d)) chunk /= 2;
    if (stream_ffn_supported(wtype, chunk, d)) return (B + chunk - 1) / chunk;
    return 3;  // union + fallback gate/up GEMV + down GEMV
}

}  // extern "C"
