// The reference's C++ host API (include/spbatch/kernel.cuh), implemented on
// the B200 kernels.  Each function keeps the reference's signature, argument
// meaning and error convention (print + exit(1)); the citations give the
// reference definition it replaces.
#include <mutex>
#include <unordered_map>

#include <vector>

#include "spb_internal.h"
#include "spbatch/kernel.cuh"

namespace {

using namespace spb;

[[noreturn]] void die(const char *what) {
    fprintf(stderr, "\nspbatch_b200: %s: %s\n", what, spb_last_error());
    exit(1);
}

#define DROPIN_OK(call)                 \
    do {                                \
        if ((call) != SPB_OK) die(#call); \
    } while (0)

// Per-device scratch that grows on demand (the reference keeps function-local
// statics sized by the first call, cuda/kernel.cu:882-905, which overflow when
// a later call is larger).
struct Scratch {
    void *ptr = nullptr;
    size_t bytes = 0;
};

void *scratch(int slot, size_t bytes) {
    static std::mutex mu;
    static std::unordered_map<int64_t, Scratch> table;
    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    Scratch &s = table[(int64_t)dev * 16 + slot];
    if (s.bytes < bytes) {
        if (s.ptr) CUDA_CHECK(cudaFree(s.ptr));
        CUDA_CHECK(cudaMalloc(&s.ptr, bytes));
        s.bytes = bytes;
    }
    return s.ptr;
}

// Sticky device error word for the drop-in kernels' bounded waits (the
// reference API returns void, so it is only there for inspection).
uint32_t *err_word() {
    static std::mutex mu;
    static std::unordered_map<int, uint32_t *> table;
    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    uint32_t *&p = table[dev];
    if (!p) {
        CUDA_CHECK(cudaMalloc(&p, 256));
        CUDA_CHECK(cudaMemset(p, 0, 256));
    }
    return p;
}

constexpr int kEw = 256;

__global__ void f32_to_f16_kernel(const float *__restrict__ x, __half *__restrict__ y, int k) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < k) y[i] = __float2half_rn(x[i]);
}

__global__ void f16_to_f32_kernel(const __half *__restrict__ x, float *__restrict__ y, int k) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < k) y[i] = __half2float(x[i]);
}

__global__ void relu_kernel(const float *__restrict__ x, float *__restrict__ y, int k) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < k) y[i] = fmaxf(x[i], 0.0f);
}

__global__ void mul_kernel(const float *__restrict__ x, const float *__restrict__ y, float *__restrict__ dst, int kx,
                           int ky) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < kx) dst[i] = x[i] * y[i % ky];
}

__global__ void relu_mul_kernel(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ dst,
                                int64_t n, int relu_u) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = fmaxf(g[i], 0.0f) * (relu_u ? fmaxf(u[i], 0.0f) : u[i]);
}

// PowerInfer-style per-token sparse GEMV (cuda/kernel.cu:358-425): warp per
// weight row; token c contributes when idx[c][row] > 0; dst accumulates.
__global__ void pi_gemv_kernel(const __half *__restrict__ w, const float *__restrict__ y, float *__restrict__ dst,
                               int ncols, int nrows, int ntok, int dst_ne0, const int *__restrict__ lst,
                               const float *__restrict__ idx) {
    const int gpu_row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gpu_row >= nrows) return;
    const int row = lst ? lst[gpu_row] : gpu_row;
    const __half *wr = w + (int64_t)gpu_row * ncols;
    for (int c = 0; c < ntok; ++c) {
        if (!(idx[(int64_t)c * dst_ne0 + row] > 0.0f)) continue;
        const float *yr = y + (int64_t)c * ncols;
        float acc = 0.0f;
        for (int k = lane; k < ncols; k += 32) acc = fmaf(__half2float(wr[k]), yr[k], acc);
        acc = warp_sum(acc);
        if (lane == 0) atomicAdd(dst + (int64_t)c * dst_ne0 + row, acc);
    }
}

// PowerInfer-style per-token sparse axpy (cuda/kernel.cu:427-502): token c
// adds W[gpu_row][:] * y[c][row] into dst[c][:] when idx[c][row] >= 0 (the
// reference tests `< dev_sparse_threshold` here, unlike the GEMV's `<= 0`).
__global__ void pi_axpy_kernel(const __half *__restrict__ w, const float *__restrict__ y, float *__restrict__ dst,
                               int ncols, int nrows, int src1_rows, int ntok, const int *__restrict__ lst,
                               const float *__restrict__ idx, int rows_per_cta) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    const int r0 = blockIdx.y * rows_per_cta, r1 = min(nrows, r0 + rows_per_cta);
    if (col >= ncols) return;
    for (int c = 0; c < ntok; ++c) {
        float acc = 0.0f;
        for (int gr = r0; gr < r1; ++gr) {
            const int row = lst ? lst[gr] : gr;
            if (idx[(int64_t)c * src1_rows + row] < dev_sparse_threshold) continue;
            acc = fmaf(__half2float(w[(int64_t)gr * ncols + col]), y[(int64_t)c * src1_rows + row], acc);
        }
        if (acc != 0.0f) atomicAdd(dst + (int64_t)c * ncols + col, acc);
    }
}

// add_f16_f32_f16_sparse (cuda/kernel.cu:818-830).
__global__ void add_sparse_kernel(const float *__restrict__ a, const __half *__restrict__ b, float *__restrict__ c,
                                  int M, int N, const int *__restrict__ act, const int *__restrict__ merge_idx) {
    const int row = blockIdx.y * blockDim.y + threadIdx.y;
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= N) return;
    const int g = col / SPARSITY_GROUP_SIZE;
    const int actM = g > 0 ? act[g] - act[g - 1] : act[g];
    if (row >= actM) return;
    c[(int64_t)col * M + row] = a[(int64_t)col * M + row] + __half2float(b[merge_idx[(int64_t)g * M + row]]);
}

// naive_mm_up_kernel semantics (cuda/kernel.cu:1079-1095), fp32 input not
// rounded; one warp per (compacted row, token).
__global__ void naive_up_kernel(const __half *__restrict__ a, const float *__restrict__ b, float *__restrict__ c,
                                int M, int N, int K, const int *__restrict__ act, const int *__restrict__ merge_idx) {
    const int row = blockIdx.y * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int col = blockIdx.x;
    const int lane = threadIdx.x & 31;
    const int g = col / SPARSITY_GROUP_SIZE;
    const int actM = g > 0 ? act[g] - act[g - 1] : act[g];
    if (row >= actM || col >= N) return;
    const __half *ar = a + (int64_t)merge_idx[(int64_t)g * M + row] * K;
    const float *br = b + (int64_t)col * K;
    float acc = 0.0f;
    for (int k = lane; k < K; k += 32) acc = fmaf(__half2float(ar[k]), br[k], acc);
    acc = warp_sum(acc);
    if (lane == 0) c[row + (int64_t)col * M] = acc;
}

// naive_mm_down_kernel semantics (cuda/kernel.cu:1097-1113).
__global__ void naive_down_kernel(const __half *__restrict__ a, const float *__restrict__ b, float *__restrict__ c,
                                  int M, int N, int K, const int *__restrict__ act,
                                  const int *__restrict__ merge_idx) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    const int col = blockIdx.y;
    if (row >= M || col >= N) return;
    const int g = col / SPARSITY_GROUP_SIZE;
    const int actK = g > 0 ? act[g] - act[g - 1] : act[g];
    const int *mi = merge_idx + (int64_t)g * K;
    const float *br = b + (int64_t)col * K;
    float acc = 0.0f;
    for (int k = 0; k < actK; ++k) acc = fmaf(__half2float(a[row + (int64_t)mi[k] * M]), br[k], acc);
    c[row + (int64_t)col * M] = acc;
}

// Dense c[M][N] = a[M][K] . fp16(b)[N][K]^T with fp32 accumulation
// (gemm_cuda, cuda/kernel.cu:1115-1248).  32x32 output tiles on CUDA cores.
__global__ void dense_gemm_kernel(const __half *__restrict__ a, const __half *__restrict__ b, float *__restrict__ c,
                                  int M, int N, int K) {
    __shared__ float as[32][33], bs[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    const int row0 = blockIdx.y * 32, col0 = blockIdx.x * 32;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < K; k0 += 32) {
        for (int i = ty; i < 32; i += 8) {
            as[i][tx] = (row0 + i < M && k0 + tx < K) ? __half2float(a[(int64_t)(row0 + i) * K + k0 + tx]) : 0.f;
            bs[i][tx] = (col0 + i < N && k0 + tx < K) ? __half2float(b[(int64_t)(col0 + i) * K + k0 + tx]) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[q] = fmaf(as[ty + 8 * q][k], bs[tx][k], acc[q]);
        __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int r = row0 + ty + 8 * q, cc = col0 + tx;
        if (r < M && cc < N) c[(int64_t)r * N + cc] = acc[q];
    }
}

inline int blocks(int64_t n, int b) { return (int)((n + b - 1) / b); }

}  // namespace

void convert_fp32_to_fp16_cuda(const void *vx, half *y, const int k, cudaStream_t stream) {
    if (k <= 0) return;
    f32_to_f16_kernel<<<blocks(k, kEw), kEw, 0, stream>>>((const float *)vx, y, k);
    CUDA_CHECK(cudaGetLastError());
}

void convert_fp16_to_fp32_cuda(const void *vx, float *y, const int k, cudaStream_t stream) {
    if (k <= 0) return;
    f16_to_f32_kernel<<<blocks(k, kEw), kEw, 0, stream>>>((const __half *)vx, y, k);
    CUDA_CHECK(cudaGetLastError());
}

void convert_mul_mat_batch_f16_cuda_sparse(const void *vx, const dfloat *y, float *dst, const int ncols,
                                           const int nrows, int src1_ncols, int dst_ne0, cudaStream_t stream,
                                           int *lst, float *idx) {
    if (nrows <= 0) return;
    pi_gemv_kernel<<<blocks(nrows, 8), 256, 0, stream>>>((const __half *)vx, y, dst, ncols, nrows, src1_ncols,
                                                          dst_ne0, lst, idx);
    CUDA_CHECK(cudaGetLastError());
}

void convert_axpy_sparse_batch_f16_cuda(const void *vx, const dfloat *y, float *dst, const int ncols,
                                        const int nrows, int src1_rows, int src1_ncols, cudaStream_t stream,
                                        int *lst, float *idx) {
    if (nrows <= 0 || ncols <= 0) return;
    const int rows_per_cta = 64;
    pi_axpy_kernel<<<dim3(blocks(ncols, 256), blocks(nrows, rows_per_cta)), 256, 0, stream>>>(
        (const __half *)vx, y, dst, ncols, nrows, src1_rows, src1_ncols, lst, idx, rows_per_cta);
    CUDA_CHECK(cudaGetLastError());
}

void relu_f32_cuda(const float *x, float *dst, const int k, cudaStream_t stream) {
    if (k <= 0) return;
    relu_kernel<<<blocks(k, kEw), kEw, 0, stream>>>(x, dst, k);
    CUDA_CHECK(cudaGetLastError());
}

void mul_f32_cuda(const float *x, const float *y, float *dst, const int kx, const int ky, cudaStream_t stream) {
    if (kx <= 0) return;
    mul_kernel<<<blocks(kx, kEw), kEw, 0, stream>>>(x, y, dst, kx, ky);
    CUDA_CHECK(cudaGetLastError());
}

// get_idx_cuda (cuda/kernel.cu:877-937): groups = M / 8 (floor, as the
// reference; tokens of a partial last group are ignored, and M < 8 is a
// no-op), act_neurons_device holds cumulative counts.  Like the reference
// (cuda/kernel.cu:936) it returns with the stream synchronised, since callers
// such as MLP_BS consume merge_idx on a second stream.
void get_idx_cuda(const float *idx, int *merge_idx, int *act_neurons_device, const int M, const int N,
                  cudaStream_t stream0) {
    const int groups = M / SPARSITY_GROUP_SIZE;
    if (groups <= 0 || N <= 0) return;
    const int Bu = groups * SPARSITY_GROUP_SIZE;
    const size_t ws_bytes = spb_ffn_workspace_bytes(Bu, 64, N, SPARSITY_GROUP_SIZE);
    void *ws = scratch(0, ws_bytes);
    DROPIN_OK(spb_union(idx, Bu, N, SPARSITY_GROUP_SIZE, merge_idx, act_neurons_device, nullptr, ws, ws_bytes,
                        stream0));
    CUDA_CHECK(cudaStreamSynchronize(stream0));
}

void up_mul_mat_cuda_sparse(const half *weight, const float *input, float *dst, int *merge_idx, const int M,
                            const int N, const int K, const int *act_neurons_device, cudaStream_t stream) {
    if (N <= 0 || M <= 0) return;
    const int Bu = (N / SPARSITY_GROUP_SIZE) * SPARSITY_GROUP_SIZE;
    if (dropin_up_stream_supported(Bu, K, SPARSITY_GROUP_SIZE)) {
        DROPIN_OK(launch_dropin_up_stream(weight, nullptr, input, dst, nullptr, merge_idx, act_neurons_device, Bu, K,
                                          M, SPARSITY_GROUP_SIZE, err_word(), stream));
        return;
    }
    DROPIN_OK(launch_dropin_up(weight, nullptr, input, dst, nullptr, merge_idx, act_neurons_device, Bu, K, M,
                               SPARSITY_GROUP_SIZE, stream));
}

// One reusable event per device and host thread for ordering stream1 after
// stream0 (cudaStreamWaitEvent captures the event's state at call time, so
// re-recording it later is safe).
static cudaEvent_t ordering_event() {
    thread_local std::vector<cudaEvent_t> events;
    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    if ((int)events.size() <= dev) events.resize(dev + 1, nullptr);
    if (!events[dev]) CUDA_CHECK(cudaEventCreateWithFlags(&events[dev], cudaEventDisableTiming));
    return events[dev];
}

void gate_and_up_mul_mat_cuda_sparse(const half *gate_w, const half *up_w, const float *input, float *gate_dst,
                                     float *up_dst, int *merge_idx, const int M, const int N, const int K,
                                     const int *act_neurons_device, cudaStream_t stream0, cudaStream_t stream1) {
    if (N <= 0 || M <= 0) return;
    const int Bu = (N / SPARSITY_GROUP_SIZE) * SPARSITY_GROUP_SIZE;
    if (dropin_up_stream_supported(Bu, K, SPARSITY_GROUP_SIZE))
        DROPIN_OK(launch_dropin_up_stream(gate_w, up_w, input, gate_dst, up_dst, merge_idx, act_neurons_device, Bu,
                                          K, M, SPARSITY_GROUP_SIZE, err_word(), stream0));
    else
        DROPIN_OK(launch_dropin_up(gate_w, up_w, input, gate_dst, up_dst, merge_idx, act_neurons_device, Bu, K, M,
                                   SPARSITY_GROUP_SIZE, stream0));
    if (stream1 != stream0) {
        // The reference computes up on stream1; order stream1 after the fused
        // launch so work queued there sees up_dst.
        cudaEvent_t ev = ordering_event();
        CUDA_CHECK(cudaEventRecord(ev, stream0));
        CUDA_CHECK(cudaStreamWaitEvent(stream1, ev, 0));
    }
}

void relu_and_mul_cuda(const float *gate, const float *up, float *dst, const int M, const int N,
                       cudaStream_t stream) {
    const int64_t n = (int64_t)M * N;
    if (n <= 0) return;
    relu_mul_kernel<<<blocks(n, kEw), kEw, 0, stream>>>(gate, up, dst, n, 0);
    CUDA_CHECK(cudaGetLastError());
}

void relu_relu_mul_cuda(const float *gate, const float *up, float *dst, const int M, const int N,
                        cudaStream_t stream) {
    const int64_t n = (int64_t)M * N;
    if (n <= 0) return;
    relu_mul_kernel<<<blocks(n, kEw), kEw, 0, stream>>>(gate, up, dst, n, 1);
    CUDA_CHECK(cudaGetLastError());
}

void down_mul_mat_cuda_sparse(const half *weight, const float *input, float *dst, int *merge_idx, const int M,
                              const int N, const int K, const int *act_neurons_device, cudaStream_t stream) {
    if (N <= 0 || M <= 0) return;
    DROPIN_OK(launch_dropin_down(weight, input, dst, merge_idx, act_neurons_device,
                                 (N / SPARSITY_GROUP_SIZE) * SPARSITY_GROUP_SIZE, M, K, SPARSITY_GROUP_SIZE, stream));
}

void add_sparse_cuda(const float *a, const half *b, float *c, const int M, const int N, const int *act_neurons_device,
                     const int *merge_idx, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return;
    add_sparse_kernel<<<dim3(blocks(N, SPARSITY_GROUP_SIZE), blocks(M, GGML_CUDA_DMMV_X)),
                        dim3(SPARSITY_GROUP_SIZE, GGML_CUDA_DMMV_X), 0, stream>>>(a, b, c, M, N, act_neurons_device,
                                                                                  merge_idx);
    CUDA_CHECK(cudaGetLastError());
}

void gemm_cuda(const half *a, const float *b, float *c, const int M, const int N, const int K, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return;
    __half *bh = (__half *)scratch(1, sizeof(__half) * (size_t)N * K);
    convert_fp32_to_fp16_cuda(b, bh, N * K, stream);
    dense_gemm_kernel<<<dim3(blocks(N, 32), blocks(M, 32)), 256, 0, stream>>>(a, bh, c, M, N, K);
    CUDA_CHECK(cudaGetLastError());
}

void naive_mm_up_cuda(const half *a, const float *b, float *c, const int M, const int N, const int K,
                      const int *act_neurons_device, int *merge_idx, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return;
    naive_up_kernel<<<dim3(N, blocks(M, 8)), 256, 0, stream>>>(a, b, c, M, N, K, act_neurons_device, merge_idx);
    CUDA_CHECK(cudaGetLastError());
}

void naive_mm_down_cuda(const half *a, const float *b, float *c, const int M, const int N, const int K,
                        const int *act_neurons_device, int *merge_idx, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return;
    naive_down_kernel<<<dim3(blocks(M, 128), N), 128, 0, stream>>>(a, b, c, M, N, K, act_neurons_device, merge_idx);
    CUDA_CHECK(cudaGetLastError());
}

// Host union (cuda/kernel.cu:1280-1297): per-group counts (not cumulative).
void naive_sparsity_div(const float *idx, int *merge_idx, int *act_neurons, int M, int N) {
    const int groups = M / SPARSITY_GROUP_SIZE;
    for (int g = 0; g < groups; ++g) {
        int n = 0;
        for (int j = 0; j < N; ++j) {
            bool any = false;
            for (int t = 0; t < SPARSITY_GROUP_SIZE && !any; ++t)
                any = idx[(int64_t)(g * SPARSITY_GROUP_SIZE + t) * N + j] > 0.0f;
            if (any) merge_idx[(int64_t)g * N + n++] = j;
        }
        act_neurons[g] = n;
    }
}
