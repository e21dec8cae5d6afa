/*
 * spb.h -- C ABI of the B200 sparse-FFN library (libspbatch_b200.so).
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no C++ or torch
 * types.  Every entry point is stream-ordered, performs no host
 * synchronisation and returns an spb_status; spb_last_error() describes the
 * last failure on the calling thread.  Scratch memory comes from a
 * caller-owned device workspace whose size spb_ffn_workspace_bytes() reports.
 * The first 4 bytes of a workspace hold a sticky device error code (0 = no
 * error): kernels whose bounded waits run out record a code there and return
 * instead of hanging the GPU; only the caller clears it.  Codes of the
 * tensor-core kernel: 1 a stage's copies never landed, 2 a stage was never
 * released, 3 accumulator hand-off, 4 the partner CTA's results never
 * arrived, 5 a cluster never published its h rows, 6 the grid barrier, 7 the
 * kernel was launched without its 2-CTA clusters (nothing was computed).
 *
 * Each entry point names the reference interface it replaces
 * (cuda/kernel.cuh / cuda/kernel.cu of SMAC-Zhang/SpBatch).  The reference's
 * own C++ signatures are kept, unchanged, in include/spbatch/kernel.cuh and
 * are implemented on top of these.
 */
#ifndef SPB_H_
#define SPB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    SPB_OK = 0,
    SPB_ERR_INVALID = 1,     /* bad shape, null pointer, unsupported combination */
    SPB_ERR_WORKSPACE = 2,   /* workspace missing or too small */
    SPB_ERR_CUDA = 3,        /* a CUDA runtime call failed */
    SPB_ERR_UNSUPPORTED = 4, /* valid request this build cannot serve */
} spb_status;

/* Weight storage formats. */
typedef enum {
    SPB_W_F16 = 0,  /* fp16 rows of d values */
    SPB_W_Q8_0 = 1, /* ggml Q8_0, split row layout (d int8 quants, then d/32 fp16 scales) */
    SPB_W_Q4_0 = 2, /* ggml Q4_0, split row layout (d/2 nibble bytes, then d/32 fp16 scales) */
} spb_wtype;

/* Activation epilogues (cuda/kernel.cu:522-538). */
typedef enum {
    SPB_ACT_RELU_MUL = 0,      /* h = max(g,0) * u           (relu_and_mul_f32)  */
    SPB_ACT_RELU_RELU_MUL = 1, /* h = max(g,0) * max(u,0)    (relu_relu_mul_f32) */
} spb_act;

/* Kernel path selection for spb_ffn_forward. */
typedef enum {
    SPB_PATH_AUTO = 0,   /* choose by batch size */
    SPB_PATH_GEMV = 1,   /* CUDA-core gather GEMV (warp per neuron row) */
    SPB_PATH_TENSOR = 2, /* tcgen05/TMEM gather GEMM */
} spb_path;

const char *spb_last_error(void);
int spb_version(void);

/*
 * Device workspace needed by spb_union / spb_ffn_forward for a batch of B
 * tokens, hidden size d, f neurons and union segments of `group` tokens
 * (group = 0 means one segment holding the whole batch).
 */
size_t spb_ffn_workspace_bytes(int B, int d, int f, int group);

/*
 * Union and compaction of active neurons.
 * Replaces get_idx_cuda (cuda/kernel.cuh:97, cuda/kernel.cu:877-937).
 *   idx       [B][f] fp32 labels, neuron j active for token t iff idx > 0
 *   group     tokens per segment: 8 = the reference's SPARSITY_GROUP_SIZE,
 *             0 = whole batch as one segment; S = ceil(B / group) segments
 *   merge_idx [S][f] out: ascending active neurons of each segment
 *   act_cum   [S]    out: cumulative inclusive counts (act_neurons_device)
 *   tok_bits  [B][ceil(f/32)] out (nullable): per-token activity bitmask
 * Unlike the reference it accepts any B >= 1 and any f >= 1, and does not
 * synchronise the stream.
 */
int spb_union(const float *idx, int B, int f, int group, int32_t *merge_idx, int32_t *act_cum,
              uint32_t *tok_bits, void *workspace, size_t workspace_bytes, void *stream);

/*
 * One sparse FFN layer, out = W_down^T (act(W_gate x, W_up x) * mask).
 * Replaces the MLP_BS composition (cuda/ffn_test.cu:129-142) of
 * get_idx_cuda + gate_and_up_mul_mat_cuda_sparse + relu_and_mul_cuda +
 * down_mul_mat_cuda_sparse (cuda/kernel.cu:877-1048) with a fused path.
 *   w_gate, w_up [f][d], w_down stored [f][d] (the d x f matrix transposed,
 *                as cuda/kernel.cu:726 reads it); format `wtype`
 *   x    [B][d] fp32 (rounded to fp16 before the products, cuda/kernel.cu:978)
 *   idx  [B][f] fp32 labels (> 0 active)
 *   per_token_mask 1: h[t][j] = 0 unless neuron j is active for token t
 *                     (the masked-dense FFN); 0: every neuron of the batch
 *                     union contributes for every token (reference BS
 *                     semantics with one segment)
 *   out  [B][d] fp32, overwritten
 *   merge_idx_out [f] (nullable): the batch union, ascending
 *   count_out     [1] (nullable): its size U
 * h is rounded to fp16 before the down projection (cuda/kernel.cu:1019);
 * accumulation is fp32.
 */
int spb_ffn_forward(const void *w_gate, const void *w_up, const void *w_down, int wtype, const float *x,
                    const float *idx, int B, int d, int f, int act, int per_token_mask, int path, float *out,
                    int32_t *merge_idx_out, int32_t *count_out, void *workspace, size_t workspace_bytes,
                    void *stream);

/*
 * spb_ffn_forward with the active sets as per-token bit words instead of fp32
 * labels: tok_bits [B][ceil(f/32)], bit (j % 32) of word j / 32 of row t set
 * iff neuron j is active for token t -- the layout spb_predict writes to
 * bits_out and spb_union to tok_bits.  Everything else, the results included,
 * is as for spb_ffn_forward.  The per-token sets cross PCIe / HBM as 1/32 of
 * the label bytes, and no pass over [B][f] labels precedes the layer: the
 * tensor-core path builds the union in every CTA from these words, with no
 * grid-wide step.  Replaces the label input of get_idx_cuda
 * (cuda/kernel.cuh:97, cuda/kernel.cu:877-937) for callers whose predictor
 * emits sets rather than labels (DejaVu_predictor/trainer_mlp.py:35-37 turns
 * logits into sets).
 */
int spb_ffn_forward_bits(const void *w_gate, const void *w_up, const void *w_down, int wtype, const float *x,
                         const uint32_t *tok_bits, int B, int d, int f, int act, int per_token_mask, int path,
                         float *out, int32_t *merge_idx_out, int32_t *count_out, void *workspace,
                         size_t workspace_bytes, void *stream);

/*
 * spb_ffn_forward with the linear layers' biases: bias_gate / bias_up [f]
 * fp16 (either nullable) are added, in fp32, to each active neuron's gate /
 * up product before the activation -- the sparse bias add of add_sparse_cuda
 * (cuda/kernel.cuh:128, cuda/kernel.cu:818-830, 1055-1063), fused into every
 * path's epilogue instead of a separate pass over the compacted [B][f]
 * products.  The sets come as labels (idx) or bit words (tok_bits): exactly
 * one of the two.
 */
int spb_ffn_forward_bias(const void *w_gate, const void *w_up, const void *w_down, int wtype, const float *x,
                         const float *idx, const uint32_t *tok_bits, const void *bias_gate, const void *bias_up, int B,
                         int d, int f, int act, int per_token_mask, int path, float *out, int32_t *merge_idx_out,
                         int32_t *count_out, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Block-quantised weights (BASELINE: ggml Q8_0 / Q4_0; the reference has only
 * the f16 instance of its block-dequantisation hook, cuda/kernel.cuh:69,
 * cuda/kernel.cu:337-356).  Rows use the "split" layout: all quant bytes of
 * the row, then its d/32 fp16 block scales.
 *   spb_weight_row_bytes  bytes of one stored row (d % 32 == 0), -1 if invalid
 *   spb_quantize          host-side quantisation of rows x d fp32 weights
 *   spb_dequantize_rows   device decoding with the gather kernels' own
 *                         in-register dequantisation (d % 256 == 0)
 * spb_ffn_forward accepts wtype SPB_W_Q8_0 / SPB_W_Q4_0 on the CUDA-core path.
 */
int64_t spb_weight_row_bytes(int wtype, int d);
int spb_quantize(const float *w, int rows, int d, int wtype, uint8_t *out);
int spb_dequantize_rows(const void *q, int wtype, int rows, int d, float *out, void *stream);

/*
 * Low-rank activity predictor (DejaVu MLP): the batch's active-neuron sets.
 * The reference has it only as a PyTorch model (DejaVu_predictor/main_mlp.py:
 * 137-141, Linear(d,D) -> ReLU -> Linear(D,f), no biases) with the decision
 * sigmoid(logit) >= 0.5 (trainer_mlp.py:35-37).
 *   p1 [D][d] fp16 (fc1.weight), p2 [f][D] fp16 (fc2.weight), x [B][d] fp32
 *   hidden = fp16(ReLU(p1 . fp16(x))), logit = p2 . hidden (fp32; up to 16
 *   tokens one fixed reduction order, so logits and index sets reproduce
 *   bit-for-bit; larger batches run both products as tensor-core GEMMs
 *   (cuBLASLt, fp32 accumulation), whose logits agree to fp32 rounding and
 *   whose sets are the exact top-k of those logits)
 *   k > 0: the k largest logits per token are active (ties -> lower id);
 *   k = 0: logit >= threshold is active (threshold 0 = sigmoid >= 0.5)
 *   labels_out [B][f] fp32 (nullable): 1 active / 0 inactive -- the label format
 *              spb_union / spb_ffn_forward consume
 *   bits_out   [B][ceil(f/32)] (nullable): the same sets as bit words, the
 *              input of spb_ffn_forward_bits; labels_out or bits_out needed
 *   idx_out    [B][k > 0 ? k : f] (nullable): ascending active ids per token
 *   count_out  [B] (nullable), logits_out [B][f] (nullable)
 * d and D must be multiples of 256; workspace: spb_predict_workspace_bytes.
 * One token with k > 0 and no idx_out is one cooperative launch of one CTA
 * per SM (P2 slices resident in shared memory, the exact top-k in the same
 * launch).  Its two grid barriers count on a counter the library keeps in
 * each device's memory.  Full-device cooperative launches do not overlap, so
 * calls on several streams of one device are serialised by the GPU.  If a
 * barrier wait ever ran out (2 s), count_out[0] is -1.
 */
size_t spb_predict_workspace_bytes(int B, int D, int f);
int spb_predict(const void *p1, const void *p2, const float *x, int B, int d, int D, int f, int k, float threshold,
                float *labels_out, uint32_t *bits_out, int32_t *idx_out, int32_t *count_out, float *logits_out,
                void *workspace, size_t workspace_bytes, void *stream);

/*
 * Allocation-free variant of spb_union for callers that cannot allocate
 * device memory (a framework allocator owns the device, a plug-in receives
 * only its input and output buffers, or a latency-critical path must not call
 * cudaMalloc).  It has no counterpart in the reference.  Same arguments and
 * results as spb_union minus the workspace: its scratch (ceil(S*W/64)*64 + S + 1
 * 32-bit words, S = segments, W = ceil(f/32)) lives in a 65536-word (256 KB)
 * device array inside the library, held by every GPU that loads the library
 * until the process exits.  Larger requests fail with SPB_ERR_UNSUPPORTED.
 * The first call on a device looks up that array's device address, so make
 * it before capturing a stream.  All calls share the array: calls that
 * overlap on the GPU (different streams, or concurrent devices' threads
 * using the same device) race; serialise them.  Every scratch word a call
 * reads is written by that same call, so no clearing is needed between calls.
 */
int spb_union_static(const float *idx, int B, int f, int group, int32_t *merge_idx, int32_t *act_cum,
                     uint32_t *tok_bits, void *stream);

/*
 * Neuron sharding's exchange step without a library collective: a one-shot
 * all-reduce of the ranks' [B][d] fp32 partial outputs over NVLink peer
 * memory.  Replaces the NCCL all-reduce the sharded layer would otherwise
 * issue after the down projection (the reference is single-GPU: ffn_test.cu
 * pins one device; its down projection ends at cuda/kernel.cu:706-816).
 *
 * Set-up, once: each rank allocates one device region holding its sync words
 * (spb_peer_sync_bytes(), zero-filled once) and its receive slots
 * [2][world][stride] fp32, exports the region's pointer with spb_peer_export
 * into spb_peer_handle_bytes() bytes, the ranks exchange the handles on the
 * host, and each rank maps its peers' regions with spb_peer_import (CUDA IPC;
 * undo with spb_peer_close).
 *
 * spb_allreduce_peer: partial = this rank's n floats (local); recv[r] /
 * syncs[r] = rank r's receive slots / sync words as this rank's GPU addresses
 * them (its own at r == rank); out receives the rank-ordered sum, bit-identical
 * on every rank.  n and stride are multiples of 4 with n <= stride; pointers
 * 16-byte aligned.  One launch, stream ordered after the kernel that wrote
 * `partial`.  Every rank makes the same sequence of calls.  Bounded waits:
 * *err (device word) receives 1 if a peer never arrived.
 */
size_t spb_peer_handle_bytes(void);
size_t spb_peer_sync_bytes(void);
int spb_peer_export(const void *dev_ptr, void *handle_out);
int spb_peer_import(const void *handle, void **dev_ptr_out);
int spb_peer_close(void *dev_ptr);
int spb_allreduce_peer(const float *partial, float *const *recv, uint32_t *const *syncs, int world, int rank,
                       int64_t stride, float *out, int64_t n, uint32_t *err, void *stream);

/*
 * Tracing: while enabled, tensor-path launches write per-CTA phase stamps
 * (%globaltimer ns, 16 u64 slots per CTA: start, union scanned, gate/up
 * issued, gate/up MMAs done, gate/up accumulators ready, h published, first
 * down tile available, down issued, down accumulator ready, end) into
 * `device_buffer` (at least grid * 16 u64 entries).  NULL disables.
 */
int spb_trace_enable(void *device_buffer, size_t slots);

/* Kernel launches one spb_ffn_forward call makes for batch B, hidden size d,
   weight format wtype and `path` (per-token mask, no index outputs). */
int spb_ffn_launches(int B, int d, int wtype, int path);

#ifdef __cplusplus
}
#endif

#endif /* SPB_H_ */
