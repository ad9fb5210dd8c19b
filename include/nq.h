/*
 * nq.h -- C ABI of the B200 quantized-matmul library (libnq.so).
 *
 * The entry points replace the quantized-linear calls that neurons' models
 * make into MLX (MLXBackend serves them today):
 *   nq_quantized_matmul  <- mx::quantized_matmul(x, w, scales, biases,
 *                           transpose=true, gs, bits, "affine")
 *                           compute/src/compute/model/mlx_ops.h:28-42 (lin)
 *   nq_dequantize        <- mx::dequantize(w, scales, biases, gs, bits)
 *                           compute/src/compute/model/llama_model.cpp:67,
 *                           gemma_model_mlx.cpp:82, qwen3_moe_model_mlx.cpp:411,
 *                           qwen3_transformer_moe_model_mlx.cpp:183
 *   nq_gather_qmm        <- mx::gather_qmm(x, w, scales, biases, lhs=nullopt,
 *                           rhs=topk_idx, transpose=true, gs, bits)
 *                           qwen3_transformer_moe_model_mlx.cpp:69-74,
 *                           qwen3_moe_model_mlx.cpp:356-364
 *   nq_moe_route         <- router of the switch step (softmax fp32, top-k,
 *                           renormalise) qwen3_transformer_moe_model_mlx.cpp:36-48
 *   nq_moe_switch        <- the whole switch-MLP step for T tokens
 *                           (gate/up gather_qmm, SwiGLU, down gather_qmm,
 *                           score-weighted sum) qwen3_transformer_moe_model_mlx.cpp:29-79;
 *                           batched over tokens instead of the token loop at
 *                           qwen3_transformer_moe_model_mlx.cpp:479-486
 *   nq_quantize          <- mx::quantize(w, gs, bits) (MLX affine; the
 *                           reference loads pre-quantized checkpoints and has
 *                           no call site of its own)
 *   nq_bits_from_shapes  <- mlx_ops::bits  compute/src/compute/model/mlx_ops.h:20-25
 *
 * Conventions
 *   - Every tensor pointer is a DEVICE pointer (cudaMalloc'd or equivalent),
 *     row-major and contiguous.  bf16 tensors are passed as uint16_t bit
 *     patterns.  Packed weights are uint32 words holding 32/bits codes, the
 *     lowest-index code in the lowest bits (MLX layout).
 *   - Weight shapes follow MLX's transpose=true layout: w [N, K*bits/32],
 *     scales and biases [N, K/group_size]; stacked experts prepend [E].
 *   - bits is 4 or 8; group_size is 32, 64 or 128; K % group_size == 0.
 *   - stream is a cudaStream_t (NULL = the legacy default stream).  Every call
 *     is asynchronous on that stream and allocates nothing.
 *   - Return value: an nq_status.  The message of the last failure on the
 *     calling thread is available from nq_last_error().
 */
#ifndef NQ_H_
#define NQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors compute::ErrorCode (compute/src/compute/core/compute_types.h:9-16). */
typedef enum nq_status {
    NQ_SUCCESS = 0,
    NQ_INVALID_INPUT = 1,
    NQ_INVALID_MODEL = 2,
    NQ_BACKEND_NOT_AVAILABLE = 3,
    NQ_COMPUTE_ERROR = 4,
    NQ_UNKNOWN_ERROR = 5
} nq_status;

/* Quantization schemes for nq_quantize. */
#define NQ_SCHEME_MLX_AFFINE 0 /* MLX affine quantizer (edge snapping) */
#define NQ_SCHEME_MINMAX 1     /* scale=(max-min)/(2^bits-1), bias=min */

/* Input dtypes for nq_quantize. */
#define NQ_DTYPE_F32 0
#define NQ_DTYPE_BF16 1
#define NQ_DTYPE_F16 2

/* Library identity / diagnostics (no reference counterpart: FFI plumbing). */
int nq_version(void);
const char *nq_last_error(void);
/* Number of CUDA devices usable by the library (0 when none); never fails. */
int nq_device_count(void);
/* Reads and clears the device-side error word of the current device (set by a
 * kernel whose bounded wait ran out, or by an out-of-range gather index).
 * 0 = no error. */
int nq_take_device_error(unsigned int *err_out);

/* mlx_ops::bits: round(32 * (w_cols / s_cols) / group_size), 4 if not positive. */
int nq_bits_from_shapes(int64_t w_cols, int64_t s_cols, int group_size);

/* mx::quantize.  w: [rows, K] fp32, bf16 or fp16 (w_dtype).  Outputs: wq
 * [rows, K*bits/32] uint32, scales/biases [rows, K/group_size] bf16 (fp16 for
 * fp16 weights: MLX keeps the weights' dtype). */
int nq_quantize(const void *w, int w_dtype, int64_t rows, int64_t K, int bits,
                int group_size, int scheme, uint32_t *wq, uint16_t *scales,
                uint16_t *biases, void *stream);

/* mx::dequantize.  out: [rows, K] bf16, bit-exact bf16(bf16(s*q) + b). */
int nq_dequantize(const uint32_t *wq, const uint16_t *scales,
                  const uint16_t *biases, int64_t rows, int64_t K, int bits,
                  int group_size, uint16_t *out, void *stream);

/* mx::dequantize with fp16 scales and biases (an fp16 checkpoint): out
 * [rows, K] fp16, bit-exact fp16(fp16(s*q) + b). */
int nq_dequantize_f16(const uint32_t *wq, const uint16_t *scales,
                      const uint16_t *biases, int64_t rows, int64_t K, int bits,
                      int group_size, uint16_t *out, void *stream);

/* mx::quantized_matmul with fp16 x, scales, biases and y (what mlx_ops::lin,
 * compute/src/compute/model/mlx_ops.h:33-39, runs for an fp16 checkpoint):
 * fp32 accumulation, fp16 out.  M <= 8 with 4-bit codes takes the decode
 * GEMV (K % 128 == 0, at most 96 KB of x); every other shape the tcgen05
 * GEMM (16-byte aligned x and packed rows). */
int nq_quantized_matmul_f16(const uint16_t *x, int64_t M, const uint32_t *wq,
                            const uint16_t *scales, const uint16_t *biases,
                            int64_t N, int64_t K, int bits, int group_size,
                            uint16_t *y, void *stream);

/* mx::quantized_matmul(x, w, scales, biases, transpose=true, gs, bits).
 * x: [M, K] bf16; y: [M, N] bf16.  fp32 accumulation.  biases must be
 * non-NULL (affine mode).  M may be 0. */
int nq_quantized_matmul(const uint16_t *x, int64_t M, const uint32_t *wq,
                        const uint16_t *scales, const uint16_t *biases,
                        int64_t N, int64_t K, int bits, int group_size,
                        uint16_t *y, void *stream);

/* Number of kernels one nq_quantized_matmul call of this shape launches on the
 * current device (no reference counterpart: profiling aid).  1 for the GEMV
 * and for most tensor-core problems; 2 when the tensor-core grid's last wave
 * is split along K (a clustered tail kernel, then the whole tiles); 0 for
 * M == 0 or N == 0; a negative status for invalid arguments. */
int nq_quantized_matmul_launches(int64_t M, int64_t N, int64_t K, int bits, int group_size);

/* mx::gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices,
 * transpose=true, gs, bits).
 *   x: [x_batch, M, K] bf16;  w: [E, N, K*bits/32];  scales/biases [E, N, K/gs]
 *   out[i] ([M, N] slice of y: [n_idx, M, N]) = x[xi] . dequant(w[rhs[i]])^T,
 *   xi = lhs[i] when lhs_indices != NULL, else i when x_batch == n_idx, else 0
 *   (x_batch == 1 broadcasts).  Index arrays are DEVICE int32 arrays; indices
 *   out of range make the affected output rows zero and raise the device error
 *   word (nq_take_device_error). */
int nq_gather_qmm(const uint16_t *x, int64_t x_batch, int64_t M,
                  const int32_t *lhs_indices, const int32_t *rhs_indices,
                  int64_t n_idx, const uint32_t *wq, const uint16_t *scales,
                  const uint16_t *biases, int64_t E, int64_t N, int64_t K,
                  int bits, int group_size, uint16_t *y, void *stream);

/* Router of the MoE switch step.  logits: [T, E] bf16 (the output of the
 * router linear).  Outputs topk_idx [T, top_k] int32 (descending probability,
 * ties -> lower expert index) and topk_scores [T, top_k] fp32 (softmax over
 * all E experts, renormalised over the selected top_k).  top_k <= 32,
 * E <= 1024. */
int nq_moe_route(const uint16_t *logits, int64_t T, int64_t E, int64_t top_k,
                 int32_t *topk_idx, float *topk_scores, void *stream);

/* Workspace bytes nq_moe_switch needs for T tokens. */
size_t nq_moe_workspace_size(int64_t T, int64_t E, int64_t top_k, int64_t H,
                             int64_t I);

/* Switch-MLP of one MoE layer for T tokens (batched over tokens):
 *   y[t] = sum_j bf16(score[t,j]) * down_e( bf16(silu(gate_e(x_t)) * up_e(x_t)) ),
 *   e = topk_idx[t, j].
 * x: [T, H] bf16; topk_idx/topk_scores as produced by nq_moe_route;
 * gate/up: w [E, I, H*bits/32], s/b [E, I, H/gs];
 * down:    w [E, H, I*bits/32], s/b [E, H, I/gs];  y: [T, H] bf16.
 * workspace: device buffer of nq_moe_workspace_size() bytes (caller-owned). */
int nq_moe_switch(const uint16_t *x, int64_t T, int64_t H, int64_t I,
                  int64_t E, int64_t top_k, const int32_t *topk_idx,
                  const float *topk_scores, const uint32_t *gate_w,
                  const uint16_t *gate_s, const uint16_t *gate_b,
                  const uint32_t *up_w, const uint16_t *up_s,
                  const uint16_t *up_b, const uint32_t *down_w,
                  const uint16_t *down_s, const uint16_t *down_b, int bits,
                  int group_size, void *workspace, size_t workspace_bytes,
                  uint16_t *y, void *stream);

/* Output fan-out of a tensor-parallel quantized matmul: the call computes
 * this rank's column shard and writes it into every rank's y through peer
 * pointers (CUDA IPC mappings), instead of leaving an all-gather to a
 * collective library.  No counterpart in the reference (one device); it is
 * the compute step of nq_tp_quantized_matmul_fused (nq_dist.h), which sets
 * these fields up and signals completion after it.  All pointers are valid in
 * this process (peer mappings for other ranks).  *epoch is the call number
 * (equal on every rank, increasing; read from device memory when the kernel
 * runs, so a captured CUDA graph stays correct when replayed); ready[q] ==
 * *epoch is set by rank q before its call (its earlier stream work has
 * completed), and the kernel waits for every ready flag (bounded, 2 s; a
 * timeout raises the device error word) before its first store.  The stores
 * are complete when the kernel is. */
#define NQ_MAX_RANKS 8
typedef struct nq_push {
    int nranks;
    int rank;
    const unsigned int *epoch;
    void *dst[NQ_MAX_RANKS];
    const unsigned int *ready;
} nq_push_t;

/* y_q[m, col0 + n] = (x . W^T)[m, n] on every rank q, y rows N_total apart
 * (W: this rank's N rows).  M <= 32 needs K % 256 == 0 (and not 8-bit with
 * group size 128); larger M takes the tensor-core path. */
int nq_quantized_matmul_push(const uint16_t *x, int64_t M, const uint32_t *wq,
                             const uint16_t *scales, const uint16_t *biases,
                             int64_t N, int64_t K, int bits, int group_size,
                             int64_t N_total, int64_t col0,
                             const nq_push_t *push, void *stream);

/* Every check nq_quantized_matmul_push makes before it launches (arguments,
 * alignment -- scales and biases included -- and whether a kernel serves the
 * shape with the fan-out), without launching anything: NQ_SUCCESS when the
 * call would be accepted, else the status and message it would fail with.
 * nq_tp_quantized_matmul_fused runs it before its ready kernel, so a rejected
 * call leaves the communicator's call count unchanged.  No counterpart in the
 * reference (part of the fused tensor-parallel plumbing). */
int nq_quantized_matmul_push_check(const uint16_t *x, int64_t M, const uint32_t *wq,
                                   const uint16_t *scales, const uint16_t *biases,
                                   int64_t N, int64_t K, int bits, int group_size,
                                   int64_t N_total, int64_t col0, const nq_push_t *push);

/* The switch step restricted to one shard of the experts, for expert
 * parallelism: the weights passed hold experts [e0, e0 + ne) of the E the
 * router chose from (gate/up w [ne, I, H*bits/32], down w [ne, H, ...]), and
 * the call writes, in fp32,
 *   y_partial[t] = sum over the slots j with e0 <= topk_idx[t,j] < e0 + ne of
 *                  bf16(score[t,j]) * down_e( bf16(silu(gate_e(x_t)) * up_e(x_t)) ).
 * Summing y_partial over all shards and rounding to bf16 gives nq_moe_switch's
 * result up to the order of the fp32 additions.  No counterpart in the
 * reference (which runs one device); it shards the switch step
 * compute/src/compute/model/qwen3_transformer_moe_model_mlx.cpp:29-79.
 * workspace: nq_moe_partial_workspace_size(T, E, ne, top_k, H, I) bytes. */
size_t nq_moe_partial_workspace_size(int64_t T, int64_t E, int64_t ne,
                                     int64_t top_k, int64_t H, int64_t I);
int nq_moe_switch_partial(const uint16_t *x, int64_t T, int64_t H, int64_t I,
                          int64_t E, int64_t top_k, const int32_t *topk_idx,
                          const float *topk_scores, int64_t e0, int64_t ne,
                          const uint32_t *gate_w, const uint16_t *gate_s,
                          const uint16_t *gate_b, const uint32_t *up_w,
                          const uint16_t *up_s, const uint16_t *up_b,
                          const uint32_t *down_w, const uint16_t *down_s,
                          const uint16_t *down_b, int bits, int group_size,
                          void *workspace, size_t workspace_bytes,
                          float *y_partial, void *stream);

/* Where nq_moe_switch_partial_push writes its fp32 partial sums: the call's
 * T tokens are nranks regions of rows_per_rank rows (T = nranks *
 * rows_per_rank); token q * rows_per_rank + i goes to row dst_row0 + i of
 * dst[q] (fp32, H per row; a peer mapping for another rank), and rows i >=
 * count[q] (device memory, read when the kernel runs) are padding and are not
 * written.  No counterpart in the reference: the combine step of the
 * expert-parallel switch (nq_ep_moe_switch_fused, nq_dist.h). */
typedef struct nq_rows_push {
    int nranks;
    int64_t rows_per_rank;
    int64_t dst_row0;
    const int32_t *count;
    float *dst[NQ_MAX_RANKS];
} nq_rows_push_t;

/* nq_moe_switch_partial with the partial sums written through `push`
 * instead of y_partial (same workspace size). */
int nq_moe_switch_partial_push(const uint16_t *x, int64_t T, int64_t H, int64_t I,
                               int64_t E, int64_t top_k, const int32_t *topk_idx,
                               const float *topk_scores, int64_t e0, int64_t ne,
                               const uint32_t *gate_w, const uint16_t *gate_s,
                               const uint16_t *gate_b, const uint32_t *up_w,
                               const uint16_t *up_s, const uint16_t *up_b,
                               const uint32_t *down_w, const uint16_t *down_s,
                               const uint16_t *down_b, int bits, int group_size,
                               void *workspace, size_t workspace_bytes,
                               const nq_rows_push_t *push, void *stream);

/* ---- Llama decode step ----
 * A Llama decode step on the GPU around the quantized matmuls, restating the
 * reference's compiled decode function
 * (compute/src/compute/model/llama_model.cpp:355-509): embedding row,
 * per layer RMSNorm -> q/k/v -> RoPE -> GQA attention over the growing KV
 * cache -> o (+ residual) -> RMSNorm -> gate/up -> SwiGLU -> down
 * (+ residual), final RMSNorm, LM head (lm_head, else the tied quantized
 * embedding) and a greedy argmax, whose token feeds the next step from
 * device memory as in mlx_generate_pipelined (:713-812).  Every call only
 * enqueues work on `stream` (no host synchronisation, no allocation): steps
 * may be captured in a CUDA graph and replayed.  Serves 4-bit codes with
 * hidden, intermediate and n_heads*head_dim multiples of 128, head_dim <= 256
 * and at most 8 query heads per KV head.  Weights are borrowed (they must
 * outlive the decoder) except q/k/v and gate/up, which are copied into
 * row-concatenated buffers at creation. */
typedef struct nq_qweight {
    const uint32_t *w;        /* packed codes [N, K*bits/32] (dense bf16 [N, K] for an
                                 unquantized embedding, with scales == NULL) */
    const uint16_t *scales;   /* bf16 [N, K/gs] */
    const uint16_t *biases;   /* bf16 [N, K/gs] */
} nq_qweight_t;

typedef struct nq_llama_config {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    int bits, group_size, max_context;
    float rms_eps, rope_theta;
} nq_llama_config_t;

typedef struct nq_llama_layer {
    const uint16_t *input_norm;  /* bf16 [hidden], 16-byte aligned */
    const uint16_t *post_norm;   /* bf16 [hidden], 16-byte aligned */
    nq_qweight_t q, k, v, o, gate, up, down;
} nq_llama_layer_t;

typedef struct nq_llama_s *nq_llama_t;

/* lm_head NULL (or lm_head->w NULL): the tied embedding is the LM head. */
int nq_llama_create(nq_llama_t *out, const nq_llama_config_t *cfg,
                    const nq_llama_layer_t *layers, const uint16_t *final_norm,
                    const nq_qweight_t *embed, const nq_qweight_t *lm_head);
int nq_llama_destroy(nq_llama_t dec);
/* Steps enqueued since the last reset (the next step's position). */
int64_t nq_llama_position(nq_llama_t dec);
/* Empties the KV cache (position 0). */
int nq_llama_reset(nq_llama_t dec, void *stream);
/* One step on token[0] (device int32; NULL: the previous step's argmax).
 * logits (fp32 [vocab], optional) and next_token (int32, optional) receive
 * the step's logits and argmax. */
int nq_llama_step(nq_llama_t dec, const int32_t *token, float *logits,
                  int32_t *next_token, void *stream);
/* n steps over the prompt tokens[0..n) (device); logits (optional) gets the
 * last position's.  Afterwards the decoder's next input is the argmax of the
 * last position (the first generated token). */
int nq_llama_prefill(nq_llama_t dec, const int32_t *tokens, int64_t n,
                     float *logits, void *stream);
/* n greedy steps, each fed the previous step's argmax (the first one token[0]
 * when token != NULL); tokens[i] (device int32 [n]) receives step i's argmax. */
int nq_llama_generate(nq_llama_t dec, const int32_t *token, int64_t n,
                      int32_t *tokens, void *stream);

/* nq_moe_switch without a workspace argument, for callers that cannot
 * allocate device memory themselves (an FFI host or a runtime that only
 * hands over the tensors it owns and exposes no allocator).  No counterpart
 * in the reference: it exists for those callers only.
 * Same arguments and result as nq_moe_switch; the scratch comes from a
 * static 4 MiB block inside the library (4,194,304 bytes; every GPU that
 * loads the library keeps that block until the process exits), so calls
 * whose nq_moe_workspace_size() exceeds it fail with NQ_INVALID_INPUT (at
 * the Qwen3-30B-A3B layer dims that allows up to ~50 tokens per call).  The
 * call allocates nothing.  The first call on a device looks up the block's
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls on a device share the one block and it keeps the last
 * call's contents (the parts that must start at zero are cleared by each
 * call): calls that overlap on the GPU -- on different streams, or from
 * different threads -- race on it, so serialise them. */
int nq_moe_switch_static(const uint16_t *x, int64_t T, int64_t H, int64_t I,
                         int64_t E, int64_t top_k, const int32_t *topk_idx,
                         const float *topk_scores, const uint32_t *gate_w,
                         const uint16_t *gate_s, const uint16_t *gate_b,
                         const uint32_t *up_w, const uint16_t *up_s,
                         const uint16_t *up_b, const uint32_t *down_w,
                         const uint16_t *down_s, const uint16_t *down_b,
                         int bits, int group_size, uint16_t *y, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NQ_H_ */
