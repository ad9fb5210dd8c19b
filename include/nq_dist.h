/* nq_dist.h -- multi-GPU sharding of the quantized-matmul path (libnq_dist.so).
 *
 * One process per GPU; collectives are NCCL's over NVLink / NVSwitch.  The
 * reference runs on a single device (MLX on one Apple GPU) and has no
 * multi-device code, so these entry points have no counterpart in it: they
 * shard the calls that replace mlx_ops::lin
 * (compute/src/compute/model/mlx_ops.h:28-42) and the MoE switch step
 * (compute/src/compute/model/qwen3_transformer_moe_model_mlx.cpp:29-79).
 *
 *   tensor parallel (linear layers): rank r holds rows [r*N/P, (r+1)*N/P) of
 *     the packed weight, its scales and biases (row slices of the MLX layout,
 *     no repacking), computes those output columns and all-gathers them, so
 *     every rank ends with the whole y [M, N];
 *   expert parallel (MoE): rank r holds experts [r*E/P, (r+1)*E/P) and tokens
 *     [r*T/P, (r+1)*T/P); tokens and their routing are all-gathered
 *     (dispatch), every rank runs the switch step for its own experts over
 *     all tokens, and the fp32 partial outputs are reduce-scattered back to
 *     the tokens' owners (combine).
 *
 * Status codes, stream semantics and pointer rules are those of nq.h; all
 * tensors are device pointers on the communicator's device.
 */
#ifndef NQ_DIST_H_
#define NQ_DIST_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NQ_COMM_ID_BYTES 128

typedef struct nq_comm_s *nq_comm_t;

/* Message of the last failed call of this library on the calling thread
 * (a failure inside libnq carries libnq's message). */
const char *nq_dist_last_error(void);

/* A fresh communicator id, made on one rank and handed to every rank by the
 * caller's own means (a store, MPI, torch.distributed). */
int nq_comm_unique_id(unsigned char id[NQ_COMM_ID_BYTES]);

/* Joins the communicator of `nranks` processes as `rank`, on the current
 * CUDA device.  Blocks until every rank has joined. */
int nq_comm_init(nq_comm_t *comm, int nranks, int rank,
                 const unsigned char id[NQ_COMM_ID_BYTES]);
int nq_comm_destroy(nq_comm_t comm);
/* Ends the communicator without waiting for outstanding collectives (after a
 * peer failed). */
int nq_comm_abort(nq_comm_t comm);
int nq_comm_rank(nq_comm_t comm);
int nq_comm_size(nq_comm_t comm);

/* Failure detection.  nq_comm_wait waits until the work enqueued on `stream`
 * so far has completed, polling the stream, NCCL's asynchronous error state
 * (ncclCommGetAsyncError) and a host deadline of timeout_ms milliseconds
 * (> 0).  A NCCL error, or the deadline passing first (a rank that left or
 * stopped making calls), aborts the NCCL communicator (ncclCommAbort, which
 * ends its collectives still waiting), waits a bounded time for the stream
 * to drain and returns NQ_COMPUTE_ERROR; every later call on the
 * communicator then fails at once, and nq_comm_destroy only releases it.
 * The fused calls' own waits on peer flags are bounded on the device (2 s,
 * bit 0 of the error word).
 * nq_comm_set_timeout(comm, ms) with ms > 0 makes every sharded call end with
 * nq_comm_wait(comm, stream, ms) (synchronous calls with a bounded wait);
 * 0, the default, leaves the calls asynchronous. */
int nq_comm_wait(nq_comm_t comm, void *stream, int64_t timeout_ms);
int nq_comm_set_timeout(nq_comm_t comm, int64_t timeout_ms);

/* Allocates this rank's share of a symmetric arena of `bytes` (collective:
 * every rank calls with the same size) and maps every other rank's share into
 * this process (CUDA IPC).  Outputs of nq_tp_quantized_matmul_fused live
 * there; nq_comm_symmetric_ptr(comm, offset) is this rank's address of a byte
 * offset (the same offset names the same buffer on every rank). */
int nq_comm_symmetric_alloc(nq_comm_t comm, size_t bytes);
void *nq_comm_symmetric_ptr(nq_comm_t comm, size_t offset);
/* Reads and clears the error word of the fused calls (bit 0: a wait for a
 * peer timed out). */
int nq_comm_take_error(nq_comm_t comm, unsigned int *value);

/* ---- plans (host only; no GPU needed) ---- */

/* Weight rows of rank `rank` of `nranks`: N must be a multiple of nranks. */
int nq_tp_shard(int64_t N, int nranks, int rank, int64_t *row0, int64_t *rows);
/* Experts of rank `rank`: E must be a multiple of nranks. */
int nq_ep_shard(int64_t E, int nranks, int rank, int64_t *e0, int64_t *ne);
/* Tokens of rank `rank`: T must be a multiple of nranks. */
int nq_ep_token_shard(int64_t T, int nranks, int rank, int64_t *t0, int64_t *nt);

/* Workspace bytes of nq_tp_quantized_matmul (0 when M == 1). */
size_t nq_tp_workspace_size(int64_t M, int64_t N, int nranks);
/* Workspace bytes of nq_ep_moe_switch for T tokens in total. */
size_t nq_ep_workspace_size(int64_t T, int64_t E, int64_t top_k, int64_t H,
                            int64_t I, int nranks);
/* Bytes of the symmetric arena that nq_ep_moe_switch_fused uses (its
 * receive and return buffers), and of its local workspace.  0 when T or E is
 * not a multiple of nranks. */
size_t nq_ep_fused_arena_size(int64_t T, int64_t top_k, int64_t H, int nranks);
size_t nq_ep_fused_workspace_size(int64_t T, int64_t E, int64_t top_k, int64_t H,
                                  int64_t I, int nranks);

/* ---- sharded calls (every rank calls, same shapes, same order) ---- */

/* y[M, N] = x[M, K] . W^T with W split by rows over the ranks: w_shard,
 * s_shard and b_shard are this rank's rows (nq_tp_shard).  x is the same on
 * every rank; y [M, N] bf16 receives the whole result on every rank. */
int nq_tp_quantized_matmul(nq_comm_t comm, const uint16_t *x, int64_t M,
                           const uint32_t *w_shard, const uint16_t *s_shard,
                           const uint16_t *b_shard, int64_t N, int64_t K,
                           int bits, int group_size, uint16_t *y,
                           void *workspace, size_t workspace_bytes,
                           void *stream);

/* nq_tp_quantized_matmul with the all-gather fused into the compute: the
 * kernel writes this rank's columns straight into every rank's y over
 * NVLink (peer stores), behind a ready barrier (every rank has finished the
 * stream work before the call) and followed by a done barrier (every rank's
 * columns have landed).  y must be a buffer of the symmetric arena, at the
 * same offset on every rank.  No workspace and no collective library call. */
int nq_tp_quantized_matmul_fused(nq_comm_t comm, const uint16_t *x, int64_t M,
                                 const uint32_t *w_shard, const uint16_t *s_shard,
                                 const uint16_t *b_shard, int64_t N, int64_t K,
                                 int bits, int group_size, uint16_t *y,
                                 void *stream);

/* The MoE switch step over T tokens in total, experts and tokens sharded
 * (nq_ep_shard, nq_ep_token_shard).  x_shard [T/P, H], topk_idx_shard and
 * topk_scores_shard [T/P, top_k] are this rank's tokens and their routing
 * (global expert ids, from nq_moe_route); gate/up/down hold this rank's
 * experts (w [E/P, ...] as in nq_moe_switch); y_shard [T/P, H] bf16 receives
 * the outputs of this rank's tokens. */
int nq_ep_moe_switch(nq_comm_t comm, const uint16_t *x_shard, int64_t T,
                     int64_t H, int64_t I, int64_t E, int64_t top_k,
                     const int32_t *topk_idx_shard,
                     const float *topk_scores_shard, const uint32_t *gate_w,
                     const uint16_t *gate_s, const uint16_t *gate_b,
                     const uint32_t *up_w, const uint16_t *up_s,
                     const uint16_t *up_b, const uint32_t *down_w,
                     const uint16_t *down_s, const uint16_t *down_b, int bits,
                     int group_size, void *workspace, size_t workspace_bytes,
                     uint16_t *y_shard, void *stream);

/* nq_ep_moe_switch with the token exchange as an all-to-all over NVLink
 * instead of an all-gather and a reduce-scatter, and no collective library
 * call: each token row goes once to every rank that holds one of its
 * experts (peer stores into that rank's receive buffer), each rank runs its
 * experts over the rows it received and writes the fp32 partial sums
 * straight back into the owners' return buffers, and each owner sums them
 * in rank order and rounds to bf16.  Three bounded barriers on flags in the
 * arena (ready, dispatched, combined; a timeout sets bit 0 of the error word
 * and skips the remaining stores).  Same arguments and result as
 * nq_ep_moe_switch, plus: the arena region at arena_offset (256-byte
 * aligned, nq_ep_fused_arena_size bytes, the same offset on every rank) and
 * a local workspace of nq_ep_fused_workspace_size bytes (256-byte aligned).
 * Requires H % 8 == 0 and 16-byte aligned x, y and weights; every check runs
 * before anything is enqueued. */
int nq_ep_moe_switch_fused(nq_comm_t comm, const uint16_t *x_shard, int64_t T,
                           int64_t H, int64_t I, int64_t E, int64_t top_k,
                           const int32_t *topk_idx_shard,
                           const float *topk_scores_shard,
                           const uint32_t *gate_w, const uint16_t *gate_s,
                           const uint16_t *gate_b, const uint32_t *up_w,
                           const uint16_t *up_s, const uint16_t *up_b,
                           const uint32_t *down_w, const uint16_t *down_s,
                           const uint16_t *down_b, int bits, int group_size,
                           size_t arena_offset, void *workspace,
                           size_t workspace_bytes, uint16_t *y_shard,
                           void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NQ_DIST_H_ */
