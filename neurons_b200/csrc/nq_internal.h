// nq_internal.h -- host-side interfaces between the C ABI (abi.cu) and the
// kernel launchers.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace nq {

struct PushDev;

// Thread-local last-error message behind nq_last_error().
void set_error(const std::string &msg);
const char *last_error();

// Device error word of the current device (a static __device__ variable;
// its address is looked up once per device).
unsigned int *device_error_word();

// Number of SMs of the current device (cached per device).
int sm_count();

// A skinny (<= 32 tokens per pass) quantized matmul problem set.
// Problem p multiplies tokens of x against expert e_p of a stacked weight
// tensor; see gemv.cu for the addressing rules.
struct GemvProblems {
    const uint32_t *w = nullptr;   // [E, N, K*bits/32]
    const uint16_t *s = nullptr;   // [E, N, K/gs]
    const uint16_t *b = nullptr;
    const uint32_t *w2 = nullptr;  // second weight set (gate/up pair), same shape
    const uint16_t *s2 = nullptr;
    const uint16_t *b2 = nullptr;
    int64_t N = 0, K = 0;
    int bits = 4, gs = 64;
    const uint16_t *x = nullptr;
    int64_t x_ld = 0;                  // elements between x rows
    int P = 1;                         // number of problems
    int M = 1;                         // tokens per problem when m_count == nullptr
    int E = 1;                         // number of experts (index range check)
    const int32_t *expert = nullptr;   // [P] expert of problem p; nullptr -> 0
    bool expert_is_p = false;          // expert of problem p is p
    const int32_t *m_count = nullptr;  // [P] tokens of problem p
    const int32_t *m_offset = nullptr; // [P] first entry of problem p in the row lists
    const int32_t *x_rows = nullptr;   // x row of (p, m); nullptr -> see x_from_offset
    bool x_from_offset = false;        // x row of (p, m) = off(p) + m (else xi(p)*M + m)
    const int32_t *lhs = nullptr;      // [P] x batch of problem p (gather_qmm lhs)
    int x_div = 0;                     // > 0 (no lhs): x batch of problem p is p / x_div
    int x_batch = 1;
    void *y = nullptr;
    int64_t y_ld = 0;                  // elements between y rows
    const int32_t *y_rows = nullptr;   // y row of (p, m); nullptr -> off(p) + m,
                                       // off(p) = m_offset[p] or p*M
    int out_f32 = 0;                   // 1: fp32 output, 0: bf16 output
    int swiglu = 0;                    // 1: y = bf16(silu(x.w^T) * (x.w2^T))
    int max_m = 1;                     // upper bound of tokens per problem
    int tile_m = 0;                    // tokens per pass to size for (0: from max_m)
    const PushDev *push = nullptr;     // tensor-parallel fan-out of the stores
};

cudaError_t launch_gemv(const GemvProblems &p, cudaStream_t stream);

// Decode-step GEMV of the row-group kernel (4-bit codes, K % 128 == 0) with a
// prologue fused into the staging of x and a residual or SwiGLU epilogue:
//   prologue 0: x as is; 1: x = bf16(norm_w * bf16(x * rsqrt(mean(x^2) + eps)))
//   (MLX rms_norm); 2: x = swiglu(g, u) for the row [g (K) | u (K)];
//   res != nullptr: y = bf16(res + bf16(x . W^T)).
// Prologues 1 and 2 need M == 1.  cudaErrorNotSupported when the kernel does
// not serve the shape.
struct RowsFusedArgs {
    const uint16_t *x = nullptr;
    int64_t x_ld = 0;
    int M = 1;
    const uint32_t *w = nullptr;
    const uint16_t *s = nullptr, *b = nullptr;
    int64_t N = 0, K = 0;
    int bits = 4, gs = 64;
    uint16_t *y = nullptr;
    int64_t y_ld = 0;
    int prologue = 0;
    const uint16_t *norm_w = nullptr;
    float eps = 0.f;
    const uint16_t *res = nullptr;
    int64_t res_ld = 0;
    // 1 (M == 1, N % 16 == 0): the weight rows come in groups of 8 gate rows
    // followed by the 8 matching up rows, and y gets the N / 2 values
    // bf16(bf16(bf16(sigmoid(g)) * g) * u) of g, u rounded to bf16
    int epi_swiglu = 0;
};
cudaError_t launch_rows_fused(const RowsFusedArgs &a, cudaStream_t stream);
// fp16 x, scales, biases and y (an fp16 checkpoint), M <= 8, 4-bit codes:
// the row-group kernel; cudaErrorNotSupported when it does not serve the shape.
cudaError_t launch_rows_f16(const uint16_t *x, int M, const uint32_t *w, const uint16_t *s,
                            const uint16_t *b, int64_t N, int64_t K, int bits, int gs, uint16_t *y,
                            cudaStream_t stream);
// Whether launch_rows_fused serves an N x K weight at M == 1 (host only).
bool rows_fused_supported(int64_t N, int64_t K, int bits);

// Why launch_gemv cannot serve p with an output fan-out (p.push), or nullptr
// when its arguments allow it (the fan-out also needs tensor maps from the
// driver: tensor_maps_available()).  Host-side only: no device work.
const char *gemv_push_unsupported(const GemvProblems &p);

// Dense path for larger M: TMA + tcgen05 GEMM with in-TMEM dequant.
struct TcGemmArgs {
    const uint16_t *x = nullptr;   // [M, K] bf16 (row stride x_ld)
    int64_t x_ld = 0;
    int64_t M = 0;
    const uint32_t *w = nullptr;   // [N, K*bits/32]
    const uint16_t *s = nullptr;
    const uint16_t *b = nullptr;
    int64_t N = 0, K = 0;
    int bits = 4, gs = 64;
    uint16_t *y = nullptr;         // [M, N] bf16 (row stride y_ld)
    int64_t y_ld = 0;
    const PushDev *push = nullptr; // tensor-parallel fan-out of the stores
    bool f16 = false;              // x, scales, biases and y are fp16 (else bf16)
};

bool tc_gemm_supported(const TcGemmArgs &a);

// cuTensorMapEncodeTiled for a 2-D row-major tensor (resolved through
// cudaGetDriverEntryPoint; false when the driver entry point is missing or the
// encoding is rejected).
bool make_map_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle sw);
cudaError_t launch_tc_gemm(const TcGemmArgs &a, cudaStream_t stream);
// Kernel launches launch_tc_gemm makes for `a` on the current device (1, or 2
// when the wave tail is split; 0 when the problem does not suit the path).
int tc_gemm_launches(const TcGemmArgs &a);

// True when cuTensorMapEncodeTiled could be resolved from the driver.
bool tensor_maps_available();

// Where the switch step of one expert shard writes its fp32 partial sums when
// they go straight to the tokens' owners: the call's tokens are n regions of
// `per` rows; token q * per + i goes to row row0 + i of dst[q] (rows i >=
// count[q] are padding and are not written).  n == 0: not used.
struct MoeRowsOut {
    int n = 0;
    int64_t per = 0, row0 = 0;
    const int32_t *count = nullptr;  // [n], device memory
    float *dst[8] = {};
};

// Expert-grouped tcgen05 GEMMs of the MoE switch step (gemm_tc_moe.cu).
// A tile is {expert, first grouped row, token count <= kMoeTileTokens, 0}.
constexpr int kMoeTileTokens = 256;
struct TcMoeArgs {
    bool up = true;                  // true: gate/up + SwiGLU -> h; false: down -> d (fp32)
    int bits = 4, gs = 64;
    int64_t E = 0, N = 0, K = 0;     // experts, weight rows per expert, reduction length
    const uint32_t *w1 = nullptr;    // [E, N, K*bits/32] (gate, or down)
    const uint16_t *s1 = nullptr, *b1 = nullptr;
    const uint32_t *w2 = nullptr;    // up (up kernel)
    const uint16_t *s2 = nullptr, *b2 = nullptr;
    const uint16_t *x = nullptr;     // token rows in grouped order: up: xg [P, K]; down: h [P, K]
    int64_t x_ld = 0;
    int64_t x_rows_total = 0;        // P
    const int32_t *rows = nullptr;   // down: pair of grouped row
    const int4 *tiles = nullptr;
    const int32_t *n_tiles = nullptr;
    int64_t max_tiles = 0;           // grid bound; CTAs past *n_tiles exit at once
    void *y = nullptr;               // up: h [P, N] bf16; down: d [P, N] fp32 (rows by pair)
    int64_t y_ld = 0;
    // down: fused score-weighted combine when fuse_cnt != nullptr ([T, ceil(N/128)]
    // arrival counters, zero at the start of the call); the tokens' sums go to
    // out [T, N] bf16, or through ro (ro.n > 0)
    int32_t *fuse_cnt = nullptr;
    const int32_t *idx = nullptr;
    const float *scores = nullptr;
    int top_k = 0, e0 = 0;
    uint16_t *out = nullptr;
    MoeRowsOut ro;
};
bool tc_moe_supported(int bits, int gs, int64_t H, int64_t I, int64_t E, const void *x,
                      int64_t x_ld);
cudaError_t launch_tc_moe(const TcMoeArgs &a, cudaStream_t stream);

cudaError_t launch_quantize(const void *w, int w_dtype, int64_t rows, int64_t K, int bits,
                            int gs, int scheme, uint32_t *wq, uint16_t *s, uint16_t *b,
                            cudaStream_t stream);
// f16: scales, biases and the output are fp16 (else bf16)
cudaError_t launch_dequantize(const uint32_t *wq, const uint16_t *s, const uint16_t *b,
                              int64_t rows, int64_t K, int bits, int gs, uint16_t *out,
                              cudaStream_t stream, bool f16 = false);

size_t moe_workspace_bytes(int64_t T, int64_t E, int64_t top_k, int64_t H, int64_t I);
size_t moe_partial_workspace_bytes(int64_t T, int64_t E, int64_t ne, int64_t top_k, int64_t H,
                                   int64_t I);
// The switch step for experts [e0, e0 + ne) of E_total (weights: those ne
// experts).  y: bf16 result (all experts); y_partial: fp32 partial sums;
// rows_out (non-null, n > 0): fp32 partial sums into other ranks' buffers.
cudaError_t launch_moe_switch(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E_total,
                              int64_t top_k, const int32_t *idx, const float *scores, int64_t e0,
                              int64_t ne, const uint32_t *gw, const uint16_t *gs_,
                              const uint16_t *gb, const uint32_t *uw, const uint16_t *us,
                              const uint16_t *ub, const uint32_t *dw, const uint16_t *ds,
                              const uint16_t *db, int bits, int gsz, void *workspace, uint16_t *y,
                              float *y_partial, cudaStream_t stream,
                              const MoeRowsOut *rows_out = nullptr);

// The switch step for a few tokens (every pair its own problem, T * top_k <=
// E, all experts on this device, 4-bit codes) in two kernels, the down one
// forming the score-weighted sum itself (moe_small.cu).  h: [T * top_k, I].
bool moe_small_supported(int64_t T, int64_t H, int64_t I, int64_t E, int64_t top_k, int bits,
                         const void *x);
cudaError_t launch_moe_small(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E,
                             int64_t top_k, const int32_t *idx, const float *scores,
                             const uint32_t *gw, const uint16_t *gs, const uint16_t *gb,
                             const uint32_t *uw, const uint16_t *us, const uint16_t *ub,
                             const uint32_t *dw, const uint16_t *ds, const uint16_t *db, int gsz,
                             uint16_t *h, uint16_t *y, cudaStream_t stream);

cudaError_t launch_moe_route(const uint16_t *logits, int64_t T, int64_t E, int64_t top_k,
                             int32_t *idx, float *scores, cudaStream_t stream);

}  // namespace nq
