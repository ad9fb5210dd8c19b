/*
 * nq_oracle.c -- CPU oracle for the MLX-affine quantized-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (neurons_b200/, include/)
 * links, loads or calls this file.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference arm use it, as the checker and as the
 * timed CPU baseline -- never as the thing measured on the GPU path.
 *
 * What it restates.  The reference (neurons) performs every quantized
 * operation through MLX, a third-party library that is not vendored in the
 * reference tree: it is fetched at configure time from a fork pinned in
 * compute/CMakeLists.txt:21-31 (MLX "0.31.2", commit
 * 1109c8ce5b14801f000fef87cb9cb75b858f8ec4) and only builds on Apple arm64
 * (compute/CMakeLists.txt:18).  The reference's call sites are:
 *   - mx::quantized_matmul(x, w, scales, biases, transpose=true, gs, bits,
 *     "affine")                      compute/src/compute/model/mlx_ops.h:39
 *   - mx::dequantize(w, scales, biases, gs, bits)
 *                                    compute/src/compute/model/llama_model.cpp:67
 *   - mx::gather_qmm(x, w, scales, biases, nullopt, topk_idx, true, gs, bits)
 *                   compute/src/compute/model/qwen3_transformer_moe_model_mlx.cpp:69-74
 *   - the MoE switch step around it (router softmax -> top-k -> renormalise,
 *     SwiGLU, score-weighted sum)
 *                   compute/src/compute/model/qwen3_transformer_moe_model_mlx.cpp:29-79
 *   - the bit width inferred from shapes   compute/src/compute/model/mlx_ops.h:20-25
 * This file restates MLX's published CPU semantics for those operations in
 * plain C, in this project's own code:
 *   - affine quantize ("mlx" scheme): per group of `gs` along K, fp32 min/max,
 *     scale = max((max-min)/n_bins, 1e-7) signed towards the larger-magnitude
 *     edge, the edge snapped to an integer code (scale = edge/q0, bias = edge,
 *     or bias = 0 when q0 rounds to 0), codes = clamp(rint((w-bias)/scale),
 *     0, n_bins) computed with the fp32 scale/bias, then scale and bias stored
 *     as bf16 (round to nearest even).
 *   - the "minmax" scheme spelled out by the benchmark workload definition:
 *     scale = (max-min)/n_bins, bias = min, same code rule (scale == 0 -> 0).
 *   - packing: 32/bits codes per uint32, element j of a word in bits
 *     [bits*j, bits*(j+1)) ("lowest index in the lowest bits").
 *   - dequantize: MLX evaluates scale*q + bias in the bf16 dtype of the
 *     scales, each op computed in fp32 and rounded to bf16, i.e.
 *     w_hat = bf16(bf16(s*q) + b).  This is the bit-exact target.
 *   - quantized_matmul: y = bf16( sum_k x[m,k] * w_hat[n,k] ), accumulated
 *     here in fp64 (the contract is "fp32 accumulation, bf16 out"; the GPU is
 *     compared against this within a tolerance).
 *   - gather_qmm: out[i] = x[lhs[i] or i or 0] . w_hat[rhs[i]]^T.
 *
 * Parity status: UNPINNED against real MLX.  MLX cannot be built or imported
 * here, and the reference's only qmm fixtures
 * (compute/tests/compute/baselines/output/attention_*_baseline.*) need the
 * TinyLlama weights, which are not in the reference tree.  The restatement is
 * cross-checked against an independent numpy restatement (oracle/np_oracle.py)
 * and against hand-derived known answers (tests/golden/).
 *
 * Build: see oracle/build.py (gcc -O2 -ffp-contract=off -fopenmp, no
 * -ffast-math, so every fp32 operation is a single IEEE-754 operation).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_OK 0
#define OR_INVALID 1

/* ---------------------------------------------------------------- bf16 */

uint16_t or_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float or_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static float round_bf16(float f) { return or_bf16_to_f32(or_f32_to_bf16(f)); }

/* ---------------------------------------------------------------- fp16
 * IEEE binary16, round to nearest even (the conversion MLX and CUDA use for
 * float16 tensors); fp16 checkpoints store scales and biases this way. */

uint16_t or_f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u, a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);   /* NaN */
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  /* >= 65520: inf */
    if (a < 0x38800000u) {                                    /* below 2^-14: subnormal */
        float af;
        memcpy(&af, &a, 4);
        const float r = rintf(af * 16777216.0f);              /* units of 2^-24, ties to even */
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t h = ((((a >> 23) - 112u)) << 10) | ((a & 0x7fffffu) >> 13);
    const uint32_t rem = a & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

float or_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t u;
    if (e == 0) {
        float f = (float)m * (1.0f / 16777216.0f);             /* exact */
        memcpy(&u, &f, 4);
        u |= sign;
    } else if (e == 31) {
        u = sign | 0x7f800000u | (m << 13);
    } else {
        u = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static float round_f16(float f) { return or_f16_to_f32(or_f32_to_f16(f)); }

/* 16-bit storage types of activations, scales and biases */
static float half_to_f32(uint16_t v, int f16) { return f16 ? or_f16_to_f32(v) : or_bf16_to_f32(v); }
static uint16_t f32_to_half(float v, int f16) { return f16 ? or_f32_to_f16(v) : or_f32_to_bf16(v); }
static float round_half(float v, int f16) { return f16 ? round_f16(v) : round_bf16(v); }

/* mlx_ops::bits (compute/src/compute/model/mlx_ops.h:20-25):
 * bits = round(32 * (w_cols / s_cols) / gs), or 4 when that is not positive. */
int or_bits_from_shapes(int64_t w_cols, int64_t s_cols, int group_size) {
    double ratio = (double)w_cols / (double)s_cols;
    int b = (int)llround(32.0 * ratio / (double)group_size);
    return b > 0 ? b : 4;
}

static int check_quant_params(int64_t rows, int64_t K, int bits, int gs) {
    if (rows < 0 || K <= 0) return OR_INVALID;
    if (bits != 4 && bits != 8) return OR_INVALID;
    if (gs != 32 && gs != 64 && gs != 128) return OR_INVALID;
    if (K % gs) return OR_INVALID;
    return OR_OK;
}

/* ------------------------------------------------------------ quantize */

/* One group of gs values -> codes, scale, bias (fp32, before bf16 storage). */
static void quantize_group(const float *w, int gs, int bits, int scheme,
                           uint8_t *codes, float *scale_out, float *bias_out) {
    const float n_bins = (float)((1 << bits) - 1);
    float w_max = -INFINITY, w_min = INFINITY;
    for (int j = 0; j < gs; ++j) {
        w_max = fmaxf(w_max, w[j]);
        w_min = fminf(w_min, w[j]);
    }
    float scale, bias;
    if (scheme == 0) {
        /* MLX affine: edge snapping so that the larger-magnitude edge and 0
         * are exactly representable. */
        const float eps = 1e-7f;
        int mask = fabsf(w_min) > fabsf(w_max);
        scale = fmaxf((w_max - w_min) / n_bins, eps);
        scale = mask ? scale : -scale;
        float edge = mask ? w_min : w_max;
        float q0 = rintf(edge / scale);
        bias = 0.0f;
        if (q0 != 0.0f) {
            scale = edge / q0;
            bias = edge;
        }
    } else {
        scale = (w_max - w_min) / n_bins;
        bias = w_min;
    }
    for (int j = 0; j < gs; ++j) {
        float q;
        if (scale == 0.0f) {
            q = 0.0f;
        } else {
            q = rintf((w[j] - bias) / scale);
            q = fminf(fmaxf(q, 0.0f), n_bins);
        }
        codes[j] = (uint8_t)q;
    }
    *scale_out = scale;
    *bias_out = bias;
}

/* w: [rows, K] fp32 (w_dtype 0), bf16 bits (w_dtype 1) or fp16 bits
 * (w_dtype 2).  wq: [rows, K*bits/32] uint32; scales, biases: [rows, K/gs],
 * bf16 bits (fp16 bits for fp16 weights, as MLX keeps the weights' dtype). */
int or_quantize(const void *w, int w_dtype, int64_t rows, int64_t K, int bits,
                int gs, int scheme, uint32_t *wq, uint16_t *scales,
                uint16_t *biases) {
    if (check_quant_params(rows, K, bits, gs) || w_dtype < 0 || w_dtype > 2 ||
        (scheme != 0 && scheme != 1))
        return OR_INVALID;
    const int f16 = w_dtype == 2;
    const int64_t groups = K / gs;
    const int64_t words = K * bits / 32;
    const int per_word = 32 / bits;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        float buf[128];
        uint8_t codes[128];
        for (int64_t g = 0; g < groups; ++g) {
            int64_t base = r * K + g * gs;
            for (int j = 0; j < gs; ++j)
                buf[j] = w_dtype == 0 ? ((const float *)w)[base + j]
                                      : half_to_f32(((const uint16_t *)w)[base + j], f16);
            float s, b;
            quantize_group(buf, gs, bits, scheme, codes, &s, &b);
            scales[r * groups + g] = f32_to_half(s, f16);
            biases[r * groups + g] = f32_to_half(b, f16);
            for (int wi = 0; wi < gs / per_word; ++wi) {
                uint32_t word = 0;
                for (int e = 0; e < per_word; ++e)
                    word |= (uint32_t)codes[wi * per_word + e] << (bits * e);
                wq[r * words + g * (gs / per_word) + wi] = word;
            }
        }
    }
    return OR_OK;
}

/* ---------------------------------------------------------- dequantize */

/* MLX-CPU dequantize of one code in the scales' dtype T (bf16 or fp16):
 * T(T(s*q) + b), each op computed in fp32 and rounded to T. */
static inline float dq_value_dt(float s, float b, uint32_t q, int f16) {
    float p = round_half(s * (float)q, f16);
    return round_half(p + b, f16);
}

static void dequant_row_dt(const uint32_t *wq_row, const uint16_t *s_row,
                           const uint16_t *b_row, int64_t K, int bits, int gs,
                           float *out, int f16) {
    const int per_word = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t k = 0; k < K; ++k) {
        uint32_t word = wq_row[k / per_word];
        uint32_t q = (word >> (bits * (k % per_word))) & mask;
        float s = half_to_f32(s_row[k / gs], f16);
        float b = b_row ? half_to_f32(b_row[k / gs], f16) : 0.0f;
        out[k] = dq_value_dt(s, b, q, f16);
    }
}

static void dequant_row_f32(const uint32_t *wq_row, const uint16_t *s_row,
                            const uint16_t *b_row, int64_t K, int bits, int gs,
                            float *out) {
    dequant_row_dt(wq_row, s_row, b_row, K, bits, gs, out, 0);
}

static int dequantize_dt(const uint32_t *wq, const uint16_t *scales,
                         const uint16_t *biases, int64_t rows, int64_t K, int bits,
                         int gs, uint16_t *out, int f16) {
    if (check_quant_params(rows, K, bits, gs) || !biases) return OR_INVALID;
    const int64_t words = K * bits / 32, groups = K / gs;
#pragma omp parallel
    {
        float *row = (float *)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            dequant_row_dt(wq + r * words, scales + r * groups, biases + r * groups,
                           K, bits, gs, row, f16);
            for (int64_t k = 0; k < K; ++k) out[r * K + k] = f32_to_half(row[k], f16);
        }
        free(row);
    }
    return OR_OK;
}

int or_dequantize(const uint32_t *wq, const uint16_t *scales,
                  const uint16_t *biases, int64_t rows, int64_t K, int bits,
                  int gs, uint16_t *out) {
    return dequantize_dt(wq, scales, biases, rows, K, bits, gs, out, 0);
}

/* fp16 scales and biases: fp16 output. */
int or_dequantize_f16(const uint32_t *wq, const uint16_t *scales,
                      const uint16_t *biases, int64_t rows, int64_t K, int bits,
                      int gs, uint16_t *out) {
    return dequantize_dt(wq, scales, biases, rows, K, bits, gs, out, 1);
}

/* ----------------------------------------------------------------- qmm */

__attribute__((target_clones("avx2", "default")))
static double dot_f32_f64(const float *a, const float *b, int64_t n) {
    /* Products of two floats are exact in double; four partial sums keep the
     * loop vectorisable (fp64 accumulation is ~2^29 times finer than the bf16
     * output, so the summation order does not matter at that precision). */
    double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int64_t k = 0;
    for (; k + 4 <= n; k += 4) {
        s0 += (double)a[k] * (double)b[k];
        s1 += (double)a[k + 1] * (double)b[k + 1];
        s2 += (double)a[k + 2] * (double)b[k + 2];
        s3 += (double)a[k + 3] * (double)b[k + 3];
    }
    for (; k < n; ++k) s0 += (double)a[k] * (double)b[k];
    return (s0 + s1) + (s2 + s3);
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

int or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* y[M,N] = x[M,K] . w_hat[N,K]^T.  x, y bf16 bits; y32 (optional) receives the
 * unrounded sums as fp32.  nthreads <= 0 keeps the OpenMP default. */
static int qmm_dt(const uint16_t *x, int64_t M, const uint32_t *wq,
                  const uint16_t *scales, const uint16_t *biases, int64_t N, int64_t K,
                  int bits, int gs, uint16_t *y, float *y32, int nthreads, int f16) {
    if (check_quant_params(N, K, bits, gs) || M < 0 || !biases) return OR_INVALID;
    set_threads(nthreads);
    const int64_t words = K * bits / 32, groups = K / gs;
    float *xf = (float *)malloc(sizeof(float) * (size_t)(M * K + 1));
    for (int64_t i = 0; i < M * K; ++i) xf[i] = half_to_f32(x[i], f16);
#pragma omp parallel
    {
        float *row = (float *)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(dynamic, 4)
        for (int64_t n = 0; n < N; ++n) {
            dequant_row_dt(wq + n * words, scales + n * groups, biases + n * groups,
                           K, bits, gs, row, f16);
            for (int64_t m = 0; m < M; ++m) {
                double acc = dot_f32_f64(xf + m * K, row, K);
                if (y) y[m * N + n] = f32_to_half((float)acc, f16);
                if (y32) y32[m * N + n] = (float)acc;
            }
        }
        free(row);
    }
    free(xf);
    return OR_OK;
}

int or_qmm(const uint16_t *x, int64_t M, const uint32_t *wq,
           const uint16_t *scales, const uint16_t *biases, int64_t N, int64_t K,
           int bits, int gs, uint16_t *y, float *y32, int nthreads) {
    return qmm_dt(x, M, wq, scales, biases, N, K, bits, gs, y, y32, nthreads, 0);
}

/* fp16 x, scales, biases and y (an fp16 checkpoint's activations). */
int or_qmm_f16(const uint16_t *x, int64_t M, const uint32_t *wq,
               const uint16_t *scales, const uint16_t *biases, int64_t N, int64_t K,
               int bits, int gs, uint16_t *y, float *y32, int nthreads) {
    return qmm_dt(x, M, wq, scales, biases, N, K, bits, gs, y, y32, nthreads, 1);
}

/* MLX gather_qmm with transpose=true:
 *   out[i] (an [M,N] slice) = x[xi] . w_hat[rhs[i]]^T,
 *   xi = lhs[i] if lhs else (x_batch == 1 ? 0 : i).
 * x: [x_batch, M, K]; w: [E, N, K*bits/32]; scales/biases: [E, N, K/gs];
 * out: [n_idx, M, N]. */
int or_gather_qmm(const uint16_t *x, int64_t x_batch, int64_t M,
                  const int32_t *lhs, const int32_t *rhs, int64_t n_idx,
                  const uint32_t *wq, const uint16_t *scales,
                  const uint16_t *biases, int64_t E, int64_t N, int64_t K,
                  int bits, int gs, uint16_t *out, float *out32, int nthreads) {
    if (check_quant_params(N, K, bits, gs) || M < 0 || E <= 0 || !biases || !rhs)
        return OR_INVALID;
    if (!lhs && x_batch != 1 && x_batch != n_idx) return OR_INVALID;
    for (int64_t i = 0; i < n_idx; ++i) {
        if (rhs[i] < 0 || rhs[i] >= E) return OR_INVALID;
        if (lhs && (lhs[i] < 0 || lhs[i] >= x_batch)) return OR_INVALID;
    }
    const int64_t words = K * bits / 32, groups = K / gs;
    for (int64_t i = 0; i < n_idx; ++i) {
        int64_t xi = lhs ? lhs[i] : (x_batch == 1 ? 0 : i);
        int64_t e = rhs[i];
        int rc = or_qmm(x + xi * M * K, M, wq + e * N * words,
                        scales + e * N * groups, biases + e * N * groups, N, K,
                        bits, gs, out ? out + i * M * N : NULL,
                        out32 ? out32 + i * M * N : NULL, nthreads);
        if (rc) return rc;
    }
    return OR_OK;
}

/* ----------------------------------------------------------------- MoE */

/* Router of the switch step (qwen3_transformer_moe_model_mlx.cpp:36-48):
 * softmax over all E experts in fp32, the top_k largest selected, their
 * probabilities renormalised to sum to 1.  Selection compares the logits
 * themselves (softmax is monotonic); equal logits prefer the lower expert
 * index.  Output order: descending probability.  logits: [T, E] bf16 bits. */
int or_moe_route(const uint16_t *logits, int64_t T, int64_t E, int64_t top_k,
                 int32_t *idx, float *scores) {
    if (T < 0 || E <= 0 || top_k <= 0 || top_k > E || top_k > 64) return OR_INVALID;
    for (int64_t t = 0; t < T; ++t) {
        const uint16_t *l = logits + t * E;
        float mx = -INFINITY;
        for (int64_t e = 0; e < E; ++e) mx = fmaxf(mx, or_bf16_to_f32(l[e]));
        float sum = 0.0f;
        for (int64_t e = 0; e < E; ++e) sum += expf(or_bf16_to_f32(l[e]) - mx);
        int32_t sel[64];
        for (int64_t j = 0; j < top_k; ++j) {
            int32_t best = -1;
            float bv = 0.0f;
            for (int64_t e = 0; e < E; ++e) {
                int taken = 0;
                for (int64_t p = 0; p < j; ++p) taken |= sel[p] == e;
                if (taken) continue;
                float v = or_bf16_to_f32(l[e]);
                if (best < 0 || v > bv) { best = (int32_t)e; bv = v; }
            }
            sel[j] = best;
        }
        float p[64], psum = 0.0f;
        for (int64_t j = 0; j < top_k; ++j) {
            p[j] = expf(or_bf16_to_f32(l[sel[j]]) - mx) / sum;
            psum += p[j];
        }
        for (int64_t j = 0; j < top_k; ++j) {
            idx[t * top_k + j] = sel[j];
            scores[t * top_k + j] = p[j] / psum;
        }
    }
    return OR_OK;
}

static float silu_f32(float g) { return g / (1.0f + expf(-g)); }

/* Switch-MLP of one MoE layer for T tokens, given the routing, in two
 * stages.  x: [T,H] bf16; idx/scores: [T,top_k]; gate/up: [E,I,H*bits/32]
 * (+ [E,I,H/gs] scales/biases); down: [E,H,I*bits/32] (+ [E,H,I/gs]).
 *
 * rounding == 0 follows MLX's op chain (qwen3_transformer_moe_model_mlx.cpp:69-78):
 *   gate_k, up_k, down_k rounded to bf16 (gather_qmm outputs),
 *   h = bf16(bf16(bf16(sigmoid(g)) * g) * u), score rounded to bf16,
 *   y = bf16(sum_k bf16(down_k * score_k)).
 * rounding == 1 states the fused GPU kernel's rounding points:
 *   gate/up sums kept in fp32, h = bf16(silu(g) * u) in fp32,
 *   down sums kept in fp32, y = bf16(sum_k bf16(score_k) * down_k). */

/* Stage 1: h[T*top_k, I] (bf16 bits) for every (token, slot) pair. */
int or_moe_hidden(const uint16_t *x, int64_t T, int64_t H, int64_t I, int64_t E,
                  int64_t top_k, const int32_t *idx, const uint32_t *wg,
                  const uint16_t *sg, const uint16_t *bg, const uint32_t *wu,
                  const uint16_t *su, const uint16_t *bu, int bits, int gs,
                  int rounding, uint16_t *h, int nthreads) {
    if (check_quant_params(I, H, bits, gs) || T < 0 || E <= 0 || top_k <= 0)
        return OR_INVALID;
    for (int64_t i = 0; i < T * top_k; ++i)
        if (idx[i] < 0 || idx[i] >= E) return OR_INVALID;
    set_threads(nthreads);
    const int64_t wgu = H * bits / 32, ggu = H / gs;
#pragma omp parallel
    {
        float *rg = (float *)malloc(sizeof(float) * (size_t)H);
        float *ru = (float *)malloc(sizeof(float) * (size_t)H);
        float *xf = (float *)malloc(sizeof(float) * (size_t)H);
#pragma omp for schedule(dynamic, 1)
        for (int64_t tk = 0; tk < T * top_k; ++tk) {
            int64_t t = tk / top_k, e = idx[tk];
            for (int64_t k = 0; k < H; ++k) xf[k] = or_bf16_to_f32(x[t * H + k]);
            for (int64_t n = 0; n < I; ++n) {
                int64_t row = e * I + n;
                dequant_row_f32(wg + row * wgu, sg + row * ggu, bg + row * ggu, H, bits, gs, rg);
                dequant_row_f32(wu + row * wgu, su + row * ggu, bu + row * ggu, H, bits, gs, ru);
                float g = (float)dot_f32_f64(xf, rg, H);
                float u = (float)dot_f32_f64(xf, ru, H);
                float hv;
                if (rounding == 0) {
                    g = round_bf16(g);
                    u = round_bf16(u);
                    float sg_ = round_bf16(1.0f / (1.0f + expf(-g)));
                    hv = round_bf16(round_bf16(sg_ * g) * u);
                } else {
                    hv = silu_f32(g) * u;
                }
                h[tk * I + n] = or_f32_to_bf16(hv);
            }
        }
        free(rg); free(ru); free(xf);
    }
    return OR_OK;
}

/* Stage 2: y[T,H] = combine over slots of the down projection of h. */
int or_moe_combine(const uint16_t *h, int64_t T, int64_t H, int64_t I, int64_t E,
                   int64_t top_k, const int32_t *idx, const float *scores,
                   const uint32_t *wd, const uint16_t *sd, const uint16_t *bd,
                   int bits, int gs, int rounding, uint16_t *y, int nthreads) {
    if (check_quant_params(H, I, bits, gs) || T < 0 || E <= 0 || top_k <= 0)
        return OR_INVALID;
    for (int64_t i = 0; i < T * top_k; ++i)
        if (idx[i] < 0 || idx[i] >= E) return OR_INVALID;
    set_threads(nthreads);
    const int64_t wdn = I * bits / 32, gdn = I / gs;
    float *hf = (float *)malloc(sizeof(float) * (size_t)(T * top_k * I + 1));
    for (int64_t i = 0; i < T * top_k * I; ++i) hf[i] = or_bf16_to_f32(h[i]);
#pragma omp parallel
    {
        float *rd = (float *)malloc(sizeof(float) * (size_t)I);
#pragma omp for schedule(dynamic, 1)
        for (int64_t t = 0; t < T; ++t) {
            for (int64_t n = 0; n < H; ++n) {
                double sum = 0.0;
                for (int64_t j = 0; j < top_k; ++j) {
                    int64_t tk = t * top_k + j, e = idx[tk];
                    int64_t row = e * H + n;
                    dequant_row_f32(wd + row * wdn, sd + row * gdn, bd + row * gdn, I, bits, gs, rd);
                    float d = (float)dot_f32_f64(hf + tk * I, rd, I);
                    float sc = round_bf16(scores[tk]);
                    if (rounding == 0) sum += (double)round_bf16(round_bf16(d) * sc);
                    else sum += (double)sc * (double)d;
                }
                y[t * H + n] = or_f32_to_bf16((float)sum);
            }
        }
        free(rd);
    }
    free(hf);
    return OR_OK;
}

int or_moe_switch(const uint16_t *x, int64_t T, int64_t H, int64_t I,
                  int64_t E, int64_t top_k, const int32_t *idx,
                  const float *scores, const uint32_t *wg, const uint16_t *sg,
                  const uint16_t *bg, const uint32_t *wu, const uint16_t *su,
                  const uint16_t *bu, const uint32_t *wd, const uint16_t *sd,
                  const uint16_t *bd, int bits, int gs, int rounding,
                  uint16_t *y, int nthreads) {
    uint16_t *h = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(T * top_k * I + 1));
    int rc = or_moe_hidden(x, T, H, I, E, top_k, idx, wg, sg, bg, wu, su, bu, bits, gs,
                           rounding, h, nthreads);
    if (!rc)
        rc = or_moe_combine(h, T, H, I, E, top_k, idx, scores, wd, sd, bd, bits, gs,
                            rounding, y, nthreads);
    free(h);
    return rc;
}
