// quant.cu -- MLX-affine quantize/pack and dequantize kernels, sm_100a.
//
// Both are HBM-bound streaming kernels: every thread owns 16 contiguous
// bytes of the narrower side (8 input values for quantize, 4 packed words for
// dequantize), loads and stores are 128-bit and coalesced across the warp,
// and a quantization group (32/64/128 values) is spread over 4/8/16
// consecutive lanes that reduce min/max with shuffles.
//
// Arithmetic is written with explicit round-to-nearest intrinsics so that the
// compiler cannot contract or reassociate it: the codes, scales and biases
// (quantize) and the dequantized bf16 values (dequantize) are bit-identical
// to MLX's CPU semantics as restated by the oracle.
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

// Quantize: one thread per 8 consecutive values along K.  IN: 0 fp32, 1 bf16,
// 2 fp16 weights; fp16 weights give fp16 scales and biases, the others bf16.
template <int BITS, int IN>
__global__ void __launch_bounds__(256) quantize_kernel(const void *__restrict__ w, int64_t rows,
                                                       int64_t K, int gs, int scheme,
                                                       uint32_t *__restrict__ wq,
                                                       uint16_t *__restrict__ scales,
                                                       uint16_t *__restrict__ biases) {
    const int64_t chunks_per_row = K / 8;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = rows * chunks_per_row;
    // Lanes of a group are consecutive and a group never straddles a row, so
    // out-of-range lanes form whole groups: they compute on a valid address
    // and do not store.
    const bool active = t < total;
    const int64_t tt = active ? t : total - 1;
    const int64_t row = tt / chunks_per_row;
    const int64_t chunk = tt % chunks_per_row;

    float v[8];
    if (IN != 0) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(w) +
                                                            row * K + chunk * 8);
        const uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = t16_to_f32<IN == 2>((uint16_t)r[i]);
            v[2 * i + 1] = t16_to_f32<IN == 2>((uint16_t)(r[i] >> 16));
        }
    } else {
        const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(w) +
                                                             row * K + chunk * 8);
        const float4 a = src[0], b = src[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    float w_max = v[0], w_min = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) {
        w_max = fmaxf(w_max, v[i]);
        w_min = fminf(w_min, v[i]);
    }
    const int lanes = gs / 8;  // 4, 8 or 16
    for (int o = 1; o < lanes; o <<= 1) {
        w_max = fmaxf(w_max, __shfl_xor_sync(0xffffffffu, w_max, o));
        w_min = fminf(w_min, __shfl_xor_sync(0xffffffffu, w_min, o));
    }
    const float n_bins = (float)((1 << BITS) - 1);
    float scale, bias;
    if (scheme == 0) {
        const float eps = 1e-7f;
        const bool mask = fabsf(w_min) > fabsf(w_max);
        scale = fmaxf(__fdiv_rn(__fsub_rn(w_max, w_min), n_bins), eps);
        scale = mask ? scale : -scale;
        const float edge = mask ? w_min : w_max;
        const float q0 = rintf(__fdiv_rn(edge, scale));
        bias = 0.0f;
        if (q0 != 0.0f) {
            scale = __fdiv_rn(edge, q0);
            bias = edge;
        }
    } else {
        scale = __fdiv_rn(__fsub_rn(w_max, w_min), n_bins);
        bias = w_min;
    }
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float qq = 0.0f;
        if (scale != 0.0f) {
            qq = rintf(__fdiv_rn(__fsub_rn(v[i], bias), scale));
            qq = fminf(fmaxf(qq, 0.0f), n_bins);
        }
        q[i] = (uint32_t)qq;
    }
    if (!active) return;
    if (BITS == 4) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) word |= q[i] << (4 * i);
        wq[row * (K / 8) + chunk] = word;
    } else {
        const uint32_t w0 = q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24);
        const uint32_t w1 = q[4] | (q[5] << 8) | (q[6] << 16) | (q[7] << 24);
        *reinterpret_cast<uint2 *>(wq + row * (K / 4) + chunk * 2) = make_uint2(w0, w1);
    }
    if ((chunk % lanes) == 0) {
        const int64_t gidx = row * (K / gs) + chunk / lanes;
        scales[gidx] = f32_to_t16<IN == 2>(scale);
        biases[gidx] = f32_to_t16<IN == 2>(bias);
    }
}

// Dequantize: one thread per 16 bytes of packed words (32 codes at 4 bits,
// 16 codes at 8 bits, always inside one group); output 64 or 32 contiguous
// bytes of bf16 (fp16 when the scales are fp16).  Codes are dequantized in
// packed pairs exactly as the matmul kernels do it (nq_common.cuh): biased
// codes, one packed fma or sub/mul and one packed add per two codes, each
// rounding the exact value once -- the same bits as T(T(s*q) + b).
template <int BITS, bool F16>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t *__restrict__ wq,
                                                         const uint16_t *__restrict__ scales,
                                                         const uint16_t *__restrict__ biases,
                                                         int64_t rows, int64_t K, int gs,
                                                         uint16_t *__restrict__ out) {
    constexpr int kCodes = 4 * 32 / BITS;  // codes per thread (4 words)
    const int64_t Kw = K * BITS / 32;
    const int64_t vec_per_row = Kw / 4;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= rows * vec_per_row) return;
    const int64_t row = t / vec_per_row;
    const int64_t vec = t % vec_per_row;
    const uint4 raw = *reinterpret_cast<const uint4 *>(wq + row * Kw + vec * 4);
    const int64_t k0 = vec * kCodes;
    const int64_t gidx = row * (K / gs) + k0 / gs;
    const uint16_t sv = scales[gidx], bv = biases[gidx];
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t outw[kCodes / 2];
    if constexpr (BITS == 4) {
        const Dq4 d = F16 ? Dq4{} : make_dq4(sv, bv);
        const Dq4h dh = make_dq4h(sv, bv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t p[4];  // (q_j, q_{j+4}) for j = 0..3
#pragma unroll
            for (int j = 0; j < 4; ++j)
                p[j] = F16 ? dqh_pair(q4_pair_biased_h(words[i], j), dh)
                           : dq4_pair(q4_pair_biased(words[i], j), d);
            outw[4 * i + 0] = prmt(p[0], p[1], 0x5410u);  // (q0, q1)
            outw[4 * i + 1] = prmt(p[2], p[3], 0x5410u);  // (q2, q3)
            outw[4 * i + 2] = prmt(p[0], p[1], 0x7632u);  // (q4, q5)
            outw[4 * i + 3] = prmt(p[2], p[3], 0x7632u);  // (q6, q7)
        }
    } else {
        const Dq4h dh = make_dq4h(sv, bv);
        const Dq8 d8 = F16 ? Dq8{} : make_dq8(sv, bv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            outw[2 * i + 0] = F16 ? dqh_pair(q8_pair_biased_h(words[i], 0, 1), dh)
                                  : dq8_pair(words[i], 0, 1, d8);
            outw[2 * i + 1] = F16 ? dqh_pair(q8_pair_biased_h(words[i], 2, 3), dh)
                                  : dq8_pair(words[i], 2, 3, d8);
        }
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out + row * K + k0);
#pragma unroll
    for (int i = 0; i < kCodes / 8; ++i)
        dst[i] = make_uint4(outw[4 * i], outw[4 * i + 1], outw[4 * i + 2], outw[4 * i + 3]);
}

}  // namespace

cudaError_t launch_quantize(const void *w, int w_dtype, int64_t rows, int64_t K, int bits,
                            int gs, int scheme, uint32_t *wq, uint16_t *s, uint16_t *b,
                            cudaStream_t stream) {
    const int64_t total = rows * (K / 8);
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    const dim3 grid((unsigned)((total + threads - 1) / threads));
#define NQ_QUANT(B, IN) \
    quantize_kernel<B, IN><<<grid, threads, 0, stream>>>(w, rows, K, gs, scheme, wq, s, b)
    if (bits == 4) {
        if (w_dtype == 2) NQ_QUANT(4, 2);
        else if (w_dtype == 1) NQ_QUANT(4, 1);
        else NQ_QUANT(4, 0);
    } else {
        if (w_dtype == 2) NQ_QUANT(8, 2);
        else if (w_dtype == 1) NQ_QUANT(8, 1);
        else NQ_QUANT(8, 0);
    }
#undef NQ_QUANT
    return cudaGetLastError();
}

cudaError_t launch_dequantize(const uint32_t *wq, const uint16_t *s, const uint16_t *b,
                              int64_t rows, int64_t K, int bits, int gs, uint16_t *out,
                              cudaStream_t stream, bool f16) {
    const int64_t total = rows * (K * bits / 32 / 4);
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    const dim3 grid((unsigned)((total + threads - 1) / threads));
    if (bits == 4 && f16)
        dequantize_kernel<4, true><<<grid, threads, 0, stream>>>(wq, s, b, rows, K, gs, out);
    else if (bits == 4)
        dequantize_kernel<4, false><<<grid, threads, 0, stream>>>(wq, s, b, rows, K, gs, out);
    else if (f16)
        dequantize_kernel<8, true><<<grid, threads, 0, stream>>>(wq, s, b, rows, K, gs, out);
    else
        dequantize_kernel<8, false><<<grid, threads, 0, stream>>>(wq, s, b, rows, K, gs, out);
    return cudaGetLastError();
}

}  // namespace nq
