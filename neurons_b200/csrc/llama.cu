// llama.cu -- a Llama decode step on the GPU around the quantized matmuls.
//
// Restates the reference's compiled decode function
// (compute/src/compute/model/llama_model.cpp:355-509) for one token:
//   h = embed[token]                                   (dequantized row, :384)
//   per layer:  x = rms_norm(h) ; q, k, v = lin(x)     (:392-402)
//               q, k = rope(q), rope(k) at pos ; append k, v to the cache
//               a = sdpa(q, K, V, 1/sqrt(head_dim))    (:446-470)
//               h = h + lin(a, o) ; x = rms_norm(h)
//               h = h + lin(sigmoid(g) * g * u, down), g, u = lin(x)  (:474-489)
//   logits = lin(rms_norm(h), lm_head or the tied embedding)  (:491-495)
//   next token = argmax(logits)                        (greedy, :745-790)
// and its pipelined generation (:713-812): the next step reads the token the
// previous step's argmax wrote to device memory, so steps queue back to back
// on the stream (or replay from a CUDA graph) with no host round trip.
//
// B200 layout: q/k/v weights are concatenated row-wise and gate/up rows
// interleaved in groups of 8 at creation, so each is one GEMV launch; RMSNorm
// runs inside the following GEMV's staging of x, SwiGLU in the gate|up GEMV's
// stores (a CTA holds each gate row with its up row), and both residual adds
// in the GEMVs' stores (launch_rows_fused).  Five launches per
// layer: qkv, attention, o, gate/up, down; then the final norm, the LM head
// and the argmax.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "nq.h"
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

constexpr int kAttnThreads = 128;
// Positions per attention CTA, 4 per warp.  Measured per layer at the
// Llama-3.2-3B dims, positions ~130-190, CUDA graph: chunks of 16 / 32 / 64 /
// 128 positions (4 / 8 / 16 / 32 per warp) take 6.9 / 7.9 / 11.3 / 17.5 us,
// and 2-warp CTAs are slower than 4-warp ones: the per-warp chain of
// dependent work, not the merge of more partials, sets the time.
constexpr int kAttnChunk = 16;
constexpr int kMaxGroup = 8;     // query heads per KV head

template <typename... Args>
cudaError_t launch_pdl_ll(void (*kern)(Args...), dim3 grid, unsigned threads, size_t smem,
                          cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// MLX dequantized value of one code: bf16(bf16(s * q) + b)
__device__ __forceinline__ uint16_t dq_value(uint32_t q, uint16_t s, uint16_t b) {
    const float p = bf16_to_f32(f32_to_bf16(__fmul_rn(bf16_to_f32(s), (float)q)));
    return f32_to_bf16(__fadd_rn(p, bf16_to_f32(b)));
}

// h = row `token` of the embedding (quantized: dequantized exactly as
// nq_dequantize; dense: copied).  The token comes from device memory.
__global__ void embed_kernel(const int32_t *tok_src, const uint32_t *ew, const uint16_t *es,
                             const uint16_t *eb, const uint16_t *dense, int64_t hidden, int bits,
                             int gs, int64_t vocab, uint16_t *h, unsigned *err) {
    pdl_launch_dependents();
    pdl_wait();  // the token may be the previous step's argmax
    int64_t t = *tok_src;
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, kErrBadIndex);
        t = 0;
    }
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < hidden;
         k += (int64_t)gridDim.x * blockDim.x) {
        if (dense) {
            h[k] = dense[t * hidden + k];
            continue;
        }
        const int per = 32 / bits;
        const uint32_t word = ew[t * (hidden / per) + k / per];
        const uint32_t q = (word >> (bits * (k % per))) & ((1u << bits) - 1u);
        const int64_t g = t * (hidden / gs) + k / gs;
        h[k] = dq_value(q, es[g], eb[g]);
    }
}

// RoPE (MLX fast::rope, traditional = false, scale 1): for i < d/2,
// angle = pos * base^(-i/(d/2)); (x_i, x_{i+d/2}) rotated by it in fp32 and
// rounded to bf16.  Returns the rotated value of element e of a head.
__device__ __forceinline__ float rope_elem(const uint16_t *head, int e, int hd, float pos,
                                           float log2_base) {
    const int half = hd / 2;
    const int i = e < half ? e : e - half;
    const float inv_freq = exp2f(-((float)i / (float)half) * log2_base);
    float sn, cs;
    sincosf(pos * inv_freq, &sn, &cs);
    const float x1 = bf16_to_f32(head[i]), x2 = bf16_to_f32(head[i + half]);
    const float r = e < half ? x1 * cs - x2 * sn : x1 * sn + x2 * cs;
    return bf16_to_f32(f32_to_bf16(r));
}

struct AttnArgs {
    const uint16_t *qkv;        // [n_heads + 2 n_kv][hd] bf16: q heads, k heads, v heads
    uint16_t *kc, *vc;          // this layer's caches [n_kv][max_ctx][hd]
    float *pm, *pl, *pacc;      // partials [n_heads][splits] (+ [hd] for pacc)
    int32_t *counter;           // [n_heads], zero between steps
    uint16_t *out;              // [n_heads][hd]
    const int32_t *pos;         // this step's position
    unsigned *err;
    int n_heads, n_kv, hd, max_ctx, splits;
    float log2_base, scale;
};

// kDpl consecutive bf16 values -> fp32 (one 4-, 8- or 16-byte load)
template <int N>
__device__ __forceinline__ void load_bf16(const uint16_t *p, float *out) {
    if constexpr (N == 2) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
        out[0] = bf16_to_f32((uint16_t)w);
        out[1] = bf16_to_f32((uint16_t)(w >> 16));
    } else if constexpr (N == 4) {
        const uint2 w = *reinterpret_cast<const uint2 *>(p);
        const uint32_t e[2] = {w.x, w.y};
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            out[2 * i] = bf16_to_f32((uint16_t)e[i]);
            out[2 * i + 1] = bf16_to_f32((uint16_t)(e[i] >> 16));
        }
    } else {
        const uint4 w = *reinterpret_cast<const uint4 *>(p);
        const uint32_t e[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[2 * i] = bf16_to_f32((uint16_t)e[i]);
            out[2 * i + 1] = bf16_to_f32((uint16_t)(e[i] >> 16));
        }
    }
}

// Flash-decoding attention: one CTA per (query head, chunk of kAttnChunk
// positions).  The query head (and, in the chunk holding `pos`, the new key)
// is rotated here; one CTA per KV head appends the new key/value to the
// cache.  Warp w takes kAttnChunk / 4 consecutive positions; each lane owns
// HD / 32 consecutive dims, so a key or value row is one coalesced load per
// warp and a warp's rows are all in flight together.  Each CTA writes its
// softmax partials (max, sum, weighted values); the last CTA of a query head
// (atomic count) merges the chunks in chunk order.  No CTA waits for another.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
    pdl_launch_dependents();
    pdl_wait();  // q, k, v come from the qkv projection
    constexpr int kDpl = HD / 32;
    constexpr int kWarps = kAttnThreads / 32;
    constexpr int kPerWarp = kAttnChunk / kWarps;
    __shared__ float qs[HD];
    __shared__ float kn[HD];
    __shared__ float sc[kAttnChunk];
    __shared__ float vred[kWarps][HD];
    __shared__ int last;
    const int hq = blockIdx.y, s = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int group = a.n_heads / a.n_kv, j = hq / group;
    const int pos = *a.pos;
    if (pos < 0 || pos >= a.max_ctx) {
        if (tid == 0 && s == 0 && hq == 0) atomicOr(a.err, kErrBadIndex);
        return;
    }
    const int n_active = pos / kAttnChunk + 1;
    if (s >= n_active) return;
    const int t0 = s * kAttnChunk, t1 = min(t0 + kAttnChunk, pos + 1);
    const float fpos = (float)pos;
    const uint16_t *qraw = a.qkv + (size_t)hq * HD;
    const uint16_t *kraw = a.qkv + (size_t)(a.n_heads + j) * HD;
    const uint16_t *vraw = a.qkv + (size_t)(a.n_heads + a.n_kv + j) * HD;
    const bool has_new = t1 == pos + 1;
    for (int d = tid; d < HD; d += kAttnThreads) {
        qs[d] = rope_elem(qraw, d, HD, fpos, a.log2_base);
        if (has_new) kn[d] = rope_elem(kraw, d, HD, fpos, a.log2_base);
    }
    uint16_t *kc = a.kc + (size_t)j * a.max_ctx * HD;
    uint16_t *vc = a.vc + (size_t)j * a.max_ctx * HD;
    __syncthreads();
    if (has_new && hq % group == 0) {
        for (int d = tid; d < HD; d += kAttnThreads) {
            kc[(size_t)pos * HD + d] = f32_to_bf16(kn[d]);
            vc[(size_t)pos * HD + d] = vraw[d];
        }
    }
    const int dim0 = lane * kDpl;
    float qv[kDpl];
#pragma unroll
    for (int i = 0; i < kDpl; ++i) qv[i] = qs[dim0 + i];
    // scores of this warp's positions
    const int tw = t0 + warp * kPerWarp;
    float sv[kPerWarp];
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
        const int t = tw + i;
        float kv[kDpl];
        if (t == pos) {
#pragma unroll
            for (int k = 0; k < kDpl; ++k) kv[k] = kn[dim0 + k];
        } else if (t < t1) {
            load_bf16<kDpl>(kc + (size_t)t * HD + dim0, kv);
        } else {
#pragma unroll
            for (int k = 0; k < kDpl; ++k) kv[k] = 0.f;
        }
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < kDpl; ++k) dot = fmaf(qv[k], kv[k], dot);
        sv[i] = dot;
    }
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sv[i] += __shfl_xor_sync(0xffffffffu, sv[i], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < kPerWarp; ++i) sc[warp * kPerWarp + i] = tw + i < t1 ? sv[i] * a.scale : -INFINITY;
    }
    __syncthreads();
    // chunk max and sum (every warp computes them over the whole chunk)
    float m = -INFINITY;
    for (int t = lane; t < kAttnChunk; t += 32) m = fmaxf(m, sc[t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int t = lane; t < kAttnChunk; t += 32) l += sc[t] == -INFINITY ? 0.f : expf(sc[t] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    // weighted values of this warp's positions
    float acc[kDpl];
#pragma unroll
    for (int k = 0; k < kDpl; ++k) acc[k] = 0.f;
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
        const int t = tw + i;
        if (t < t1) {
            float vv[kDpl];
            if (t == pos) {
#pragma unroll
                for (int k = 0; k < kDpl; ++k) vv[k] = bf16_to_f32(vraw[dim0 + k]);
            } else {
                load_bf16<kDpl>(vc + (size_t)t * HD + dim0, vv);
            }
            const float p = expf(sc[t - t0] - m);
#pragma unroll
            for (int k = 0; k < kDpl; ++k) acc[k] = fmaf(p, vv[k], acc[k]);
        }
    }
#pragma unroll
    for (int k = 0; k < kDpl; ++k) vred[warp][dim0 + k] = acc[k];
    __syncthreads();
    if (n_active == 1) {
        // one chunk holds every position: its sums are the result (the merge
        // below would compute the same values: a factor exp(0) = 1)
        for (int d = tid; d < HD; d += kAttnThreads) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += vred[w][d];
            a.out[(size_t)hq * HD + d] = f32_to_bf16(v / l);
        }
        return;
    }
    const size_t pb = (size_t)hq * a.splits + s;
    for (int d = tid; d < HD; d += kAttnThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += vred[w][d];
        a.pacc[pb * HD + d] = v;
    }
    if (tid == 0) {
        a.pm[pb] = m;
        a.pl[pb] = l;
    }
    // the last chunk of this query head to finish merges all of them
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&a.counter[hq], 1) == n_active - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int d = tid; d < HD; d += kAttnThreads) {
        const size_t p0 = (size_t)hq * a.splits;
        float mm = -INFINITY;
#pragma unroll 4
        for (int c = 0; c < n_active; ++c) mm = fmaxf(mm, __ldcg(&a.pm[p0 + c]));
        float ll = 0.f, o = 0.f;
#pragma unroll 4
        for (int c = 0; c < n_active; ++c) {
            const float f = expf(__ldcg(&a.pm[p0 + c]) - mm);
            ll = fmaf(__ldcg(&a.pl[p0 + c]), f, ll);
            o = fmaf(__ldcg(&a.pacc[(p0 + c) * HD + d]), f, o);
        }
        a.out[(size_t)hq * HD + d] = f32_to_bf16(o / ll);
    }
    if (tid == 0) a.counter[hq] = 0;
}

// next = argmax over the bf16 logits (first index of the maximum), over
// kArgmaxBlocks CTAs that each reduce a slice and the last one to finish
// (atomic count) reducing their results; logits also copied out as fp32 when
// asked; tokens_out[0] records the token; the position advances for the
// next step.  No CTA waits for another.
constexpr int kArgmaxBlocks = 128, kArgmaxThreads = 256;

__device__ __forceinline__ void better(float &bv, int64_t &bi, float v, int64_t i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(
    const uint16_t *logits, int64_t vocab, float *logits_f32, float *part_v, int32_t *part_i,
    int32_t *counter, int32_t *next, int32_t *tokens_out, int32_t *pos) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float wv[kArgmaxThreads / 32];
    __shared__ int64_t wi[kArgmaxThreads / 32];
    __shared__ int last;
    const int64_t per = (vocab + gridDim.x - 1) / gridDim.x;
    const int64_t lo = (int64_t)blockIdx.x * per, hi = min(vocab, lo + per);
    float best = -INFINITY;
    int64_t besti = vocab;  // (no finite logit: token 0)
#pragma unroll 4
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = bf16_to_f32(logits[i]);
        if (logits_f32) logits_f32[i] = v;
        if (v > best) {  // increasing i: ties keep the first index
            best = v;
            besti = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        better(best, besti, __shfl_xor_sync(0xffffffffu, best, o),
               __shfl_xor_sync(0xffffffffu, besti, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        wv[warp] = best;
        wi[warp] = besti;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; ++w) better(best, besti, wv[w], wi[w]);
        part_v[blockIdx.x] = best;
        part_i[blockIdx.x] = (int32_t)(besti < vocab ? besti : vocab);
        __threadfence();
        last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    best = -INFINITY;
    besti = vocab;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x)
        better(best, besti, __ldcg(&part_v[b]), __ldcg(&part_i[b]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        better(best, besti, __shfl_xor_sync(0xffffffffu, best, o),
               __shfl_xor_sync(0xffffffffu, besti, o));
    __syncthreads();
    if (lane == 0) {
        wv[warp] = best;
        wi[warp] = besti;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; ++w) better(best, besti, wv[w], wi[w]);
        const int32_t tok = besti < vocab ? (int32_t)besti : 0;
        *next = tok;
        if (tokens_out) tokens_out[0] = tok;
        *pos = *pos + 1;
        *counter = 0;
    }
}

__global__ void set_pos_kernel(int32_t *pos, int32_t v) { *pos = v; }

// xn = bf16(w * bf16(x * 1/sqrt(mean(x^2) + eps))) for one row (MLX rms_norm
// rounding, as the GEMV's fused prologue), one CTA.  Used before the LM head,
// whose thousands of CTAs would each recompute the norm in a fused prologue.
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const uint16_t *x, const uint16_t *w,
                                                       int64_t n, float eps, uint16_t *y) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float part[32];
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = bf16_to_f32(x[i]);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += part[i];
    const float inv = 1.0f / sqrtf(tot / (float)n + eps);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
        y[i] = f32_to_bf16(bf16_to_f32(w[i]) * bf16_to_f32(f32_to_bf16(bf16_to_f32(x[i]) * inv)));
}

}  // namespace

struct LlamaDecoder {
    nq_llama_config_t c{};
    // per layer: concatenated q|k|v and gate|up weights (owned), o and down borrowed
    struct Layer {
        const uint16_t *in_norm, *post_norm;
        uint32_t *qkv_w;
        uint16_t *qkv_s, *qkv_b;
        const uint32_t *o_w;
        const uint16_t *o_s, *o_b;
        uint32_t *gu_w;
        uint16_t *gu_s, *gu_b;
        const uint32_t *d_w;
        const uint16_t *d_s, *d_b;
    };
    std::vector<Layer> layers;
    const uint16_t *final_norm = nullptr;
    nq_qweight_t embed{}, head{};
    const uint16_t *embed_dense = nullptr;
    // device state
    uint16_t *kc = nullptr, *vc = nullptr;  // [layers][n_kv][max_ctx][hd]
    uint16_t *h = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr, *logits = nullptr;
    uint16_t *xn = nullptr;  // the final norm's output (LM head input)
    float *pm = nullptr, *pl = nullptr, *pacc = nullptr;
    int32_t *counter = nullptr, *pos = nullptr, *tok = nullptr;
    float *part_v = nullptr;  // argmax partials [kArgmaxBlocks]
    int32_t *part_i = nullptr, *amax_counter = nullptr;
    int splits = 1;
    int64_t host_pos = 0;  // steps enqueued since the last reset
    std::vector<void *> owned;

    ~LlamaDecoder() {
        for (void *p : owned) cudaFree(p);
    }
    template <typename T>
    cudaError_t alloc(T **p, size_t n) {
        void *v = nullptr;
        cudaError_t e = cudaMalloc(&v, n * sizeof(T));
        if (e == cudaSuccess) owned.push_back(v);
        *p = static_cast<T *>(v);
        return e;
    }
};

namespace {

cudaError_t concat_rows(const nq_qweight_t *parts, const int64_t *rows, int n, int64_t K, int bits,
                        int gs, uint32_t **w, uint16_t **s, uint16_t **b, LlamaDecoder &d) {
    int64_t total = 0;
    for (int i = 0; i < n; ++i) total += rows[i];
    const int64_t kw = K * bits / 32, G = K / gs;
    cudaError_t e;
    if ((e = d.alloc(w, (size_t)(total * kw))) != cudaSuccess) return e;
    if ((e = d.alloc(s, (size_t)(total * G))) != cudaSuccess) return e;
    if ((e = d.alloc(b, (size_t)(total * G))) != cudaSuccess) return e;
    int64_t r = 0;
    for (int i = 0; i < n; ++i) {
        if ((e = cudaMemcpy(*w + r * kw, parts[i].w, rows[i] * kw * 4, cudaMemcpyDeviceToDevice)))
            return e;
        if ((e = cudaMemcpy(*s + r * G, parts[i].scales, rows[i] * G * 2, cudaMemcpyDeviceToDevice)))
            return e;
        if ((e = cudaMemcpy(*b + r * G, parts[i].biases, rows[i] * G * 2, cudaMemcpyDeviceToDevice)))
            return e;
        r += rows[i];
    }
    return cudaSuccess;
}

// gate and up rows interleaved in groups of 8 (8 gate rows, the matching 8 up
// rows, ...): the row-group GEMV then holds each gate row and its up row in one
// CTA and forms SwiGLU in its stores
cudaError_t interleave_gate_up(const nq_qweight_t &gate, const nq_qweight_t &up, int64_t I,
                               int64_t K, int bits, int gs, uint32_t **w, uint16_t **s,
                               uint16_t **b, LlamaDecoder &d) {
    const int64_t kw = K * bits / 32, G = K / gs;
    cudaError_t e;
    if ((e = d.alloc(w, (size_t)(2 * I * kw))) != cudaSuccess) return e;
    if ((e = d.alloc(s, (size_t)(2 * I * G))) != cudaSuccess) return e;
    if ((e = d.alloc(b, (size_t)(2 * I * G))) != cudaSuccess) return e;
    const nq_qweight_t *src[2] = {&gate, &up};
    for (int h = 0; h < 2; ++h) {
        // rows [8i, 8i + 8) of the source -> rows [16i + 8h, 16i + 8h + 8)
        const size_t wrow = kw * 4, srow = G * 2;
        if ((e = cudaMemcpy2D(reinterpret_cast<char *>(*w) + 8 * h * wrow, 16 * wrow, src[h]->w,
                              8 * wrow, 8 * wrow, (size_t)(I / 8), cudaMemcpyDeviceToDevice)))
            return e;
        if ((e = cudaMemcpy2D(reinterpret_cast<char *>(*s) + 8 * h * srow, 16 * srow,
                              src[h]->scales, 8 * srow, 8 * srow, (size_t)(I / 8),
                              cudaMemcpyDeviceToDevice)))
            return e;
        if ((e = cudaMemcpy2D(reinterpret_cast<char *>(*b) + 8 * h * srow, 16 * srow,
                              src[h]->biases, 8 * srow, 8 * srow, (size_t)(I / 8),
                              cudaMemcpyDeviceToDevice)))
            return e;
    }
    return cudaSuccess;
}

cudaError_t gemv(const LlamaDecoder &d, const uint16_t *x, int64_t x_ld, const uint32_t *w,
                 const uint16_t *s, const uint16_t *b, int64_t N, int64_t K, uint16_t *y,
                 int prologue, const uint16_t *nw, const uint16_t *res, cudaStream_t st,
                 int epi_swiglu = 0) {
    RowsFusedArgs a;
    a.x = x;
    a.x_ld = x_ld;
    a.M = 1;
    a.w = w;
    a.s = s;
    a.b = b;
    a.N = N;
    a.K = K;
    a.bits = d.c.bits;
    a.gs = d.c.group_size;
    a.y = y;
    a.y_ld = N;
    a.prologue = prologue;
    a.norm_w = nw;
    a.eps = d.c.rms_eps;
    a.res = res;
    a.res_ld = N;
    a.epi_swiglu = epi_swiglu;
    return launch_rows_fused(a, st);
}

}  // namespace

cudaError_t launch_attention(int hd, dim3 grid, const AttnArgs &aa, cudaStream_t st) {
    if (hd == 64) return launch_pdl_ll(attn_kernel<64>, grid, kAttnThreads, 0, st, aa);
    if (hd == 128) return launch_pdl_ll(attn_kernel<128>, grid, kAttnThreads, 0, st, aa);
    return launch_pdl_ll(attn_kernel<256>, grid, kAttnThreads, 0, st, aa);
}

// One decode step: tok_src holds the input token (device); the argmax goes to
// d.tok (and tokens_out when given), logits_f32 (optional) gets the logits.
cudaError_t llama_step(LlamaDecoder &d, const int32_t *tok_src, float *logits_f32,
                       int32_t *tokens_out, cudaStream_t st) {
    const auto &c = d.c;
    unsigned *err = device_error_word();
    const int64_t H = c.hidden, hd = c.head_dim, nq_ = (int64_t)c.n_heads * hd,
                  nkv = (int64_t)c.n_kv_heads * hd, I = c.intermediate;
    cudaError_t e;
    if ((e = launch_pdl_ll(embed_kernel, dim3((unsigned)((H + 255) / 256)), 256, 0, st, tok_src,
                           d.embed.w, d.embed.scales, d.embed.biases, d.embed_dense, H, c.bits,
                           c.group_size, (int64_t)c.vocab, d.h, err)) != cudaSuccess)
        return e;
    AttnArgs aa;
    aa.qkv = d.qkv;
    aa.pm = d.pm;
    aa.pl = d.pl;
    aa.pacc = d.pacc;
    aa.counter = d.counter;
    aa.out = d.attn;
    aa.pos = d.pos;
    aa.err = err;
    aa.n_heads = c.n_heads;
    aa.n_kv = c.n_kv_heads;
    aa.hd = c.head_dim;
    aa.max_ctx = c.max_context;
    aa.splits = d.splits;
    aa.log2_base = log2f(c.rope_theta);
    aa.scale = 1.0f / sqrtf((float)c.head_dim);
    const size_t layer_cache = (size_t)c.n_kv_heads * c.max_context * hd;
    for (int l = 0; l < c.n_layers; ++l) {
        const auto &L = d.layers[l];
        if ((e = gemv(d, d.h, H, L.qkv_w, L.qkv_s, L.qkv_b, nq_ + 2 * nkv, H, d.qkv, 1, L.in_norm,
                      nullptr, st)) != cudaSuccess)
            return e;
        aa.kc = d.kc + (size_t)l * layer_cache;
        aa.vc = d.vc + (size_t)l * layer_cache;
        const dim3 agrid((unsigned)d.splits, (unsigned)c.n_heads);
        e = launch_attention(c.head_dim, agrid, aa, st);
        if (e != cudaSuccess) return e;
        if ((e = gemv(d, d.attn, nq_, L.o_w, L.o_s, L.o_b, H, nq_, d.h, 0, nullptr, d.h, st)) !=
            cudaSuccess)
            return e;
        // gate|up (interleaved) with the norm in its prologue and SwiGLU in its
        // stores: d.gu gets the I activations; down adds the residual
        if ((e = gemv(d, d.h, H, L.gu_w, L.gu_s, L.gu_b, 2 * I, H, d.gu, 1, L.post_norm, nullptr,
                      st, 1)) != cudaSuccess)
            return e;
        if ((e = gemv(d, d.gu, I, L.d_w, L.d_s, L.d_b, H, I, d.h, 0, nullptr, d.h, st)) !=
            cudaSuccess)
            return e;
    }
    if ((e = launch_pdl_ll(rmsnorm_kernel, dim3(1), 1024, 0, st, (const uint16_t *)d.h,
                           d.final_norm, H, c.rms_eps, d.xn)) != cudaSuccess)
        return e;
    if ((e = gemv(d, d.xn, H, d.head.w, d.head.scales, d.head.biases, c.vocab, H, d.logits, 0,
                  nullptr, nullptr, st)) != cudaSuccess)
        return e;
    const unsigned ablocks =
        (unsigned)std::min<int64_t>(kArgmaxBlocks, (c.vocab + kArgmaxThreads - 1) / kArgmaxThreads);
    return launch_pdl_ll(argmax_kernel, dim3(ablocks), kArgmaxThreads, 0, st,
                         (const uint16_t *)d.logits, (int64_t)c.vocab, logits_f32, d.part_v,
                         d.part_i, d.amax_counter, d.tok, tokens_out, d.pos);
}

cudaError_t llama_reset(LlamaDecoder &d, cudaStream_t st) {
    d.host_pos = 0;
    set_pos_kernel<<<1, 1, 0, st>>>(d.pos, 0);
    return cudaGetLastError();
}

const char *llama_unsupported(const nq_llama_config_t &c) {
    if (c.n_layers <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
        c.head_dim <= 0 || c.intermediate <= 0 || c.vocab <= 0 || c.max_context <= 0)
        return "every size must be positive";
    if (c.bits != 4) return "the decode step serves 4-bit codes";
    if (c.group_size != 32 && c.group_size != 64 && c.group_size != 128)
        return "group size must be 32, 64 or 128";
    if (c.n_heads % c.n_kv_heads || c.n_heads / c.n_kv_heads > kMaxGroup)
        return "n_heads must be a multiple of n_kv_heads, at most 8 query heads per KV head";
    if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
        return "head_dim must be 64, 128 or 256";
    const int64_t nq_ = (int64_t)c.n_heads * c.head_dim;
    if (c.hidden % 128 || c.intermediate % 128 || nq_ % 128)
        return "hidden, intermediate and n_heads * head_dim must be multiples of 128";
    if (c.hidden % c.group_size || c.intermediate % c.group_size || nq_ % c.group_size)
        return "the group size must divide hidden, intermediate and n_heads * head_dim";
    if ((int64_t)c.max_context > (int64_t)1 << 24) return "max_context too large";
    const int64_t nkv = (int64_t)c.n_kv_heads * c.head_dim;
    const int64_t shapes[5][2] = {{nq_ + 2 * nkv, c.hidden}, {c.hidden, nq_},
                                  {2 * (int64_t)c.intermediate, c.hidden},
                                  {c.hidden, c.intermediate}, {c.vocab, c.hidden}};
    for (const auto &sh : shapes)
        if (!rows_fused_supported(sh[0], sh[1], c.bits))
            return "a projection's shape is not served by the decode GEMV (K must split into "
                   "4..16 warps of 2..8 blocks of 128 codes, K <= 49152)";
    if (!(c.rope_theta > 0.f) || !(c.rms_eps >= 0.f)) return "rope_theta > 0 and rms_eps >= 0";
    return nullptr;
}

cudaError_t llama_create(LlamaDecoder &d, const nq_llama_config_t &c,
                         const nq_llama_layer_t *layers, const uint16_t *final_norm,
                         nq_qweight_t embed, const uint16_t *embed_dense, nq_qweight_t head) {
    d.c = c;
    d.final_norm = final_norm;
    d.embed = embed;
    d.embed_dense = embed_dense;
    d.head = head.w ? head : embed;
    const int64_t H = c.hidden, hd = c.head_dim, nq_ = (int64_t)c.n_heads * hd,
                  nkv = (int64_t)c.n_kv_heads * hd, I = c.intermediate;
    cudaError_t e;
    d.layers.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        const nq_llama_layer_t &s = layers[l];
        auto &L = d.layers[l];
        L.in_norm = s.input_norm;
        L.post_norm = s.post_norm;
        const nq_qweight_t qkv[3] = {s.q, s.k, s.v};
        const int64_t qkv_rows[3] = {nq_, nkv, nkv};
        if ((e = concat_rows(qkv, qkv_rows, 3, H, c.bits, c.group_size, &L.qkv_w, &L.qkv_s,
                             &L.qkv_b, d)) != cudaSuccess)
            return e;
        if ((e = interleave_gate_up(s.gate, s.up, I, H, c.bits, c.group_size, &L.gu_w, &L.gu_s,
                                    &L.gu_b, d)) != cudaSuccess)
            return e;
        L.o_w = s.o.w;
        L.o_s = s.o.scales;
        L.o_b = s.o.biases;
        L.d_w = s.down.w;
        L.d_s = s.down.scales;
        L.d_b = s.down.biases;
    }
    d.splits = (c.max_context + kAttnChunk - 1) / kAttnChunk;
    const size_t cache = (size_t)c.n_layers * c.n_kv_heads * c.max_context * hd;
    if ((e = d.alloc(&d.kc, cache)) || (e = d.alloc(&d.vc, cache)) || (e = d.alloc(&d.h, H)) ||
        (e = d.alloc(&d.xn, H)) ||
        (e = d.alloc(&d.qkv, nq_ + 2 * nkv)) || (e = d.alloc(&d.attn, nq_)) ||
        (e = d.alloc(&d.gu, 2 * I)) || (e = d.alloc(&d.logits, (size_t)c.vocab)) ||
        (e = d.alloc(&d.pm, (size_t)c.n_heads * d.splits)) ||
        (e = d.alloc(&d.pl, (size_t)c.n_heads * d.splits)) ||
        (e = d.alloc(&d.pacc, (size_t)c.n_heads * d.splits * hd)) ||
        (e = d.alloc(&d.counter, (size_t)c.n_heads)) || (e = d.alloc(&d.pos, 1)) ||
        (e = d.alloc(&d.tok, 1)) || (e = d.alloc(&d.part_v, kArgmaxBlocks)) ||
        (e = d.alloc(&d.part_i, kArgmaxBlocks)) || (e = d.alloc(&d.amax_counter, 1)))
        return e;
    if ((e = cudaMemset(d.amax_counter, 0, sizeof(int32_t)))) return e;
    if ((e = cudaMemset(d.counter, 0, sizeof(int32_t) * c.n_heads)) ||
        (e = cudaMemset(d.pos, 0, sizeof(int32_t))) || (e = cudaMemset(d.tok, 0, sizeof(int32_t))))
        return e;
    return cudaDeviceSynchronize();
}

}  // namespace nq

// ---------------------------------------------------------------------------
// C ABI (include/nq.h, "Llama decode step")
// ---------------------------------------------------------------------------
struct nq_llama_s {
    nq::LlamaDecoder d;
};

namespace {
int llama_fail(int status, const std::string &msg) {
    nq::set_error(msg);
    return status;
}
int llama_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return NQ_SUCCESS;
    cudaGetLastError();
    return llama_fail(NQ_COMPUTE_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
}
bool qw_ok(const nq_qweight_t &q) { return q.w && q.scales && q.biases; }
}  // namespace

extern "C" {

int nq_llama_create(nq_llama_t *out, const nq_llama_config_t *cfg, const nq_llama_layer_t *layers,
                    const uint16_t *final_norm, const nq_qweight_t *embed,
                    const nq_qweight_t *lm_head) {
    const char *what = "nq_llama_create";
    if (!out || !cfg || !layers || !final_norm || !embed)
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": NULL argument");
    *out = nullptr;
    if (const char *why = nq::llama_unsupported(*cfg))
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": " + why);
    const bool dense_embed = embed->w && !embed->scales;
    if (!embed->w || (!dense_embed && !qw_ok(*embed)))
        return llama_fail(NQ_INVALID_MODEL, std::string(what) + ": embedding weights missing");
    if (dense_embed && !(lm_head && qw_ok(*lm_head)))
        return llama_fail(NQ_INVALID_MODEL,
                          std::string(what) + ": an unquantized embedding needs a quantized lm_head");
    if (lm_head && lm_head->w && !qw_ok(*lm_head))
        return llama_fail(NQ_INVALID_MODEL, std::string(what) + ": lm_head scales/biases missing");
    for (int l = 0; l < cfg->n_layers; ++l) {
        const nq_llama_layer_t &L = layers[l];
        if (!L.input_norm || !L.post_norm || !qw_ok(L.q) || !qw_ok(L.k) || !qw_ok(L.v) ||
            !qw_ok(L.o) || !qw_ok(L.gate) || !qw_ok(L.up) || !qw_ok(L.down))
            return llama_fail(NQ_INVALID_MODEL, std::string(what) + ": layer " + std::to_string(l) +
                                                    ": a weight is missing");
        if ((reinterpret_cast<uintptr_t>(L.input_norm) | reinterpret_cast<uintptr_t>(L.post_norm)) &
            15)
            return llama_fail(NQ_INVALID_INPUT,
                              std::string(what) + ": norm weights must be 16-byte aligned");
    }
    if (reinterpret_cast<uintptr_t>(final_norm) & 15)
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": norm weights must be 16-byte aligned");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return llama_fail(NQ_BACKEND_NOT_AVAILABLE, std::string(what) + ": no CUDA device");
    }
    auto *h = new nq_llama_s;
    nq_qweight_t head{};
    if (lm_head && lm_head->w) head = *lm_head;
    nq_qweight_t emb = *embed;
    const uint16_t *dense = nullptr;
    if (dense_embed) {
        dense = reinterpret_cast<const uint16_t *>(embed->w);
        emb = nq_qweight_t{};
    }
    if (int rc = llama_cuda(nq::llama_create(h->d, *cfg, layers, final_norm, emb, dense, head), what)) {
        delete h;
        return rc;
    }
    *out = h;
    return NQ_SUCCESS;
}

int nq_llama_destroy(nq_llama_t dec) {
    delete dec;
    return NQ_SUCCESS;
}

int64_t nq_llama_position(nq_llama_t dec) { return dec ? dec->d.host_pos : -1; }

int nq_llama_reset(nq_llama_t dec, void *stream) {
    if (!dec) return llama_fail(NQ_INVALID_INPUT, "nq_llama_reset: NULL decoder");
    return llama_cuda(nq::llama_reset(dec->d, static_cast<cudaStream_t>(stream)), "nq_llama_reset");
}

int nq_llama_step(nq_llama_t dec, const int32_t *token, float *logits, int32_t *next_token,
                  void *stream) {
    const char *what = "nq_llama_step";
    if (!dec) return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": NULL decoder");
    auto &d = dec->d;
    if (d.host_pos >= d.c.max_context)
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": context full (max_context " +
                                                std::to_string(d.c.max_context) + ")");
    const int32_t *src = token ? token : d.tok;
    if (int rc = llama_cuda(nq::llama_step(d, src, logits, next_token,
                                           static_cast<cudaStream_t>(stream)),
                            what))
        return rc;
    ++d.host_pos;
    return NQ_SUCCESS;
}

int nq_llama_prefill(nq_llama_t dec, const int32_t *tokens, int64_t n, float *logits,
                     void *stream) {
    const char *what = "nq_llama_prefill";
    if (!dec || !tokens || n <= 0)
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": need a decoder and n > 0 tokens");
    auto &d = dec->d;
    if (d.host_pos + n > d.c.max_context)
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": context full");
    for (int64_t i = 0; i < n; ++i) {
        if (int rc = llama_cuda(nq::llama_step(d, tokens + i, i + 1 == n ? logits : nullptr,
                                               nullptr, static_cast<cudaStream_t>(stream)),
                                what))
            return rc;
        ++d.host_pos;
    }
    return NQ_SUCCESS;
}

int nq_llama_generate(nq_llama_t dec, const int32_t *token, int64_t n, int32_t *tokens,
                      void *stream) {
    const char *what = "nq_llama_generate";
    if (!dec || !tokens || n <= 0)
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": need a decoder, n > 0, tokens");
    auto &d = dec->d;
    if (d.host_pos + n > d.c.max_context)
        return llama_fail(NQ_INVALID_INPUT, std::string(what) + ": context full");
    for (int64_t i = 0; i < n; ++i) {
        const int32_t *src = (i == 0 && token) ? token : d.tok;
        if (int rc = llama_cuda(nq::llama_step(d, src, nullptr, tokens + i,
                                               static_cast<cudaStream_t>(stream)),
                                what))
            return rc;
        ++d.host_pos;
    }
    return NQ_SUCCESS;
}

}  // extern "C"
