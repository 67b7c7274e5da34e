// CUDA-core (SIMT) kernels for the three attention operators.
//
// These cover every dtype and shape the C ABI accepts. They are the production path
// for float32 (whose 1e-4 parity bound rules out tf32 tensor-core math) and for shapes
// outside the tensor-core kernels' envelope. Numerics follow the reference plugins:
// scores accumulate in fp32 and are stored to the I/O dtype where the reference's
// cuBLAS GEMMs store them; softmax runs in fp32.
#include <algorithm>

#include "fga_common.cuh"
#include "fga_kernels.h"

namespace fga {
namespace {

constexpr int kSimtWarps = 4;  // warps per block; one row per warp

// ---------------------------------------------------------------------------------------
// Zipformer relative-attention weights.
//
// One warp owns one (n, h, q) row. Pass 1 computes every valid key's logit
//   round_T(q . k) + sum_i pq_i * pos[T-1-q+k, h, i]
// and accumulates an online (max, sum); pass 2 recomputes the logit and writes the
// normalised weight. Masked keys are written as 0; a row whose keys are all masked is
// all zero; rows inside the padded-query halo (q >= 7 and mask[q-7]) are all zero.
// Reference: zipformer_relative_attention_plugin.cu:238-327 and
// export/model/zipformer/attention.py:253-289.
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kSimtWarps * kWarp)
zipformer_weights_simt_kernel(const T* __restrict__ proj, const T* __restrict__ pos,
                              const uint8_t* __restrict__ mask, T* __restrict__ out,
                              int batch, int heads, int length, int qd) {
    extern __shared__ float smem_q[];  // [kSimtWarps][qd]
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t rows = static_cast<int64_t>(batch) * heads * length;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kSimtWarps + warp;
    if (row >= rows) return;
    const int q = static_cast<int>(row % length);
    const int h = static_cast<int>((row / length) % heads);
    const int n = static_cast<int>(row / (static_cast<int64_t>(length) * heads));
    const int pdim = heads * (2 * qd + 4);
    T* orow = out + row * length;
    const uint8_t* mrow = mask + static_cast<int64_t>(n) * length;

    if (q >= 7 && mrow[q - 7]) {
        for (int k = lane; k < length; k += kWarp) orow[k] = from_f32<T>(0.0f);
        return;
    }
    const T* qrow = proj + (static_cast<int64_t>(n) * length + q) * pdim;
    float* sq = smem_q + warp * qd;
    for (int d = lane; d < qd; d += kWarp) sq[d] = ldf(qrow + h * qd + d);
    const T* pq = qrow + 2 * heads * qd + h * 4;
    const float pq0 = ldf(pq), pq1 = ldf(pq + 1), pq2 = ldf(pq + 2), pq3 = ldf(pq + 3);
    __syncwarp();

    const T* kbase = proj + static_cast<int64_t>(n) * length * pdim + heads * qd + h * qd;
    auto logit = [&](int k) {
        const T* krow = kbase + static_cast<int64_t>(k) * pdim;
        float s = 0.0f;
        for (int d = 0; d < qd; ++d) s = fmaf(sq[d], ldf(krow + d), s);
        const T* pr = pos + (static_cast<int64_t>(length - 1 - q + k) * heads + h) * 4;
        float r = round_to<T>(s);
        r = fmaf(pq0, ldf(pr), r);
        r = fmaf(pq1, ldf(pr + 1), r);
        r = fmaf(pq2, ldf(pr + 2), r);
        r = fmaf(pq3, ldf(pr + 3), r);
        return r;
    };

    float m = -INFINITY, l = 0.0f;
    for (int k = lane; k < length; k += kWarp) {
        if (mrow[k]) continue;
        const float s = logit(k);
        const float mn = fmaxf(m, s);
        l = l * __expf(m - mn) + __expf(s - mn);
        m = mn;
    }
    // Combine the lanes' (max, sum) pairs.
    const float mw = warp_max(m);
    l = (m == -INFINITY) ? 0.0f : l * __expf(m - mw);
    l = warp_sum(l);
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    for (int k = lane; k < length; k += kWarp) {
        float w = 0.0f;
        if (!mrow[k]) w = __expf(logit(k) - mw) * inv;
        orow[k] = from_f32<T>(w);
    }
}

// ---------------------------------------------------------------------------------------
// Zipformer attention-value.
//   out[n,q,h,d] = sum_k A[n, h_a, q, k] * V[n, k, h*hd + d],  h_a = (value_heads==1 ? 0 : h)
// Narrow heads (hd <= 32): lanes split the keys, each lane accumulates all hd channels,
// and a butterfly reduction combines them (the access pattern of the reference's
// attentionValueHead12, zipformer_attention_value_plugin.cu:118-181, for any hd).
// Wide heads (NonlinAttention, hd = 3E/4): lanes split the channels in chunks of 32*CPL
// and broadcast 32 coalesced attention weights at a time with shuffles.
// ---------------------------------------------------------------------------------------
template <typename T, int MAXD>
__global__ void __launch_bounds__(kSimtWarps * kWarp)
value_keysplit_kernel(const T* __restrict__ att, const T* __restrict__ val, T* __restrict__ out,
                      int batch, int att_heads, int value_heads, int length, int channels) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int hd = channels / value_heads;
    const int64_t rows = static_cast<int64_t>(batch) * value_heads * length;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kSimtWarps + warp;
    if (row >= rows) return;
    const int q = static_cast<int>(row % length);
    const int h = static_cast<int>((row / length) % value_heads);
    const int n = static_cast<int>(row / (static_cast<int64_t>(length) * value_heads));
    const T* arow = att + ((static_cast<int64_t>(n) * att_heads + h) * length + q) * length;
    const T* vbase = val + static_cast<int64_t>(n) * length * channels + h * hd;
    float acc[MAXD];
#pragma unroll
    for (int d = 0; d < MAXD; ++d) acc[d] = 0.0f;
    for (int k = lane; k < length; k += kWarp) {
        const float w = ldf(arow + k);
        const T* vr = vbase + static_cast<int64_t>(k) * channels;
#pragma unroll
        for (int d = 0; d < MAXD; ++d)
            if (d < hd) acc[d] = fmaf(w, ldf(vr + d), acc[d]);
    }
#pragma unroll
    for (int d = 0; d < MAXD; ++d) acc[d] = warp_sum(acc[d]);
    T* orow = out + (static_cast<int64_t>(n) * length + q) * channels + h * hd;
#pragma unroll
    for (int d = 0; d < MAXD; ++d)
        if (d < hd && lane == (d & 31)) orow[d] = from_f32<T>(acc[d]);
}

template <typename T, int CPL>
__global__ void __launch_bounds__(kSimtWarps * kWarp)
value_chansplit_kernel(const T* __restrict__ att, const T* __restrict__ val, T* __restrict__ out,
                       int batch, int att_heads, int value_heads, int length, int channels) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int hd = channels / value_heads;
    const int c0 = blockIdx.y * (kWarp * CPL);  // first channel of this chunk within the head
    const int64_t rows = static_cast<int64_t>(batch) * value_heads * length;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kSimtWarps + warp;
    if (row >= rows) return;
    const int q = static_cast<int>(row % length);
    const int h = static_cast<int>((row / length) % value_heads);
    const int n = static_cast<int>(row / (static_cast<int64_t>(length) * value_heads));
    const T* arow = att + ((static_cast<int64_t>(n) * att_heads + h) * length + q) * length;
    const T* vbase = val + static_cast<int64_t>(n) * length * channels + h * hd + c0;
    float acc[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[c] = 0.0f;
    for (int k0 = 0; k0 < length; k0 += kWarp) {
        const int kk = k0 + lane;
        const float wl = kk < length ? ldf(arow + kk) : 0.0f;
        const int kend = min(kWarp, length - k0);
        for (int j = 0; j < kend; ++j) {
            const float w = __shfl_sync(0xffffffffu, wl, j);
            const T* vr = vbase + static_cast<int64_t>(k0 + j) * channels;
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const int ch = lane + kWarp * c;
                if (c0 + ch < hd) acc[c] = fmaf(w, ldf(vr + ch), acc[c]);
            }
        }
    }
    T* orow = out + (static_cast<int64_t>(n) * length + q) * channels + h * hd + c0;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int ch = lane + kWarp * c;
        if (c0 + ch < hd) orow[ch] = from_f32<T>(acc[c]);
    }
}

// ---------------------------------------------------------------------------------------
// Parakeet relative-position MHSA, flash-style on CUDA cores.
//
// One warp owns one (n, h, q) row. Biased queries q+u and q+v are formed in fp32 and
// rounded to T (parakeet_relative_attention_plugin.cu:268-281, 339-345). Keys are
// visited in chunks of 32 (one key per lane): content and positional dots accumulate
// in fp32 and are rounded to T like the reference's GEMM outputs, summed and scaled in
// fp32 (the reference's score promotion, .cu:503-508), and folded into an online
// softmax; lanes then split the head channels to accumulate P.V. Only keys
// k < min(T, valid_length) are visited; valid_length <= 0 gives a zero row.
// NaN and infinite logits propagate as in the reference softmax (.cu:480-537).
// ---------------------------------------------------------------------------------------
template <typename T, int CPL>
__global__ void __launch_bounds__(kSimtWarps * kWarp)
parakeet_simt_kernel(const T* __restrict__ qkv, const T* __restrict__ pos,
                     const T* __restrict__ ubias, const T* __restrict__ vbias,
                     const int32_t* __restrict__ lengths, T* __restrict__ out, int batch,
                     int heads, int length, int head_dim, float scale) {
    extern __shared__ float smem[];  // [kSimtWarps][2][head_dim]
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t rows = static_cast<int64_t>(batch) * heads * length;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kSimtWarps + warp;
    if (row >= rows) return;
    // Row order (n, q, h) keeps the warps of one block on one query frame.
    const int h = static_cast<int>(row % heads);
    const int q = static_cast<int>((row / heads) % length);
    const int n = static_cast<int>(row / (static_cast<int64_t>(heads) * length));
    const int C = heads * head_dim;
    const int64_t C3 = 3LL * C;
    T* orow = out + (static_cast<int64_t>(n) * length + q) * C + h * head_dim;
    const int valid = min(lengths[n], length);
    if (valid <= 0) {
        for (int d = lane; d < head_dim; d += kWarp) orow[d] = from_f32<T>(0.0f);
        return;
    }
    float* su = smem + warp * 2 * head_dim;
    float* sv = su + head_dim;
    const T* qrow = qkv + (static_cast<int64_t>(n) * length + q) * C3 + h * head_dim;
    for (int d = lane; d < head_dim; d += kWarp) {
        const float x = ldf(qrow + d);
        su[d] = round_to<T>(x + ldf(ubias + h * head_dim + d));
        sv[d] = round_to<T>(x + ldf(vbias + h * head_dim + d));
    }
    __syncwarp();
    const T* kbase = qkv + static_cast<int64_t>(n) * length * C3 + C + h * head_dim;
    const T* vbase = qkv + static_cast<int64_t>(n) * length * C3 + 2 * C + h * head_dim;
    const T* pbase = pos + h * head_dim;

    float m = -INFINITY, l = 0.0f;
    float acc[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[c] = 0.0f;
    for (int k0 = 0; k0 < valid; k0 += kWarp) {
        const int k = k0 + lane;
        float s = -INFINITY;
        if (k < valid) {
            const T* kr = kbase + static_cast<int64_t>(k) * C3;
            const T* pr = pbase + static_cast<int64_t>(length - 1 - q + k) * C;
            float sc = 0.0f, sp = 0.0f;
            for (int d = 0; d < head_dim; ++d) {
                sc = fmaf(su[d], ldf(kr + d), sc);
                sp = fmaf(sv[d], ldf(pr + d), sp);
            }
            s = (round_to<T>(sc) + round_to<T>(sp)) * scale;
        }
        const float mn = fmaxf(m, warp_max(s));
        const float alpha = __expf(m - mn);
        const float p = k < valid ? __expf(s - mn) : 0.0f;
        l = l * alpha + warp_sum(p);
#pragma unroll
        for (int c = 0; c < CPL; ++c) acc[c] *= alpha;
        m = mn;
        const int kend = min(kWarp, valid - k0);
        for (int j = 0; j < kend; ++j) {
            const float w = __shfl_sync(0xffffffffu, p, j);
            const T* vr = vbase + static_cast<int64_t>(k0 + j) * C3;
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const int d = lane + kWarp * c;
                if (d < head_dim) acc[c] = fmaf(w, ldf(vr + d), acc[c]);
            }
        }
    }
    const float inv = 1.0f / l;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int d = lane + kWarp * c;
        if (d < head_dim) orow[d] = from_f32<T>(acc[c] * inv);
    }
}

template <typename T>
cudaError_t parakeet_simt_typed(const ParakeetProblem& p, cudaStream_t stream) {
    const int64_t rows = static_cast<int64_t>(p.batch) * p.heads * p.length;
    const dim3 grid(static_cast<unsigned>((rows + kSimtWarps - 1) / kSimtWarps));
    const size_t smem = sizeof(float) * kSimtWarps * 2 * p.head_dim;
    const int cpl = (p.head_dim + kWarp - 1) / kWarp;
    auto args = [&](auto kernel) {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        kernel<<<grid, kSimtWarps * kWarp, smem, stream>>>(
            static_cast<const T*>(p.qkv), static_cast<const T*>(p.position),
            static_cast<const T*>(p.content_bias), static_cast<const T*>(p.position_bias),
            p.valid_lengths, static_cast<T*>(p.output), p.batch, p.heads, p.length,
            p.head_dim, p.scale);
    };
    if (cpl <= 1) args(parakeet_simt_kernel<T, 1>);
    else if (cpl <= 2) args(parakeet_simt_kernel<T, 2>);
    else if (cpl <= 4) args(parakeet_simt_kernel<T, 4>);
    else if (cpl <= 8) args(parakeet_simt_kernel<T, 8>);
    else args(parakeet_simt_kernel<T, 16>);
    return cudaGetLastError();
}

template <typename T>
cudaError_t zipformer_weights_simt_typed(const ZipformerWeightsProblem& p, cudaStream_t stream) {
    const int64_t rows = static_cast<int64_t>(p.batch) * p.heads * p.length;
    const dim3 grid(static_cast<unsigned>((rows + kSimtWarps - 1) / kSimtWarps));
    const size_t smem = sizeof(float) * kSimtWarps * p.query_dim;
    zipformer_weights_simt_kernel<T><<<grid, kSimtWarps * kWarp, smem, stream>>>(
        static_cast<const T*>(p.projection), static_cast<const T*>(p.position), p.mask,
        static_cast<T*>(p.weights), p.batch, p.heads, p.length, p.query_dim);
    return cudaGetLastError();
}

template <typename T>
cudaError_t zipformer_value_simt_typed(const ZipformerValueProblem& p, cudaStream_t stream) {
    const int64_t rows = static_cast<int64_t>(p.batch) * p.value_heads * p.length;
    const unsigned blocks = static_cast<unsigned>((rows + kSimtWarps - 1) / kSimtWarps);
    const int hd = p.channels / p.value_heads;
    const T* a = static_cast<const T*>(p.attention);
    const T* v = static_cast<const T*>(p.value);
    T* o = static_cast<T*>(p.output);
    if (hd <= 16) {
        value_keysplit_kernel<T, 16><<<blocks, kSimtWarps * kWarp, 0, stream>>>(
            a, v, o, p.batch, p.attention_heads, p.value_heads, p.length, p.channels);
    } else if (hd <= 32) {
        value_keysplit_kernel<T, 32><<<blocks, kSimtWarps * kWarp, 0, stream>>>(
            a, v, o, p.batch, p.attention_heads, p.value_heads, p.length, p.channels);
    } else {
        constexpr int kCpl = 8;
        const dim3 grid(blocks, static_cast<unsigned>((hd + kWarp * kCpl - 1) / (kWarp * kCpl)));
        value_chansplit_kernel<T, kCpl><<<grid, kSimtWarps * kWarp, 0, stream>>>(
            a, v, o, p.batch, p.attention_heads, p.value_heads, p.length, p.channels);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_parakeet_simt(const ParakeetProblem& p, cudaStream_t s) {
    switch (p.dtype) {
        case FGA_FLOAT: return parakeet_simt_typed<float>(p, s);
        case FGA_HALF: return parakeet_simt_typed<__half>(p, s);
        case FGA_BF16: return parakeet_simt_typed<__nv_bfloat16>(p, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_zipformer_weights_simt(const ZipformerWeightsProblem& p, cudaStream_t s) {
    switch (p.dtype) {
        case FGA_FLOAT: return zipformer_weights_simt_typed<float>(p, s);
        case FGA_HALF: return zipformer_weights_simt_typed<__half>(p, s);
        case FGA_BF16: return zipformer_weights_simt_typed<__nv_bfloat16>(p, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_zipformer_value_simt(const ZipformerValueProblem& p, cudaStream_t s) {
    switch (p.dtype) {
        case FGA_FLOAT: return zipformer_value_simt_typed<float>(p, s);
        case FGA_HALF: return zipformer_value_simt_typed<__half>(p, s);
        case FGA_BF16: return zipformer_value_simt_typed<__nv_bfloat16>(p, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace fga
