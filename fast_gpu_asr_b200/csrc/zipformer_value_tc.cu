// Zipformer attention-value on tcgen05 tensor cores (f16/bf16):
//   out[n, q, h*hd + d] = sum_k A[n, ha, q, k] * V[n, k, h*hd + d],   ha = (heads == 1 ? 0 : h)
//
// One CTA computes 128 query rows of one (utterance n, value head h) (two CTAs per SM).
// The attention rows are the dominant HBM stream. Their NHTT row stride (T*2 bytes) is
// not 16-byte aligned for the encoder's lengths, so they are read by the threads: eight
// lanes share one row's 64-key chunk, each loading two consecutive aligned 16-byte
// pieces (so one warp instruction reads four 128-byte row segments), shifting its 8 keys
// into place (rows start at any 2-byte boundary) and storing them into a K-major
// SWIZZLE_128B tile. The next chunk's loads are issued before the current chunk is
// shifted, so two chunks of loads are in flight per thread.
//
// Warps 0-7 load and repack (16 rows each); warp 8 issues the MMAs and the V loads. V
// arrives by TMA as MN-major SWIZZLE_128B tiles of 64 channels starting at the head's
// first channel rounded down to 8 (one tile for a 12-channel self-attention head,
// ceil(C/64) for the NonlinAttention value); A tiles and V tiles are double-buffered.
// The epilogue reads the fp32 accumulator from TMEM and stores the head's channels.
//
// All waits are bounded; a timeout raises the CTA's abort word, after which every warp
// skips its work but keeps its loop. Reference: zipformer_attention_value_plugin.cu:
// 118-181 (fp32 accumulation; one value head consumes attention head 0, :85).
#include <cuda.h>

#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;        // query rows per CTA
constexpr int kKc = 64;        // keys per chunk (one 128-byte swizzle atom of A)
constexpr int kLoadWarps = 8;
constexpr int kThreads = (kLoadWarps + 1) * 32;
constexpr int kMaxCpad = 512;  // TMEM columns
constexpr uint32_t kATile = kM * 128;   // 16 KB: 128 rows x 64 keys
constexpr uint32_t kVAtom = kKc * 128;  // 8 KB: 64 keys x 64 channels

__device__ unsigned int g_value_tc_error = 0;

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

struct Layout {
    uint32_t a0, v0, vstage, bar, bytes, tmem_cols;
};

__host__ __device__ constexpr uint32_t pow2_cols(uint32_t n) {
    return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512;
}

__host__ __device__ constexpr Layout make_layout(int cpad) {
    Layout l{};
    l.vstage = static_cast<uint32_t>(cpad / 64) * kVAtom;
    l.a0 = 0;
    l.v0 = 2 * kATile;
    l.bar = l.v0 + 2 * l.vstage;
    l.bytes = l.bar + 64;
    l.tmem_cols = pow2_cols(cpad);
    return l;
}

// Bounded wait with a warp-uniform result; a failure raises the CTA's abort word.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity,
                                          volatile uint32_t* abort) {
    bool ok = (*abort == 0u) && mbar_wait(bar, parity);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && (threadIdx.x & 31) == 0) {
        *abort = 1u;
        atomicExch(&g_value_tc_error, 1u);
    }
    return ok;
}

// This lane's share of one row chunk: the aligned 16-byte pieces at s and s+8 elements
// (s = aligned span start + 8m). Elements past the end of the tensor read as zero.
template <typename T>
__device__ __forceinline__ void load_piece(const T* __restrict__ att, int64_t s,
                                           int64_t att_elems, uint4 (&p)[2]) {
    if (s + 16 <= att_elems) {
        p[0] = __ldg(reinterpret_cast<const uint4*>(att + s));
        p[1] = __ldg(reinterpret_cast<const uint4*>(att + s + 8));
    } else {
        uint32_t w[8];
        const uint16_t* g = reinterpret_cast<const uint16_t*>(att);
#pragma unroll
        for (int x = 0; x < 8; ++x) {
            const uint32_t lo = s + 2 * x < att_elems ? g[s + 2 * x] : 0u;
            const uint32_t hi = s + 2 * x + 1 < att_elems ? g[s + 2 * x + 1] : 0u;
            w[x] = lo | (hi << 16);
        }
        p[0] = make_uint4(w[0], w[1], w[2], w[3]);
        p[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// Keys 8m..8m+7 of the chunk from the two pieces, shifted by a elements; keys at or past
// nk (the end of the row) are zero.
__device__ __forceinline__ uint4 shift_piece(const uint4 (&p)[2], int a, int m, int nk) {
    const uint32_t w[8] = {p[0].x, p[0].y, p[0].z, p[0].w, p[1].x, p[1].y, p[1].z, p[1].w};
    const uint32_t o = static_cast<uint32_t>(a) >> 1;
    uint32_t x[7], y[5];
#pragma unroll
    for (int k = 0; k < 7; ++k) x[k] = (o & 1u) ? w[k + 1] : w[k];
#pragma unroll
    for (int k = 0; k < 5; ++k) y[k] = (o & 2u) ? x[k + 2] : x[k];
    const uint32_t sh = (a & 1) ? 16u : 0u;
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = __funnelshift_r(y[i], y[i + 1], sh);
    if (8 * m + 8 > nk) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = 8 * m + 2 * i;
            if (k >= nk) out[i] = 0u;
            else if (k + 1 >= nk) out[i] &= 0xFFFFu;
        }
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
zipformer_value_tc_kernel(const __grid_constant__ CUtensorMap v_map, const T* __restrict__ att,
                          T* __restrict__ out, int seq, int att_heads, int value_heads,
                          int channels, int cpad, int64_t att_elems) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const Layout L = make_layout(cpad);
    const uint32_t bar_afull = sbase + L.bar;        // + 8 * buffer (count kLoadWarps)
    const uint32_t bar_aempty = sbase + L.bar + 16;  // + 8 * buffer (MMA commit)
    const uint32_t bar_vfull = sbase + L.bar + 32;   // + 8 * buffer (TMA)
    const uint32_t bar_acc = sbase + L.bar + 48;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 56);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(smem + L.bar + 60);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int nqb = (seq + kM - 1) / kM;
    const int q0 = (blockIdx.x % nqb) * kM;
    const int h = (blockIdx.x / nqb) % value_heads;
    const int n = blockIdx.x / (nqb * value_heads);
    const int hd = channels / value_heads;
    const int ha = value_heads == 1 ? 0 : h;
    const int nchunks = (seq + kKc - 1) / kKc;
    const int col0 = h * hd;
    const int col_base = col0 & ~7;

    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_value_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar_afull + 8 * b, kLoadWarps);
            mbar_init(bar_aempty + 8 * b, 1);
            mbar_init(bar_vfull + 8 * b, 1);
        }
        mbar_init(bar_acc, 1);
        *abort = 0u;
        fence_mbar_init();
        prefetch_tensormap(&v_map);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), L.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kLoadWarps) {
        // ---------------- MMA issuer and V producer ----------------
        auto load_v = [&](int c) {
            const uint32_t b = c & 1;
            mbar_expect_tx(bar_vfull + 8 * b, L.vstage);
            for (int x = 0; x < cpad / 64; ++x)
                tma_load_3d(sbase + L.v0 + b * L.vstage + x * kVAtom, &v_map, bar_vfull + 8 * b,
                            col_base + x * 64, c * kKc, n);
        };
        if (lane == 0) {
            load_v(0);
            if (nchunks > 1) load_v(1);
        }
        __syncwarp();
        const uint32_t idesc_base = idesc_f16(Fmt<T>::v, kM, 16, 0, 1);  // N patched per part
        int last_issued = -1;
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
            const uint32_t b = c & 1;
            bool ok = warp_wait(bar_afull + 8 * b, (c >> 1) & 1, abort);
            ok = ok && warp_wait(bar_vfull + 8 * b, (c >> 1) & 1, abort);
            if (ok) {
                tc_fence_after();
                if (elect_one()) {
                    const uint64_t da = sw128_desc(sbase + L.a0 + b * kATile, 16, 1024);
                    for (int part = 0; part * 256 < cpad; ++part) {
                        const int nw = min(256, cpad - part * 256);
                        const uint32_t idesc = idesc_base + ((static_cast<uint32_t>(nw) >> 3) << 17) -
                                               ((16u >> 3) << 17);
                        // V: MN-major, 64-channel atoms kVAtom bytes apart, 16 keys = 2048 B.
                        const uint64_t dv =
                            sw128_desc(sbase + L.v0 + b * L.vstage + part * 4 * kVAtom, kVAtom, 1024);
#pragma unroll
                        for (int ks = 0; ks < kKc / 16; ++ks)
                            umma_f16_ss(tmem + part * 256, da + ks * 2, dv + ks * (2048 >> 4), idesc,
                                        (c > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(bar_aempty + 8 * b);
                    if (c == nchunks - 1) umma_commit(bar_acc);
                }
                __syncwarp();
                last_issued = c;
            }
            // V buffer b is free once this MMA completes: queue chunk c+2 into it.
            if (c + 2 < nchunks && warp_wait(bar_aempty + 8 * b, (c >> 1) & 1, abort)) {
                if (lane == 0) load_v(c + 2);
                __syncwarp();
            }
        }
        // Teardown: the last issued MMA completes before TMEM is released.
        if (last_issued >= 0 &&
            !mbar_wait(bar_aempty + 8 * (last_issued & 1), (last_issued >> 1) & 1) && lane == 0)
            atomicExch(&g_value_tc_error, 1u);
    } else {
        // ---------------- loaders: 16 rows per warp, 4 rows per instruction ----------------
        const int m = lane & 7;
        int64_t ea[4];
        int shift[4];
        bool live[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int r = 16 * warp + 4 * g + (lane >> 3);
            const int q = q0 + r;
            live[g] = q < seq;
            const int64_t e =
                ((static_cast<int64_t>(n) * att_heads + ha) * seq + (live[g] ? q : 0)) * seq;
            ea[g] = e & ~static_cast<int64_t>(7);
            shift[g] = static_cast<int>(e - ea[g]);
        }
        uint4 in0[4][2], in1[4][2];
        auto load = [&](int c, uint4 (&buf)[4][2]) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                if (live[g]) {
                    load_piece<T>(att, ea[g] + c * kKc + 8 * m, att_elems, buf[g]);
                } else {
                    buf[g][0] = make_uint4(0u, 0u, 0u, 0u);
                    buf[g][1] = make_uint4(0u, 0u, 0u, 0u);
                }
            }
        };
        auto step = [&](int c, const uint4 (&buf)[4][2]) {
            const uint32_t b = c & 1;
            if (c >= 2) warp_wait(bar_aempty + 8 * b, ((c >> 1) - 1) & 1, abort);
            uint8_t* tile = smem + L.a0 + b * kATile;
            const int nk = min(kKc, seq - c * kKc);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int r = 16 * warp + 4 * g + (lane >> 3);
                const uint4 v =
                    live[g] ? shift_piece(buf[g], shift[g], m, nk) : make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(tile + sw128_offset(r, m)) = v;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_afull + 8 * b);
        };
        load(0, in0);
#pragma unroll 1
        for (int c = 0; c < nchunks; c += 2) {
            if (c + 1 < nchunks) load(c + 1, in1);
            step(c, in0);
            if (c + 1 < nchunks) {
                if (c + 2 < nchunks) load(c + 2, in0);
                step(c + 1, in1);
            }
        }
        // Epilogue: warp w reads TMEM lanes 32*(w%4).. and every other 32-column block of
        // the head's columns; only the head's hd columns are stored.
        const int qtr = warp & 3;
        const int r = qtr * 32 + lane;
        const int q = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(qtr * 32) << 16;
        const int off = col0 - col_base;
        if (warp_wait(bar_acc, 0, abort)) {
            tc_fence_after();
            T* orow = out + (static_cast<int64_t>(n) * seq + q) * channels + col0;
            const bool vec = off == 0 && channels % 8 == 0 && hd % 8 == 0;
            int blk = 0;
            for (int cb = off & ~31; cb < off + hd; cb += 32, ++blk) {
                if ((blk & 1) != (warp >> 2)) continue;
                uint32_t v[32];
                tmem_ld32(tmem + lane_off + cb, v);
                tmem_wait_ld();
                reg_fence(v);
                if (q >= seq) continue;
                if (vec && cb + 32 <= hd) {
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 o;
                        o.x = pack2<T>(__uint_as_float(v[e]), __uint_as_float(v[e + 1]));
                        o.y = pack2<T>(__uint_as_float(v[e + 2]), __uint_as_float(v[e + 3]));
                        o.z = pack2<T>(__uint_as_float(v[e + 4]), __uint_as_float(v[e + 5]));
                        o.w = pack2<T>(__uint_as_float(v[e + 6]), __uint_as_float(v[e + 7]));
                        *reinterpret_cast<uint4*>(orow + cb + e) = o;
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const int col = cb + e - off;
                        if (col >= 0 && col < hd) orow[col] = from_f32<T>(__uint_as_float(v[e]));
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, L.tmem_cols);
    }
}

// ---- host side ------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

template <typename T>
cudaError_t value_tc_typed(const ZipformerValueProblem& p, int cpad, cudaStream_t stream) {
    EncodeTiledFn encode = encode_fn();
    if (encode == nullptr) return cudaErrorNotSupported;
    const CUtensorMapDataType dt = Fmt<T>::v == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap map;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.channels),
                                static_cast<cuuint64_t>(p.length),
                                static_cast<cuuint64_t>(p.batch)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.channels) * sizeof(T),
                                   static_cast<cuuint64_t>(p.channels) * sizeof(T) * p.length};
    const cuuint32_t box[3] = {64, kKc, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode(&map, dt, 3, const_cast<void*>(p.value), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return cudaErrorNotSupported;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(zipformer_value_tc_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(make_layout(kMaxCpad).bytes));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const Layout L = make_layout(cpad);
    const int64_t att_elems =
        static_cast<int64_t>(p.batch) * p.attention_heads * p.length * p.length;
    const int64_t tiles =
        static_cast<int64_t>(p.batch) * p.value_heads * ((p.length + kM - 1) / kM);
    zipformer_value_tc_kernel<T><<<static_cast<unsigned int>(tiles), kThreads, L.bytes, stream>>>(
        map, static_cast<const T*>(p.attention), static_cast<T*>(p.output), p.length,
        p.attention_heads, p.value_heads, p.channels, cpad, att_elems);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_zipformer_value_tc(const ZipformerValueProblem& p, cudaStream_t stream) {
    if (p.dtype != FGA_HALF && p.dtype != FGA_BF16) return cudaErrorNotSupported;
    // TMA needs 16-byte V row strides.
    if (p.channels % 8 != 0 || p.value_heads < 1 || p.channels % p.value_heads != 0)
        return cudaErrorNotSupported;
    // Accumulator columns: the widest head span from its first channel rounded down to 8
    // (the offset repeats with period 8 in the head index), rounded up to 64.
    const int hd = p.channels / p.value_heads;
    int span = 0;
    for (int h = 0; h < p.value_heads && h < 8; ++h) span = max(span, ((h * hd) & 7) + hd);
    const int cpad = (span + 63) / 64 * 64;
    if (cpad > kMaxCpad) return cudaErrorNotSupported;
    if (static_cast<int64_t>(p.batch) * p.value_heads * ((p.length + kM - 1) / kM) > 0x7FFFFFFF)
        return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(p.attention) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.value) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.output) & 15u) != 0)
        return cudaErrorNotSupported;
    return p.dtype == FGA_HALF ? value_tc_typed<__half>(p, cpad, stream)
                               : value_tc_typed<__nv_bfloat16>(p, cpad, stream);
}

}  // namespace fga
