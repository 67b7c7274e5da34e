// Parakeet relative-position MHSA on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA computes a 128-query tile of one (utterance n, head h), head_dim D = 128:
//
//   S_c  = (Q+u) K_j^T                128 x 128   tcgen05.mma -> TMEM cols [0,128)
//   S_b  = (Q+v) Pband_j^T            128 x 256   tcgen05.mma -> TMEM cols [128,384)
//   logit(q,k) = scale * (S_c[q,k] + S_b[q, 127 - q + k])      (Transformer-XL shift)
//   online softmax over keys k < valid_length (fp32, exp2)
//   O   += P_j V_j                    128 x 128   tcgen05.mma -> TMEM cols [384,512)
//
// Pband_j holds the 256 rows of the positional projection that the tile's (q, k)
// pairs touch: relative index T-1-q+k ranges over [T-128-q0+k0, T-1-q0+k0+127]. Row i
// of S_b therefore needs columns 127-i .. 255-i; each warp loads the 64-column window
// its 32 rows span and every thread shifts its own row into place with a 5-stage
// predicated barrel shift (no shared-memory round trip).
//
// Reference semantics (parakeet_relative_attention_plugin.cu): biased queries are
// formed in fp32 and rounded to the I/O dtype (:268-281); scores are summed and scaled
// in fp32 (:503-508); only keys below the valid length contribute; valid_length <= 0
// gives zero rows (:478-486); every query row < T is produced (:472-476). Scores stay in
// fp32 between the two GEMMs (the reference stores them in the I/O dtype).
//
// Data movement: Q, K and V tiles arrive by TMA from the fused [N, T, 3C] projection
// through a 3-D tensor map (rows past T of an utterance read as zero), the positional
// band through a 2-D map over [2T-1, C] (rows outside the table read as zero). All
// operand tiles use the 128-byte-swizzled canonical UMMA layouts.
#include <cuda.h>

#include <cstdint>
#include <cstring>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;       // query rows per CTA
constexpr int kN = 128;       // keys per tile
constexpr int kD = 128;       // head dim
constexpr int kBand = 256;    // positional rows per tile (kM + kN - 1, rounded to 256)
constexpr int kThreads = 128;

// Shared-memory map (bytes from the 1024-aligned base).
constexpr uint32_t kAtom = kM * 128;                 // one 64-column swizzle atom of a 128-row tile
constexpr uint32_t kSmemQu = 0;                      // 2 atoms
constexpr uint32_t kSmemQv = kSmemQu + 2 * kAtom;    // 2 atoms
constexpr uint32_t kSmemK = kSmemQv + 2 * kAtom;     // 2 atoms
constexpr uint32_t kSmemV = kSmemK + 2 * kAtom;      // 2 atoms
constexpr uint32_t kBandAtom = kBand * 128;
constexpr uint32_t kSmemBand = kSmemV + 2 * kAtom;   // 2 atoms of 256 rows
constexpr uint32_t kSmemP = kSmemBand + 2 * kBandAtom;  // 2 atoms
constexpr uint32_t kSmemBar = kSmemP + 2 * kAtom;
constexpr uint32_t kSmemBytes = kSmemBar + 64 + 1024;  // + barriers + alignment slack

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSc = 0, kColSb = 128, kColO = 384;

constexpr uint32_t kTileTxBytes = 4 * kAtom + 2 * kBandAtom;  // K + V + band

__device__ unsigned int g_parakeet_tc_error = 0;

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
    return __half22float2(*reinterpret_cast<__half2*>(&w));
}
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w));
}

// out[j] = v[j + s] for j < 32, s in [0, 31]: five predicated stages (16, 8, 4, 2, 1).
__device__ __forceinline__ void barrel_shift(float (&v)[64], uint32_t s) {
#pragma unroll
    for (int j = 0; j < 47; ++j) v[j] = (s & 16u) ? v[j + 16] : v[j];
#pragma unroll
    for (int j = 0; j < 39; ++j) v[j] = (s & 8u) ? v[j + 8] : v[j];
#pragma unroll
    for (int j = 0; j < 35; ++j) v[j] = (s & 4u) ? v[j + 4] : v[j];
#pragma unroll
    for (int j = 0; j < 33; ++j) v[j] = (s & 2u) ? v[j + 2] : v[j];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (s & 1u) ? v[j + 1] : v[j];
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
parakeet_tc_kernel(const __grid_constant__ CUtensorMap qkv_map,
                   const __grid_constant__ CUtensorMap pos_map, const T* __restrict__ ubias,
                   const T* __restrict__ vbias, const int32_t* __restrict__ lengths,
                   T* __restrict__ out, int length, int heads, float scale) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_q = sbase + kSmemBar;
    const uint32_t bar_kv = bar_q + 8;
    const uint32_t bar_s = bar_q + 16;
    const uint32_t bar_o = bar_q + 24;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + 32);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int q0 = blockIdx.x * kM;
    const int h = blockIdx.y;
    const int n = blockIdx.z;
    const int C = heads * kD;
    const int valid = min(lengths[n], length);
    const int row_q = q0 + tid;
    T* orow = out + (static_cast<int64_t>(n) * length + row_q) * C + h * kD;

    if (valid <= 0) {  // no valid key: the reference defines the rows as zero
        if (row_q < length) {
            const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int c = 0; c < kD * 2 / 16; ++c) reinterpret_cast<uint4*>(orow)[c] = z;
        }
        return;
    }

    if (tid == 0) {
        mbar_init(bar_q, 1);
        mbar_init(bar_kv, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        fence_mbar_init();
        prefetch_tensormap(&qkv_map);
        prefetch_tensormap(&pos_map);
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    // Thread 0's outstanding asynchronous work, drained (bounded) on an abort.
    bool kv_pending = false, s_pending = false, o_pending = false;
    uint32_t pending_parity = 0;
    bool aborted = false;

    // ---- Q tile -> (Q+u), (Q+v) in smem -----------------------------------------------------
    if (tid == 0) {
        mbar_expect_tx(bar_q, 2 * kAtom);
        tma_load_3d(sbase + kSmemQu, &qkv_map, bar_q, h * kD, q0, n);
        tma_load_3d(sbase + kSmemQu + kAtom, &qkv_map, bar_q, h * kD + 64, q0, n);
    }
    if (__syncthreads_or(!mbar_wait(bar_q, 0))) {
        aborted = true;
    } else {
        const T* ub = ubias + h * kD;
        const T* vb = vbias + h * kD;
#pragma unroll 1
        for (int c = 0; c < 16; ++c) {
            const uint32_t off = (c >> 3) * kAtom + sw128_offset(tid, c & 7);
            const uint4 qw = *reinterpret_cast<const uint4*>(smem + kSmemQu + off);
            const uint4 uw4 = *reinterpret_cast<const uint4*>(ub + c * 8);
            const uint4 vw4 = *reinterpret_cast<const uint4*>(vb + c * 8);
            const uint32_t qs[4] = {qw.x, qw.y, qw.z, qw.w};
            const uint32_t us[4] = {uw4.x, uw4.y, uw4.z, uw4.w};
            const uint32_t vs[4] = {vw4.x, vw4.y, vw4.z, vw4.w};
            uint32_t a[4], b[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 q = unpack2<T>(qs[e]);
                const float2 u = unpack2<T>(us[e]);
                const float2 v = unpack2<T>(vs[e]);
                a[e] = pack2<T>(q.x + u.x, q.y + u.y);
                b[e] = pack2<T>(q.x + v.x, q.y + v.y);
            }
            *reinterpret_cast<uint4*>(smem + kSmemQu + off) = make_uint4(a[0], a[1], a[2], a[3]);
            *reinterpret_cast<uint4*>(smem + kSmemQv + off) = make_uint4(b[0], b[1], b[2], b[3]);
        }
        fence_proxy_async_smem();
        __syncthreads();
    }

    constexpr uint32_t idesc_s = idesc_f16(Fmt<T>::v, kM, kN, 0, 0);
    constexpr uint32_t idesc_b = idesc_f16(Fmt<T>::v, kM, kBand, 0, 0);
    constexpr uint32_t idesc_o = idesc_f16(Fmt<T>::v, kM, kD, 0, 1);

    float m_run = -INFINITY;  // running max of the scaled logits
    float l_run = 0.0f;       // running sum of exp(logit - m_run)
    const int tiles = (valid + kN - 1) / kN;
    const uint32_t shift = 31u - static_cast<uint32_t>(lane);

#pragma unroll 1
    for (int j = 0; j < tiles && !aborted; ++j) {
        const int k0 = j * kN;
        const uint32_t parity = j & 1;
        bool ok = true;
        if (tid == 0) {
            const int r0 = length - kM - q0 + k0;  // first positional row of the band
            mbar_expect_tx(bar_kv, kTileTxBytes);
            tma_load_3d(sbase + kSmemK, &qkv_map, bar_kv, C + h * kD, k0, n);
            tma_load_3d(sbase + kSmemK + kAtom, &qkv_map, bar_kv, C + h * kD + 64, k0, n);
            tma_load_3d(sbase + kSmemV, &qkv_map, bar_kv, 2 * C + h * kD, k0, n);
            tma_load_3d(sbase + kSmemV + kAtom, &qkv_map, bar_kv, 2 * C + h * kD + 64, k0, n);
            tma_load_2d(sbase + kSmemBand, &pos_map, bar_kv, h * kD, r0);
            tma_load_2d(sbase + kSmemBand + kBandAtom, &pos_map, bar_kv, h * kD + 64, r0);
            kv_pending = true;
            pending_parity = parity;
            ok = mbar_wait(bar_kv, parity);
            if (ok) {
                kv_pending = false;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < kD / 16; ++ks) {
                    const uint32_t a = ks >> 2, koff = (ks & 3) * 32;
                    const uint64_t qu = sw128_desc(sbase + kSmemQu + a * kAtom + koff, 16, 1024);
                    const uint64_t qv = sw128_desc(sbase + kSmemQv + a * kAtom + koff, 16, 1024);
                    const uint64_t kd = sw128_desc(sbase + kSmemK + a * kAtom + koff, 16, 1024);
                    const uint64_t bd =
                        sw128_desc(sbase + kSmemBand + a * kBandAtom + koff, 16, 1024);
                    umma_f16_ss(tmem + kColSc, qu, kd, idesc_s, ks > 0);
                    umma_f16_ss(tmem + kColSb, qv, bd, idesc_b, ks > 0);
                }
                umma_commit(bar_s);
                s_pending = true;
            }
        }
        if (ok) ok = mbar_wait(bar_s, parity);
        if (__syncthreads_or(!ok)) { aborted = true; break; }
        s_pending = false;
        tc_fence_after();

        // ---- logits of this thread's row over the tile's kN keys ----------------------------
        float s[kN];
#pragma unroll
        for (int c = 0; c < kN / 32; ++c) {
            uint32_t sc[32], b0[32], b1[32];
            const uint32_t base = 96u - 32u * warp + 32u * c;
            tmem_ld32(tmem + lane_off + kColSc + c * 32, sc);
            tmem_ld32(tmem + lane_off + kColSb + base, b0);
            tmem_ld32(tmem + lane_off + kColSb + base + 32, b1);
            tmem_wait_ld();
            reg_fence(sc);
            reg_fence(b0);
            reg_fence(b1);
            float band[64];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                band[e] = __uint_as_float(b0[e]);
                band[e + 32] = __uint_as_float(b1[e]);
            }
            barrel_shift(band, shift);
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const int k = k0 + c * 32 + e;
                s[c * 32 + e] = k < valid ? (__uint_as_float(sc[e]) + band[e]) * scale : -INFINITY;
            }
        }
        float m_tile = -INFINITY;
#pragma unroll
        for (int e = 0; e < kN; ++e) m_tile = fmaxf(m_tile, s[e]);
        const float m_new = fmaxf(m_run, m_tile);
        // Subtract the max before converting to base 2 so that large finite logits cannot
        // overflow (the reference softmax does the same, .cu:520-523).
        const float corr = exp2f((m_run - m_new) * kLog2e);
        float l_tile = 0.0f;
#pragma unroll
        for (int c = 0; c < kN / 8; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int k = c * 8 + 2 * e;
                const float p0 = (k0 + k < valid) ? exp2f((s[k] - m_new) * kLog2e) : 0.0f;
                const float p1 = (k0 + k + 1 < valid) ? exp2f((s[k + 1] - m_new) * kLog2e) : 0.0f;
                l_tile += p0 + p1;
                w[e] = pack2<T>(p0, p1);
            }
            const uint32_t off = (c >> 3) * kAtom + sw128_offset(tid, c & 7);
            *reinterpret_cast<uint4*>(smem + kSmemP + off) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l_run = l_run * corr + l_tile;
        m_run = m_new;

        // Rescale the running output when the max moved (not on the first tile).
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll
            for (int c = 0; c < kD / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_off + kColO + c * 32, o);
                tmem_wait_ld();
                reg_fence(o);
                float of[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) of[e] = __uint_as_float(o[e]) * corr;
                tmem_st32(tmem + lane_off + kColO + c * 32, of);
            }
            tmem_wait_st();
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        ok = true;
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < kN / 16; ++ks) {
                const uint32_t a = ks >> 2, koff = (ks & 3) * 32;
                const uint64_t pd = sw128_desc(sbase + kSmemP + a * kAtom + koff, 16, 1024);
                // V tile is MN-major (head dim contiguous): 16 keys = 2 row groups = 2048 B,
                // the two 64-channel halves are kAtom apart.
                const uint64_t vd = sw128_desc(sbase + kSmemV + ks * 2048, kAtom, 1024);
                umma_f16_ss(tmem + kColO, pd, vd, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
            }
            umma_commit(bar_o);
            o_pending = true;
        }
        ok = mbar_wait(bar_o, parity);
        if (__syncthreads_or(!ok)) { aborted = true; break; }
        o_pending = false;
        tc_fence_after();
    }

    if (aborted) {
        // Drain this CTA's own asynchronous work (bounded) before releasing TMEM.
        if (tid == 0) {
            atomicExch(&g_parakeet_tc_error, 1u);
            if (kv_pending) mbar_wait(bar_kv, pending_parity);
            if (s_pending) mbar_wait(bar_s, pending_parity);
            if (o_pending) mbar_wait(bar_o, pending_parity);
        }
    } else {
        // ---- epilogue: O / l -> output row ------------------------------------------------
        // Every thread of the warp executes the (warp-collective, .aligned) TMEM loads;
        // only rows inside the sequence are stored.
        const float inv = 1.0f / l_run;
        const bool store = row_q < length;
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_off + kColO + c * 32, o);
            tmem_wait_ld();
            reg_fence(o);
            if (!store) continue;
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
                const uint4 w = make_uint4(
                    pack2<T>(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv),
                    pack2<T>(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv),
                    pack2<T>(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv),
                    pack2<T>(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv));
                *reinterpret_cast<uint4*>(orow + c * 32 + e) = w;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
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
cudaError_t parakeet_tc_typed(const ParakeetProblem& p, cudaStream_t stream) {
    EncodeTiledFn encode = encode_fn();
    if (encode == nullptr) return cudaErrorNotSupported;
    const CUtensorMapDataType dt = Fmt<T>::v == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t C = static_cast<uint64_t>(p.heads) * kD;
    CUtensorMap qkv_map, pos_map;
    {
        const cuuint64_t dims[3] = {3 * C, static_cast<cuuint64_t>(p.length),
                                    static_cast<cuuint64_t>(p.batch)};
        const cuuint64_t strides[2] = {3 * C * sizeof(T), 3 * C * sizeof(T) * p.length};
        const cuuint32_t box[3] = {64, kM, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (encode(&qkv_map, dt, 3, const_cast<void*>(p.qkv), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return cudaErrorNotSupported;
    }
    {
        const cuuint64_t dims[2] = {C, static_cast<cuuint64_t>(2 * p.length - 1)};
        const cuuint64_t strides[1] = {C * sizeof(T)};
        const cuuint32_t box[2] = {64, kBand};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&pos_map, dt, 2, const_cast<void*>(p.position), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return cudaErrorNotSupported;
    }
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(parakeet_tc_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const dim3 grid((p.length + kM - 1) / kM, p.heads, p.batch);
    parakeet_tc_kernel<T><<<grid, kThreads, kSmemBytes, stream>>>(
        qkv_map, pos_map, static_cast<const T*>(p.content_bias),
        static_cast<const T*>(p.position_bias), p.valid_lengths, static_cast<T*>(p.output),
        p.length, p.heads, p.scale);
    return cudaGetLastError();
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

cudaError_t launch_parakeet_tc(const ParakeetProblem& p, cudaStream_t stream) {
    if (p.head_dim != kD || (p.dtype != FGA_HALF && p.dtype != FGA_BF16)) return cudaErrorNotSupported;
    if (p.batch > 65535 || p.heads > 65535) return cudaErrorNotSupported;
    if (!aligned16(p.qkv) || !aligned16(p.position) || !aligned16(p.output) ||
        !aligned16(p.content_bias) || !aligned16(p.position_bias))
        return cudaErrorNotSupported;
    return p.dtype == FGA_HALF ? parakeet_tc_typed<__half>(p, stream)
                               : parakeet_tc_typed<__nv_bfloat16>(p, stream);
}

}  // namespace fga
