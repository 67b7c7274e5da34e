// Zipformer attention-value on tcgen05 tensor cores (f16/bf16):
//   out[n, q, h*hd + d] = sum_k A[n, ha, q, k] * V[n, k, h*hd + d],   ha = (heads == 1 ? 0 : h)
//
// One CTA computes 128 query rows of one (utterance n, value head h). The attention
// rows are the dominant HBM stream. They cannot be fetched by TMA: the NHTT row stride T
// is not a multiple of 16 bytes for the encoder's lengths. So every thread streams its own
// row with aligned 16-byte loads, shifts it into place (rows start at any 2-byte
// boundary) and writes it into a K-major SWIZZLE_128B tile (64 keys per chunk). V arrives
// by TMA as an MN-major SWIZZLE_128B tile holding *all* C channels of the chunk's keys,
// zero-padded to a multiple of 64; the MMA computes all C_pad output columns into TMEM
// and the epilogue keeps the head's hd columns. At 4-12 MACs per attention element the
// MMA is far from the limit; the extra columns cost nothing measurable.
//
// Both A and V tiles are double-buffered: chunk c+1 is loaded while the MMA of chunk c
// runs. Reference: zipformer_attention_value_plugin.cu:118-181 (fp32 accumulation; one
// value head consumes attention head 0, :85).
#include <cuda.h>

#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;       // query rows per CTA
constexpr int kKc = 64;       // keys per chunk (one 128-byte swizzle atom of A)
constexpr int kThreads = 128;
constexpr int kMaxCpad = 512;  // TMEM columns

constexpr uint32_t kATile = kM * 128;        // 16 KB: 128 rows x 64 keys
constexpr uint32_t kVAtom = kKc * 128;       // 8 KB: 64 keys x 64 channels

__device__ unsigned int g_value_tc_error = 0;

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

struct Layout {
    uint32_t a0, v0, bar, bytes, vtile;
};

__host__ __device__ constexpr Layout make_layout(int cpad) {
    Layout l{};
    l.vtile = static_cast<uint32_t>(cpad / 64) * kVAtom;
    l.a0 = 0;
    l.v0 = 2 * kATile;
    l.bar = l.v0 + 2 * l.vtile;
    l.bytes = l.bar + 64;
    return l;
}

// Copy this thread's 64 attention values [e, e+64) (element offset e into the flat
// attention tensor, any 2-byte alignment) into row `row` of the K-major swizzled tile.
// Elements at or beyond `limit` (end of the row's valid keys) are zero.
template <typename T>
__device__ __forceinline__ void stage_row(uint8_t* tile, int row, const T* __restrict__ base,
                                         int64_t e, int nkeys) {
    const int a = static_cast<int>(e & 7);  // misalignment in elements
    const uint4* src = reinterpret_cast<const uint4*>(base + (e - a));
    uint32_t w[36];
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        // The 9th vector is only needed when the row is misaligned.
        const uint4 v = (i < 8 || a != 0) ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
    }
    // Shift by a elements: whole words (a >> 1) with a predicated barrel, then half a
    // word with a funnel shift.
    const uint32_t sw = static_cast<uint32_t>(a) >> 1;
#pragma unroll
    for (int i = 0; i < 34; ++i) w[i] = (sw & 2u) ? w[i + 2] : w[i];
#pragma unroll
    for (int i = 0; i < 33; ++i) w[i] = (sw & 1u) ? w[i + 1] : w[i];
    const uint32_t sh = (a & 1) ? 16u : 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = __funnelshift_r(w[i], w[i + 1], sh);
    // Zero keys beyond the row's end (last chunk).
    if (nkeys < kKc) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int k = 2 * i;
            if (k >= nkeys) w[i] = 0u;
            else if (k + 1 >= nkeys) w[i] &= 0xFFFFu;
        }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(tile + sw128_offset(row, c)) =
            make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
zipformer_value_tc_kernel(const __grid_constant__ CUtensorMap v_map, const T* __restrict__ att,
                          T* __restrict__ out, int length, int att_heads, int value_heads,
                          int channels, int cpad, int64_t att_elems) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const Layout L = make_layout(cpad);
    const uint32_t bar_v0 = sbase + L.bar;        // + 8 * buffer: V tile loaded
    const uint32_t bar_mma0 = sbase + L.bar + 16;  // + 8 * buffer: MMA of that buffer done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 32);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int q0 = blockIdx.x * kM;
    const int h = blockIdx.y;
    const int n = blockIdx.z;
    const int seq = length;
    const int hd = channels / value_heads;
    const int ha = value_heads == 1 ? 0 : h;
    const int q = q0 + tid;
    const int nchunks = (seq + kKc - 1) / kKc;
    const uint32_t tcols = cpad <= 64 ? 64 : cpad <= 128 ? 128 : cpad <= 256 ? 256 : 512;

    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_value_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        mbar_init(bar_v0, 1);
        mbar_init(bar_v0 + 8, 1);
        mbar_init(bar_mma0, 1);
        mbar_init(bar_mma0 + 8, 1);
        fence_mbar_init();
        prefetch_tensormap(&v_map);
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), tcols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto load_v = [&](int c) {  // V chunk c -> buffer c & 1 (all channels, zero-padded)
        const uint32_t b = c & 1;
        mbar_expect_tx(bar_v0 + 8 * b, L.vtile);
        for (int x = 0; x < cpad / 64; ++x)
            tma_load_3d(sbase + L.v0 + b * L.vtile + x * kVAtom, &v_map, bar_v0 + 8 * b, x * 64,
                        c * kKc, n);
    };
    if (tid == 0) {
        load_v(0);
        if (nchunks > 1) load_v(1);
    }
    // Row q of this CTA: element offset of A[n, ha, q, 0].
    const int64_t row_e = ((static_cast<int64_t>(n) * att_heads + ha) * seq + q) * seq;
    const bool row_live = q < seq;
    const T* arow_base = att;
    const uint32_t idesc_base = idesc_f16(Fmt<T>::v, kM, 16, 0, 1);  // N patched per part
    bool ok = true;

#pragma unroll 1
    for (int c = 0; c < nchunks && ok; ++c) {
        const uint32_t b = c & 1;
        // A buffer b was last read by the MMA of chunk c-2.
        if (c >= 2 && !mbar_wait(bar_mma0 + 8 * b, ((c - 2) >> 1) & 1)) ok = false;
        if (__syncthreads_or(!ok)) { ok = false; break; }
        uint8_t* tile = smem + L.a0 + b * kATile;
        const int k0 = c * kKc;
        const int nk = min(kKc, seq - k0);
        if (row_live) {
            // Stay inside the tensor: the last row's tail must not read past its end.
            const int64_t e = row_e + k0;
            const int a = static_cast<int>(e & 7);
            if (e - a + 72 <= att_elems) {
                stage_row<T>(tile, tid, arow_base, e, nk);
            } else {
                for (int cc = 0; cc < 8; ++cc) {
                    uint32_t w[4];
                    for (int x = 0; x < 4; ++x) {
                        const int k = cc * 8 + 2 * x;
                        const T lo = k < nk ? att[e + k] : from_f32<T>(0.f);
                        const T hi = k + 1 < nk ? att[e + k + 1] : from_f32<T>(0.f);
                        w[x] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
                               (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
                    }
                    *reinterpret_cast<uint4*>(tile + sw128_offset(tid, cc)) =
                        make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        } else {
#pragma unroll
            for (int cc = 0; cc < 8; ++cc)
                *reinterpret_cast<uint4*>(tile + sw128_offset(tid, cc)) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            bool vok = mbar_wait(bar_v0 + 8 * b, (c >> 1) & 1);
            vok = __all_sync(0xffffffffu, vok);
            if (!vok) {
                ok = false;
            } else {
                tc_fence_after();
                if (elect_one()) {
                    const uint64_t da = sw128_desc(sbase + L.a0 + b * kATile, 16, 1024);
                    for (int part = 0; part * 256 < cpad; ++part) {
                        const int nw = min(256, cpad - part * 256);
                        const uint32_t idesc = idesc_base + ((static_cast<uint32_t>(nw) >> 3) << 17) -
                                               ((16u >> 3) << 17);
                        // V: MN-major, 64-channel atoms kKc*128 bytes apart, 16 keys = 2048 B.
                        const uint64_t dv = sw128_desc(
                            sbase + L.v0 + b * L.vtile + part * 4 * kVAtom, kVAtom, 1024);
#pragma unroll
                        for (int ks = 0; ks < kKc / 16; ++ks)
                            umma_f16_ss(tmem + part * 256, da + ks * 2, dv + ks * (2048 >> 4),
                                        idesc, (c > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(bar_mma0 + 8 * b);
                    // V buffer b is free once this MMA completes: queue chunk c+2 into it.
                    if (c + 2 < nchunks) {
                        mbar_wait(bar_mma0 + 8 * b, (c >> 1) & 1);
                        load_v(c + 2);
                    }
                }
                __syncwarp();
            }
        }
    }
    // Epilogue: wait for the last MMA, then keep this head's hd columns.
    const int last = nchunks - 1;
    bool done = ok && mbar_wait(bar_mma0 + 8 * (last & 1), (last >> 1) & 1);
    done = !__syncthreads_or(!done);
    if (!done) {
        if (tid == 0) atomicExch(&g_value_tc_error, 1u);
    } else {
        tc_fence_after();
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        T* orow = out + (static_cast<int64_t>(n) * seq + q) * channels + h * hd;
        const int col0 = h * hd;  // first output column of this head in the C_pad block
        for (int cb = (col0 / 32) * 32; cb < col0 + hd; cb += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + lane_off + cb, r);
            tmem_wait_ld();
            reg_fence(r);
            if (!row_live) continue;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const int col = cb + e;
                if (col >= col0 && col < col0 + hd) orow[col - col0] = from_f32<T>(__uint_as_float(r[e]));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, tcols);
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
    const Layout L = make_layout(cpad);
    static int attr_bytes = 0;
    if (attr_bytes < static_cast<int>(L.bytes)) {
        cudaError_t e = cudaFuncSetAttribute(zipformer_value_tc_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(make_layout(kMaxCpad).bytes));
        if (e != cudaSuccess) return e;
        attr_bytes = static_cast<int>(make_layout(kMaxCpad).bytes);
    }
    const int64_t att_elems =
        static_cast<int64_t>(p.batch) * p.attention_heads * p.length * p.length;
    const dim3 grid((p.length + kM - 1) / kM, p.value_heads, p.batch);
    zipformer_value_tc_kernel<T><<<grid, kThreads, L.bytes, stream>>>(
        map, static_cast<const T*>(p.attention), static_cast<T*>(p.output), p.length,
        p.attention_heads, p.value_heads, p.channels, cpad, att_elems);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_zipformer_value_tc(const ZipformerValueProblem& p, cudaStream_t stream) {
    if (p.dtype != FGA_HALF && p.dtype != FGA_BF16) return cudaErrorNotSupported;
    // TMA needs 16-byte V row strides; TMEM holds at most 512 fp32 columns.
    if (p.channels % 8 != 0 || p.channels > kMaxCpad) return cudaErrorNotSupported;
    if (p.batch > 65535 || p.value_heads > 65535) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(p.attention) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.value) & 15u) != 0)
        return cudaErrorNotSupported;
    const int cpad = (p.channels + 63) / 64 * 64;
    return p.dtype == FGA_HALF ? value_tc_typed<__half>(p, cpad, stream)
                               : value_tc_typed<__nv_bfloat16>(p, cpad, stream);
}

}  // namespace fga
