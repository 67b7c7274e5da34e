// Zipformer relative-position attention weights on tcgen05 tensor cores (f16/bf16).
//
// One CTA produces the weights of 128 query rows (q0 .. q0+127) of one (utterance n,
// head h): W[n, h, q, k] for every key k < T. The content scores Q K^T (query head dim
// 32, i.e. two K=16 steps) are computed by tcgen05.mma into TMEM, 128 keys at a time,
// double-buffered (2 x 128 columns) so the next chunk's MMA runs while the threads
// consume the current one. Thread i owns row q0+i (TMEM lane i) and adds the 4-dim
// positional term sum_i pq[q,i] * pos[T-1-q+k, i] from an fp32 copy of the CTA's
// positional band in shared memory (relative rows T-1-q0-127 .. T-1-q0+T-1).
//
// Two passes over the key chunks (the QK^T MMAs are re-issued; at K = 32 they are far
// cheaper than the output write):
//   pass 1: logits -> online (max, sum) per row, masked keys excluded;
//   pass 2: logits again -> exp(logit - max) / sum -> I/O dtype -> shared staging tile,
//           then every warp writes whole row segments (coalesced, any alignment: the
//           NHTT row stride T is not a multiple of 16 bytes for the encoder's lengths).
//
// Reference semantics (zipformer_relative_attention_plugin.cu:238-327): the content
// score is stored in the I/O dtype by the reference's GEMM, so it is rounded to T here
// before the fp32 positional add; masked keys get weight 0; a row whose keys are all
// masked is zero; rows q >= 7 with mask[q-7] (the padded-query halo) are zero; a row
// whose sum is not positive (all logits -inf, or NaN) is zero.
#include <cuda.h>

#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;        // query rows per CTA
constexpr int kChunk = 128;    // keys per MMA chunk
constexpr int kQd = 32;        // query/key head dim served by this kernel
constexpr int kMaxT = 768;     // keys held in shared memory (K tile rows)
constexpr int kThreads = 128;
constexpr int kHalo = 7;

// Shared memory (bytes from the 1024-aligned base).
constexpr uint32_t kRowBytes = kQd * 2;                   // 64 B rows, 64-byte swizzle
constexpr uint32_t kSmemQ = 0;                            // 128 rows
constexpr uint32_t kSmemK = kSmemQ + kM * kRowBytes;      // up to kMaxT rows
constexpr uint32_t kSmemStage = kSmemK + kMaxT * kRowBytes;  // [128 rows][128 keys] T
constexpr uint32_t kStageRowBytes = kChunk * 2;
constexpr uint32_t kSmemPos = kSmemStage + kM * kStageRowBytes;  // fp32x4 band rows
constexpr uint32_t kMaxBandRows = kMaxT + kM;
constexpr uint32_t kSmemMask = kSmemPos + kMaxBandRows * 16;     // valid-key bits
constexpr uint32_t kSmemBar = kSmemMask + kMaxT / 8;
constexpr uint32_t kSmemBytes = kSmemBar + 64;

constexpr uint32_t kTmemCols = 256;

__device__ unsigned int g_zipformer_tc_error = 0;

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// SWIZZLE_64B K-major descriptor: 64-byte rows, 8-row groups of 512 bytes.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;                   // LBO (unused for swizzled K-major)
    d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;  // SBO: 8 rows x 64 B
    d |= 1ull << 46;
    d |= 4ull << 61;                                        // SWIZZLE_64B
    return d;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
zipformer_weights_tc_kernel(const __grid_constant__ CUtensorMap proj_map,
                            const T* __restrict__ proj, const T* __restrict__ pos,
                            const uint8_t* __restrict__ mask, T* __restrict__ out, int length,
                            int heads) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_load = sbase + kSmemBar;
    const uint32_t bar_mma0 = sbase + kSmemBar + 8;  // + 8 * buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + 24);
    float4* pos_band = reinterpret_cast<float4*>(smem + kSmemPos);
    uint32_t* valid_bits = reinterpret_cast<uint32_t*>(smem + kSmemMask);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int q0 = blockIdx.x * kM;
    const int h = blockIdx.y;
    const int n = blockIdx.z;
    const int seq = length;
    const int pdim = heads * (2 * kQd + 4);
    const int nchunks = (seq + kChunk - 1) / kChunk;
    const int band_lo = seq - 1 - q0 - (kM - 1);  // relative row of band entry 0
    const int band_rows = seq + kM - 1;
    const int q = q0 + tid;
    const uint8_t* mrow = mask + static_cast<int64_t>(n) * seq;

    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_zipformer_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        mbar_init(bar_load, 1);
        mbar_init(bar_mma0, 1);
        mbar_init(bar_mma0 + 8, 1);
        fence_mbar_init();
        prefetch_tensormap(&proj_map);
        // Q rows q0.. (head h), then all K rows of head h. Rows past T read as zero.
        mbar_expect_tx(bar_load, (kM + nchunks * kChunk) * kRowBytes);
        tma_load_3d(sbase + kSmemQ, &proj_map, bar_load, h * kQd, q0, n);
        for (int c = 0; c < nchunks; ++c)
            tma_load_3d(sbase + kSmemK + c * kChunk * kRowBytes, &proj_map, bar_load,
                        heads * kQd + h * kQd, c * kChunk, n);
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    // Positional band (fp32) and valid-key bits, while the TMA runs.
    for (int r = tid; r < band_rows; r += kThreads) {
        const int rel = band_lo + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rel >= 0 && rel < 2 * seq - 1) {
            const T* pr = pos + (static_cast<int64_t>(rel) * heads + h) * 4;
            v = make_float4(to_f32<T>(pr[0]), to_f32<T>(pr[1]), to_f32<T>(pr[2]),
                            to_f32<T>(pr[3]));
        }
        pos_band[r] = v;
    }
    for (int w = tid; w < (nchunks * kChunk) / 32; w += kThreads) {
        uint32_t bits = 0;
        for (int b = 0; b < 32; ++b) {
            const int k = w * 32 + b;
            if (k < seq && !mrow[k]) bits |= 1u << b;
        }
        valid_bits[w] = bits;
    }
    // This row's positional query and halo state.
    float pq0 = 0.f, pq1 = 0.f, pq2 = 0.f, pq3 = 0.f;
    bool row_live = q < seq;
    if (row_live) {
        const T* pr = proj + (static_cast<int64_t>(n) * seq + q) * pdim + 2 * heads * kQd + h * 4;
        pq0 = to_f32<T>(pr[0]);
        pq1 = to_f32<T>(pr[1]);
        pq2 = to_f32<T>(pr[2]);
        pq3 = to_f32<T>(pr[3]);
        if (q >= kHalo && mrow[q - kHalo]) row_live = false;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const bool loaded = mbar_wait(bar_load, 0);
    bool ok = !__syncthreads_or(!loaded);

    constexpr uint32_t idesc = idesc_f16(Fmt<T>::v, kM, kChunk, 0, 0);
    const uint64_t dq = sw64_desc(sbase + kSmemQ);
    auto issue = [&](int it) {  // MMA for pass-iteration it into buffer it % 2
        const int c = it % nchunks;
        const uint64_t dk = sw64_desc(sbase + kSmemK + c * kChunk * kRowBytes);
        const uint32_t d = tmem + (it & 1) * kChunk;
        umma_f16_ss(d, dq, dk, idesc, 0);
        umma_f16_ss(d, dq + 2, dk + 2, idesc, 1);  // second K=16 step: +32 bytes
        umma_commit(bar_mma0 + 8 * (it & 1));
    };
    if (ok && warp == 0) {
        tc_fence_after();
        if (elect_one()) issue(0);
        __syncwarp();
    }

    float m_run = -INFINITY, l_run = 0.0f, inv = 0.0f;
    const int iters = 2 * nchunks;
    const int prow = (kM - 1) - tid;  // band entry of key 0 for this row: seq-1-q - band_lo
#pragma unroll 1
    for (int it = 0; it < iters && ok; ++it) {
        const int c = it % nchunks;
        const bool pass2 = it >= nchunks;
        const int k0 = c * kChunk;
        // Buffer (it+1)%2 was last read at it-1: every thread has passed that point.
        tc_fence_before();
        __syncthreads();
        if (it + 1 < iters && warp == 0) {
            tc_fence_after();
            if (elect_one()) issue(it + 1);
            __syncwarp();
        }
        // A row whose sum is not positive (no valid key, all -inf, or NaN) is zero, as in
        // the reference (sum > 0 ? v / sum : 0).
        if (pass2 && c == 0) inv = (l_run > 0.0f) ? 1.0f / l_run : 0.0f;
        if (!mbar_wait(bar_mma0 + 8 * (it & 1), (it >> 1) & 1)) {
            atomicExch(&g_zipformer_tc_error, 1u);
            ok = false;
        }
        if (__syncthreads_or(!ok)) {
            ok = false;
            break;
        }
        tc_fence_after();
        const uint32_t buf = tmem + lane_off + (it & 1) * kChunk;
        uint8_t* srow = smem + kSmemStage + tid * kStageRowBytes;
        float m_chunk = -INFINITY;
        float s[32];
#pragma unroll 1
        for (int sub = 0; sub < kChunk / 32; ++sub) {
            const uint32_t vbits = valid_bits[(k0 >> 5) + sub];
            // Skip decisions are warp-uniform: tcgen05.ld is a warp-collective instruction.
            const bool lane_any = row_live && vbits != 0u && (!pass2 || inv > 0.0f);
            if (!__any_sync(0xffffffffu, lane_any)) {
                if (pass2) {  // fully masked group or dead rows: zeros
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        const uint32_t chunk = (sub * 4 + (e >> 3)) ^ (tid & 15);
                        *reinterpret_cast<uint4*>(srow + chunk * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                continue;
            }
            uint32_t r[32];
            tmem_ld32(buf + sub * 32, r);
            tmem_wait_ld();
            reg_fence(r);
            const float4* pb = pos_band + prow + k0 + sub * 32;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const float4 p = pb[e];
                float v = round_to<T>(__uint_as_float(r[e]));
                v = fmaf(pq0, p.x, v);
                v = fmaf(pq1, p.y, v);
                v = fmaf(pq2, p.z, v);
                v = fmaf(pq3, p.w, v);
                const bool valid = lane_any && ((vbits >> e) & 1u);
                s[e] = valid ? v : -INFINITY;
            }
            if (!pass2) {
                float mm = -INFINITY;
#pragma unroll
                for (int e = 0; e < 32; ++e) mm = fmaxf(mm, s[e]);
                const float m_new = fmaxf(m_run, mm);
                if (m_new != -INFINITY) {
                    const float mb = m_new * kLog2e;
                    float acc = 0.0f;
#pragma unroll
                    for (int e = 0; e < 32; ++e) acc += fast_exp2(fmaf(s[e], kLog2e, -mb));
                    l_run = l_run * fast_exp2(fmaf(m_run, kLog2e, -mb)) + acc;
                    m_run = m_new;
                }
                (void)m_chunk;
            } else {
                const float mb = m_run * kLog2e;
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                    uint32_t w[4];
#pragma unroll
                    for (int x = 0; x < 4; ++x) {
                        const float a = s[e + 2 * x] == -INFINITY
                                            ? 0.0f
                                            : fast_exp2(fmaf(s[e + 2 * x], kLog2e, -mb)) * inv;
                        const float b = s[e + 2 * x + 1] == -INFINITY
                                            ? 0.0f
                                            : fast_exp2(fmaf(s[e + 2 * x + 1], kLog2e, -mb)) * inv;
                        const T ta = from_f32<T>(a), tb = from_f32<T>(b);
                        w[x] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&ta)) |
                               (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&tb)) << 16);
                    }
                    // 16-byte chunk (sub*4 + e/8) of this row, XOR-swizzled by row.
                    const uint32_t chunk = (sub * 4 + (e >> 3)) ^ (tid & 15);
                    *reinterpret_cast<uint4*>(srow + chunk * 16) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
        if (pass2) {
            // Staging tile complete: write whole row segments, coalesced.
            __syncthreads();
            const int width = min(kChunk, seq - k0);
            const int rows = min(kM, seq - q0);
            T* obase = out + ((static_cast<int64_t>(n) * heads + h) * seq + q0) * seq + k0;
#pragma unroll 1
            for (int rr = warp; rr < rows; rr += kThreads / 32) {
                const uint8_t* src = smem + kSmemStage + rr * kStageRowBytes;
                T* dst = obase + static_cast<int64_t>(rr) * seq;
                for (int k = lane; k < width; k += 32) {
                    const uint32_t chunk = (k >> 3) ^ (rr & 15);
                    dst[k] = *reinterpret_cast<const T*>(src + chunk * 16 + (k & 7) * 2);
                }
            }
        }
    }
    // Drain: the last issued MMA is waited on in the loop; on an abort wait (bounded)
    // for any outstanding one before releasing TMEM.
    if (!ok && warp == 0 && elect_one()) {
        mbar_wait(bar_mma0, 0);
        mbar_wait(bar_mma0 + 8, 0);
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
cudaError_t weights_tc_typed(const ZipformerWeightsProblem& p, cudaStream_t stream) {
    EncodeTiledFn encode = encode_fn();
    if (encode == nullptr) return cudaErrorNotSupported;
    const CUtensorMapDataType dt = Fmt<T>::v == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t pdim = static_cast<uint64_t>(p.heads) * (2 * kQd + 4);
    CUtensorMap map;
    const cuuint64_t dims[3] = {pdim, static_cast<cuuint64_t>(p.length),
                                static_cast<cuuint64_t>(p.batch)};
    const cuuint64_t strides[2] = {pdim * sizeof(T), pdim * sizeof(T) * p.length};
    const cuuint32_t box[3] = {kQd, kChunk, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode(&map, dt, 3, const_cast<void*>(p.projection), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return cudaErrorNotSupported;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(zipformer_weights_tc_kernel<T>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const dim3 grid((p.length + kM - 1) / kM, p.heads, p.batch);
    zipformer_weights_tc_kernel<T><<<grid, kThreads, kSmemBytes, stream>>>(
        map, static_cast<const T*>(p.projection), static_cast<const T*>(p.position), p.mask,
        static_cast<T*>(p.weights), p.length, p.heads);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_zipformer_weights_tc(const ZipformerWeightsProblem& p, cudaStream_t stream) {
    if (p.query_dim != kQd || (p.dtype != FGA_HALF && p.dtype != FGA_BF16))
        return cudaErrorNotSupported;
    if (p.length > kMaxT || p.batch > 65535 || p.heads > 65535) return cudaErrorNotSupported;
    // TMA needs 16-byte row strides: H * (2*32+4) * 2 bytes = 136 H.
    const int64_t row_bytes = static_cast<int64_t>(p.heads) * (2 * kQd + 4) * 2;
    if (row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(p.projection) & 15u) != 0)
        return cudaErrorNotSupported;
    return p.dtype == FGA_HALF ? weights_tc_typed<__half>(p, stream)
                               : weights_tc_typed<__nv_bfloat16>(p, stream);
}

}  // namespace fga
