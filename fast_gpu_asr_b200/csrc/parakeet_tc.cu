// Parakeet relative-position MHSA on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Work item = one 128-query tile of one (utterance n, head h), head_dim D = 128. For
// each 128-key tile j of the utterance's valid keys:
//
//   S_c  = (Q+u) K_j^T                128 x 128   tcgen05.mma -> TMEM cols [0,128)
//   S_b  = (Q+v) Pband_j^T            128 x 256   tcgen05.mma -> TMEM cols [128,384)
//   logit(q,k) = scale * (S_c[q,k] + S_b[q, 127 - q + k])      (Transformer-XL shift)
//   online softmax over keys k < valid_length (fp32, base 2)
//   O   += P_j V_j                    128 x 128   tcgen05.mma -> TMEM cols [384,512)
//
// Pband_j holds the 256 rows of the positional projection that the tile's (q, k) pairs
// touch: relative index T-1-q+k ranges over [T-128-q0+k0, T-1-q0+k0+127], so row i of
// S_b needs columns 127-i .. 255-i. A warp loads the 64-column window its 32 rows span
// and every thread shifts its own row into place with a 5-stage predicated barrel shift.
//
// CTA organisation (persistent: one CTA per SM walks the work items):
//   warps 0-7  softmax. Warp w owns TMEM lanes 32*(w%4).. (rows) and key half w/4
//              (64 keys of each tile); the two warps of a row group exchange the row
//              max through shared memory behind a 64-thread named barrier.
//   warp 8     TMA producer: lane 0 loads Q and K + positional band, lane 1 loads V.
//   warp 9     MMA issuer (one thread) and TMEM owner.
// The next tile's score MMAs are issued as soon as the softmax warps have copied the
// current scores to registers, so S(j+1) overlaps the exponentials of tile j. O is
// rescaled only when a row max grows by more than 2^8 (the unnormalised probabilities
// stay <= 256, exact in f16/bf16 range).
//
// Reference semantics (parakeet_relative_attention_plugin.cu): biased queries are
// formed in fp32 and rounded to the I/O dtype (:268-281); scores are summed and scaled
// in fp32 (:503-508); only keys below the valid length contribute; valid_length <= 0
// gives zero rows (:478-486); every query row < T is produced (:472-476). Scores stay
// in fp32 between the two GEMMs (the reference stores them in the I/O dtype). The log2(e)
// factor is folded into the scale, so this kernel serves scale <= 1 (every real model:
// 1/sqrt(D)); larger scales run on the SIMT kernel, which subtracts the row max before
// converting to base 2 exactly like the reference.
//
// Data movement: Q, K and V tiles arrive by TMA from the fused [N, T, 3C] projection
// through a 3-D tensor map (rows past T of an utterance read as zero), the positional
// band through a 2-D map over [2T-1, C] (rows outside the table read as zero). All
// operand tiles use the 128-byte-swizzled canonical UMMA layouts.
#include <cuda.h>

#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;       // query rows per work item
constexpr int kN = 128;       // keys per tile
constexpr int kD = 128;       // head dim
constexpr int kBand = 256;    // positional rows per tile (kM + kN - 1, rounded to 256)
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kHalfKeys = kN / 2;

// Shared-memory map (bytes from the 1024-aligned dynamic base).
constexpr uint32_t kAtom = kM * 128;                 // one 64-column swizzle atom of a 128-row tile
constexpr uint32_t kSmemQu = 0;                      // 2 atoms (TMA lands Q here first)
constexpr uint32_t kSmemQv = kSmemQu + 2 * kAtom;    // 2 atoms
constexpr uint32_t kSmemK = kSmemQv + 2 * kAtom;     // 2 atoms
constexpr uint32_t kSmemV = kSmemK + 2 * kAtom;      // 2 atoms
constexpr uint32_t kBandAtom = kBand * 128;
constexpr uint32_t kSmemBand = kSmemV + 2 * kAtom;   // 2 atoms of 256 rows
constexpr uint32_t kSmemP = kSmemBand + 2 * kBandAtom;  // 2 atoms
constexpr uint32_t kSmemXchg = kSmemP + 2 * kAtom;   // [2 halves][128 rows] fp32
constexpr uint32_t kSmemBar = kSmemXchg + 2 * kM * 4;
constexpr uint32_t kNumBars = 13;
constexpr uint32_t kSmemBytes = kSmemBar + kNumBars * 8 + 16;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSc = 0, kColSb = 128, kColO = 384;

constexpr uint32_t kKBandTxBytes = 2 * kAtom + 2 * kBandAtom;
constexpr uint32_t kVTxBytes = 2 * kAtom;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

enum : uint32_t {
    kBarQFull = 0, kBarQReady, kBarQEmpty, kBarKBFull, kBarKBEmpty, kBarVFull, kBarVEmpty,
    kBarSFull, kBarSFree, kBarPFull, kBarODone, kBarOFree, kBarDrain
};

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

// 2^x on the MUFU unit (ex2.approx, relative error ~2^-22; -inf -> 0).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
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

struct Item {
    int n, h, q0, valid, tiles;
};

__device__ __forceinline__ Item decode_item(int item, int qtiles, int heads, int length,
                                            const int32_t* __restrict__ lengths) {
    Item it;
    const int qt = item % qtiles;
    const int nh = item / qtiles;
    it.h = nh % heads;
    it.n = nh / heads;
    it.q0 = qt * kM;
    it.valid = min(lengths[it.n], length);
    it.tiles = it.valid > 0 ? (it.valid + kN - 1) / kN : 0;
    return it;
}

// mbarrier waits with a shared abort word: once any role gives up on a wait (time
// limit), every other role stops waiting and the CTA tears down.
struct Sync {
    uint32_t bars;
    volatile int* abort;
    __device__ __forceinline__ uint32_t bar(uint32_t i) const { return bars + 8 * i; }
    __device__ __forceinline__ bool wait(uint32_t i, uint32_t parity) const {
        if (mbar_try_wait(bar(i), parity)) return true;
        const uint64_t start = global_timer_ns();
        while (!mbar_try_wait(bar(i), parity)) {
            if (*abort) return false;
            if (global_timer_ns() - start > kWaitLimitNs) {
                *abort = 1;
                atomicExch(&g_parakeet_tc_error, 1u);
                return false;
            }
        }
        return true;
    }
    // Warp-uniform wait (all lanes agree before any warp-collective instruction).
    __device__ __forceinline__ bool wait_warp(uint32_t i, uint32_t parity) const {
        const bool ok = wait(i, parity);
        return __all_sync(0xffffffffu, ok);
    }
};

// Scaled base-2 logits of this thread's 64 keys of the tile (two 32-key chunks).
template <bool kMasked>
__device__ __forceinline__ void load_logits(float (&s)[kHalfKeys], uint32_t tmem_row,
                                            int group, int half, uint32_t shift,
                                            float scale_log2, int nvalid) {
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;  // 32-key chunk of the tile
        uint32_t sc[32], b0[32], b1[32];
        const uint32_t base = 96u - 32u * group + 32u * c;
        tmem_ld32(tmem_row + kColSc + c * 32, sc);
        tmem_ld32(tmem_row + kColSb + base, b0);
        tmem_ld32(tmem_row + kColSb + base + 32, b1);
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
            const float v = (__uint_as_float(sc[e]) + band[e]) * scale_log2;
            s[cc * 32 + e] = (!kMasked || c * 32 + e < nvalid) ? v : -INFINITY;
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
parakeet_tc_kernel(const __grid_constant__ CUtensorMap qkv_map,
                   const __grid_constant__ CUtensorMap pos_map, const T* __restrict__ ubias,
                   const T* __restrict__ vbias, const int32_t* __restrict__ lengths,
                   T* __restrict__ out, int batch, int length, int heads, float scale_log2) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + kNumBars * 8);
    int* abort_word = reinterpret_cast<int*>(smem + kSmemBar + kNumBars * 8 + 4);
    float* xchg = reinterpret_cast<float*>(smem + kSmemXchg);
    const Sync sync{sbase + kSmemBar, abort_word};

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int C = heads * kD;
    const int qtiles = (length + kM - 1) / kM;
    const int num_items = qtiles * heads * batch;

    // The swizzled layouts need a 1024-byte aligned base; report and stop otherwise.
    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_parakeet_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        const uint32_t counts[kNumBars] = {1, kSoftmaxWarps, 1, 1, 1, 1, 1, 1, kSoftmaxWarps,
                                           kSoftmaxWarps, 1, kSoftmaxWarps, 1};
        for (uint32_t i = 0; i < kNumBars; ++i) mbar_init(sync.bar(i), counts[i]);
        *abort_word = 0;
        fence_mbar_init();
        prefetch_tensormap(&qkv_map);
        prefetch_tensormap(&pos_map);
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kProducerWarp) {
        // ---- TMA producer: lane 0 loads Q and K+band, lane 1 loads V ------------------------
        if (lane == 0) {
            uint32_t q_iter = 0, kb_iter = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
                const Item it = decode_item(item, qtiles, heads, length, lengths);
                if (it.tiles == 0) continue;
                if (q_iter > 0 && !(ok = sync.wait(kBarQEmpty, (q_iter - 1) & 1))) break;
                mbar_expect_tx(sync.bar(kBarQFull), 2 * kAtom);
                tma_load_3d(sbase + kSmemQu, &qkv_map, sync.bar(kBarQFull), it.h * kD, it.q0, it.n);
                tma_load_3d(sbase + kSmemQu + kAtom, &qkv_map, sync.bar(kBarQFull),
                            it.h * kD + 64, it.q0, it.n);
                ++q_iter;
                for (int j = 0; j < it.tiles; ++j) {
                    if (kb_iter > 0 && !(ok = sync.wait(kBarKBEmpty, (kb_iter - 1) & 1))) break;
                    const int k0 = j * kN;
                    const int r0 = length - kM - it.q0 + k0;  // first positional row of the band
                    const uint32_t b = sync.bar(kBarKBFull);
                    mbar_expect_tx(b, kKBandTxBytes);
                    tma_load_3d(sbase + kSmemK, &qkv_map, b, C + it.h * kD, k0, it.n);
                    tma_load_3d(sbase + kSmemK + kAtom, &qkv_map, b, C + it.h * kD + 64, k0, it.n);
                    tma_load_2d(sbase + kSmemBand, &pos_map, b, it.h * kD, r0);
                    tma_load_2d(sbase + kSmemBand + kBandAtom, &pos_map, b, it.h * kD + 64, r0);
                    ++kb_iter;
                }
            }
            if (!ok) {  // drain our own copies in flight (bounded) before teardown
                if (q_iter) mbar_wait(sync.bar(kBarQFull), (q_iter - 1) & 1);
                if (kb_iter) mbar_wait(sync.bar(kBarKBFull), (kb_iter - 1) & 1);
            }
        } else if (lane == 1) {
            uint32_t v_iter = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
                const Item it = decode_item(item, qtiles, heads, length, lengths);
                for (int j = 0; j < it.tiles; ++j) {
                    if (v_iter > 0 && !(ok = sync.wait(kBarVEmpty, (v_iter - 1) & 1))) break;
                    const uint32_t b = sync.bar(kBarVFull);
                    mbar_expect_tx(b, kVTxBytes);
                    tma_load_3d(sbase + kSmemV, &qkv_map, b, 2 * C + it.h * kD, j * kN, it.n);
                    tma_load_3d(sbase + kSmemV + kAtom, &qkv_map, b, 2 * C + it.h * kD + 64,
                                j * kN, it.n);
                    ++v_iter;
                }
            }
            if (!ok && v_iter) mbar_wait(sync.bar(kBarVFull), (v_iter - 1) & 1);
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issuer (one thread) -------------------------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_f16(Fmt<T>::v, kM, kN, 0, 0);
            constexpr uint32_t idesc_b = idesc_f16(Fmt<T>::v, kM, kBand, 0, 0);
            constexpr uint32_t idesc_o = idesc_f16(Fmt<T>::v, kM, kD, 0, 1);
            uint32_t q_iter = 0, kb_iter = 0, v_iter = 0, s_iter = 0, items_done = 0;
            bool ok = true;
            auto issue_s = [&](bool last_of_item) -> bool {
                if (!sync.wait(kBarKBFull, kb_iter & 1)) return false;
                if (s_iter > 0 && !sync.wait(kBarSFree, (s_iter - 1) & 1)) return false;
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
                umma_commit(sync.bar(kBarSFull));
                umma_commit(sync.bar(kBarKBEmpty));
                if (last_of_item) umma_commit(sync.bar(kBarQEmpty));
                ++kb_iter;
                ++s_iter;
                return true;
            };
            for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
                const Item it = decode_item(item, qtiles, heads, length, lengths);
                if (it.tiles == 0) continue;
                if (!(ok = sync.wait(kBarQReady, q_iter & 1))) break;
                ++q_iter;
                if (!(ok = issue_s(it.tiles == 1))) break;
                for (int j = 0; j < it.tiles && ok; ++j) {
                    const bool more = j + 1 < it.tiles;
                    if (more && !(ok = issue_s(j + 2 == it.tiles))) break;
                    if (!(ok = sync.wait(kBarPFull, (s_iter - (more ? 2 : 1)) & 1))) break;
                    if (!(ok = sync.wait(kBarVFull, v_iter & 1))) break;
                    if (j == 0 && items_done > 0 &&
                        !(ok = sync.wait(kBarOFree, (items_done - 1) & 1)))
                        break;
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kN / 16; ++ks) {
                        const uint32_t a = ks >> 2, koff = (ks & 3) * 32;
                        const uint64_t pd = sw128_desc(sbase + kSmemP + a * kAtom + koff, 16, 1024);
                        // V is MN-major (head dim contiguous): 16 keys = 2 row groups = 2048 B;
                        // the two 64-channel halves are kAtom apart.
                        const uint64_t vd = sw128_desc(sbase + kSmemV + ks * 2048, kAtom, 1024);
                        umma_f16_ss(tmem + kColO, pd, vd, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(sync.bar(kBarVEmpty));
                    umma_commit(sync.bar(kBarODone));
                    ++v_iter;
                }
                ++items_done;
            }
            // Drain every MMA this thread issued before the CTA releases TMEM.
            umma_commit(sync.bar(kBarDrain));
            mbar_wait(sync.bar(kBarDrain), 0);
        }
    } else {
        // ---- softmax warps ---------------------------------------------------------------
        const int group = warp & 3;      // TMEM lane group == rows 32*group ..
        const int half = warp >> 2;      // keys [64*half, 64*half + 64) of every tile
        const int row = group * 32 + lane;
        const uint32_t tmem_row = tmem + (static_cast<uint32_t>(group * 32) << 16);
        const uint32_t shift = 31u - static_cast<uint32_t>(lane);
        const uint32_t pair_bar = 1 + group;  // named barrier of the two warps sharing rows
        uint32_t q_iter = 0, s_iter = 0, o_iter = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
            const Item it = decode_item(item, qtiles, heads, length, lengths);
            const int row_q = it.q0 + row;
            T* orow = out + (static_cast<int64_t>(it.n) * length + row_q) * C + it.h * kD +
                      half * 64;
            if (it.tiles == 0) {  // no valid key: the reference defines the rows as zero
                if (row_q < length) {
                    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(orow)[c] = z;
                }
                continue;
            }
            // (Q+u), (Q+v) in fp32, rounded to T (reference .cu:268-281); this warp does
            // head channels [64*half, 64*half+64) of its 32 rows.
            if (!(ok = sync.wait_warp(kBarQFull, q_iter & 1))) break;
            ++q_iter;
            {
                const T* ub = ubias + it.h * kD;
                const T* vb = vbias + it.h * kD;
#pragma unroll 2
                for (int c8 = 0; c8 < 8; ++c8) {
                    const int c = half * 8 + c8;
                    const uint32_t off = half * kAtom + sw128_offset(row, c8);
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
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(sync.bar(kBarQReady));

            float m_run = -INFINITY;  // reference max (base-2 logits)
            float l_run = 0.0f;       // this half's running sum of 2^(logit - m_run)
            for (int j = 0; j < it.tiles; ++j) {
                const int k0 = j * kN;
                if (!(ok = sync.wait_warp(kBarSFull, s_iter & 1))) break;
                ++s_iter;
                tc_fence_after();
                float s[kHalfKeys];
                const int nvalid = it.valid - k0;  // valid keys in this tile (>= 1)
                if (nvalid >= kN)
                    load_logits<false>(s, tmem_row, group, half, shift, scale_log2, nvalid);
                else
                    load_logits<true>(s, tmem_row, group, half, shift, scale_log2, nvalid);
                // Scores are in registers: the MMA warp may overwrite S with the next tile.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(sync.bar(kBarSFree));

                float m_half = -INFINITY;
#pragma unroll
                for (int e = 0; e < kHalfKeys; ++e) m_half = fmaxf(m_half, s[e]);
                xchg[half * kM + row] = m_half;
                named_barrier(pair_bar, 64);
                const float m_tile = fmaxf(m_half, xchg[(1 - half) * kM + row]);
                named_barrier(pair_bar, 64);  // the slot is rewritten next tile
                // Move the reference max only when it grows by more than 2^8.
                const bool grow = (m_tile - m_run) > kRescaleThreshold;
                const float m_new = grow ? m_tile : m_run;
                const float corr = grow ? fast_exp2(m_run - m_new) : 1.0f;

                // P(j-1) has been consumed and O(j-1) is final once PV(j-1) completed.
                if (j > 0) {
                    if (!(ok = sync.wait_warp(kBarODone, o_iter & 1))) break;
                    ++o_iter;
                    tc_fence_after();
                }
                float l_tile = 0.0f;
#pragma unroll
                for (int c = 0; c < kHalfKeys / 8; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float p0 = fast_exp2(s[c * 8 + 2 * e] - m_new);
                        const float p1 = fast_exp2(s[c * 8 + 2 * e + 1] - m_new);
                        l_tile += p0 + p1;
                        w[e] = pack2<T>(p0, p1);
                    }
                    const uint32_t off = half * kAtom + sw128_offset(row, c);
                    *reinterpret_cast<uint4*>(smem + kSmemP + off) =
                        make_uint4(w[0], w[1], w[2], w[3]);
                }
                l_run = l_run * corr + l_tile;
                m_run = m_new;
                if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const uint32_t col = kColO + half * 64 + c * 32;
                        uint32_t o[32];
                        tmem_ld32(tmem_row + col, o);
                        tmem_wait_ld();
                        reg_fence(o);
                        float of[32];
#pragma unroll
                        for (int e = 0; e < 32; ++e) of[e] = __uint_as_float(o[e]) * corr;
                        tmem_st32(tmem_row + col, of);
                    }
                    tmem_wait_st();
                }
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(sync.bar(kBarPFull));
            }
            if (!ok) break;
            // ---- epilogue: combine the two halves' sums, wait for the last PV, O / l ------------
            xchg[half * kM + row] = l_run;
            named_barrier(pair_bar, 64);
            const float l_total = l_run + xchg[(1 - half) * kM + row];
            named_barrier(pair_bar, 64);
            if (!(ok = sync.wait_warp(kBarODone, o_iter & 1))) break;
            ++o_iter;
            tc_fence_after();
            const float inv = 1.0f / l_total;
            const bool store = row_q < length;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t o[32];
                tmem_ld32(tmem_row + kColO + half * 64 + c * 32, o);
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sync.bar(kBarOFree));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
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

int sm_count() {
    static int count = [] {
        int dev = 0, n = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n > 0 ? n : 148;
    }();
    return count;
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
    const int64_t items = static_cast<int64_t>((p.length + kM - 1) / kM) * p.heads * p.batch;
    const dim3 grid(static_cast<unsigned>(items < sm_count() ? items : sm_count()));
    parakeet_tc_kernel<T><<<grid, kThreads, kSmemBytes, stream>>>(
        qkv_map, pos_map, static_cast<const T*>(p.content_bias),
        static_cast<const T*>(p.position_bias), p.valid_lengths, static_cast<T*>(p.output),
        p.batch, p.length, p.heads, p.scale * kLog2e);
    return cudaGetLastError();
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

cudaError_t launch_parakeet_tc(const ParakeetProblem& p, cudaStream_t stream) {
    if (p.head_dim != kD || (p.dtype != FGA_HALF && p.dtype != FGA_BF16)) return cudaErrorNotSupported;
    // log2(e) is folded into the scale; keep scaled logits far from the fp32 range limit.
    if (!(p.scale <= 1.0f)) return cudaErrorNotSupported;
    if (static_cast<int64_t>((p.length + kM - 1) / kM) * p.heads * p.batch > 0x7fffffff)
        return cudaErrorNotSupported;
    if (!aligned16(p.qkv) || !aligned16(p.position) || !aligned16(p.output) ||
        !aligned16(p.content_bias) || !aligned16(p.position_bias))
        return cudaErrorNotSupported;
    return p.dtype == FGA_HALF ? parakeet_tc_typed<__half>(p, stream)
                               : parakeet_tc_typed<__nv_bfloat16>(p, stream);
}

}  // namespace fga
