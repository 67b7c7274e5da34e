// Parakeet relative-position MHSA on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Work item = one 128-query tile (rows q0..q0+127) of one (utterance n, head h), head
// dim D = 128. Keys are visited in tiles of 128 (k0 = 128 j) up to the valid length.
//
//   S_c(j) = (Q+u) K_j^T      128 x 128   tcgen05.mma -> TMEM cols [0,128)
//   band   = (Q+v) Pband^T                 tcgen05.mma -> TMEM band ring
//   logit(q,k) = scale * (S_c[q,k] + band[q, T-1-q+k])     (Transformer-XL shift)
//   online softmax over keys k < valid_length (fp32, base 2)
//   O     += P_j V_j          128 x 128   tcgen05.mma -> TMEM cols [384,512)
//
// Positional band. Key tile j touches relative rows r0 + 128 j + [0, 256) with
// r0 = T-128-q0; row i of the tile needs band column 127-i+kk for key kk. The 256
// columns of tile j are two 128-row "halves" m = j and m = j+1 of the item's band
// (half m = positional rows r0 + 128 m + [0,128)), and tile j+1 reuses half j+1. So each
// half is computed once, by an N=128 MMA into a two-slot TMEM ring (slot m % 2):
// halves 0 and 1 together with S_c(0), half j+2 together with S_c(j+1). The score MMAs
// then do exactly the algorithmic work (no band recomputation).
//
// Skew. A warp loads the 96-column band window its 32 rows and 64 keys span (three
// 32-column pieces, each inside one half) together with its S_c columns, releases S at
// once, and every thread then shifts its own row into place with a 5-stage predicated
// barrel shift while the MMA warp computes the next tile's scores.
//
// CTA organisation (persistent: one CTA per SM walks the work items):
//   warps 0-7  softmax. Warp w owns TMEM lanes 32*(w%4).. (rows) and key half w/4 (64
//              keys of each tile); the two warps of a row group exchange the row max
//              through shared memory behind a 64-thread named barrier. After reading the
//              scores of an item's last tile they form the next item's biased queries,
//              so the next item's first MMAs overlap this item's exponentials and
//              epilogue.
//   warp 8     TMA producer: lane 0 loads Q, K and positional chunks, lane 1 loads V.
//   warp 9     MMA issuer (one thread) and TMEM owner.
// O is rescaled only when a row max grows by more than 2^8 (the unnormalised
// probabilities stay <= 256, exact in f16/bf16 range).
//
// Reference semantics (parakeet_relative_attention_plugin.cu): biased queries are
// formed in fp32 and rounded to the I/O dtype (:268-281); scores are summed and scaled
// in fp32 (:503-508); only keys below the valid length contribute; valid_length <= 0
// gives zero rows (:478-486); every query row < T is produced (:472-476). Scores stay
// in fp32 between the GEMMs (the reference stores them in the I/O dtype). log2(e) is
// folded into the scale and the row max is taken before scaling, so this kernel serves
// 0 < scale <= 1 (every real model: 1/sqrt(D)); other scales run on the SIMT kernel,
// which subtracts the row max before converting to base 2 exactly like the reference.
//
// Data movement: Q, K and V tiles arrive by TMA from the fused [N, T, 3C] projection
// through a 3-D tensor map (rows past T of an utterance read as zero), positional
// chunks through a 2-D map over [2T-1, C] (rows outside the table read as zero), the
// head's u and v rows by bulk copy with Q. All operand tiles use the 128-byte-swizzled
// canonical UMMA layouts. Each softmax warp stages its 32 x 64 block of O / l in its own
// rows of the P tile and writes it with one TMA store (rows past T are not written).
#include <cuda.h>

#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "host_util.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;       // query rows per work item
constexpr int kN = 128;       // keys per tile (= rows per positional half)
constexpr int kD = 128;       // head dim
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kHalfKeys = kN / 2;

// Shared-memory map (bytes from the 1024-aligned dynamic base). Every tile is
// 128 rows x 128 channels = two 64-channel swizzle atoms of 16 KB.
constexpr uint32_t kAtom = 128 * 128;
constexpr uint32_t kTile = 2 * kAtom;
constexpr uint32_t kSmemQu = 0;                 // TMA lands Q here first
constexpr uint32_t kSmemQv = kSmemQu + kTile;
constexpr uint32_t kSmemK = kSmemQv + kTile;
constexpr uint32_t kSmemV = kSmemK + kTile;
constexpr uint32_t kSmemB0 = kSmemV + kTile;    // positional chunk slots 0 and 1
constexpr uint32_t kSmemP = kSmemB0 + 2 * kTile;
constexpr uint32_t kSmemXchg = kSmemP + kTile;  // [2 halves][128 rows] fp32
constexpr uint32_t kLenCache = 256;             // valid lengths of utterances 0..255
constexpr uint32_t kSmemLen = kSmemXchg + 2 * kM * 4;
constexpr uint32_t kSmemBias = kSmemLen + kLenCache * 4;  // [u | v] of the item's head
constexpr uint32_t kBiasBytes = 2 * kD * 2;
constexpr uint32_t kSmemBar = kSmemBias + kBiasBytes;
constexpr uint32_t kNumBars = 17;
constexpr uint32_t kSmemBytes = kSmemBar + kNumBars * 8 + 16;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSc = 0, kColBand = 128, kColO = 384;  // band ring: 2 x 128 cols

constexpr float kRescaleThreshold = 8.0f;  // log2 units

enum : uint32_t {
    kBarQFull = 0, kBarQReady, kBarQEmpty, kBarKFull, kBarKEmpty, kBarVFull, kBarVEmpty,
    kBarSFull, kBarSFree, kBarPFull, kBarODone, kBarOFree, kBarDrain,
    kBarBFull0, kBarBFull1,  // positional chunk slot s full: kBarBFull0 + s
    kBarBEmpty0              // slot s empty: kBarBEmpty0 + s (entries 15 and 16)
};
static_assert(kBarBEmpty0 + 2 == kNumBars, "barrier table");
static_assert(kSmemBias % 16 == 0 && kSmemBytes <= 227 * 1024, "shared-memory map");

// Per-device error word of this file's kernel: 1 = a bounded wait gave up, 2 = the dynamic
// shared memory was not 1024-byte aligned. Read and cleared by fga_device_status.
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
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The positional band is held as packed pairs of the storage type T (element 2i in the
// low half of word i): the reference's positional-score GEMM writes T as well
// (parakeet_relative_attention_plugin.cu:1062-1087), and a 32-bit select then moves two
// elements. out[e] = v[e + s] for e < 64, s in [0, 31]: four predicated word stages (8, 4,
// 2 and 1 words = 16, 8, 4 and 2 elements), each touching only the words the later stages
// still read, then one byte permute per word for an odd shift.
template <typename T> __device__ __forceinline__ uint32_t pack_band(float a, float b);
template <> __device__ __forceinline__ uint32_t pack_band<__half>(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
    return r;
}
template <> __device__ __forceinline__ uint32_t pack_band<__nv_bfloat16>(float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void band_shift_words(uint32_t (&w)[48], uint32_t s) {
#pragma unroll
    for (int j = 0; j < 40; ++j) w[j] = (s & 16u) ? w[j + 8] : w[j];
#pragma unroll
    for (int j = 0; j < 36; ++j) w[j] = (s & 8u) ? w[j + 4] : w[j];
#pragma unroll
    for (int j = 0; j < 34; ++j) w[j] = (s & 4u) ? w[j + 2] : w[j];
#pragma unroll
    for (int j = 0; j < 33; ++j) w[j] = (s & 2u) ? w[j + 1] : w[j];
}
__device__ __forceinline__ void band_shift_odd(uint32_t (&w)[48], uint32_t s) {
    // Selector 0x5432: the high element of word j and the low element of word j + 1.
    const uint32_t sel = (s & 1u) ? 0x5432u : 0x3210u;
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = __byte_perm(w[j], w[j + 1], sel);
}

// a + float(h) with the 16-bit value h of type T converted exactly (fma with 1.0).
template <typename T> __device__ __forceinline__ float add_t16(float a, uint16_t h);
template <> __device__ __forceinline__ float add_t16<__half>(float a, uint16_t h) {
    float r;
    asm("{\n\t.reg .b16 one;\n\tmov.b16 one, 0x3C00;\n\t"
        "fma.rn.f32.f16 %0, %1, one, %2;\n\t}" : "=f"(r) : "h"(h), "f"(a));
    return r;
}
template <> __device__ __forceinline__ float add_t16<__nv_bfloat16>(float a, uint16_t h) {
    float r;
    asm("{\n\t.reg .b16 one;\n\tmov.b16 one, 0x3F80;\n\t"
        "fma.rn.f32.bf16 %0, %1, one, %2;\n\t}" : "=f"(r) : "h"(h), "f"(a));
    return r;
}

// Maximum of 64 values with three-input max instructions (eight independent chains).
__device__ __forceinline__ float tree_max(const float (&x)[64]) {
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmax3(x[i], x[i + 8], x[i + 16]);
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmax3(m[i], x[i + 24], x[i + 32]);
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmax3(m[i], x[i + 40], x[i + 48]);
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], x[i + 56]);
    return fmax3(fmax3(m[0], m[1], m[2]), fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

struct Item {
    int n, h, q0, valid, tiles;
};

// Valid lengths: utterances below kLenCache come from the shared-memory copy made at
// kernel start (an item's length is on every role's critical path), the rest from global.
struct Lengths {
    const int32_t* __restrict__ global;
    const int32_t* cached;
    __device__ __forceinline__ int operator[](int n) const {
        return n < static_cast<int>(kLenCache) ? cached[n] : __ldg(global + n);
    }
};

__device__ __forceinline__ Item decode_item(int item, int qtiles, int heads, int length,
                                            const Lengths& lengths) {
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

// TMEM column of virtual band column x (0..255) of a tile whose lower half lives in
// ring slot `slot_lo` (the upper half is in the other slot).
__device__ __forceinline__ uint32_t band_col(uint32_t x, uint32_t slot_lo) {
    const uint32_t slot = (x < 128u) ? slot_lo : (slot_lo ^ 1u);
    return kColBand + slot * 128u + (x & 127u);
}

// This thread's row of the tile as it sits in TMEM: the 96 band columns its 64 keys
// reach (rows of a warp span 32 band columns, so the window is [base, base + 96) with
// base = 96 - 32 group + 64 half, in three 32-column pieces that each lie inside one ring
// slot), packed to T pairs, then S_c of those keys. The word shift stages run between
// the two loads so that fewer values are live at once. Every load completes here, so the
// caller can release S before the rest of the arithmetic and the next tile's score MMAs
// overlap the skew and the exponentials.
template <typename T>
__device__ __forceinline__ void load_tile(uint32_t (&sc)[kHalfKeys], uint32_t (&band)[48],
                                          uint32_t tmem_row, int group, int half,
                                          uint32_t slot_lo, uint32_t shift) {
    const uint32_t base = 96u - 32u * group + 64u * half;
    uint32_t raw[96];
#pragma unroll
    for (int p = 0; p < 3; ++p)
        tmem_ld32(tmem_row + band_col(base + 32u * p, slot_lo),
                  *reinterpret_cast<uint32_t(*)[32]>(raw + 32 * p));
    tmem_wait_ld();
#pragma unroll
    for (int p = 0; p < 3; ++p) reg_fence(*reinterpret_cast<uint32_t(*)[32]>(raw + 32 * p));
#pragma unroll
    for (int i = 0; i < 48; ++i)
        band[i] = pack_band<T>(__uint_as_float(raw[2 * i]), __uint_as_float(raw[2 * i + 1]));
    band_shift_words(band, shift);
    tmem_ld64(tmem_row + kColSc + half * 64, sc);
    tmem_wait_ld();
    reg_fence(sc);
}

// Unscaled logits S_c + band of this thread's 64 keys (row lane of its warp reads band
// column base + key + 31 - lane); keys at or past the valid length are -inf.
template <typename T, bool kMasked>
__device__ __forceinline__ void form_logits(float (&s)[kHalfKeys],
                                            const uint32_t (&sc)[kHalfKeys],
                                            uint32_t (&band)[48], uint32_t shift, int nvalid) {
    band_shift_odd(band, shift);
#pragma unroll
    for (int e = 0; e < kHalfKeys; e += 2) {
        const uint32_t w = band[e >> 1];
        const float v0 = add_t16<T>(__uint_as_float(sc[e]), static_cast<uint16_t>(w & 0xFFFFu));
        const float v1 = add_t16<T>(__uint_as_float(sc[e + 1]), static_cast<uint16_t>(w >> 16));
        s[e] = (!kMasked || e < nvalid) ? v0 : -INFINITY;
        s[e + 1] = (!kMasked || e + 1 < nvalid) ? v1 : -INFINITY;
    }
}

// Two packed T values added with one round-to-nearest packed add. The reference forms
// the biased queries in fp32 and rounds the sum to T (reference .cu:268-281). For f16
// (11-bit significand) and bf16 (8-bit) inputs the fp32 sum rounded to T equals the
// correctly rounded T sum: double rounding through a format of p' >= 2p + 1 significand
// bits is innocuous for addition (S. A. Figueroa, "When is double rounding innocuous?",
// SIGNUM Newsletter 30(3), 1995), and fp32 has p' = 24.
template <typename T> __device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b);
template <> __device__ __forceinline__ uint32_t add2<__half>(uint32_t a, uint32_t b) {
    __half2 r = __hadd2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
template <> __device__ __forceinline__ uint32_t add2<__nv_bfloat16>(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hadd2(*reinterpret_cast<__nv_bfloat162*>(&a),
                               *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// Q+u and Q+v rounded to T (see add2) for this thread's row and head channels
// [64*half, 64*half+64), in place in the Qu tile and into the Qv tile. The item's u and v
// rows arrive in shared memory with its Q tile.
template <typename T>
__device__ __forceinline__ void bias_queries(uint8_t* smem, int row, int half) {
    const uint4* ub = reinterpret_cast<const uint4*>(smem + kSmemBias) + half * 8;
    const uint4* vb = reinterpret_cast<const uint4*>(smem + kSmemBias + 2 * kD) + half * 8;
#pragma unroll 4
    for (int c = 0; c < 8; ++c) {
        const uint32_t off = half * kAtom + sw128_offset(row, c);
        const uint4 q = *reinterpret_cast<const uint4*>(smem + kSmemQu + off);
        const uint4 u = ub[c], v = vb[c];
        *reinterpret_cast<uint4*>(smem + kSmemQu + off) = make_uint4(
            add2<T>(q.x, u.x), add2<T>(q.y, u.y), add2<T>(q.z, u.z), add2<T>(q.w, u.w));
        *reinterpret_cast<uint4*>(smem + kSmemQv + off) = make_uint4(
            add2<T>(q.x, v.x), add2<T>(q.y, v.y), add2<T>(q.z, v.z), add2<T>(q.w, v.w));
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
parakeet_tc_kernel(const __grid_constant__ CUtensorMap qkv_map,
                   const __grid_constant__ CUtensorMap pos_map,
                   const __grid_constant__ CUtensorMap out_map, const T* __restrict__ ubias,
                   const T* __restrict__ vbias, const int32_t* __restrict__ lengths_global,
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
    int32_t* len_cache = reinterpret_cast<int32_t*>(smem + kSmemLen);
    for (int i = tid; i < batch && i < static_cast<int>(kLenCache); i += kThreads)
        len_cache[i] = lengths_global[i];
    const Lengths lengths{lengths_global, len_cache};
    if (tid == 0) {
        for (uint32_t i = 0; i < kNumBars; ++i) {
            const bool per_warp = i == kBarQReady || i == kBarSFree || i == kBarPFull ||
                                  i == kBarOFree;
            mbar_init(sync.bar(i), per_warp ? kSoftmaxWarps : 1);
        }
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
        // ---- TMA producer: lane 0 loads Q, K and positional chunks, lane 1 loads V ---------
        if (lane == 0) {
            uint32_t q_iter = 0, k_iter = 0, c_iter = 0;
            bool ok = true;
            auto load_chunk = [&](const Item& it, int m) -> bool {
                const uint32_t slot = c_iter & 1;
                if (c_iter >= 2 && !sync.wait(kBarBEmpty0 + slot, ((c_iter >> 1) - 1) & 1))
                    return false;
                const int r = length - kM - it.q0 + m * kN;  // first positional row
                const uint32_t b = sync.bar(kBarBFull0 + slot);
                mbar_expect_tx(b, kTile);
                tma_load_2d(sbase + kSmemB0 + slot * kTile, &pos_map, b, it.h * kD, r);
                tma_load_2d(sbase + kSmemB0 + slot * kTile + kAtom, &pos_map, b,
                            it.h * kD + 64, r);
                ++c_iter;
                return true;
            };
            auto load_k = [&](const Item& it, int j) -> bool {
                if (k_iter > 0 && !sync.wait(kBarKEmpty, (k_iter - 1) & 1)) return false;
                const uint32_t b = sync.bar(kBarKFull);
                mbar_expect_tx(b, kTile);
                tma_load_3d(sbase + kSmemK, &qkv_map, b, C + it.h * kD, j * kN, it.n);
                tma_load_3d(sbase + kSmemK + kAtom, &qkv_map, b, C + it.h * kD + 64, j * kN,
                            it.n);
                ++k_iter;
                return true;
            };
            // Warm L2 with everything an item will load (Q, K and V tiles, positional
            // chunks), one item ahead, so the SMEM loads that wait for a free buffer
            // hit L2 instead of HBM.
            auto prefetch_item = [&](int item) {
                if (item >= num_items) return;
                const Item it = decode_item(item, qtiles, heads, length, lengths);
                if (it.tiles == 0) return;
                for (int a = 0; a < 2; ++a) {
                    const int x = it.h * kD + 64 * a;
                    tma_prefetch_3d(&qkv_map, x, it.q0, it.n);
                    for (int j = 0; j < it.tiles; ++j) {
                        tma_prefetch_3d(&qkv_map, C + x, j * kN, it.n);
                        tma_prefetch_3d(&qkv_map, 2 * C + x, j * kN, it.n);
                    }
                    for (int m = 0; m <= it.tiles; ++m)
                        tma_prefetch_2d(&pos_map, x, length - kM - it.q0 + m * kN);
                }
            };
            prefetch_item(blockIdx.x);
            for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
                const Item it = decode_item(item, qtiles, heads, length, lengths);
                if (it.tiles == 0) continue;
                prefetch_item(item + gridDim.x);
                if (q_iter > 0 && !(ok = sync.wait(kBarQEmpty, (q_iter - 1) & 1))) break;
                mbar_expect_tx(sync.bar(kBarQFull), kTile + kBiasBytes);
                tma_load_3d(sbase + kSmemQu, &qkv_map, sync.bar(kBarQFull), it.h * kD, it.q0, it.n);
                tma_load_3d(sbase + kSmemQu + kAtom, &qkv_map, sync.bar(kBarQFull),
                            it.h * kD + 64, it.q0, it.n);
                bulk_load(sbase + kSmemBias, ubias + it.h * kD, 2 * kD, sync.bar(kBarQFull));
                bulk_load(sbase + kSmemBias + 2 * kD, vbias + it.h * kD, 2 * kD,
                          sync.bar(kBarQFull));
                ++q_iter;
                // In the order the MMA consumes them: K(0), chunk 0, chunk 1, then
                // K(j), chunk j+1 for j >= 1.
                if (!(ok = load_k(it, 0)) || !(ok = load_chunk(it, 0)) ||
                    !(ok = load_chunk(it, 1)))
                    break;
                for (int j = 1; j < it.tiles && ok; ++j)
                    ok = load_k(it, j) && load_chunk(it, j + 1);
            }
            if (!ok) {  // drain our own copies in flight (bounded) before teardown
                if (q_iter) mbar_wait(sync.bar(kBarQFull), (q_iter - 1) & 1);
                if (k_iter) mbar_wait(sync.bar(kBarKFull), (k_iter - 1) & 1);
                for (uint32_t s = 0; s < 2 && s < c_iter; ++s) {
                    const uint32_t last = c_iter - 1 - s;  // the last load into slot last&1
                    mbar_wait(sync.bar(kBarBFull0 + (last & 1)), (last >> 1) & 1);
                }
            }
        } else if (lane == 1) {
            uint32_t v_iter = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
                const Item it = decode_item(item, qtiles, heads, length, lengths);
                for (int j = 0; j < it.tiles; ++j) {
                    if (v_iter > 0 && !(ok = sync.wait(kBarVEmpty, (v_iter - 1) & 1))) break;
                    const uint32_t b = sync.bar(kBarVFull);
                    mbar_expect_tx(b, kTile);
                    tma_load_3d(sbase + kSmemV, &qkv_map, b, 2 * C + it.h * kD, j * kN, it.n);
                    tma_load_3d(sbase + kSmemV + kAtom, &qkv_map, b, 2 * C + it.h * kD + 64,
                                j * kN, it.n);
                    ++v_iter;
                }
            }
            if (!ok && v_iter) mbar_wait(sync.bar(kBarVFull), (v_iter - 1) & 1);
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issuer: the whole warp runs this loop (uniform control flow, warp-
        // uniform descriptors); one elected lane issues each tcgen05 instruction. A
        // single-thread issuer is starved of issue slots by the busy softmax warps.
        constexpr uint32_t idesc_s = idesc_f16(Fmt<T>::v, kM, kN, 0, 0);
        constexpr uint32_t idesc_o = idesc_f16(Fmt<T>::v, kM, kD, 0, 1);
        // Base descriptors (K-major operands: +32 B per 16-channel K step inside an
        // atom, +kAtom per atom; V is MN-major: +2048 B per 16-key step).
        const uint64_t d_qu = sw128_desc(sbase + kSmemQu, 16, 1024);
        const uint64_t d_qv = sw128_desc(sbase + kSmemQv, 16, 1024);
        const uint64_t d_k = sw128_desc(sbase + kSmemK, 16, 1024);
        const uint64_t d_b0 = sw128_desc(sbase + kSmemB0, 16, 1024);
        const uint64_t d_p = sw128_desc(sbase + kSmemP, 16, 1024);
        const uint64_t d_v = sw128_desc(sbase + kSmemV, kAtom, 1024);
        auto kstep = [](uint32_t ks) -> uint64_t {  // descriptor offset (16-byte units)
            return static_cast<uint64_t>(((ks >> 2) * kAtom + (ks & 3) * 32) >> 4);
        };
        uint32_t q_iter = 0, k_iter = 0, c_iter = 0, h_iter = 0, v_iter = 0, s_iter = 0,
                 items_done = 0;
        bool ok = true;
        auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, sync.wait(bar, parity));
        };
        // One positional half: band ring slot (h_iter % 2) = Qv . chunk(c_iter)^T.
        auto band_half = [&]() -> bool {
            const uint32_t slot = c_iter & 1;
            if (!wait(kBarBFull0 + slot, (c_iter >> 1) & 1)) return false;
            tc_fence_after();
            const uint32_t d = tmem + kColBand + (h_iter & 1) * 128;
            const uint64_t b = d_b0 + ((slot * kTile) >> 4);
            if (elect_one()) {
#pragma unroll
                for (uint32_t ks = 0; ks < kD / 16; ++ks)
                    umma_f16_ss(d, d_qv + kstep(ks), b + kstep(ks), idesc_s, ks > 0);
                umma_commit(sync.bar(kBarBEmpty0 + slot));
            }
            __syncwarp();
            ++c_iter;
            ++h_iter;
            return true;
        };
        // Score MMAs of one tile: content S_c and the new positional half(s).
        auto issue_s = [&](bool first_of_item, bool last_of_item) -> bool {
            if (!wait(kBarKFull, k_iter & 1)) return false;
            if (s_iter > 0 && !wait(kBarSFree, (s_iter - 1) & 1)) return false;
            tc_fence_after();
            if (elect_one()) {
#pragma unroll
                for (uint32_t ks = 0; ks < kD / 16; ++ks)
                    umma_f16_ss(tmem + kColSc, d_qu + kstep(ks), d_k + kstep(ks), idesc_s, ks > 0);
                umma_commit(sync.bar(kBarKEmpty));
            }
            __syncwarp();
            ++k_iter;
            if (first_of_item && !band_half()) return false;
            if (!band_half()) return false;
            if (elect_one()) {
                umma_commit(sync.bar(kBarSFull));
                if (last_of_item) umma_commit(sync.bar(kBarQEmpty));
            }
            __syncwarp();
            ++s_iter;
            return true;
        };
        auto next_item = [&](int from) -> int {
            int item = from;
            while (item < num_items &&
                   decode_item(item, qtiles, heads, length, lengths).tiles == 0)
                item += gridDim.x;
            return item;
        };
        // The first score MMAs of an item: wait for its biased queries, then S(0).
        auto start_item = [&](int item) -> bool {
            const Item it = decode_item(item, qtiles, heads, length, lengths);
            if (!wait(kBarQReady, q_iter & 1)) return false;
            ++q_iter;
            return issue_s(true, it.tiles == 1);
        };
        int item = next_item(blockIdx.x);
        if (item < num_items) ok = start_item(item);
        while (ok && item < num_items) {
            const Item it = decode_item(item, qtiles, heads, length, lengths);
            // The candidate's length load is issued now and consumed at the last tile.
            const int cand = item + gridDim.x;
            const int cand_len = cand < num_items ? lengths[cand / (qtiles * heads)] : 0;
            int next = num_items;
            for (int j = 0; j < it.tiles && ok; ++j) {
                if (j + 1 == it.tiles && cand < num_items)
                    next = cand_len > 0 ? cand : next_item(cand);
                // Keep the tensor pipe fed: the next tile's score MMAs go ahead of this
                // tile's P.V. (The next item's first score MMAs follow the last P.V: its
                // biased queries are formed while that P.V runs.)
                if (j + 1 < it.tiles && !(ok = issue_s(false, j + 2 == it.tiles))) break;
                if (!(ok = wait(kBarPFull, v_iter & 1))) break;
                if (!(ok = wait(kBarVFull, v_iter & 1))) break;
                if (j == 0 && items_done > 0 && !(ok = wait(kBarOFree, (items_done - 1) & 1)))
                    break;
                tc_fence_after();
                if (elect_one()) {
#pragma unroll
                    for (uint32_t ks = 0; ks < kN / 16; ++ks)
                        umma_f16_ss(tmem + kColO, d_p + kstep(ks),
                                    d_v + static_cast<uint64_t>((ks * 2048) >> 4), idesc_o,
                                    (j > 0 || ks > 0) ? 1u : 0u);
                    umma_commit(sync.bar(kBarVEmpty));
                    umma_commit(sync.bar(kBarODone));
                }
                __syncwarp();
                ++v_iter;
                if (j + 1 == it.tiles && next < num_items && !(ok = start_item(next))) break;
            }
            ++items_done;
            item = next;
        }
        // Drain every MMA this warp issued before the CTA releases TMEM.
        if (elect_one()) {
            umma_commit(sync.bar(kBarDrain));
            mbar_wait(sync.bar(kBarDrain), 0);
        }
        __syncwarp();
    } else {
        // ---- softmax warps ---------------------------------------------------------------
        const int group = warp & 3;      // TMEM lane group == rows 32*group ..
        const int half = warp >> 2;      // keys [64*half, 64*half + 64) of every tile
        const int row = group * 32 + lane;
        const uint32_t tmem_row = tmem + (static_cast<uint32_t>(group * 32) << 16);
        const uint32_t shift = 31u - static_cast<uint32_t>(lane);
        const uint32_t pair_bar = 1 + group;  // named barrier of the two warps sharing rows
        uint32_t q_iter = 0, s_iter = 0, o_iter = 0, h_base = 0;
        bool ok = true;

        // Items with no valid key are zero rows (reference :478-486); they need no MMA.
        auto next_item = [&](int from) -> int {
            int item = from;
            for (; item < num_items; item += gridDim.x) {
                const Item it = decode_item(item, qtiles, heads, length, lengths);
                if (it.tiles > 0) break;
                const int row_q = it.q0 + row;
                if (row_q < length) {
                    T* orow = out + (static_cast<int64_t>(it.n) * length + row_q) * C +
                              it.h * kD + half * 64;
                    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(orow)[c] = z;
                }
            }
            return item;
        };
        auto prepare_queries = [&]() -> bool {
            if (!sync.wait_warp(kBarQFull, q_iter & 1)) return false;
            ++q_iter;
            bias_queries<T>(smem, row, half);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(sync.bar(kBarQReady));
            return true;
        };

        int item = next_item(blockIdx.x);
        if (item < num_items) ok = prepare_queries();
        while (ok && item < num_items) {
            const Item it = decode_item(item, qtiles, heads, length, lengths);
            // The candidate's length load is issued now and consumed at the last tile.
            const int cand = item + gridDim.x;
            const int cand_len = cand < num_items ? lengths[cand / (qtiles * heads)] : 0;
            int next = num_items;
            float m_run = -INFINITY;  // reference max (base-2 logits)
            float l_run = 0.0f;       // this half's running sum of 2^(logit - m_run)
            for (int j = 0; j < it.tiles; ++j) {
                const int k0 = j * kN;
                if (!(ok = sync.wait_warp(kBarSFull, s_iter & 1))) break;
                ++s_iter;
                tc_fence_after();
                const int nvalid = it.valid - k0;  // valid keys in this tile (>= 1)
                const uint32_t slot_lo = (h_base + j) & 1;
                float s[kHalfKeys];
                {
                    uint32_t sc[kHalfKeys], band[48];
                    load_tile<T>(sc, band, tmem_row, group, half, slot_lo, shift);
                    // Scores are in registers: the MMA warp may overwrite S with the next tile.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(sync.bar(kBarSFree));
                    if (nvalid >= kN)
                        form_logits<T, false>(s, sc, band, shift, kHalfKeys);
                    else
                        form_logits<T, true>(s, sc, band, shift, nvalid - half * kHalfKeys);
                }

                const float m_half = tree_max(s);
                xchg[half * kM + row] = m_half;
                named_barrier(pair_bar, 64);
                // Scaled base-2 tile max: scale_log2 > 0, so scaling commutes with max.
                const float m_tile = fmaxf(m_half, xchg[(1 - half) * kM + row]) * scale_log2;
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
                // The item's first P overwrites the rows this warp staged the previous
                // item's output in: that store must have read them.
                if (j == 0) {
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                }
                // Exponent arguments and the running sums on packed fp32 pairs.
                const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
                const uint64_t neg_m2 = f2_pack(-m_new, -m_new);
                uint64_t lsum2[4] = {0, 0, 0, 0};  // +0.0f pairs
#pragma unroll
                for (int c = 0; c < kHalfKeys / 8; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 a = f2_unpack(
                            f2_fma(f2_pack(s[c * 8 + 2 * e], s[c * 8 + 2 * e + 1]), scale2, neg_m2));
                        const float p0 = fast_exp2(a.x);
                        const float p1 = fast_exp2(a.y);
                        lsum2[e] = f2_add(lsum2[e], f2_pack(p0, p1));
                        w[e] = pack2<T>(p0, p1);
                    }
                    const uint32_t off = half * kAtom + sw128_offset(row, c);
                    *reinterpret_cast<uint4*>(smem + kSmemP + off) =
                        make_uint4(w[0], w[1], w[2], w[3]);
                }
                const float2 l2 = f2_unpack(f2_add(f2_add(lsum2[0], lsum2[1]),
                                                   f2_add(lsum2[2], lsum2[3])));
                l_run = l_run * corr + (l2.x + l2.y);
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
                // After the last tile's P, prepare the next item's queries while the
                // last P.V runs; its first score MMAs then run under this epilogue.
                if (j + 1 == it.tiles && cand < num_items) {
                    next = cand_len > 0 ? cand : next_item(cand);
                    if (next < num_items && !(ok = prepare_queries())) break;
                }
            }
            if (!ok) break;
            h_base += it.tiles + 1;
            // ---- epilogue: combine the two halves' sums, wait for the last PV, O / l ------------
            xchg[half * kM + row] = l_run;
            named_barrier(pair_bar, 64);
            const float l_total = l_run + xchg[(1 - half) * kM + row];
            named_barrier(pair_bar, 64);
            if (!(ok = sync.wait_warp(kBarODone, o_iter & 1))) break;
            ++o_iter;
            tc_fence_after();
            const float inv = 1.0f / l_total;
            // O / l goes to this warp's own rows of the P tile (free once the last P.V has
            // completed; the same 32 rows x 64 channels this warp writes P into), then one
            // TMA store per warp writes them out. Rows past T fall outside the tensor map.
            const uint32_t stage = kSmemP + half * kAtom;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t o[32];
                tmem_ld32(tmem_row + kColO + half * 64 + c * 32, o);
                tmem_wait_ld();
                reg_fence(o);
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                    const uint4 w = make_uint4(
                        pack2<T>(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv),
                        pack2<T>(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv),
                        pack2<T>(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv),
                        pack2<T>(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv));
                    *reinterpret_cast<uint4*>(smem + stage + sw128_offset(row, c * 4 + e / 8)) = w;
                }
            }
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && it.q0 + group * 32 < length) {
                tma_store_3d(&out_map, sbase + stage + group * 32 * 128, it.h * kD + half * 64,
                             it.q0 + group * 32, it.n);
                bulk_commit_group();
            }
            if (lane == 0) mbar_arrive(sync.bar(kBarOFree));
            item = next;
        }
    }

    if (warp < kSoftmaxWarps && lane == 0) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---- host side ------------------------------------------------------------------------------
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
        const cuuint32_t box[2] = {64, kN};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&pos_map, dt, 2, const_cast<void*>(p.position), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return cudaErrorNotSupported;
    }
    CUtensorMap out_map;
    {
        const cuuint64_t dims[3] = {C, static_cast<cuuint64_t>(p.length),
                                    static_cast<cuuint64_t>(p.batch)};
        const cuuint64_t strides[2] = {C * sizeof(T), C * sizeof(T) * p.length};
        const cuuint32_t box[3] = {64, 32, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (encode(&out_map, dt, 3, p.output, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return cudaErrorNotSupported;
    }
    static SmemAttr attr;
    if (cudaError_t e = attr.ensure(reinterpret_cast<const void*>(parakeet_tc_kernel<T>),
                                    static_cast<int>(kSmemBytes));
        e != cudaSuccess)
        return e;
    const int64_t items = static_cast<int64_t>((p.length + kM - 1) / kM) * p.heads * p.batch;
    const int sms = sm_count();
    if (sms <= 0) return cudaErrorNotSupported;
    const dim3 grid(static_cast<unsigned>(items < sms ? items : sms));
    parakeet_tc_kernel<T><<<grid, kThreads, kSmemBytes, stream>>>(
        qkv_map, pos_map, out_map, static_cast<const T*>(p.content_bias),
        static_cast<const T*>(p.position_bias), p.valid_lengths, static_cast<T*>(p.output),
        p.batch, p.length, p.heads, p.scale * kLog2e);
    return cudaGetLastError();
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

uint32_t take_parakeet_tc_error(cudaStream_t stream, bool clear, cudaError_t* err) {
    return take_error_word(g_parakeet_tc_error, stream, clear, err);
}

cudaError_t launch_parakeet_tc(const ParakeetProblem& p, cudaStream_t stream) {
    if (p.head_dim != kD || (p.dtype != FGA_HALF && p.dtype != FGA_BF16)) return cudaErrorNotSupported;
    // log2(e) is folded into the scale; keep scaled logits far from the fp32 range limit.
    // The tile max is taken before scaling, which needs a positive scale.
    if (!(p.scale > 0.0f && p.scale <= 1.0f)) return cudaErrorNotSupported;
    if (static_cast<int64_t>((p.length + kM - 1) / kM) * p.heads * p.batch > 0x7fffffff)
        return cudaErrorNotSupported;
    if (!aligned16(p.qkv) || !aligned16(p.position) || !aligned16(p.output) ||
        !aligned16(p.content_bias) || !aligned16(p.position_bias))
        return cudaErrorNotSupported;
    return p.dtype == FGA_HALF ? parakeet_tc_typed<__half>(p, stream)
                               : parakeet_tc_typed<__nv_bfloat16>(p, stream);
}

}  // namespace fga
