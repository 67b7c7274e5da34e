// Depthwise temporal convolution of the encoders' convolution modules, NTC storage:
//   parakeet_conformer_convolution: masked depthwise convolution with the evaluation-mode
//     BatchNorm folded into weight and bias, then SiLU;
//   zipformer_convolution: masked depthwise convolution, then Swoosh-R.
//
//   y[n,t,c] = act( bias[c] + sum_k w[k,c] * xm[n, t+k-K/2, c] )
//
// xm is x on the frames below the utterance's valid length (clamped to [0, T]) and zero
// elsewhere; output frames past the valid length are written too (not re-masked).
//
// Reference semantics (parakeet_convolution_plugin.cu:105-157, 241-352, 598-623;
// zipformer_convolution_plugin.cu:104-109, 156-199, 275-509, 790-835):
// - f16/bf16 accumulate in the storage type: starting from the bias, one packed fused
//   multiply-add per tap in tap order, each rounding to the storage type; the activation
//   is evaluated in fp32 on the rounded sum and rounded once at the store. fp32 uses one
//   fmaf per tap in the same order.
// - A tap on a padded or out-of-range frame is a multiply-add with a zero input, except
//   in the Parakeet paths that skip it (fp32, and f16/bf16 when C % 8 != 0). The two differ
//   only for non-finite weights or a -0 sum; this library takes the same path as the
//   reference for every (dtype, C).
//
// Launch shape: a warp computes kFrames consecutive output frames x 64 channels of one
// utterance; lane l holds channel pair l of the slab, so each frame is read and written as
// one coalesced 128-byte row (16-bit types). Groups of 8 warps stage a tile's input frames
// in shared memory once and apply each to every output frame of the tile it reaches; a
// block holds several groups and the activation table they share. Groups take equal
// contiguous runs of the tiles ordered (channel slab, utterance, frame tile): a group
// reloads weights only when its slab changes.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <cstdint>
#include <type_traits>

#include "fga_kernels.h"
#include "host_util.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kConvThreads = 256;
constexpr int kSlabPairs = 32;  // channel pairs per warp tile (64 channels)

template <typename T> struct PairOps;
template <> struct PairOps<__half> {
    using P = __half2;
    static __device__ __forceinline__ P fma(P x, P w, P acc) { return __hfma2(x, w, acc); }
    static __device__ __forceinline__ float2 to_float2(P v) { return __half22float2(v); }
    static __device__ __forceinline__ P from_float2(float a, float b) {
        return __floats2half2_rn(a, b);
    }
    static __device__ __forceinline__ P zero() { return __float2half2_rn(0.0f); }
};
template <> struct PairOps<__nv_bfloat16> {
    using P = __nv_bfloat162;
    static __device__ __forceinline__ P fma(P x, P w, P acc) { return __hfma2(x, w, acc); }
    static __device__ __forceinline__ float2 to_float2(P v) { return __bfloat1622float2(v); }
    static __device__ __forceinline__ P from_float2(float a, float b) {
        return __floats2bfloat162_rn(a, b);
    }
    static __device__ __forceinline__ P zero() { return __float2bfloat162_rn(0.0f); }
};
template <> struct PairOps<float> {
    using P = float2;
    static __device__ __forceinline__ P fma(P x, P w, P acc) {
        return make_float2(fmaf(x.x, w.x, acc.x), fmaf(x.y, w.y, acc.y));
    }
    static __device__ __forceinline__ float2 to_float2(P v) { return v; }
    static __device__ __forceinline__ P from_float2(float a, float b) { return make_float2(a, b); }
    static __device__ __forceinline__ P zero() { return make_float2(0.0f, 0.0f); }
};

// SiLU and Swoosh-R (softplus(v - 1) - 0.08 v - 0.313261687), evaluated in fp32 with the
// same operations as the reference kernels.
enum Activation : int { kSilu = 0, kSwooshR = 1 };

__device__ __forceinline__ float silu(float v) { return v / (1.0f + __expf(-v)); }

__device__ __forceinline__ float swoosh_r(float v) {
    const float shifted = v - 1.0f;
    const float softplus = fmaxf(shifted, 0.0f) + log1pf(__expf(-fabsf(shifted)));
    return softplus - 0.08f * v - 0.313261687f;
}

template <typename T, int kAct>
__device__ __forceinline__ typename PairOps<T>::P activate(typename PairOps<T>::P v) {
    const float2 f = PairOps<T>::to_float2(v);
    if constexpr (kAct == kSilu) return PairOps<T>::from_float2(silu(f.x), silu(f.y));
    else return PairOps<T>::from_float2(swoosh_r(f.x), swoosh_r(f.y));
}

// Activation tables for the 16-bit types. The activation's input is the sum rounded to
// the storage type and its output is rounded to it, so it is a function of 16 bits. A table
// holds it for every magnitude below 2^e_hi (bf16: from 2^-20) of the type: one 32-bit
// entry per magnitude with act(+v) in its low half and act(-v) in its high half.
//   bf16: [2^-20, 2^8), 28 binades x 128 significands =  3584 entries, 14 KB;
//   f16:  [0, 2^4), zero, subnormals and 18 binades    = 19456 entries, 76 KB.
// The ranges reach down far enough that the sums of padded frames (the bias alone) of
// almost every channel are in them: a warp with one lane outside the range evaluates the
// activation for that lane.
// Entries are computed by the same `silu` / `swoosh_r` code the direct path runs, so a
// looked-up value equals the computed one bit for bit. Inputs outside the range (zeros,
// tiny and large magnitudes, inf, NaN) are computed. A block keeps the table in shared
// memory for all of its warps.
//
// Each device holds one copy per (type, activation) in global memory, built by the first
// launch that finds its ready flag clear: every block of that launch computes the table
// itself, writes it to shared memory and to the global copy, and publishes the flag with a
// release store after a fence. Later blocks that read the flag set (acquire) copy the table
// from L2 instead. Concurrent builders write identical values.
template <typename T> struct LutSpec;
template <> struct LutSpec<__nv_bfloat16> {
    static constexpr uint32_t kMant = 7, kExpLo = 107, kExps = 28;  // 107: biased 2^-20
    static __device__ __forceinline__ float to_float(uint32_t bits) {
        return __uint_as_float(bits << 16);
    }
    static __device__ __forceinline__ uint32_t round(float a) {
        return __bfloat16_as_ushort(__float2bfloat16_rn(a));
    }
};
template <> struct LutSpec<__half> {
    static constexpr uint32_t kMant = 10, kExpLo = 0, kExps = 19;  // 0: zero and subnormals
    static __device__ __forceinline__ float to_float(uint32_t bits) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
    }
    static __device__ __forceinline__ uint32_t round(float a) {
        return __half_as_ushort(__float2half_rn(a));
    }
};
template <typename T> struct Lut {
    static constexpr uint32_t kBase = LutSpec<T>::kExpLo << LutSpec<T>::kMant;  // first magnitude
    static constexpr uint32_t kSpan = LutSpec<T>::kExps << LutSpec<T>::kMant;   // entries
    static constexpr int kBytes = static_cast<int>(kSpan) * 4;
};
template <typename T> constexpr int lut_bytes() {
    if constexpr (sizeof(T) == 2) return Lut<T>::kBytes;
    else return 0;
}

__device__ __align__(16) uint32_t g_bf16_act_lut[2][Lut<__nv_bfloat16>::kSpan];
__device__ __align__(16) uint32_t g_f16_act_lut[2][Lut<__half>::kSpan];
__device__ unsigned int g_act_lut_ready[2][2];  // [bf16, f16][activation]

template <typename T> __device__ __forceinline__ uint32_t* global_lut(int act) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) return g_bf16_act_lut[act];
    else return g_f16_act_lut[act];
}
template <typename T> __device__ __forceinline__ unsigned int* lut_ready(int act) {
    return &g_act_lut_ready[std::is_same<T, __nv_bfloat16>::value ? 0 : 1][act];
}

template <typename T, int kAct> __device__ __forceinline__ uint32_t lut_entry(int i) {
    const float v = LutSpec<T>::to_float(Lut<T>::kBase + static_cast<uint32_t>(i));
    const float pos = kAct == kSilu ? silu(v) : swoosh_r(v);
    const float neg = kAct == kSilu ? silu(-v) : swoosh_r(-v);
    return LutSpec<T>::round(pos) | (LutSpec<T>::round(neg) << 16);
}

template <typename T, int kAct>
__device__ __forceinline__ typename PairOps<T>::P activate_lut(typename PairOps<T>::P v,
                                                              const uint32_t* lut) {
    constexpr uint32_t kBase = Lut<T>::kBase, kSpan = Lut<T>::kSpan;
    const uint32_t w = *reinterpret_cast<const uint32_t*>(&v);
    // Both magnitudes less the table base at once: a borrow out of the low half happens only
    // when the low magnitude is below the base, and then the low offset is out of range.
    const uint32_t off = (w & 0x7FFF7FFFu) - kBase * 0x10001u;
    const uint32_t o0 = off & 0xFFFFu, o1 = off >> 16;
    if (o0 < kSpan && o1 < kSpan) {
        // Result bytes 0-1: the half of lut[o0] the low sign picks; bytes 2-3: the half of
        // lut[o1] the high sign picks.
        const uint32_t sel = 0x5410u + (((w >> 14) & 2u) | ((w >> 22) & 0x200u)) * 0x11u;
        const uint32_t r = __byte_perm(lut[o0], lut[o1], sel);
        return *reinterpret_cast<const typename PairOps<T>::P*>(&r);
    }
    return activate<T, kAct>(v);
}

template <typename T> __device__ __forceinline__ typename PairOps<T>::P load_pair(const T* p) {
    return *reinterpret_cast<const typename PairOps<T>::P*>(p);
}

// Frames per warp tile: 16 for the packed 16-bit types, 8 for fp32 (twice the registers
// per pair).
template <typename T> __host__ __device__ constexpr int frames_per_tile() { return sizeof(T) == 4 ? 8 : 16; }

// Shape of the fixed-K kernel for storage type T and kK taps. A group is 8 warps (256
// threads) computing a tile of 64 channels x kTileFrames output frames of one utterance; a
// block holds kGroups groups (four, or three where four would not fit shared memory) and
// the activation table they share. All shared memory is dynamic:
//   [table (16-bit types)] [group 0: kStages input tiles, weights] [group 1 ...] ...
template <typename T, int kK> struct ConvShape {
    using P = typename PairOps<T>::P;
    static constexpr int kFrames = frames_per_tile<T>();       // output frames per warp
    static constexpr int kTileFrames = 8 * kFrames;
    static constexpr int kRows = kTileFrames + kK - 1;           // staged input rows
    static constexpr int kRowBytes = kSlabPairs * static_cast<int>(sizeof(P));
    // 16-bit types stage the next tile while the current one is computed (two buffers);
    // fp32 tiles are twice as large and use one.
    static constexpr int kStages = sizeof(T) == 2 ? 2 : 1;
    static constexpr int kStageBytes = kRows * kRowBytes;
    static constexpr int kGroupBytes = kStages * kStageBytes + kK * kRowBytes;
    static constexpr int kTableBytes = lut_bytes<T>();
    static constexpr int kMaxSmem = 227 * 1024;
    static constexpr int kGroups = kTableBytes + 4 * kGroupBytes <= kMaxSmem ? 4 : 3;
    static constexpr int kThreads = 256 * kGroups;
    static constexpr int kSmemBytes = kTableBytes + kGroups * kGroupBytes;
    static_assert(kSmemBytes <= kMaxSmem, "convolution tile does not fit shared memory");
};

// Compile-time tap count kK (the kernel sizes of the encoders: 9, 15, 31).
//
// One block per SM. Each group of 8 warps runs the tile loop below on its own staging
// buffers and weights, synchronised by its own named barrier, so the groups are as
// independent as separate blocks; they share the activation table, filled once per block.
// Groups take equal contiguous runs of the tiles ordered (channel slab, utterance, frame
// tile). A group stages a tile's input frames (kTileFrames + kK - 1 rows of 64 channels,
// zeros where a frame is padded or outside [0, T)) and the slab's weights, then warp w
// computes kFrames of the output frames with lane l on channel pair l. Taps are the outer
// loop: for tap k output frame j takes staged row j + k, so a warp's rows form a window of
// kFrames that slides by one row per tap (one shared-memory load per tap) and every
// accumulator receives its taps in tap order; each tap's weight is read from shared memory
// (keeping them in registers spilled at the 64 registers per thread that four groups allow).
template <typename T, int kK, int kAct, bool kSkip>
__global__ void __launch_bounds__(ConvShape<T, kK>::kThreads, 1)
depthwise_conv_kernel(const T* __restrict__ x, const int32_t* __restrict__ lens,
                      const T* __restrict__ w, const T* __restrict__ bias, T* __restrict__ y,
                      int batch, int seq, int channels, int tiles, int64_t tasks) {
    using S = ConvShape<T, kK>;
    using Ops = PairOps<T>;
    using P = typename Ops::P;
    constexpr int kFrames = S::kFrames;
    constexpr int kTileFrames = S::kTileFrames;
    constexpr int kRows = S::kRows;
    constexpr int kPad = kK / 2;
    constexpr int kRowBytes = S::kRowBytes;
    constexpr int kChunks = kRowBytes / 16;                      // 16-byte pieces of a row
    constexpr int kChunkElems = 16 / static_cast<int>(sizeof(T));
    constexpr int kStages = S::kStages;
    constexpr int kGroupThreads = 256;
    constexpr bool kLut = sizeof(T) == 2;
    extern __shared__ __align__(16) unsigned char smem[];

    const int tid = threadIdx.x, lane = tid & 31;
    const int group = tid / kGroupThreads, gtid = tid % kGroupThreads, warp = gtid >> 5;
    const uint32_t group_bar = 1 + static_cast<uint32_t>(group);  // 0 is __syncthreads
    uint32_t* const lut = reinterpret_cast<uint32_t*>(smem);
    unsigned char* const s_x = smem + S::kTableBytes + group * S::kGroupBytes;
    unsigned char* const s_w = s_x + kStages * S::kStageBytes;

    const int npairs = channels / 2;
    const int64_t per_slab = static_cast<int64_t>(batch) * tiles;
    const int64_t groups_total = static_cast<int64_t>(gridDim.x) * S::kGroups;
    const int64_t per = (tasks + groups_total - 1) / groups_total;
    const int64_t t_begin = (static_cast<int64_t>(blockIdx.x) * S::kGroups + group) * per;
    const int64_t t_end = t_begin + per < tasks ? t_begin + per : tasks;
    // 16-byte staging needs every row piece aligned: 8 (16-bit) or 4 (fp32) channels.
    const bool vec16 = (channels % kChunkElems) == 0 &&
                       (reinterpret_cast<uintptr_t>(x) & 15u) == 0;

    // A task's (slab, utterance, frame tile): the group's first task is decoded once, each
    // next one is its predecessor advanced by one tile (no division per tile).
    struct Tile {
        int slab, n, f0;
    };
    auto decode = [&](int64_t task) {
        Tile t;
        t.slab = static_cast<int>(task / per_slab);
        const int64_t rem = task - t.slab * per_slab;
        t.n = static_cast<int>(rem / tiles);
        t.f0 = static_cast<int>(rem - static_cast<int64_t>(t.n) * tiles) * kTileFrames;
        return t;
    };
    auto advance = [&](Tile t) {
        t.f0 += kTileFrames;
        if (t.f0 >= tiles * kTileFrames) {
            t.f0 = 0;
            if (++t.n == batch) {
                t.n = 0;
                ++t.slab;
            }
        }
        return t;
    };
    // The tile's input rows (frames f0 - kPad ...) into buffer `buf`: zeros where a frame is
    // padded or outside [0, T). 16-byte asynchronous copies (the zeros by a zero source
    // size), or pair loads and stores when rows are not 16-byte aligned. One commit group.
    auto stage = [&](const Tile& t, int buf) {
        const int requested = __ldg(lens + t.n);
        const int vl = requested < 0 ? 0 : (requested < seq ? requested : seq);
        const T* xb = x + static_cast<int64_t>(t.n) * seq * channels;
        unsigned char* sx = s_x + buf * S::kStageBytes;
        if (vec16) {
            const int c_slab = t.slab * 2 * kSlabPairs;
            for (int i = gtid; i < kRows * kChunks; i += kGroupThreads) {
                const int r = i / kChunks, c = c_slab + (i % kChunks) * kChunkElems;
                const int fi = t.f0 - kPad + r;
                const bool valid = static_cast<unsigned>(fi) < static_cast<unsigned>(vl) &&
                                   c < channels;
                const T* src = valid ? xb + static_cast<int64_t>(fi) * channels + c : x;
                cp_async16_zfill(smem_u32(sx + i * 16), src, valid ? 16u : 0u);
            }
        } else {
            for (int i = gtid; i < kRows * kSlabPairs; i += kGroupThreads) {
                const int r = i / kSlabPairs, q = t.slab * kSlabPairs + i % kSlabPairs;
                const int fi = t.f0 - kPad + r;
                P v = Ops::zero();
                if (static_cast<unsigned>(fi) < static_cast<unsigned>(vl) && q < npairs)
                    v = load_pair(xb + static_cast<int64_t>(fi) * channels + 2 * q);
                *reinterpret_cast<P*>(sx + i * sizeof(P)) = v;
            }
        }
        cp_async_commit();
    };

    P b0 = Ops::zero();
    int cur_slab = -1;
    Tile cur = t_begin < t_end ? decode(t_begin) : Tile{0, 0, 0};
    if (kStages == 2 && t_begin < t_end) stage(cur, 0);
    if constexpr (kLut) {
        // Fill the activation table (under the first tiles' copies), all groups together.
        constexpr int kEntries = static_cast<int>(Lut<T>::kSpan);
        __shared__ unsigned int s_lut_ready;
        if (tid == 0) s_lut_ready = ld_acquire_gpu(lut_ready<T>(kAct));
        __syncthreads();
        const bool ready = s_lut_ready != 0u;
        uint32_t* const glut = global_lut<T>(kAct);
        if (ready) {
            const uint4* src = reinterpret_cast<const uint4*>(glut);
            for (int i = tid; i < Lut<T>::kBytes / 16; i += S::kThreads)
                reinterpret_cast<uint4*>(lut)[i] = __ldcg(src + i);
        } else {
            for (int i = tid; i < kEntries; i += S::kThreads) {
                const uint32_t e = lut_entry<T, kAct>(i);
                lut[i] = e;
                glut[i] = e;
            }
            __threadfence();
        }
        __syncthreads();
        if (!ready && tid == 0) st_release_gpu(lut_ready<T>(kAct), 1u);
    }
    int buf = 0;
    for (int64_t task = t_begin; task < t_end; ++task) {
        const Tile tile = cur;
        const Tile next = advance(cur);
        const int slab = tile.slab, n = tile.n, f0 = tile.f0;
        const int p = slab * kSlabPairs + lane;
        const bool ok = p < npairs;
        const bool new_slab = slab != cur_slab;
        // Every warp of the group finished reading the other buffer and the weights (end of
        // the previous iteration), so they can be refilled.
        const bool prefetch = kStages == 2 && task + 1 < t_end;
        if (prefetch) stage(next, buf ^ 1);
        if (kStages == 1) stage(tile, 0);
        if (new_slab) {
            for (int i = gtid; i < kK * kSlabPairs; i += kGroupThreads) {
                const int k = i / kSlabPairs, q = slab * kSlabPairs + i % kSlabPairs;
                *reinterpret_cast<P*>(s_w + i * sizeof(P)) =
                    q < npairs ? load_pair(w + static_cast<int64_t>(k) * channels + 2 * q)
                               : Ops::zero();
            }
            b0 = ok ? load_pair(bias + 2 * p) : Ops::zero();
        }
        const int requested = __ldg(lens + n);
        const int vl = requested < 0 ? 0 : (requested < seq ? requested : seq);
        if (prefetch) cp_async_wait<1>();  // this tile's group is complete
        else cp_async_wait<0>();
        named_barrier(group_bar, kGroupThreads);
        const int fw = f0 + warp * kFrames;  // this warp's first output frame
        const unsigned char* xs =
            s_x + buf * S::kStageBytes + warp * kFrames * kRowBytes + lane * sizeof(P);
        P acc[kFrames], win[kFrames];
#pragma unroll
        for (int j = 0; j < kFrames; ++j) {
            acc[j] = b0;
            win[j] = *reinterpret_cast<const P*>(xs + j * kRowBytes);
        }
#pragma unroll
        for (int k = 0; k < kK; ++k) {
            const P wk = *reinterpret_cast<const P*>(s_w + k * kRowBytes + lane * sizeof(P));
            // win[(j + k) % kFrames] holds staged row j + k (input frame fw - kPad + j + k).
#pragma unroll
            for (int j = 0; j < kFrames; ++j) {
                const int fi = fw - kPad + j + k;
                if (kSkip && static_cast<unsigned>(fi) >= static_cast<unsigned>(vl)) continue;
                acc[j] = Ops::fma(win[(j + k) % kFrames], wk, acc[j]);
            }
            // Slide: the slot of row k takes row k + kFrames.
            if (k + 1 < kK)
                win[k % kFrames] = *reinterpret_cast<const P*>(xs + (k + kFrames) * kRowBytes);
        }
        if (ok) {
            T* yp = y + (static_cast<int64_t>(n) * seq + fw) * channels + 2 * p;
            // The frame check is hoisted out of the common case (the warp's frames all
            // below T), which leaves the loop with no per-frame range test.
            if (fw + kFrames <= seq) {
#pragma unroll
                for (int j = 0; j < kFrames; ++j) {
                    P out;
                    if constexpr (kLut) out = activate_lut<T, kAct>(acc[j], lut);
                    else out = activate<T, kAct>(acc[j]);
                    *reinterpret_cast<P*>(yp + static_cast<int64_t>(j) * channels) = out;
                }
            } else {
#pragma unroll
                for (int j = 0; j < kFrames; ++j)
                    if (fw + j < seq) {
                        P out;
                        if constexpr (kLut) out = activate_lut<T, kAct>(acc[j], lut);
                        else out = activate<T, kAct>(acc[j]);
                        *reinterpret_cast<P*>(yp + static_cast<int64_t>(j) * channels) = out;
                    }
            }
        }
        cur_slab = slab;
        cur = next;
        named_barrier(group_bar, kGroupThreads);  // this tile's rows and the weights are read
        buf ^= kStages - 1;
    }
    cp_async_wait<0>();  // nothing left in flight (a group with no tile committed none)
}

// Any odd tap count: one output frame pair per thread per step, weights read per tap
// (through L1), the same per-output arithmetic and order.
template <typename T, int kAct, bool kSkip>
__global__ void __launch_bounds__(kConvThreads)
depthwise_conv_any_kernel(const T* __restrict__ x, const int32_t* __restrict__ lens,
                          const T* __restrict__ w, const T* __restrict__ bias, T* __restrict__ y,
                          int batch, int seq, int channels, int taps) {
    using Ops = PairOps<T>;
    using P = typename Ops::P;
    const int npairs = channels / 2;
    const int64_t total = static_cast<int64_t>(batch) * seq * npairs;
    const int pad = taps / 2;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(i % npairs);
        const int64_t frame_index = i / npairs;
        const int f = static_cast<int>(frame_index % seq);
        const int n = static_cast<int>(frame_index / seq);
        const int requested = __ldg(lens + n);
        const int vl = requested < 0 ? 0 : (requested < seq ? requested : seq);
        P acc = load_pair(bias + 2 * p);
        for (int k = 0; k < taps; ++k) {
            const int fi = f + k - pad;
            const bool valid = static_cast<unsigned>(fi) < static_cast<unsigned>(vl);
            if (kSkip && !valid) continue;
            const P xv = valid ? load_pair(x + (static_cast<int64_t>(n) * seq + fi) * channels + 2 * p)
                               : Ops::zero();
            acc = Ops::fma(xv, load_pair(w + static_cast<int64_t>(k) * channels + 2 * p), acc);
        }
        *reinterpret_cast<P*>(y + frame_index * channels + 2 * p) = activate<T, kAct>(acc);
    }
}

// Resident blocks per SM of `kKernel` launched with `threads` threads and `dyn_smem` bytes of
// dynamic shared memory, looked up once per (kernel, device).
template <auto kKernel> int blocks_per_sm(int threads, int dyn_smem = 0) {
    static std::atomic<int> cache[kMaxCachedDevices];
    const auto kernel = kKernel;
    const int dev = current_device();
    if (dev >= 0 && dev < kMaxCachedDevices) {
        if (const int v = cache[dev].load(std::memory_order_relaxed)) return v;
    }
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, threads, dyn_smem) !=
            cudaSuccess ||
        v < 1)
        v = 1;
    if (dev >= 0 && dev < kMaxCachedDevices) cache[dev].store(v, std::memory_order_relaxed);
    return v;
}

template <typename T, int kK, int kAct, bool kSkip>
cudaError_t launch_fixed(const ConvolutionProblem& p, cudaStream_t stream) {
    using S = ConvShape<T, kK>;
    const int tiles = (p.length + S::kTileFrames - 1) / S::kTileFrames;
    const int slabs = (p.channels / 2 + kSlabPairs - 1) / kSlabPairs;
    const int64_t tasks = static_cast<int64_t>(slabs) * p.batch * tiles;
    auto kernel = depthwise_conv_kernel<T, kK, kAct, kSkip>;
    const int sms = sm_count();
    if (sms <= 0) return cudaErrorNotSupported;
    static SmemAttr attr;
    const cudaError_t e = attr.ensure(reinterpret_cast<const void*>(kernel), S::kSmemBytes);
    if (e != cudaSuccess) return e;
    // Enough blocks for every group to have a tile, at most the resident ones.
    int64_t grid = static_cast<int64_t>(sms) *
                   blocks_per_sm<depthwise_conv_kernel<T, kK, kAct, kSkip>>(S::kThreads,
                                                                            S::kSmemBytes);
    const int64_t needed = (tasks + S::kGroups - 1) / S::kGroups;
    if (grid > needed) grid = needed;
    kernel<<<static_cast<unsigned>(grid), S::kThreads, S::kSmemBytes, stream>>>(
        static_cast<const T*>(p.x), p.valid_lengths, static_cast<const T*>(p.weight),
        static_cast<const T*>(p.bias), static_cast<T*>(p.output), p.batch, p.length, p.channels,
        tiles, tasks);
    return cudaGetLastError();
}

template <typename T, int kAct, bool kSkip>
cudaError_t launch_any(const ConvolutionProblem& p, cudaStream_t stream) {
    const int64_t total = static_cast<int64_t>(p.batch) * p.length * (p.channels / 2);
    const int sms = sm_count();
    if (sms <= 0) return cudaErrorNotSupported;
    auto kernel = depthwise_conv_any_kernel<T, kAct, kSkip>;
    int64_t grid =
        static_cast<int64_t>(sms) * blocks_per_sm<depthwise_conv_any_kernel<T, kAct, kSkip>>(kConvThreads);
    const int64_t needed = (total + kConvThreads - 1) / kConvThreads;
    if (grid > needed) grid = needed;
    kernel<<<static_cast<unsigned>(grid), kConvThreads, 0, stream>>>(
        static_cast<const T*>(p.x), p.valid_lengths, static_cast<const T*>(p.weight),
        static_cast<const T*>(p.bias), static_cast<T*>(p.output), p.batch, p.length, p.channels,
        p.taps);
    return cudaGetLastError();
}

template <typename T, int kAct, bool kSkip>
cudaError_t launch_typed(const ConvolutionProblem& p, cudaStream_t stream, const char** variant) {
    switch (p.taps) {
        case 9: *variant = "conv-k9"; return launch_fixed<T, 9, kAct, kSkip>(p, stream);
        case 15: *variant = "conv-k15"; return launch_fixed<T, 15, kAct, kSkip>(p, stream);
        case 31: *variant = "conv-k31"; return launch_fixed<T, 31, kAct, kSkip>(p, stream);
        default: *variant = "conv-any"; return launch_any<T, kAct, kSkip>(p, stream);
    }
}

template <int kAct, bool kSkip>
cudaError_t launch_dtype(const ConvolutionProblem& p, cudaStream_t stream, const char** variant) {
    switch (p.dtype) {
        case 1: return launch_typed<__half, kAct, kSkip>(p, stream, variant);
        case 7: return launch_typed<__nv_bfloat16, kAct, kSkip>(p, stream, variant);
        default: return launch_typed<float, kAct, kSkip>(p, stream, variant);
    }
}

}  // namespace

cudaError_t launch_convolution(const ConvolutionProblem& p, cudaStream_t stream,
                               const char** variant) {
    if (p.kind == ConvolutionProblem::kZipformer) return launch_dtype<kSwooshR, false>(p, stream, variant);
    // The reference's Parakeet kernels multiply padded taps as zeros only in the packed
    // eight-channel path (f16/bf16 with C % 8 == 0); the others skip them.
    const bool zero_taps = p.dtype != 0 && p.channels % 8 == 0;
    return zero_taps ? launch_dtype<kSilu, false>(p, stream, variant)
                     : launch_dtype<kSilu, true>(p, stream, variant);
}

}  // namespace fga
