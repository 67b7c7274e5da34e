// Zipformer relative-position attention weights on tcgen05 tensor cores (f16/bf16, query
// head dim 32): T <= 768 with an exponential cache in TMEM (zipformer_weights_tc_kernel,
// below); 768 < T <= 1536 recomputing the scores (zipformer_weights_long_kernel, at the
// end of the file).
//
// W[n, h, q, k] = softmax_k( round_T(Q[q] . K[k]) + sum_i pq[q,i] * pos[T-1-q+k, i] ),
// masked keys excluded, written as the I/O dtype T in the NHTT layout.
//
// Launch shape: a persistent grid of one CTA per SM. A CTA draws (utterance, head) pairs
// from a work counter and produces all query blocks (128 rows) of the pair, so Q and K of
// the head are loaded once per pair by TMA (SWIZZLE_64B, rows past T read as zero).
// 16 compute warps (four per TMEM lane quarter; the fused variant: 8, two per quarter) + 1
// control warp that issues TMA and MMAs.
//
// TMEM (512 columns, one CTA per SM):
//   [0, 128)    two 64-key score buffers (content scores Q K^T, fp32), filled by the
//               control warp, drained by the compute warps (mbarrier ring);
//   [128, 512)  the row's exponentials as packed f16 pairs, key k at column 128 + k/2.
//
// Per query block (thread = query row, warp sub-slot = which kGroup keys of each chunk:
// 16 in the weights kernel, 32 in the fused one):
//   pass 1: logits -> group max -> exp2(logit - running max) in fp32, summed in fp32 and
//           cached in TMEM as f16 (no logit is computed twice); the running max of every
//           group is kept in shared memory;
//   combine the sub-slots' (max, sum) per row;
//   pass 2: cached exps x exp(group max - row max) / sum -> T, staged per warp in shared
//           memory and written as 16-byte stores aligned to the global NHTT addresses
//           (the row stride T*2 bytes is not 16-byte aligned for the encoder's lengths, so
//           each row's slots are re-aligned from the staging tile with byte permutes; the
//           partial slots at range ends are written element-wise).
//
// Fused variant (kFused, entry point fga_zipformer_attention_fused_enqueue, no reference
// plugin): pass 2 writes each piece of rounded weights into a P tile and the control
// warp multiplies it by both value tensors' V pieces (tcgen05, N = 16 each); O1 and O2
// accumulate in a drained score buffer. The [N, H, T, T] weights are never written, except
// head 0's ([N, 1, T, T], for NonlinAttention), staged per warp in the band region.
//
// Reference semantics (zipformer_relative_attention_plugin.cu:238-327 and 490-566): the
// content score is stored in T by the reference GEMM (rounded here before the fp32
// positional add, accumulated in the same order); max over valid keys; exp(x - max);
// sum > 0 ? e / sum : 0; masked keys weigh 0; rows q >= 7 with mask[q-7] (the padded-
// query halo) are zero; a row with no valid key is zero. The f16 exp cache perturbs a
// weight by at most 2^-11 relative before the final rounding (at most one ulp of the
// output type).
#include <cuda.h>

#include <atomic>
#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "host_util.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kQd = 32;             // query/key head dim served by this kernel
constexpr int kMaxT = 768;          // keys held in shared memory / TMEM cache columns
constexpr int kM = 128;             // query rows per block
constexpr int kChunk = 64;          // keys per MMA (score buffer width)
constexpr int kWord = 32;           // keys per key-validity word
constexpr int kMaxWords = kMaxT / kWord;
constexpr int kHalo = 7;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kCacheCol = 2 * kChunk;
constexpr uint32_t kRowBytes = kQd * 2;  // 64-byte K-major rows (SWIZZLE_64B)

// Positional band, kept in the I/O type (the positions are T values, so this is exact):
// 4 planes (one per positional dim) x 4 copies shifted by 0..3 entries, so that every
// thread reads 4 consecutive keys' values of a plane with one aligned 8-byte load. A
// copy's stride is 16 (mod 64) elements, so the 16 lanes of a load phase (consecutive
// rows, hence consecutive shifts) fall in distinct bank pairs.
constexpr int kPlane = 904;
constexpr int kCopy = 4 * kPlane + 48;
constexpr int kBandFill = kMaxT + kM + 4;  // band entries written per block

// Fused variant (weights applied to two value tensors in the same kernel): pass 2 writes
// each 64-key piece of rounded weights into a P tile (one per warp sub-slot, 128 rows x
// 64 keys, SWIZZLE_128B K-major) and the control warp multiplies it by the head's V
// pieces, which stay resident for the whole pair (64 keys x 16 channels per piece,
// SWIZZLE_32B MN-major, both value tensors).
constexpr int kFusedPiece = 64;
constexpr uint32_t kPTile = kM * kFusedPiece * 2;
constexpr uint32_t kVPiece = kFusedPiece * 16 * 2;
constexpr int kVBox = 256;  // keys per V TMA box (four pieces)
constexpr uint32_t kVTensor = (kMaxT / kFusedPiece) * kVPiece;

// Dynamic pair scheduling: the CTAs draw pairs from one 32-bit counter in the caller's
// workspace, which the launcher zeroes on the launch's stream just before the kernel.

// Work split and shared memory of each variant. kSub compute warps share a TMEM lane
// quarter: in pass 1 each takes kGroup = 64 / kSub keys of every 64-key score chunk, in
// pass 2 a contiguous range of kPiece-key pieces. The weights kernel runs four per quarter
// (16 compute warps: enough warps in flight to hide the TMEM, shared-memory and MUFU
// latencies of both passes) with 32-key pieces; the fused kernel two, with the 64-key
// pieces of its P tiles.
template <bool kFused> struct Cfg {
    static constexpr int kSub = kFused ? 2 : 4;
    static constexpr int kGroup = kChunk / kSub;  // keys per thread group
    static constexpr int kMaxGroups = kMaxT / kGroup;
    static constexpr int kComputeWarps = 4 * kSub;
    static constexpr int kComputeThreads = 32 * kComputeWarps;
    static constexpr int kThreads = kComputeThreads + 32;  // + control warp
    // Pass 2 works in kPiece-key pieces. Per-warp staging tile: 32 rows x (16-byte carry
    // chunk + kPiece keys), rows an odd number of 16-byte chunks long, so row-parallel
    // 16-byte stores are bank-conflict free.
    static constexpr int kPiece = kFused ? kFusedPiece : 32;
    static constexpr int kStageRow = 16 + kPiece * 2;
    static constexpr int kStageWarp = 32 * kStageRow;
    // Shared memory (bytes from the 1024-aligned base). The variant region holds the
    // pass-2 staging tiles (weights kernel) or the P tiles and resident V (fused kernel).
    static constexpr uint32_t kSmemQ = 0;
    static constexpr uint32_t kSmemK = kSmemQ + kMaxT * kRowBytes;
    static constexpr uint32_t kSmemBand = kSmemK + kMaxT * kRowBytes;
    static constexpr uint32_t kSmemHist = kSmemBand + 4u * kCopy * 2u;
    static constexpr uint32_t kSmemStats = kSmemHist + kMaxGroups * kM * 4;
    static constexpr uint32_t kSmemKb = kSmemStats + kSub * kM * 8;        // 2 buffers (pair parity)
    static constexpr uint32_t kSmemValid = kSmemKb + 2 * kMaxT * 4;         // 2 buffers
    static constexpr uint32_t kSmemLive = kSmemValid + 2 * kMaxWords * 4;   // 2 buffers x 8 words
    static constexpr uint32_t kSmemVariant = (kSmemLive + 2 * 8 * 4 + 1023u) & ~1023u;
    static constexpr uint32_t kSmemStage = kSmemVariant;
    static constexpr uint32_t kSmemP = kSmemVariant;
    static constexpr uint32_t kSmemV = kSmemP + kSub * kPTile;  // value v at + v * kVTensor
    // Barriers: [0, 64) shared by both variants; fused adds a_full[2], a_empty[2], v_full,
    // o_full, o_free at [64, 120).
    static constexpr uint32_t bar =
        kFused ? kSmemV + 2 * kVTensor : kSmemStage + kComputeWarps * kStageWarp + 16;
    static constexpr uint32_t bytes = bar + (kFused ? 128u : 64u);
    static_assert(kStageRow % 32 == 16, "staging rows: an odd number of 16-byte chunks");
    static_assert(kPiece == 2 * kGroup, "two thread groups per pass-2 piece");
    static_assert(bytes <= 227 * 1024, "shared memory budget");
    static_assert(kMaxT / kM <= kComputeWarps, "one warp per query block computes its liveness");
};
static_assert(kCopy % 64 == 16, "band copy stride");

// Per-device error word of this file's kernels: 1 = a bounded wait gave up, 2 = the
// dynamic shared memory was not 1024-byte aligned. Read and cleared by fga_device_status.
__device__ unsigned int g_zipformer_tc_error = 0;

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

// a0 += q * lo(w), a1 += q * hi(w): T x T products accumulated in fp32 (exact products,
// the same arithmetic as converting both operands to fp32 first).
template <typename T> __device__ __forceinline__ void fma_pair(float& a0, float& a1, uint16_t q,
                                                               uint32_t w);
template <> __device__ __forceinline__ void fma_pair<__nv_bfloat16>(float& a0, float& a1,
                                                                    uint16_t q, uint32_t w) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "fma.rn.f32.bf16 %0, %3, l, %0;\n\tfma.rn.f32.bf16 %1, %3, h, %1;\n\t}"
        : "+f"(a0), "+f"(a1) : "r"(w), "h"(q));
}
template <> __device__ __forceinline__ void fma_pair<__half>(float& a0, float& a1, uint16_t q,
                                                             uint32_t w) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "fma.rn.f32.f16 %0, %3, l, %0;\n\tfma.rn.f32.f16 %1, %3, h, %1;\n\t}"
        : "+f"(a0), "+f"(a1) : "r"(w), "h"(q));
}

// Round two fp32 values to T and return them as fp32 (a GEMM that writes T).
template <typename T> __device__ __forceinline__ float2 round_pair(float a, float b);
template <> __device__ __forceinline__ float2 round_pair<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    const uint32_t u = *reinterpret_cast<const uint32_t*>(&v);
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}
template <> __device__ __forceinline__ float2 round_pair<__half>(float a, float b) {
    return __half22float2(__floats2half2_rn(a, b));
}

template <typename T> __device__ __forceinline__ uint32_t pack_pair(float a, float b);
template <> __device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack_pair<__half>(float a, float b) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
}

// SWIZZLE_64B K-major descriptor: 64-byte rows, 8-row groups of 512 bytes.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;                     // LBO (unused, swizzled K-major)
    d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;  // SBO: 8 rows x 64 B
    d |= 1ull << 46;
    d |= 4ull << 61;                                          // SWIZZLE_64B
    return d;
}

// Bounded wait with a warp-uniform result; a failure raises the CTA's abort word (the
// CTA then skips all further work but keeps every barrier, so no thread is stranded).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity,
                                          volatile uint32_t* abort, uint64_t limit_ns) {
    bool ok = (*abort == 0u) && mbar_wait(bar, parity, limit_ns);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && (threadIdx.x & 31) == 0) {
        *abort = 1u;
        atomicExch(&g_zipformer_tc_error, 1u);
    }
    return ok;
}

// Fused variant, head 0: one 32-key half (keys k0h..k0h+31) of this warp's 32 rows of the
// [N, 1, T, T] weights, restricted to [kb_w, ke_w). The halves are staged per warp in
// the positional-band region (dead during pass 2): 80-byte rows (an odd number of
// 16-byte chunks, so the row-parallel 16-byte accesses are bank-conflict free) holding
// the previous 8 keys (carry) and the half, then written as 16-byte stores aligned to
// the global addresses, as in pass 2 of the weights kernel.
constexpr int kHalfStageRow = 16 + 32 * 2;
constexpr int kHalfStageWarp = 32 * kHalfStageRow;
static_assert(Cfg<true>::kComputeWarps * kHalfStageWarp + 16 <= 4 * kCopy * 2,
              "head-0 staging fits the band");

template <typename T>
__device__ __forceinline__ void store_head0_half(T* __restrict__ out, uint8_t* stage_w,
                                                 uint4& carry, const uint32_t (&w)[32], int hf,
                                                 int64_t e_base, int seq, int rows_here,
                                                 int k0h, int kb_w, int ke_w, bool last) {
    const int lane = threadIdx.x & 31;
    uint8_t* srow = stage_w + lane * kHalfStageRow;
    *reinterpret_cast<uint4*>(srow) = carry;
#pragma unroll
    for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(srow + 16 + 16 * i) =
            make_uint4(w[16 * hf + 4 * i], w[16 * hf + 4 * i + 1], w[16 * hf + 4 * i + 2],
                       w[16 * hf + 4 * i + 3]);
    carry = make_uint4(w[16 * hf + 12], w[16 * hf + 13], w[16 * hf + 14], w[16 * hf + 15]);
    __syncwarp();
    // Staging element i of a row holds key k0h - 8 + i; slot m starts at key k0h - d + 8m.
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int row = it * 8 + (lane >> 2);
        const int m = lane & 3;
        if (row < rows_here) {
            const int64_t e_row = e_base + static_cast<int64_t>(row) * seq;
            const int d = static_cast<int>(e_row & 7);
            const int lo = k0h - d + 8 * m;
            const uint8_t* sr = stage_w + row * kHalfStageRow;
            if (lo >= kb_w && lo + 8 <= ke_w) {
                const int s0 = 8 - d + 8 * m;
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(sr) + (s0 >> 1);
                const uint32_t a0 = wp[0], a1 = wp[1], a2 = wp[2], a3 = wp[3], a4 = wp[4];
                const uint32_t sel = (s0 & 1) ? 0x5432u : 0x3210u;
                *reinterpret_cast<uint4*>(out + e_row + lo) =
                    make_uint4(__byte_perm(a0, a1, sel), __byte_perm(a1, a2, sel),
                               __byte_perm(a2, a3, sel), __byte_perm(a3, a4, sel));
            } else if (lo + 8 > kb_w && lo < ke_w) {
                const T* se = reinterpret_cast<const T*>(sr);
                for (int k = max(lo, kb_w); k < min(lo + 8, ke_w); ++k)
                    out[e_row + k] = se[k - k0h + 8];
            }
        }
    }
    if (last && lane < rows_here) {
        // Keys after the last slot of the range (slot m = 4, always partial).
        const int64_t e_row = e_base + static_cast<int64_t>(lane) * seq;
        const int d = static_cast<int>(e_row & 7);
        const int lo = k0h - d + 32;
        const T* se = reinterpret_cast<const T*>(srow);
        for (int k = max(lo, kb_w); k < min(lo + 8, ke_w); ++k) out[e_row + k] = se[k - k0h + 8];
    }
    __syncwarp();
}

// kFused = false: the attention weights, written as [N, H, T, T].
// kFused = true: the weights of every head applied to two value
// tensors [N, T, heads * vd] (v1_map, v2_map) into out1 and out2, and, when `out` is not
// null, head 0's weights written as [N, 1, T, T].
template <typename T, bool kFused>
__global__ void __launch_bounds__(Cfg<kFused>::kThreads, 1)
zipformer_weights_tc_kernel(const __grid_constant__ CUtensorMap proj_map,
                            const __grid_constant__ CUtensorMap v1_map,
                            const __grid_constant__ CUtensorMap v2_map,
                            const T* __restrict__ proj, const T* __restrict__ pos,
                            const uint8_t* __restrict__ mask, T* __restrict__ out,
                            T* __restrict__ out1, T* __restrict__ out2, int seq, int heads,
                            int vd, int num_pairs, unsigned int* __restrict__ sched,
                            uint64_t wait_limit) {
    using C = Cfg<kFused>;
    constexpr int kSub = C::kSub, kGroup = C::kGroup;
    constexpr int kComputeWarps = C::kComputeWarps, kComputeThreads = C::kComputeThreads;
    constexpr int kThreads = C::kThreads, kPiece = C::kPiece;
    constexpr int kStageRow = C::kStageRow, kStageWarp = C::kStageWarp;
    constexpr uint32_t kSmemQ = C::kSmemQ, kSmemK = C::kSmemK, kSmemBand = C::kSmemBand;
    constexpr uint32_t kSmemHist = C::kSmemHist, kSmemStats = C::kSmemStats;
    constexpr uint32_t kSmemKb = C::kSmemKb, kSmemValid = C::kSmemValid, kSmemLive = C::kSmemLive;
    constexpr uint32_t kSmemStage = C::kSmemStage, kSmemP = C::kSmemP, kSmemV = C::kSmemV;
    constexpr uint32_t kSmemBar = C::bar;
    // Validity bits of a thread group's keys when all of them are valid.
    constexpr uint32_t kGroupFull = kGroup == 32 ? 0xffffffffu : (1u << kGroup) - 1u;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_kq = sbase + kSmemBar;
    const uint32_t bar_full = sbase + kSmemBar + 8;   // + 8 * buffer
    const uint32_t bar_free = sbase + kSmemBar + 24;  // + 8 * buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + 40);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(smem + kSmemBar + 44);
    uint16_t* band = reinterpret_cast<uint16_t*>(smem + kSmemBand);
    volatile int* next_pair = reinterpret_cast<volatile int*>(smem + kSmemBar + 48);  // [2]
    const uint32_t bar_drain = sbase + kSmemBar + 56;  // teardown: every MMA completed
    // Fused variant only.
    const uint32_t bar_a_full = sbase + kSmemBar + 64;    // + 8 * sub-slot
    const uint32_t bar_a_empty = sbase + kSmemBar + 80;   // + 8 * sub-slot
    const uint32_t bar_v_full = sbase + kSmemBar + 96;
    const uint32_t bar_o_full = sbase + kSmemBar + 104;
    const uint32_t bar_o_free = sbase + kSmemBar + 112;
    float* hist = reinterpret_cast<float*>(smem + kSmemHist);
    float2* stats = reinterpret_cast<float2*>(smem + kSmemStats);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const bool control = warp == kComputeWarps;
    const int qtr = warp & 3;
    const int sub = warp >> 2;
    const int q_local = qtr * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(qtr * 32) << 16;
    const int pdim = heads * (2 * kQd + 4);
    const int ngroups = (seq + kGroup - 1) / kGroup;
    const int nwords = (seq + kWord - 1) / kWord;
    const int nchunks = (seq + kChunk - 1) / kChunk;
    const int nqb = (seq + kM - 1) / kM;
    const int npieces = (seq + kPiece - 1) / kPiece;
    const int split = (npieces + 1) / 2;  // pass-2 piece ranges: [0, split), [split, npieces)

    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_zipformer_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        mbar_init(bar_kq, 1);
        mbar_init(bar_full, 1);
        mbar_init(bar_full + 8, 1);
        mbar_init(bar_free, kComputeWarps);
        mbar_init(bar_free + 8, kComputeWarps);
        mbar_init(bar_drain, 1);
        if constexpr (kFused) {
            for (int i = 0; i < kSub; ++i) {
                mbar_init(bar_a_full + 8 * i, 4);  // the sub-slot's four warps
                mbar_init(bar_a_empty + 8 * i, 1);
            }
            mbar_init(bar_v_full, 1);
            mbar_init(bar_o_full, 1);
            mbar_init(bar_o_free, kComputeWarps);
            prefetch_tensormap(&v1_map);
            prefetch_tensormap(&v2_map);
        }
        *abort = 0u;
        fence_mbar_init();
        prefetch_tensormap(&proj_map);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    uint32_t ucount = 0;    // score-buffer uses so far (both roles count identically)
    // Fused variant: P-tile uses per sub-slot (both roles count identically), the control
    // warp's o_full commits / o_free and v_full waits, and the score buffer holding the
    // accumulators of an output tile whose epilogue has not been waited for (-1: none).
    uint32_t a_uses[kSub] = {0, 0};  // control warp
    uint32_t p_uses = 0;             // compute warp: P tiles of its sub-slot written
    uint32_t o_fulls = 0, o_frees = 0, v_waits = 0;
    int o_buf = -1;
    bool v_pending = false;
    uint32_t kq_phase = 0;  // control warp: Q/K loads waited for so far
    int kq_pair = -1;       // control warp: pair whose Q/K loads are in flight, if any
    // Control warp: TMA loads of Q and K of every query block of pair p.
    auto load_qk = [&](int p) {
        if (lane == 0) {
            const int pn = p / heads, ph = p - pn * heads;
            mbar_expect_tx(bar_kq, 2u * nqb * kM * kRowBytes);
            for (int b = 0; b < nqb; ++b) {
                tma_load_3d(sbase + kSmemQ + b * kM * kRowBytes, &proj_map, bar_kq, ph * kQd,
                            b * kM, pn);
                tma_load_3d(sbase + kSmemK + b * kM * kRowBytes, &proj_map, bar_kq,
                            heads * kQd + ph * kQd, b * kM, pn);
            }
        }
        __syncwarp();
        kq_pair = p;
    };
    // Pair tickets are drawn one pair ahead, so the atomic's round trip overlaps the work.
    if (tid == 0) next_pair[0] = static_cast<int>(atomicAdd(sched, 1u));
#pragma unroll 1
    for (int iter = 0;; ++iter) {
        named_barrier(1, kThreads);
        const int pair = next_pair[iter & 1];
        if (pair >= num_pairs) break;
        // Every thread read slot (iter+1)&1 of the previous pair before this barrier.
        if (tid == 0)
            next_pair[(iter + 1) & 1] = static_cast<int>(atomicAdd(sched, 1u));
        const int n = pair / heads;
        const int h = pair - n * heads;
        const uint8_t* mrow = mask + static_cast<int64_t>(n) * seq;
        const int buf = iter & 1;
        float* kb = reinterpret_cast<float*>(smem + kSmemKb) + buf * kMaxT;
        uint32_t* valid = reinterpret_cast<uint32_t*>(smem + kSmemValid) + buf * kMaxWords;
        uint32_t* live_q = reinterpret_cast<uint32_t*>(smem + kSmemLive) + buf * 8;

        if (!control) {
            // Key validity (bit per key, +-inf bias per key) and query-block liveness. Every
            // mask byte a thread needs is loaded before any is used (one memory round trip).
            constexpr int kWordIters = (kMaxWords + kComputeWarps - 1) / kComputeWarps;
            uint8_t mk[kWordIters], mq[kM / 32];
#pragma unroll
            for (int i = 0; i < kWordIters; ++i) {
                const int k = (warp + i * kComputeWarps) * kWord + lane;
                mk[i] = k < seq ? __ldg(mrow + k) : 1;
            }
#pragma unroll
            for (int i = 0; i < kM / 32; ++i) {
                const int q = warp * kM + lane + 32 * i;
                mq[i] = (warp < nqb && q < seq && q >= kHalo) ? __ldg(mrow + q - kHalo) : 0;
            }
#pragma unroll
            for (int i = 0; i < kWordIters; ++i) {
                const int wd = warp + i * kComputeWarps;
                if (wd < nwords) {
                    const int k = wd * kWord + lane;
                    const bool v = mk[i] == 0;
                    const uint32_t bits = __ballot_sync(0xffffffffu, v);
                    kb[k] = v ? INFINITY : -INFINITY;
                    if (lane == 0) valid[wd] = bits;
                }
            }
            if (warp < nqb) {
                bool any = false;
#pragma unroll
                for (int i = 0; i < kM / 32; ++i) {
                    const int q = warp * kM + lane + 32 * i;
                    any |= q < seq && mq[i] == 0;
                }
                any = __any_sync(0xffffffffu, any);
                if (lane == 0) live_q[warp] = any ? 1u : 0u;
            }
        } else if (ucount > 0) {
            // Q/K of the previous pair are read by its MMAs: wait for the last one.
            const uint32_t u = ucount - 1;
            warp_wait(bar_full + 8 * (u & 1), (u >> 1) & 1, abort, wait_limit);
        }
        named_barrier(1, kThreads);  // mask information of this pair is visible

        bool any_valid = false;
        for (int wd = 0; wd < nwords; ++wd) any_valid |= valid[wd] != 0u;
        // Validity bits of the keys of thread group g (g < ngroups).
        auto group_bits = [&](int g) -> uint32_t {
            if constexpr (kGroup == kWord) return valid[g];
            else return (valid[g / (kWord / kGroup)] >> ((g % (kWord / kGroup)) * kGroup)) &
                        kGroupFull;
        };
        uint32_t live_mask = 0;
        for (int b = 0; b < nqb; ++b)
            if (any_valid && live_q[b] != 0u) live_mask |= 1u << b;

        if (control) {
            // ---- control warp: Q/K loads and the score MMAs of every live block ----
            // The loads were normally issued one pair ahead (end of the previous pair).
            if (kq_pair != pair && live_mask != 0u && __all_sync(0xffffffffu, *abort == 0u))
                load_qk(pair);
            if (kq_pair == pair && warp_wait(bar_kq, kq_phase & 1, abort, wait_limit)) {
                // (After a failed wait the loads stay in flight: teardown drains them.)
                ++kq_phase;
                kq_pair = -1;
            }
            if constexpr (kFused) {
                // The head's V pieces of both value tensors, resident for the pair, once the
                // previous pair's last P.V MMAs have read theirs. They land under pass 1.
                if (live_mask != 0u && __all_sync(0xffffffffu, *abort == 0u)) {
                    bool ok = true;
                    if (o_fulls > 0) ok = warp_wait(bar_o_full, (o_fulls - 1) & 1, abort, wait_limit);
                    if (ok) {
                        if (lane == 0) {
                            const int nvb = (seq + kVBox - 1) / kVBox;
                            const int cb = (h * vd) & ~7;
                            mbar_expect_tx(bar_v_full, 2u * nvb * kVBox * 32u);
                            for (int vb = 0; vb < nvb; ++vb) {
                                tma_load_3d(sbase + kSmemV + vb * kVBox * 32u, &v1_map,
                                            bar_v_full, cb, vb * kVBox, n);
                                tma_load_3d(sbase + kSmemV + kVTensor + vb * kVBox * 32u,
                                            &v2_map, bar_v_full, cb, vb * kVBox, n);
                            }
                        }
                        __syncwarp();
                        v_pending = true;
                    }
                }
            }
            constexpr uint32_t idesc = idesc_f16(Fmt<T>::v, kM, kChunk, 0, 0);
#pragma unroll 1
            for (int b = 0; b < nqb; ++b) {
                if (!((live_mask >> b) & 1u)) continue;
                const uint64_t dq = sw64_desc(sbase + kSmemQ + b * kM * kRowBytes);
#pragma unroll 1
                for (int j = 0; j < nchunks; ++j) {
                    const uint32_t u = ucount + j;
                    const uint32_t sb = u & 1;
                    bool ok = __all_sync(0xffffffffu, *abort == 0u);
                    if (ok && u >= 2) ok = warp_wait(bar_free + 8 * sb, ((u >> 1) - 1) & 1, abort, wait_limit);
                    if constexpr (kFused) {
                        // This buffer holds the accumulators of an earlier output tile.
                        if (ok && static_cast<int>(sb) == o_buf) {
                            ok = warp_wait(bar_o_free, o_frees & 1, abort, wait_limit);
                            ++o_frees;
                            o_buf = -1;
                        }
                    }
                    if (ok) {
                        tc_fence_after();
                        if (elect_one()) {
                            const uint64_t dk = sw64_desc(sbase + kSmemK + j * kChunk * kRowBytes);
                            const uint32_t d = tmem + sb * kChunk;
                            umma_f16_ss(d, dq, dk, idesc, 0);
                            umma_f16_ss(d, dq + 2, dk + 2, idesc, 1);  // second K=16 step
                            umma_commit(bar_full + 8 * sb);
                        }
                        __syncwarp();
                    }
                }
                ucount += nchunks;
                if constexpr (kFused) {
                    // P.V of this block: O1, O2 (16 columns each) accumulate in the score
                    // buffer of the block's last chunk, which pass 1 has drained by the
                    // time the first P tile is full. Steps alternate the two sub-slots.
                    constexpr uint32_t idesc_pv = idesc_f16(Fmt<T>::v, kM, 16, 0, 1);
                    bool ok = __all_sync(0xffffffffu, *abort == 0u);
                    if (ok && o_buf >= 0) {
                        ok = warp_wait(bar_o_free, o_frees & 1, abort, wait_limit);
                        ++o_frees;
                        o_buf = -1;
                    }
                    if (ok && v_pending) {
                        ok = warp_wait(bar_v_full, v_waits & 1, abort, wait_limit);
                        if (ok) {  // otherwise the loads stay in flight: teardown drains them
                            ++v_waits;
                            v_pending = false;
                        }
                    }
                    const uint32_t ob = (ucount & 1u) ^ 1u;
                    const int cnt[kSub] = {split, npieces - split};
                    const int steps = max(cnt[0], cnt[1]);
                    bool first = true;
#pragma unroll 1
                    for (int i = 0; i < steps; ++i) {
#pragma unroll
                        for (int sl = 0; sl < kSub; ++sl) {
                            if (i >= cnt[sl]) continue;
                            const int piece = sl == 0 ? i : split + i;
                            if (ok) ok = warp_wait(bar_a_full + 8 * sl, a_uses[sl] & 1, abort, wait_limit);
                            if (ok) {
                                tc_fence_after();
                                if (elect_one()) {
                                    const uint64_t da =
                                        sw128_desc(sbase + kSmemP + sl * kPTile, 16, 1024);
#pragma unroll
                                    for (int v = 0; v < 2; ++v) {
                                        const uint64_t dv = smem_desc(
                                            sbase + kSmemV + v * kVTensor + piece * kVPiece,
                                            kVPiece, 256, 6);
#pragma unroll
                                        for (uint32_t ks = 0; ks < kPiece / 16; ++ks)
                                            umma_f16_ss(tmem + ob * kChunk + v * 16,
                                                        da + ((ks * 32) >> 4),
                                                        dv + ((ks * 512) >> 4), idesc_pv,
                                                        (first && ks == 0) ? 0u : 1u);
                                    }
                                    umma_commit(bar_a_empty + 8 * sl);
                                }
                                __syncwarp();
                            }
                            ++a_uses[sl];
                            first = false;
                        }
                    }
                    if (elect_one()) umma_commit(bar_o_full);
                    __syncwarp();
                    ++o_fulls;
                    o_buf = static_cast<int>(ob);
                }
            }
            // Once this pair's MMAs have read Q and K, load the next pair's (its ticket was
            // drawn at the start of this pair and published by the barrier above).
            const int nxt = next_pair[(iter + 1) & 1];
            if (nxt < num_pairs && __all_sync(0xffffffffu, *abort == 0u)) {
                bool ok = true;
                if (ucount > 0) {
                    const uint32_t u = ucount - 1;
                    ok = warp_wait(bar_full + 8 * (u & 1), (u >> 1) & 1, abort, wait_limit);
                }
                if (ok) load_qk(nxt);
            }
            continue;
        }

        // ---- compute warps ----
#pragma unroll 1
        for (int b = 0; b < nqb; ++b) {
            const int q0 = b * kM;
            const int q = q0 + q_local;
            const bool block_live = (live_mask >> b) & 1u;
            bool row_live = false;
            float m_fin = -INFINITY, inv = 0.0f;
            if (block_live) {
                named_barrier(2, kComputeThreads);  // previous block's band/cache readers done
                // Positional band of this block: entry i is relative row T-1-q0-127+i. Pass 1
                // reads entries below 127 + kGroup * ngroups.
                const int band_lo = seq - 1 - q0 - (kM - 1);
                const int band_fill = min(kBandFill, kM + ngroups * kGroup + 4);
                // All of this thread's positional rows and its query's positional
                // projection are requested before any is used (one memory round trip).
                constexpr int kBandIters = (kBandFill + kComputeThreads - 1) / kComputeThreads;
                uint2 raw_band[kBandIters];
#pragma unroll
                for (int it = 0; it < kBandIters; ++it) {
                    const int i = tid + it * kComputeThreads;
                    const int rel = band_lo + i;
                    raw_band[it] = make_uint2(0u, 0u);
                    if (i < band_fill && i < seq + kM - 1 && rel >= 0 && rel < 2 * seq - 1)
                        raw_band[it] = __ldg(reinterpret_cast<const uint2*>(
                            pos + (static_cast<int64_t>(rel) * heads + h) * 4));
                }
                uint2 raw_pq = make_uint2(0u, 0u);
                uint8_t halo_mask = 0;
                if (q < seq) {
                    raw_pq = __ldg(reinterpret_cast<const uint2*>(
                        proj + (static_cast<int64_t>(n) * seq + q) * pdim + 2 * heads * kQd + h * 4));
                    if (q >= kHalo) halo_mask = __ldg(mrow + q - kHalo);
                }
#pragma unroll
                for (int it = 0; it < kBandIters; ++it) {
                    const int i = tid + it * kComputeThreads;
                    if (i >= band_fill) break;
                    const uint2 raw = raw_band[it];
                    const uint16_t v[4] = {static_cast<uint16_t>(raw.x & 0xFFFFu),
                                           static_cast<uint16_t>(raw.x >> 16),
                                           static_cast<uint16_t>(raw.y & 0xFFFFu),
                                           static_cast<uint16_t>(raw.y >> 16)};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (i >= c) {
#pragma unroll
                            for (int pl = 0; pl < 4; ++pl)
                                band[c * kCopy + pl * kPlane + i - c] = v[pl];
                        }
                    }
                }
                uint16_t pq[4] = {0, 0, 0, 0};
                if (q < seq) {
                    const uint2 raw = raw_pq;
                    pq[0] = static_cast<uint16_t>(raw.x & 0xFFFFu);
                    pq[1] = static_cast<uint16_t>(raw.x >> 16);
                    pq[2] = static_cast<uint16_t>(raw.y & 0xFFFFu);
                    pq[3] = static_cast<uint16_t>(raw.y >> 16);
                    row_live = halo_mask == 0;
                }
                const bool warp_live = __any_sync(0xffffffffu, row_live);
                named_barrier(3, kComputeThreads);  // band complete
                tc_fence_after();

                // ---- pass 1 ----
                const float2 l2e = make_float2(kLog2e, kLog2e);
                const int prow = (kM - 1) - q_local;
                float m_run = -INFINITY, l_run = 0.0f;
#pragma unroll 1
                for (int j = 0; j < nchunks; ++j) {
                    const uint32_t u = ucount + j;
                    const uint32_t sb = u & 1;
                    const int g = kSub * j + sub;
                    const uint32_t vb = g < ngroups ? group_bits(g) : 0u;
                    const bool math = warp_live && vb != 0u;
                    const bool ok = warp_wait(bar_full + 8 * sb, (u >> 1) & 1, abort, wait_limit);
                    uint32_t r[kGroup];
                    if (ok && math) {
                        tmem_ld_cols(tmem + lane_off + sb * kChunk + sub * kGroup, r);
                        tmem_wait_ld();
                        reg_fence(r);
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_free + 8 * sb);
                    if (!(ok && math)) {
                        if (g < ngroups) hist[g * kM + q_local] = -INFINITY;
                        continue;
                    }
                    float s[kGroup];
#pragma unroll
                    for (int i = 0; i < kGroup / 2; ++i) {
                        const float2 f = round_pair<T>(__uint_as_float(r[2 * i]),
                                                       __uint_as_float(r[2 * i + 1]));
                        s[2 * i] = f.x;
                        s[2 * i + 1] = f.y;
                    }
                    // Positional term, accumulated in the reference's order (dims 0..3).
                    const int b0 = prow + g * kGroup;
                    const int cpy = b0 & 3;
                    const uint16_t* bp = band + cpy * kCopy + (b0 - cpy);
#pragma unroll
                    for (int t = 0; t < kGroup / 4; ++t) {
#pragma unroll
                        for (int pl = 0; pl < 4; ++pl) {
                            const uint2 v = *reinterpret_cast<const uint2*>(bp + pl * kPlane + 4 * t);
                            fma_pair<T>(s[4 * t], s[4 * t + 1], pq[pl], v.x);
                            fma_pair<T>(s[4 * t + 2], s[4 * t + 3], pq[pl], v.y);
                        }
                    }
                    if (vb != kGroupFull) {
                        // Some keys of the group are masked or past T: min with -inf
                        // removes them whatever their score (NaN included).
                        const float* kp = kb + g * kGroup;
#pragma unroll
                        for (int t = 0; t < kGroup / 4; ++t) {
                            const float4 m4 = *reinterpret_cast<const float4*>(kp + 4 * t);
                            s[4 * t] = fminf(s[4 * t], m4.x);
                            s[4 * t + 1] = fminf(s[4 * t + 1], m4.y);
                            s[4 * t + 2] = fminf(s[4 * t + 2], m4.z);
                            s[4 * t + 3] = fminf(s[4 * t + 3], m4.w);
                        }
                    }
                    // Group max and sum as trees (four independent chains each), so the
                    // dependent-instruction latency does not serialise the group's keys.
                    float m4[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) m4[i] = s[i];
#pragma unroll
                    for (int t = 1; t + 1 < kGroup / 4; t += 2) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) m4[i] = fmax3(m4[i], s[i + 4 * t], s[i + 4 * t + 4]);
                    }
                    if constexpr ((kGroup / 4) % 2 == 0) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) m4[i] = fmaxf(m4[i], s[i + kGroup - 4]);
                    }
                    const float gm = fmaxf(fmax3(m4[0], m4[1], m4[2]), m4[3]);
                    const float m_new = fmaxf(m_run, gm);
                    const float mb = m_new == -INFINITY ? 0.0f : m_new * kLog2e;
                    const float2 nb = make_float2(-mb, -mb);
                    float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                                     make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
                    uint32_t c16[kGroup / 2];
#pragma unroll
                    for (int i = 0; i < kGroup / 2; ++i) {
                        const float2 x = __ffma2_rn(make_float2(s[2 * i], s[2 * i + 1]), l2e, nb);
                        const float e0 = fast_exp2(x.x), e1 = fast_exp2(x.y);
                        acc[i & 3] = __fadd2_rn(acc[i & 3], make_float2(e0, e1));
                        c16[i] = pack_half2(e0, e1);
                    }
                    const float2 accs = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
                    const float alpha =
                        m_run == m_new ? 1.0f : fast_exp2((m_run - m_new) * kLog2e);
                    l_run = fmaf(l_run, alpha, accs.x + accs.y);
                    m_run = m_new;
                    hist[g * kM + q_local] = m_new;
                    tmem_st_cols(tmem + lane_off + kCacheCol + g * (kGroup / 2), c16);
                }
                ucount += nchunks;
                tmem_wait_st();
                stats[sub * kM + q_local] = make_float2(m_run, l_run);
                tc_fence_before();
                named_barrier(4, kComputeThreads);  // stats and the exp cache complete
                tc_fence_after();
                float l_fin = 0.0f;
#pragma unroll
                for (int s2 = 0; s2 < kSub; ++s2) m_fin = fmaxf(m_fin, stats[s2 * kM + q_local].x);
#pragma unroll
                for (int s2 = 0; s2 < kSub; ++s2) {
                    const float2 st = stats[s2 * kM + q_local];
                    l_fin += st.y * (st.x == m_fin ? 1.0f : fast_exp2((st.x - m_fin) * kLog2e));
                }
                // sum > 0 ? e / sum : 0 (no valid key, all -inf, NaN or +inf logits -> 0)
                inv = l_fin > 0.0f ? 1.0f / l_fin : 0.0f;
                row_live = row_live && inv > 0.0f;
            }

            // Fused: this warp's value tensor (sub-slot 0: first, 1: second) and its output
            // row; the head's vd channels start `och` columns into its 16-column tile.
            T* const orow = sub == 0 ? out1 : out2;
            const int64_t orow_off = (static_cast<int64_t>(n) * seq + q) * heads * vd + h * vd;
            const int och = h * vd - ((h * vd) & ~7);
            const bool write_w0 = kFused && h == 0 && out != nullptr;
            const int64_t e0_base = (static_cast<int64_t>(n) * seq + q0 + qtr * 32) * seq;
            uint8_t* const stage_h0 = smem + kSmemBand + warp * kHalfStageWarp;
            if constexpr (kFused) {
                if (!block_live) {
                    // No live row: the block's outputs are zero (rows past T excluded).
                    if (q < seq)
                        for (int cpair = 0; 2 * cpair < vd; ++cpair)
                            *reinterpret_cast<uint32_t*>(orow + orow_off + 2 * cpair) = 0u;
                    if (write_w0) {
                        const int p_lo = sub == 0 ? 0 : split;
                        const int p_hi = sub == 0 ? split : npieces;
                        const int rows_here = min(32, seq - (q0 + qtr * 32));
                        uint32_t zw[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) zw[i] = 0u;
                        uint4 zc = make_uint4(0u, 0u, 0u, 0u);
                        for (int pc = p_lo; pc < p_hi; ++pc)
#pragma unroll
                            for (int hf = 0; hf < 2; ++hf)
                                store_head0_half<T>(out, stage_h0, zc, zw, hf, e0_base, seq,
                                                    rows_here, pc * kPiece + 32 * hf,
                                                    p_lo * kPiece, min(p_hi * kPiece, seq),
                                                    pc + 1 == p_hi && hf == 1);
                    }
                    continue;
                }
            }

            // ---- pass 2: this warp writes keys [kb_w, ke_w) of its 32 rows ----
            const bool all_live = __all_sync(0xffffffffu, row_live);
            const bool use_tmem = block_live && __any_sync(0xffffffffu, row_live) &&
                                  __all_sync(0xffffffffu, *abort == 0u);
            const int p_lo = (sub * npieces + kSub - 1) / kSub;
            const int p_hi = ((sub + 1) * npieces + kSub - 1) / kSub;
            const int kb_w = p_lo * kPiece;
            const int ke_w = min(p_hi * kPiece, seq);
            const int rows_here = min(32, seq - (q0 + qtr * 32));
            const int64_t e_base =
                (static_cast<int64_t>(n * heads + h) * seq + q0 + qtr * 32) * seq;
            uint8_t* stage_w = smem + kSmemStage + warp * kStageWarp;
            uint8_t* srow = stage_w + lane * kStageRow;
            auto group_valid = [&](int g) { return g < ngroups && group_bits(g) != 0u; };
            auto piece_cached = [&](int pc) {
                return use_tmem && (group_valid(2 * pc) || group_valid(2 * pc + 1));
            };
            constexpr int kGw = kGroup / 2;  // cache words (f16 pairs) of a thread group
            uint32_t c[kPiece / 2];
            if (p_lo < p_hi && piece_cached(p_lo))
                tmem_ld_cols(tmem + lane_off + kCacheCol + p_lo * (kPiece / 2), c);
            uint4 carry = make_uint4(0u, 0u, 0u, 0u);
            // Staging element i of a row holds key k0 - 8 + i. A slot is an 8-element run
            // whose start is 16-byte aligned in the output; slot m of a piece starts at key
            // k0 - d + 8m, d = (row's element offset) mod 8. Each lane writes one slot of
            // kRowSlots rows (kRowSlots lanes cover a row). What a lane's slots need that
            // does not change from piece to piece is computed once per block: the slot's
            // element offset from the block's first output element at piece 0, the
            // staging word it starts in and the byte selector of its re-alignment.
            constexpr int kRowSlots = kPiece / 8;
            int slot_off[kRowSlots];
            uint32_t slot_word[kRowSlots], slot_sel[kRowSlots];
            uint32_t slot_live = 0;
            if constexpr (!kFused) {
#pragma unroll
                for (int it = 0; it < kRowSlots; ++it) {
                    const int row = it * (32 / kRowSlots) + lane / kRowSlots;
                    const int m = lane % kRowSlots;
                    const int d = static_cast<int>((e_base + static_cast<int64_t>(row) * seq) & 7);
                    const int s0 = 8 - d + 8 * m;
                    slot_off[it] = row * seq - d + 8 * m;
                    slot_word[it] = static_cast<uint32_t>(row * kStageRow) / 4u + (s0 >> 1);
                    slot_sel[it] = (s0 & 1) ? 0x5432u : 0x3210u;
                    if (row < rows_here) slot_live |= 1u << it;
                }
            }
#pragma unroll 1
            for (int pc = p_lo; pc < p_hi; ++pc) {
                const int k0 = pc * kPiece;
                uint32_t w[kPiece / 2];
                if (piece_cached(pc)) {
                    tmem_wait_ld();
                    reg_fence(c);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int g = 2 * pc + half;
                        if (group_valid(g)) {
                            const float hm = hist[g * kM + q_local];
                            const float scale =
                                row_live ? fast_exp2((hm - m_fin) * kLog2e) * inv : 0.0f;
                            const float2 sc = make_float2(scale, scale);
#pragma unroll
                            for (int i = 0; i < kGw; ++i) {
                                const float2 f = __fmul2_rn(unpack_half2(c[kGw * half + i]), sc);
                                w[kGw * half + i] = pack_pair<T>(f.x, f.y);
                            }
                            if (!all_live) {
#pragma unroll
                                for (int i = 0; i < kGw; ++i)
                                    w[kGw * half + i] = row_live ? w[kGw * half + i] : 0u;
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < kGw; ++i) w[kGw * half + i] = 0u;
                        }
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < kPiece / 2; ++i) w[i] = 0u;
                }
                // Next piece's exps are read from TMEM while this one is written out.
                if (pc + 1 < p_hi && piece_cached(pc + 1))
                    tmem_ld_cols(tmem + lane_off + kCacheCol + (pc + 1) * (kPiece / 2), c);
                if constexpr (kFused) {
                    // The piece's rounded weights go to this sub-slot's P tile (row q_local,
                    // keys k0..k0+63) once the control warp's previous P.V has read it.
                    if (p_uses > 0) warp_wait(bar_a_empty + 8 * sub, (p_uses - 1) & 1, abort, wait_limit);
                    uint8_t* pt = smem + kSmemP + sub * kPTile;
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *reinterpret_cast<uint4*>(pt + sw128_offset(q_local, i)) =
                            make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_a_full + 8 * sub);
                    ++p_uses;
                    if (write_w0) {
                        // Head 0's weights of the same piece, for NonlinAttention.
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf)
                            store_head0_half<T>(out, stage_h0, carry, w, hf, e0_base, seq,
                                                rows_here, k0 + 32 * hf, kb_w, ke_w,
                                                pc + 1 == p_hi && hf == 1);
                    }
                    continue;
                }
                *reinterpret_cast<uint4*>(srow) = carry;
#pragma unroll
                for (int i = 0; i < kPiece / 8; ++i)
                    *reinterpret_cast<uint4*>(srow + 16 + 16 * i) =
                        make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                carry = make_uint4(w[kPiece / 2 - 4], w[kPiece / 2 - 3], w[kPiece / 2 - 2],
                                   w[kPiece / 2 - 1]);
                __syncwarp();
                if (pc > p_lo && pc + 1 < p_hi) {
                    // An inner piece of the range: every slot lies inside [kb_w, ke_w).
                    const uint32_t* sw = reinterpret_cast<const uint32_t*>(stage_w);
                    T* const ob = out + e_base + k0;
#pragma unroll
                    for (int it = 0; it < kRowSlots; ++it) {
                        if ((slot_live >> it) & 1u) {
                            const uint32_t* wp = sw + slot_word[it];
                            const uint32_t a0 = wp[0], a1 = wp[1], a2 = wp[2], a3 = wp[3], a4 = wp[4];
                            const uint32_t sel = slot_sel[it];
                            *reinterpret_cast<uint4*>(ob + slot_off[it]) =
                                make_uint4(__byte_perm(a0, a1, sel), __byte_perm(a1, a2, sel),
                                           __byte_perm(a2, a3, sel), __byte_perm(a3, a4, sel));
                        }
                    }
                    __syncwarp();
                    continue;
                }
#pragma unroll
                for (int it = 0; it < kRowSlots; ++it) {
                    const int row = it * (32 / kRowSlots) + lane / kRowSlots;
                    const int m = lane % kRowSlots;
                    if (row < rows_here) {
                        const int64_t e_row = e_base + static_cast<int64_t>(row) * seq;
                        const int d = static_cast<int>(e_row & 7);
                        const int lo = k0 - d + 8 * m;
                        const uint8_t* sr = stage_w + row * kStageRow;
                        if (lo >= kb_w && lo + 8 <= ke_w) {
                            const int s0 = 8 - d + 8 * m;
                            const uint32_t* wp = reinterpret_cast<const uint32_t*>(sr) + (s0 >> 1);
                            const uint32_t a0 = wp[0], a1 = wp[1], a2 = wp[2], a3 = wp[3], a4 = wp[4];
                            const uint32_t sel = (s0 & 1) ? 0x5432u : 0x3210u;
                            const uint4 o = make_uint4(__byte_perm(a0, a1, sel), __byte_perm(a1, a2, sel),
                                                       __byte_perm(a2, a3, sel), __byte_perm(a3, a4, sel));
                            *reinterpret_cast<uint4*>(out + e_row + lo) = o;
                        } else if (lo + 8 > kb_w && lo < ke_w) {
                            const T* se = reinterpret_cast<const T*>(sr);
                            for (int k = max(lo, kb_w); k < min(lo + 8, ke_w); ++k)
                                out[e_row + k] = se[k - k0 + 8];
                        }
                    }
                }
                if (pc + 1 == p_hi && lane < rows_here) {
                    // Keys after the last slot of the range (slot m = kRowSlots, always partial).
                    const int64_t e_row = e_base + static_cast<int64_t>(lane) * seq;
                    const int d = static_cast<int>(e_row & 7);
                    const int lo = k0 - d + kPiece;
                    const T* se = reinterpret_cast<const T*>(srow);
                    for (int k = max(lo, kb_w); k < min(lo + 8, ke_w); ++k)
                        out[e_row + k] = se[k - k0 + 8];
                }
                __syncwarp();
            }
            if constexpr (kFused) {
                // O row of this warp's value tensor: accumulator columns of the block's last
                // score buffer, rounded to T like the attention-value plugin's output.
                const uint32_t ocol = ((ucount & 1u) ^ 1u) * kChunk + sub * 16;
                const bool ok = warp_wait(bar_o_full, o_fulls & 1, abort, wait_limit);
                ++o_fulls;
                uint32_t r[16];
                if (ok) {
                    tc_fence_after();
                    tmem_ld16(tmem + lane_off + ocol, r);
                    tmem_wait_ld();
                    reg_fence(r);
                    if (q < seq) {
#pragma unroll
                        for (int cpair = 0; cpair < 8; ++cpair) {
                            if (2 * cpair >= vd) break;
                            // och is 0 or 4 (vd is a multiple of 4).
                            const float a = __uint_as_float(
                                och == 0 ? r[2 * cpair] : r[(2 * cpair + 4) & 15]);
                            const float b2 = __uint_as_float(
                                och == 0 ? r[2 * cpair + 1] : r[(2 * cpair + 5) & 15]);
                            *reinterpret_cast<uint32_t*>(orow + orow_off + 2 * cpair) =
                                pack_pair<T>(a, b2);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_o_free);
            }
            tc_fence_before();
        }
    }

    // Teardown, with the default time limit whatever the launch's: the control warp waits
    // for every MMA it issued (one commit tracks them all, so MMAs skipped after an abort
    // do not matter) before TMEM is freed, and for TMA loads still in flight (only after
    // an abort) before shared memory is.
    if (control) {
        bool ok = true;
        if (elect_one()) {
            umma_commit(bar_drain);
            ok = mbar_wait(bar_drain, 0);
        }
        __syncwarp();
        if (kq_pair >= 0) ok = mbar_wait(bar_kq, kq_phase & 1) && ok;
        if constexpr (kFused) {
            if (v_pending) ok = mbar_wait(bar_v_full, v_waits & 1) && ok;
        }
        if (!ok) atomicExch(&g_zipformer_tc_error, 1u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---- long rows: 768 < T <= 1536 ----------------------------------------------------------------
// The exponential cache of zipformer_weights_tc_kernel needs T/2 TMEM columns next to the
// 128 score columns, so it ends at T = 768. Past it this kernel keeps nothing per key: each
// query block's score MMAs run twice. Pass 1 reduces every row to its running max and sum;
// pass 2 recomputes the same logits (the same code, so the same values), writes
// exp(logit - max) / sum rounded to T, and never caches a key. K of the head stays in shared
// memory for the pair (T x 64 bytes); Q is loaded per block into two alternating buffers.
// Pass 2 stores 64-key pieces: the two warps of a TMEM lane quarter each form one 32-key
// half of the piece into a shared staging tile (two tiles alternate per chunk), meet at a
// 64-thread named barrier, and write half of the tile's rows each with 16-byte stores
// aligned to the global addresses, as the short-row kernel does.
namespace lg {
constexpr int kMaxT = 1536;
constexpr int kSub = 2;                     // compute warps per lane quarter: 32-key groups
constexpr int kGroup = kChunk / kSub;
constexpr int kComputeWarps = 4 * kSub;
constexpr int kComputeThreads = 32 * kComputeWarps;
constexpr int kThreads = kComputeThreads + 32;
constexpr int kMaxWords = kMaxT / kWord;
constexpr int kBandFill = kMaxT + kM + 4;
constexpr int kPlane = 1672;                // >= kBandFill
constexpr int kCopy = 4 * kPlane + 48;
constexpr int kPiece = kChunk;
constexpr int kStageRow = 16 + kPiece * 2;  // 9 x 16 bytes (odd: conflict-free row stores)
constexpr int kStageTile = 32 * kStageRow;  // one lane quarter's 32 rows
constexpr uint32_t kTmemCols = 128;         // two 64-key score buffers
constexpr uint32_t kSmemK = 0;
constexpr uint32_t kSmemQ = kSmemK + kMaxT * kRowBytes;                // 2 buffers
constexpr uint32_t kSmemBand = kSmemQ + 2 * kM * kRowBytes;
constexpr uint32_t kSmemKb = kSmemBand + 4u * kCopy * 2u;              // 2 buffers (pair parity)
constexpr uint32_t kSmemValid = kSmemKb + 2 * kMaxT * 4;
constexpr uint32_t kSmemLive = kSmemValid + 2 * kMaxWords * 4;
constexpr uint32_t kSmemStats = kSmemLive + 2 * 16 * 4;               // [2 subs][rows]
constexpr uint32_t kSmemStage = (kSmemStats + kSub * kM * 8 + 15u) & ~15u;  // [4][2] tiles
constexpr uint32_t kSmemBar = kSmemStage + 4 * 2 * kStageTile + 16;
constexpr uint32_t kBytes = kSmemBar + 128;
static_assert(kPlane >= kBandFill && kCopy % 64 == 16, "positional band layout");
static_assert(kBytes <= 227 * 1024, "shared memory budget");
static_assert(kMaxT / kM <= 16, "block liveness words");
}  // namespace lg

template <typename T>
__global__ void __launch_bounds__(lg::kThreads, 1)
zipformer_weights_long_kernel(const __grid_constant__ CUtensorMap proj_map,
                              const T* __restrict__ proj, const T* __restrict__ pos,
                              const uint8_t* __restrict__ mask, T* __restrict__ out, int seq,
                              int heads, int num_pairs, unsigned int* __restrict__ sched,
                              uint64_t wait_limit) {
    // This kernel's sizes (they shadow the short-row kernel's of the same names).
    constexpr int kMaxT = lg::kMaxT, kSub = lg::kSub, kGroup = lg::kGroup;
    constexpr int kComputeWarps = lg::kComputeWarps, kComputeThreads = lg::kComputeThreads;
    constexpr int kThreads = lg::kThreads, kMaxWords = lg::kMaxWords, kBandFill = lg::kBandFill;
    constexpr int kPlane = lg::kPlane, kCopy = lg::kCopy, kPiece = lg::kPiece;
    constexpr int kStageRow = lg::kStageRow, kStageTile = lg::kStageTile;
    constexpr uint32_t kTmemCols = lg::kTmemCols;
    constexpr uint32_t kSmemK = lg::kSmemK, kSmemQ = lg::kSmemQ, kSmemBand = lg::kSmemBand;
    constexpr uint32_t kSmemKb = lg::kSmemKb, kSmemValid = lg::kSmemValid, kSmemLive = lg::kSmemLive;
    constexpr uint32_t kSmemStats = lg::kSmemStats, kSmemStage = lg::kSmemStage;
    constexpr uint32_t kSmemBar = lg::kSmemBar;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_k = sbase + kSmemBar;          // K of the pair
    const uint32_t bar_q = sbase + kSmemBar + 8;      // + 8 * Q buffer
    const uint32_t bar_full = sbase + kSmemBar + 24;  // + 8 * score buffer
    const uint32_t bar_free = sbase + kSmemBar + 40;  // + 8 * score buffer
    const uint32_t bar_drain = sbase + kSmemBar + 56;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + 64);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(smem + kSmemBar + 68);
    volatile int* next_pair = reinterpret_cast<volatile int*>(smem + kSmemBar + 72);  // [2]
    uint16_t* band = reinterpret_cast<uint16_t*>(smem + kSmemBand);
    float2* stats = reinterpret_cast<float2*>(smem + kSmemStats);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const bool control = warp == kComputeWarps;
    const int qtr = warp & 3;
    const int sub = warp >> 2;
    const int q_local = qtr * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(qtr * 32) << 16;
    const int pdim = heads * (2 * kQd + 4);
    const int ngroups = (seq + kGroup - 1) / kGroup;
    const int nwords = (seq + kWord - 1) / kWord;
    const int nchunks = (seq + kChunk - 1) / kChunk;
    const int nqb = (seq + kM - 1) / kM;

    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_zipformer_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        mbar_init(bar_k, 1);
        mbar_init(bar_q, 1);
        mbar_init(bar_q + 8, 1);
        mbar_init(bar_full, 1);
        mbar_init(bar_full + 8, 1);
        mbar_init(bar_free, kComputeWarps);
        mbar_init(bar_free + 8, kComputeWarps);
        mbar_init(bar_drain, 1);
        *abort = 0u;
        fence_mbar_init();
        prefetch_tensormap(&proj_map);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    uint32_t ucount = 0;                  // score-buffer uses (both roles count identically)
    uint32_t k_phase = 0, q_loads[2] = {0, 0}, q_waits[2] = {0, 0};  // control warp
    bool k_pending = false;
    int qi = 0;                           // control warp: live blocks of the run so far
    int prefetched = -1;                  // control warp: block whose Q is already loading
    uint32_t pieces = 0;                  // compute warps: pass-2 pieces written so far
    auto load_q = [&](int b, int pn, int ph) {
        const int qs = qi & 1;  // the buffer the next live block uses
        if (lane == 0) {
            mbar_expect_tx(bar_q + 8 * qs, kM * kRowBytes);
            tma_load_3d(sbase + kSmemQ + qs * kM * kRowBytes, &proj_map, bar_q + 8 * qs, ph * kQd,
                        b * kM, pn);
        }
        __syncwarp();
        ++q_loads[qs];
    };
    // Waits for the MMA that used score-buffer slot u (the control warp's own commits).
    auto wait_use = [&](uint32_t u) {
        return warp_wait(bar_full + 8 * (u & 1), (u >> 1) & 1, abort, wait_limit);
    };

    if (tid == 0) next_pair[0] = static_cast<int>(atomicAdd(sched, 1u));
#pragma unroll 1
    for (int iter = 0;; ++iter) {
        named_barrier(1, kThreads);
        const int pair = next_pair[iter & 1];
        if (pair >= num_pairs) break;
        if (tid == 0) next_pair[(iter + 1) & 1] = static_cast<int>(atomicAdd(sched, 1u));
        const int n = pair / heads;
        const int h = pair - n * heads;
        const uint8_t* mrow = mask + static_cast<int64_t>(n) * seq;
        const int buf = iter & 1;
        float* kb = reinterpret_cast<float*>(smem + kSmemKb) + buf * kMaxT;
        uint32_t* valid = reinterpret_cast<uint32_t*>(smem + kSmemValid) + buf * kMaxWords;
        uint32_t* live_q = reinterpret_cast<uint32_t*>(smem + kSmemLive) + buf * 16;
        if (!control) {
            for (int wd = warp; wd < nwords; wd += kComputeWarps) {
                const int k = wd * kWord + lane;
                const bool v = k < seq && __ldg(mrow + k) == 0;
                const uint32_t bits = __ballot_sync(0xffffffffu, v);
                kb[k] = v ? INFINITY : -INFINITY;
                if (lane == 0) valid[wd] = bits;
            }
            for (int b = warp; b < nqb; b += kComputeWarps) {
                bool any = false;
#pragma unroll
                for (int i = 0; i < kM / 32; ++i) {
                    const int q = b * kM + lane + 32 * i;
                    any |= q < seq && (q < kHalo || __ldg(mrow + q - kHalo) == 0);
                }
                any = __any_sync(0xffffffffu, any);
                if (lane == 0) live_q[b] = any ? 1u : 0u;
            }
        } else if (ucount > 0) {
            wait_use(ucount - 1);  // K and both Q buffers are free after the last MMA
        }
        named_barrier(1, kThreads);  // mask information of this pair is visible

        bool any_valid = false;
        for (int wd = 0; wd < nwords; ++wd) any_valid |= valid[wd] != 0u;
        uint32_t live_mask = 0;
        for (int b = 0; b < nqb; ++b)
            if (any_valid && live_q[b] != 0u) live_mask |= 1u << b;

        if (control) {
            // ---- control warp: K of the pair, Q per live block, two rounds of score MMAs ----
            if (live_mask != 0u && __all_sync(0xffffffffu, *abort == 0u)) {
                if (lane == 0) {
                    mbar_expect_tx(bar_k, nqb * kM * kRowBytes);
                    for (int b = 0; b < nqb; ++b)
                        tma_load_3d(sbase + kSmemK + b * kM * kRowBytes, &proj_map, bar_k,
                                    heads * kQd + h * kQd, b * kM, n);
                }
                __syncwarp();
                k_pending = true;
            }
            constexpr uint32_t idesc = idesc_f16(Fmt<T>::v, kM, kChunk, 0, 0);
            prefetched = -1;
#pragma unroll 1
            for (int b = 0; b < nqb; ++b) {
                if (!((live_mask >> b) & 1u)) continue;
                bool ok = __all_sync(0xffffffffu, *abort == 0u);
                if (ok && prefetched != b) load_q(b, n, h);  // the pair's first live block
                const int qs = qi & 1;
                // The next live block's Q goes to the other buffer, once the MMAs of the block
                // that used it last have completed.
                int nb = b + 1;
                while (nb < nqb && !((live_mask >> nb) & 1u)) ++nb;
                if (ok && nb < nqb) {
                    if (ucount > 0) ok = wait_use(ucount - 1);
                    if (ok) {
                        ++qi;
                        load_q(nb, n, h);
                        --qi;
                        prefetched = nb;
                    }
                }
                if (ok && k_pending) {
                    ok = warp_wait(bar_k, k_phase & 1, abort, wait_limit);
                    if (ok) {
                        ++k_phase;
                        k_pending = false;
                    }
                }
                if (ok) {
                    ok = warp_wait(bar_q + 8 * qs, q_waits[qs] & 1, abort, wait_limit);
                    if (ok) ++q_waits[qs];
                }
                const uint64_t dq = sw64_desc(sbase + kSmemQ + qs * kM * kRowBytes);
#pragma unroll 1
                for (int pass = 0; pass < 2; ++pass) {
#pragma unroll 1
                    for (int j = 0; j < nchunks; ++j) {
                        const uint32_t u = ucount++;
                        const uint32_t sb = u & 1;
                        bool go = ok && __all_sync(0xffffffffu, *abort == 0u);
                        if (go && u >= 2)
                            go = warp_wait(bar_free + 8 * sb, ((u >> 1) - 1) & 1, abort, wait_limit);
                        if (go) {
                            tc_fence_after();
                            if (elect_one()) {
                                const uint64_t dk = sw64_desc(sbase + kSmemK + j * kChunk * kRowBytes);
                                const uint32_t d = tmem + sb * kChunk;
                                umma_f16_ss(d, dq, dk, idesc, 0);
                                umma_f16_ss(d, dq + 2, dk + 2, idesc, 1);
                                umma_commit(bar_full + 8 * sb);
                            }
                            __syncwarp();
                        }
                    }
                }
                ++qi;
            }
            continue;
        }

        // ---- compute warps ----
#pragma unroll 1
        for (int b = 0; b < nqb; ++b) {
            const int q0 = b * kM;
            const int q = q0 + q_local;
            const bool block_live = (live_mask >> b) & 1u;
            bool row_live = false;
            float inv = 0.0f, mlog = 0.0f;
            uint16_t pq[4] = {0, 0, 0, 0};
            bool warp_live = false;
            if (block_live) {
                named_barrier(2, kComputeThreads);  // previous block's band readers done
                const int band_lo = seq - 1 - q0 - (kM - 1);
                const int band_fill = min(kBandFill, kM + ngroups * kGroup + 4);
                constexpr int kBandIters = (kBandFill + kComputeThreads - 1) / kComputeThreads;
                uint2 raw_band[kBandIters];
#pragma unroll
                for (int it = 0; it < kBandIters; ++it) {
                    const int i = tid + it * kComputeThreads;
                    const int rel = band_lo + i;
                    raw_band[it] = make_uint2(0u, 0u);
                    if (i < band_fill && i < seq + kM - 1 && rel >= 0 && rel < 2 * seq - 1)
                        raw_band[it] = __ldg(reinterpret_cast<const uint2*>(
                            pos + (static_cast<int64_t>(rel) * heads + h) * 4));
                }
                uint2 raw_pq = make_uint2(0u, 0u);
                uint8_t halo_mask = 0;
                if (q < seq) {
                    raw_pq = __ldg(reinterpret_cast<const uint2*>(
                        proj + (static_cast<int64_t>(n) * seq + q) * pdim + 2 * heads * kQd + h * 4));
                    if (q >= kHalo) halo_mask = __ldg(mrow + q - kHalo);
                }
#pragma unroll
                for (int it = 0; it < kBandIters; ++it) {
                    const int i = tid + it * kComputeThreads;
                    if (i >= band_fill) break;
                    const uint2 raw = raw_band[it];
                    const uint16_t v[4] = {static_cast<uint16_t>(raw.x & 0xFFFFu),
                                           static_cast<uint16_t>(raw.x >> 16),
                                           static_cast<uint16_t>(raw.y & 0xFFFFu),
                                           static_cast<uint16_t>(raw.y >> 16)};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (i >= c) {
#pragma unroll
                            for (int pl = 0; pl < 4; ++pl)
                                band[c * kCopy + pl * kPlane + i - c] = v[pl];
                        }
                    }
                }
                if (q < seq) {
                    pq[0] = static_cast<uint16_t>(raw_pq.x & 0xFFFFu);
                    pq[1] = static_cast<uint16_t>(raw_pq.x >> 16);
                    pq[2] = static_cast<uint16_t>(raw_pq.y & 0xFFFFu);
                    pq[3] = static_cast<uint16_t>(raw_pq.y >> 16);
                    row_live = halo_mask == 0;
                }
                warp_live = __any_sync(0xffffffffu, row_live);
                named_barrier(3, kComputeThreads);  // band complete
                tc_fence_after();
            }
            const int prow = (kM - 1) - q_local;
            // Logits of this thread's 32-key group g from the content scores r (the same code
            // in both passes, so both passes see the same values).
            auto logits = [&](int g, uint32_t vb, const uint32_t (&r)[32], float (&s)[32]) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float2 f = round_pair<T>(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
                    s[2 * i] = f.x;
                    s[2 * i + 1] = f.y;
                }
                const int b0 = prow + g * kGroup;
                const int cpy = b0 & 3;
                const uint16_t* bp = band + cpy * kCopy + (b0 - cpy);
#pragma unroll
                for (int t = 0; t < 8; ++t) {
#pragma unroll
                    for (int pl = 0; pl < 4; ++pl) {
                        const uint2 v = *reinterpret_cast<const uint2*>(bp + pl * kPlane + 4 * t);
                        fma_pair<T>(s[4 * t], s[4 * t + 1], pq[pl], v.x);
                        fma_pair<T>(s[4 * t + 2], s[4 * t + 3], pq[pl], v.y);
                    }
                }
                if (vb != 0xffffffffu) {
                    const float* kp = kb + g * kGroup;
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const float4 m4 = *reinterpret_cast<const float4*>(kp + 4 * t);
                        s[4 * t] = fminf(s[4 * t], m4.x);
                        s[4 * t + 1] = fminf(s[4 * t + 1], m4.y);
                        s[4 * t + 2] = fminf(s[4 * t + 2], m4.z);
                        s[4 * t + 3] = fminf(s[4 * t + 3], m4.w);
                    }
                }
            };
            // The content scores of use u for this thread's group; false: no math needed.
            auto scores = [&](uint32_t u, bool math, uint32_t (&r)[32]) {
                const uint32_t sb = u & 1;
                const bool ok = warp_wait(bar_full + 8 * sb, (u >> 1) & 1, abort, wait_limit);
                if (ok && math) {
                    tmem_ld32(tmem + lane_off + sb * kChunk + sub * kGroup, r);
                    tmem_wait_ld();
                    reg_fence(r);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_free + 8 * sb);
                return ok && math;
            };

            if (block_live) {
                // ---- pass 1: running max and sum of every row ----
                const float2 l2e = make_float2(kLog2e, kLog2e);
                float m_run = -INFINITY, l_run = 0.0f;
#pragma unroll 1
                for (int j = 0; j < nchunks; ++j) {
                    const int g = 2 * j + sub;
                    const uint32_t vb = g < ngroups ? valid[g] : 0u;
                    uint32_t r[32];
                    if (!scores(ucount + j, warp_live && vb != 0u, r)) continue;
                    float s[32];
                    logits(g, vb, r, s);
                    float m4[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) m4[i] = fmax3(s[i], s[i + 4], s[i + 8]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) m4[i] = fmax3(m4[i], s[i + 12], s[i + 16]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) m4[i] = fmax3(m4[i], s[i + 20], s[i + 24]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) m4[i] = fmaxf(m4[i], s[i + 28]);
                    const float m_new = fmaxf(m_run, fmaxf(fmax3(m4[0], m4[1], m4[2]), m4[3]));
                    const float mb = m_new == -INFINITY ? 0.0f : m_new * kLog2e;
                    const float2 nb = make_float2(-mb, -mb);
                    float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                                     make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = __ffma2_rn(make_float2(s[2 * i], s[2 * i + 1]), l2e, nb);
                        acc[i & 3] = __fadd2_rn(acc[i & 3], make_float2(fast_exp2(x.x), fast_exp2(x.y)));
                    }
                    const float2 accs =
                        __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
                    const float alpha = m_run == m_new ? 1.0f : fast_exp2((m_run - m_new) * kLog2e);
                    l_run = fmaf(l_run, alpha, accs.x + accs.y);
                    m_run = m_new;
                }
                ucount += nchunks;
                stats[sub * kM + q_local] = make_float2(m_run, row_live ? l_run : 0.0f);
                named_barrier(4, kComputeThreads);  // both sub-slots' statistics written
                float m_fin = -INFINITY, l_fin = 0.0f;
#pragma unroll
                for (int s2 = 0; s2 < kSub; ++s2) m_fin = fmaxf(m_fin, stats[s2 * kM + q_local].x);
#pragma unroll
                for (int s2 = 0; s2 < kSub; ++s2) {
                    const float2 st = stats[s2 * kM + q_local];
                    l_fin += st.y * (st.x == m_fin ? 1.0f : fast_exp2((st.x - m_fin) * kLog2e));
                }
                inv = l_fin > 0.0f ? 1.0f / l_fin : 0.0f;
                row_live = row_live && inv > 0.0f;
                mlog = m_fin == -INFINITY ? 0.0f : m_fin * kLog2e;
                named_barrier(4, kComputeThreads);  // statistics read before the next block
            }

            // ---- pass 2: recompute the logits, normalise, write 64-key pieces ----
            const int rows_here = min(32, seq - (q0 + qtr * 32));
            const int64_t e_base =
                (static_cast<int64_t>(n * heads + h) * seq + q0 + qtr * 32) * seq;
            uint4 carry = make_uint4(0u, 0u, 0u, 0u);  // sub-slot 1: last 8 keys of the previous piece
#pragma unroll 1
            for (int j = 0; j < nchunks; ++j, ++pieces) {
                const int k0 = j * kPiece;
                const int g = 2 * j + sub;
                const uint32_t vb = g < ngroups ? valid[g] : 0u;
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = 0u;
                if (block_live) {
                    uint32_t r[32];
                    if (scores(ucount + j, warp_live && vb != 0u, r) && row_live) {
                        float s[32];
                        logits(g, vb, r, s);
                        const float2 l2e = make_float2(kLog2e, kLog2e);
                        const float2 nb = make_float2(-mlog, -mlog);
                        const float2 sc = make_float2(inv, inv);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float2 x = __ffma2_rn(make_float2(s[2 * i], s[2 * i + 1]), l2e, nb);
                            const float2 e = __fmul2_rn(make_float2(fast_exp2(x.x), fast_exp2(x.y)), sc);
                            w[i] = pack_pair<T>(e.x, e.y);
                        }
                    }
                }
                // Stage this warp's half of the piece (sub-slot 1 adds the carry), then write
                // half of the quarter's rows each.
                // The two tiles alternate over every piece of the run (blocks included), so a
                // tile is refilled only after both warps have passed the next piece's barrier.
                uint8_t* tile = smem + kSmemStage + (qtr * 2 + (pieces & 1u)) * kStageTile;
                uint8_t* srow = tile + lane * kStageRow;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    *reinterpret_cast<uint4*>(srow + 16 + 64 * sub + 16 * i) =
                        make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                if (sub == 1) {
                    *reinterpret_cast<uint4*>(srow) = carry;
                    carry = make_uint4(w[12], w[13], w[14], w[15]);
                }
                named_barrier(5 + qtr, 64);  // both halves of the quarter's piece are staged
#pragma unroll
                for (int it = 4 * sub; it < 4 * sub + 4; ++it) {
                    const int row = it * 4 + (lane >> 3);
                    const int m = lane & 7;
                    if (row < rows_here) {
                        const int64_t e_row = e_base + static_cast<int64_t>(row) * seq;
                        const int d = static_cast<int>(e_row & 7);
                        const int lo = k0 - d + 8 * m;
                        const uint8_t* sr = tile + row * kStageRow;
                        if (lo >= 0 && lo + 8 <= seq) {
                            const int s0 = 8 - d + 8 * m;
                            const uint32_t* wp = reinterpret_cast<const uint32_t*>(sr) + (s0 >> 1);
                            const uint32_t a0 = wp[0], a1 = wp[1], a2 = wp[2], a3 = wp[3], a4 = wp[4];
                            const uint32_t sel = (s0 & 1) ? 0x5432u : 0x3210u;
                            *reinterpret_cast<uint4*>(out + e_row + lo) =
                                make_uint4(__byte_perm(a0, a1, sel), __byte_perm(a1, a2, sel),
                                           __byte_perm(a2, a3, sel), __byte_perm(a3, a4, sel));
                        } else if (lo + 8 > 0 && lo < seq) {
                            const T* se = reinterpret_cast<const T*>(sr);
                            for (int k = max(lo, 0); k < min(lo + 8, seq); ++k)
                                out[e_row + k] = se[k - k0 + 8];
                        }
                    }
                }
                if (j + 1 == nchunks && lane < 16 && 16 * sub + lane < rows_here) {
                    // Keys after the last slot of the row (slot m = 8, always partial).
                    const int row = 16 * sub + lane;
                    const int64_t e_row = e_base + static_cast<int64_t>(row) * seq;
                    const int d = static_cast<int>(e_row & 7);
                    const int lo = k0 - d + kPiece;
                    const T* se = reinterpret_cast<const T*>(tile + row * kStageRow);
                    for (int k = max(lo, 0); k < min(lo + 8, seq); ++k) out[e_row + k] = se[k - k0 + 8];
                }
            }
            if (block_live) ucount += nchunks;
            tc_fence_before();
        }
    }

    // Teardown, with the default time limit whatever the launch's: the control warp waits
    // for every MMA it issued and for loads still in flight (only after an abort).
    if (control) {
        bool ok = true;
        if (elect_one()) {
            umma_commit(bar_drain);
            ok = mbar_wait(bar_drain, 0);
        }
        __syncwarp();
        if (k_pending) ok = mbar_wait(bar_k, k_phase & 1) && ok;
        for (int s2 = 0; s2 < 2; ++s2)
            if (q_loads[s2] > q_waits[s2]) ok = mbar_wait(bar_q + 8 * s2, q_waits[s2] & 1) && ok;
        if (!ok) atomicExch(&g_zipformer_tc_error, 1u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---- host side ------------------------------------------------------------------------------
CUtensorMapDataType map_type(int32_t dtype) {
    return dtype == FGA_HALF ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Projection map: Q and K rows of one head, 128 rows per box, SWIZZLE_64B.
bool encode_proj_map(EncodeTiledFn encode, CUtensorMap* map, const void* proj, int32_t dtype,
                     int batch, int seq, int heads) {
    const uint64_t pdim = static_cast<uint64_t>(heads) * (2 * kQd + 4);
    const cuuint64_t dims[3] = {pdim, static_cast<cuuint64_t>(seq), static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[2] = {pdim * 2, pdim * 2 * seq};
    const cuuint32_t box[3] = {kQd, kM, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return encode(map, map_type(dtype), 3, const_cast<void*>(proj), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// Value map [N, T, H*vd]: boxes of 16 channels x 256 keys, SWIZZLE_32B (MN-major pieces).
bool encode_value_map(EncodeTiledFn encode, CUtensorMap* map, const void* value, int32_t dtype,
                      int batch, int seq, int channels) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(channels), static_cast<cuuint64_t>(seq),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(channels) * 2,
                                   static_cast<cuuint64_t>(channels) * 2 * seq};
    const cuuint32_t box[3] = {16, kVBox, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return encode(map, map_type(dtype), 3, const_cast<void*>(value), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

template <typename T, bool kFused>
cudaError_t set_smem_attr() {
    static SmemAttr attr;
    return attr.ensure(reinterpret_cast<const void*>(zipformer_weights_tc_kernel<T, kFused>),
                       static_cast<int>(Cfg<kFused>::bytes));
}

// The work counter starts at zero for every launch: a 4-byte memset on the same stream,
// ordered before the kernel (and captured with it in a CUDA graph).
cudaError_t zero_counter(unsigned int* sched, cudaStream_t stream) {
    return cudaMemsetAsync(sched, 0, sizeof(unsigned int), stream);
}

template <typename T>
cudaError_t weights_tc_typed(const ZipformerWeightsProblem& p, cudaStream_t stream) {
    EncodeTiledFn encode = encode_fn();
    if (encode == nullptr) return cudaErrorNotSupported;
    CUtensorMap map, unused{};
    if (!encode_proj_map(encode, &map, p.projection, p.dtype, p.batch, p.length, p.heads))
        return cudaErrorNotSupported;
    if (cudaError_t e = set_smem_attr<T, false>(); e != cudaSuccess) return e;
    const int64_t pairs = static_cast<int64_t>(p.batch) * p.heads;
    const int sms = sm_count();
    if (sms <= 0) return cudaErrorNotSupported;
    const int grid = static_cast<int>(pairs < sms ? pairs : sms);
    if (cudaError_t e = zero_counter(p.sched, stream); e != cudaSuccess) return e;
    zipformer_weights_tc_kernel<T, false><<<grid, Cfg<false>::kThreads, Cfg<false>::bytes, stream>>>(
        map, unused, unused, static_cast<const T*>(p.projection),
        static_cast<const T*>(p.position), p.mask, static_cast<T*>(p.weights), nullptr, nullptr,
        p.length, p.heads, 0, static_cast<int>(pairs), p.sched, wait_limit_ns());
    return cudaGetLastError();
}

template <typename T>
cudaError_t weights_long_typed(const ZipformerWeightsProblem& p, cudaStream_t stream) {
    EncodeTiledFn encode = encode_fn();
    if (encode == nullptr) return cudaErrorNotSupported;
    CUtensorMap map;
    if (!encode_proj_map(encode, &map, p.projection, p.dtype, p.batch, p.length, p.heads))
        return cudaErrorNotSupported;
    static SmemAttr attr;
    if (cudaError_t e = attr.ensure(reinterpret_cast<const void*>(zipformer_weights_long_kernel<T>),
                                    static_cast<int>(lg::kBytes));
        e != cudaSuccess)
        return e;
    const int64_t pairs = static_cast<int64_t>(p.batch) * p.heads;
    const int sms = sm_count();
    if (sms <= 0) return cudaErrorNotSupported;
    const int grid = static_cast<int>(pairs < sms ? pairs : sms);
    if (cudaError_t e = zero_counter(p.sched, stream); e != cudaSuccess) return e;
    zipformer_weights_long_kernel<T><<<grid, lg::kThreads, lg::kBytes, stream>>>(
        map, static_cast<const T*>(p.projection), static_cast<const T*>(p.position), p.mask,
        static_cast<T*>(p.weights), p.length, p.heads, static_cast<int>(pairs), p.sched,
        wait_limit_ns());
    return cudaGetLastError();
}

template <typename T>
cudaError_t fused_tc_typed(const ZipformerFusedProblem& p, cudaStream_t stream) {
    EncodeTiledFn encode = encode_fn();
    if (encode == nullptr) return cudaErrorNotSupported;
    const int channels = p.heads * p.value_dim;
    CUtensorMap map, v1, v2;
    if (!encode_proj_map(encode, &map, p.projection, p.dtype, p.batch, p.length, p.heads) ||
        !encode_value_map(encode, &v1, p.value1, p.dtype, p.batch, p.length, channels) ||
        !encode_value_map(encode, &v2, p.value2, p.dtype, p.batch, p.length, channels))
        return cudaErrorNotSupported;
    if (cudaError_t e = set_smem_attr<T, true>(); e != cudaSuccess) return e;
    const int64_t pairs = static_cast<int64_t>(p.batch) * p.heads;
    const int sms = sm_count();
    if (sms <= 0) return cudaErrorNotSupported;
    const int grid = static_cast<int>(pairs < sms ? pairs : sms);
    if (cudaError_t e = zero_counter(p.sched, stream); e != cudaSuccess) return e;
    zipformer_weights_tc_kernel<T, true><<<grid, Cfg<true>::kThreads, Cfg<true>::bytes, stream>>>(
        map, v1, v2, static_cast<const T*>(p.projection), static_cast<const T*>(p.position),
        p.mask, static_cast<T*>(p.weights0), static_cast<T*>(p.output1),
        static_cast<T*>(p.output2), p.length, p.heads, p.value_dim, static_cast<int>(pairs),
        p.sched, wait_limit_ns());
    return cudaGetLastError();
}

}  // namespace

uint32_t take_zipformer_tc_error(cudaStream_t stream, bool clear, cudaError_t* err) {
    return take_error_word(g_zipformer_tc_error, stream, clear, err);
}

// Scratch of fga_zipformer_relative_attention_enqueue_no_workspace, for callers that cannot
// allocate device memory: the weights kernel's work counter lives here instead of in a
// caller-provided workspace. Every device that loads the library holds these bytes until
// the process exits, and every call of that entry point on a device shares them, so two
// such calls must not overlap on the GPU (the counter would be shared).
static __device__ __align__(256) unsigned char g_no_workspace_scratch[FGA_NO_WORKSPACE_SCRATCH_BYTES];

// Device address of the scratch on the current device. The name above is a host-side
// stand-in, not a device address, so the address is looked up with cudaGetSymbolAddress,
// once per device with that device current, and cached (devices past the cache are looked
// up on every call).
cudaError_t no_workspace_scratch(void** ptr) {
    static std::atomic<void*> cache[kMaxCachedDevices];
    const int dev = current_device();
    if (dev < 0) return cudaErrorNoDevice;
    if (dev < kMaxCachedDevices) {
        if (void* p = cache[dev].load(std::memory_order_acquire)) {
            *ptr = p;
            return cudaSuccess;
        }
    }
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_no_workspace_scratch);
    if (e != cudaSuccess) return e;
    if (dev < kMaxCachedDevices) cache[dev].store(p, std::memory_order_release);
    *ptr = p;
    return cudaSuccess;
}

cudaError_t launch_zipformer_weights_tc(const ZipformerWeightsProblem& p, cudaStream_t stream) {
    if (p.query_dim != kQd || (p.dtype != FGA_HALF && p.dtype != FGA_BF16))
        return cudaErrorNotSupported;
    if (p.length > lg::kMaxT || p.length < 1) return cudaErrorNotSupported;
    if (static_cast<int64_t>(p.batch) * p.heads > (1ll << 30)) return cudaErrorNotSupported;
    // TMA needs 16-byte row strides (H * (2*32+4) * 2 bytes = 136 H) and a 16-byte aligned
    // base; the aligned row writes need a 16-byte aligned output.
    const int64_t row_bytes = static_cast<int64_t>(p.heads) * (2 * kQd + 4) * 2;
    if (row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(p.projection) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.weights) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.position) & 7u) != 0)
        return cudaErrorNotSupported;
    if (p.length > kMaxT)  // past the exponential cache: two rounds of score MMAs
        return p.dtype == FGA_HALF ? weights_long_typed<__half>(p, stream)
                                   : weights_long_typed<__nv_bfloat16>(p, stream);
    return p.dtype == FGA_HALF ? weights_tc_typed<__half>(p, stream)
                               : weights_tc_typed<__nv_bfloat16>(p, stream);
}

cudaError_t launch_zipformer_fused(const ZipformerFusedProblem& p, cudaStream_t stream) {
    if (p.query_dim != kQd || (p.dtype != FGA_HALF && p.dtype != FGA_BF16))
        return cudaErrorNotSupported;
    if (p.length > kMaxT || p.length < 1) return cudaErrorNotSupported;
    if (static_cast<int64_t>(p.batch) * p.heads > (1ll << 30)) return cudaErrorNotSupported;
    // One 16-channel V atom per head: vd a multiple of 4 up to 16 puts the head's channels
    // at offset 0 or 4 of the atom that starts at its first channel rounded down to 8.
    if (p.value_dim < 4 || p.value_dim > 16 || p.value_dim % 4 != 0) return cudaErrorNotSupported;
    const int64_t row_bytes = static_cast<int64_t>(p.heads) * (2 * kQd + 4) * 2;
    const int64_t v_row_bytes = static_cast<int64_t>(p.heads) * p.value_dim * 2;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if (row_bytes % 16 != 0 || v_row_bytes % 16 != 0 || !a16(p.projection) || !a16(p.value1) ||
        !a16(p.value2) || (reinterpret_cast<uintptr_t>(p.output1) & 3u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.output2) & 3u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.position) & 7u) != 0 ||
        (p.weights0 != nullptr && !a16(p.weights0)))
        return cudaErrorNotSupported;
    return p.dtype == FGA_HALF ? fused_tc_typed<__half>(p, stream)
                               : fused_tc_typed<__nv_bfloat16>(p, stream);
}

}  // namespace fga
