// Zipformer attention-value on tcgen05 tensor cores (f16/bf16):
//   out[n, q, h*hd + d] = sum_k A[n, ha, q, k] * V[n, k, h*hd + d],   ha = (heads == 1 ? 0 : h)
//
// A persistent, warp-specialized streaming kernel (one CTA per SM). A tile is 128 query
// rows of one (utterance n, value head h); the CTAs take tiles in a static stride and run
// one continuous pipeline over their tiles' 64-key chunks:
//
//   warp 0      A producer: the attention rows are the dominant HBM stream. Their NHTT row
//               stride (T*2 bytes) is not 16-byte aligned for the encoder's lengths, but
//               rows R and R+8 of the flattened [N*Ha*T, T] tensor are 16*T bytes apart.
//               So the rows are split into 8 residue classes (R mod 8), each described by
//               its own 2-D tensor map (16-byte aligned base, row stride 16*T bytes, the
//               class's row start at element offset (r*T) mod 8). One TMA box of 16 rows x
//               (64*S + 8) elements per class fetches the segments of S consecutive 64-key
//               chunks of 16 rows (8 boxes per super-chunk of 128 rows; S = 3 for narrow
//               value tiles, 1 when the V tiles are wide) into a raw staging ring, several
//               super-chunks ahead. Wide boxes keep the number of TMA row requests low.
//   warps 1-4   repack: one thread per row. Shift the row segment into place (by its class
//               offset) and write it into a K-major tile without swizzle (8x16-byte core
//               matrices, 8-row groups 1040 bytes apart, so both the staging reads and the
//               tile writes are bank-conflict free).
//   warps 7-10  epilogue: after the last chunk of a tile, read the accumulator from TMEM
//               and store the head's output columns, while the next tile streams in.
//   warp 5      MMA issuer; warp 6 V producer. V arrives by TMA as MN-major SWIZZLE_128B
//               tiles of 64 channels starting at the head's first channel (rounded down
//               to 8), so a self-attention head (12 channels) needs one 64-wide tile and
//               the NonlinAttention value (3E/4 channels, head 0) ceil(C/64) of them.
//               Accumulators (fp32, TMEM) are double-buffered across tiles when they fit.
//
// All waits are bounded; a timeout raises the CTA's abort word, after which every role
// skips its work but keeps its loop, so nothing waits on a role that has stopped.
// Reference: zipformer_attention_value_plugin.cu:118-181 (fp32 accumulation; one value
// head consumes attention head 0, :85).
#include <cuda.h>

#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;        // query rows per tile
constexpr int kKc = 64;        // keys per chunk (one 128-byte swizzle atom of A)
constexpr int kThreads = 352;  // 11 warps
constexpr int kMaxCpad = 512;  // TMEM columns
// Raw staging for a super-chunk of S 64-key chunks: per row a TMA box row of 64*S + 8
// elements (the class offset is at most 7), 16 rows per residue class, 8 classes.
__host__ __device__ constexpr uint32_t raw_row_bytes(int sup) { return (64u * sup + 8u) * 2u; }
__host__ __device__ constexpr uint32_t raw_stage_bytes(int sup) { return 128u * raw_row_bytes(sup); }
constexpr uint32_t kSbo = 1040;               // 8-row core-matrix groups (16 mod 128)
constexpr uint32_t kATile = 16 * kSbo;        // 128 rows x 64 keys, no swizzle
constexpr uint32_t kVAtom = kKc * 128;        // 8 KB: 64 keys x 64 channels
constexpr uint32_t kSmemLimit = 227 * 1024;

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
    uint32_t sup, raw_row, raw_stage, raw_stages, v_stages, acc_bufs;
    uint32_t raw0, a0, v0, vstage, bar, bytes, tmem_cols;
};

__host__ __device__ constexpr uint32_t pow2_cols(uint32_t n) {
    return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512;
}

// Shared-memory plan for `cpad` accumulator columns: narrow V tiles (cpad <= 128) get
// 3-chunk super-chunks in a 3-deep raw ring; wide ones single chunks in a 4-deep ring
// (2 when needed); then two A tiles and up to 4 V stages in what is left.
__host__ __device__ constexpr Layout make_layout(int cpad) {
    Layout l{};
    l.vstage = static_cast<uint32_t>(cpad / 64) * kVAtom;
    l.sup = cpad <= 128 ? 3 : 1;
    l.raw_row = raw_row_bytes(static_cast<int>(l.sup));
    l.raw_stage = raw_stage_bytes(static_cast<int>(l.sup));
    l.raw_stages = l.sup == 3 ? 3 : 4;
    uint32_t fixed = l.raw_stages * l.raw_stage + 2 * kATile + 1024 + 256;
    l.v_stages = (kSmemLimit - fixed) / l.vstage;
    if (l.v_stages < 2) {
        l.raw_stages = 2;
        fixed = l.raw_stages * l.raw_stage + 2 * kATile + 1024 + 256;
        l.v_stages = (kSmemLimit - fixed) / l.vstage;
    }
    if (l.v_stages > 4) l.v_stages = 4;
    l.acc_bufs = 2 * cpad <= kMaxCpad ? 2 : 1;
    l.raw0 = 0;
    l.a0 = l.raw_stages * l.raw_stage;
    l.v0 = (l.a0 + 2 * kATile + 1023u) & ~1023u;  // SWIZZLE_128B atoms: 1024-byte aligned
    l.bar = l.v0 + l.v_stages * l.vstage;
    l.bytes = l.bar + 256;
    l.tmem_cols = pow2_cols(l.acc_bufs * cpad);
    return l;
}

struct Bars {  // mbarrier addresses (shared window)
    uint32_t base;
    __device__ uint32_t raw_full(uint32_t s) const { return base + 8 * s; }
    __device__ uint32_t raw_empty(uint32_t s) const { return base + 32 + 8 * s; }
    __device__ uint32_t a_full(uint32_t t) const { return base + 64 + 8 * t; }
    __device__ uint32_t a_empty(uint32_t t) const { return base + 80 + 8 * t; }
    __device__ uint32_t v_full(uint32_t s) const { return base + 96 + 8 * s; }
    __device__ uint32_t v_empty(uint32_t s) const { return base + 128 + 8 * s; }
    __device__ uint32_t acc_full(uint32_t b) const { return base + 160 + 8 * b; }
    __device__ uint32_t acc_empty(uint32_t b) const { return base + 176 + 8 * b; }
};

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

// One tensor map per residue class r = R mod 8 of the flattened attention rows.
struct AMaps {
    CUtensorMap m[8];
};

// Element offset of a row start inside its class's 16-byte aligned map row.
__device__ __forceinline__ int class_offset(int r, int seq) { return (r * seq) & 7; }

// K-major, no swizzle: core matrices of 8 rows x 16 bytes; LBO = next core matrix along K
// (128 bytes), SBO = next 8-row group (kSbo).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((128u >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((kSbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;  // version; layout type 0 = no swizzle
    return d;
}

// Byte offset of 16-byte chunk cc (8 keys) of row j in the A tile.
__device__ __forceinline__ uint32_t a_offset(int j, int cc) {
    return static_cast<uint32_t>(j >> 3) * kSbo + static_cast<uint32_t>(cc) * 128u +
           static_cast<uint32_t>(j & 7) * 16u;
}

struct TileInfo {
    int n, h, q0;
};

__device__ __forceinline__ TileInfo tile_info(int tile, int heads, int nqb) {
    TileInfo t;
    t.q0 = (tile % nqb) * kM;
    const int nh = tile / nqb;
    t.h = nh % heads;
    t.n = nh / heads;
    return t;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
zipformer_value_tc_kernel(const __grid_constant__ CUtensorMap v_map,
                          const __grid_constant__ AMaps a_maps, T* __restrict__ out, int seq,
                          int att_heads, int value_heads, int channels, int cpad,
                          int num_tiles) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const Layout L = make_layout(cpad);
    const Bars B{sbase + L.bar};
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 192);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(smem + L.bar + 196);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int hd = channels / value_heads;
    const int nqb = (seq + kM - 1) / kM;
    const int nchunks = (seq + kKc - 1) / kKc;
    const int my_tiles = (num_tiles - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1;
    const int total = my_tiles * nchunks;

    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_value_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        for (uint32_t s = 0; s < L.raw_stages; ++s) {
            mbar_init(B.raw_full(s), 1);
            mbar_init(B.raw_empty(s), 4);
        }
        for (uint32_t t = 0; t < 2; ++t) {
            mbar_init(B.a_full(t), 4);
            mbar_init(B.a_empty(t), 1);
            mbar_init(B.acc_full(t), 1);
            mbar_init(B.acc_empty(t), 4);
        }
        for (uint32_t s = 0; s < L.v_stages; ++s) {
            mbar_init(B.v_full(s), 1);
            mbar_init(B.v_empty(s), 1);
        }
        *abort = 0u;
        fence_mbar_init();
        prefetch_tensormap(&v_map);
        for (int r = 0; r < 8; ++r) prefetch_tensormap(&a_maps.m[r]);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), L.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int nsup = (nchunks + static_cast<int>(L.sup) - 1) / static_cast<int>(L.sup);
    const int total_sup = my_tiles * nsup;
    if (warp == 0) {
        // ---------------- A producer: one super-chunk per raw stage ----------------
#pragma unroll 1
        for (int gs = 0; gs < total_sup; ++gs) {
            const int i = gs / nsup, sc = gs - i * nsup;
            const TileInfo ti = tile_info(blockIdx.x + i * gridDim.x, value_heads, nqb);
            const int ha = value_heads == 1 ? 0 : ti.h;
            const uint32_t s = gs % L.raw_stages;
            if (gs >= static_cast<int>(L.raw_stages) &&
                !warp_wait(B.raw_empty(s), ((gs / L.raw_stages) - 1) & 1, abort))
                continue;
            if (__any_sync(0xffffffffu, *abort != 0u)) continue;
            // Rows j = slot + 8i (i < 16) of the tile form one box of class (R0+slot) mod 8.
            if (lane < 8) {
                const int64_t R = (static_cast<int64_t>(ti.n) * att_heads + ha) * seq + ti.q0 + lane;
                if (lane == 0) mbar_expect_tx(B.raw_full(s), L.raw_stage);
                __syncwarp(0xffu);
                tma_load_2d(sbase + L.raw0 + s * L.raw_stage + lane * 16 * L.raw_row,
                            &a_maps.m[R & 7], B.raw_full(s), sc * kKc * static_cast<int>(L.sup),
                            static_cast<int32_t>(R >> 3));
            }
            __syncwarp();
        }
    } else if (warp == 6) {
        // ---------------- V producer: up to v_stages chunks ahead of the MMAs ----------------
#pragma unroll 1
        for (int g = 0; g < total; ++g) {
            const int i = g / nchunks, c = g - i * nchunks;
            const uint32_t vs = g % L.v_stages;
            if (g >= static_cast<int>(L.v_stages) &&
                !warp_wait(B.v_empty(vs), ((g / L.v_stages) - 1) & 1, abort))
                continue;
            if (lane == 0) {
                const TileInfo ti = tile_info(blockIdx.x + i * gridDim.x, value_heads, nqb);
                const int col_base = (ti.h * hd) & ~7;
                mbar_expect_tx(B.v_full(vs), L.vstage);
                for (int x = 0; x < cpad / 64; ++x)
                    tma_load_3d(sbase + L.v0 + vs * L.vstage + x * kVAtom, &v_map, B.v_full(vs),
                                col_base + x * 64, c * kKc, ti.n);
            }
            __syncwarp();
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        const uint32_t idesc_base = idesc_f16(Fmt<T>::v, kM, 16, 0, 1);  // N patched per part
#pragma unroll 1
        for (int gc = 0; gc < total; ++gc) {
            const int i = gc / nchunks, c = gc - i * nchunks;
            const uint32_t t = gc & 1, vs = gc % L.v_stages, b = i % L.acc_bufs;
            bool ok = warp_wait(B.a_full(t), (gc >> 1) & 1, abort);
            ok = ok && warp_wait(B.v_full(vs), (gc / L.v_stages) & 1, abort);
            if (ok && c == 0 && i >= static_cast<int>(L.acc_bufs))
                ok = warp_wait(B.acc_empty(b), ((i / L.acc_bufs) - 1) & 1, abort);
            if (ok) {
                tc_fence_after();
                if (elect_one()) {
                    const uint64_t da = kmajor_desc(sbase + L.a0 + t * kATile);
                    for (int part = 0; part * 256 < cpad; ++part) {
                        const int nw = min(256, cpad - part * 256);
                        const uint32_t idesc = idesc_base + ((static_cast<uint32_t>(nw) >> 3) << 17) -
                                               ((16u >> 3) << 17);
                        // V: MN-major, 64-channel atoms kVAtom bytes apart, 16 keys = 2048 B.
                        const uint64_t dv = sw128_desc(
                            sbase + L.v0 + vs * L.vstage + part * 4 * kVAtom, kVAtom, 1024);
#pragma unroll
                        for (int ks = 0; ks < kKc / 16; ++ks)
                            umma_f16_ss(tmem + b * cpad + part * 256, da + ks * (256 >> 4),
                                        dv + ks * (2048 >> 4), idesc, (c > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(B.a_empty(t));
                    umma_commit(B.v_empty(vs));
                    if (c == nchunks - 1) umma_commit(B.acc_full(b));
                }
                __syncwarp();
            }
        }
        // Teardown: every MMA of this CTA completes before TMEM is released.
        if (total > 0) {
            const int last = total - 1;
            if (!mbar_wait(B.a_empty(last & 1), (last >> 1) & 1) && lane == 0)
                atomicExch(&g_value_tc_error, 1u);
        }
    } else if (warp >= 7) {
        // ---------------- epilogue warps 7..10 ----------------
        const int qtr = warp & 3;
        const int r = qtr * 32 + lane;  // output row = TMEM lane
        const uint32_t lane_off = static_cast<uint32_t>(qtr * 32) << 16;
        auto epilogue = [&](int i) {
            const TileInfo ti = tile_info(blockIdx.x + i * gridDim.x, value_heads, nqb);
            const uint32_t b = i % L.acc_bufs;
            if (warp_wait(B.acc_full(b), (i / L.acc_bufs) & 1, abort)) {
                tc_fence_after();
                const int q = ti.q0 + r;
                const int col0 = ti.h * hd;
                const int off = col0 & 7;  // first head column inside the V tile
                T* orow = out + (static_cast<int64_t>(ti.n) * seq + q) * channels + col0;
                const bool vec = off == 0 && channels % 8 == 0 && hd % 8 == 0;
                for (int cb = off & ~31; cb < off + hd; cb += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem + lane_off + b * cpad + cb, v);
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(B.acc_empty(b));
        };
#pragma unroll 1
        for (int i = 0; i < my_tiles; ++i) epilogue(i);
    } else {
        // ---------------- repack warps 1..4 ----------------
        // Repack row: thread t = 16 * slot + i handles row j = slot + 8i, so that the 8
        // lanes of a shared-memory phase read 8 consecutive box rows of one class and
        // write 8 consecutive core-matrix groups.
        const int rt = (warp - 1) * 32 + lane;
        const int slot = rt >> 4, bi = rt & 15;
        const int j = slot + 8 * bi;
        int gc = 0;
#pragma unroll 1
        for (int gs = 0; gs < total_sup; ++gs) {
            const int i = gs / nsup, sc = gs - i * nsup;
            const TileInfo ti = tile_info(blockIdx.x + i * gridDim.x, value_heads, nqb);
            const int ha = value_heads == 1 ? 0 : ti.h;
            const uint32_t s = gs % L.raw_stages;
            const bool raw_ok = warp_wait(B.raw_full(s), (gs / L.raw_stages) & 1, abort);
            const int c_end = min(nchunks, (sc + 1) * static_cast<int>(L.sup));
#pragma unroll 1
            for (int c = sc * static_cast<int>(L.sup); c < c_end; ++c, ++gc) {
                const int sub = c - sc * static_cast<int>(L.sup);
                const uint32_t t = gc & 1;
                bool ok = raw_ok;
                if (ok && gc >= 2) ok = warp_wait(B.a_empty(t), ((gc >> 1) - 1) & 1, abort);
                if (ok) {
                    const int q = ti.q0 + j;
                    const int k0 = c * kKc;
                    const int nk = min(kKc, seq - k0);
                    uint32_t w[36];
                    if (q < seq) {
                        const int64_t R0 =
                            (static_cast<int64_t>(ti.n) * att_heads + ha) * seq + ti.q0;
                        const int a = class_offset(static_cast<int>((R0 + slot) & 7), seq);
                        const uint4* raw = reinterpret_cast<const uint4*>(
                            smem + L.raw0 + s * L.raw_stage + (slot * 16 + bi) * L.raw_row +
                            sub * 128);
#pragma unroll
                        for (int x = 0; x < 9; ++x) {
                            const uint4 v = raw[x];
                            w[4 * x] = v.x;
                            w[4 * x + 1] = v.y;
                            w[4 * x + 2] = v.z;
                            w[4 * x + 3] = v.w;
                        }
                        // Shift by a elements: whole words (a >> 1) with a predicated
                        // barrel, then half a word with a funnel shift.
                        const uint32_t sw = static_cast<uint32_t>(a) >> 1;
#pragma unroll
                        for (int x = 0; x < 34; ++x) w[x] = (sw & 2u) ? w[x + 2] : w[x];
#pragma unroll
                        for (int x = 0; x < 33; ++x) w[x] = (sw & 1u) ? w[x + 1] : w[x];
                        const uint32_t sh = (a & 1) ? 16u : 0u;
#pragma unroll
                        for (int x = 0; x < 32; ++x) w[x] = __funnelshift_r(w[x], w[x + 1], sh);
                        if (nk < kKc) {
#pragma unroll
                            for (int x = 0; x < 32; ++x) {
                                const int k = 2 * x;
                                if (k >= nk) w[x] = 0u;
                                else if (k + 1 >= nk) w[x] &= 0xFFFFu;
                            }
                        }
                    } else {
#pragma unroll
                        for (int x = 0; x < 32; ++x) w[x] = 0u;
                    }
                    uint8_t* tile = smem + L.a0 + t * kATile;
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc)
                        *reinterpret_cast<uint4*>(tile + a_offset(j, cc)) =
                            make_uint4(w[4 * cc], w[4 * cc + 1], w[4 * cc + 2], w[4 * cc + 3]);
                    fence_proxy_async_smem();
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(B.a_full(t));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(B.raw_empty(s));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
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

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 0;
    return n;
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
                                             static_cast<int>(kSmemLimit));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    // Attention rows by residue class r = R mod 8 of the flattened row index R: class r's
    // rows start at element r*T + 8*T*m; its map begins at the 16-byte boundary below r*T.
    AMaps amaps;
    const int64_t rows = static_cast<int64_t>(p.batch) * p.attention_heads * p.length;
    for (int r = 0; r < 8; ++r) {
        const int64_t start = static_cast<int64_t>(r) * p.length;
        const int64_t base = start & ~static_cast<int64_t>(7);
        const int64_t class_rows = r < rows ? (rows - 1 - r) / 8 + 1 : 1;
        const cuuint64_t adims[2] = {static_cast<cuuint64_t>(p.length + (start - base)),
                                     static_cast<cuuint64_t>(class_rows)};
        const cuuint64_t astrides[1] = {static_cast<cuuint64_t>(p.length) * 8 * sizeof(T)};
        const cuuint32_t abox[2] = {make_layout(cpad).raw_row / 2, 16};
        const cuuint32_t aestr[2] = {1, 1};
        if (encode(&amaps.m[r], dt, 2,
                   const_cast<T*>(static_cast<const T*>(p.attention)) + base, adims, astrides,
                   abox, aestr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return cudaErrorNotSupported;
    }
    const Layout L = make_layout(cpad);
    const int64_t tiles =
        static_cast<int64_t>(p.batch) * p.value_heads * ((p.length + kM - 1) / kM);
    const int sms = sm_count();
    if (sms <= 0) return cudaErrorNotSupported;
    const int grid = static_cast<int>(tiles < sms ? tiles : sms);
    zipformer_value_tc_kernel<T><<<grid, kThreads, L.bytes, stream>>>(
        map, amaps, static_cast<T*>(p.output), p.length, p.attention_heads, p.value_heads,
        p.channels, cpad, static_cast<int>(tiles));
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_zipformer_value_tc(const ZipformerValueProblem& p, cudaStream_t stream) {
    if (p.dtype != FGA_HALF && p.dtype != FGA_BF16) return cudaErrorNotSupported;
    // TMA needs 16-byte V row strides.
    if (p.channels % 8 != 0 || p.value_heads < 1 || p.channels % p.value_heads != 0)
        return cudaErrorNotSupported;
    // Rows shorter than one 64-key chunk use the SIMT kernel.
    if (p.length < kKc) return cudaErrorNotSupported;
    // Accumulator columns: the widest head span from its first channel rounded down to 8
    // (the offset repeats with period 8 in the head index), rounded up to 64.
    const int hd = p.channels / p.value_heads;
    int span = 0;
    for (int h = 0; h < p.value_heads && h < 8; ++h) span = max(span, ((h * hd) & 7) + hd);
    const int cpad = (span + 63) / 64 * 64;
    if (cpad > kMaxCpad) return cudaErrorNotSupported;
    if (static_cast<int64_t>(p.batch) * p.value_heads * ((p.length + kM - 1) / kM) > (1ll << 30))
        return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(p.attention) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.value) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(p.output) & 15u) != 0)
        return cudaErrorNotSupported;
    return p.dtype == FGA_HALF ? value_tc_typed<__half>(p, cpad, stream)
                               : value_tc_typed<__nv_bfloat16>(p, cpad, stream);
}

}  // namespace fga
