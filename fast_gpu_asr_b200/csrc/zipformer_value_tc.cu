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
//   warp 5      MMA issuer; warp 6 V producer. A V tile holds the chunk's 64 keys of the
//               channels from the head's first channel (rounded down to 8) in MN-major
//               swizzled atoms, as narrow as the head allows: a self-attention head (12
//               channels) is one 16-channel SWIZZLE_32B atom (2 KB per chunk) and an N = 16
//               MMA. Tiles up to 64 channels wide are copied by the V warp with 16-byte
//               cp.async straight into their swizzled slots, several chunks ahead, so V
//               takes no place in the SM's TMA queue: there every V key would be one box row
//               (64 per chunk, more than the A boxes' 43), and the A stream would wait
//               behind them. Wider tiles (the NonlinAttention value, 3E/4 channels of head
//               0) arrive by TMA in ceil(C/64) 64-channel SWIZZLE_128B atoms. Accumulators
//               (fp32, TMEM) are double-buffered across tiles when they fit.
//
// All waits are bounded; a timeout raises the CTA's abort word, after which every role
// skips its work but keeps its loop, so nothing waits on a role that has stopped.
// Reference: zipformer_attention_value_plugin.cu:118-181 (fp32 accumulation; one value
// head consumes attention head 0, :85).
#include <cuda.h>

#include <cstdint>

#include "fga_common.cuh"
#include "fga_kernels.h"
#include "host_util.h"
#include "sm100_ptx.cuh"

namespace fga {
namespace {

using namespace sm100;

constexpr int kM = 128;        // query rows per tile
constexpr int kKc = 64;        // keys per chunk (one 128-byte swizzle atom of A)
constexpr int kThreads = 480;  // 15 warps
constexpr int kRepackWarps = 8;
constexpr int kMaxCpad = 512;  // TMEM columns
// Raw staging for a super-chunk of S 64-key chunks: per row a TMA box row of 64*S + 8
// elements (the class offset is at most 7), 16 rows per residue class, 8 classes.
__host__ __device__ constexpr uint32_t raw_row_bytes(int sup) { return (64u * sup + 8u) * 2u; }
__host__ __device__ constexpr uint32_t raw_stage_bytes(int sup) { return 128u * raw_row_bytes(sup); }
constexpr uint32_t kSbo = 1040;               // 8-row core-matrix groups (16 mod 128)
constexpr uint32_t kATile = 16 * kSbo;        // 128 rows x 64 keys, no swizzle
constexpr uint32_t kSmemLimit = 227 * 1024;
constexpr uint32_t kMaxVStages = 8;   // streaming V ring
constexpr uint32_t kMaxVRes = 16;     // resident V: chunks per row (keys <= 1024)
constexpr uint32_t kBarBytes = 512;

// Per-device error word of this file's kernel: 1 = a bounded wait gave up, 2 = the dynamic
// shared memory was not 1024-byte aligned. Read and cleared by fga_device_status.
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
    uint32_t sup, raw_row, raw_stage, raw_stages, a_tiles, v_stages, acc_bufs, acc_stride;
    uint32_t vw, vatom, vstage;  // V atom width (channels) and bytes; bytes per V stage
    uint32_t vres;               // 1: one V stage per chunk, loaded once per (n, h) run
    uint32_t raw0, a0, v0, bar, bytes, tmem_cols;
};

__host__ __device__ constexpr uint32_t pow2_cols(uint32_t n) {
    return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512;
}

// Shared-memory plan for `cpad` accumulator columns (16, 32 or a multiple of 64) and
// rows of `seq` keys. A V atom is 64 keys x vw channels (vw = cpad up to 64): rows of
// 2*vw bytes, swizzled over 2*vw bytes (SWIZZLE_32B, 64B or 128B). Narrow V tiles
// (cpad <= 128) get 3-chunk super-chunks in a 3-deep raw ring, wide ones single chunks in
// a 4-deep raw ring. Three A tiles keep the repack and the MMAs from waiting on each
// other; two when space is short. When a V stage per chunk of the whole row fits (at most
// kMaxVRes chunks), V is resident: each chunk's stage is loaded once per run of tiles of
// one (utterance, head) and serves all its query blocks. Otherwise up to kMaxVStages V
// stages stream; while fewer than 2 fit, the raw ring gives up stages.
__host__ __device__ constexpr Layout make_layout(int cpad, int seq) {
    Layout l{};
    l.vw = cpad < 64 ? static_cast<uint32_t>(cpad) : 64u;
    l.vatom = static_cast<uint32_t>(kKc) * l.vw * 2u;
    l.vstage = (static_cast<uint32_t>(cpad) / l.vw) * l.vatom;
    const bool narrow = cpad <= 128;
    const uint32_t nchunks = static_cast<uint32_t>((seq + kKc - 1) / kKc);
    // A super-chunk never spans more chunks than the row has (short rows would otherwise
    // fill boxes that are mostly past the row's end).
    l.sup = narrow ? (nchunks < 3u ? nchunks : 3u) : 1u;
    l.raw_row = raw_row_bytes(static_cast<int>(l.sup));
    l.raw_stage = raw_stage_bytes(static_cast<int>(l.sup));
    l.raw_stages = narrow ? 3u : 4u;
    for (l.a_tiles = 3; l.a_tiles >= 2 && l.vres == 0; --l.a_tiles) {
        const uint32_t fixed = l.raw_stages * l.raw_stage + l.a_tiles * kATile + 1024 + kBarBytes;
        if (nchunks <= kMaxVRes && fixed + nchunks * l.vstage <= kSmemLimit) {
            l.vres = 1;
            l.v_stages = nchunks;
            break;
        }
    }
    if (l.vres == 0) {
        l.a_tiles = 3;
        uint32_t fixed = l.raw_stages * l.raw_stage + l.a_tiles * kATile + 1024 + kBarBytes;
        if (fixed + 3 * l.vstage > kSmemLimit) {
            l.a_tiles = 2;
            fixed -= kATile;
        }
        for (;;) {
            l.v_stages = fixed < kSmemLimit ? (kSmemLimit - fixed) / l.vstage : 0u;
            if (l.v_stages >= 2 || l.raw_stages == 2) break;
            --l.raw_stages;
            fixed = l.raw_stages * l.raw_stage + l.a_tiles * kATile + 1024 + kBarBytes;
        }
        if (l.v_stages > kMaxVStages) l.v_stages = kMaxVStages;
    }
    // The epilogue reads 32 accumulator columns at a time.
    l.acc_stride = cpad < 32 ? 32u : static_cast<uint32_t>(cpad);
    l.acc_bufs = 2 * l.acc_stride <= kMaxCpad ? 2 : 1;
    l.raw0 = 0;
    l.a0 = l.raw_stages * l.raw_stage;
    l.v0 = (l.a0 + l.a_tiles * kATile + 1023u) & ~1023u;  // swizzle atoms: 1024-byte aligned
    l.bar = l.v0 + l.v_stages * l.vstage;
    l.bytes = l.bar + kBarBytes;
    l.tmem_cols = pow2_cols(l.acc_bufs * l.acc_stride);
    return l;
}

struct Bars {  // mbarrier addresses (shared window); the TMEM slot and abort word follow
    uint32_t base;
    __device__ uint32_t raw_full(uint32_t s) const { return base + 8 * s; }        // <= 5
    __device__ uint32_t raw_empty(uint32_t s) const { return base + 40 + 8 * s; }
    __device__ uint32_t a_full(uint32_t t) const { return base + 80 + 8 * t; }         // <= 4
    __device__ uint32_t a_empty(uint32_t t) const { return base + 112 + 8 * t; }
    __device__ uint32_t acc_full(uint32_t b) const { return base + 144 + 8 * b; }      // <= 2
    __device__ uint32_t acc_empty(uint32_t b) const { return base + 160 + 8 * b; }
    __device__ uint32_t v_full(uint32_t s) const { return base + 176 + 8 * s; }        // <= 16
    __device__ uint32_t v_empty(uint32_t s) const { return base + 304 + 8 * s; }
};
constexpr uint32_t kTmemSlotOff = 432, kAbortOff = 436, kDrainOff = 440;

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

// Walks a CTA's contiguous range of tiles; tile = (n * heads + h) * nqb + qb, so the query
// blocks of one (utterance, head) are consecutive.
struct TileCursor {
    int qb, h, n;
    __device__ void init(int tile, int heads, int nqb) {
        qb = tile % nqb;
        const int nh = tile / nqb;
        h = nh % heads;
        n = nh / heads;
    }
    __device__ void next(int heads, int nqb) {
        if (++qb == nqb) {
            qb = 0;
            if (++h == heads) {
                h = 0;
                ++n;
            }
        }
    }
};

// Ring position: slot and the parity of its current phase.
struct Ring {
    uint32_t slot = 0, phase = 0;
    __device__ void next(uint32_t n) {
        if (++slot == n) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
zipformer_value_tc_kernel(const __grid_constant__ CUtensorMap v_map,
                          const __grid_constant__ AMaps a_maps, T* __restrict__ out, int seq,
                          int att_heads, int value_heads, int channels, int cpad,
                          int num_tiles) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const Layout L = make_layout(cpad, seq);
    const Bars B{sbase + L.bar};
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + kTmemSlotOff);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(smem + L.bar + kAbortOff);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int hd = channels / value_heads;
    const int nqb = (seq + kM - 1) / kM;
    const int nchunks = (seq + kKc - 1) / kKc;
    const int sup = static_cast<int>(L.sup);
    const int nsup = (nchunks + sup - 1) / sup;
    // A contiguous, balanced range of tiles per CTA (grid <= tiles, so none is empty).
    const int t_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * num_tiles / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * num_tiles / gridDim.x);
    const int my_tiles = t_end - t_begin;

    if ((sbase & 1023u) != 0) {
        if (tid == 0) atomicExch(&g_value_tc_error, 2u);
        return;
    }
    if (tid == 0) {
        for (uint32_t s = 0; s < L.raw_stages; ++s) {
            mbar_init(B.raw_full(s), 1);
            mbar_init(B.raw_empty(s), kRepackWarps);
        }
        for (uint32_t t = 0; t < L.a_tiles; ++t) {
            mbar_init(B.a_full(t), kRepackWarps);
            mbar_init(B.a_empty(t), 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(B.acc_full(b), 1);
            mbar_init(B.acc_empty(b), 4);
        }
        for (uint32_t s = 0; s < L.v_stages; ++s) {
            mbar_init(B.v_full(s), 1);
            mbar_init(B.v_empty(s), 1);
        }
        mbar_init(sbase + L.bar + kDrainOff, 1);
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

    if (warp == 0) {
        // ---------------- A producer: one super-chunk per raw stage ----------------
        TileCursor cur;
        cur.init(t_begin, value_heads, nqb);
        Ring rs;
        int gs = 0;
        uint32_t issued = 0, issued_par = 0;  // per raw slot: loaded, and that load's parity
#pragma unroll 1
        for (int i = 0; i < my_tiles; ++i, cur.next(value_heads, nqb)) {
            const int ha = value_heads == 1 ? 0 : cur.h;
            // Rows j = slot + 8m (m < 16) of the tile form one box of class (R0+slot) mod 8.
            const int64_t R = (static_cast<int64_t>(cur.n) * att_heads + ha) * seq + cur.qb * kM + lane;
#pragma unroll 1
            for (int sc = 0; sc < nsup; ++sc, ++gs, rs.next(L.raw_stages)) {
                if (gs >= static_cast<int>(L.raw_stages) &&
                    !warp_wait(B.raw_empty(rs.slot), rs.phase ^ 1u, abort))
                    continue;
                if (__any_sync(0xffffffffu, *abort != 0u)) continue;
                if (lane < 8) {
                    if (lane == 0) mbar_expect_tx(B.raw_full(rs.slot), L.raw_stage);
                    __syncwarp(0xffu);
                    tma_load_2d(sbase + L.raw0 + rs.slot * L.raw_stage + lane * 16 * L.raw_row,
                                &a_maps.m[R & 7], B.raw_full(rs.slot), sc * kKc * sup,
                                static_cast<int32_t>(R >> 3));
                }
                __syncwarp();
                issued |= 1u << rs.slot;
                issued_par = (issued_par & ~(1u << rs.slot)) | (rs.phase << rs.slot);
            }
        }
        // Teardown (default time limit): every slot's last load has landed before shared
        // memory is released. Without an abort the consumers already waited for them all.
        if (lane == 0) {
            bool ok = true;
            for (uint32_t st = 0; st < L.raw_stages; ++st)
                if ((issued >> st) & 1u) ok = mbar_wait(B.raw_full(st), (issued_par >> st) & 1u) && ok;
            if (!ok) atomicExch(&g_value_tc_error, 1u);
        }
        __syncwarp();
    } else if (warp == 6) {
        // ---------------- V producer ----------------
        // Resident: at the start of each run of tiles of one (n, h), chunk c's stage c is
        // reloaded once the MMAs of the previous run's last tile have released it.
        // Streaming: one stage per chunk of every tile, up to v_stages ahead of the MMAs.
        TileCursor cur;
        cur.init(t_begin, value_heads, nqb);
        Ring vr;
        int run = 0, g = 0;
        uint32_t issued = 0, issued_par = 0;  // per V stage: loaded, and that load's parity
#pragma unroll 1
        for (int i = 0; i < my_tiles; ++i, cur.next(value_heads, nqb)) {
            const bool run_start = i == 0 || cur.qb == 0;
            if (L.vres && !run_start) continue;
            const int col_base = (cur.h * hd) & ~7;
#pragma unroll 1
            for (int c = 0; c < nchunks; ++c, ++g) {
                uint32_t vs, vpar;
                bool ok;
                if (L.vres) {
                    vs = static_cast<uint32_t>(c);
                    vpar = static_cast<uint32_t>(run & 1);
                    ok = run == 0 || warp_wait(B.v_empty(vs), (run - 1) & 1, abort);
                } else {
                    vs = vr.slot;
                    vpar = vr.phase;
                    ok = g < static_cast<int>(L.v_stages) ||
                         warp_wait(B.v_empty(vs), vr.phase ^ 1u, abort);
                    vr.next(L.v_stages);
                }
                // (the first loads of a run skip the wait: check the abort word for them too)
                ok = ok && __all_sync(0xffffffffu, *abort == 0u);
                if (ok && lane == 0) {
                    mbar_expect_tx(B.v_full(vs), L.vstage);
                    for (int x = 0; x < cpad / static_cast<int>(L.vw); ++x)
                        tma_load_3d(sbase + L.v0 + vs * L.vstage + x * L.vatom, &v_map,
                                    B.v_full(vs), col_base + x * static_cast<int>(L.vw), c * kKc,
                                    cur.n);
                }
                __syncwarp();
                if (ok) {
                    issued |= 1u << vs;
                    issued_par = (issued_par & ~(1u << vs)) | (vpar << vs);
                }
            }
            ++run;
        }
        // Teardown (default time limit): every stage's last load has landed.
        if (lane == 0) {
            bool ok = true;
            for (uint32_t st = 0; st < L.v_stages; ++st)
                if ((issued >> st) & 1u) ok = mbar_wait(B.v_full(st), (issued_par >> st) & 1u) && ok;
            if (!ok) atomicExch(&g_value_tc_error, 1u);
        }
        __syncwarp();
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        // V: MN-major atoms of vw channels, vatom bytes apart along N; 8-key groups of
        // 16*vw bytes; one 16-key step = 32*vw bytes. Descriptor start addresses advance in
        // 16-byte units.
        const uint32_t vlayout = L.vw == 16 ? 6u : L.vw == 32 ? 4u : 2u;  // SWIZZLE_32B/64B/128B
        const uint64_t da0 = kmajor_desc(sbase + L.a0);
        const uint64_t dv0 = smem_desc(sbase + L.v0, L.vatom, 16 * L.vw, vlayout);
        const uint32_t part_atoms = (256u / L.vw) * L.vatom;
        const uint32_t idesc_full = idesc_f16(Fmt<T>::v, kM, 256, 0, 1);
        const uint32_t idesc_last = idesc_f16(Fmt<T>::v, kM, ((cpad - 1) & 255) + 1, 0, 1);
        const int parts = (cpad + 255) / 256;
        TileCursor cur;
        cur.init(t_begin, value_heads, nqb);
        Ring ar, vr, acc;
        int run = -1;
#pragma unroll 1
        for (int i = 0; i < my_tiles; ++i, cur.next(value_heads, nqb)) {
            const bool run_start = i == 0 || cur.qb == 0;
            if (run_start) ++run;
            const bool run_end = i + 1 == my_tiles || cur.qb == nqb - 1;
            // Resident V is waited for once per run: it stays until the run's last tile.
            const bool wait_v = !L.vres || run_start;
            bool tile_ok = true;
            if (i >= static_cast<int>(L.acc_bufs))
                tile_ok = warp_wait(B.acc_empty(acc.slot), acc.phase ^ 1u, abort);
            const uint32_t d_acc = tmem + acc.slot * L.acc_stride;
#pragma unroll 1
            for (int c = 0; c < nchunks; ++c, ar.next(L.a_tiles)) {
                const uint32_t vs = L.vres ? static_cast<uint32_t>(c) : vr.slot;
                const uint32_t vph = L.vres ? static_cast<uint32_t>(run & 1) : vr.phase;
                if (!L.vres) vr.next(L.v_stages);
                bool ok = tile_ok && warp_wait(B.a_full(ar.slot), ar.phase, abort);
                if (wait_v) ok = ok && warp_wait(B.v_full(vs), vph, abort);
                if (!ok) continue;
                tc_fence_after();
                if (elect_one()) {
                    const uint64_t da = da0 + ar.slot * (kATile >> 4);
                    const uint64_t dv = dv0 + ((vs * L.vstage) >> 4);
                    for (int part = 0; part < parts; ++part) {
                        const uint32_t idesc = part + 1 == parts ? idesc_last : idesc_full;
#pragma unroll
                        for (int ks = 0; ks < kKc / 16; ++ks)
                            umma_f16_ss(d_acc + part * 256, da + ks * (256 >> 4),
                                        dv + ((part * part_atoms + ks * 32 * L.vw) >> 4), idesc,
                                        (c > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(B.a_empty(ar.slot));
                    if (!L.vres || run_end) umma_commit(B.v_empty(vs));
                    if (c == nchunks - 1) umma_commit(B.acc_full(acc.slot));
                }
                __syncwarp();
            }
            acc.next(L.acc_bufs);
        }
        // Teardown: every MMA of this CTA completes before TMEM is released (one commit
        // tracks all MMAs this thread issued, including when some were skipped after an abort).
        bool drained = true;
        if (elect_one()) {
            umma_commit(sbase + L.bar + kDrainOff);
            drained = mbar_wait(sbase + L.bar + kDrainOff, 0);
        }
        __syncwarp();
        if (!drained) atomicExch(&g_value_tc_error, 1u);
    } else if (warp >= 7 && warp <= 10) {
        // ---------------- epilogue warps 7..10 ----------------
        const int qtr = warp & 3;
        const int r = qtr * 32 + lane;  // output row = TMEM lane
        const uint32_t lane_off = static_cast<uint32_t>(qtr * 32) << 16;
        TileCursor cur;
        cur.init(t_begin, value_heads, nqb);
        Ring acc;
#pragma unroll 1
        for (int i = 0; i < my_tiles; ++i, cur.next(value_heads, nqb), acc.next(L.acc_bufs)) {
            if (warp_wait(B.acc_full(acc.slot), acc.phase, abort)) {
                tc_fence_after();
                const int q = cur.qb * kM + r;
                const int col0 = cur.h * hd;
                const int off = col0 & 7;  // first head column inside the V tile
                T* orow = out + (static_cast<int64_t>(cur.n) * seq + q) * channels + col0;
                const bool vec = off == 0 && channels % 8 == 0 && hd % 8 == 0;
                for (int cb = off & ~31; cb < off + hd; cb += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem + lane_off + acc.slot * L.acc_stride + cb, v);
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
            if (lane == 0) mbar_arrive(B.acc_empty(acc.slot));
        }
    } else {
        // ---------------- repack warps 1..4 and 11..14 ----------------
        // Repack thread rt (0..255) moves keys [32 half, 32 half + 32) of row
        // j = slot + 8 m, with half = rt / 128, slot = (rt / 16) mod 8, m = rt mod 16, so
        // that the 8 lanes of a shared-memory phase read 8 consecutive box rows of one
        // class and write 8 consecutive core-matrix groups.
        const int rt = (warp <= 4 ? warp - 1 : warp - 7) * 32 + lane;
        const int half = rt >> 7, slot = (rt >> 4) & 7, bi = rt & 15;
        const int j = slot + 8 * bi;
        const uint32_t a_row = static_cast<uint32_t>(j >> 3) * kSbo + static_cast<uint32_t>(j & 7) * 16u +
                               static_cast<uint32_t>(half) * 512u;
        TileCursor cur;
        cur.init(t_begin, value_heads, nqb);
        Ring rs, ar;
        int gc = 0;
#pragma unroll 1
        for (int i = 0; i < my_tiles; ++i, cur.next(value_heads, nqb)) {
            const int ha = value_heads == 1 ? 0 : cur.h;
            const int q = cur.qb * kM + j;
            const int64_t R = (static_cast<int64_t>(cur.n) * att_heads + ha) * seq + q;
            const int a = class_offset(static_cast<int>(R & 7), seq);
            // Shift by a elements: whole words (a >> 1) with a predicated barrel, then half a
            // word with a funnel shift.
            const uint32_t sw = static_cast<uint32_t>(a) >> 1;
            const uint32_t sh = (a & 1) ? 16u : 0u;
            int c = 0;
#pragma unroll 1
            for (int sc = 0; sc < nsup; ++sc, rs.next(L.raw_stages)) {
                const bool raw_ok = warp_wait(B.raw_full(rs.slot), rs.phase, abort);
                const uint8_t* raw_row = smem + L.raw0 + rs.slot * L.raw_stage +
                                         (slot * 16 + bi) * L.raw_row + half * 64;
#pragma unroll 1
                for (int sub = 0; sub < sup && c < nchunks; ++sub, ++c, ++gc, ar.next(L.a_tiles)) {
                    bool ok = raw_ok;
                    if (ok && gc >= static_cast<int>(L.a_tiles))
                        ok = warp_wait(B.a_empty(ar.slot), ar.phase ^ 1u, abort);
                    if (ok) {
                        const int nk = min(kKc, seq - c * kKc) - 32 * half;  // keys of this half
                        uint32_t w[20];
                        if (q < seq) {
                            const uint4* src = reinterpret_cast<const uint4*>(raw_row + sub * 128);
#pragma unroll
                            for (int x = 0; x < 5; ++x) {
                                const uint4 v = src[x];
                                w[4 * x] = v.x;
                                w[4 * x + 1] = v.y;
                                w[4 * x + 2] = v.z;
                                w[4 * x + 3] = v.w;
                            }
#pragma unroll
                            for (int x = 0; x < 18; ++x) w[x] = (sw & 2u) ? w[x + 2] : w[x];
#pragma unroll
                            for (int x = 0; x < 17; ++x) w[x] = (sw & 1u) ? w[x + 1] : w[x];
#pragma unroll
                            for (int x = 0; x < 16; ++x) w[x] = __funnelshift_r(w[x], w[x + 1], sh);
                            if (nk < 32) {
#pragma unroll
                                for (int x = 0; x < 16; ++x) {
                                    const int k = 2 * x;
                                    if (k >= nk) w[x] = 0u;
                                    else if (k + 1 >= nk) w[x] &= 0xFFFFu;
                                }
                            }
                        } else {
#pragma unroll
                            for (int x = 0; x < 16; ++x) w[x] = 0u;
                        }
                        uint8_t* tile = smem + L.a0 + ar.slot * kATile + a_row;
#pragma unroll
                        for (int cc = 0; cc < 4; ++cc)
                            *reinterpret_cast<uint4*>(tile + cc * 128) =
                                make_uint4(w[4 * cc], w[4 * cc + 1], w[4 * cc + 2], w[4 * cc + 3]);
                        fence_proxy_async_smem();
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(B.a_full(ar.slot));
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(B.raw_empty(rs.slot));
            }
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
    const Layout L = make_layout(cpad, p.length);
    const cuuint32_t box[3] = {L.vw, kKc, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle vswz = L.vw == 16   ? CU_TENSOR_MAP_SWIZZLE_32B
                                    : L.vw == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                 : CU_TENSOR_MAP_SWIZZLE_128B;
    if (encode(&map, dt, 3, const_cast<void*>(p.value), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, vswz,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return cudaErrorNotSupported;
    static SmemAttr attr;
    if (cudaError_t e = attr.ensure(reinterpret_cast<const void*>(zipformer_value_tc_kernel<T>),
                                    static_cast<int>(kSmemLimit));
        e != cudaSuccess)
        return e;
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
        const cuuint32_t abox[2] = {L.raw_row / 2, 16};
        const cuuint32_t aestr[2] = {1, 1};
        if (encode(&amaps.m[r], dt, 2,
                   const_cast<T*>(static_cast<const T*>(p.attention)) + base, adims, astrides,
                   abox, aestr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return cudaErrorNotSupported;
    }
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

uint32_t take_value_tc_error(cudaStream_t stream, bool clear, cudaError_t* err) {
    return take_error_word(g_value_tc_error, stream, clear, err);
}

cudaError_t launch_zipformer_value_tc(const ZipformerValueProblem& p, cudaStream_t stream) {
    if (p.dtype != FGA_HALF && p.dtype != FGA_BF16) return cudaErrorNotSupported;
    // TMA needs 16-byte V row strides.
    if (p.channels % 8 != 0 || p.value_heads < 1 || p.channels % p.value_heads != 0)
        return cudaErrorNotSupported;
    // Rows shorter than one 64-key chunk use the SIMT kernel.
    if (p.length < kKc) return cudaErrorNotSupported;
    // Accumulator columns: the widest head span from its first channel rounded down to 8
    // (the offset repeats with period 8 in the head index), rounded up to the V atom width
    // (16, 32 or 64 channels).
    const int hd = p.channels / p.value_heads;
    int span = 0;
    for (int h = 0; h < p.value_heads && h < 8; ++h) span = max(span, ((h * hd) & 7) + hd);
    const int vw = span <= 16 ? 16 : span <= 32 ? 32 : 64;
    const int cpad = (span + vw - 1) / vw * vw;
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
