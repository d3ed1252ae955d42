// K2: persistent, warp-specialised tcgen05 GEMM with a fused epilogue.
//
//   y[m, n] = act( x[m, :] . w[n, :] + bias[n] ) (+ residual[m, n])
//
// x: fp16 [M, K] (K-major activations, Re half then Im half of each row),
// w: fp16 [N, K] (the dense coefficient matrix [[rr, ir], [ri, ii]] decoded
// from the packed phase codes by K1), y / residual: fp16 or fp32 [M, N] (the
// residual has y's dtype; y may alias it: each element is read and written by
// the same thread, before its TMA store). fp32 accumulation in TMEM. One real
// GEMM carries the whole widely-linear map (four real blocks, 2*M*K*N flops),
// which is the minimum for U x + W conj(x).
//
// CTA = 12 warps in 3 warpgroups, one CTA per SM, persistent over 128 x BN
// output tiles:
//   WG0  warp 0   TMA producer: x tile [128 x 64] and w tile [BN x 64] per
//                 k-block into a STAGES-deep ring (128-byte swizzle).
//        warp 1   TMEM owner + MMA issuer: one thread issues 4 x tcgen05.mma
//                 (K = 16 each) per k-block into one of two TMEM accumulators
//                 (2 x BN fp32 columns), so the epilogue of tile i overlaps
//                 the main loop of tile i+1.
//        (WG0 runs with 40 registers per thread: setmaxnreg.dec)
//   WG1  warps 4..7   epilogue, tile columns [0, BN/2)
//   WG2  warps 8..11  epilogue, tile columns [BN/2, BN)   (232 registers: setmaxnreg.inc)
//        Each epilogue warp owns the 32 TMEM lanes (tile rows) of quarter
//        warp % 4 and walks its column half in steps of 128 bytes of output
//        per row: tcgen05.ld, bias, GELU, residual, pack, 128-B-swizzled smem
//        staging, TMA store of a [32 rows x 128 B] box. The residual step is
//        TMA-loaded into the warp's staging slot one step ahead (two slots
//        per warp) and the output is written over it. (An L2 prefetch of each
//        tile's residual two tiles ahead was measured: its lines were evicted
//        before use, so the residual came from DRAM twice — fc2 633 against
//        482 MB read, proj + 8 % time — and it was taken out.)
// Register split: 128 x 40 + 256 x 232 = 64512 = 384 threads x 168 at launch.
//
// Split-K (one CTA per tile, p.splits > 1; small M, where the tiles alone
// would leave most SMs idle and each busy SM would stream a long K at the
// per-SM load rate): the launch is a grid of tiles x splits CTAs in clusters
// of `splits` CTAs; cluster rank s accumulates k-blocks
// [s num_k / S, (s + 1) num_k / S) of its tile into TMEM and writes the raw
// fp32 partial to the workspace in the epilogue warps' own order (every
// store instruction of a warp covers 512 contiguous bytes). After a cluster
// barrier (release / acquire) each CTA reduces 1/S of the tile over the S
// partials in the fixed order 0..S-1 (deterministic) and applies bias, GELU
// and residual to it.
//
// Stream-K tail (p.sk_tiles > 0; CTA pairs or single CTAs, no split-K): when
// the tiles do not fill whole waves of the persistent grid, the last
// sk_tiles tiles (between one and two waves' worth) are not dealt out whole.
// Their k-blocks, in tile order, are cut into one contiguous share per unit
// (a CTA pair or a CTA): every unit first runs its data-parallel tiles, then
// its share. A share is at least one tile long, so a tile is cut at most
// once, into a head (its first k-blocks, the end of one unit's share) and a
// tail (the rest, the start of the next unit's share). A unit runs its head
// first of all (before its data-parallel tiles), then its data-parallel and
// whole tiles, then its tail. The head's unit writes its raw fp32 accumulator to its workspace
// slot in the epilogue warps' own layout and raises one flag per epilogue
// warp. For the tail, the epilogue warps wait for the flags (bounded, like
// every wait here) and load that accumulator into the tail's TMEM buffer
// (tcgen05.st) while the item before it is still in its main loop, and the
// MMAs continue on it: a cut tile goes through exactly the operations of an
// uncut one, so the result is the same bit for bit whatever the schedule (an
// image's outputs do not depend on the batch around it). Then the usual
// epilogue runs and the reader clears the flags. All units are resident at
// once (the grid is the co-resident cluster count), and a head never waits
// for anything, so every wait ends.
//
// Narrow tail (p.pieces = P > 0; CTA pairs): when the tiles leave a last wave
// at most half full, the last p.tail_tiles tiles are cut into P column pieces
// of BN / P (64 or 128) columns each — one MMA of N = BN / P per k-block, the
// weight rows through a second tensor map with that box — and the pieces are
// dealt out over the units after their whole tiles. Every output element is
// still accumulated over all of K in one TMEM buffer, in the same order, so
// the results are those of whole tiles; no exchange between units.
#pragma once

#include "ptx.cuh"

namespace rpfq {

enum : int { kActNone = 0, kActGelu = 1 };

struct GemmParams {
    const void* bias;        // [N] fp16 (fp32 with bias_f32) or nullptr
    const void* residual;    // [M, N], same dtype as y (row stride ldr), or nullptr
    int64_t ldr;
    int64_t m;
    int32_t n, k;
    int32_t activation;
    int32_t bias_f32;        // bias holds fp32 values (no per-element conversion in the epilogue)
    int32_t splits;          // K splits per tile (1: none; > 1 only with PAIR = false, cluster = splits)
    float* ws;               // split-K partials: [tiles * splits][128 * BN] fp32 (splits > 1);
                             // stream-K partials: [units * ranks][128 * BN] fp32 (sk_tiles > 0)
    void* y;                 // the output (y's dtype, row stride ldy): split-K stores it directly
    int64_t ldy;
    int* err;                // device error word
    int32_t sk_tiles;        // stream-K: tiles shared out by k-blocks over all units (0: none)
    int32_t tail_tiles;      // narrow tail: the last tail_tiles tiles are cut into `pieces` column pieces
    int32_t pieces;          // 0: none; else 2 or 4 (BN / pieces columns per piece)
    int* sk_flags;           // stream-K: [units * ranks][8] flags (partial of an epilogue warp written); zero
                             // between calls
};

// One unit's work list: data-parallel tiles (strided over the units), then
// its contiguous share of the stream-K k-blocks. Every role of the CTA walks
// the same list.
struct WorkItem {
    int tile;
    int kb_lo, kb_hi;  // k-blocks [kb_lo, kb_hi) of the tile
    int mode;          // kItemWhole, kItemHead or kItemTail
    int n_off;         // first column of the item within the tile (narrow-tail pieces)
    int width;         // columns of the item: BN, or BN / pieces
};
// kItemHead: k-blocks [0, kb_hi < num_k) of a cut tile, the accumulator goes to
// the workspace; kItemTail: k-blocks [kb_lo > 0, num_k), the accumulator starts
// from the head's and the epilogue follows.
enum : int { kItemWhole = 0, kItemHead = 1, kItemTail = 2 };

template <int BN>
struct Schedule {
    int units, num_k, dp_tiles, dp_kb_lo, dp_kb_hi;
    int next_dp;
    int pieces, piece_items, next_piece;  // narrow tail
    int lo, hi;              // this unit's stream-K k-blocks [lo, hi) (tiles x k-blocks < 2^31)
    int whole, whole_end;    // whole tiles of the share: [whole, whole_end) in k-blocks
    int phase;               // 0 head, 1 data-parallel and pieces, 2 whole tiles, 3 tail, 4 done

    __device__ __forceinline__ Schedule(int unit, int units_, int num_tiles, int num_k_, int sk_tiles, int kb_lo,
                                        int kb_hi, int tail_tiles = 0, int pieces_ = 0)
        : units(units_), num_k(num_k_), dp_tiles(num_tiles - sk_tiles - (pieces_ > 0 ? tail_tiles : 0)),
          dp_kb_lo(kb_lo), dp_kb_hi(kb_hi), next_dp(unit), pieces(pieces_),
          piece_items(pieces_ > 0 ? tail_tiles * pieces_ : 0), next_piece(unit), phase(0) {
        const int64_t total = static_cast<int64_t>(sk_tiles) * num_k;
        lo = static_cast<int>(static_cast<int64_t>(unit) * total / units_);
        hi = static_cast<int>(static_cast<int64_t>(unit + 1) * total / units_);
        whole = (lo + num_k - 1) / num_k * num_k;  // first tile boundary at or after lo
        whole_end = hi / num_k * num_k;            // last tile boundary at or before hi
    }

    __device__ __forceinline__ void set(WorkItem& w, int a, int b, int mode) const {
        const int j = a / num_k;
        w.tile = dp_tiles + j;
        w.kb_lo = a - j * num_k;
        w.kb_hi = b - j * num_k;
        w.mode = mode;
        w.n_off = 0;
        w.width = BN;
    }

    // Order: the head first of all (the next unit's tail waits for it, and its
    // accumulator store then overlaps the main loops that follow), the
    // data-parallel tiles and narrow-tail pieces, the share's whole tiles, the
    // tail last (it waits for the previous unit's head, loaded while the item
    // before it computes).
    __device__ __forceinline__ bool next(WorkItem& w) {
        if (phase == 0) {
            phase = 1;
            if (lo < hi && whole_end < hi) {  // the share ends inside a tile
                set(w, whole_end, hi, kItemHead);
                return true;
            }
        }
        if (phase == 1) {
            if (next_dp < dp_tiles) {
                w.tile = next_dp;
                w.kb_lo = dp_kb_lo;
                w.kb_hi = dp_kb_hi;
                w.mode = kItemWhole;
                w.n_off = 0;
                w.width = BN;
                next_dp += units;
                return true;
            }
            if (next_piece < piece_items) {  // narrow tail: pieces after the whole tiles
                const int pw = BN / pieces;
                w.tile = dp_tiles + next_piece / pieces;
                w.kb_lo = dp_kb_lo;
                w.kb_hi = dp_kb_hi;
                w.mode = kItemWhole;
                w.n_off = (next_piece % pieces) * pw;
                w.width = pw;
                next_piece += units;
                return true;
            }
            phase = lo < hi ? 2 : 4;
        }
        if (phase == 2) {
            if (whole < whole_end) {
                set(w, whole, whole + num_k, kItemWhole);
                whole += num_k;
                return true;
            }
            phase = 3;
        }
        if (phase == 3) {
            phase = 4;
            if (lo % num_k != 0) {  // starts inside a tile
                set(w, lo, (lo / num_k + 1) * num_k, kItemTail);
                return true;
            }
        }
        return false;
    }
};

// Stream-K flag handshake (one flag per epilogue warp and partial).
__device__ __forceinline__ void sk_signal(int* flag) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(1) : "memory");
}
__device__ __forceinline__ int sk_poll(const int* flag) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    return v;
}
// Bounded wait for a partial; false (error word = site, abort raised) when the
// limit runs out or another role has raised abort.
__device__ __forceinline__ bool sk_wait(const int* flag, volatile int* abort_flag, int* gerr, int site) {
    if (sk_poll(flag)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (sk_poll(flag)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1;
            atomicCAS(gerr, 0, site);
            return false;
        }
    }
}

// RES = residual slots per epilogue warp: 0 (no residual), 1 (the residual
// step lands in the single staging slot just before it is used: fine when a
// long main loop hides the epilogue), 2 (the next step's residual lands in the
// second slot while this step runs: for short main loops, at the price of one
// main-loop stage of shared memory).
// PAIR: a cluster of two CTAs computes a 256 x BN tile with cta_group::2
// MMAs; each CTA loads its 128 rows of x and half (BN/2 rows) of w, so the
// operand bytes each SM streams per flop drop by a third.
template <int BN, int RES, bool PAIR = false>
struct GemmCfg {
    static_assert(BN == 128 || BN == 256, "tile width");
    static_assert(RES >= 0 && RES <= 2, "residual slots");
    static_assert(!PAIR || BN == 256, "CTA pairs use 256-wide tiles");
    static constexpr int BM = 128;      // rows per CTA (TMEM lanes)
    static constexpr int TILE_M = PAIR ? 256 : 128;
    static constexpr int BK = 64;  // 64 fp16 = 128 B = one swizzle row
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of w per CTA and stage
    static constexpr int STAGES = PAIR ? (RES == 2 ? 5 : 6) : (BN == 256 ? (RES == 2 ? 3 : 4) : (RES == 2 ? 5 : 6));
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = B_ROWS * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_WARPS = 8;
    static constexpr int EPI_SLOTS = RES == 2 ? 2 : 1;  // staging slots per epilogue warp
    static constexpr int EPI_BUF_BYTES = 32 * 128;  // one slot: 32 rows x 128 B
    static constexpr int EPI_BYTES = EPI_WARPS * EPI_SLOTS * EPI_BUF_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator (power of two)
    static constexpr int BAR_BYTES = 512;
    static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
    static constexpr int THREADS = 384;
    static constexpr int LAUNCH_REGS = 168;  // 65536 / 384, rounded down to the allocation granule
    static constexpr int REGS_PRODUCER = 40;
    static constexpr int REGS_EPILOGUE = 232;
    static_assert(128 * REGS_PRODUCER + 256 * REGS_EPILOGUE <= THREADS * LAUNCH_REGS,
                  "register split exceeds the launch allocation");
    static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM cols");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

// GELU(v) = v/2 (1 + erf(v / sqrt 2)) with erf from Abramowitz & Stegun
// 7.1.26 (Hastings): for z = |v| / sqrt 2,
//   1 - erf(z) = tail = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^{-z^2},  t = 1 / (1 + p z),
// |error of erf| <= 1.5e-7. Since erf(v / sqrt 2) = sign(v) (1 - tail),
//   GELU(v) = (v + |v|) / 2 - |v| tail / 2,
// evaluated on pairs of values with the packed fp32x2 instructions of sm_100
// (one reciprocal and one exponential per value on the special-function unit).
__device__ __forceinline__ void gelu_erf_pair(float& v0, float& v1) {
    constexpr float kP = 0.3275911f * 0.70710678118654752f;  // p / sqrt 2 (acts on |v|)
    constexpr float kE = -0.5f * 1.4426950408889634f;        // -z^2 = -v^2 / 2, in base 2
    const uint64_t v = f2_pack(v0, v1);
    const uint64_t a = v & 0x7fffffff7fffffffull;  // |v| of both lanes
    const uint64_t den = f2_fma(f2_pack(kP, kP), a, f2_pack(1.0f, 1.0f));
    float d0, d1;
    f2_unpack(den, d0, d1);
    const uint64_t t = f2_pack(rcp_approx(d0), rcp_approx(d1));
    uint64_t poly = f2_fma(t, f2_pack(1.061405429f, 1.061405429f), f2_pack(-1.453152027f, -1.453152027f));
    poly = f2_fma(t, poly, f2_pack(1.421413741f, 1.421413741f));
    poly = f2_fma(t, poly, f2_pack(-0.284496736f, -0.284496736f));
    poly = f2_fma(t, poly, f2_pack(0.254829592f, 0.254829592f));
    poly = f2_mul(t, poly);
    const uint64_t q = f2_mul(f2_mul(v, v), f2_pack(kE, kE));
    float q0, q1;
    f2_unpack(q, q0, q1);
    const uint64_t tail = f2_mul(poly, f2_pack(ex2_approx(q0), ex2_approx(q1)));
    const uint64_t half_a = f2_mul(a, f2_pack(-0.5f, -0.5f));
    const uint64_t pos = f2_mul(f2_add(v, a), f2_pack(0.5f, 0.5f));
    f2_unpack(f2_fma(half_a, tail, pos), v0, v1);
}

__device__ __forceinline__ void setmaxnreg_dec40() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
}
__device__ __forceinline__ void setmaxnreg_inc232() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 232;\n" ::: "memory");
}

// Split-K reduction of tile `tile` by its split `split`: float4 granules
// [split E / S, (split + 1) E / S) of the S partials (E = 128 BN / 4, laid out
// as the epilogue warps write them) are summed in the order 0..S-1, then
// bias, GELU and residual are applied as in the one-pass epilogue and the
// four outputs of each granule stored (256 threads, tid 0..255). Each thread
// takes kRedBatch granules at a time and issues all their partial, bias and
// residual loads before the first use, so a batch costs one memory latency.
constexpr int kRedMaxSplits = 8;
constexpr int kRedBatch = 4;

template <int BN, bool OUT_F32>
__device__ __forceinline__ void splitk_reduce(const GemmParams& p, int tile, int split, int num_n, int tid) {
    constexpr int E = 128 * BN / 4;
    constexpr int NS = BN / 64;  // 32-column steps per epilogue warp (half a tile row)
    const int S = p.splits;
    const int64_t m0 = static_cast<int64_t>(tile / num_n) * 128;
    const int n0 = (tile % num_n) * BN;
    const float4* __restrict__ part = reinterpret_cast<const float4*>(p.ws) + static_cast<size_t>(tile) * S * E;
    const int lo = split * E / S, hi = (split + 1) * E / S;
    for (int e0 = lo + tid; e0 < hi; e0 += 256 * kRedBatch) {
        int64_t row[kRedBatch];
        int col[kRedBatch];
        bool live[kRedBatch];
        float4 buf[kRedMaxSplits][kRedBatch];
        float4 bb[kRedBatch];
        float4 rr[kRedBatch];
#pragma unroll
        for (int b = 0; b < kRedBatch; ++b) {
            const int e = e0 + 256 * b;
            const int l = e & 31, g = (e >> 5) & 7, rest = e >> 8;
            const int ew = rest / NS, step = rest - ew * NS;
            row[b] = m0 + 32 * (ew & 3) + l;
            col[b] = n0 + (ew >> 2) * (BN / 2) + 32 * step + 4 * g;
            // n is a multiple of 8: a granule is all in or all out
            live[b] = e < hi && row[b] < p.m && col[b] < p.n;
#pragma unroll
            for (int s = 0; s < kRedMaxSplits; ++s)
                if (live[b] && s < S) buf[s][b] = __ldcg(part + static_cast<size_t>(s) * E + e);
            bb[b] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (live[b] && p.bias != nullptr) {
                if (p.bias_f32) {
                    bb[b] = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.bias) + col[b]));
                } else {
                    const uint2 h = __ldg(reinterpret_cast<const uint2*>(static_cast<const __half*>(p.bias) + col[b]));
                    const float2 b0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                    const float2 b1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                    bb[b] = make_float4(b0.x, b0.y, b1.x, b1.y);
                }
            }
            rr[b] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (live[b] && p.residual != nullptr) {
                if constexpr (OUT_F32) {
                    rr[b] = *reinterpret_cast<const float4*>(static_cast<const float*>(p.residual) + row[b] * p.ldr + col[b]);
                } else {
                    const uint2 h = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p.residual) + row[b] * p.ldr + col[b]);
                    const float2 r0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                    const float2 r1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                    rr[b] = make_float4(r0.x, r0.y, r1.x, r1.y);
                }
            }
        }
#pragma unroll
        for (int b = 0; b < kRedBatch; ++b) {
            if (!live[b]) continue;
            float4 a = buf[0][b];
#pragma unroll
            for (int s = 1; s < kRedMaxSplits; ++s) {
                if (s < S) {
                    a.x += buf[s][b].x;
                    a.y += buf[s][b].y;
                    a.z += buf[s][b].z;
                    a.w += buf[s][b].w;
                }
            }
            float v[4] = {a.x, a.y, a.z, a.w};
            if (p.bias != nullptr) {
                v[0] += bb[b].x;
                v[1] += bb[b].y;
                v[2] += bb[b].z;
                v[3] += bb[b].w;
            }
            if (p.activation == kActGelu) {
                gelu_erf_pair(v[0], v[1]);
                gelu_erf_pair(v[2], v[3]);
            }
            if (p.residual != nullptr) {
                v[0] += rr[b].x;
                v[1] += rr[b].y;
                v[2] += rr[b].z;
                v[3] += rr[b].w;
            }
            if constexpr (OUT_F32) {
                *reinterpret_cast<float4*>(static_cast<float*>(p.y) + row[b] * p.ldy + col[b]) =
                    make_float4(v[0], v[1], v[2], v[3]);
            } else {
                __half2 h0 = __floats2half2_rn(v[0], v[1]);
                __half2 h1 = __floats2half2_rn(v[2], v[3]);
                uint2 o;
                o.x = *reinterpret_cast<uint32_t*>(&h0);
                o.y = *reinterpret_cast<uint32_t*>(&h1);
                *reinterpret_cast<uint2*>(static_cast<__half*>(p.y) + row[b] * p.ldy + col[b]) = o;
            }
        }
    }
}

template <int BN, bool OUT_F32, int RES, bool PAIR>
__global__ void __launch_bounds__(384, 1)
    gemm_f16_sm100_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                          const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_r,
                          const __grid_constant__ CUtensorMap tm_wp, const GemmParams p) {
    using C = GemmCfg<BN, RES, PAIR>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_base = smem;
    uint8_t* epi_base = smem + C::STAGES * C::STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi_base + C::EPI_BYTES);
    uint64_t* full_bar = bars;                       // [STAGES]
    uint64_t* empty_bar = bars + C::STAGES;          // [STAGES]
    uint64_t* tfull_bar = bars + 2 * C::STAGES;      // [2]
    uint64_t* tempty_bar = bars + 2 * C::STAGES + 2; // [2]
    uint64_t* drain_bar = bars + 2 * C::STAGES + 4;  // [1] teardown drain of MMAs
    uint64_t* res_bar = bars + 2 * C::STAGES + 5;    // [EPI_WARPS * 2] residual slot landed
    uint64_t* loaded_bar = bars + 2 * C::STAGES + 5 + 2 * C::EPI_WARPS;  // [1] stream-K tail: head loaded into TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::STAGES + 6 + 2 * C::EPI_WARPS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // CTA pairs: rank 0 (leader) issues the MMAs; tiles are scheduled per pair.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    // split-K: CTA blockIdx.x = tile * splits + s takes k-blocks [kb_lo, kb_hi) of one tile
    const int splits = PAIR ? 1 : p.splits;
    const int split = PAIR ? 0 : static_cast<int>(blockIdx.x) % splits;
    const int first_tile = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x) / splits;
    const int tile_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x) / splits;

    const int num_m = static_cast<int>((p.m + C::TILE_M - 1) / C::TILE_M);
    const int num_n = (p.n + BN - 1) / BN;
    const int num_k = (p.k + C::BK - 1) / C::BK;
    const int num_tiles = num_m * num_n;
    const int kb_lo = split * num_k / splits;
    const int kb_hi = (split + 1) * num_k / splits;
    const bool use_res = p.residual != nullptr && splits == 1;  // split-K adds the residual in its reduction
    // units: CTA pairs or CTAs (split-K: tiles); stream-K only without split-K
    constexpr int RANKS = PAIR ? 2 : 1;
    const int sk_tiles = splits == 1 ? p.sk_tiles : 0;
    const int pieces = (PAIR && splits == 1 && sk_tiles == 0) ? p.pieces : 0;
    auto schedule = [&]() {
        return Schedule<BN>(first_tile, tile_step, num_tiles, num_k, sk_tiles, kb_lo, kb_hi, p.tail_tiles, pieces);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull_bar[b], 1);
            mbar_init(&tempty_bar[b], PAIR ? 2 * C::EPI_WARPS : C::EPI_WARPS);
        }
        mbar_init(drain_bar, 1);
        for (int b = 0; b < 2 * C::EPI_WARPS; ++b) mbar_init(&res_bar[b], 1);
        mbar_init(loaded_bar, PAIR ? 2 * C::EPI_WARPS : C::EPI_WARPS);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tm_x);
        prefetch_tmap(&tm_w);
        if (pieces) prefetch_tmap(&tm_wp);
        prefetch_tmap(&tm_y);
        if (use_res) prefetch_tmap(&tm_r);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, C::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // the predecessor's outputs (x, residual) are complete from here on
    pdl_launch_dependents();

    if (warp < 4) {
        setmaxnreg_dec40();
        if (warp == 0 && lane == 0) {
            // -------------------------------------------------------- producer
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            auto sched = schedule();
            WorkItem w;
            while (ok && sched.next(w)) {
                const int tile = w.tile;
                const bool piece = w.width != BN;
                // a piece's weight rows: width / 2 per CTA of a pair, through tm_wp
                const int b_rows = PAIR ? w.width / 2 : w.width;
                const uint32_t stage_bytes = static_cast<uint32_t>(C::A_BYTES + b_rows * C::BK * 2);
                const int m0 = (tile / num_n) * C::TILE_M + static_cast<int>(rank) * C::BM;
                const int n0 = (tile % num_n) * BN + w.n_off + static_cast<int>(rank) * b_rows;
                const CUtensorMap* tw = piece ? &tm_wp : &tm_w;
                for (int kb = w.kb_lo; kb < w.kb_hi; ++kb) {
                    if (!wait_bar(&empty_bar[stage], phase ^ 1, abort_flag, p.err, 101)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = stage_base + stage * C::STAGE_BYTES;
                    if constexpr (PAIR) {
                        // both CTAs' bytes complete on the leader's full barrier
                        if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * stage_bytes);
                        const uint32_t leader_full = mapa_shared(smem_u32(&full_bar[stage]), 0);
                        tma_load_2d_pair(sa, &tm_x, leader_full, kb * C::BK, m0);
                        tma_load_2d_pair(sa + C::A_BYTES, tw, leader_full, kb * C::BK, n0);
                    } else {
                        mbar_arrive_expect_tx(&full_bar[stage], stage_bytes);
                        tma_load_2d(sa, &tm_x, &full_bar[stage], kb * C::BK, m0);
                        tma_load_2d(sa + C::A_BYTES, tw, &full_bar[stage], kb * C::BK, n0);
                    }
                    ++issued;
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Drain: every load issued into the ring must have landed before the
            // CTA may exit (normally already consumed by the MMA warp). With CTA
            // pairs the peer's bytes complete on the leader's barriers, so the
            // leader drains for both (the peer waits at the final cluster barrier).
            const int pending = (PAIR && rank != 0) ? 0 : (issued < C::STAGES ? issued : C::STAGES);
            for (int i = 1; i <= pending; ++i) {
                int s = stage - i;
                uint32_t ph = phase;
                if (s < 0) {
                    s += C::STAGES;
                    ph ^= 1;
                }
                volatile int no_abort = 0;
                wait_bar(&full_bar[s], ph, &no_abort, p.err, 102);
            }
        } else if (warp == 1 && lane == 0 && rank == 0) {
            // -------------------------------------------------------- MMA issuer
            constexpr uint32_t idesc_full = umma_idesc_f16(C::TILE_M, BN);
            // commits go to this CTA's barrier and, for pairs, to the peer's as well
            auto commit_both = [&](uint64_t* bar) {
                if constexpr (PAIR) {
                    const uint32_t a = smem_u32(bar);
                    umma_commit_pair(a);
                    umma_commit_pair(mapa_shared(a, 1));
                } else {
                    umma_commit(bar);
                }
            };
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            auto sched = schedule();
            WorkItem w;
            while (ok && sched.next(w)) {
                if (!wait_bar<PAIR>(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.err, 201)) break;
                // a stream-K tail continues from the head's accumulator, which the
                // epilogue warps (of both CTAs of a pair) load into this buffer first
                const bool cont = w.mode == kItemTail;
                if (cont && !wait_bar<PAIR>(loaded_bar, 0, abort_flag, p.err, 204)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                // a narrow-tail piece: N = its width (the accumulator's first columns)
                const uint32_t idesc = w.width == BN ? idesc_full : umma_idesc_f16(C::TILE_M, w.width);
                for (int kb = w.kb_lo; kb < w.kb_hi; ++kb) {
                    if (!wait_bar(&full_bar[stage], phase, abort_flag, p.err, 202)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(stage_base + stage * C::STAGE_BYTES);
                    const uint64_t a_desc = umma_desc_sw128_kmajor(a_addr);
                    const uint64_t b_desc = umma_desc_sw128_kmajor(a_addr + C::A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < C::BK / 16; ++kk) {
                        // +32 B per K step of 16 fp16 inside the 128-B swizzle row
                        const bool accumulate = cont || (kb - w.kb_lo) + kk != 0;
                        if constexpr (PAIR)
                            umma_f16_pair(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, accumulate);
                        else
                            umma_f16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, accumulate);
                    }
                    commit_both(&empty_bar[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                commit_both(&tfull_bar[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            // Teardown: make sure no MMA is still writing TMEM before it is freed.
            if constexpr (PAIR)
                umma_commit_pair(smem_u32(drain_bar));
            else
                umma_commit(drain_bar);
            volatile int no_abort = 0;
            wait_bar(drain_bar, 0, &no_abort, p.err, 203);
        }
        if constexpr (!PAIR) {
            if (splits > 1) {
                __syncwarp();
                cluster_sync();  // the split-K exchange barrier, which every thread of the cluster joins
            }
        }
    } else {
        setmaxnreg_inc232();
        // ------------------------------------------------------------ epilogue
        // CW output columns per step = 128 bytes per row (64 fp16 or 32 fp32).
        constexpr int CW = OUT_F32 ? 32 : 64;
        constexpr int HALF = BN / 2;
        static_assert(HALF % CW == 0, "column half must hold whole steps");
        const int q = warp & 3;                // TMEM lane quarter accessible to this warp
        const int col_half = (warp - 4) >> 2;  // 0: columns [0, BN/2), 1: [BN/2, BN)
        const int ew = warp - 4;               // epilogue warp index 0..7
        uint8_t* slots = epi_base + ew * C::EPI_SLOTS * C::EPI_BUF_BYTES;
        // TMA load of residual step (row0, col0) into slot s of this warp
        auto load_residual = [&](int s, int col0, int64_t row0) {
            mbar_arrive_expect_tx(&res_bar[2 * ew + s], C::EPI_BUF_BYTES);
            tma_load_2d(slots + s * C::EPI_BUF_BYTES, &tm_r, &res_bar[2 * ew + s], col0,
                        static_cast<int32_t>(row0));
        };
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t j = 0;  // running step counter of this warp (slot = j & 1 with a residual)
        // the accumulator is released to the leader's MMA warp (both CTAs' warps)
        const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
        const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty_bar[1]), 0);
        // stream-K partials and flags of this CTA's unit (slot = unit * RANKS + rank)
        constexpr int NS = HALF / 32;  // 32-column partial steps per warp
        const size_t sk_slot = static_cast<size_t>(first_tile) * RANKS + rank;
        // the previous unit's head (same rank, rows and columns, same layout) into
        // accumulator buffer `buf`; false when the bounded wait gave up
        auto preload_tail = [&](int buf) -> bool {
            const size_t hslot = sk_slot - RANKS;
            int* hflag = p.sk_flags + hslot * C::EPI_WARPS + ew;
            const float4* src = reinterpret_cast<const float4*>(p.ws) + hslot * (C::BM * BN / 4) +
                                static_cast<size_t>(ew) * NS * 256 + lane;
            const uint32_t t_dst = tmem_base + (static_cast<uint32_t>(32 * q) << 16) +
                                   static_cast<uint32_t>(buf * BN + col_half * HALF);
            bool got = true;
            if (lane == 0) got = sk_wait(hflag, abort_flag, p.err, 303);
            if (__shfl_sync(0xffffffffu, got ? 1 : 0, 0) == 0) return false;
#pragma unroll 1
            for (int c = 0; c < NS; ++c) {
                float4 pv[8];
#pragma unroll
                for (int g = 0; g < 8; ++g) pv[g] = __ldcg(src + (c * 8 + g) * 32);
                uint32_t r0[16], r1[16];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    r0[4 * g + 0] = __float_as_uint(pv[g].x);
                    r0[4 * g + 1] = __float_as_uint(pv[g].y);
                    r0[4 * g + 2] = __float_as_uint(pv[g].z);
                    r0[4 * g + 3] = __float_as_uint(pv[g].w);
                    r1[4 * g + 0] = __float_as_uint(pv[g + 4].x);
                    r1[4 * g + 1] = __float_as_uint(pv[g + 4].y);
                    r1[4 * g + 2] = __float_as_uint(pv[g + 4].z);
                    r1[4 * g + 3] = __float_as_uint(pv[g + 4].w);
                }
                tmem_st_32x32b_x16(t_dst + 32 * c, r0);
                tmem_st_32x32b_x16(t_dst + 32 * c + 16, r1);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                *reinterpret_cast<volatile int*>(hflag) = 0;  // read: zero again for the next call
                if constexpr (PAIR)
                    mbar_arrive_cluster(mapa_shared(smem_u32(loaded_bar), 0));
                else
                    mbar_arrive(loaded_bar);
            }
            return true;
        };
        bool tail_loaded = false;
        auto sched = schedule();
        WorkItem w;
        while (sched.next(w)) {
            const int tile = w.tile;
            const int64_t m0 = static_cast<int64_t>(tile / num_n) * C::TILE_M + static_cast<int64_t>(rank) * C::BM;
            // a narrow-tail piece (width <= HALF) is drained by the first column half's warps
            const bool piece = w.width != BN;
            const int c_begin = (tile % num_n) * BN + w.n_off + (piece ? 0 : col_half * HALF);
            const int64_t row0 = m0 + 32 * q;
            const int valid = piece ? (col_half == 0 ? min(w.width, p.n - c_begin) : 0)
                                    : min(HALF, p.n - c_begin);  // may be <= 0 for the last tile
            const int nsteps = (valid > 0 && row0 < p.m) ? (valid + CW - 1) / CW : 0;
            // raw accumulator out instead of an epilogue: split-K, or the head of a cut stream-K tile
            const bool partial = splits > 1 || w.mode == kItemHead;
            if constexpr (RES > 0) {
                // first residual step of the tile lands while the main loop runs
                if (lane == 0 && nsteps > 0 && !partial) {
                    bulk_wait_group_read<0>();
                    load_residual(RES == 2 ? (j & 1) : 0, c_begin, row0);
                }
            }
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16) +
                                   static_cast<uint32_t>(acc * BN + (piece ? 0 : col_half * HALF));
            // stream-K tail: the previous unit's head goes into the tail's TMEM buffer
            // before the tail's MMAs start, while the item before it is still being
            // computed (that buffer was freed by this warp's previous epilogue). When
            // the item before the tail is this unit's own head, the load waits until
            // that head is written and flagged, so no unit's head ever waits.
            bool preload_after_head = false;
            if (splits == 1) {
                if (w.mode == kItemTail && !tail_loaded) {
                    if (!preload_tail(acc)) break;
                    tail_loaded = true;
                }
                WorkItem nx;
                auto look = sched;
                if (look.next(nx) && nx.mode == kItemTail) {
                    if (w.mode == kItemHead) {
                        preload_after_head = true;
                    } else {
                        if (!preload_tail(acc ^ 1)) break;
                        tail_loaded = true;
                    }
                }
            }
            if (!wait_bar(&tfull_bar[acc], acc_phase, abort_flag, p.err, 301)) break;
            tc_fence_after();
            bool ok = true;
            if (partial) {
                // the raw accumulator, 32 columns per step; granule (ew, step, g) of
                // lane l at float4 ((ew * NS + step) * 8 + g) * 32 + l of the slot
                const size_t slot = splits > 1 ? static_cast<size_t>(blockIdx.x) : sk_slot;
                float4* dst = reinterpret_cast<float4*>(p.ws) + slot * (C::BM * BN / 4) +
                              static_cast<size_t>(ew) * NS * 256 + lane;
#pragma unroll 1
                for (int c = 0; c < NS; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + 32 * c, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        __stcg(dst + (c * 8 + g) * 32, make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                                                   __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3])));
                }
                if (splits == 1) {
                    // stream-K: every lane's stores are visible device-wide before the flag
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) sk_signal(p.sk_flags + sk_slot * C::EPI_WARPS + ew);
                    if (preload_after_head) {
                        ok = preload_tail(acc ^ 1);
                        tail_loaded = true;
                    }
                }
            }
#pragma unroll 1
            for (int c = 0; c < (partial ? 0 : nsteps); ++c, ++j) {
                const int col0 = c_begin + c * CW;
                if constexpr (RES == 2) {
                    // next residual step into the other slot, once that slot's
                    // previous store has been read out
                    if (lane == 0 && c + 1 < nsteps) {
                        bulk_wait_group_read<0>();
                        load_residual((j + 1) & 1, col0 + CW, row0);
                    }
                } else if constexpr (RES == 1) {
                    // single slot: this step's residual (the first one of the tile
                    // was issued before the accumulator wait)
                    if (lane == 0 && c > 0) {
                        bulk_wait_group_read<0>();
                        load_residual(0, col0, row0);
                    }
                }
                // this step's bias words are requested before the TMEM wait, so the two
                // latencies overlap (every lane reads the same 16 B: one broadcast each);
                // only a step that crosses n needs per-word bounds
                uint4 bq[CW / 4];
                if (p.bias != nullptr) {
                    const bool whole = col0 + CW <= p.n;
                    if (p.bias_f32) {
                        const uint4* bp = reinterpret_cast<const uint4*>(static_cast<const float*>(p.bias) + col0);
                        if (whole) {
#pragma unroll
                            for (int g = 0; g < CW / 4; ++g) bq[g] = __ldg(bp + g);
                        } else {
#pragma unroll
                            for (int g = 0; g < CW / 4; ++g)
                                bq[g] = col0 + 4 * g < p.n ? __ldg(bp + g) : make_uint4(0u, 0u, 0u, 0u);
                        }
                    } else {
                        const uint4* bp = reinterpret_cast<const uint4*>(static_cast<const __half*>(p.bias) + col0);
                        if (whole) {
#pragma unroll
                            for (int g = 0; g < CW / 8; ++g) bq[g] = __ldg(bp + g);
                        } else {
#pragma unroll
                            for (int g = 0; g < CW / 8; ++g)
                                bq[g] = col0 + 8 * g < p.n ? __ldg(bp + g) : make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
                }
                uint32_t r[CW];
#pragma unroll
                for (int h = 0; h < CW / 32; ++h)
                    tmem_ld_32x32b_x32(t_row + c * CW + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * h]));
                tmem_ld_wait();
                float v[CW];
#pragma unroll
                for (int jj = 0; jj < CW; ++jj) v[jj] = __uint_as_float(r[jj]);
                if (p.bias != nullptr && p.bias_f32) {
#pragma unroll
                    for (int g = 0; g < CW / 4; ++g) {
                        v[4 * g + 0] += __uint_as_float(bq[g].x);
                        v[4 * g + 1] += __uint_as_float(bq[g].y);
                        v[4 * g + 2] += __uint_as_float(bq[g].z);
                        v[4 * g + 3] += __uint_as_float(bq[g].w);
                    }
                } else if (p.bias != nullptr) {
#pragma unroll
                    for (int g = 0; g < CW / 8; ++g) {
                        const __half2* bh = reinterpret_cast<const __half2*>(&bq[g]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(bh[e]);
                            v[8 * g + 2 * e] += f.x;
                            v[8 * g + 2 * e + 1] += f.y;
                        }
                    }
                }
                if (p.activation == kActGelu) {
#pragma unroll
                    for (int jj = 0; jj < CW; jj += 2) gelu_erf_pair(v[jj], v[jj + 1]);
                }
                const uint32_t slot = RES == 2 ? (j & 1) : 0;
                uint8_t* buf = slots + slot * C::EPI_BUF_BYTES;
                if constexpr (RES > 0) {
                    // uses of this slot so far: j / 2 (two slots) or j (one slot)
                    const uint32_t parity = RES == 2 ? ((j >> 1) & 1) : (j & 1);
                    if (!wait_bar(&res_bar[2 * ew + slot], parity, abort_flag, p.err, 302)) {
                        ok = false;
                        break;
                    }
                    // this thread's row of the residual step (128-B swizzle)
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const uint4 rv = *reinterpret_cast<const uint4*>(buf + lane * 128 + ((g ^ (lane & 7)) << 4));
                        if constexpr (OUT_F32) {
                            v[4 * g + 0] += __uint_as_float(rv.x);
                            v[4 * g + 1] += __uint_as_float(rv.y);
                            v[4 * g + 2] += __uint_as_float(rv.z);
                            v[4 * g + 3] += __uint_as_float(rv.w);
                        } else {
                            const __half2* rh = reinterpret_cast<const __half2*>(&rv);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = __half22float2(rh[e]);
                                v[8 * g + 2 * e] += f.x;
                                v[8 * g + 2 * e + 1] += f.y;
                            }
                        }
                    }
                    __syncwarp();  // every lane has read its row before any lane overwrites the slot
                } else {
                    // single slot: wait until the previous TMA store has read it
                    if (lane == 0) bulk_wait_group_read<0>();
                    __syncwarp();
                }
#pragma unroll
                for (int g = 0; g < 8; ++g) {  // eight 16-B granules per 128-B row
                    uint4 pk;
                    if constexpr (OUT_F32) {
                        pk.x = __float_as_uint(v[4 * g + 0]);
                        pk.y = __float_as_uint(v[4 * g + 1]);
                        pk.z = __float_as_uint(v[4 * g + 2]);
                        pk.w = __float_as_uint(v[4 * g + 3]);
                    } else {
                        __half2 h0 = __floats2half2_rn(v[8 * g + 0], v[8 * g + 1]);
                        __half2 h1 = __floats2half2_rn(v[8 * g + 2], v[8 * g + 3]);
                        __half2 h2 = __floats2half2_rn(v[8 * g + 4], v[8 * g + 5]);
                        __half2 h3 = __floats2half2_rn(v[8 * g + 6], v[8 * g + 7]);
                        pk.x = *reinterpret_cast<uint32_t*>(&h0);
                        pk.y = *reinterpret_cast<uint32_t*>(&h1);
                        pk.z = *reinterpret_cast<uint32_t*>(&h2);
                        pk.w = *reinterpret_cast<uint32_t*>(&h3);
                    }
                    // 128-B swizzle: 16-B granule g of row `lane` lives at g ^ (lane & 7)
                    *reinterpret_cast<uint4*>(buf + lane * 128 + ((g ^ (lane & 7)) << 4)) = pk;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tm_y, buf, col0, static_cast<int32_t>(row0));
                    bulk_commit_group();
                }
            }
            if (!ok) break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR)
                    mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
                else
                    mbar_arrive(&tempty_bar[acc]);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
        if constexpr (!PAIR) {
            if (splits > 1) {
                // every split's partial is written (release) and visible here (acquire);
                // the reduction runs in this register-rich region
                cluster_sync();
                if (first_tile < num_tiles) splitk_reduce<BN, OUT_F32>(p, first_tile, split, num_n, threadIdx.x - 128);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // the peer is done with TMEM and with our barriers
    tc_fence_after();
    if (warp == 1) {
        if constexpr (PAIR)
            tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
        else
            tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

}  // namespace rpfq
