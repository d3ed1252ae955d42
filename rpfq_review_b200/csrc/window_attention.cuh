// Swin window attention on tcgen05: softmax(Q K^T / sqrt(32) + bias) V for
// every (7x7 window, head), head dim 32, where bias = relative position bias
// (+ the shift mask on shifted blocks), the attention of the blocks the
// reference's Swin models wrap (RPFQ-ViT-main/quant_models/quant_rpfq_swin.py:64-91;
// timm's WindowAttention, restated in oracle/swin_ref.py).
//
// Input: the qkv GEMM output in window order, [windows * 49, 3 C] fp16 (per
// token q heads, k heads, v heads, 32 columns each; C = 32 heads), read
// through a 2-D tensor map with [64 rows x 64 columns] boxes: one box is one
// window's 49 tokens (the 15 rows after them belong to the next window or lie
// past the end and read as zeros; they only ever meet zero weights) for a
// pair of heads. bias_mask: log2(e) (bias + mask) as fp32, per (window entry,
// head) a [16][49][4] block (key column j of query row i at ((j / 4) 49 + i) 4 +
// j % 4, so that the 49 rows of a column group are consecutive), -inf in key
// columns 49..63; it reaches shared memory with the item's Q / K / V (one bulk
// copy per window) and every softmax thread reads its row conflict-free.
// Output: [windows * 49, ldo] fp16, head h in columns [32 h, 32 h + 32) (the
// proj GEMM's input).
//
// Work item = (pair of windows, pair of heads): a 128-row tile stacks the two
// windows (rows 0..63 and 64..127), so
//   S_g = Q_g K_g^T   M = 128, N = 128 keys, K = 32 (head g's half of the tile)
//   O_g = P_g V       M = 128, N = 64 (both heads' V columns; head g keeps its
//                     32), K = 128 keys; P_g from TMEM
// where a query row only weighs the keys of its own window (the others and
// the padding get weight exactly 0).
// Persistent CTAs, 10 warps:
//   warp 0    TMA producer into two shared-memory stages (Q, K, V of an item)
//   warp 1    TMEM (512 columns: two item buffers x two heads x 128) and the
//             MMA issue, software-pipelined: S of item k is issued before
//             P V of item k - 1, so the tensor core works while the softmax
//             warps do
//   warps 2-9 group g = head slot g of each item, one query row per thread:
//             t = S c + bias_mask, row max, p = 2^(t - max) (SFU ex2) packed
//             as fp16 over the first 64 columns of S_g, row sum of the rounded
//             p, then O_g / sum to global.
// Every wait is bounded (wait_bar) and reports through the device error word.
#pragma once

#include "ptx.cuh"

namespace rpfq {

struct WinAttnParams {
    const float* bias_mask;  // [bm_windows, heads, 16, 49, 4] fp32, log2(e) scaled
    __half* out;             // [windows * 49, ldo]
    int64_t ldo;
    int32_t windows;
    int32_t heads;
    int32_t bm_windows;      // window w uses bias_mask entry w % bm_windows
    float scale_log2;        // log2(e) / sqrt(32)
    int* err;
};

struct WinAttnCfg {
    static constexpr int L = 49;                // tokens per window
    static constexpr int LP = 64;               // padded rows / keys per window
    static constexpr int HD = 32;
    static constexpr int BOX = LP * 64 * 2;     // one [64 rows x 64 fp16] box = 8 KB
    static constexpr int TILE = 2 * BOX;        // two windows = 128 rows
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = TILE;
    static constexpr int V_OFF = 2 * TILE;
    static constexpr int BM_HEAD = L * LP * 4;    // one head's bias rows: 12544 B
    static constexpr int BM_OFF = 3 * TILE;       // [window half][head slot] blocks
    static constexpr int STAGE_BYTES = 3 * TILE + 4 * BM_HEAD;  // 98 KB (a multiple of 1024)
    static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
    static constexpr int STAGES = 2;
    static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
    static constexpr int SMEM_BYTES = 1024 + BAR_OFF + 512;
    static constexpr int THREADS = 320;
    static constexpr int TMEM_COLS = 512;       // buffer b, head slot g: [256 b + 128 g, + 128)
    static constexpr int O_COL = 64;            // O next to P (P: columns 0..63 of the region)
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

__global__ void __launch_bounds__(320, 1)
    attn_window_sm100_kernel(const __grid_constant__ CUtensorMap tm_qkv, const WinAttnParams p) {
    using C = WinAttnCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* load_full = bars;         // [stage]
    uint64_t* stage_free = bars + 2;    // [stage]
    uint64_t* s_full = bars + 4;        // [buffer * 2 + slot]
    uint64_t* p_full = bars + 8;        // [buffer * 2 + slot] (4 warps)
    uint64_t* o_full = bars + 12;       // [buffer * 2 + slot]
    uint64_t* tmem_free = bars + 16;    // [buffer * 2 + slot] (4 warps)
    uint64_t* drain = bars + 20;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpairs = (p.windows + 1) >> 1;
    const int hpairs = (p.heads + 1) >> 1;
    const int items = wpairs * hpairs;
    const int cdim = p.heads * C::HD;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&load_full[i], 1);
            mbar_init(&stage_free[i], 1);
        }
        for (int i = 0; i < 4; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&o_full[i], 1);
            mbar_init(&tmem_free[i], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tm_qkv);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // the predecessor's outputs (qkv) are complete from here on
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------ producer
            int issued = 0;
            for (int item = blockIdx.x, k = 0; item < items; item += gridDim.x, ++k) {
                const int st = k & 1;
                if (k >= 2 && !wait_bar(&stage_free[st], static_cast<uint32_t>((k >> 1) - 1) & 1, abort_flag, p.err, 831))
                    break;
                const int wp = item / hpairs, hp = item - wp * hpairs;
                const int nslots = min(2, p.heads - 2 * hp);
                const int nwin = min(2, p.windows - 2 * wp);
                uint8_t* sm = smem + st * C::STAGE_BYTES;
                mbar_arrive_expect_tx(&load_full[st], 3 * C::TILE + nwin * nslots * C::BM_HEAD);
                for (int t = 0; t < 2; ++t) {
                    // window 2 wp + t (past the last window: rows past the end, zero-filled)
                    const int32_t row = (2 * wp + t) * C::L;
                    tma_load_2d(sm + C::Q_OFF + t * C::BOX, &tm_qkv, &load_full[st], 64 * hp, row);
                    tma_load_2d(sm + C::K_OFF + t * C::BOX, &tm_qkv, &load_full[st], cdim + 64 * hp, row);
                    tma_load_2d(sm + C::V_OFF + t * C::BOX, &tm_qkv, &load_full[st], 2 * cdim + 64 * hp, row);
                    if (t < nwin) {
                        // this window's bias rows of both heads (consecutive in bias_mask)
                        const float* bsrc = p.bias_mask + (static_cast<int64_t>((2 * wp + t) % p.bm_windows) * p.heads +
                                                           2 * hp) * (C::BM_HEAD / 4);
                        bulk_load_1d(sm + C::BM_OFF + t * 2 * C::BM_HEAD, bsrc, nslots * C::BM_HEAD, &load_full[st]);
                    }
                }
                ++issued;
            }
            for (int k = issued - 1; k >= 0 && k >= issued - 2; --k) {
                volatile int no_abort = 0;
                wait_bar(&load_full[k & 1], static_cast<uint32_t>(k >> 1) & 1, &no_abort, p.err, 832);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            const uint32_t base = smem_u32(smem);
            constexpr uint32_t idesc_s = umma_idesc_f16(128, 2 * C::LP);
            constexpr uint32_t idesc_o = umma_idesc_f16(128, 64) | (1u << 16);  // B (= V) MN-major
            // issued P V per (buffer, slot): one byte each of a register (only the
            // parity and "any so far" are used; a count saturates at 255 -> kept below)
            uint32_t uses = 0;
            auto uses_of = [&](int slot) { return (uses >> (8 * slot)) & 0xffu; };
            auto bump = [&](int slot) {
                const uint32_t u = uses_of(slot);
                // keep the parity, stay nonzero: 255 -> 254
                const uint32_t nu = u == 255u ? 254u : u + 1u;
                uses = (uses & ~(0xffu << (8 * slot))) | (nu << (8 * slot));
            };
            bool ok = true;
            int prev_item = -1;
            for (int item = blockIdx.x, k = 0; ok; item += gridDim.x, ++k) {
                const bool have = item < items;
                if (have) {
                    const int st = k & 1;
                    const int hp = item % hpairs;
                    const int nslots = min(2, p.heads - 2 * hp);
                    if (!wait_bar(&load_full[st], static_cast<uint32_t>(k >> 1) & 1, abort_flag, p.err, 833)) break;
                    const uint32_t sb = base + st * C::STAGE_BYTES;
                    const uint64_t qdesc = umma_desc_sw128_kmajor(sb + C::Q_OFF);
                    const uint64_t kdesc = umma_desc_sw128_kmajor(sb + C::K_OFF);
                    for (int g = 0; g < nslots; ++g) {
                        const int slot = 2 * st + g;
                        if (uses_of(slot) > 0 &&
                            !wait_bar(&tmem_free[slot], (uses_of(slot) - 1) & 1, abort_flag, p.err, 834)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // head slot g: columns 32 g .. 32 g + 31 of the tile = K steps 2 g, 2 g + 1
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk)
                            umma_f16(tmem_base + 128 * slot, qdesc + 2 * (2 * g + kk), kdesc + 2 * (2 * g + kk),
                                     idesc_s, kk != 0);
                        umma_commit(&s_full[slot]);
                    }
                    if (!ok) break;
                }
                if (k >= 1) {
                    // P V of the previous item
                    const int stp = (k - 1) & 1;
                    const int hp = prev_item % hpairs;
                    const int nslots = min(2, p.heads - 2 * hp);
                    const uint32_t sb = base + stp * C::STAGE_BYTES;
                    for (int g = 0; g < nslots; ++g) {
                        const int slot = 2 * stp + g;
                        if (!wait_bar(&p_full[slot], uses_of(slot) & 1, abort_flag, p.err, 835)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        for (int kk = 0; kk < 2 * C::LP / 16; ++kk) {
                            const uint64_t vdesc = umma_desc_sw128_mnmajor(sb + C::V_OFF + kk * 2048);
                            // A = P from TMEM: keys 16 kk .. 16 kk + 15 are columns 8 kk .. 8 kk + 7
                            umma_f16_ts(tmem_base + 128 * slot + C::O_COL, tmem_base + 128 * slot + 8 * kk, vdesc,
                                        idesc_o, kk != 0);
                        }
                        umma_commit(&o_full[slot]);
                        bump(slot);
                    }
                    if (!ok) break;
                    umma_commit(&stage_free[stp]);
                }
                if (!have) break;
                prev_item = item;
            }
            umma_commit(drain);
            volatile int no_abort = 0;
            wait_bar(drain, 0, &no_abort, p.err, 836);
        }
    } else {
        // ---------------------------------------------------------------- softmax + output
        const int g = (warp - 2) >> 2;  // head slot of this warp group
        const int q = warp & 3;         // TMEM lane quarter
        const int row = 32 * q + lane;  // tile row: window half row / 64, query row % 64
        const int half = row >> 6, i = row & 63;
        const bool real_row = i < C::L;
        const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
        uint32_t uses0 = 0, uses1 = 0;  // this group's uses of its slot in buffer 0 / 1
        for (int item = blockIdx.x, k = 0; item < items; item += gridDim.x, ++k) {
            const int wp = item / hpairs, hp = item - wp * hpairs;
            const int h = 2 * hp + g;
            if (h >= p.heads) continue;  // odd head count: no second head in the last pair
            const int b = k & 1, slot = 2 * b + g;
            const uint32_t ub = b ? uses1 : uses0;
            const int w = 2 * wp + half;
            const bool live = real_row && w < p.windows;
            // this row's bias (+ mask) in the item's stage: column group u at (u 49 + i) 16 B
            const float4* bm4 = reinterpret_cast<const float4*>(smem + b * C::STAGE_BYTES + C::BM_OFF +
                                                                (2 * half + g) * C::BM_HEAD) + i;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(128 * slot);
            if (!wait_bar(&s_full[slot], ub & 1, abort_flag, p.err, 837)) break;
            tc_fence_after();
            // S columns of this row's window: 64 half .. 64 half + 63
            uint32_t r[2][32];
            tmem_ld_32x32b_x32(t_row + 64 * half, r[0]);
            tmem_ld_32x32b_x32(t_row + 64 * half + 32, r[1]);
            tmem_ld_wait();
            float inv_sum = 0.0f;
            uint32_t pw[2][16];  // p of the own window's keys, packed fp16 pairs
            if (live) {
                // t = S c + bias_mask, in place over the S registers
                float m8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) m8[u] = -INFINITY;
#pragma unroll
                for (int u = 0; u < C::LP / 4; ++u) {
                    const float4 bq = bm4[u * C::L];
                    const float bv[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
                    for (int e2 = 0; e2 < 4; e2 += 2) {
                        const int e = 4 * u + e2;
                        float a0, a1;
                        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[e >> 5][e & 31]), __uint_as_float(r[e >> 5][(e & 31) + 1])),
                                         c2, f2_pack(bv[e2], bv[e2 + 1])),
                                  a0, a1);
                        r[e >> 5][e & 31] = __float_as_uint(a0);
                        r[e >> 5][(e & 31) + 1] = __float_as_uint(a1);
                        m8[e & 7] = fmaxf(m8[e & 7], a0);
                        m8[(e + 1) & 7] = fmaxf(m8[(e + 1) & 7], a1);
                    }
                }
                const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                       fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
                const uint64_t nm2 = f2_pack(-mx, -mx);
                float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int u = 0; u < C::LP / 2; ++u) {
                    float a0, a1;
                    const int e = 2 * u;
                    f2_unpack(f2_add(f2_pack(__uint_as_float(r[e >> 5][e & 31]), __uint_as_float(r[e >> 5][(e & 31) + 1])),
                                     nm2),
                              a0, a1);
                    // masked keys: t = -inf, 2^-inf = 0
                    const __half2 hh = __floats2half2_rn(ex2_approx(a0), ex2_approx(a1));
                    const float2 f = __half22float2(hh);
                    s4[u & 3] += f.x + f.y;
                    pw[u >> 4][u & 15] = *reinterpret_cast<const uint32_t*>(&hh);
                }
                inv_sum = 1.0f / ((s4[0] + s4[1]) + (s4[2] + s4[3]));
            } else {
#pragma unroll
                for (int u = 0; u < 16; ++u) pw[0][u] = pw[1][u] = 0u;
            }
            // P over columns 0..63 (keys 0..127): the own window's 32 columns carry p,
            // the other window's 32 columns are zero
            uint32_t zero[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) zero[u] = 0u;
            tmem_st_32x32b_x16(t_row + 32 * half, pw[0]);
            tmem_st_32x32b_x16(t_row + 32 * half + 16, pw[1]);
            tmem_st_32x32b_x16(t_row + 32 * (1 - half), zero);
            tmem_st_32x32b_x16(t_row + 32 * (1 - half) + 16, zero);
            tmem_st_wait();
            tc_fence_before();  // P is in TMEM; O will land next to it
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[slot]);
            if (!wait_bar(&o_full[slot], ub & 1, abort_flag, p.err, 838)) break;
            tc_fence_after();
            uint32_t o[32];
            tmem_ld_32x32b_x32(t_row + C::O_COL + 32 * g, o);  // head g's 32 of the 64 V columns
            tmem_ld_wait();
            if (live) {
                __half* orow = p.out + (static_cast<int64_t>(w) * C::L + i) * p.ldo + h * C::HD;
#pragma unroll
                for (int gg = 0; gg < 4; ++gg) {
                    uint32_t o4[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const __half2 hh = __floats2half2_rn(__uint_as_float(o[8 * gg + 2 * u]) * inv_sum,
                                                             __uint_as_float(o[8 * gg + 2 * u + 1]) * inv_sum);
                        o4[u] = *reinterpret_cast<const uint32_t*>(&hh);
                    }
                    *reinterpret_cast<uint4*>(orow + 8 * gg) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_free[slot]);
            if (b)
                ++uses1;
            else
                ++uses0;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace rpfq
