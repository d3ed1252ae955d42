// Short-sequence multi-head attention on tcgen05 for the ViT / DeiT token
// counts (L <= 256 keys, head dim 64): softmax(Q K^T / sqrt(64)) V per
// (image, head), all keys in one tile, so O is never rescaled (only the
// weights already written, in the rare case described at the softmax).
//
// Input: the qkv GEMM output [B, L, 3 d] (fp16; per token q heads, k heads, v
// heads, 64 columns each), read through a 3-D tensor map [B][L][3 d] so that
// rows past L are zero-filled. Output: [B, L, d] fp16 (heads concatenated),
// the proj GEMM's input. Mirrors timm's Attention.forward as used by the
// reference models (RPFQ-ViT-main/quant_models/quant_rpfq_vit.py; runtime
// restatement RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:612-614).
//
// Persistent CTAs (10 warps, one per SM), lk = L rounded up to 16, query tile g:
//   warp 0    TMA: Q (one or two 128-row tiles), K and V (one or two boxes
//             each) into one of two shared-memory stages
//   warp 1    TMEM (512 columns) + MMA issue:
//               S_g = Q_g K^T   M=128, N=lk, K=64   -> TMEM cols [256 g, 256 g + lk)
//               O_g = P_g V     M=128, N=64, K=lk   -> TMEM cols [256 g + 128, 256 g + 192)
//             (P_g is the TMEM A operand; V the B operand in its natural
//             [key][dim] layout: MN-major)
//   warps 2-9 group g = query tile g, one query row per thread, one pass over
//             S: p = 2^((s - m) c) (SFU ex2) against a reference m raised only
//             when a chunk of keys exceeds it by 2^12, row sum of the
//             fp16-rounded p, P as packed fp16 over the first lk/2 columns of
//             S_g, then O_g / sum to global.
// Every wait is bounded (wait_bar) and reports through the device error word.
#pragma once

#include "ptx.cuh"

namespace rpfq {

struct AttnParams {
    __half* out;       // [B * L, ldo]
    int64_t ldo;
    int32_t images;
    int32_t L;         // tokens per image (<= 256)
    int32_t heads;     // d = 64 * heads
    float scale_log2;  // log2(e) / sqrt(head_dim)
    int* err;
};

struct AttnCfg {
    static constexpr int HD = 64;
    static constexpr int LK = 256;             // largest key tile
    static constexpr int TILE = 128 * HD * 2;  // one 128-row x 64 fp16 tile = 16 KB
    // One stage per (image, head): Q0 | Q1 | K (2 tiles) | V (2 tiles) = 96 KB.
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = 2 * TILE;
    static constexpr int V_OFF = 4 * TILE;
    static constexpr int STAGE_BYTES = 6 * TILE;
    static constexpr int STAGES = 2;
    static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
    static constexpr int SMEM_BYTES = 1024 + BAR_OFF + 256;
    static constexpr int THREADS = 320;
    static constexpr int TMEM_COLS = 512;  // query tile g: S / P at 256 g, O at 256 g + 128
    static constexpr int O_COL = 128;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

__device__ __forceinline__ uint64_t umma_desc_sw128_mnmajor(uint32_t smem_addr) {
    // MN-major, 128-B swizzle: 64 contiguous MN elements per 128-B row, 8 K
    // rows per 1024-B atom. With an MN extent of exactly one atom (64) only
    // the K-direction atom stride is used; both offset fields hold it.
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1024 >> 4) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Persistent, one CTA per SM: CTA c takes (image, head) items c, c + grid, ...;
// its k-th item uses shared-memory stage k % 2, so the next item's Q, K, V
// load while the current one computes. Both 128-query tiles of an item share
// one K / V load.
__global__ void __launch_bounds__(320, 1)
    attn_short_sm100_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnParams p) {
    using C = AttnCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* load_full = bars;        // [stage] Q, K, V landed
    uint64_t* stage_free = bars + 2;   // [stage] the item's MMAs are done reading it
    uint64_t* s_full = bars + 4;       // [tile] S in TMEM
    uint64_t* p_full = bars + 6;       // [tile] P in TMEM (4 warps)
    uint64_t* o_full = bars + 8;       // [tile] O in TMEM
    uint64_t* tmem_free = bars + 10;   // [tile] O read out (4 warps)
    uint64_t* drain = bars + 12;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = p.images * p.heads;
    const int d = p.heads * C::HD;
    const int lk = (p.L + 15) & ~15;  // keys the MMAs cover (N of S, K of P V)
    const int kboxes = (lk + 127) >> 7;
    const int qtiles = (p.L + 127) >> 7;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&load_full[i], 1);
            mbar_init(&stage_free[i], 1);
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
                const uint32_t use = static_cast<uint32_t>(k >> 1);
                if (use > 0 && !wait_bar(&stage_free[st], (use - 1) & 1, abort_flag, p.err, 811)) break;
                const int b = item / p.heads, h = item % p.heads;
                uint8_t* sm = smem + st * C::STAGE_BYTES;
                mbar_arrive_expect_tx(&load_full[st], (qtiles + 2 * kboxes) * C::TILE);
                for (int t = 0; t < qtiles; ++t)
                    tma_load_3d(sm + C::Q_OFF + t * C::TILE, &tm_qkv, &load_full[st], h * C::HD, 128 * t, b);
                for (int t = 0; t < kboxes; ++t) {
                    tma_load_3d(sm + C::K_OFF + t * C::TILE, &tm_qkv, &load_full[st], d + h * C::HD, 128 * t, b);
                    tma_load_3d(sm + C::V_OFF + t * C::TILE, &tm_qkv, &load_full[st], 2 * d + h * C::HD, 128 * t, b);
                }
                ++issued;
            }
            for (int k = issued - 1; k >= 0 && k >= issued - 2; --k) {
                volatile int no_abort = 0;
                wait_bar(&load_full[k & 1], static_cast<uint32_t>(k >> 1) & 1, &no_abort, p.err, 812);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            const uint32_t base = smem_u32(smem);
            const uint32_t idesc_s = umma_idesc_f16(128, lk);
            constexpr uint32_t idesc_o = umma_idesc_f16(128, C::HD) | (1u << 16);  // B (= V) MN-major
            bool ok = true;
            for (int item = blockIdx.x, k = 0; item < items && ok; item += gridDim.x, ++k) {
                const int st = k & 1;
                const uint32_t sb = base + st * C::STAGE_BYTES;
                if (!wait_bar(&load_full[st], static_cast<uint32_t>(k >> 1) & 1, abort_flag, p.err, 813)) break;
                const uint64_t kdesc = umma_desc_sw128_kmajor(sb + C::K_OFF);
                for (int g = 0; g < qtiles; ++g) {
                    if (k > 0 && !wait_bar(&tmem_free[g], (k - 1) & 1, abort_flag, p.err, 814)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t qdesc = umma_desc_sw128_kmajor(sb + C::Q_OFF + g * C::TILE);
#pragma unroll
                    for (int kk = 0; kk < C::HD / 16; ++kk)
                        umma_f16(tmem_base + 256 * g, qdesc + 2 * kk, kdesc + 2 * kk, idesc_s, kk != 0);
                    umma_commit(&s_full[g]);
                }
                for (int g = 0; g < qtiles && ok; ++g) {
                    if (!wait_bar(&p_full[g], k & 1, abort_flag, p.err, 815)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int kk = 0; kk < lk / 16; ++kk) {
                        const uint64_t vdesc = umma_desc_sw128_mnmajor(sb + C::V_OFF + kk * 2048);
                        // A = P from TMEM: keys 16 kk .. 16 kk + 15 are columns 8 kk .. 8 kk + 7
                        umma_f16_ts(tmem_base + 256 * g + C::O_COL, tmem_base + 256 * g + 8 * kk, vdesc, idesc_o,
                                    kk != 0);
                    }
                    umma_commit(&o_full[g]);
                }
                if (ok) umma_commit(&stage_free[st]);
            }
            umma_commit(drain);
            volatile int no_abort = 0;
            wait_bar(drain, 0, &no_abort, p.err, 816);
        }
    } else {
        // ---------------------------------------------------------------- softmax + output
        const int g = (warp - 2) >> 2;  // query tile of this warp group
        const int q = warp & 3;         // TMEM lane quarter
        const int row = 32 * q + lane;  // query row within the tile
        const int nchunk = (lk + 31) >> 5;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(256 * g);
        const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
        const bool group_live = g < qtiles;
        const bool warp_live = 128 * g + 32 * q < p.L;  // some row of this warp is a real query
        const int l = 128 * g + row;
        for (int item = blockIdx.x, k = 0; item < items && group_live; item += gridDim.x, ++k) {
            const int b = item / p.heads, h = item % p.heads;
            if (!wait_bar(&s_full[g], k & 1, abort_flag, p.err, 817)) break;
            tc_fence_after();
            float inv_sum = 0.0f;
            if (warp_live) {
                // One pass over S, 32 keys per TMEM load. The weights are taken
                // relative to a reference m (p = 2^((s - m) c)) that starts at the
                // first chunk's maximum and is raised only when a later chunk
                // exceeds it by more than 2^kLazyLog2 (p then stays <= 4096, well
                // inside fp16): softmax is invariant to m, and fp16's relative
                // rounding does not depend on the scale. When a lane's m is raised
                // the warp rescales the P chunks already written (rare: never for
                // keys whose scaled logits stay within 8.3 of the first chunk's).
                constexpr float kLazyLog2 = 12.0f;
                const float lazy = kLazyLog2 / p.scale_log2;  // the same bound on raw S
                float m_run = -INFINITY;
                uint64_t m2 = f2_pack(INFINITY, INFINITY);
                float s8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) s8[u] = 0.0f;
                for (int c = 0; c < nchunk; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + 32 * c, r);
                    tmem_ld_wait();
                    const bool full = 32 * c + 32 <= p.L;
                    float cm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                    if (full) {
#pragma unroll
                        for (int e = 0; e < 32; e += 2)
                            cm[(e >> 1) & 3] = fmax3(cm[(e >> 1) & 3], __uint_as_float(r[e]), __uint_as_float(r[e + 1]));
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            const float v0 = 32 * c + e < p.L ? __uint_as_float(r[e]) : -INFINITY;
                            const float v1 = 32 * c + e + 1 < p.L ? __uint_as_float(r[e + 1]) : -INFINITY;
                            cm[(e >> 1) & 3] = fmax3(cm[(e >> 1) & 3], v0, v1);
                        }
                    }
                    const float cmax = fmaxf(fmax3(cm[0], cm[1], cm[2]), cm[3]);
                    const bool raise = cmax > m_run + lazy;  // always for chunk 0
                    if (__any_sync(0xffffffffu, raise)) {
                        const float m_new = raise ? cmax : m_run;
                        if (c > 0) {
                            // P of chunks 0 .. c-1 (columns 0 .. 16 c - 1) times
                            // 2^((m_run - m_new) c), re-rounded to fp16; the row sum
                            // is rebuilt from the re-rounded weights
                            const float f = raise ? ex2_approx((m_run - m_new) * p.scale_log2) : 1.0f;
                            tmem_st_wait();
#pragma unroll
                            for (int u = 0; u < 8; ++u) s8[u] = 0.0f;
                            for (int cc = 0; cc < c; ++cc) {
                                uint32_t pw[16];
                                tmem_ld_32x32b_x16(t_row + 16 * cc, pw);
                                tmem_ld_wait();
#pragma unroll
                                for (int u = 0; u < 16; ++u) {
                                    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&pw[u]));
                                    const __half2 hh = __floats2half2_rn(v.x * f, v.y * f);
                                    s8[2 * (u & 3)] = add_f32_f16(__low2half(hh), s8[2 * (u & 3)]);
                                    s8[2 * (u & 3) + 1] = add_f32_f16(__high2half(hh), s8[2 * (u & 3) + 1]);
                                    pw[u] = *reinterpret_cast<const uint32_t*>(&hh);
                                }
                                tmem_st_32x32b_x16(t_row + 16 * cc, pw);
                            }
                        }
                        m_run = m_new;
                        const float nm = -m_run * p.scale_log2;
                        m2 = f2_pack(nm, nm);
                    }
                    // p = 2^(s c - m c) (fp32x2 fma, ex2 on the SFU), packed as fp16 pairs
                    // over the first columns of S (chunk c -> columns 16 c .. 16 c + 15,
                    // all of whose S values this thread has already read); the row sum
                    // adds the fp16-rounded weights the MMA sees
                    uint32_t pw[16];
#pragma unroll
                    for (int u = 0; u < 16; ++u) {
                        const int e = 2 * u;
                        float a0, a1;
                        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), c2, m2), a0, a1);
                        a0 = ex2_approx(a0);
                        a1 = ex2_approx(a1);
                        if (!full) {
                            if (32 * c + e >= p.L) a0 = 0.0f;
                            if (32 * c + e + 1 >= p.L) a1 = 0.0f;
                        }
                        const __half2 hh = __floats2half2_rn(a0, a1);
                        s8[2 * (u & 3)] = add_f32_f16(__low2half(hh), s8[2 * (u & 3)]);
                        s8[2 * (u & 3) + 1] = add_f32_f16(__high2half(hh), s8[2 * (u & 3) + 1]);
                        pw[u] = *reinterpret_cast<const uint32_t*>(&hh);
                    }
                    tmem_st_32x32b_x16(t_row + 16 * c, pw);
                }
                tmem_st_wait();
                inv_sum = 1.0f / (((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])));
            }
            tc_fence_before();  // P is in TMEM; O will land next to it
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[g]);
            if (!wait_bar(&o_full[g], k & 1, abort_flag, p.err, 818)) break;
            tc_fence_after();
            uint32_t r0[32], r1[32];
            if (warp_live) {
                tmem_ld_32x32b_x32(t_row + C::O_COL, r0);
                tmem_ld_32x32b_x32(t_row + C::O_COL + 32, r1);
                tmem_ld_wait();
            }
            // O is in registers: the tile's TMEM may take the next item's S now,
            // while this item's output is scaled and stored
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_free[g]);
            if (warp_live) {
                if (l < p.L) {
                    __half* orow = p.out + (static_cast<int64_t>(b) * p.L + l) * p.ldo + h * C::HD;
#pragma unroll
                    for (int gg = 0; gg < 8; ++gg) {
                        const uint32_t* rr = gg < 4 ? &r0[8 * gg] : &r1[8 * (gg - 4)];
                        uint32_t o4[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const __half2 hh = __floats2half2_rn(__uint_as_float(rr[2 * u]) * inv_sum,
                                                                 __uint_as_float(rr[2 * u + 1]) * inv_sum);
                            o4[u] = *reinterpret_cast<const uint32_t*>(&hh);
                        }
                        *reinterpret_cast<uint4*>(orow + 8 * gg) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace rpfq
