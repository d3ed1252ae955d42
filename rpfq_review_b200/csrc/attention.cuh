// Short-sequence multi-head attention on tcgen05 for the ViT / DeiT token
// counts (L <= 256 keys, head dim 64): softmax(Q K^T / sqrt(64)) V for one
// (image, head, 128-query tile) per CTA, all keys in one tile, so no online
// rescaling; two CTAs per SM overlap one's loads and MMAs with the other's
// softmax.
//
// Input: the qkv GEMM output [B, L, 3 d] (fp16; per token q heads, k heads, v
// heads, 64 columns each), read through a 3-D tensor map [B][L][3 d] so that
// rows past L are zero-filled. Output: [B, L, d] fp16 (heads concatenated),
// the proj GEMM's input. Mirrors timm's Attention.forward as used by the
// reference models (RPFQ-ViT-main/quant_models/quant_rpfq_vit.py; runtime
// restatement RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:612-614).
//
// Per CTA (6 warps), lk = L rounded up to 16:
//   warp 0    TMA: the Q tile, K and V (one or two 128-row boxes each)
//   warp 1    TMEM (256 columns) + MMA issue:
//               S = Q K^T      M=128, N=lk, K=64   -> TMEM cols [0, lk)
//               O = P V        M=128, N=64, K=lk   -> TMEM cols [0, 64)
//             (V is the B operand in its natural [key][dim] layout: MN-major)
//   warps 2-5 one query row per thread: row max over the valid keys,
//             p = 2^((s - max) c) (SFU ex2), row sum of the fp16-rounded p,
//             fp16 P into shared memory (128-B swizzled K-major A operand, over
//             the dead Q / K tiles), then O / sum to global.
// Every wait is bounded (wait_bar) and reports through the device error word.
#pragma once

#include "ptx.cuh"

namespace rpfq {

struct AttnParams {
    __half* out;       // [B * L, ldo]
    int64_t ldo;
    int32_t L;         // tokens per image (<= 256)
    int32_t heads;     // d = 64 * heads
    float scale_log2;  // log2(e) / sqrt(head_dim)
    int* err;
};

struct AttnCfg {
    static constexpr int HD = 64;
    static constexpr int LK = 256;             // largest key tile
    static constexpr int TILE = 128 * HD * 2;  // one 128-row x 64 fp16 tile = 16 KB
    // Q 16 KB | K 32 KB | V 32 KB. P stays in tensor memory: it overwrites the
    // first lk / 2 columns of S as packed fp16 pairs, the A operand of O = P V.
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = TILE;
    static constexpr int V_OFF = 3 * TILE;
    static constexpr int BAR_OFF = 5 * TILE;
    static constexpr int O_COL = 128;  // O = P V lands in TMEM columns [128, 192)
    static constexpr int SMEM_BYTES = 1024 + BAR_OFF + 128;  // two CTAs per SM (80 KB each)
    static constexpr int THREADS = 192;
    static constexpr int TMEM_COLS = 256;
    static_assert(2 * SMEM_BYTES <= 232448, "two CTAs per SM");
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

// One (image, head, 128-query tile) per CTA; 6 warps: 0 TMA, 1 TMEM + MMA,
// 2-5 softmax and output (one query row per thread).
__global__ void __launch_bounds__(192, 2)
    attn_short_sm100_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnParams p) {
    using C = AttnCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* load_bar = bars;  // Q, K, V landed
    uint64_t* s_full = bars + 1;
    uint64_t* p_full = bars + 2;  // 4 softmax warps
    uint64_t* o_full = bars + 3;
    uint64_t* drain = bars + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qtiles = (p.L + 127) >> 7;
    const int qt = blockIdx.x % qtiles;
    const int bh = blockIdx.x / qtiles;
    const int b = bh / p.heads, h = bh % p.heads;
    const int d = p.heads * C::HD;
    const int lk = (p.L + 15) & ~15;  // keys the MMAs cover (N of S, K of P V)

    if (threadIdx.x == 0) {
        mbar_init(load_bar, 1);
        mbar_init(s_full, 1);
        mbar_init(p_full, 4);
        mbar_init(o_full, 1);
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
    pdl_wait();  // the predecessor's outputs (x, residual) are complete from here on
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            const int kboxes = (lk + 127) >> 7;
            mbar_arrive_expect_tx(load_bar, (1 + 2 * kboxes) * C::TILE);
            tma_load_3d(smem + C::Q_OFF, &tm_qkv, load_bar, h * C::HD, 128 * qt, b);
            for (int t = 0; t < kboxes; ++t) {
                tma_load_3d(smem + C::K_OFF + t * C::TILE, &tm_qkv, load_bar, d + h * C::HD, 128 * t, b);
                tma_load_3d(smem + C::V_OFF + t * C::TILE, &tm_qkv, load_bar, 2 * d + h * C::HD, 128 * t, b);
            }
            volatile int no_abort = 0;
            wait_bar(load_bar, 0, &no_abort, p.err, 801);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = wait_bar(load_bar, 0, abort_flag, p.err, 802);
            if (ok) {
                tc_fence_after();
                const uint32_t base = smem_u32(smem);
                const uint32_t idesc_s = umma_idesc_f16(128, lk);
                const uint64_t kdesc = umma_desc_sw128_kmajor(base + C::K_OFF);
                const uint64_t qdesc = umma_desc_sw128_kmajor(base + C::Q_OFF);
#pragma unroll
                for (int kk = 0; kk < C::HD / 16; ++kk)
                    umma_f16(tmem_base, qdesc + 2 * kk, kdesc + 2 * kk, idesc_s, kk != 0);
                umma_commit(s_full);
                ok = wait_bar(p_full, 0, abort_flag, p.err, 803);
                if (ok) {
                    tc_fence_after();
                    constexpr uint32_t idesc_o = umma_idesc_f16(128, C::HD) | (1u << 16);  // B (= V) MN-major
                    for (int kk = 0; kk < lk / 16; ++kk) {
                        const uint64_t vdesc = umma_desc_sw128_mnmajor(base + C::V_OFF + kk * 2048);
                        // A = P from TMEM: keys 16 kk .. 16 kk + 15 are columns 8 kk .. 8 kk + 7
                        umma_f16_ts(tmem_base + C::O_COL, tmem_base + 8 * kk, vdesc, idesc_o, kk != 0);
                    }
                    umma_commit(o_full);
                }
            }
            umma_commit(drain);
            volatile int no_abort = 0;
            wait_bar(drain, 0, &no_abort, p.err, 804);
        }
    } else {
        const int q = warp & 3;         // TMEM lane quarter
        const int row = 32 * q + lane;  // query row within the tile
        const int l = 128 * qt + row;
        const bool warp_live = 128 * qt + 32 * q < p.L;  // some row of this warp is a real query
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
        const int nchunk = (lk + 31) >> 5;
        bool ok = wait_bar(s_full, 0, abort_flag, p.err, 805);
        float inv_sum = 0.0f;
        if (ok) {
            tc_fence_after();
            if (warp_live) {
                // pass 1: row max over the valid keys
                float mx = -INFINITY;
                for (int c = 0; c < nchunk; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + 32 * c, r);
                    tmem_ld_wait();
                    if (32 * c + 32 <= p.L) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) mx = fmaxf(mx, __uint_as_float(r[e]));
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (32 * c + e < p.L) mx = fmaxf(mx, __uint_as_float(r[e]));
                    }
                }
                const float nmx = -mx * p.scale_log2;
                const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2), m2 = f2_pack(nmx, nmx);
                // pass 2: p = 2^(s c - max c) (fp32x2 fma, ex2 on the SFU), packed as fp16
                // pairs over the first columns of S (chunk c -> columns 16 c .. 16 c + 15, all
                // of whose S values this thread has already read); the row sum adds the
                // fp16-rounded weights the MMA sees
                float sum = 0.0f;
                for (int c = 0; c < nchunk; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + 32 * c, r);
                    tmem_ld_wait();
                    const bool full = 32 * c + 32 <= p.L;
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
                        const float2 f = __half22float2(hh);
                        sum += f.x + f.y;
                        pw[u] = *reinterpret_cast<const uint32_t*>(&hh);
                    }
                    tmem_st_32x32b_x16(t_row + 16 * c, pw);
                }
                tmem_st_wait();
                inv_sum = 1.0f / sum;
            }
            tc_fence_before();  // P is in TMEM; O will land next to it
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            ok = wait_bar(o_full, 0, abort_flag, p.err, 806);
        }
        if (ok && warp_live) {
            tc_fence_after();
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(t_row + C::O_COL, r0);
            tmem_ld_32x32b_x32(t_row + C::O_COL + 32, r1);
            tmem_ld_wait();
            if (l < p.L) {
                __half* orow = p.out + (static_cast<int64_t>(b) * p.L + l) * p.ldo + h * C::HD;
#pragma unroll
                for (int gg = 0; gg < 8; ++gg) {
                    const uint32_t* rr = gg < 4 ? &r0[8 * gg] : &r1[8 * (gg - 4)];
                    uint32_t pw[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const __half2 hh = __floats2half2_rn(__uint_as_float(rr[2 * u]) * inv_sum,
                                                             __uint_as_float(rr[2 * u + 1]) * inv_sum);
                        pw[u] = *reinterpret_cast<const uint32_t*>(&hh);
                    }
                    *reinterpret_cast<uint4*>(orow + 8 * gg) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
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
