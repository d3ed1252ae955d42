// K3: fused decode + tcgen05 GEMM for small M (the weight-bound regime).
//
// The packed phase codes are the weight stream: TMA stages one tile of codes
// (4 planes x RB complex rows x 64 complex columns = 2 bits per real weight),
// decode warps unpack it in shared memory into the two fp16 B-operand tiles
//   B_re = [rr; ri]  (x_re -> y_re, y_im)      B_im = [ir; ii]  (x_im -> y_re, y_im)
// written directly in the UMMA 128-B-swizzled K-major layout, and one thread
// issues tcgen05.mma against the x tiles (x_re and x_im halves of the same 64
// complex columns, TMA-loaded from a [M][2][k_c] view), accumulating
//   acc[m][0:RB)   = y_re rows r0..r0+RB,   acc[m][RB:2RB) = y_im rows r0..r0+RB
// in TMEM. The decoded coefficients are bit-identical to K1's (same fp32 sum
// order and rounding), so this path computes the same products as the
// prepacked one without ever writing the dense matrix to HBM.
//
// Work item = one block of RB complex output rows over all of K; persistent
// CTAs loop over items. M <= 256 (two 128-row sub-tiles).
// Split-K (p.splits = S > 1, for layers whose row blocks alone leave most SMs
// idle): a cluster of S CTAs per item, CTA s takes k-blocks
// [s num_k / S, (s + 1) num_k / S) and writes its raw fp32 accumulator to the
// workspace; after a cluster barrier each CTA reduces 1/S of the item's
// outputs over the S partials in the fixed order 0..S-1 (deterministic) and
// applies bias / GELU / residual. 10 warps:
//   warp 0    TMA producer (x_re, x_im per sub-tile + the code planes per stage)
//   warp 1    TMEM owner + MMA issuer
//   warps 2-9 decode in two groups that take alternate stages (one 16-byte
//             granule of one row per thread and stage), then the epilogue of
//             the item (bias, GELU, residual, fp16/fp32 store)
#pragma once

#include "gemm.cuh"
#include "prepack.cuh"

namespace rpfq {

struct DecodeGemmParams {
    const __half* gamma_re[8];  // u_s0.., w_s0.. (stages each), [n_cp, k_cp/256]
    const __half* gamma_im[8];
    int32_t stages;
    int32_t n_c, k_c, n_cp, k_cp;
    int32_t rows_per_item;  // RB (16, 32 or 64)
    const void* bias;       // [2 n_c] fp16 (fp32 with bias_f32) or nullptr
    int32_t bias_f32;
    const void* residual;   // [m, 2 n_c] (y's dtype) or nullptr
    int64_t ldr;
    void* y;                // [m, 2 n_c]
    int64_t ldy;
    int64_t m;
    int32_t activation;
    int32_t out_f32;
    int32_t splits;         // K splits per item (cluster size), 1 = none
    float* ws;              // split-K partials [items * splits][nsub * 128][2 RB] fp32
    int* err;
};

struct DecodeCodeMaps {
    CUtensorMap plane[8];  // u_s0.., w_s0..: codes [n_cp rows][k_cp/4 bytes], box {16 B, RB rows}
};

template <int RB>
struct DecodeCfg {
    static_assert(RB == 16 || RB == 32 || RB == 64, "row block");
    static constexpr int NT = 2 * RB;           // accumulator columns per sub-tile
    static constexpr int KB = 64;               // complex columns per stage
    static constexpr int A_BYTES = 128 * KB * 2;  // one x half-tile of a 128-row sub-tile
    static constexpr int B_BYTES = NT * KB * 2;   // one decoded tile (B_re or B_im)
    static constexpr int CODE_BYTES = RB * 16;    // one plane's code tile
    // stage: [A_re0, A_im0, A_re1, A_im1][B_re, B_im][codes x 8 planes]
    static constexpr int STAGE_BYTES =
        4 * A_BYTES + 2 * B_BYTES + ((8 * CODE_BYTES + 1023) / 1024) * 1024;
    static constexpr int STAGES =
        (230 * 1024 - 1280) / STAGE_BYTES >= 4 ? 4 : (230 * 1024 - 1280) / STAGE_BYTES;
    static constexpr int TMEM_COLS = NT * 2 <= 32 ? 32 : NT * 2;  // two sub-tiles
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
    static constexpr int THREADS = 320;
    static_assert(STAGES >= 2, "at least two stages");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

// Split-K reduction of item `item` by split `split` of S: float4 granules
// [split E / S, (split + 1) E / S) of the item's m x 2 RB outputs (E = m RB / 2)
// are summed over the S partials in the order 0..S-1, then bias, GELU and
// residual are applied and the four outputs of each granule stored (256
// threads, tid 0..255). Accumulator column j < RB is output column r0 + j
// (y_re), j >= RB is n_c + r0 + j - RB (y_im).
template <int RB>
__device__ __forceinline__ void decode_splitk_reduce(const DecodeGemmParams& p, int item, int split, int nsub, int tid) {
    constexpr int G = 2 * RB / 4;  // granules per row
    const int S = p.splits;
    const int64_t E = p.m * G;
    const int r0 = item * RB;
    const int valid = min(RB, p.n_c - r0);
    const float4* base = reinterpret_cast<const float4*>(p.ws) + static_cast<size_t>(item) * S * nsub * 128 * G;
    const size_t part_stride = static_cast<size_t>(nsub) * 128 * G;  // float4 per partial
    for (int64_t e = split * E / S + tid; e < (split + 1) * E / S; e += 256) {
        const int64_t row = e / G;
        const int jg = static_cast<int>(e - row * G);
        const int j = 4 * jg;                       // accumulator column
        const int half = j >= RB ? 1 : 0;
        const int jc = j - half * RB;               // column within the half
        if (jc >= valid) continue;
        const int64_t col = static_cast<int64_t>(half) * p.n_c + r0 + jc;
        float4 a = __ldcg(base + static_cast<size_t>(row) * G + jg);
        for (int s = 1; s < S; ++s) {
            const float4 b = __ldcg(base + s * part_stride + static_cast<size_t>(row) * G + jg);
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        float v[4] = {a.x, a.y, a.z, a.w};
        if (p.bias != nullptr) {
            if (p.bias_f32) {
                const float4 bb = *reinterpret_cast<const float4*>(static_cast<const float*>(p.bias) + col);
                v[0] += bb.x; v[1] += bb.y; v[2] += bb.z; v[3] += bb.w;
            } else {
                const uint2 h = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p.bias) + col);
                const float2 b0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                const float2 b1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                v[0] += b0.x; v[1] += b0.y; v[2] += b1.x; v[3] += b1.y;
            }
        }
        if (p.activation == kActGelu) {
            gelu_erf_pair(v[0], v[1]);
            gelu_erf_pair(v[2], v[3]);
        }
        if (p.out_f32) {
            float* y = static_cast<float*>(p.y) + row * p.ldy + col;
            if (p.residual != nullptr) {
                const float4 r = *reinterpret_cast<const float4*>(static_cast<const float*>(p.residual) + row * p.ldr + col);
                v[0] += r.x; v[1] += r.y; v[2] += r.z; v[3] += r.w;
            }
            *reinterpret_cast<float4*>(y) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
            __half* y = static_cast<__half*>(p.y) + row * p.ldy + col;
            if (p.residual != nullptr) {
                const uint2 h = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p.residual) + row * p.ldr + col);
                const float2 r0f = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                const float2 r1f = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                v[0] += r0f.x; v[1] += r0f.y; v[2] += r1f.x; v[3] += r1f.y;
            }
            __half2 h0 = __floats2half2_rn(v[0], v[1]);
            __half2 h1 = __floats2half2_rn(v[2], v[3]);
            uint2 o;
            o.x = *reinterpret_cast<uint32_t*>(&h0);
            o.y = *reinterpret_cast<uint32_t*>(&h1);
            *reinterpret_cast<uint2*>(y) = o;
        }
    }
}

template <int RB>
__global__ void __launch_bounds__(320, 1)
    decode_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ DecodeCodeMaps cm,
                             const DecodeGemmParams p) {
    using C = DecodeCfg<RB>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t* full_bar = bars;                     // [STAGES] TMA landed
    uint64_t* dec_bar = bars + C::STAGES;          // [STAGES] decode written
    uint64_t* empty_bar = bars + 2 * C::STAGES;    // [STAGES] MMAs done reading
    uint64_t* tfull_bar = bars + 3 * C::STAGES;    // accumulators complete
    uint64_t* tempty_bar = tfull_bar + 1;          // accumulators read out
    uint64_t* drain_bar = tfull_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull_bar + 3);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nsub = p.m > 128 ? 2 : 1;
    const int num_items = (p.n_c + RB - 1) / RB;
    const int num_k_all = (p.k_c + C::KB - 1) / C::KB;
    const int planes = 2 * p.stages;
    // split-K: one item per cluster, this CTA's k-blocks [kb_lo, kb_lo + num_k)
    const int S = p.splits;
    const int split = S > 1 ? static_cast<int>(blockIdx.x) % S : 0;
    const int first_item = S > 1 ? static_cast<int>(blockIdx.x) / S : static_cast<int>(blockIdx.x);
    const int item_step = S > 1 ? num_items : static_cast<int>(gridDim.x);
    const int kb_lo = split * num_k_all / S;
    const int num_k = (split + 1) * num_k_all / S - kb_lo;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&dec_bar[s], 4);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(tfull_bar, 1);
        mbar_init(tempty_bar, 8);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tm_x);
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

    auto stage_ptr = [&](int s) { return smem + s * C::STAGE_BYTES; };

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------ producer (split-K: see the end of the branch)
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            const uint32_t bytes = static_cast<uint32_t>(2 * nsub * C::A_BYTES + planes * C::CODE_BYTES);
            for (int item = first_item; item < num_items && ok; item += item_step) {
                const int r0 = item * RB;
                for (int kb = kb_lo; kb < kb_lo + num_k; ++kb) {
                    if (!wait_bar(&empty_bar[stage], phase ^ 1, abort_flag, p.err, 501)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = stage_ptr(stage);
                    mbar_arrive_expect_tx(&full_bar[stage], bytes);
                    for (int sub = 0; sub < nsub; ++sub) {
                        tma_load_3d(st + (2 * sub) * C::A_BYTES, &tm_x, &full_bar[stage], kb * C::KB, 0, sub * 128);
                        tma_load_3d(st + (2 * sub + 1) * C::A_BYTES, &tm_x, &full_bar[stage], kb * C::KB, 1,
                                    sub * 128);
                    }
                    uint8_t* codes = st + 4 * C::A_BYTES + 2 * C::B_BYTES;
                    for (int pl = 0; pl < planes; ++pl)
                        tma_load_2d(codes + pl * C::CODE_BYTES, &cm.plane[pl], &full_bar[stage], kb * (C::KB / 4), r0);
                    ++issued;
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            const int pending = issued < C::STAGES ? issued : C::STAGES;
            for (int i = 1; i <= pending; ++i) {
                int s = stage - i;
                uint32_t ph = phase;
                if (s < 0) {
                    s += C::STAGES;
                    ph ^= 1;
                }
                volatile int no_abort = 0;
                wait_bar(&full_bar[s], ph, &no_abort, p.err, 502);
            }
        }
        if (S > 1) {
            __syncwarp();
            cluster_sync();  // the split-K exchange barrier
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = umma_idesc_f16(128, C::NT);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t item_phase = 0;
            bool ok = true;
            for (int item = first_item; item < num_items && ok; item += item_step) {
                if (!wait_bar(tempty_bar, item_phase ^ 1, abort_flag, p.err, 601)) break;
                tc_fence_after();
                for (int kb = kb_lo; kb < kb_lo + num_k; ++kb) {
                    // the x tiles come from TMA (full), the weight tiles from the decode warps (dec)
                    if (!wait_bar(&full_bar[stage], phase, abort_flag, p.err, 604) ||
                        !wait_bar(&dec_bar[stage], phase, abort_flag, p.err, 602)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t base = smem_u32(stage_ptr(stage));
                    const uint64_t b_re = umma_desc_sw128_kmajor(base + 4 * C::A_BYTES);
                    const uint64_t b_im = umma_desc_sw128_kmajor(base + 4 * C::A_BYTES + C::B_BYTES);
                    for (int sub = 0; sub < nsub; ++sub) {
                        const uint32_t d = tmem_base + static_cast<uint32_t>(sub * C::NT);
                        const uint64_t a_re = umma_desc_sw128_kmajor(base + (2 * sub) * C::A_BYTES);
                        const uint64_t a_im = umma_desc_sw128_kmajor(base + (2 * sub + 1) * C::A_BYTES);
#pragma unroll
                        for (int kk = 0; kk < C::KB / 16; ++kk)
                            umma_f16(d, a_re + 2 * kk, b_re + 2 * kk, idesc, ((kb - kb_lo) | kk) != 0);
#pragma unroll
                        for (int kk = 0; kk < C::KB / 16; ++kk) umma_f16(d, a_im + 2 * kk, b_im + 2 * kk, idesc, 1);
                    }
                    umma_commit(&empty_bar[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(tfull_bar);
                item_phase ^= 1;
            }
            umma_commit(drain_bar);
            volatile int no_abort = 0;
            wait_bar(drain_bar, 0, &no_abort, p.err, 603);
        }
        if (S > 1) {
            __syncwarp();
            cluster_sync();  // the split-K exchange barrier, which every thread of the cluster joins
        }
    } else {
        // -------------------------------------------------------------- decode + epilogue
        // Two groups of four warps take alternate ring stages (more warps in
        // flight per scheduler); in the epilogue group 0 writes the y_re
        // block of the item and group 1 the y_im block.
        constexpr int ROWS_PER_THREAD = RB * 8 / 128;  // decode items per thread and stage
        const int group = (warp - 2) >> 2;
        const int dt = (threadIdx.x - 64) & 127;  // thread within the group
        const int q = warp & 3;                   // TMEM lane quarter
        int n = 0;                                // ring iteration (same sequence as producer and MMA)
        uint32_t item_phase = 0;
        bool ok = true;
        // 1/gamma of this thread's rows for the current 256-column block, all
        // planes, as fp32 bit patterns; reloaded when the block changes
        uint32_t inv_r[ROWS_PER_THREAD][8], inv_i[ROWS_PER_THREAD][8];
        for (int item = first_item; item < num_items && ok; item += item_step) {
            const int r0 = item * RB;
            int cached_blk = -1;
            for (int kb = kb_lo; kb < kb_lo + num_k; ++kb) {
                const int it = n++;
                if ((it & 1) != group) continue;
                const int stage = it % C::STAGES;
                const uint32_t phase = static_cast<uint32_t>(it / C::STAGES) & 1u;
                const int gblk = (kb * C::KB) >> 8;  // 256-column gamma block
                if (gblk != cached_blk) {
                    cached_blk = gblk;
                    __half gr[ROWS_PER_THREAD][8], gi[ROWS_PER_THREAD][8];
#pragma unroll
                    for (int t = 0; t < ROWS_PER_THREAD; ++t) {
                        const int row = r0 + ((dt + 128 * t) >> 3);
                        const int gidx = row * (p.k_cp >> 8) + gblk;
#pragma unroll
                        for (int pl = 0; pl < 8; ++pl) {
                            gr[t][pl] = pl < planes ? p.gamma_re[pl][gidx] : __float2half(1.0f);
                            gi[t][pl] = pl < planes ? p.gamma_im[pl][gidx] : __float2half(1.0f);
                        }
                    }
#pragma unroll
                    for (int t = 0; t < ROWS_PER_THREAD; ++t)
#pragma unroll
                        for (int pl = 0; pl < 8; ++pl) {
                            inv_r[t][pl] = __float_as_uint(__frcp_rn(__half2float(gr[t][pl])));
                            inv_i[t][pl] = __float_as_uint(__frcp_rn(__half2float(gi[t][pl])));
                        }
                }
                if (!wait_bar(&full_bar[stage], phase, abort_flag, p.err, 701)) {
                    ok = false;
                    break;
                }
                uint8_t* st = stage_ptr(stage);
                uint8_t* b_re = st + 4 * C::A_BYTES;
                uint8_t* b_im = b_re + C::B_BYTES;
                const uint8_t* codes = b_im + C::B_BYTES;
                // items of this stage: RB rows x 8 granules of 8 complex columns
#pragma unroll
                for (int t = 0; t < ROWS_PER_THREAD; ++t) {
                    const int itm = dt + 128 * t;
                    const int i = itm >> 3;  // row within the block
                    const int g = itm & 7;   // granule: complex columns 8g..8g+7 of the stage
                    // Per element, as fp32x2 pairs: p = (rr, ri), q = (ii, ir).
                    // Code c of a plane: re = c==0 ? -a : c==1 ? a : +0, im = c==2 ? -b : c==3 ? b : +0,
                    // built from the code bits: bit 0 clear -> negative, bit 1 -> imaginary axis.
                    uint64_t acc_p[8], acc_q[8];
                    const uint8_t* crow = codes + i * 16 + 2 * g;
                    {
                        const uint32_t two = *reinterpret_cast<const uint16_t*>(crow);
                        const uint32_t nb = ~two;
                        const uint32_t a = inv_r[t][0], b = inv_i[t][0];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const uint32_t sgn = (nb << (31 - 2 * e)) & 0x80000000u;
                            const uint32_t m1 = static_cast<uint32_t>(static_cast<int32_t>(two << (30 - 2 * e)) >> 31);
                            const uint32_t re = (a | sgn) & ~m1;
                            const uint32_t im = (b | sgn) & m1;
                            // first U plane: rr = re, ri = im, ii = re, ir = -im
                            acc_p[e] = (static_cast<uint64_t>(im) << 32) | re;
                            acc_q[e] = (static_cast<uint64_t>(im ^ 0x80000000u) << 32) | re;
                        }
                    }
#pragma unroll
                    for (int pl = 1; pl < 8; ++pl) {
                        if (pl >= planes) break;
                        const uint32_t two = *reinterpret_cast<const uint16_t*>(crow + pl * C::CODE_BYTES);
                        const uint32_t nb = ~two;
                        const uint32_t a = inv_r[t][pl], b = inv_i[t][pl];
                        // U planes: (ii, ir) += (re, -im); W planes: (ii, ir) += (-re, im).
                        // x*(+-1) is exact, so each fma rounds exactly like the scalar add / sub.
                        const uint64_t sgnq = pl < p.stages ? 0xBF8000003F800000ull : 0x3F800000BF800000ull;
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const uint32_t sgn = (nb << (31 - 2 * e)) & 0x80000000u;
                            const uint32_t m1 = static_cast<uint32_t>(static_cast<int32_t>(two << (30 - 2 * e)) >> 31);
                            const uint32_t re = (a | sgn) & ~m1;
                            const uint32_t im = (b | sgn) & m1;
                            const uint64_t v = (static_cast<uint64_t>(im) << 32) | re;
                            acc_p[e] = f2_add(acc_p[e], v);
                            acc_q[e] = f2_fma(v, sgnq, acc_q[e]);
                        }
                    }
                    float rr[8], ri[8], ii[8], ir[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        f2_unpack(acc_p[e], rr[e], ri[e]);
                        f2_unpack(acc_q[e], ii[e], ir[e]);
                    }
                    auto pack8 = [](const float (&v)[8]) {
                        uint4 o;
                        __half2 h0 = __floats2half2_rn(v[0], v[1]);
                        __half2 h1 = __floats2half2_rn(v[2], v[3]);
                        __half2 h2 = __floats2half2_rn(v[4], v[5]);
                        __half2 h3 = __floats2half2_rn(v[6], v[7]);
                        o.x = *reinterpret_cast<uint32_t*>(&h0);
                        o.y = *reinterpret_cast<uint32_t*>(&h1);
                        o.z = *reinterpret_cast<uint32_t*>(&h2);
                        o.w = *reinterpret_cast<uint32_t*>(&h3);
                        return o;
                    };
                    // rows i (y_re) and RB + i (y_im) of both tiles, 128-B swizzle
                    const int n0 = i, n1 = RB + i;
                    *reinterpret_cast<uint4*>(b_re + n0 * 128 + ((g ^ (n0 & 7)) << 4)) = pack8(rr);
                    *reinterpret_cast<uint4*>(b_re + n1 * 128 + ((g ^ (n1 & 7)) << 4)) = pack8(ri);
                    *reinterpret_cast<uint4*>(b_im + n0 * 128 + ((g ^ (n0 & 7)) << 4)) = pack8(ir);
                    *reinterpret_cast<uint4*>(b_im + n1 * 128 + ((g ^ (n1 & 7)) << 4)) = pack8(ii);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&dec_bar[stage]);
            }
            if (!ok) break;
            // ---- epilogue of the item: this warp's 32 rows of each sub-tile,
            //      columns [group*RB, group*RB + RB) of the accumulator
            if (!wait_bar(tfull_bar, item_phase, abort_flag, p.err, 702)) break;
            tc_fence_after();
            const int valid = min(RB, p.n_c - r0);
            const int64_t col0 = static_cast<int64_t>(group) * p.n_c + r0;
            if (S > 1) {
                // split-K partial: this warp's 32 rows x RB columns of each sub-tile, raw
                float* part = p.ws + (static_cast<size_t>(blockIdx.x) * nsub * 128) * (2 * RB) + group * RB;
                for (int sub = 0; sub < nsub; ++sub) {
                    uint32_t r[RB];
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16) +
                                           static_cast<uint32_t>(sub * C::NT + group * RB);
                    if constexpr (RB == 16) {
                        tmem_ld_32x32b_x16(taddr, r);
                    } else {
#pragma unroll
                        for (int h = 0; h < RB / 32; ++h)
                            tmem_ld_32x32b_x32(taddr + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * h]));
                    }
                    tmem_ld_wait();
                    float4* dst = reinterpret_cast<float4*>(part + static_cast<size_t>(sub * 128 + 32 * q + lane) * (2 * RB));
#pragma unroll
                    for (int j = 0; j < RB / 4; ++j)
                        __stcg(dst + j, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                    __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty_bar);
                item_phase ^= 1;
                continue;
            }
            for (int sub = 0; sub < nsub; ++sub) {
                const int64_t row = static_cast<int64_t>(sub) * 128 + 32 * q + lane;
                uint32_t r[RB];
                const uint32_t taddr =
                    tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(sub * C::NT + group * RB);
                if constexpr (RB == 16) {
                    tmem_ld_32x32b_x16(taddr, r);
                } else {
#pragma unroll
                    for (int h = 0; h < RB / 32; ++h)
                        tmem_ld_32x32b_x32(taddr + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * h]));
                }
                tmem_ld_wait();
                if (row >= p.m) continue;
#pragma unroll
                for (int j0 = 0; j0 < RB; j0 += 8) {
                    if (j0 >= valid) break;
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[j0 + e]);
                    if (p.bias != nullptr && p.bias_f32) {
                        const float* bf = static_cast<const float*>(p.bias) + col0 + j0;
                        const float4 b0 = *reinterpret_cast<const float4*>(bf);
                        const float4 b1 = *reinterpret_cast<const float4*>(bf + 4);
                        v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
                        v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
                    } else if (p.bias != nullptr) {
                        const uint4 bv = *reinterpret_cast<const uint4*>(static_cast<const __half*>(p.bias) + col0 + j0);
                        const __half2* bh = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(bh[e]);
                            v[2 * e] += f.x;
                            v[2 * e + 1] += f.y;
                        }
                    }
                    if (p.activation == kActGelu) {
#pragma unroll
                        for (int e = 0; e < 8; e += 2) gelu_erf_pair(v[e], v[e + 1]);
                    }
                    if (p.out_f32) {
                        float* yrow = static_cast<float*>(p.y) + row * p.ldy + col0 + j0;
                        if (p.residual != nullptr) {
                            const float* rrow = static_cast<const float*>(p.residual) + row * p.ldr + col0 + j0;
                            const float4 a = *reinterpret_cast<const float4*>(rrow);
                            const float4 b = *reinterpret_cast<const float4*>(rrow + 4);
                            v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
                            v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
                        }
                        *reinterpret_cast<float4*>(yrow) = make_float4(v[0], v[1], v[2], v[3]);
                        *reinterpret_cast<float4*>(yrow + 4) = make_float4(v[4], v[5], v[6], v[7]);
                    } else {
                        __half* yrow = static_cast<__half*>(p.y) + row * p.ldy + col0 + j0;
                        if (p.residual != nullptr) {
                            const __half* rrow = static_cast<const __half*>(p.residual) + row * p.ldr + col0 + j0;
                            const uint4 rv = *reinterpret_cast<const uint4*>(rrow);
                            const __half2* rh = reinterpret_cast<const __half2*>(&rv);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = __half22float2(rh[e]);
                                v[2 * e] += f.x;
                                v[2 * e + 1] += f.y;
                            }
                        }
                        uint4 o;
                        __half2 h0 = __floats2half2_rn(v[0], v[1]);
                        __half2 h1 = __floats2half2_rn(v[2], v[3]);
                        __half2 h2 = __floats2half2_rn(v[4], v[5]);
                        __half2 h3 = __floats2half2_rn(v[6], v[7]);
                        o.x = *reinterpret_cast<uint32_t*>(&h0);
                        o.y = *reinterpret_cast<uint32_t*>(&h1);
                        o.z = *reinterpret_cast<uint32_t*>(&h2);
                        o.w = *reinterpret_cast<uint32_t*>(&h3);
                        *reinterpret_cast<uint4*>(yrow) = o;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar);
            item_phase ^= 1;
        }
        if (S > 1) {
            __syncwarp();
            cluster_sync();  // every split's partial is written (release) and visible (acquire)
            if (first_item < num_items) decode_splitk_reduce<RB>(p, first_item, split, nsub, threadIdx.x - 64);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace rpfq
