// LayerNorm of the fp32 residual stream into the fp16 input of the next
// packed GEMM, optionally followed by the activation quantization of that
// GEMM's complex input (ActivationQuantSTE, quant_i.py:442-455 of the
// reference), so that the quantized activations are produced in the same
// pass: one warp per row, the row held in registers.
//
//   mean = sum(x) / d;  var = sum((x - mean)^2) / d;  h = (x - mean) * rsqrt(var + eps) * w + b
//   act_bits > 0:  per Re / Im half of h: s = fl(fl(1 / max(amax, 1e-5)) * qmax),
//                  h' = fl(clamp(rint(fl(h * s)), qmin, qmax) / s)
//
// Layout: G lanes per row (a warp takes 32 / G rows), VW = 4, 2 or 1
// consecutive floats per lane and step (by row length).
#pragma once

#include "ptx.cuh"

namespace rpfq {

// Lanes per row: Swin's 96- and 192-wide rows get 8 / 16 lanes (three 16-byte
// loads per lane, a 3- / 4-level shuffle reduction; a warp takes 4 / 2 rows),
// every other row length a whole warp. The layout depends on the row length
// only, so every variant of a given length (plain, gathered, fused quantizer)
// sums in the same order and their outputs agree bit for bit.
__host__ __device__ constexpr int ln_lanes_per_row(int d) { return d == 96 ? 8 : (d == 192 ? 16 : 32); }

// Dynamic shared memory of the fused quantizer: per row of a block, both
// halves' tables of fl(q / s) for the 2^act_bits values of q and -0.
__host__ __device__ constexpr int ln_qtab_floats(int d, int warps, int act_bits) {
    return warps * (32 / ln_lanes_per_row(d)) * 2 * ((1 << act_bits) + 1);
}

struct LayerNormParams {
    const float* x;       // [x_rows, ldx] fp32
    const __half* w;
    const __half* b;
    __half* y;            // fp16 output [m, ldy], or nullptr
    float* y32;           // fp32 output [m, ldy32], or nullptr (may be x: in-place, plain row mapping only)
    int64_t ldx, ldy, ldy32;
    int64_t m;
    float eps;
    int32_t act_bits;
    const int32_t* rows;  // optional gather: output row r normalizes input row rows[r]
    int64_t x_rows;       // rows of x (gather indices outside [0, x_rows) are rejected)
    const float* add;     // optional: the row is x[r] + add[add_rows[r]] (a row-permuted residual add)
    const int32_t* add_rows;
    int64_t ld_add, add_bound;
    int32_t y32_prenorm;  // y32 receives the row before normalization (the updated residual) instead of after
    int32_t merge_side;   // > 0: 2x2 patch merging of a [images, side, side, D / 4] grid (see below)
    int* err;
};

// VW consecutive floats at p (16-, 8- or 4-byte aligned by the caller).
template <int VW>
__device__ __forceinline__ void load_row_part(const float* p, float (&v)[VW]) {
    if constexpr (VW == 4) {
        const float4 t = *reinterpret_cast<const float4*>(p);
        v[0] = t.x;
        v[1] = t.y;
        v[2] = t.z;
        v[3] = t.w;
    } else if constexpr (VW == 2) {
        const float2 t = *reinterpret_cast<const float2*>(p);
        v[0] = t.x;
        v[1] = t.y;
    } else {
        v[0] = p[0];
    }
}

// One warp per output row. Row sources:
//   plain        x[row]
//   rows         x[rows[row]] (Swin's cyclic shift + window partition)
//   merge_side   the concatenation of the four D/4-wide rows (2i, 2j), (2i+1, 2j),
//                (2i, 2j+1), (2i+1, 2j+1) of image row / (side/2)^2 of the
//                [side, side] token grid, (i, j) = that image's merged token
//                (Swin PatchMerging's strided slices and concatenation)
//   add          plus add[add_rows[row]] (Swin's window reverse + un-shift +
//                residual add of the attention branch)
// Outputs: fp16 y (normalized, optionally activation-quantized) and / or
// fp32 y32 (normalized, or with y32_prenorm the row before normalization).
// PLAIN instances (row source x[row], fp16 output only: every LayerNorm of
// the ViT / DeiT blocks) compile without the source selection.
// QUANT instances (act_bits > 0) carry the fused activation quantizer.
template <int D, bool PLAIN, bool QUANT>
__global__ void __launch_bounds__(256) layernorm_f32_f16_kernel(const LayerNormParams p) {
    static_assert(D % 32 == 0, "row length must be a multiple of 32");
    constexpr int G = ln_lanes_per_row(D);
    constexpr int R = 32 / G;  // rows per warp
    // VW consecutive floats per lane and step: element e of step j of lane l of
    // a row group sits at column G VW j + VW l + e (coalesced, 16-/8-/4-byte loads)
    constexpr int VW = G < 32 ? 4 : (D % 128 == 0 ? 4 : (D % 64 == 0 ? 2 : 1));
    constexpr int J = D / (G * VW);
    static_assert(J * G * VW == D, "row layout");
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rg = lane / G;  // this lane's row within the warp
    const int sl = lane % G;  // this lane within its row
    // Rows are taken last to first: the GEMM that wrote x finished with its
    // highest row blocks, which are the ones still in L2, and the GEMM that
    // reads y starts with the lowest rows, the ones written last here.
    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5)) * R + rg;
    const int64_t row = p.m - 1 - slot;
    // per row: the activation quantizer's fl(q / s) for both halves, see below
    // (dynamic shared memory, present only when act_bits > 0)
    extern __shared__ float ln_qtab[];
    const int qstride = (1 << p.act_bits) + 1;
    float* qtab_re = ln_qtab + (static_cast<int>(threadIdx.x >> 5) * R + rg) * 2 * qstride;
    float* qtab_im = qtab_re + qstride;
    pdl_wait();
    pdl_launch_dependents();
    // a row group past the last row stays in the warp's shuffles without touching memory
    bool live = slot < p.m;
    if (!__any_sync(0xffffffffu, live)) return;
    // source row of each quarter of the output row (all four equal unless merging)
    int64_t src[4] = {row, row, row, row};
    const float* ar = nullptr;
    if (!PLAIN && live) {
        if (p.merge_side > 0) {
            const int64_t half = p.merge_side >> 1;
            const int64_t img = row / (half * half), t = row - img * half * half;
            const int64_t i = t / half, j = t - i * half;
            const int64_t base = img * p.merge_side * p.merge_side + 2 * i * p.merge_side + 2 * j;
            src[0] = base;
            src[1] = base + p.merge_side;
            src[2] = base + 1;
            src[3] = base + p.merge_side + 1;
        } else {
            int64_t s0 = row;
            if (p.rows != nullptr) {
                s0 = p.rows[row];
                if (s0 < 0 || s0 >= p.x_rows) {  // bad gather index: report, touch nothing
                    if (sl == 0) atomicCAS(p.err, 0, 901);
                    live = false;
                    s0 = 0;
                }
            }
            src[0] = src[1] = src[2] = src[3] = s0;
        }
        if (live && p.add != nullptr) {
            const int64_t a = p.add_rows != nullptr ? p.add_rows[row] : row;
            if (a < 0 || a >= p.add_bound) {
                if (sl == 0) atomicCAS(p.err, 0, 902);
                live = false;
            } else {
                ar = p.add + a * p.ld_add;
            }
        }
    }
    // every load of the row is issued before the first use (x, then the add
    // rows), with no branch between them
    float v[J][VW];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int col = G * VW * j + VW * sl;
        const int q = col / (D / 4);  // quarter (VW divides D / 4 whenever merging is allowed)
        const int64_t sq = PLAIN ? row : (q == 0 ? src[0] : (q == 1 ? src[1] : (q == 2 ? src[2] : src[3])));
        const float* xr = p.x + sq * p.ldx + (!PLAIN && p.merge_side > 0 ? col - q * (D / 4) : col);
        if (live) {
            load_row_part<VW>(xr, v[j]);
        } else {
#pragma unroll
            for (int e = 0; e < VW; ++e) v[j][e] = 0.0f;
        }
    }
    if (!PLAIN && ar != nullptr) {
        float u[J][VW];
#pragma unroll
        for (int j = 0; j < J; ++j) load_row_part<VW>(ar + G * VW * j + VW * sl, u[j]);
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int e = 0; e < VW; ++e) v[j][e] += u[j][e];
    }
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        if constexpr (VW == 4)
            sum += (v[j][0] + v[j][1]) + (v[j][2] + v[j][3]);
        else if constexpr (VW == 2)
            sum += v[j][0] + v[j][1];
        else
            sum += v[j][0];
    }
    if (!PLAIN && live && p.y32 != nullptr && p.y32_prenorm) {
        // the updated residual row (in place when y32 == x: these lanes have read their whole row)
        float* zr = p.y32 + row * p.ldy32;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int col = G * VW * j + VW * sl;
            if constexpr (VW == 4)
                *reinterpret_cast<float4*>(zr + col) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
            else if constexpr (VW == 2)
                *reinterpret_cast<float2*>(zr + col) = make_float2(v[j][0], v[j][1]);
            else
                zr[col] = v[j][0];
        }
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(D);
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int e = 0; e < VW; ++e) {
            const float dlt = v[j][e] - mean;
            sq += dlt * dlt;
        }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq / static_cast<float>(D) + p.eps);
    float amax_re = 0.0f, amax_im = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int col = G * VW * j + VW * sl;
        float wf[VW], bf[VW];
        if constexpr (VW == 4) {
            const uint2 wv = *reinterpret_cast<const uint2*>(p.w + col);
            const uint2 bv = *reinterpret_cast<const uint2*>(p.b + col);
            const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
            const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
            const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&bv.x));
            const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&bv.y));
            wf[0] = w01.x; wf[1] = w01.y; wf[2] = w23.x; wf[3] = w23.y;
            bf[0] = b01.x; bf[1] = b01.y; bf[2] = b23.x; bf[3] = b23.y;
        } else {
#pragma unroll
            for (int e = 0; e < VW; ++e) {
                wf[e] = __half2float(p.w[col + e]);
                bf[e] = __half2float(p.b[col + e]);
            }
        }
#pragma unroll
        for (int e = 0; e < VW; ++e) {
            v[j][e] = (v[j][e] - mean) * rstd * wf[e] + bf[e];
            const float a = fabsf(v[j][e]);
            if (col + e < D / 2)
                amax_re = fmaxf(amax_re, a);
            else
                amax_im = fmaxf(amax_im, a);
        }
    }
    if (!PLAIN && live && p.y32 != nullptr && !p.y32_prenorm) {
        float* zr = p.y32 + row * p.ldy32;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int col = G * VW * j + VW * sl;
            if constexpr (VW == 4)
                *reinterpret_cast<float4*>(zr + col) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
            else if constexpr (VW == 2)
                *reinterpret_cast<float2*>(zr + col) = make_float2(v[j][0], v[j][1]);
            else
                zr[col] = v[j][0];
        }
    }
    if (p.y == nullptr) return;
    float s_re = 0.0f, s_im = 0.0f, qmax = 0.0f, qmin = 0.0f;
    if (QUANT) {
#pragma unroll
        for (int o = G / 2; o > 0; o >>= 1) {
            amax_re = fmaxf(amax_re, __shfl_xor_sync(0xffffffffu, amax_re, o));
            amax_im = fmaxf(amax_im, __shfl_xor_sync(0xffffffffu, amax_im, o));
        }
        qmax = static_cast<float>((1 << (p.act_bits - 1)) - 1);
        qmin = -static_cast<float>(1 << (p.act_bits - 1));
        // The quantizer sees the fp16 GEMM input, as in the unfused path.
        s_re = __fmul_rn(__frcp_rn(fmaxf(__half2float(__float2half_rn(amax_re)), 1e-5f)), qmax);
        s_im = __fmul_rn(__frcp_rn(fmaxf(__half2float(__float2half_rn(amax_im)), 1e-5f)), qmax);
        // q takes the 2^act_bits integers in [qmin, qmax] and -0 (rint of a small
        // negative h): the row's lanes divide each once (IEEE, as per element) into
        // its table, slot 2^act_bits holding fl(-0 / s)
        const int nq = 1 << p.act_bits;
        for (int t = sl; t < nq; t += G) {
            qtab_re[t] = __fdiv_rn(qmin + static_cast<float>(t), s_re);
            qtab_im[t] = __fdiv_rn(qmin + static_cast<float>(t), s_im);
        }
        if (sl == 0) {
            qtab_re[nq] = __fdiv_rn(-0.0f, s_re);
            qtab_im[nq] = __fdiv_rn(-0.0f, s_im);
        }
        __syncwarp();
    }
    if (!live) return;
    __half* yr = p.y + row * p.ldy;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int col = G * VW * j + VW * sl;
        float o[VW];
#pragma unroll
        for (int e = 0; e < VW; ++e) {
            o[e] = v[j][e];
            if (QUANT) {
                const float s = (col + e < D / 2) ? s_re : s_im;
                const float h = __half2float(__float2half_rn(o[e]));
                const float q = fminf(fmaxf(rintf(__fmul_rn(h, s)), qmin), qmax);
                const float* tab = (col + e < D / 2) ? qtab_re : qtab_im;
                o[e] = tab[__float_as_uint(q) == 0x80000000u ? (1 << p.act_bits) : static_cast<int>(q - qmin)];
            }
        }
        if constexpr (VW == 4) {
            __half2 h01 = __floats2half2_rn(o[0], o[1]);
            __half2 h23 = __floats2half2_rn(o[2], o[3]);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&h01);
            pk.y = *reinterpret_cast<uint32_t*>(&h23);
            *reinterpret_cast<uint2*>(yr + col) = pk;
        } else if constexpr (VW == 2) {
            *reinterpret_cast<__half2*>(yr + col) = __floats2half2_rn(o[0], o[1]);
        } else {
            yr[col] = __float2half_rn(o[0]);
        }
    }
}

}  // namespace rpfq
