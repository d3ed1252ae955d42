// K1: decode the packed phase planes into the dense fp16 coefficient matrix
//
//   W[2 n_c, 2 k_c] = [[rr, ir], [ri, ii]]
//
// rr: x_re -> y_re, ir: x_im -> y_re, ri: x_re -> y_im, ii: x_im -> y_im.
// Per element the stage values are decoded with a float32 reciprocal of the
// fp16 gamma (phase_linear.cpp:82-83 of the reference Android runtime) and
// summed left to right in float32 in the order of buildFusedWideLinearCache
// (phase_linear_cache.cpp:119-126): U stages first, then W stages. The sum is
// rounded to fp16 either to nearest even (IEEE, default) or with ties away
// from zero (the reference's floatToHalfBits, phase_linear_cache.cpp:58-82),
// so both are reproducible bit for bit.
//
// 2-bit codes use the reference codebook 0:-1, 1:+1, 2:-i, 3:+i
// (export_rpfq_vit_to_mlx.py:598-603). 3- and 4-bit codes are this library's
// extension: code c is the phase exp(2 pi i c / 2^b), value
// (cos / gamma_real, sin / gamma_imag), packed LSB-first as a bit stream.
//
// One thread per (output complex row, 4 consecutive complex columns): reads
// one code byte per plane (b = 2) and writes 4 x 8 B into the four quadrants.
// Runs once per layer at load time.
#pragma once

#include "ptx.cuh"

namespace rpfq {

enum : int { kRoundNearestEven = 0, kRoundTiesAway = 1 };

struct PrepackPlane {
    const uint8_t* codes;
    const __half* gamma_re;
    const __half* gamma_im;
};

struct PrepackParams {
    PrepackPlane u[4];
    PrepackPlane w[4];
    int32_t stages;
    int32_t code_bits;
    int32_t n_c, k_c, n_cp, k_cp;
    int32_t rounding;
    float cos_tab[16];
    float sin_tab[16];
    __half* out;  // [2 n_c, 2 k_c]
};

// float32 -> fp16 bits, ties away from zero (same steps as the reference's
// floatToHalfBits: truncate, add one ulp when the first dropped bit is set).
__device__ __forceinline__ uint16_t f32_to_f16_ties_away(float x) {
    const uint32_t bits = __float_as_uint(x);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const int32_t exp = static_cast<int32_t>((bits >> 23) & 0xffu) - 127 + 15;
    uint32_t mant = bits & 0x7fffffu;
    if (exp <= 0) {
        if (exp < -10) return static_cast<uint16_t>(sign);
        mant |= 0x800000u;
        const int shift = 14 - exp;
        uint32_t hm = mant >> shift;
        if ((mant >> (shift - 1)) & 1u) ++hm;
        return static_cast<uint16_t>(sign | hm);
    }
    if (exp >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    uint32_t h = sign | (static_cast<uint32_t>(exp) << 10) | (mant >> 13);
    if (mant & 0x1000u) ++h;
    return static_cast<uint16_t>(h);
}

__device__ __forceinline__ uint16_t to_f16_bits(float x, int rounding) {
    if (rounding == kRoundTiesAway) return f32_to_f16_ties_away(x);
    return __half_as_ushort(__float2half_rn(x));
}

// Code of complex column `col` in a row of a b-bit plane (LSB-first stream).
__device__ __forceinline__ uint32_t read_code(const uint8_t* row, int col, int bits) {
    const int bit = col * bits;
    const int byte = bit >> 3;
    const int sh = bit & 7;
    uint32_t v = row[byte];
    if (sh + bits > 8) v |= static_cast<uint32_t>(row[byte + 1]) << 8;
    return (v >> sh) & ((1u << bits) - 1u);
}

__device__ __forceinline__ void decode_value(const PrepackParams& p, uint32_t code, float inv_r, float inv_i,
                                             float& re, float& im) {
    if (p.code_bits == 2) {
        re = code == 0 ? -inv_r : (code == 1 ? inv_r : 0.0f);
        im = code == 2 ? -inv_i : (code == 3 ? inv_i : 0.0f);
    } else {
        re = __fmul_rn(p.cos_tab[code], inv_r);
        im = __fmul_rn(p.sin_tab[code], inv_i);
    }
}

__global__ void __launch_bounds__(256) prepack_kernel(const PrepackParams p) {
    const int n = blockIdx.y;
    const int col4 = blockIdx.x * blockDim.x + threadIdx.x;  // group of 4 complex columns
    const int k_base = col4 * 4;
    if (n >= p.n_c || k_base >= p.k_c) return;
    const int blocks = p.k_cp / 256;
    const int gidx = n * blocks + (k_base >> 8);
    const int row_bytes = p.k_cp * p.code_bits / 8;

    float rr[4], ir[4], ri[4], ii[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) rr[e] = ir[e] = ri[e] = ii[e] = 0.0f;

    // U stages: y = U x  ->  rr += Ur, ir -= Ui, ri += Ui, ii += Ur
    for (int s = 0; s < p.stages; ++s) {
        const PrepackPlane& pl = p.u[s];
        const float inv_r = __frcp_rn(__half2float(pl.gamma_re[gidx]));
        const float inv_i = __frcp_rn(__half2float(pl.gamma_im[gidx]));
        const uint8_t* row = pl.codes + static_cast<int64_t>(n) * row_bytes;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float re, im;
            decode_value(p, read_code(row, k_base + e, p.code_bits), inv_r, inv_i, re, im);
            if (s == 0) {
                rr[e] = re;
                ir[e] = -im;
                ri[e] = im;
                ii[e] = re;
            } else {
                rr[e] = __fadd_rn(rr[e], re);
                ir[e] = __fsub_rn(ir[e], im);
                ri[e] = __fadd_rn(ri[e], im);
                ii[e] = __fadd_rn(ii[e], re);
            }
        }
    }
    // W stages: y += W conj(x)  ->  rr += Wr, ir += Wi, ri += Wi, ii -= Wr
    for (int s = 0; s < p.stages; ++s) {
        const PrepackPlane& pl = p.w[s];
        const float inv_r = __frcp_rn(__half2float(pl.gamma_re[gidx]));
        const float inv_i = __frcp_rn(__half2float(pl.gamma_im[gidx]));
        const uint8_t* row = pl.codes + static_cast<int64_t>(n) * row_bytes;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float re, im;
            decode_value(p, read_code(row, k_base + e, p.code_bits), inv_r, inv_i, re, im);
            rr[e] = __fadd_rn(rr[e], re);
            ir[e] = __fadd_rn(ir[e], im);
            ri[e] = __fadd_rn(ri[e], im);
            ii[e] = __fsub_rn(ii[e], re);
        }
    }

    const int64_t K = 2 * static_cast<int64_t>(p.k_c);
    uint16_t* out = reinterpret_cast<uint16_t*>(p.out);
    uint16_t* o_rr = out + static_cast<int64_t>(n) * K + k_base;
    uint16_t* o_ir = o_rr + p.k_c;
    uint16_t* o_ri = out + static_cast<int64_t>(n + p.n_c) * K + k_base;
    uint16_t* o_ii = o_ri + p.k_c;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        if (k_base + e < p.k_c) {
            o_rr[e] = to_f16_bits(rr[e], p.rounding);
            o_ir[e] = to_f16_bits(ir[e], p.rounding);
            o_ri[e] = to_f16_bits(ri[e], p.rounding);
            o_ii[e] = to_f16_bits(ii[e], p.rounding);
        }
    }
}

}  // namespace rpfq
