// Exporter algorithm on the device: float weight -> packed 2-bit axial planes.
//
// Restates save_quantized_linear / quantize_complex_weight of the reference
// exporter (RPFQ-ViTApple/scripts/export_rpfq_vit_to_mlx.py:257-289,317-333,
// 384-423): the real weight [2 n_c, 2 k_c] = [[A11, A12], [A21, A22]] is split
// into the widely-linear parts
//   U = 0.5 (A11 + A22) + i 0.5 (A21 - A12),   W = 0.5 (A11 - A22) + i 0.5 (A12 + A21)
// and each part gets `stages` residual axial quantization steps. One step
// (export...py:189-224): per element the dominant axis with quadrant
// tie-breaking (:127-145) gives the code (0:-1, 1:+1, 2:-i, 3:+i); one scale
// per axis for the whole matrix is the masked mean |value| clamped at 1e-6
// (:121-124); gamma = fp16(1 / scale); the dequantized value +-1/gamma
// (:227-254) is subtracted from the residual.
//
// Two kernels per step, for U and W together:
//   pack_stats_kernel  masked |value| sums and counts, fp64, one partial per CTA
//   pack_codes_kernel  every CTA reduces the partials in the same fixed order,
//                      derives the gammas, writes one code byte per thread
//                      (padding included) and the residual for the next step.
// HBM-bound: per step one read of the parts (16 B per complex element for the
// first step, from the weight; from the residual planes after) and one write
// of the residual, plus n_cp*k_cp/2 code bytes.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace rpfq {

constexpr int kPackThreads = 256;
constexpr int kPackPartials = 8;  // per CTA: (sum, count) x (U re, U im, W re, W im)
constexpr int kPackMaxStatsCtas = 1024;

struct PackParams {
    const float* weight;  // [2 n_c, 2 k_c], row stride ldw (first step only)
    int64_t ldw;
    int32_t n_c, k_c, n_cp, k_cp;
    int32_t first;        // 1: read the parts from the weight, 0: from res
    int32_t write_res;    // 0 on the last step
    float* res;           // [4][n_c * k_c]: U re, U im, W re, W im
    double* partials;     // [stats grid][kPackPartials]
    int32_t stats_ctas;
    uint8_t* codes[2];    // this step's U, W code planes [n_cp, k_cp/4]
    uint16_t* gre[2];     // [n_cp, k_cp/256]
    uint16_t* gim[2];
};

// U re, U im, W re, W im of complex element (row, col), as the exporter's
// fp32 tensor expressions 0.5 * (a + b).
__device__ __forceinline__ void pack_load_parts(const PackParams& p, int row, int col, float (&v)[4]) {
    if (p.first) {
        const float* r0 = p.weight + static_cast<int64_t>(row) * p.ldw;
        const float* r1 = p.weight + static_cast<int64_t>(row + p.n_c) * p.ldw;
        const float a11 = r0[col], a12 = r0[p.k_c + col], a21 = r1[col], a22 = r1[p.k_c + col];
        v[0] = __fmul_rn(0.5f, __fadd_rn(a11, a22));
        v[1] = __fmul_rn(0.5f, __fsub_rn(a21, a12));
        v[2] = __fmul_rn(0.5f, __fsub_rn(a11, a22));
        v[3] = __fmul_rn(0.5f, __fadd_rn(a12, a21));
    } else {
        const int64_t nk = static_cast<int64_t>(p.n_c) * p.k_c;
        const int64_t e = static_cast<int64_t>(row) * p.k_c + col;
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = p.res[j * nk + e];
    }
}

// Dominant-axis code with the exporter's quadrant tie-breaking
// (export...py:127-145); in_r / in_i: the element counts toward the real /
// imaginary scale. NaN falls in no mask (code 0), as in the reference.
__device__ __forceinline__ uint32_t axial_code(float re, float im, bool& in_r, bool& in_i) {
    const float ar = fabsf(re), ai = fabsf(im);
    const bool real_dom = ar > ai, imag_dom = ai > ar;
    const bool tie = !(real_dom || imag_dom);
    const bool zero_tie = tie && re == 0.0f && im == 0.0f;
    const bool q1 = tie && re > 0.0f && im > 0.0f;
    const bool q2 = tie && re < 0.0f && im > 0.0f;
    const bool q3 = tie && re < 0.0f && im < 0.0f;
    const bool q4 = tie && re > 0.0f && im < 0.0f;
    const bool rp = (real_dom && re >= 0.0f) || q4 || zero_tie;
    const bool rn = (real_dom && re < 0.0f) || q2;
    const bool ip = (imag_dom && im >= 0.0f) || q1;
    const bool ineg = (imag_dom && im < 0.0f) || q3;
    in_r = rp || rn;
    in_i = ip || ineg;
    return rp ? 1u : (ineg ? 2u : (ip ? 3u : 0u));
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(kPackThreads) pack_stats_kernel(const PackParams p) {
    double acc[kPackPartials];
#pragma unroll
    for (int j = 0; j < kPackPartials; ++j) acc[j] = 0.0;
    const int64_t total = static_cast<int64_t>(p.n_c) * p.k_c;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int row = static_cast<int>(e / p.k_c), col = static_cast<int>(e % p.k_c);
        float v[4];
        pack_load_parts(p, row, col, v);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
            bool in_r, in_i;
            axial_code(v[2 * part], v[2 * part + 1], in_r, in_i);
            if (in_r) {
                acc[4 * part + 0] += fabs(static_cast<double>(v[2 * part]));
                acc[4 * part + 1] += 1.0;
            }
            if (in_i) {
                acc[4 * part + 2] += fabs(static_cast<double>(v[2 * part + 1]));
                acc[4 * part + 3] += 1.0;
            }
        }
    }
    __shared__ double red[kPackThreads / 32][kPackPartials];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < kPackPartials; ++j) {
        const double s = warp_sum_f64(acc[j]);
        if (lane == 0) red[warp][j] = s;
    }
    __syncthreads();
    if (threadIdx.x < kPackPartials) {
        double s = 0.0;
        for (int w = 0; w < kPackThreads / 32; ++w) s += red[w][threadIdx.x];
        p.partials[static_cast<int64_t>(blockIdx.x) * kPackPartials + threadIdx.x] = s;
    }
}

// fp16 bits of 1 / scale for the masked mean sum / count: mean and clamp in
// fp32 (torch: (|x| * m).sum() / m.sum().clamp_min(1)).clamp_min(1e-6)), the
// reciprocal as a Python float (fp64) division, stored through torch.full
// (fp64 -> fp32 -> fp16).
__device__ __forceinline__ uint16_t pack_gamma_bits(double sum, double count) {
    const float c = fmaxf(static_cast<float>(count), 1.0f);
    const float mean = fmaxf(__fdiv_rn(static_cast<float>(sum), c), 1e-6f);
    const double inv = 1.0 / static_cast<double>(mean);
    return __half_as_ushort(__float2half_rn(static_cast<float>(inv)));
}

__global__ void __launch_bounds__(kPackThreads) pack_codes_kernel(const PackParams p) {
    __shared__ uint16_t g_sh[4];  // U re, U im, W re, W im gamma bits
    if (threadIdx.x < 4) {
        double s = 0.0, c = 0.0;
        for (int b = 0; b < p.stats_ctas; ++b) {
            s += p.partials[static_cast<int64_t>(b) * kPackPartials + 2 * threadIdx.x];
            c += p.partials[static_cast<int64_t>(b) * kPackPartials + 2 * threadIdx.x + 1];
        }
        g_sh[threadIdx.x] = pack_gamma_bits(s, c);
    }
    __syncthreads();
    const uint16_t gbits[4] = {g_sh[0], g_sh[1], g_sh[2], g_sh[3]};
    // +-1 / gamma in fp32 (torch: w / gamma.float(), w in {-1, 0, 1})
    float inv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) inv[j] = __fdiv_rn(1.0f, __half2float(__ushort_as_half(gbits[j])));

    const int bytes_per_row = p.k_cp / 4;
    const int64_t total = static_cast<int64_t>(p.n_cp) * bytes_per_row;
    const int64_t nk = static_cast<int64_t>(p.n_c) * p.k_c;
    const int blocks = p.k_cp / 256;
    const int64_t gamma_total = static_cast<int64_t>(p.n_cp) * blocks;
    for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < total;
         b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int row = static_cast<int>(b / bytes_per_row);
        const int cb = static_cast<int>(b % bytes_per_row);
        uint32_t byte[2] = {0u, 0u};
        if (row < p.n_c) {
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const int col = 4 * cb + l;
                if (col >= p.k_c) break;
                float v[4];
                pack_load_parts(p, row, col, v);
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    bool in_r, in_i;
                    const uint32_t code = axial_code(v[2 * part], v[2 * part + 1], in_r, in_i);
                    byte[part] |= code << (2 * l);
                    if (p.write_res) {
                        const float ir = inv[2 * part], ii = inv[2 * part + 1];
                        const float d_r = code == 0 ? -ir : (code == 1 ? ir : 0.0f);
                        const float d_i = code == 2 ? -ii : (code == 3 ? ii : 0.0f);
                        const int64_t e = static_cast<int64_t>(row) * p.k_c + col;
                        p.res[(2 * part) * nk + e] = __fsub_rn(v[2 * part], d_r);
                        p.res[(2 * part + 1) * nk + e] = __fsub_rn(v[2 * part + 1], d_i);
                    }
                }
            }
        }
        p.codes[0][b] = static_cast<uint8_t>(byte[0]);
        p.codes[1][b] = static_cast<uint8_t>(byte[1]);
        if (b < gamma_total) {
            p.gre[0][b] = gbits[0];
            p.gim[0][b] = gbits[1];
            p.gre[1][b] = gbits[2];
            p.gim[1][b] = gbits[3];
        }
    }
}

}  // namespace rpfq
