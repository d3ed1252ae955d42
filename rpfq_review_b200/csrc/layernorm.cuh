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
// Loads: VW = 4, 2 or 1 consecutive floats per lane and step (by row length).
#pragma once

#include "ptx.cuh"

namespace rpfq {

struct LayerNormParams {
    const float* x;
    const __half* w;
    const __half* b;
    __half* y;
    int64_t ldx, ldy;
    int64_t m;
    float eps;
    int32_t act_bits;
    const int32_t* rows;  // optional gather: output row r normalizes input row rows[r]
    int64_t x_rows;       // rows of x (gather indices outside [0, x_rows) are rejected)
    int* err;
};

template <int D>
__global__ void __launch_bounds__(256) layernorm_f32_f16_kernel(const LayerNormParams p) {
    static_assert(D % 32 == 0, "row length must be a multiple of 32");
    // VW consecutive floats per lane and step: element e of step j of lane l
    // sits at column 32 VW j + VW l + e (coalesced, 16-/8-/4-byte loads)
    constexpr int VW = D % 128 == 0 ? 4 : (D % 64 == 0 ? 2 : 1);
    constexpr int J = D / (32 * VW);
    const int warps = blockDim.x >> 5;
    // Rows are taken last to first: the GEMM that wrote x finished with its
    // highest row blocks, which are the ones still in L2, and the GEMM that
    // reads y starts with the lowest rows, the ones written last here.
    const int64_t slot = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5);
    const int64_t row = p.m - 1 - slot;
    const int lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    if (slot >= p.m) return;
    int64_t src = row;
    if (p.rows != nullptr) {
        src = p.rows[row];
        if (src < 0 || src >= p.x_rows) {  // bad gather index: report, touch nothing
            if ((threadIdx.x & 31) == 0) atomicCAS(p.err, 0, 901);
            return;
        }
    }
    const float* xr = p.x + src * p.ldx;
    float v[J][VW];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int col = 32 * VW * j + VW * lane;
        if constexpr (VW == 4) {
            const float4 t = *reinterpret_cast<const float4*>(xr + col);
            v[j][0] = t.x;
            v[j][1] = t.y;
            v[j][2] = t.z;
            v[j][3] = t.w;
            sum += (t.x + t.y) + (t.z + t.w);
        } else if constexpr (VW == 2) {
            const float2 t = *reinterpret_cast<const float2*>(xr + col);
            v[j][0] = t.x;
            v[j][1] = t.y;
            sum += t.x + t.y;
        } else {
            v[j][0] = xr[col];
            sum += v[j][0];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
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
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq / static_cast<float>(D) + p.eps);
    float amax_re = 0.0f, amax_im = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int col = 32 * VW * j + VW * lane;
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
    float s_re = 0.0f, s_im = 0.0f, qmax = 0.0f, qmin = 0.0f;
    if (p.act_bits > 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            amax_re = fmaxf(amax_re, __shfl_xor_sync(0xffffffffu, amax_re, o));
            amax_im = fmaxf(amax_im, __shfl_xor_sync(0xffffffffu, amax_im, o));
        }
        qmax = static_cast<float>((1 << (p.act_bits - 1)) - 1);
        qmin = -static_cast<float>(1 << (p.act_bits - 1));
        // The quantizer sees the fp16 GEMM input, as in the unfused path.
        s_re = __fmul_rn(__frcp_rn(fmaxf(__half2float(__float2half_rn(amax_re)), 1e-5f)), qmax);
        s_im = __fmul_rn(__frcp_rn(fmaxf(__half2float(__float2half_rn(amax_im)), 1e-5f)), qmax);
    }
    __half* yr = p.y + row * p.ldy;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int col = 32 * VW * j + VW * lane;
        float o[VW];
#pragma unroll
        for (int e = 0; e < VW; ++e) {
            o[e] = v[j][e];
            if (p.act_bits > 0) {
                const float s = (col + e < D / 2) ? s_re : s_im;
                const float h = __half2float(__float2half_rn(o[e]));
                const float q = fminf(fmaxf(rintf(__fmul_rn(h, s)), qmin), qmax);
                o[e] = __fdiv_rn(q, s);
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
