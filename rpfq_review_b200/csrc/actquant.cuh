// Activation quantization of the complex input (ActivationQuantSTE.forward,
// quant_i.py:442-455 of the reference), one warp per row:
//
//   per row and separately for the Re half [0, k_c) and the Im half [k_c, 2 k_c):
//   s  = fl(fl(1 / max(amax, 1e-5)) * qmax)      (torch evaluates qmax / t as
//                                                 reciprocal(t) * qmax)
//   q  = clamp(rint(fl(x * s)), qmin, qmax)       (round half to even)
//   x' = fl(q / s)                               -> fp16 (round to nearest even)
//
// Row amax: 16-byte vector loads, per-lane max, warp-shuffle max reduction.
// The row is re-read for the quantize pass (it is L1/L2 resident). q takes
// only 2^num_bits values per half row (plus -0, which rint gives for small
// negative x and which divides to -0), so the warp divides each of them once
// (IEEE division, as torch) into a shared-memory table of the fp16 results and
// every element looks its q up: the same bits as dividing per element, without
// a division subroutine per element. Table slot 2^num_bits holds fl(-0 / s).
#pragma once

#include "ptx.cuh"

namespace rpfq {

struct ActQuantParams {
    const __half* x;
    __half* y;
    int64_t ldx, ldy;
    int64_t m;
    int32_t k_c;  // half width (row has 2 k_c values)
    int32_t num_bits;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Table slot of an integer-valued q in [qmin, qmax]: q - qmin, or nq for -0.
__device__ __forceinline__ int qslot(float q, float qmin, int nq) {
    return __float_as_uint(q) == 0x80000000u ? nq : static_cast<int>(q - qmin);
}

__global__ void __launch_bounds__(256) act_quant_kernel(const ActQuantParams p) {
    __shared__ __half qtab[8][2][264];  // per warp and half: fp16(q / s) for q = qmin .. qmax, then q = -0
    const int warps_per_block = blockDim.x >> 5;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * warps_per_block + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    if (row >= p.m) return;
    const __half* xr = p.x + row * p.ldx;
    __half* yr = p.y + row * p.ldy;
    const int k_c = p.k_c;
    const bool vec = (k_c % 8 == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(yr) & 15) == 0);
    const float qmax = static_cast<float>((1 << (p.num_bits - 1)) - 1);
    const float qmin = -static_cast<float>(1 << (p.num_bits - 1));

    float amax[2] = {0.0f, 0.0f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const __half* src = xr + h * k_c;
        float a = 0.0f;
        if (vec) {
            for (int i = lane * 8; i < k_c; i += 32 * 8) {
                const uint4 v = *reinterpret_cast<const uint4*>(src + i);
                const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hv[e]);
                    a = fmaxf(a, fmaxf(fabsf(f.x), fabsf(f.y)));
                }
            }
        } else {
            for (int i = lane; i < k_c; i += 32) a = fmaxf(a, fabsf(__half2float(src[i])));
        }
        amax[h] = warp_max(a);
    }

    __half(*tab)[264] = qtab[threadIdx.x >> 5];
    const int nq = 1 << p.num_bits;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float s = __fmul_rn(__frcp_rn(fmaxf(amax[h], 1e-5f)), qmax);
        for (int t = lane; t < nq; t += 32) tab[h][t] = __float2half_rn(__fdiv_rn(qmin + static_cast<float>(t), s));
        if (lane == 0) tab[h][nq] = __float2half_rn(__fdiv_rn(-0.0f, s));
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float s = __fmul_rn(__frcp_rn(fmaxf(amax[h], 1e-5f)), qmax);
        const __half* th = tab[h];
        const __half* src = xr + h * k_c;
        __half* dst = yr + h * k_c;
        if (vec) {
            for (int i = lane * 8; i < k_c; i += 32 * 8) {
                const uint4 v = *reinterpret_cast<const uint4*>(src + i);
                const __half2* hv = reinterpret_cast<const __half2*>(&v);
                uint4 o;
                uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hv[e]);
                    const float q0 = fminf(fmaxf(rintf(__fmul_rn(f.x, s)), qmin), qmax);
                    const float q1 = fminf(fmaxf(rintf(__fmul_rn(f.y, s)), qmin), qmax);
                    __half2 r = __halves2half2(th[qslot(q0, qmin, nq)], th[qslot(q1, qmin, nq)]);
                    ov[e] = *reinterpret_cast<uint32_t*>(&r);
                }
                *reinterpret_cast<uint4*>(dst + i) = o;
            }
        } else {
            for (int i = lane; i < k_c; i += 32) {
                const float f = __half2float(src[i]);
                const float q = fminf(fmaxf(rintf(__fmul_rn(f, s)), qmin), qmax);
                dst[i] = th[qslot(q, qmin, nq)];
            }
        }
    }
}

}  // namespace rpfq
