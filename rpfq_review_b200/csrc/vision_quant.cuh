// Vision-aware activation quantization (token saliency).
//
// Restates VisionAwareActivationQuantizer.forward of the reference
// (RPFQ-ViT-main/quant_models/quant_rpfq_vit_vision.py:26-171) for the fp16
// input of a packed layer, x[t] = [Re | Im] (k_c columns each):
//   A  per token (one warp each, all images at once): amax of |Re| and |Im| and the energy
//      mean_j sqrt(re^2 + im^2 + 1e-6)                               (:63-64, :80)
//   B  per image (one CTA), per patch token on the g x g grid: contrast = mean |energy step| to
//      its 4-neighbours, summed up, down, left, right (:83-98); score =
//      w * e / max(mean e, eps) + (1 - w) * c / max(mean c, eps)   (:99-106)
//   C  the k highest scores (ties: lower patch index first) are salient; the
//      CLS token is salient iff protect_cls                           (:108-143)
//   D  background amax per half over the non-salient tokens        (:145-149)
//   E  per element (all rows at once): s = 127 * rcp(max(amax_token or background * clip, eps)),
//      q = rint(x s) clamped to [-128, 127], out = x + (q / s - x), to fp16
//                                                                      (:57-64, :156-167)
// Inputs without a square patch grid (grid = 0) use the per-token scale for
// every token (:151-154). fp32 everywhere with the reference's operation
// order; only the energy / contrast sums differ in summation order, which
// moves scores by ulps (the saliency order, not the quantized values).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace rpfq {

constexpr int kVisionThreads = 512;
constexpr int kVisionMaxTokens = 16385;  // 1 + 128 x 128 patches with a saliency grid
constexpr float kVisionEps = 1e-6f;

struct VisionQuantParams {
    const __half* x;
    int64_t ldx;
    __half* y;
    int64_t ldy;
    int32_t tokens;       // per image
    int32_t k_c;          // complex columns (Re and Im halves of k_c each)
    int32_t grid;         // g, or 0: per-token scales for every token
    int32_t num_salient;  // salient patches per image
    int32_t protect_cls;
    float clip;           // background_clip_ratio
    float w_energy;       // energy_score_weight
    float w_contrast;     // 1 - energy_score_weight (rounded once from double)
    uint8_t* mask_out;    // [images * tokens] or nullptr
};

__device__ __forceinline__ float vq_scale(float amax) {
    return __fmul_rn(__frcp_rn(fmaxf(amax, kVisionEps)), 127.0f);
}

__device__ __forceinline__ float block_sum_f32(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int w = 0; w < kVisionThreads / 32; ++w) s = __fadd_rn(s, red[w]);
    return s;
}

__device__ __forceinline__ float block_max_f32(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = 0.0f;
    for (int w = 0; w < kVisionThreads / 32; ++w) m = fmaxf(m, red[w]);
    return m;
}

// One token row: per-half amax (and the energy when `energy` is set).
__device__ __forceinline__ void vq_row_stats(const VisionQuantParams& p, const __half* row, bool energy,
                                             float& amax_re, float& amax_im, float& esum) {
    const int lane = threadIdx.x & 31;
    float ar = 0.0f, ai = 0.0f, es = 0.0f;
    for (int j0 = lane * 8; j0 < p.k_c; j0 += 256) {
        const uint4 vr = *reinterpret_cast<const uint4*>(row + j0);
        const uint4 vi = *reinterpret_cast<const uint4*>(row + p.k_c + j0);
        const __half2* hr = reinterpret_cast<const __half2*>(&vr);
        const __half2* hi = reinterpret_cast<const __half2*>(&vi);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 r = __half22float2(hr[e]);
            const float2 i = __half22float2(hi[e]);
            ar = fmaxf(ar, fmaxf(fabsf(r.x), fabsf(r.y)));
            ai = fmaxf(ai, fmaxf(fabsf(i.x), fabsf(i.y)));
            if (energy) {
                es = __fadd_rn(es, __fsqrt_rn(__fadd_rn(__fadd_rn(__fmul_rn(r.x, r.x), __fmul_rn(i.x, i.x)), kVisionEps)));
                es = __fadd_rn(es, __fsqrt_rn(__fadd_rn(__fadd_rn(__fmul_rn(r.y, r.y), __fmul_rn(i.y, i.y)), kVisionEps)));
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ar = fmaxf(ar, __shfl_xor_sync(0xffffffffu, ar, o));
        ai = fmaxf(ai, __shfl_xor_sync(0xffffffffu, ai, o));
        es = __fadd_rn(es, __shfl_xor_sync(0xffffffffu, es, o));
    }
    amax_re = ar;
    amax_im = ai;
    esum = es;
}

__device__ __forceinline__ void vq_quantize_row(const VisionQuantParams& p, const __half* row, __half* out, float sr,
                                                float si) {
    const int lane = threadIdx.x & 31;
    for (int c0 = lane * 8; c0 < 2 * p.k_c; c0 += 256) {
        const float s = c0 < p.k_c ? sr : si;
        const uint4 v = *reinterpret_cast<const uint4*>(row + c0);
        const __half2* h = reinterpret_cast<const __half2*>(&v);
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(h[e]);
            float r[2] = {f.x, f.y};
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float q = fminf(fmaxf(rintf(__fmul_rn(r[u], s)), -128.0f), 127.0f);
                const float qx = __fdiv_rn(q, s);
                r[u] = __fadd_rn(r[u], __fsub_rn(qx, r[u]));
            }
            const __half2 hh = __floats2half2_rn(r[0], r[1]);
            ow[e] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        *reinterpret_cast<uint4*>(out + c0) = o;
    }
}

// vq_quantize_row with the quotients q / s taken from a table: tab[h][q + 128]
// = fl(q / s_h) for the integers q in [-128, 127] (the only values q takes), so
// the IEEE division runs once per table entry instead of once per element.
// q = -0 reads the +0 entry; x + (q / s - x) is +0 for either sign of zero, so
// the output bits equal vq_quantize_row's. Eight 16-byte chunks of the row per
// lane are loaded before the first is used.
__device__ __forceinline__ void vq_quantize_row_tab(const VisionQuantParams& p, const __half* row, __half* out,
                                                    float sr, float si, const float (*tab)[256]) {
    const int lane = threadIdx.x & 31;
    const int n = 2 * p.k_c;
    for (int c00 = lane * 8; c00 < n; c00 += 8 * 256) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (c00 + u * 256 < n) v[u] = *reinterpret_cast<const uint4*>(row + c00 + u * 256);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c0 = c00 + u * 256;
            if (c0 >= n) break;
            const bool re = c0 < p.k_c;  // k_c % 8 == 0: a chunk lies in one half
            const float s = re ? sr : si;
            const float* th = tab[re ? 0 : 1];
            const __half2* h = reinterpret_cast<const __half2*>(&v[u]);
            uint4 o;
            uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(h[e]);
                float r[2] = {f.x, f.y};
#pragma unroll
                for (int w = 0; w < 2; ++w) {
                    const float q = fminf(fmaxf(rintf(__fmul_rn(r[w], s)), -128.0f), 127.0f);
                    const float qx = th[static_cast<int>(q) + 128];
                    r[w] = __fadd_rn(r[w], __fsub_rn(qx, r[w]));
                }
                const __half2 hh = __floats2half2_rn(r[0], r[1]);
                ow[e] = *reinterpret_cast<const uint32_t*>(&hh);
            }
            *reinterpret_cast<uint4*>(out + c0) = o;
        }
    }
}

constexpr int kVisionApplyRun = 4;  // consecutive rows per warp (one image's background rows share scales)

// grid = 0: one warp per token, no shared state (any token count).
__global__ void __launch_bounds__(kVisionThreads) vision_quant_tokenwise_kernel(const VisionQuantParams p,
                                                                               int64_t rows) {
    pdl_wait();  // the producer of x (or of the statistics) has completed
    pdl_launch_dependents();
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kVisionThreads / 32);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (kVisionThreads / 32) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const __half* row = p.x + r * p.ldx;
        float ar, ai, es;
        vq_row_stats(p, row, false, ar, ai, es);
        vq_quantize_row(p, row, p.y + r * p.ldy, vq_scale(ar), vq_scale(ai));
        if (p.mask_out != nullptr && (threadIdx.x & 31) == 0) p.mask_out[r] = 1;
    }
}

// grid > 0, three kernels so that every pass over x runs on the whole GPU:
//   vision_stats_kernel   one warp per row, all images: amax re / im, energy
//   vision_select_kernel  one CTA per image over its T statistics only:
//                         contrast, scores, rank selection, background amax,
//                         the two scales of every token
//   vision_apply_kernel   elementwise over all rows: quantize with the scales
struct VisionTokenStats {
    float amax_re, amax_im, energy, pad;
};

__global__ void __launch_bounds__(kVisionThreads) vision_stats_kernel(const VisionQuantParams p, int64_t rows,
                                                                     VisionTokenStats* stats) {
    pdl_wait();  // the producer of x (or of the statistics) has completed
    pdl_launch_dependents();
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kVisionThreads / 32);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (kVisionThreads / 32) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const bool patch = (r % p.tokens) != 0;
        float ar, ai, es;
        vq_row_stats(p, p.x + r * p.ldx, patch, ar, ai, es);
        if ((threadIdx.x & 31) == 0)
            stats[r] = VisionTokenStats{ar, ai, patch ? __fdiv_rn(es, static_cast<float>(p.k_c)) : 0.0f, 0.0f};
    }
}

// Dynamic shared memory: 2 floats per patch (energy then score, contrast) + 1 byte per token.
__global__ void __launch_bounds__(kVisionThreads) vision_select_kernel(const VisionQuantParams p,
                                                                      const VisionTokenStats* stats, float2* scales) {
    pdl_wait();  // the producer of x (or of the statistics) has completed
    pdl_launch_dependents();
    extern __shared__ float vsm[];
    const int T = p.tokens;
    const int P = T - 1;
    const int g = p.grid;
    float* energy = vsm;  // patch energies, then scores
    float* contrast = vsm + P;
    uint8_t* mask = reinterpret_cast<uint8_t*>(vsm + 2 * P);
    __shared__ float red[kVisionThreads / 32];
    const int64_t img_row0 = static_cast<int64_t>(blockIdx.x) * T;
    const VisionTokenStats* st = stats + img_row0;
    for (int q = threadIdx.x; q < P; q += kVisionThreads) energy[q] = st[q + 1].energy;
    __syncthreads();
    // contrast on the patch grid (up, down, left, right), then the two means
    float esum = 0.0f, csum = 0.0f;
    for (int q = threadIdx.x; q < P; q += kVisionThreads) {
        const int i = q / g, j = q % g;
        const float e = energy[q];
        float c = 0.0f, n = 0.0f;
        if (i > 0) { c = __fadd_rn(c, fabsf(__fsub_rn(e, energy[q - g]))); n += 1.0f; }
        if (i + 1 < g) { c = __fadd_rn(c, fabsf(__fsub_rn(energy[q + g], e))); n += 1.0f; }
        if (j > 0) { c = __fadd_rn(c, fabsf(__fsub_rn(e, energy[q - 1]))); n += 1.0f; }
        if (j + 1 < g) { c = __fadd_rn(c, fabsf(__fsub_rn(energy[q + 1], e))); n += 1.0f; }
        c = __fdiv_rn(c, fmaxf(n, 1.0f));
        contrast[q] = c;
        esum = __fadd_rn(esum, e);
        csum = __fadd_rn(csum, c);
    }
    const float emean = fmaxf(__fdiv_rn(block_sum_f32(esum, red), static_cast<float>(P)), kVisionEps);
    const float cmean = fmaxf(__fdiv_rn(block_sum_f32(csum, red), static_cast<float>(P)), kVisionEps);
    __syncthreads();
    for (int q = threadIdx.x; q < P; q += kVisionThreads)
        energy[q] = __fadd_rn(__fmul_rn(p.w_energy, __fdiv_rn(energy[q], emean)),
                              __fmul_rn(p.w_contrast, __fdiv_rn(contrast[q], cmean)));
    __syncthreads();
    // rank selection of the salient patches (ties: lower index first)
    for (int q = threadIdx.x; q < P; q += kVisionThreads) {
        const float s = energy[q];
        int rank = 0;
        for (int o = 0; o < P; ++o) {
            const float so = energy[o];
            rank += (so > s) || (so == s && o < q);
        }
        mask[q + 1] = rank < p.num_salient ? 1 : 0;
    }
    if (threadIdx.x == 0) mask[0] = p.protect_cls ? 1 : 0;
    __syncthreads();
    // background amax over the non-salient tokens, per half
    float br = 0.0f, bi = 0.0f;
    for (int t = threadIdx.x; t < T; t += kVisionThreads)
        if (!mask[t]) {
            br = fmaxf(br, st[t].amax_re);
            bi = fmaxf(bi, st[t].amax_im);
        }
    const float s_bg_re = vq_scale(__fmul_rn(block_max_f32(br, red), p.clip));
    const float s_bg_im = vq_scale(__fmul_rn(block_max_f32(bi, red), p.clip));
    for (int t = threadIdx.x; t < T; t += kVisionThreads) {
        const bool sal = mask[t] != 0;
        scales[img_row0 + t] = sal ? make_float2(vq_scale(st[t].amax_re), vq_scale(st[t].amax_im))
                                   : make_float2(s_bg_re, s_bg_im);
        if (p.mask_out != nullptr) p.mask_out[img_row0 + t] = mask[t];
    }
}

// One warp per row (no index division), 16 bytes per lane and step.
__global__ void __launch_bounds__(kVisionThreads) vision_apply_kernel(const VisionQuantParams p, int64_t rows,
                                                                     const float2* scales) {
    pdl_wait();  // the producer of x (or of the statistics) has completed
    pdl_launch_dependents();
    __shared__ float qtab[kVisionThreads / 32][2][256];  // per warp: fl(q / s) of the scales it holds
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float(*tab)[256] = qtab[warp];
    float tab_sr = 0.0f, tab_si = 0.0f;  // scales are > 0: 0 marks an empty table
    const int64_t step = static_cast<int64_t>(gridDim.x) * (kVisionThreads / 32) * kVisionApplyRun;
    for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * (kVisionThreads / 32) + warp) * kVisionApplyRun; r0 < rows;
         r0 += step) {
        for (int64_t r = r0; r < r0 + kVisionApplyRun && r < rows; ++r) {
            const float2 sc = scales[r];
            if (sc.x != tab_sr || sc.y != tab_si) {
                __syncwarp();  // every lane is done with the previous table
                for (int t = lane; t < 256; t += 32) {
                    tab[0][t] = __fdiv_rn(static_cast<float>(t - 128), sc.x);
                    tab[1][t] = __fdiv_rn(static_cast<float>(t - 128), sc.y);
                }
                __syncwarp();
                tab_sr = sc.x;
                tab_si = sc.y;
            }
            vq_quantize_row_tab(p, p.x + r * p.ldx, p.y + r * p.ldy, sc.x, sc.y, tab);
        }
    }
}

}  // namespace rpfq
