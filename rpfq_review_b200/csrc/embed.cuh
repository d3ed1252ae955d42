// Patch unfold of the ViT / DeiT input: images [B, C, H, W] (fp16 or fp32,
// contiguous) -> the patch-embedding GEMM's fp16 rows
//
//   patches[b * gh * gw + i * gw + j][c * P * P + y * P + x] = image[b][c][i * P + y][j * P + x]
//
// (gh = H / P, gw = W / P), the CHW patch order of the reference's
// patchify_tensor (RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:125-134)
// and of Conv2d(C, d, P, stride P) weights flattened to [d, C P P].
//
// One thread per CH = 8 (P a multiple of 8: ViT / DeiT) or CH = 4 (P a
// multiple of 4: Swin's 4x4 patches) consecutive pixels of an image row, which
// stay inside one patch: coalesced 2·CH-byte (fp16) or 4·CH-byte (fp32) loads
// and one 2·CH-byte store into a 2·P-byte run of the patch row.
// HBM-bound: (2 or 4) + 2 bytes per pixel.
#pragma once

#include "ptx.cuh"

namespace rpfq {

struct PatchUnfoldParams {
    const void* images;
    __half* out;
    int64_t ldo;
    int64_t chunks;  // B * C * H * W / CH
    int32_t c, h, w, patch;
    int32_t f32;     // images are fp32 (converted to fp16, round to nearest even)
};

template <int CH>
__global__ void __launch_bounds__(256) patch_unfold_kernel(const PatchUnfoldParams p) {
    static_assert(CH == 8 || CH == 4, "chunk of 8 or 4 pixels");
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    if (t >= p.chunks) return;
    const int64_t e = t * CH;  // first pixel of the chunk, in [B][C][H][W] order
    const int xw = static_cast<int>(e % p.w);
    const int64_t r = e / p.w;  // image row index over (b, c, y)
    const int yh = static_cast<int>(r % p.h);
    const int64_t bc = r / p.h;
    const int ch = static_cast<int>(bc % p.c);
    const int64_t b = bc / p.c;
    const int P = p.patch;
    const int gw = p.w / P, gh = p.h / P;
    const int64_t row = (b * gh + yh / P) * gw + xw / P;
    const int64_t col = static_cast<int64_t>(ch) * P * P + (yh % P) * P + (xw % P);
    __half* dst = p.out + row * p.ldo + col;
    if constexpr (CH == 8) {
        uint4 o;
        if (p.f32) {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.images) + e);
            const float4 a = __ldg(src), c = __ldg(src + 1);
            __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            __half2 h2 = __floats2half2_rn(c.x, c.y), h3 = __floats2half2_rn(c.z, c.w);
            o.x = *reinterpret_cast<uint32_t*>(&h0);
            o.y = *reinterpret_cast<uint32_t*>(&h1);
            o.z = *reinterpret_cast<uint32_t*>(&h2);
            o.w = *reinterpret_cast<uint32_t*>(&h3);
        } else {
            o = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(p.images) + e));
        }
        *reinterpret_cast<uint4*>(dst) = o;
    } else {
        uint2 o;
        if (p.f32) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.images) + e));
            __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            o.x = *reinterpret_cast<uint32_t*>(&h0);
            o.y = *reinterpret_cast<uint32_t*>(&h1);
        } else {
            o = __ldg(reinterpret_cast<const uint2*>(static_cast<const __half*>(p.images) + e));
        }
        *reinterpret_cast<uint2*>(dst) = o;
    }
}

}  // namespace rpfq
