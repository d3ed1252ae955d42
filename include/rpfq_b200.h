/*
 * rpfq_b200.h — C ABI of the B200 (sm_100a) packed complex-phase linear layer.
 *
 * Drop-in boundary for the hot path of RPFQ-ViT (Fmylalala/RPFQ-review): the
 * widely-linear layer y = U x + W conj(x) whose U and W are stored as
 * residual stages of 2-bit phase codes plus fp16 magnitude scales, in the
 * exporter's packed layout. All entry points take plain device pointers and
 * sizes, launch on the given CUDA stream, never synchronise the device and
 * never allocate (the caller owns every buffer). They return RPFQ_OK or a
 * nonzero status; rpfq_last_error() gives the message (thread-local).
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   - QATLinearComplexPhase.forward           RPFQ-ViT-main/quant_models/quant_i.py:513-554
 *   - torch.ops.quant.QATLinearComplexPhaseV2_forward
 *                                             RPFQ-ViT-main/quant_models/kernel.py:599-605
 *   - wideLinear / wideLinearReference        RPFQ-ViTAndroid/app/src/main/cpp/ops/phase_linear.h:59-68
 *   - buildFusedWideLinearCache               RPFQ-ViTAndroid/app/src/main/cpp/kernels/phase_linear_cache.h:30-31
 *   - ActivationQuantSTE.forward              RPFQ-ViT-main/quant_models/quant_i.py:442-455
 *   - save_quantized_linear (exporter packing) RPFQ-ViTApple/scripts/export_rpfq_vit_to_mlx.py:384-423
 *   - VisionAwareActivationQuantizer.forward  RPFQ-ViT-main/quant_models/quant_rpfq_vit_vision.py:26-171
 *
 * Layout conventions (unchanged from the reference):
 *   real Linear(in = K, out = N) = complex map k_c = K/2 -> n_c = N/2;
 *   x[:, 0:k_c] = Re(x), x[:, k_c:K] = Im(x); y likewise with n_c.
 *   Packed plane (one residual stage of U or W):
 *     codes       uint8 [n_cp, k_cp * code_bits / 8], codes LSB-first
 *                 (2-bit codebook 0:-1, 1:+1, 2:-i, 3:+i)
 *     gamma_real  fp16  [n_cp, k_cp / 256]   (1 / scale, per row and 256-column block)
 *     gamma_imag  fp16  [n_cp, k_cp / 256]
 *   with n_cp, k_cp the complex dims rounded up to 256
 *   (RPFQ-ViTApple/scripts/export_rpfq_vit_to_mlx.py:148-159,189-224,384-423).
 */
#ifndef RPFQ_B200_H
#define RPFQ_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* rpfq_stream_t; /* a cudaStream_t; NULL = the legacy default stream */

enum {
    RPFQ_OK = 0,
    RPFQ_ERR_INVALID = 1,     /* bad argument (shape, alignment, null pointer)        */
    RPFQ_ERR_UNSUPPORTED = 2, /* valid but not supported on this path                 */
    RPFQ_ERR_CUDA = 3,        /* a CUDA runtime call failed (message has the details) */
    RPFQ_ERR_DEVICE = 4       /* a kernel reported a device-side error (bounded wait) */
};

enum { RPFQ_ACT_NONE = 0, RPFQ_ACT_GELU = 1 };               /* epilogue activation */
/* RpfqGemmArgs.flags / RpfqWideLinearArgs.flags: fp32 output, fp32 residual,
 * fp32 bias (the same bias values widened once by the caller: the epilogue
 * then adds them without a conversion per element). */
enum { RPFQ_GEMM_OUT_F32 = 1, RPFQ_GEMM_RESIDUAL_F32 = 2, RPFQ_GEMM_BIAS_F32 = 4 };
enum { RPFQ_ROUND_NEAREST_EVEN = 0, RPFQ_ROUND_TIES_AWAY = 1 }; /* fp32 -> fp16 of K1 */

/* One residual stage of U or W. Replaces PhaseLinearParams
 * (RPFQ-ViTAndroid/app/src/main/cpp/ops/phase_linear.h:15-26). */
typedef struct RpfqPhasePlane {
    const uint8_t* codes;
    const uint16_t* gamma_real; /* fp16 bits */
    const uint16_t* gamma_imag; /* fp16 bits */
} RpfqPhasePlane;

/* A packed widely-linear layer. Replaces WideLinearParams
 * (RPFQ-ViTAndroid/app/src/main/cpp/ops/phase_linear.h:28-40). */
typedef struct RpfqPackedLinear {
    int32_t n_c, k_c;   /* complex output / input dims (unpadded)           */
    int32_t n_cp, k_cp; /* padded dims, multiples of 256                    */
    int32_t stages;     /* residual stages per U and per W, 1..4            */
    int32_t code_bits;  /* 2 (reference codebook); 3 or 4 (uniform phases)  */
    RpfqPhasePlane u[4];
    RpfqPhasePlane w[4];
} RpfqPackedLinear;

/* K1 — decode a packed layer into the dense fp16 coefficient matrix
 * dense[2 n_c, 2 k_c] = [[rr, ir], [ri, ii]] (row-major), the B operand of
 * rpfq_gemm_sm100. Bit-exact with the reference's fp16 coefficient cache:
 * buildFusedWideLinearCache, RPFQ-ViTAndroid/app/src/main/cpp/kernels/phase_linear_cache.cpp:84-133
 * (rounding = RPFQ_ROUND_TIES_AWAY reproduces its floatToHalfBits, :91-115;
 * RPFQ_ROUND_NEAREST_EVEN is the IEEE conversion). Runs once per layer. */
int rpfq_prepack_sm100(const RpfqPackedLinear* layer, uint16_t* dense_out, int32_t rounding,
                       rpfq_stream_t stream);

/* K2 — y[m, n] = act(x[m, :] . w[n, :] + bias[n]) + residual[m, n], fp16
 * operands, fp32 accumulation on tcgen05 tensor cores, fp16 or fp32 output
 * and residual (flags). Replaces the dense product F.linear(x, q_weight, bias)
 * of QATLinearComplexPhase.forward (RPFQ-ViT-main/quant_models/quant_i.py:554)
 * and the F.linear call of QATLinearComplexPhaseV2_autograd.forward
 * (kernel.py:573). y may alias residual (in-place residual add); the residual
 * has the output's dtype (RPFQ_GEMM_RESIDUAL_F32 iff RPFQ_GEMM_OUT_F32).
 * Requirements: k % 8 == 0, n % 8 == 0, ldx % 8 == 0, ldy % 8 == 0,
 * ldr % 8 == 0, 16-byte aligned x / w / y / bias / residual.
 * Split-K: when few output tiles would leave most SMs idle (small m), the
 * K dimension of each tile is split over a cluster of up to 8 CTAs whose
 * fp32 partials meet in `workspace` (device memory, 16-byte aligned, at
 * least rpfq_gemm_workspace_bytes(m, n, k) bytes; calls that run
 * concurrently need their own). Stream-K: when the 256 x 256 tiles of CTA
 * pairs fill at least one wave but not a whole number of waves, the k-blocks
 * of the last one to two waves are shared out evenly over all pairs and a
 * tile cut between two pairs meets in the same workspace; its last 8192
 * bytes are flag words that must be zero before the first call (allocate the
 * workspace zeroed) and that every call which completes without a device
 * error leaves zero. rpfq_gemm_workspace_bytes(0, 0, 0) is a size that fits
 * every shape. With workspace == NULL the call neither splits nor uses
 * stream-K. split_k: 0 = automatic, 1 = never, 2..8 = that many splits
 * (needs the workspace). Partials are summed in a fixed order: results are
 * deterministic for a given shape. RPFQ_STREAM_K=0 in the environment turns
 * the stream-K tail off. Narrow tail (no workspace needed, takes precedence):
 * when the CTA-pair tiles leave a last wave at most half full, those tiles
 * are cut into 2 or 4 column pieces dealt out over the idle pairs; every
 * output is still accumulated over all of K in one pass, so the results are
 * those of whole tiles. RPFQ_NARROW_TAIL=0 turns it off. */
typedef struct RpfqGemmArgs {
    const uint16_t* x;        /* fp16 [m, k], row stride ldx (elements)                */
    int64_t ldx;
    const uint16_t* w;        /* fp16 [n, k], contiguous                                */
    const void* bias;         /* fp16 [n] (fp32 with RPFQ_GEMM_BIAS_F32) or NULL         */
    const void* residual;     /* [m, n] fp16 (fp32 with RPFQ_GEMM_RESIDUAL_F32) or NULL */
    int64_t ldr;
    void* y;                  /* [m, n] fp16 (fp32 with RPFQ_GEMM_OUT_F32), stride ldy  */
    int64_t ldy;
    int64_t m;
    int32_t n, k;
    int32_t activation;       /* RPFQ_ACT_NONE or RPFQ_ACT_GELU (erf)                   */
    int32_t block_n;          /* 0 = automatic; else 128 or 256                         */
    int32_t flags;            /* RPFQ_GEMM_OUT_F32 | RPFQ_GEMM_RESIDUAL_F32 | RPFQ_GEMM_BIAS_F32 */
    int32_t cta_pair;         /* 0 = automatic; 1 = one CTA per tile; 2 = CTA pairs      */
    int32_t split_k;          /* 0 = automatic; 1 = off; 2..8 = K splits per tile       */
    int32_t reserved;
    void* workspace;          /* split-K / stream-K partials and flags, or NULL         */
    uint64_t workspace_bytes;
} RpfqGemmArgs;
int rpfq_gemm_sm100(const RpfqGemmArgs* args, rpfq_stream_t stream);
/* Workspace bytes that rpfq_gemm_sm100 (split_k = 0) uses for an m x n x k
 * product on the current device (0: it does not split); m == 0 returns the
 * largest amount any shape uses, so one buffer of that size serves every
 * call on a stream. */
uint64_t rpfq_gemm_workspace_bytes(int64_t m, int32_t n, int32_t k);

/* The tile plan rpfq_gemm_sm100 would run for these arguments (validated the
 * same way; nothing is launched and no memory is touched). A diagnostic with
 * no counterpart in the reference: benchmarks and tests read which schedule
 * a shape takes. */
typedef struct RpfqGemmPlan {
    int32_t block_n;         /* tile width: 128 or 256                                    */
    int32_t cta_pair;        /* 1: one CTA per 128-row tile, 2: CTA pairs, 256-row tiles  */
    int32_t split_k;         /* K splits per tile (1: none)                               */
    int32_t stream_k_tiles;  /* tiles of the stream-K tail (0: whole tiles only)          */
    int32_t units;           /* persistent CTAs / CTA pairs (split-K: tiles)             */
    int32_t tiles;           /* output tiles                                              */
    int32_t tail_tiles;      /* narrow tail: last-wave tiles cut into column pieces      */
    int32_t pieces;          /* narrow tail: pieces per such tile (0: none; 2 or 4)      */
} RpfqGemmPlan;
int rpfq_gemm_plan_sm100(const RpfqGemmArgs* args, RpfqGemmPlan* plan);

/* Activation quantization of a complex input (per row, Re and Im halves
 * separately), fp16 in / fp16 out. Replaces ActivationQuantSTE.forward
 * (RPFQ-ViT-main/quant_models/quant_i.py:442-455). x and xq may alias.
 * num_bits in 2..8; k = 2 k_c real columns. */
int rpfq_act_quant_sm100(const uint16_t* x, int64_t ldx, uint16_t* xq, int64_t ldq, int64_t m, int32_t k,
                         int32_t num_bits, rpfq_stream_t stream);

/* Patch unfold of the ViT / DeiT input: images [batch, channels, height,
 * width] (fp16, or fp32 with images_f32 != 0, contiguous) -> fp16 rows
 * patches[b * gh * gw + i * gw + j][c * patch^2 + y * patch + x] =
 * image[b][c][i * patch + y][j * patch + x], the input of the patch-embedding
 * GEMM (row stride ldp >= channels * patch^2, a multiple of 8, or of 4 when
 * patch is not a multiple of 8). Replaces the
 * reference's patchify_tensor (RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:
 * 125-134), the CHW patch order of Conv2d(C, d, patch, stride patch) weights
 * flattened to [d, C patch^2]. patch must be a multiple of 4 (ViT / DeiT 16,
 * Swin 4) dividing height and width; both pointers 16-byte aligned. */
int rpfq_patch_unfold_sm100(const void* images, int32_t images_f32, int64_t batch, int32_t channels,
                            int32_t height, int32_t width, int32_t patch, uint16_t* patches, int64_t ldp,
                            rpfq_stream_t stream);

/* LayerNorm of an fp32 residual stream row (d = 96, 192, 384, 768, 1024, 1536
 * or 3072: the ViT / DeiT / Swin widths and Swin's patch-merging 4C) into the
 * fp16 input of the next packed GEMM; with act_bits > 0 the activation
 * quantization of that GEMM's complex input (ActivationQuantSTE,
 * RPFQ-ViT-main/quant_models/quant_i.py:442-455) is applied in the same pass.
 * Replaces the LayerNorm -> quantizer pair in front of the reference's
 * complex linears (timm Block norm1 / norm2; Android ops/layernorm.cpp:8). */
int rpfq_layernorm_sm100(const float* x, int64_t ldx, const uint16_t* weight, const uint16_t* bias, uint16_t* y,
                         int64_t ldy, int64_t m, int32_t d, float eps, int32_t act_bits, rpfq_stream_t stream);

/* rpfq_layernorm_sm100 with a row gather: output row r is the normalized
 * input row rows[r] (int32 [m], device memory; x has x_rows rows). Lets a
 * token permutation (a Swin window partition with its cyclic shift) ride on
 * the LayerNorm pass. An index outside [0, x_rows) leaves its output row
 * untouched and records code 901 in the device error word. */
int rpfq_layernorm_rows_sm100(const float* x, int64_t ldx, int64_t x_rows, const int32_t* rows,
                              const uint16_t* weight, const uint16_t* bias, uint16_t* y, int64_t ldy, int64_t m,
                              int32_t d, float eps, int32_t act_bits, rpfq_stream_t stream);

/* The LayerNorm pass with every row source and output it offers; the two
 * entry points above are special cases. Row sources (one per output row):
 *   plain      x[r]
 *   rows       x[rows[r]] (as rpfq_layernorm_rows_sm100)
 *   merge_side > 0: Swin PatchMerging (the swin stages' downsample in front of
 *              the packed `reduction` linear): output row r is token (i, j) of
 *              image r / (side/2)^2 and concatenates the d/4-wide rows
 *              (2i, 2j), (2i+1, 2j), (2i, 2j+1), (2i+1, 2j+1) of that image's
 *              [side, side] grid in x (torch.cat of the four strided slices);
 *              d % 16 == 0, x_rows >= images * side^2
 *   add        x[r] + add[add_rows[r]] (add_rows NULL: add[r]): a row-permuted
 *              residual add, e.g. Swin's window reverse + un-shift + residual
 *              of the attention branch; needs y32 with y32_prenorm, which then
 *              receives the updated row (y32 == x: in place). An index outside
 *              [0, add_bound) records code 902.
 * Outputs: y (fp16, normalized, activation-quantized with act_bits > 0)
 * and / or y32 (fp32: the normalized row, or with y32_prenorm the row before
 * normalization). y32 may alias x only with the plain row mapping. */
typedef struct RpfqLayerNormArgs {
    const float* x;           /* fp32 [x_rows, ldx] */
    int64_t ldx;
    int64_t x_rows;
    const int32_t* rows;      /* optional gather */
    const float* add;         /* optional row-permuted addend [add_bound, ld_add] */
    int64_t ld_add;
    int64_t add_bound;
    const int32_t* add_rows;  /* optional indices into add */
    const uint16_t* weight;   /* fp16 [d] */
    const uint16_t* bias;     /* fp16 [d] */
    uint16_t* y;              /* fp16 [m, ldy] or NULL */
    int64_t ldy;
    float* y32;               /* fp32 [m, ldy32] or NULL */
    int64_t ldy32;
    int64_t m;
    int32_t d;
    float eps;
    int32_t act_bits;
    int32_t merge_side;
    int32_t y32_prenorm;
    int32_t reserved;
} RpfqLayerNormArgs;
int rpfq_layernorm_ex_sm100(const RpfqLayerNormArgs* args, rpfq_stream_t stream);

/* Whole layer — QATLinearComplexPhase.forward on packed weights
 * (RPFQ-ViT-main/quant_models/quant_i.py:513-554; Android wideLinear,
 * phase_linear.cpp:209-258): optional activation quantization, then the
 * tcgen05 GEMM over the dense coefficients `dense` (from rpfq_prepack_sm100),
 * bias and optional GELU / residual in the epilogue. With dense == NULL and
 * m <= 256 (2-bit codes, n_c and k_c multiples of 8) the layer runs the fused
 * decode path instead: the packed codes are TMA-staged and unpacked in shared
 * memory into the MMA operand tiles, so only the packed weights are read.
 * When act_bits > 0, `scratch` must hold m * 2 k_c fp16 values (the quantized
 * activations); otherwise it may be NULL. */
typedef struct RpfqWideLinearArgs {
    const RpfqPackedLinear* layer; /* shapes; the planes are read when dense == NULL */
    const uint16_t* dense;         /* fp16 [2 n_c, 2 k_c] from rpfq_prepack_sm100, or NULL (m <= 256) */
    const uint16_t* x;             /* fp16 [m, 2 k_c], row stride ldx */
    int64_t ldx;
    const void* bias;              /* fp16 [2 n_c] (fp32 with RPFQ_GEMM_BIAS_F32) or NULL */
    const void* residual;          /* [m, 2 n_c] or NULL, row stride ldr (fp32 with RPFQ_GEMM_RESIDUAL_F32) */
    int64_t ldr;
    void* y;                       /* [m, 2 n_c], row stride ldy (fp32 with RPFQ_GEMM_OUT_F32) */
    int64_t ldy;
    int64_t m;
    int32_t act_bits;              /* 0 = no activation quantization, else 2..8 */
    int32_t activation;            /* RPFQ_ACT_NONE or RPFQ_ACT_GELU */
    uint16_t* scratch;             /* fp16 [m, 2 k_c] when act_bits > 0 */
    int32_t flags;                 /* RPFQ_GEMM_OUT_F32 | RPFQ_GEMM_RESIDUAL_F32 | RPFQ_GEMM_BIAS_F32 */
    int32_t split_k;               /* as RpfqGemmArgs.split_k (dense path) */
    void* workspace;               /* as RpfqGemmArgs.workspace, or NULL */
    uint64_t workspace_bytes;
} RpfqWideLinearArgs;
int rpfq_wide_linear_sm100(const RpfqWideLinearArgs* args, rpfq_stream_t stream);

/* Multi-head self-attention for short sequences: qkv is the qkv GEMM output
 * [images * tokens, 3 * heads * 64] fp16 (row = token: q heads, k heads,
 * v heads), out[images * tokens, ldo] receives softmax(q k^T / 8) v with the
 * heads concatenated (the proj GEMM's input). tokens <= 256 (all keys in one
 * tensor-core tile), head_dim = 64. Replaces the attention of the timm blocks
 * the reference models wrap (RPFQ-ViT-main/quant_models/quant_rpfq_vit.py,
 * quant_rpfq_deit.py; runtime restatement
 * RPFQ-ViTApple/scripts/audit_rpfq_vit_ios_parity.py:612-614). */
int rpfq_attention_sm100(const uint16_t* qkv, int64_t images, int32_t tokens, int32_t heads, int32_t head_dim,
                         uint16_t* out, int64_t ldo, rpfq_stream_t stream);

/* Swin window attention (7x7 windows, head dim 32): for every window w and
 * head h, softmax(q k^T / sqrt(32) + bias) v over the window's 49 tokens, the
 * attention of the timm Swin blocks the reference wraps
 * (RPFQ-ViT-main/quant_models/quant_rpfq_swin.py:64-91). qkv is the qkv
 * GEMM output in window order, [windows * 49, 3 * 32 * heads] fp16 (row =
 * token: q heads, k heads, v heads); out[windows * 49, ldo] receives the heads
 * concatenated (the proj GEMM's input). bias_mask is fp32
 * [bm_windows, heads, 16, 49, 4]: log2(e) * (relative position bias + shift
 * mask) of query row i and key column j at [.., j / 4, i, j % 4], -inf for
 * the padding keys 49..63; window w uses entry w % bm_windows (1 for unshifted
 * blocks, the windows per image for shifted ones). */
int rpfq_window_attention_sm100(const uint16_t* qkv, int64_t windows, int32_t heads, int32_t head_dim,
                                int32_t window_tokens, const float* bias_mask, int32_t bm_windows, uint16_t* out,
                                int64_t ldo, rpfq_stream_t stream);

/* Vision-aware activation quantization of `images` x `tokens` rows of fp16
 * x[row] = [Re | Im] (k = 2 k_c columns, k_c a multiple of 8) into xq (may
 * alias x): the reference's VisionAwareActivationQuantizer.forward
 * (RPFQ-ViT-main/quant_models/quant_rpfq_vit_vision.py:26-171). With
 * tokens = 1 + g*g the ceil(g*g * salient_ratio) most salient patch tokens per
 * image (energy and 4-neighbour contrast score) and, if protect_cls_token,
 * the CLS token keep per-token int8 scales; the other tokens share one
 * per-image scale from their amax times background_clip_ratio. Any other
 * token count quantizes every row with its own int8 scale, like the
 * reference's fallback. mask_out (optional, [images * tokens]) receives 1 for
 * salient rows. The ratios are doubles as in the reference (Python floats);
 * saliency grids up to 128 x 128 patches. With a saliency grid the call
 * needs `workspace`: rpfq_vision_workspace_bytes(images, tokens) bytes of
 * device memory, 16-byte aligned (per-token statistics and scales); it may be
 * NULL otherwise. */
uint64_t rpfq_vision_workspace_bytes(int64_t images, int32_t tokens);
int rpfq_vision_act_quant_sm100(const uint16_t* x, int64_t ldx, uint16_t* xq, int64_t ldq, int64_t images,
                                int32_t tokens, int32_t k, double salient_ratio, double background_clip_ratio,
                                double energy_score_weight, int32_t protect_cls_token, uint8_t* mask_out,
                                void* workspace, uint64_t workspace_bytes, rpfq_stream_t stream);

/* Output buffers of one residual stage of U or W for rpfq_pack_linear_sm100:
 * codes uint8 [n_cp, k_cp/4], gammas fp16 [n_cp, k_cp/256]. */
typedef struct RpfqPhasePlaneOut {
    uint8_t* codes;
    uint16_t* gamma_real;
    uint16_t* gamma_imag;
} RpfqPhasePlaneOut;

/* Device memory rpfq_pack_linear_sm100 needs as workspace for a layer with
 * complex dims (n_c, k_c): the four fp32 residual planes plus the partial
 * sums of the scale reductions. 0 for non-positive dims. */
uint64_t rpfq_pack_workspace_bytes(int32_t n_c, int32_t k_c);

/* The exporter's packing on the device: float weight [2 n_c, 2 k_c] (fp32,
 * row stride ldw elements) -> `stages` residual stages of 2-bit axial codes and
 * fp16 gammas for U and for W (u_out[0..stages), w_out[0..stages)), padding
 * included, bit-identical to the reference exporter: save_quantized_linear /
 * quantize_complex_weight / phase_quantize_axis,
 * RPFQ-ViTApple/scripts/export_rpfq_vit_to_mlx.py:189-224,257-289,317-333,384-423.
 * The bias is not touched (the exporter stores fp16(bias)). The scale of each
 * axis is a mean over the whole matrix, reduced on the device: no host sync.
 * workspace: rpfq_pack_workspace_bytes(n_c, k_c) bytes, 16-byte aligned. */
int rpfq_pack_linear_sm100(const float* weight, int64_t ldw, int32_t n_c, int32_t k_c, int32_t stages,
                           const RpfqPhasePlaneOut* u_out, const RpfqPhasePlaneOut* w_out, void* workspace,
                           uint64_t workspace_bytes, rpfq_stream_t stream);

/* Allocation-free variant of rpfq_wide_linear_sm100 — no counterpart in the
 * reference. For callers that cannot allocate device memory when they run a
 * layer (server request paths that must not call cudaMalloc / cudaFree, which
 * can synchronise the whole device, and plugin or embedded hosts that give a
 * library no allocator):
 * with act_bits > 0 the quantized activations go to an 8 MiB scratch array
 * built into the library (m * 2 k_c fp16 values at most; larger m is rejected
 * with RPFQ_ERR_INVALID), args->scratch is ignored, and nothing is allocated.
 * Every GPU that loads the library holds the array until the process exits.
 * The first call on a device looks up the array's device address (set-up,
 * once per device); make that first call before any stream capture. All calls
 * share the array: calls that overlap on the GPU race on it. */
int rpfq_wide_linear_noalloc_sm100(const RpfqWideLinearArgs* args, rpfq_stream_t stream);

/* Message of the last failed call on this host thread ("" if none). */
const char* rpfq_last_error(void);

/* Reads and clears the device-side error word of the current device (a
 * bounded wait inside a kernel that ran out records its site there).
 * Synchronises the device. *code_out = 0 when no kernel reported an error. */
int rpfq_device_error(int32_t* code_out);

/* Library ABI version (major * 100 + minor). */
int rpfq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* RPFQ_B200_H */
