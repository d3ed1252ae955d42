// C ABI of the B200 packed complex-phase linear layer (declared in
// include/rpfq_b200.h). Host-side validation, TMA descriptor encoding and
// launches; the kernels live in the included .cuh files. One translation unit
// so that all kernels share the device error word without relocatable code.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/rpfq_b200.h"
#include "actquant.cuh"
#include "attention.cuh"
#include "window_attention.cuh"
#include "decode_gemm.cuh"
#include "embed.cuh"
#include "gemm.cuh"
#include "layernorm.cuh"
#include "pack.cuh"
#include "vision_quant.cuh"
#include "prepack.cuh"

namespace rpfq {

// Device-side error word: the first bounded wait that runs out records its
// site code here (see ptx.cuh wait_bar). Read and cleared by rpfq_device_error.
__device__ int g_device_error;

namespace {

constexpr int kMaxDevices = 64;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define RPFQ_CUDA(call)                                                                                    \
    do {                                                                                                   \
        cudaError_t e_ = (call);                                                                           \
        if (e_ != cudaSuccess) return fail(RPFQ_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

// ---------------------------------------------------------------- per-device state
struct DeviceState {
    std::once_flag once;
    int status = RPFQ_OK;
    std::string error;
    int sm_count = 0;
    int* err_word = nullptr;  // device address of g_device_error
};
DeviceState g_dev[kMaxDevices];

template <int BN, bool OUT_F32, int RES, bool PAIR = false>
cudaError_t configure_one() {
    return cudaFuncSetAttribute(gemm_f16_sm100_kernel<BN, OUT_F32, RES, PAIR>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN, RES, PAIR>::SMEM_BYTES);
}

template <int BN>
cudaError_t configure_gemm() {
    cudaError_t e = cudaSuccess;
    for (cudaError_t r : {configure_one<BN, false, 0>(), configure_one<BN, true, 0>(), configure_one<BN, false, 1>(),
                          configure_one<BN, true, 1>(), configure_one<BN, false, 2>(), configure_one<BN, true, 2>()})
        if (e == cudaSuccess) e = r;
    if constexpr (BN == 256) {
        for (cudaError_t r :
             {configure_one<BN, false, 0, true>(), configure_one<BN, true, 0, true>(), configure_one<BN, false, 1, true>(),
              configure_one<BN, true, 1, true>(), configure_one<BN, false, 2, true>(), configure_one<BN, true, 2, true>()})
            if (e == cudaSuccess) e = r;
    }
    return e;
}

// Per-device set-up, done once with that device current: SM count, device
// error word address, kernel shared-memory limits, arch check.
int device_state(DeviceState** out) {
    int dev = 0;
    RPFQ_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(RPFQ_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    DeviceState& st = g_dev[dev];
    std::call_once(st.once, [&st, dev]() {
        cudaDeviceProp prop;
        cudaError_t e = cudaGetDeviceProperties(&prop, dev);
        if (e != cudaSuccess) {
            st.status = RPFQ_ERR_CUDA;
            st.error = std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e);
            return;
        }
        if (prop.major != 10 || prop.minor != 0) {
            st.status = RPFQ_ERR_UNSUPPORTED;
            st.error = "this library is built for sm_100a (B200); device is sm_" + std::to_string(prop.major) +
                       std::to_string(prop.minor);
            return;
        }
        st.sm_count = prop.multiProcessorCount;
        void* addr = nullptr;
        e = cudaGetSymbolAddress(&addr, g_device_error);
        if (e == cudaSuccess) e = configure_gemm<256>();
        if (e == cudaSuccess) e = configure_gemm<128>();
        if (e != cudaSuccess) {
            st.status = RPFQ_ERR_CUDA;
            st.error = std::string("device set-up: ") + cudaGetErrorString(e);
            return;
        }
        st.err_word = static_cast<int*>(addr);
    });
    if (st.status != RPFQ_OK) return fail(st.status, "%s", st.error.c_str());
    *out = &st;
    return RPFQ_OK;
}

// ---------------------------------------------------------------- TMA descriptors
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out) {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    static std::string err;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
            err = "cuTensorMapEncodeTiled is not available from the driver";
            return;
        }
        fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) return fail(RPFQ_ERR_CUDA, "%s", err.c_str());
    *out = fn;
    return RPFQ_OK;
}

// Row-major matrix [rows, cols] of fp16 (esize 2) or fp32 (esize 4), row
// stride ld elements, box [box_rows, box_cols], 128-B swizzle.
int make_tmap_f16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                  int box_cols, int esize = 2, bool swizzle = true) {
    EncodeTiledFn fn;
    int rc = encode_fn(&fn);
    if (rc) return rc;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(RPFQ_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for a [%lld x %lld] matrix", (int)r,
                    (long long)rows, (long long)cols);
    return RPFQ_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Programmatic dependent launch for the per-layer kernels (on unless the
// environment sets RPFQ_PDL=0): a kernel's launch and prologue overlap the
// tail of its predecessor in the stream; every such kernel calls pdl_wait()
// before touching global memory.
bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("RPFQ_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          int cluster_x, Args... args) {
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster_x;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// x [m][2][k_c] view of the fp16 activations (Re half, Im half), box {64, 1, 128}, 128-B swizzle.
int make_tmap_x_halves(CUtensorMap* m, const void* base, int64_t rows, int32_t k_c, int64_t ld) {
    EncodeTiledFn fn;
    int rc = encode_fn(&fn);
    if (rc) return rc;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(k_c), 2, static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(k_c) * 2, static_cast<cuuint64_t>(ld) * 2};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RPFQ_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for the x halves view", (int)r);
    return RPFQ_OK;
}

// packed codes [rows][bytes_per_row] uint8, box {16 bytes, box_rows}, no swizzle.
int make_tmap_codes(CUtensorMap* m, const void* base, int64_t rows, int64_t bytes_per_row, int box_rows) {
    EncodeTiledFn fn;
    int rc = encode_fn(&fn);
    if (rc) return rc;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(bytes_per_row), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(bytes_per_row)};
    cuuint32_t box[2] = {16, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RPFQ_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for packed codes", (int)r);
    return RPFQ_OK;
}

// ---------------------------------------------------------------- GEMM launch
// Stream-K tail length for `tiles` tiles over `units` co-resident units: the
// last wave plus one full wave (so every unit's share is at least one tile),
// when the last wave is at most 85 % full; 0 = data-parallel only.
int sk_tail(int64_t tiles, int units) {
    if (units <= 0 || tiles <= units || tiles % units == 0) return 0;
    const double fill = static_cast<double>(tiles % units) / units;
    if (fill > 0.85) return 0;
    return static_cast<int>(tiles - (tiles / units - 1) * units);
}

// Narrow tail for `tiles` tiles over `units` units: when the last wave is at
// most half full, its tiles are cut into pieces (4 of BN / 4 columns, or 2 of
// BN / 2 when four would exceed the units); 0 = none.
int narrow_pieces(int64_t tiles, int units) {
    if (units <= 0 || tiles < units) return 0;
    const int64_t rem = tiles % units;
    if (rem == 0 || 2 * rem > units) return 0;
    return 4 * rem <= units ? 4 : 2;
}

// Narrow tail on by default; RPFQ_NARROW_TAIL=0 turns it off (measurement).
bool narrow_tail_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("RPFQ_NARROW_TAIL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Workspace: split-K / stream-K partials, then the stream-K flag words.
uint64_t ws_partial_bytes(const DeviceState* st) { return static_cast<uint64_t>(st->sm_count) * 128u * 256u * 4u; }
constexpr uint64_t kSkFlagBytes = 8192;  // >= SMs x 8 epilogue warps x 4 B

// Units of the persistent grid that are resident at once: CTA pairs (queried
// once per device and kernel variant) or CTAs (one per SM). 0 on error.
template <int BN, bool OUT_F32, int RES, bool PAIR>
int gemm_units(DeviceState* st) {
    using C = GemmCfg<BN, RES, PAIR>;
    if constexpr (!PAIR) {
        return st->sm_count;
    } else {
        static int max_pairs[kMaxDevices] = {};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
        if (max_pairs[dev] == 0) {
            cudaLaunchConfig_t q = {};
            cudaLaunchAttribute qa[1];
            qa[0].id = cudaLaunchAttributeClusterDimension;
            qa[0].val.clusterDim.x = 2;
            qa[0].val.clusterDim.y = 1;
            qa[0].val.clusterDim.z = 1;
            q.gridDim = dim3(st->sm_count);
            q.blockDim = dim3(C::THREADS);
            q.dynamicSmemBytes = C::SMEM_BYTES;
            q.attrs = qa;
            q.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, gemm_f16_sm100_kernel<BN, OUT_F32, RES, true>, &q) != cudaSuccess) {
                cudaGetLastError();
                return 0;
            }
            max_pairs[dev] = n > 0 ? n : 1;
        }
        return max_pairs[dev];
    }
}

// Stream-K tail of a launch: only when every unit of the grid can be resident
// together (owners wait for their peers).
template <int BN, bool OUT_F32, int RES, bool PAIR>
int gemm_sk_tiles(int64_t tiles, DeviceState* st) {
    const int units = gemm_units<BN, OUT_F32, RES, PAIR>(st);
    if (units <= 0 || (PAIR ? 2 * units : units) > st->sm_count) return 0;
    return sk_tail(tiles, units);
}

template <int BN, bool OUT_F32, int RES, bool PAIR>
int launch_gemm(const RpfqGemmArgs* a, DeviceState* st, cudaStream_t stream, int splits, bool stream_k,
                bool narrow, RpfqGemmPlan* dry) {
    using C = GemmCfg<BN, RES, PAIR>;
    constexpr int CW = OUT_F32 ? 32 : 64;   // output / residual columns per 128-B step
    constexpr int ESZ = OUT_F32 ? 4 : 2;
    GemmParams p;
    p.bias = a->bias;
    p.bias_f32 = (a->flags & RPFQ_GEMM_BIAS_F32) ? 1 : 0;
    p.residual = a->residual;
    p.ldr = a->ldr;
    p.m = a->m;
    p.n = a->n;
    p.k = a->k;
    p.activation = a->activation;
    p.splits = PAIR ? 1 : splits;
    p.ws = static_cast<float*>(a->workspace);
    p.y = a->y;
    p.ldy = a->ldy;
    p.err = st->err_word;
    p.sk_tiles = 0;
    p.sk_flags = stream_k ? reinterpret_cast<int*>(static_cast<uint8_t*>(a->workspace) + ws_partial_bytes(st))
                          : nullptr;
    p.tail_tiles = 0;
    p.pieces = 0;
    const int64_t tiles = ((a->m + C::TILE_M - 1) / C::TILE_M) * ((a->n + BN - 1) / BN);
    if constexpr (PAIR) {
        // narrow tail first (no exchange between units); stream-K otherwise
        if (narrow && splits <= 1) {
            const int units = gemm_units<BN, OUT_F32, RES, true>(st);
            p.pieces = narrow_pieces(tiles, units);
            if (p.pieces) p.tail_tiles = static_cast<int32_t>(tiles % units);
        }
    }
    if (stream_k && !p.pieces) p.sk_tiles = gemm_sk_tiles<BN, OUT_F32, RES, PAIR>(tiles, st);
    // grid: persistent units (CTA pairs or CTAs, as many as are resident at once; with a
    // stream-K tail exactly that many), or tiles x splits CTAs for split-K
    int units;
    if constexpr (PAIR) {
        const int max_pairs = gemm_units<BN, OUT_F32, RES, true>(st);
        if (max_pairs <= 0) return fail(RPFQ_ERR_CUDA, "rpfq_gemm_sm100: occupancy query for CTA pairs failed");
        units = p.sk_tiles ? max_pairs : static_cast<int>(tiles < max_pairs ? tiles : max_pairs);
    } else if (p.splits > 1) {
        units = static_cast<int>(tiles);
    } else {
        units = p.sk_tiles ? st->sm_count : static_cast<int>(tiles < st->sm_count ? tiles : st->sm_count);
    }
    if (dry) {
        dry->block_n = BN;
        dry->cta_pair = PAIR ? 2 : 1;
        dry->split_k = p.splits;
        dry->stream_k_tiles = p.sk_tiles;
        dry->units = units;
        dry->tiles = static_cast<int32_t>(tiles);
        dry->tail_tiles = p.tail_tiles;
        dry->pieces = p.pieces;
        return RPFQ_OK;
    }
    CUtensorMap tx, tw, ty, tr, twp;
    int rc = make_tmap_f16(&tx, a->x, a->m, a->k, a->ldx, C::BM, C::BK);
    if (!rc) rc = make_tmap_f16(&tw, a->w, a->n, a->k, a->k, C::B_ROWS, C::BK);
    // narrow-tail pieces: BN / pieces columns, half of them per CTA of a pair
    if (!rc && p.pieces) rc = make_tmap_f16(&twp, a->w, a->n, a->k, a->k, C::B_ROWS / p.pieces, C::BK);
    if (!rc) rc = make_tmap_f16(&ty, a->y, a->m, a->n, a->ldy, 32, CW, ESZ);
    // residual: same [32 rows x 128 B] boxes as the output (TMA loads + L2 prefetches)
    if (!rc && RES > 0) rc = make_tmap_f16(&tr, a->residual, a->m, a->n, a->ldr, 32, CW, ESZ);
    if (rc) return rc;
    if (RES == 0) tr = ty;
    if (!p.pieces) twp = tw;
    if constexpr (PAIR) {
        RPFQ_CUDA(launch_kernel(gemm_f16_sm100_kernel<BN, OUT_F32, RES, true>, dim3(2 * units), dim3(C::THREADS),
                                C::SMEM_BYTES, stream, 2, tx, tw, ty, tr, twp, p));
    } else {
        // split-K: one CTA per (tile, split), the splits of a tile in one cluster
        RPFQ_CUDA(launch_kernel(gemm_f16_sm100_kernel<BN, OUT_F32, RES, false>, dim3(units * p.splits),
                                dim3(C::THREADS), C::SMEM_BYTES, stream, p.splits, tx, tw, ty, tr, twp, p));
    }
    return RPFQ_OK;
}

// ---------------------------------------------------------------- split-K choice
constexpr int kMaxSplits = 8;        // portable cluster size
constexpr int kMinSplitKBlocks = 2;  // k-blocks (of 64) per split, automatic choice

// Clusters of `s` one-CTA-per-tile GEMM CTAs that fit on the device at once
// (queried once per device, tile width and s).
template <int BN>
int max_clusters(int s, DeviceState* st) {
    static int cache[kMaxDevices][kMaxSplits + 1] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cache[dev][s] == 0) {
        cudaLaunchConfig_t q = {};
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = s;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        q.gridDim = dim3(s * (st->sm_count / s));
        q.blockDim = dim3(GemmCfg<BN, 0, false>::THREADS);
        q.dynamicSmemBytes = GemmCfg<BN, 0, false>::SMEM_BYTES;
        q.attrs = qa;
        q.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_f16_sm100_kernel<BN, false, 0, false>, &q) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        cache[dev][s] = n > 0 ? n : -1;
    }
    return cache[dev][s] > 0 ? cache[dev][s] : 0;
}

int64_t gemm_tiles(int64_t m, int n, int bn) { return ((m + 127) / 128) * ((n + bn - 1) / bn); }

uint64_t splitk_bytes(int64_t m, int n, int bn, int s) {
    return static_cast<uint64_t>(gemm_tiles(m, n, bn)) * static_cast<uint64_t>(s) * 128u * static_cast<uint64_t>(bn) * 4u;
}

// Residual slots: two (one main-loop stage less) when the main loop is short
// and the epilogue must hide the residual latency itself; one otherwise.
// Split-K reads the residual in its reduction: no staging slots.
template <int BN, bool PAIR>
int launch_gemm_bn(const RpfqGemmArgs* a, DeviceState* st, cudaStream_t stream, int splits, bool sk, bool narrow,
                   RpfqGemmPlan* dry) {
    const bool f32 = (a->flags & RPFQ_GEMM_OUT_F32) != 0;
    const int res = (a->residual == nullptr || splits > 1) ? 0 : (a->k <= 1024 ? 2 : 1);
    if (f32) {
        if (res == 2) return launch_gemm<BN, true, 2, PAIR>(a, st, stream, splits, sk, narrow, dry);
        if (res == 1) return launch_gemm<BN, true, 1, PAIR>(a, st, stream, splits, sk, narrow, dry);
        return launch_gemm<BN, true, 0, PAIR>(a, st, stream, splits, sk, narrow, dry);
    }
    if (res == 2) return launch_gemm<BN, false, 2, PAIR>(a, st, stream, splits, sk, narrow, dry);
    if (res == 1) return launch_gemm<BN, false, 1, PAIR>(a, st, stream, splits, sk, narrow, dry);
    return launch_gemm<BN, false, 0, PAIR>(a, st, stream, splits, sk, narrow, dry);
}

// ---------------------------------------------------------------- K3 fused decode launch
constexpr int64_t kDecodeMaxRows = 256;

template <int RB>
int launch_decode(const RpfqWideLinearArgs* a, const uint16_t* xin, int64_t ldx, DeviceState* st, cudaStream_t stream,
                  int splits_forced) {
    using C = DecodeCfg<RB>;
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr_status[kMaxDevices];
    int dev = 0;
    RPFQ_CUDA(cudaGetDevice(&dev));
    std::call_once(once[dev], [dev]() {
        attr_status[dev] = cudaFuncSetAttribute(decode_gemm_sm100_kernel<RB>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    });
    RPFQ_CUDA(attr_status[dev]);
    const RpfqPackedLinear* L = a->layer;
    CUtensorMap tx;
    DecodeCodeMaps cm;
    std::memset(&cm, 0, sizeof(cm));
    int rc = make_tmap_x_halves(&tx, xin, a->m, L->k_c, ldx);
    DecodeGemmParams p;
    std::memset(&p, 0, sizeof(p));
    for (int s = 0; s < L->stages && !rc; ++s) {
        rc = make_tmap_codes(&cm.plane[s], L->u[s].codes, L->n_cp, L->k_cp / 4, RB);
        if (!rc) rc = make_tmap_codes(&cm.plane[L->stages + s], L->w[s].codes, L->n_cp, L->k_cp / 4, RB);
        p.gamma_re[s] = reinterpret_cast<const __half*>(L->u[s].gamma_real);
        p.gamma_im[s] = reinterpret_cast<const __half*>(L->u[s].gamma_imag);
        p.gamma_re[L->stages + s] = reinterpret_cast<const __half*>(L->w[s].gamma_real);
        p.gamma_im[L->stages + s] = reinterpret_cast<const __half*>(L->w[s].gamma_imag);
    }
    if (rc) return rc;
    p.stages = L->stages;
    p.n_c = L->n_c;
    p.k_c = L->k_c;
    p.n_cp = L->n_cp;
    p.k_cp = L->k_cp;
    p.rows_per_item = RB;
    p.bias = a->bias;
    p.bias_f32 = (a->flags & RPFQ_GEMM_BIAS_F32) ? 1 : 0;
    p.residual = a->residual;
    p.ldr = a->ldr;
    p.y = a->y;
    p.ldy = a->ldy;
    p.m = a->m;
    p.activation = a->activation;
    p.out_f32 = (a->flags & RPFQ_GEMM_OUT_F32) ? 1 : 0;
    p.err = st->err_word;
    const int items = (L->n_c + RB - 1) / RB;
    // Split-K when the row blocks alone leave most SMs idle (fewer than a third
    // of the SMs: ViT-B proj / fc2 at one image, 24 blocks; measured slower for
    // qkv's 72): S CTAs per item (a cluster), at least two k-blocks each, items x
    // S within the SM count, the partials within the caller's workspace.
    const int num_k = (L->k_c + DecodeCfg<RB>::KB - 1) / DecodeCfg<RB>::KB;
    const int nsub = a->m > 128 ? 2 : 1;
    int S = std::min({kMaxSplits, num_k / 2, st->sm_count / items});
    if (S < 2 || splits_forced == 1 || (splits_forced == 0 && 3 * items >= st->sm_count)) S = 1;
    if (splits_forced > 1) S = std::min(splits_forced, num_k);
    const uint64_t part_bytes = static_cast<uint64_t>(items) * S * nsub * 128 * 2 * RB * 4;
    if (S > 1 && (!a->workspace || part_bytes > std::min<uint64_t>(a->workspace_bytes, ws_partial_bytes(st)))) S = 1;
    p.splits = S;
    p.ws = S > 1 ? static_cast<float*>(a->workspace) : nullptr;
    const int grid = S > 1 ? items * S : (items < st->sm_count ? items : st->sm_count);
    RPFQ_CUDA(launch_kernel(decode_gemm_sm100_kernel<RB>, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, stream, S, tx,
                            cm, p));
    return RPFQ_OK;
}

int decode_path(const RpfqWideLinearArgs* a, const uint16_t* xin, int64_t ldx, cudaStream_t stream) {
    const RpfqPackedLinear* L = a->layer;
    if (L->code_bits != 2)
        return fail(RPFQ_ERR_UNSUPPORTED, "fused decode path: 2-bit codes only (decode 3/4-bit layers with rpfq_prepack_sm100)");
    if (a->m > kDecodeMaxRows)
        return fail(RPFQ_ERR_UNSUPPORTED, "fused decode path: m <= %lld rows (got %lld); prepack for larger m",
                    (long long)kDecodeMaxRows, (long long)a->m);
    if (L->k_c % 8 || L->n_c % 8)
        return fail(RPFQ_ERR_UNSUPPORTED, "fused decode path: n_c and k_c must be multiples of 8");
    if (ldx % 8 || a->ldy % 8 || (a->residual && a->ldr % 8) || !aligned16(xin) || !aligned16(a->y) ||
        (a->bias && !aligned16(a->bias)) || (a->residual && !aligned16(a->residual)))
        return fail(RPFQ_ERR_INVALID, "fused decode path: 16-byte aligned pointers and strides required");
    if (a->residual && (((a->flags & RPFQ_GEMM_RESIDUAL_F32) != 0) != ((a->flags & RPFQ_GEMM_OUT_F32) != 0)))
        return fail(RPFQ_ERR_UNSUPPORTED, "fused decode path: the residual must have the output's dtype");
    if (a->split_k < 0 || a->split_k > kMaxSplits)
        return fail(RPFQ_ERR_INVALID, "fused decode path: split_k must be 0..%d (got %d)", kMaxSplits, a->split_k);
    if (a->workspace && !aligned16(a->workspace))
        return fail(RPFQ_ERR_INVALID, "fused decode path: the workspace must be 16-byte aligned");
    for (int s = 0; s < L->stages; ++s) {
        const RpfqPhasePlane* ps[2] = {&L->u[s], &L->w[s]};
        for (const RpfqPhasePlane* pl : ps)
            if (!pl->codes || !pl->gamma_real || !pl->gamma_imag || !aligned16(pl->codes))
                return fail(RPFQ_ERR_INVALID, "fused decode path: stage %d needs 16-byte aligned codes and gammas", s);
    }
    if (a->m == 0) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    // Row block: the smallest block that still fills the SMs (more x reuse per
    // weight tile with larger blocks, more CTAs with smaller ones).
    static const int forced_rows = [] {
        const char* e = std::getenv("RPFQ_DECODE_ROWS");
        return e ? std::atoi(e) : 0;
    }();
    int rb = forced_rows;
    if (rb != 16 && rb != 32 && rb != 64) {
        const int64_t n_c = L->n_c;
        rb = (n_c + 63) / 64 >= st->sm_count ? 64 : ((n_c + 31) / 32 >= st->sm_count ? 32 : 16);
    }
    // split_k as for the GEMM: 0 automatic, 1 never, 2..8 forced
    const int sf = a->split_k;
    if (rb == 64) return launch_decode<64>(a, xin, ldx, st, stream, sf);
    if (rb == 32) return launch_decode<32>(a, xin, ldx, st, stream, sf);
    return launch_decode<16>(a, xin, ldx, st, stream, sf);
}

int pick_block_n(int64_t m, int n, int sm_count) {
    // Estimated time ~ waves of the persistent grid x tile width / relative
    // per-tile efficiency (measured on B200: 128-wide tiles run at ~0.78 of
    // the flop rate of 256-wide tiles).
    const int64_t mt = (m + 127) / 128;
    int best = 256;
    double best_cost = -1.0;
    for (int bn : {256, 128}) {
        const double eff = bn == 256 ? 1.0 : 0.78;
        const int64_t ntiles = (n + bn - 1) / bn;
        const int64_t waves = (mt * ntiles + sm_count - 1) / sm_count;
        const double cost = static_cast<double>(waves) * bn / eff;
        if (best_cost < 0 || cost < best_cost * 0.999) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

struct GemmPlan {
    int bn;          // tile width
    bool pair;       // CTA pairs (256 x 256 tiles)
    int splits;      // K splits per tile (one CTA per tile)
    bool stream_k;   // a stream-K tail when the tiles do not fill whole waves
    bool narrow;     // a narrow tail (last-wave tiles cut into column pieces)
};

constexpr double kSkMinIdleKBlocks = 24.0;  // see plan_gemm

// Stream-K: RPFQ_STREAM_K=0 off (data-parallel waves only), 1 (default) by the
// cost rule of plan_gemm, 2 whenever the tiles leave a tail (measurement).
int stream_k_mode() {
    static const int mode = [] {
        const char* e = std::getenv("RPFQ_STREAM_K");
        if (!e || !e[0]) return 1;
        return e[0] == '0' ? 0 : (e[0] == '2' ? 2 : 1);
    }();
    return mode;
}

// Time (us) of a one-CTA-per-tile plan when few tiles leave SMs idle, fitted
// to CUDA-event timings on B200 (M = 198..1584, K = 384..4096): a fixed
// launch-to-store cost (4.8 us for 128-wide tiles, 7.3 us for 256-wide ones:
// twice the epilogue), 0.28 us per k-block of the busiest CTA (each SM then
// streams its operands on its own), and for split-K the partial round trip
// (write, cluster barrier, batched reads) of 0.9 + 6 (bn / 128) / s us.
// < 0 when the plan does not fit one wave of clusters.
double small_m_cost(int64_t m, int n, int k, int bn, int s, DeviceState* st) {
    const int64_t tiles = gemm_tiles(m, n, bn);
    const int num_k = (k + 63) / 64;
    if (s > num_k || (s > 1 && num_k / s < kMinSplitKBlocks)) return -1.0;
    int64_t waves = (tiles + st->sm_count - 1) / st->sm_count;
    if (s > 1) {
        const int fit = bn == 256 ? max_clusters<256>(s, st) : max_clusters<128>(s, st);
        if (tiles > fit) return -1.0;
        waves = 1;
    }
    const double fixed = bn == 256 ? 7.3 : 4.8;
    const double reduce = s > 1 ? 0.9 + 6.0 * (bn / 128.0) / s : 0.0;
    return static_cast<double>(waves) * (fixed + 0.28 * ((num_k + s - 1) / s) + reduce);
}

// Tile width, CTA pairs and K splits of one call. Without a workspace (or
// split_k = 1) the tile width comes from the wave-quantisation model of
// pick_block_n; with one, shapes whose 128-wide tiles do not fill the SMs are
// planned by small_m_cost over tile widths and split counts.
GemmPlan plan_gemm(int64_t m, int n, int k, int block_n, int cta_pair, int split_k, bool have_ws, DeviceState* st,
                   bool sk_ws = false) {
    GemmPlan g;
    g.stream_k = false;
    g.narrow = false;
    const int64_t pair_tiles = ((m + 255) / 256) * ((n + 255) / 256);
    // A stream-K tail turns the last, partly idle wave of 256 x 256 pair tiles into
    // an even share per pair, at the price of moving each cut tile's fp32
    // accumulator (128 KiB per CTA) through L2 before its second part can start:
    // about 10 us on B200 (CUDA events, m = 6304). A pair k-block takes about
    // 0.5 us, so the tail is taken only when the idle part of the last wave is at
    // least 24 k-blocks long (ViT-B fc2 at 32 images: 0.99 x 48; qkv, fc1 and proj
    // with K = 768 lose).
    // The tails below force 256-wide pair tiles, so they apply only when n
    // fills such tiles (Swin's 96- to 576-column layers keep the width chosen by
    // pick_block_n: forcing 256 there cost 6 % of the Swin-T step).
    const bool full_width = n % 256 == 0;
    // A last wave at most half full: CTA pairs with the narrow tail (the last
    // wave's tiles cut into column pieces), which needs no workspace.
    if (full_width && narrow_tail_enabled() && block_n == 0 && cta_pair == 0 && split_k <= 1 &&
        pair_tiles >= st->sm_count / 2 && narrow_pieces(pair_tiles, gemm_units<256, false, 0, true>(st)) > 0) {
        g.bn = 256;
        g.pair = true;
        g.splits = 1;
        g.narrow = true;
        return g;
    }
    if (full_width && sk_ws && stream_k_mode() > 0 && block_n == 0 && cta_pair == 0 && split_k <= 1 &&
        pair_tiles >= st->sm_count / 2) {
        const int units = gemm_units<256, false, 0, true>(st);
        const int num_k = (k + 63) / 64;
        if (units > 0 && sk_tail(pair_tiles, units) > 0) {
            const int64_t waves = (pair_tiles + units - 1) / units;
            const double idle = static_cast<double>(waves) - static_cast<double>(pair_tiles) / units;
            if (stream_k_mode() == 2 || idle * num_k >= kSkMinIdleKBlocks) {
                g.bn = 256;
                g.pair = true;
                g.splits = 1;
                g.stream_k = true;
                return g;
            }
        }
    }
    g.bn = block_n ? block_n : pick_block_n(m, n, st->sm_count);
    g.pair = g.bn == 256 && (cta_pair == 2 || (cta_pair == 0 && split_k <= 1 && pair_tiles >= st->sm_count / 2));
    g.splits = 1;
    if (g.pair || !have_ws || split_k == 1) return g;
    const int num_k = (k + 63) / 64;
    if (split_k > 1) {
        g.splits = std::min(split_k, num_k);
        return g;
    }
    if (gemm_tiles(m, n, 128) > st->sm_count) return g;
    double best = -1.0;
    for (int bn : {128, 256}) {
        if (block_n && bn != block_n) continue;
        for (int s = 1; s <= kMaxSplits; ++s) {
            const double c = small_m_cost(m, n, k, bn, s, st);
            if (c >= 0 && (best < 0 || c < best - 1e-9)) {
                best = c;
                g.bn = bn;
                g.splits = s;
            }
        }
    }
    return g;
}

int gemm(const RpfqGemmArgs* a, cudaStream_t stream, RpfqGemmPlan* dry = nullptr) {
    if (!a) return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: null args");
    if (!a->x || !a->w || !a->y) return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: x, w and y are required");
    if (a->m < 0 || a->n <= 0 || a->k <= 0) return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: bad shape m=%lld n=%d k=%d", (long long)a->m, a->n, a->k);
    if (a->k % 8 || a->n % 8)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: k (%d) and n (%d) must be multiples of 8", a->k, a->n);
    if (a->flags & ~(RPFQ_GEMM_OUT_F32 | RPFQ_GEMM_RESIDUAL_F32 | RPFQ_GEMM_BIAS_F32))
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: unknown flags 0x%x", a->flags);
    if (a->ldx < a->k || a->ldx % 8 || a->ldy < a->n || a->ldy % 8)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: row strides must be >= the row length and multiples of 8");
    if (a->residual && (a->ldr < a->n || a->ldr % 8))
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: residual row stride must be >= n and a multiple of 8");
    if (a->residual && (((a->flags & RPFQ_GEMM_RESIDUAL_F32) != 0) != ((a->flags & RPFQ_GEMM_OUT_F32) != 0)))
        return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_gemm_sm100: the residual must have the output's dtype");
    if (!aligned16(a->x) || !aligned16(a->w) || !aligned16(a->y) || (a->bias && !aligned16(a->bias)) ||
        (a->residual && !aligned16(a->residual)))
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: all pointers must be 16-byte aligned");
    if (a->activation != RPFQ_ACT_NONE && a->activation != RPFQ_ACT_GELU)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: unknown activation %d", a->activation);
    if (a->split_k < 0 || a->split_k > kMaxSplits)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: split_k must be 0..%d (got %d)", kMaxSplits, a->split_k);
    if (a->workspace && !aligned16(a->workspace))
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: the workspace must be 16-byte aligned");
    if (a->split_k > 1 && a->cta_pair == 2)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: split_k > 1 runs one CTA per tile (cta_pair 2 given)");
    if (a->split_k > 1 && !a->workspace)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: split_k %d needs a workspace", a->split_k);
    if (a->m > (int64_t(1) << 31) - 256) return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_gemm_sm100: m too large");
    if (a->m == 0 && !dry) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    if (a->cta_pair < 0 || a->cta_pair > 2)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: cta_pair must be 0, 1 or 2 (got %d)", a->cta_pair);
    if (a->block_n != 0 && a->block_n != 128 && a->block_n != 256)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: block_n must be 0, 128 or 256 (got %d)", a->block_n);
    // CTA pairs (256 x 256 tiles over two SMs) when the 256-wide tile is chosen
    // and there are enough row pairs to fill the GPU; cta_pair forces either way.
    const bool sk_ws = a->workspace != nullptr && a->workspace_bytes >= ws_partial_bytes(st) + kSkFlagBytes;
    GemmPlan g = plan_gemm(a->m, a->n, a->k, a->block_n, a->cta_pair, a->split_k, a->workspace != nullptr, st, sk_ws);
    if (a->split_k == 0 && g.splits > 1 && splitk_bytes(a->m, a->n, g.bn, g.splits) > a->workspace_bytes)
        g = plan_gemm(a->m, a->n, a->k, a->block_n, a->cta_pair, 1, false, st);  // too small a workspace: no split
    const int splits = g.splits;
    if (splits > 1 && splitk_bytes(a->m, a->n, g.bn, splits) > a->workspace_bytes)
        return fail(RPFQ_ERR_INVALID, "rpfq_gemm_sm100: %d K splits need a workspace of %llu bytes (got %llu)", splits,
                    (unsigned long long)splitk_bytes(a->m, a->n, g.bn, splits), (unsigned long long)a->workspace_bytes);
    if (g.bn == 256)
        return g.pair ? launch_gemm_bn<256, true>(a, st, stream, 1, g.stream_k, g.narrow, dry)
                      : launch_gemm_bn<256, false>(a, st, stream, splits, false, false, dry);
    return launch_gemm_bn<128, false>(a, st, stream, splits, false, false, dry);
}

// ---------------------------------------------------------------- packed-layer validation
int check_layer(const RpfqPackedLinear* l, const char* who) {
    if (!l) return fail(RPFQ_ERR_INVALID, "%s: null layer", who);
    if (l->n_c <= 0 || l->k_c <= 0) return fail(RPFQ_ERR_INVALID, "%s: n_c and k_c must be positive", who);
    if (l->n_cp % 256 || l->k_cp % 256 || l->n_cp < l->n_c || l->k_cp < l->k_c)
        return fail(RPFQ_ERR_INVALID,
                    "%s: padded dims must be multiples of 256 covering the valid dims (n_c=%d n_cp=%d k_c=%d k_cp=%d)",
                    who, l->n_c, l->n_cp, l->k_c, l->k_cp);
    if (l->stages < 1 || l->stages > 4) return fail(RPFQ_ERR_INVALID, "%s: stages must be 1..4 (got %d)", who, l->stages);
    if (l->code_bits < 2 || l->code_bits > 4)
        return fail(RPFQ_ERR_INVALID, "%s: code_bits must be 2, 3 or 4 (got %d)", who, l->code_bits);
    return RPFQ_OK;
}

int check_planes(const RpfqPackedLinear* l, const char* who) {
    for (int s = 0; s < l->stages; ++s) {
        const RpfqPhasePlane* ps[2] = {&l->u[s], &l->w[s]};
        for (const RpfqPhasePlane* p : ps)
            if (!p->codes || !p->gamma_real || !p->gamma_imag)
                return fail(RPFQ_ERR_INVALID, "%s: stage %d has a null codes/gamma pointer", who, s);
    }
    return RPFQ_OK;
}

}  // namespace
}  // namespace rpfq

using namespace rpfq;

extern "C" {

int rpfq_version(void) { return 100; }

const char* rpfq_last_error(void) { return g_last_error.c_str(); }

int rpfq_device_error(int32_t* code_out) {
    if (!code_out) return fail(RPFQ_ERR_INVALID, "rpfq_device_error: null output");
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    RPFQ_CUDA(cudaDeviceSynchronize());
    int v = 0, zero = 0;
    RPFQ_CUDA(cudaMemcpy(&v, st->err_word, sizeof(int), cudaMemcpyDeviceToHost));
    RPFQ_CUDA(cudaMemcpy(st->err_word, &zero, sizeof(int), cudaMemcpyHostToDevice));
    *code_out = v;
    return RPFQ_OK;
}

int rpfq_prepack_sm100(const RpfqPackedLinear* layer, uint16_t* dense_out, int32_t rounding,
                       rpfq_stream_t stream) {
    int rc = check_layer(layer, "rpfq_prepack_sm100");
    if (!rc) rc = check_planes(layer, "rpfq_prepack_sm100");
    if (rc) return rc;
    if (!dense_out) return fail(RPFQ_ERR_INVALID, "rpfq_prepack_sm100: null output");
    if (rounding != RPFQ_ROUND_NEAREST_EVEN && rounding != RPFQ_ROUND_TIES_AWAY)
        return fail(RPFQ_ERR_INVALID, "rpfq_prepack_sm100: unknown rounding %d", rounding);
    DeviceState* st;
    rc = device_state(&st);
    if (rc) return rc;
    PrepackParams p;
    std::memset(&p, 0, sizeof(p));
    for (int s = 0; s < layer->stages; ++s) {
        p.u[s] = {layer->u[s].codes, reinterpret_cast<const __half*>(layer->u[s].gamma_real),
                  reinterpret_cast<const __half*>(layer->u[s].gamma_imag)};
        p.w[s] = {layer->w[s].codes, reinterpret_cast<const __half*>(layer->w[s].gamma_real),
                  reinterpret_cast<const __half*>(layer->w[s].gamma_imag)};
    }
    p.stages = layer->stages;
    p.code_bits = layer->code_bits;
    p.n_c = layer->n_c;
    p.k_c = layer->k_c;
    p.n_cp = layer->n_cp;
    p.k_cp = layer->k_cp;
    p.rounding = rounding;
    // Uniform-phase tables for the 3/4-bit extension: cos/sin of 2 pi c / 2^b
    // in double, exact zeros kept exact, rounded once to float.
    const int nphase = 1 << layer->code_bits;
    for (int c = 0; c < 16; ++c) {
        double a = 2.0 * M_PI * (c % nphase) / nphase;
        double cs = std::cos(a), sn = std::sin(a);
        if (std::fabs(cs) < 1e-12) cs = 0.0;
        if (std::fabs(sn) < 1e-12) sn = 0.0;
        p.cos_tab[c] = static_cast<float>(cs);
        p.sin_tab[c] = static_cast<float>(sn);
    }
    p.out = reinterpret_cast<__half*>(dense_out);
    const int groups = (layer->k_c + 3) / 4;
    dim3 block(128);
    dim3 grid((groups + 127) / 128, layer->n_c);
    prepack_kernel<<<grid, block, 0, static_cast<cudaStream_t>(stream)>>>(p);
    RPFQ_CUDA(cudaGetLastError());
    return RPFQ_OK;
}

int rpfq_gemm_sm100(const RpfqGemmArgs* args, rpfq_stream_t stream) {
    return gemm(args, static_cast<cudaStream_t>(stream));
}

int rpfq_gemm_plan_sm100(const RpfqGemmArgs* args, RpfqGemmPlan* plan) {
    if (!plan) return fail(RPFQ_ERR_INVALID, "rpfq_gemm_plan_sm100: null plan");
    std::memset(plan, 0, sizeof(*plan));
    return gemm(args, nullptr, plan);
}

uint64_t rpfq_gemm_workspace_bytes(int64_t m, int32_t n, int32_t k) {
    DeviceState* st;
    if (device_state(&st)) return 0;
    // split-K partials (tiles x splits <= SMs) or stream-K partials (units x ranks
    // <= SMs), then the stream-K flags
    if (m == 0) return ws_partial_bytes(st) + kSkFlagBytes;
    if (m < 0 || n <= 0 || k <= 0) return 0;
    const GemmPlan g = plan_gemm(m, n, k, 0, 0, 0, true, st, true);
    if (g.stream_k) {
        // the tail exists only when the pair tiles do not fill whole waves (every
        // pair-kernel variant has the same resident pair count)
        const int64_t tiles = ((m + 255) / 256) * ((n + 255) / 256);
        return gemm_sk_tiles<256, false, 0, true>(tiles, st) ? ws_partial_bytes(st) + kSkFlagBytes : 0;
    }
    return g.splits > 1 ? splitk_bytes(m, n, g.bn, g.splits) : 0;
}

int rpfq_act_quant_sm100(const uint16_t* x, int64_t ldx, uint16_t* xq, int64_t ldq, int64_t m, int32_t k,
                         int32_t num_bits, rpfq_stream_t stream) {
    if (!x || !xq) return fail(RPFQ_ERR_INVALID, "rpfq_act_quant_sm100: null pointer");
    if (k <= 0 || k % 2) return fail(RPFQ_ERR_INVALID, "rpfq_act_quant_sm100: k must be positive and even (got %d)", k);
    if (m < 0 || ldx < k || ldq < k) return fail(RPFQ_ERR_INVALID, "rpfq_act_quant_sm100: bad shape or stride");
    if (num_bits < 2 || num_bits > 8)
        return fail(RPFQ_ERR_INVALID, "rpfq_act_quant_sm100: num_bits must be 2..8 (got %d)", num_bits);
    if (m == 0) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    ActQuantParams p;
    p.x = reinterpret_cast<const __half*>(x);
    p.y = reinterpret_cast<__half*>(xq);
    p.ldx = ldx;
    p.ldy = ldq;
    p.m = m;
    p.k_c = k / 2;
    p.num_bits = num_bits;
    const int warps = 8;
    const int64_t blocks = (m + warps - 1) / warps;
    if (blocks > 0x7fffffff) return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_act_quant_sm100: m too large");
    RPFQ_CUDA(launch_kernel(act_quant_kernel, dim3(static_cast<unsigned>(blocks)), dim3(warps * 32), 0,
                            static_cast<cudaStream_t>(stream), 1, p));
    RPFQ_CUDA(cudaGetLastError());
    return RPFQ_OK;
}

int rpfq_patch_unfold_sm100(const void* images, int32_t images_f32, int64_t batch, int32_t channels,
                            int32_t height, int32_t width, int32_t patch, uint16_t* patches, int64_t ldp,
                            rpfq_stream_t stream) {
    if (!images || !patches) return fail(RPFQ_ERR_INVALID, "rpfq_patch_unfold_sm100: null pointer");
    if (batch < 0 || channels <= 0 || patch <= 0 || patch % 4 || height <= 0 || width <= 0 || height % patch ||
        width % patch)
        return fail(RPFQ_ERR_INVALID,
                    "rpfq_patch_unfold_sm100: patch must be a positive multiple of 4 that divides height and width "
                    "(got %d for %dx%d)", patch, height, width);
    const int chunk = patch % 8 == 0 ? 8 : 4;  // pixels per thread (one 16- or 8-byte store)
    const int64_t k = static_cast<int64_t>(channels) * patch * patch;
    if (ldp < k || ldp % chunk)
        return fail(RPFQ_ERR_INVALID,
                    "rpfq_patch_unfold_sm100: ldp must be >= channels * patch^2 and a multiple of %d", chunk);
    if (!aligned16(images) || !aligned16(patches))
        return fail(RPFQ_ERR_INVALID, "rpfq_patch_unfold_sm100: images and patches must be 16-byte aligned");
    const int64_t chunks = batch * channels * static_cast<int64_t>(height) * width / chunk;
    if (chunks == 0) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    PatchUnfoldParams p;
    p.images = images;
    p.out = reinterpret_cast<__half*>(patches);
    p.ldo = ldp;
    p.chunks = chunks;
    p.c = channels;
    p.h = height;
    p.w = width;
    p.patch = patch;
    p.f32 = images_f32 ? 1 : 0;
    const int64_t blocks = (chunks + 255) / 256;
    if (blocks > 0x7fffffff) return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_patch_unfold_sm100: too many images");
    RPFQ_CUDA(chunk == 8 ? launch_kernel(patch_unfold_kernel<8>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                                         static_cast<cudaStream_t>(stream), 1, p)
                         : launch_kernel(patch_unfold_kernel<4>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                                         static_cast<cudaStream_t>(stream), 1, p));
    RPFQ_CUDA(cudaGetLastError());
    return RPFQ_OK;
}

int rpfq_layernorm_sm100(const float* x, int64_t ldx, const uint16_t* weight, const uint16_t* bias, uint16_t* y,
                         int64_t ldy, int64_t m, int32_t d, float eps, int32_t act_bits, rpfq_stream_t stream) {
    return rpfq_layernorm_rows_sm100(x, ldx, m, nullptr, weight, bias, y, ldy, m, d, eps, act_bits, stream);
}

int rpfq_layernorm_rows_sm100(const float* x, int64_t ldx, int64_t x_rows, const int32_t* rows,
                              const uint16_t* weight, const uint16_t* bias, uint16_t* y, int64_t ldy, int64_t m,
                              int32_t d, float eps, int32_t act_bits, rpfq_stream_t stream) {
    if (!y) return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_sm100: null pointer");
    RpfqLayerNormArgs a;
    std::memset(&a, 0, sizeof(a));
    a.x = x;
    a.ldx = ldx;
    a.x_rows = x_rows;
    a.rows = rows;
    a.weight = weight;
    a.bias = bias;
    a.y = y;
    a.ldy = ldy;
    a.m = m;
    a.d = d;
    a.eps = eps;
    a.act_bits = act_bits;
    return rpfq_layernorm_ex_sm100(&a, stream);
}

int rpfq_layernorm_ex_sm100(const RpfqLayerNormArgs* a, rpfq_stream_t stream) {
    if (!a) return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_sm100: null args");
    const int32_t d = a->d;
    const int64_t m = a->m;
    if (a->rows != nullptr && ((reinterpret_cast<uintptr_t>(a->rows) & 3) || a->x_rows < 0))
        return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_rows_sm100: rows must be 4-byte aligned, x_rows >= 0");
    if (!a->x || !a->weight || !a->bias || (!a->y && !a->y32))
        return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_sm100: null pointer (x, weight, bias and y or y32 are required)");
    if (m < 0 || a->ldx < (a->merge_side > 0 ? d / 4 : d) || a->ldx % 4 || (a->y && (a->ldy < d || a->ldy % 4)) ||
        (a->y32 && (a->ldy32 < d || a->ldy32 % 4)))
        return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_sm100: bad shape or stride (strides must be multiples of 4)");
    if (!aligned16(a->x) || (a->y && (reinterpret_cast<uintptr_t>(a->y) & 7)) || (a->y32 && !aligned16(a->y32)) ||
        (reinterpret_cast<uintptr_t>(a->weight) & 7) || (reinterpret_cast<uintptr_t>(a->bias) & 7))
        return fail(RPFQ_ERR_INVALID,
                    "rpfq_layernorm_sm100: x and y32 must be 16-byte and y, weight, bias 8-byte aligned");
    if (a->act_bits != 0 && (a->act_bits < 2 || a->act_bits > 8))
        return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_sm100: act_bits must be 0 or 2..8 (got %d)", a->act_bits);
    if (d % 2) return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_sm100: odd row length %d", d);
    if (a->merge_side < 0 || a->merge_side % 2)
        return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_ex_sm100: merge_side must be 0 or even (got %d)", a->merge_side);
    if (a->merge_side > 0) {
        const int64_t half = a->merge_side / 2;
        if (a->rows || a->add || d % 16 || m % (half * half) ||
            a->x_rows < (m / (half * half)) * a->merge_side * a->merge_side)
            return fail(RPFQ_ERR_INVALID,
                        "rpfq_layernorm_ex_sm100: patch merging needs no gather / add, d %% 16 == 0, m a multiple of "
                        "(side/2)^2 and x_rows >= images * side^2");
    }
    if (a->add) {
        if (!a->y32 || !a->y32_prenorm || a->ld_add < d || a->ld_add % 4 || !aligned16(a->add) ||
            (a->add_rows && (reinterpret_cast<uintptr_t>(a->add_rows) & 3)) || a->add_bound < 0)
            return fail(RPFQ_ERR_INVALID,
                        "rpfq_layernorm_ex_sm100: add needs y32 with y32_prenorm, a 16-byte aligned add "
                        "with ld_add >= d (a multiple of 4) and 4-byte aligned add_rows");
    }
    if (a->y32 && static_cast<const void*>(a->y32) == static_cast<const void*>(a->x) &&
        (a->rows || a->merge_side || a->ldy32 != a->ldx))
        return fail(RPFQ_ERR_INVALID, "rpfq_layernorm_ex_sm100: y32 may alias x only with the plain row mapping");
    if (m == 0) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    LayerNormParams p;
    p.x = a->x;
    p.w = reinterpret_cast<const __half*>(a->weight);
    p.b = reinterpret_cast<const __half*>(a->bias);
    p.y = reinterpret_cast<__half*>(a->y);
    p.y32 = a->y32;
    p.ldx = a->ldx;
    p.ldy = a->ldy;
    p.ldy32 = a->ldy32;
    p.m = m;
    p.eps = a->eps;
    p.act_bits = a->act_bits;
    p.rows = a->rows;
    p.x_rows = a->rows ? a->x_rows : 0;
    p.add = a->add;
    p.add_rows = a->add_rows;
    p.ld_add = a->ld_add;
    p.add_bound = a->add_rows ? a->add_bound : m;
    p.y32_prenorm = a->y32_prenorm ? 1 : 0;
    p.merge_side = a->merge_side;
    p.err = st->err_word;
    const int warps = 8;
    const int64_t rows_per_block = static_cast<int64_t>(warps) * (32 / ln_lanes_per_row(d));
    const int64_t blocks = (m + rows_per_block - 1) / rows_per_block;
    if (blocks > 0x7fffffff) return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_layernorm_sm100: m too large");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned nb = static_cast<unsigned>(blocks);
    const bool plain = !a->rows && !a->add && !a->merge_side && !a->y32;
    // the fused quantizer's per-row quotient tables (dynamic shared memory)
    const bool quant = a->act_bits > 0;
    const size_t qtab = quant ? static_cast<size_t>(ln_qtab_floats(d, warps, a->act_bits)) * sizeof(float) : 0;
    switch (d) {
#define RPFQ_LN_LAUNCH(D, PL, Q) launch_kernel(layernorm_f32_f16_kernel<D, PL, Q>, dim3(nb), dim3(warps * 32), qtab, s, 1, p)
#define RPFQ_LN_CASE(D)                                                                                            \
    case D:                                                                                                        \
        RPFQ_CUDA(plain ? (quant ? RPFQ_LN_LAUNCH(D, true, true) : RPFQ_LN_LAUNCH(D, true, false))                  \
                        : (quant ? RPFQ_LN_LAUNCH(D, false, true) : RPFQ_LN_LAUNCH(D, false, false)));              \
        break;
        RPFQ_LN_CASE(96)
        RPFQ_LN_CASE(192)
        RPFQ_LN_CASE(384)
        RPFQ_LN_CASE(768)
        RPFQ_LN_CASE(1024)
        RPFQ_LN_CASE(1536)
        RPFQ_LN_CASE(3072)
#undef RPFQ_LN_CASE
#undef RPFQ_LN_LAUNCH
        default:
            return fail(RPFQ_ERR_UNSUPPORTED,
                        "rpfq_layernorm_sm100: row length %d (supported: 96, 192, 384, 768, 1024, 1536, 3072)", d);
    }
    RPFQ_CUDA(cudaGetLastError());
    return RPFQ_OK;
}

int rpfq_attention_sm100(const uint16_t* qkv, int64_t images, int32_t tokens, int32_t heads, int32_t head_dim,
                         uint16_t* out, int64_t ldo, rpfq_stream_t stream) {
    if (!qkv || !out) return fail(RPFQ_ERR_INVALID, "rpfq_attention_sm100: null pointer");
    if (images < 0 || tokens <= 0 || heads <= 0)
        return fail(RPFQ_ERR_INVALID, "rpfq_attention_sm100: bad shape (images %lld, tokens %d, heads %d)",
                    (long long)images, tokens, heads);
    if (head_dim != 64) return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_attention_sm100: head_dim %d (only 64)", head_dim);
    if (tokens > AttnCfg::LK)
        return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_attention_sm100: %d tokens (at most %d keys in one tile)", tokens,
                    AttnCfg::LK);
    const int64_t d = static_cast<int64_t>(heads) * head_dim;
    if (ldo < d || ldo % 8 || !aligned16(qkv) || !aligned16(out))
        return fail(RPFQ_ERR_INVALID, "rpfq_attention_sm100: 16-byte aligned rows required (ldo >= d, ldo %% 8 == 0)");
    if (images * heads * 2 > 0x7fffffff) return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_attention_sm100: grid too large");
    if (images == 0) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr[kMaxDevices];
    int dev = 0;
    RPFQ_CUDA(cudaGetDevice(&dev));
    std::call_once(once[dev], [dev]() {
        attr[dev] = cudaFuncSetAttribute(attn_short_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         AttnCfg::SMEM_BYTES);
    });
    RPFQ_CUDA(attr[dev]);
    EncodeTiledFn fn;
    rc = encode_fn(&fn);
    if (rc) return rc;
    CUtensorMap tm;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(3 * d), static_cast<cuuint64_t>(tokens),
                          static_cast<cuuint64_t>(images)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(3 * d * 2), static_cast<cuuint64_t>(3 * d * 2 * tokens)};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t*>(qkv), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RPFQ_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for qkv", (int)r);
    AttnParams p;
    p.out = reinterpret_cast<__half*>(out);
    p.ldo = ldo;
    p.L = tokens;
    p.heads = heads;
    p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(head_dim)));
    p.err = st->err_word;
    p.images = static_cast<int32_t>(images);
    const int64_t items = images * heads;
    const int grid = static_cast<int>(std::min<int64_t>(items, st->sm_count));
    RPFQ_CUDA(launch_kernel(attn_short_sm100_kernel, dim3(grid), dim3(AttnCfg::THREADS), AttnCfg::SMEM_BYTES,
                            static_cast<cudaStream_t>(stream), 1, tm, p));
    return RPFQ_OK;
}

int rpfq_window_attention_sm100(const uint16_t* qkv, int64_t windows, int32_t heads, int32_t head_dim,
                                int32_t window_tokens, const float* bias_mask, int32_t bm_windows, uint16_t* out,
                                int64_t ldo, rpfq_stream_t stream) {
    using C = WinAttnCfg;
    if (!qkv || !out || !bias_mask) return fail(RPFQ_ERR_INVALID, "rpfq_window_attention_sm100: null pointer");
    if (head_dim != C::HD || window_tokens != C::L)
        return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_window_attention_sm100: head_dim %d / %d tokens per window "
                    "(supported: 32 / 49, the 7x7 windows of Swin)", head_dim, window_tokens);
    if (windows < 0 || heads <= 0 || bm_windows <= 0 || heads > 4096)
        return fail(RPFQ_ERR_INVALID, "rpfq_window_attention_sm100: bad shape (windows %lld, heads %d, bm_windows %d)",
                    (long long)windows, heads, bm_windows);
    const int64_t d = static_cast<int64_t>(heads) * head_dim;
    if (ldo < d || ldo % 8 || !aligned16(qkv) || !aligned16(out) || !aligned16(bias_mask))
        return fail(RPFQ_ERR_INVALID,
                    "rpfq_window_attention_sm100: 16-byte aligned qkv, out and bias_mask, ldo >= heads * 32, ldo %% 8 == 0");
    if (windows * C::L > 0x7fffffff - 128)
        return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_window_attention_sm100: too many windows");
    if (windows == 0) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr[kMaxDevices];
    int dev = 0;
    RPFQ_CUDA(cudaGetDevice(&dev));
    std::call_once(once[dev], [dev]() {
        attr[dev] = cudaFuncSetAttribute(attn_window_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         WinAttnCfg::SMEM_BYTES);
    });
    RPFQ_CUDA(attr[dev]);
    // qkv [windows * 49, 3 d], [64 rows x 64 columns] boxes (128-B swizzle)
    CUtensorMap tm;
    rc = make_tmap_f16(&tm, qkv, windows * C::L, 3 * d, 3 * d, C::LP, 64);
    if (rc) return rc;
    WinAttnParams p;
    p.bias_mask = bias_mask;
    p.out = reinterpret_cast<__half*>(out);
    p.ldo = ldo;
    p.windows = static_cast<int32_t>(windows);
    p.heads = heads;
    p.bm_windows = bm_windows;
    p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(head_dim)));
    p.err = st->err_word;
    const int64_t items = ((windows + 1) / 2) * ((heads + 1) / 2);
    const int grid = static_cast<int>(std::min<int64_t>(items, st->sm_count));
    RPFQ_CUDA(launch_kernel(attn_window_sm100_kernel, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES,
                            static_cast<cudaStream_t>(stream), 1, tm, p));
    return RPFQ_OK;
}

uint64_t rpfq_vision_workspace_bytes(int64_t images, int32_t tokens) {
    if (images <= 0 || tokens <= 0) return 0;
    return 24ull * static_cast<uint64_t>(images) * static_cast<uint64_t>(tokens);
}

int rpfq_vision_act_quant_sm100(const uint16_t* x, int64_t ldx, uint16_t* xq, int64_t ldq, int64_t images,
                                int32_t tokens, int32_t k, double salient_ratio, double background_clip_ratio,
                                double energy_score_weight, int32_t protect_cls_token, uint8_t* mask_out,
                                void* workspace, uint64_t workspace_bytes, rpfq_stream_t stream) {
    if (!x || !xq) return fail(RPFQ_ERR_INVALID, "rpfq_vision_act_quant_sm100: null pointer");
    if (images < 0 || tokens <= 0 || k <= 0 || k % 16)
        return fail(RPFQ_ERR_INVALID, "rpfq_vision_act_quant_sm100: need images >= 0, tokens > 0, k a multiple of 16");
    if (ldx < k || ldq < k || ldx % 8 || ldq % 8 || !aligned16(x) || !aligned16(xq))
        return fail(RPFQ_ERR_INVALID, "rpfq_vision_act_quant_sm100: rows must be 16-byte aligned (strides % 8)");
    if (!(salient_ratio >= 0.0 && salient_ratio <= 1.0))
        return fail(RPFQ_ERR_INVALID, "salient_token_ratio must be in [0, 1].");
    if (!(background_clip_ratio > 0.0)) return fail(RPFQ_ERR_INVALID, "background_clip_ratio must be > 0.");
    if (!(energy_score_weight >= 0.0 && energy_score_weight <= 1.0))
        return fail(RPFQ_ERR_INVALID, "energy_score_weight must be in [0, 1].");
    if (images == 0) return RPFQ_OK;
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    VisionQuantParams p;
    std::memset(&p, 0, sizeof(p));
    p.x = reinterpret_cast<const __half*>(x);
    p.ldx = ldx;
    p.y = reinterpret_cast<__half*>(xq);
    p.ldy = ldq;
    p.tokens = tokens;
    p.k_c = k / 2;
    p.protect_cls = protect_cls_token ? 1 : 0;
    p.clip = static_cast<float>(background_clip_ratio);
    p.w_energy = static_cast<float>(energy_score_weight);
    p.w_contrast = static_cast<float>(1.0 - energy_score_weight);
    p.mask_out = mask_out;
    const int patches = tokens - 1;
    int g = 0;
    if (patches > 0) {
        g = static_cast<int>(std::sqrt(static_cast<double>(patches)));
        while (g * g > patches) --g;
        while ((g + 1) * (g + 1) <= patches) ++g;
        if (g * g != patches) g = 0;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (g == 0) {
        p.grid = 0;
        const int64_t rows = images * tokens;
        const int64_t ctas = std::min<int64_t>((rows + 15) / 16, 8 * st->sm_count);
        RPFQ_CUDA(launch_kernel(vision_quant_tokenwise_kernel, dim3(static_cast<unsigned>(ctas)), dim3(kVisionThreads), 0, s,
                                1, p, rows));
        RPFQ_CUDA(cudaGetLastError());
        return RPFQ_OK;
    }
    if (tokens > kVisionMaxTokens)
        return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_vision_act_quant_sm100: saliency grid of %d patches (max %d)", patches,
                    kVisionMaxTokens - 1);
    if (images > 0x7fffffff) return fail(RPFQ_ERR_UNSUPPORTED, "rpfq_vision_act_quant_sm100: too many images");
    p.grid = g;
    // the reference: max(1, ceil(P * ratio)) capped at P, 0 when the ratio is 0 (Python floats)
    p.num_salient = salient_ratio <= 0.0
                        ? 0
                        : static_cast<int>(std::min<double>(patches, std::max(1.0, std::ceil(patches * salient_ratio))));
    if (!workspace || workspace_bytes < rpfq_vision_workspace_bytes(images, tokens) || !aligned16(workspace))
        return fail(RPFQ_ERR_INVALID,
                    "rpfq_vision_act_quant_sm100: a 16-byte aligned workspace of rpfq_vision_workspace_bytes() bytes "
                    "is required for a saliency grid");
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr[kMaxDevices];
    int dev = 0;
    RPFQ_CUDA(cudaGetDevice(&dev));
    const int max_smem = 2 * (kVisionMaxTokens - 1) * 4 + kVisionMaxTokens + 16;
    std::call_once(once[dev], [dev, max_smem]() {
        attr[dev] = cudaFuncSetAttribute(vision_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    });
    RPFQ_CUDA(attr[dev]);
    const int64_t rows = images * tokens;
    VisionTokenStats* stats = static_cast<VisionTokenStats*>(workspace);
    float2* scales = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) + 16 * rows);
    const int64_t stat_ctas = std::min<int64_t>((rows + 15) / 16, 16 * st->sm_count);
    RPFQ_CUDA(launch_kernel(vision_stats_kernel, dim3(static_cast<unsigned>(stat_ctas)), dim3(kVisionThreads), 0, s, 1, p,
                            rows, stats));
    RPFQ_CUDA(cudaGetLastError());
    const int smem = 2 * patches * 4 + tokens;
    RPFQ_CUDA(launch_kernel(vision_select_kernel, dim3(static_cast<unsigned>(images)), dim3(kVisionThreads),
                            static_cast<size_t>(smem), s, 1, p, stats, scales));
    RPFQ_CUDA(cudaGetLastError());
    const int64_t apply_ctas =
        std::min<int64_t>((rows + 16 * kVisionApplyRun - 1) / (16 * kVisionApplyRun), 2 * st->sm_count);  // resident CTAs
    RPFQ_CUDA(launch_kernel(vision_apply_kernel, dim3(static_cast<unsigned>(apply_ctas)), dim3(kVisionThreads), 0, s, 1, p,
                            rows, scales));
    RPFQ_CUDA(cudaGetLastError());
    return RPFQ_OK;
}

uint64_t rpfq_pack_workspace_bytes(int32_t n_c, int32_t k_c) {
    if (n_c <= 0 || k_c <= 0) return 0;
    return 16ull * static_cast<uint64_t>(n_c) * static_cast<uint64_t>(k_c) +
           static_cast<uint64_t>(kPackMaxStatsCtas) * kPackPartials * sizeof(double);
}

int rpfq_pack_linear_sm100(const float* weight, int64_t ldw, int32_t n_c, int32_t k_c, int32_t stages,
                           const RpfqPhasePlaneOut* u_out, const RpfqPhasePlaneOut* w_out, void* workspace,
                           uint64_t workspace_bytes, rpfq_stream_t stream) {
    if (!weight || !u_out || !w_out || !workspace) return fail(RPFQ_ERR_INVALID, "rpfq_pack_linear_sm100: null pointer");
    if (n_c <= 0 || k_c <= 0)
        return fail(RPFQ_ERR_INVALID, "rpfq_pack_linear_sm100: complex dims must be positive (got %d, %d)", n_c, k_c);
    if (stages < 1 || stages > 4)
        return fail(RPFQ_ERR_INVALID, "rpfq_pack_linear_sm100: stages must be 1..4 (got %d)", stages);
    if (ldw < 2 * static_cast<int64_t>(k_c))
        return fail(RPFQ_ERR_INVALID, "rpfq_pack_linear_sm100: ldw %lld < 2 k_c", (long long)ldw);
    if ((reinterpret_cast<uintptr_t>(weight) & 3) || !aligned16(workspace))
        return fail(RPFQ_ERR_INVALID, "rpfq_pack_linear_sm100: weight must be 4-byte, workspace 16-byte aligned");
    if (workspace_bytes < rpfq_pack_workspace_bytes(n_c, k_c))
        return fail(RPFQ_ERR_INVALID, "rpfq_pack_linear_sm100: workspace of %llu bytes, need %llu",
                    (unsigned long long)workspace_bytes, (unsigned long long)rpfq_pack_workspace_bytes(n_c, k_c));
    for (int s = 0; s < stages; ++s)
        for (const RpfqPhasePlaneOut* o : {&u_out[s], &w_out[s]})
            if (!o->codes || !o->gamma_real || !o->gamma_imag || (reinterpret_cast<uintptr_t>(o->gamma_real) & 1) ||
                (reinterpret_cast<uintptr_t>(o->gamma_imag) & 1))
                return fail(RPFQ_ERR_INVALID, "rpfq_pack_linear_sm100: stage %d output buffers missing or misaligned", s);
    DeviceState* st;
    int rc = device_state(&st);
    if (rc) return rc;
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    PackParams p;
    std::memset(&p, 0, sizeof(p));
    p.weight = weight;
    p.ldw = ldw;
    p.n_c = n_c;
    p.k_c = k_c;
    p.n_cp = (n_c + 255) / 256 * 256;
    p.k_cp = (k_c + 255) / 256 * 256;
    p.res = static_cast<float*>(workspace);
    p.partials = reinterpret_cast<double*>(static_cast<uint8_t*>(workspace) +
                                           16ull * static_cast<uint64_t>(n_c) * static_cast<uint64_t>(k_c));
    const int64_t elems = static_cast<int64_t>(n_c) * k_c;
    int64_t sc = (elems + kPackThreads - 1) / kPackThreads;
    const int stats_ctas = static_cast<int>(std::min<int64_t>(sc, std::min(kPackMaxStatsCtas, 4 * st->sm_count)));
    const int64_t bytes = static_cast<int64_t>(p.n_cp) * (p.k_cp / 4);
    const int code_ctas =
        static_cast<int>(std::min<int64_t>((bytes + kPackThreads - 1) / kPackThreads, 16 * st->sm_count));
    p.stats_ctas = stats_ctas;
    for (int s = 0; s < stages; ++s) {
        p.first = s == 0;
        p.write_res = s + 1 < stages;
        p.codes[0] = u_out[s].codes;
        p.codes[1] = w_out[s].codes;
        p.gre[0] = u_out[s].gamma_real;
        p.gim[0] = u_out[s].gamma_imag;
        p.gre[1] = w_out[s].gamma_real;
        p.gim[1] = w_out[s].gamma_imag;
        pack_stats_kernel<<<stats_ctas, kPackThreads, 0, strm>>>(p);
        RPFQ_CUDA(cudaGetLastError());
        pack_codes_kernel<<<code_ctas, kPackThreads, 0, strm>>>(p);
        RPFQ_CUDA(cudaGetLastError());
    }
    return RPFQ_OK;
}

int rpfq_wide_linear_sm100(const RpfqWideLinearArgs* a, rpfq_stream_t stream) {
    if (!a) return fail(RPFQ_ERR_INVALID, "rpfq_wide_linear_sm100: null args");
    int rc = check_layer(a->layer, "rpfq_wide_linear_sm100");
    if (rc) return rc;
    if (!a->dense && a->m > kDecodeMaxRows)
        return fail(RPFQ_ERR_INVALID,
                    "rpfq_wide_linear_sm100: for m > %lld the dense coefficients are required (decode them once with "
                    "rpfq_prepack_sm100)", (long long)kDecodeMaxRows);
    const int32_t K = 2 * a->layer->k_c;
    const int32_t N = 2 * a->layer->n_c;
    const uint16_t* xin = a->x;
    int64_t ldx = a->ldx;
    if (a->act_bits != 0) {
        if (!a->scratch)
            return fail(RPFQ_ERR_INVALID, "rpfq_wide_linear_sm100: act_bits > 0 needs a scratch buffer of m x %d fp16", K);
        rc = rpfq_act_quant_sm100(a->x, a->ldx, a->scratch, K, a->m, K, a->act_bits, stream);
        if (rc) return rc;
        xin = a->scratch;
        ldx = K;
    }
    if (!a->dense) return decode_path(a, xin, ldx, static_cast<cudaStream_t>(stream));
    RpfqGemmArgs g;
    std::memset(&g, 0, sizeof(g));
    g.x = xin;
    g.ldx = ldx;
    g.w = a->dense;
    g.bias = a->bias;
    g.residual = a->residual;
    g.ldr = a->ldr;
    g.y = a->y;
    g.ldy = a->ldy;
    g.m = a->m;
    g.n = N;
    g.k = K;
    g.activation = a->activation;
    g.flags = a->flags;
    g.split_k = a->split_k;
    g.workspace = a->workspace;
    g.workspace_bytes = a->workspace_bytes;
    return gemm(&g, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of the whole-layer entry point.
//
// Some callers cannot allocate device memory at the moment they run a layer:
// inference servers whose request path must not call cudaMalloc / cudaFree
// because those calls can synchronise the device and stall every other
// stream, and embedded or plugin hosts that own a fixed device budget and give
// a kernel library no allocator at all. With activation quantization on, the
// layer needs a scratch buffer for the quantized activations; this variant
// takes it from a fixed array compiled into the library instead of from the
// caller.
//
// The array is a file-scope static __device__ array of
// kNoAllocScratchBytes (8 MiB). Every GPU that loads this library holds it
// until the process exits. All calls share it and it keeps the last call's
// contents; nothing in it needs to start at zero, because the quantization
// kernel writes every element the GEMM then reads. Calls that overlap on the
// GPU (for example on two streams at once) race on it.
namespace rpfq {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) uint16_t g_noalloc_scratch[kNoAllocScratchBytes / sizeof(uint16_t)];

struct NoAllocState {
    std::once_flag once;
    cudaError_t status = cudaSuccess;
    uint16_t* ptr = nullptr;  // device address of g_noalloc_scratch on this device
};
NoAllocState g_noalloc[kMaxDevices];

// In host code the array's name is only a host-side stand-in, so its device
// address is looked up once per device, with that device current.
int noalloc_scratch(uint16_t** out) {
    int dev = 0;
    RPFQ_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(RPFQ_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    NoAllocState& st = g_noalloc[dev];
    std::call_once(st.once, [&st]() {
        void* p = nullptr;
        st.status = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        st.ptr = static_cast<uint16_t*>(p);
    });
    if (st.status != cudaSuccess || st.ptr == nullptr)
        return fail(RPFQ_ERR_CUDA, "cudaGetSymbolAddress of the no-alloc scratch failed: %s",
                    cudaGetErrorString(st.status));
    *out = st.ptr;
    return RPFQ_OK;
}

}  // namespace
}  // namespace rpfq

extern "C" int rpfq_wide_linear_noalloc_sm100(const RpfqWideLinearArgs* a, rpfq_stream_t stream) {
    if (!a) return fail(RPFQ_ERR_INVALID, "rpfq_wide_linear_noalloc_sm100: null args");
    int rc = check_layer(a->layer, "rpfq_wide_linear_noalloc_sm100");
    if (rc) return rc;
    if (a->m < 0) return fail(RPFQ_ERR_INVALID, "rpfq_wide_linear_noalloc_sm100: negative m");
    RpfqWideLinearArgs local = *a;
    local.scratch = nullptr;
    if (a->act_bits != 0) {
        // rows that fit: compared by division, so no product of caller sizes can wrap
        const int64_t row_bytes = 2 * static_cast<int64_t>(a->layer->k_c) * static_cast<int64_t>(sizeof(uint16_t));
        const int64_t max_rows = static_cast<int64_t>(kNoAllocScratchBytes) / row_bytes;
        if (a->m > max_rows)
            return fail(RPFQ_ERR_INVALID,
                        "rpfq_wide_linear_noalloc_sm100: the quantized activations of m=%lld rows x %d fp16 do not fit "
                        "the built-in scratch of %zu bytes (at most %lld rows for this layer); use "
                        "rpfq_wide_linear_sm100 with a caller buffer",
                        (long long)a->m, 2 * a->layer->k_c, kNoAllocScratchBytes, (long long)max_rows);
        uint16_t* scratch = nullptr;
        rc = noalloc_scratch(&scratch);
        if (rc) return rc;
        local.scratch = scratch;
    }
    return rpfq_wide_linear_sm100(&local, stream);
}
