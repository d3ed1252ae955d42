// C-ABI shim over the reference's own C++ CPU runtime for the packed
// complex-phase linear layer (TEST INFRASTRUCTURE ONLY).
//
// This file is compiled together with the reference's unmodified sources
// (RPFQ-ViTAndroid/app/src/main/cpp: ops/phase_linear.cpp, kernels/*.cpp,
// runtime/*.cpp, tensor.cpp, json_utils.cpp, safetensors_loader.cpp) by
// oracle/Makefile into oracle/_ref/librpfq_ref.so. The library is the second,
// independent oracle and the "reference" CPU baseline; nothing in the product
// links it.
//
// The shim builds a SafeTensorStore in memory (the same struct the reference
// fills from a safetensors file, safetensors_loader.h:10-18) and calls
// loadWideParams (phase_linear.cpp:90-117) with the argument meaning used by
// the reference engine (rpfq_vit_engine.cpp:240-275): real dims, padded
// complex dims, and the unpadded complex output count.

#include "ops/phase_linear.h"
#include "kernels/phase_linear_cache.h"
#include "kernels/phase_linear_fused.h"
#include "kernels/wide_linear_cache_neon.h"
#include "runtime/thread_pool.h"
#include "safetensors_loader.h"
#include "tensor.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <string>

using namespace rpfq_vit;

namespace {

thread_local std::string g_error;

const char* kPlanes[4] = {"u_s0", "u_s1", "w_s0", "w_s1"};

struct Layer {
    SafeTensorStore store;
    WideLinearParams params;
};

std::unique_ptr<Layer> makeLayer(int n_c, int k_c, int n_cp, int k_cp,
                                 const uint8_t* const* codes,
                                 const uint16_t* const* gamma_re,
                                 const uint16_t* const* gamma_im,
                                 const uint16_t* bias) {
    auto layer = std::make_unique<Layer>();
    const int blocks = k_cp / 256;
    for (int p = 0; p < 4; ++p) {
        std::string prefix = std::string("layer.") + kPlanes[p];
        UInt8Tensor c;
        c.shape = {n_cp, k_cp / 4};
        c.data.assign(codes[p], codes[p] + static_cast<size_t>(n_cp) * (k_cp / 4));
        layer->store.u8[prefix + ".codes"] = std::move(c);
        Tensor gr({n_cp, blocks});
        Tensor gi({n_cp, blocks});
        for (size_t i = 0; i < gr.data.size(); ++i) {
            gr.data[i] = halfToFloat(gamma_re[p][i]);
            gi.data[i] = halfToFloat(gamma_im[p][i]);
        }
        layer->store.f32[prefix + ".gamma_real"] = std::move(gr);
        layer->store.f32[prefix + ".gamma_imag"] = std::move(gi);
    }
    Tensor b({2 * n_c});
    for (int i = 0; i < 2 * n_c; ++i) b.data[i] = bias ? halfToFloat(bias[i]) : 0.0f;
    layer->store.f32["layer.bias"] = std::move(b);
    layer->params = loadWideParams(layer->store, "layer", 2 * k_c, 2 * n_c, k_cp, n_cp, n_c, 256);
    return layer;
}

ThreadPool& pool(int threads) {
    static std::mutex mu;
    static std::map<int, std::unique_ptr<ThreadPool>> pools;
    std::lock_guard<std::mutex> lock(mu);
    auto& slot = pools[threads];
    if (!slot) slot = std::make_unique<ThreadPool>(threads);
    return *slot;
}

}  // namespace

extern "C" {

const char* rpfq_ref_last_error() { return g_error.c_str(); }

// mode 0: wideLinearReference (scalar, fp32, phase_linear.cpp:166-207)
// mode 1: wideLinearOptimized (fused scalar, phase_linear_fused.cpp:120-148)
// mode 2: fp16 coefficient cache (wide_linear_cache_neon.cpp:69-161)
int rpfq_ref_wide_linear(const float* x, int tokens, int n_c, int k_c, int n_cp, int k_cp,
                         const uint8_t* const* codes, const uint16_t* const* gamma_re,
                         const uint16_t* const* gamma_im, const uint16_t* bias,
                         int mode, int threads, float* y) {
    try {
        auto layer = makeLayer(n_c, k_c, n_cp, k_cp, codes, gamma_re, gamma_im, bias);
        Tensor xt({tokens, 2 * k_c});
        std::memcpy(xt.data.data(), x, sizeof(float) * static_cast<size_t>(tokens) * 2 * k_c);
        Tensor out;
        if (mode == 0) {
            out = wideLinearReference(xt, layer->params);
        } else if (mode == 1) {
            out = wideLinearOptimized(xt, layer->params, threads);
        } else {
            layer->params.fusedCache = buildFusedWideLinearCache(layer->params);
            out = Tensor({tokens, 2 * n_c});
            wideLinearFusedCacheFp16Neon(xt, layer->params, out, pool(threads));
        }
        std::memcpy(y, out.data.data(), sizeof(float) * out.data.size());
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

// Four fp16 coefficient planes [n_c, k_c] from buildFusedWideLinearCache
// (phase_linear_cache.cpp:84-133): rr = XrToRe, ir = XiToRe, ri = XrToIm,
// ii = XiToIm.
int rpfq_ref_coefficient_planes(int n_c, int k_c, int n_cp, int k_cp,
                                const uint8_t* const* codes, const uint16_t* const* gamma_re,
                                const uint16_t* const* gamma_im, uint16_t* rr, uint16_t* ir,
                                uint16_t* ri, uint16_t* ii) {
    try {
        auto layer = makeLayer(n_c, k_c, n_cp, k_cp, codes, gamma_re, gamma_im, nullptr);
        auto cache = buildFusedWideLinearCache(layer->params);
        size_t count = static_cast<size_t>(n_c) * k_c;
        std::memcpy(rr, cache->coeffXrToReFp16.data(), count * 2);
        std::memcpy(ir, cache->coeffXiToReFp16.data(), count * 2);
        std::memcpy(ri, cache->coeffXrToImFp16.data(), count * 2);
        std::memcpy(ii, cache->coeffXiToImFp16.data(), count * 2);
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

// Prepared layer for repeated timing of the fp16-cache path (the CPU baseline):
// the cache is built once, as the reference runtime does at load time
// (phase_linear.cpp:113-115), and only the GEMM is timed.
void* rpfq_ref_prepare(int n_c, int k_c, int n_cp, int k_cp, const uint8_t* const* codes,
                       const uint16_t* const* gamma_re, const uint16_t* const* gamma_im,
                       const uint16_t* bias) {
    try {
        auto layer = makeLayer(n_c, k_c, n_cp, k_cp, codes, gamma_re, gamma_im, bias);
        layer->params.fusedCache = buildFusedWideLinearCache(layer->params);
        return layer.release();
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

int rpfq_ref_run_prepared(void* handle, const float* x, int tokens, int threads, float* y) {
    try {
        auto* layer = static_cast<Layer*>(handle);
        Tensor xt({tokens, layer->params.realInDim});
        std::memcpy(xt.data.data(), x, sizeof(float) * xt.data.size());
        Tensor out({tokens, layer->params.realOutDim});
        wideLinearFusedCacheFp16Neon(xt, layer->params, out, pool(threads));
        std::memcpy(y, out.data.data(), sizeof(float) * out.data.size());
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

void rpfq_ref_release(void* handle) { delete static_cast<Layer*>(handle); }

}  // extern "C"
