// C ABI (include/gptoss.h). Exceptions become -1 plus a thread-local message, as the reference's guard() does
// (runtime/src/capi.cpp:19-32). Kernel entry points run on the legacy default stream and synchronize before
// returning (runtime/src/capi.cpp:34-37).
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gptoss.h"
#include "kernels.h"

namespace {

thread_local std::string g_error;

template <class F>
int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
    } catch (...) {
        g_error = "unknown error";
    }
    return -1;
}

void sync_check(const char* what) {
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Grow-only scratch owned by the calling thread, one per device: the kernel entry points reuse it across calls
// instead of allocating per call. Freed at thread exit.
struct Scratch {
    void* p[64] = {};
    size_t n[64] = {};
    ~Scratch() {
        for (int d = 0; d < 64; ++d)
            if (p[d]) cudaFree(p[d]);
    }
    void* get(size_t bytes) {
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        if (dev < 0 || dev >= 64) throw std::runtime_error("device index out of range");
        if (n[dev] < bytes) {
            if (p[dev]) GPT_CHECK(cudaFree(p[dev]));
            p[dev] = nullptr;
            n[dev] = 0;
            GPT_CHECK(cudaMalloc(&p[dev], bytes));
            n[dev] = bytes;
        }
        return p[dev];
    }
};
thread_local Scratch g_scratch;

int g_moe_impl = 1;

[[noreturn]] void not_built(const char* what) {
    throw std::runtime_error(std::string(what) + ": not part of this build (the B200 MoE path); see gptoss.h");
}

}  // namespace

extern "C" {

const char* gptoss_last_error(void) { return g_error.c_str(); }

gptoss_engine* gptoss_create(const char* model_dir, int max_ctx, long long vram_budget_bytes) {
    (void)model_dir; (void)max_ctx; (void)vram_budget_bytes;
    guard([&] { not_built("gptoss_create"); });
    return nullptr;
}
void gptoss_destroy(gptoss_engine* e) { (void)e; }
int gptoss_vocab(const gptoss_engine*) { return -1; }
int gptoss_position(const gptoss_engine*) { return -1; }
long long gptoss_device_bytes(const gptoss_engine*) { return -1; }
int gptoss_reset(gptoss_engine*) { return guard([] { not_built("gptoss_reset"); }); }
int gptoss_use_graph(gptoss_engine*, int) { return guard([] { not_built("gptoss_use_graph"); }); }
int gptoss_step(gptoss_engine*, int) { return guard([] { not_built("gptoss_step"); }); }
int gptoss_logits(gptoss_engine*, float*) { return guard([] { not_built("gptoss_logits"); }); }
int gptoss_prefill(gptoss_engine*, const int32_t*, int, const int32_t*, int, float*, int32_t*, float*) {
    return guard([] { not_built("gptoss_prefill"); });
}
int gptoss_score(gptoss_engine*, const int32_t*, int, int, float*, int32_t*, float*, float*) {
    return guard([] { not_built("gptoss_score"); });
}
int gptoss_set_position(gptoss_engine*, int) { return guard([] { not_built("gptoss_set_position"); }); }
int gptoss_bench_steps(gptoss_engine*, int, int) { return guard([] { not_built("gptoss_bench_steps"); }); }

int gptoss_kernel_gemv_bf16(const void*, const float*, const float*, const float*, float*, int, int) {
    return guard([] { not_built("gptoss_kernel_gemv_bf16"); });
}
int gptoss_kernel_rope_append(float*, const float*, const float*, int, void*, void*, int) {
    return guard([] { not_built("gptoss_kernel_rope_append"); });
}
int gptoss_kernel_attention(const float*, const void*, const void*, const float*, int, int, int, float*) {
    return guard([] { not_built("gptoss_kernel_attention"); });
}

int gptoss_kernel_rmsnorm(const float* x, const float* w, float* y, int n, float eps) {
    return guard([&] {
        gpt::launch_rmsnorm(x, w, y, 1, n, eps, nullptr);
        sync_check("rmsnorm");
    });
}

int gptoss_kernel_router(const void* W, const float* b, const float* x, int E, int H, int k, int32_t* ids,
                         float* weights) {
    return guard([&] {
        gpt::launch_router_decode(static_cast<const __nv_bfloat16*>(W), b, x, E, H, k, ids, weights, nullptr);
        sync_check("router");
    });
}

int gptoss_kernel_moe(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                      const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias, const float* x_norm,
                      const int32_t* ids, const float* weights, float* x_resid, int k, int H, int I, float alpha,
                      float limit) {
    return guard([&] {
        if (k < 1 || k > 8) throw std::runtime_error("moe: k must be in 1..8");
        void* scratch = g_scratch.get(gpt::moe_decode_scratch_bytes(k, I));
        gpt::launch_moe_decode_simt(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, x_norm, ids,
                                    weights, x_resid, k, H, I, alpha, limit, scratch, nullptr);
        sync_check("moe");
    });
}

int gptoss_kernel_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, float* out, long long n_blocks) {
    return guard([&] {
        int* bad = static_cast<int*>(g_scratch.get(sizeof(int)));
        GPT_CHECK(cudaMemset(bad, 0, sizeof(int)));
        gpt::launch_mxfp4_dequant(blocks, scales, out, n_blocks, bad, nullptr);
        sync_check("mxfp4_dequant");
        int h = 0;
        GPT_CHECK(cudaMemcpy(&h, bad, sizeof(int), cudaMemcpyDeviceToHost));
        if (h) throw std::runtime_error("mxfp4_dequant: E8M0 scale 0xFF encodes NaN; refusing to decode it");
    });
}

int gptoss_moe_block_async(const float* x, const float* norm_w, float eps, const void* router_w,
                           const float* router_b, const uint8_t* gu_blocks, const uint8_t* gu_scales,
                           const float* gu_bias, const uint8_t* dn_blocks, const uint8_t* dn_scales,
                           const float* dn_bias, float* x_resid, int E, int k, int H, int I, float alpha, float limit,
                           void* stream, void* const* events) {
    return guard([&] {
        if (k < 1 || k > 8) throw std::runtime_error("moe: k must be in 1..8");
        if (H < 1 || I < 1) throw std::runtime_error("moe: H and I must be positive");
        const size_t h_bytes = (size_t(H) * sizeof(float) + 255) & ~size_t(255);
        char* ws = static_cast<char*>(g_scratch.get(h_bytes + 256 + gpt::moe_decode_scratch_bytes(k, I)));
        float* h = reinterpret_cast<float*>(ws);
        int* ids = reinterpret_cast<int*>(ws + h_bytes);
        float* w = reinterpret_cast<float*>(ws + h_bytes + 128);
        void* a = ws + h_bytes + 256;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        auto rec = [&](int i) {
            if (events) GPT_CHECK(cudaEventRecord(static_cast<cudaEvent_t>(events[i]), s));
        };
        gpt::launch_rmsnorm(x, norm_w, h, 1, H, eps, s);
        rec(0);
        gpt::launch_router_decode(static_cast<const __nv_bfloat16*>(router_w), router_b, h, E, H, k, ids, w, s);
        rec(1);
        gpt::launch_moe_decode_simt(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, h, ids, w, x_resid,
                                    k, H, I, alpha, limit, a, s, events ? events[2] : nullptr);
        rec(3);
    });
}

int gptoss_selftest_mxf4_gemm(const uint8_t* a_blocks, const uint8_t* a_scales, const uint8_t* b_blocks,
                              const uint8_t* b_scales, float* d, int N, int K) {
    return guard([&] {
        const size_t bytes = size_t(1) << 22;
        void* scratch = g_scratch.get(bytes);
        gpt::selftest_mxf4_gemm(a_blocks, a_scales, b_blocks, b_scales, d, N, K, scratch, bytes, nullptr);
    });
}

int gptoss_set_moe_impl(int impl) {
    if (impl != 0 && impl != 1) {
        g_error = "gptoss_set_moe_impl: impl must be 0 (SIMT) or 1 (tensor cores)";
        return -1;
    }
    const int prev = g_moe_impl;
    g_moe_impl = impl;
    return prev;
}

}  // extern "C"
