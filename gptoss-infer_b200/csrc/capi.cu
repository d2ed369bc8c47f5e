// C ABI (include/gptoss.h). Exceptions become -1 plus a thread-local message, as the reference's guard() does
// (runtime/src/capi.cpp:19-32). Kernel entry points run on the legacy default stream and synchronize before
// returning (runtime/src/capi.cpp:34-37).
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "common.cuh"
#include "gptoss.h"
#include "engine.h"
#include "kernels.h"
#include "tma.h"

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
thread_local Scratch g_flag;                // one device int for the NaN-scale check

// Error code the scale repack stores when it meets an E8M0 byte 0xFF (NaN): the reference refuses such a scale at
// load (runtime/src/engine.cu:119-122); here every path that repacks scales refuses it.
constexpr int kNanScaleCode = 200;

// Runs f(flag) with a zeroed device int and throws if f's kernels stored kNanScaleCode into it (synchronizes).
template <class F>
void with_nan_scale_check(const char* what, F&& f) {
    int* flag = static_cast<int*>(g_flag.get(sizeof(int)));
    GPT_CHECK(cudaMemset(flag, 0, sizeof(int)));
    f(flag);
    sync_check(what);
    int h = 0;
    GPT_CHECK(cudaMemcpy(&h, flag, sizeof(int), cudaMemcpyDeviceToHost));
    if (h == kNanScaleCode)
        throw std::runtime_error(std::string(what) + ": an E8M0 scale byte is 0xFF (NaN); refusing the weights");
}

// Workspace of the tensor-core decode path (activation terms, epoch-tagged partial sums, grid-barrier words, gathered
// scales), owned by the calling thread, one per device. Zero-filled whenever it is (re)allocated. The words that carry
// state from one launch to the next (barrier counters that reset themselves, the launch epoch, the tagged partial
// sums) sit at offsets that depend on the shape (k, H, I), so they are valid only for the layout that last used them:
// for_layout() zeroes the new layout's range of them, on the call's stream, whenever the shape changes.
struct DecodeWs {
    void* p[64] = {};
    size_t n[64] = {};
    unsigned long long shape[64] = {};        // (k, H, I) whose layout the state words follow; 0: none yet
    ~DecodeWs() {
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
            GPT_CHECK(cudaMemset(p[dev], 0, bytes));
            n[dev] = bytes;
            shape[dev] = 0;
        }
        return p[dev];
    }
    void* for_layout(const gpt::DecodeTcLayout& L, int k, int H, int I, cudaStream_t s) {
        void* w = get(L.bytes);
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        const unsigned long long key =
            (static_cast<unsigned long long>(k) << 48) | (static_cast<unsigned long long>(H) << 24) | unsigned(I);
        if (shape[dev] != key) {
            GPT_CHECK(cudaMemsetAsync(static_cast<char*>(w) + L.zero_bytes_from, 0, L.zero_bytes_to - L.zero_bytes_from,
                                      s));
            shape[dev] = key;
        }
        return w;
    }
};
thread_local DecodeWs g_dws;

// Decode MoE implementation: 0 SIMT, 1 tensor cores (the row-job kernel where its shape conditions hold, else the
// stream-K kernel), 2 tensor cores with the stream-K kernel only.
int g_moe_impl = 1;
int decode_plan() { return g_moe_impl == 2 ? 1 : 0; }
bool moe_impl_tc() { return g_moe_impl == 1 || g_moe_impl == 2; }

bool tc_shape_ok(int k, int H, int I) { return k >= 1 && k <= 8 && H % 64 == 0 && I % 64 == 0 && H >= 64 && I >= 64; }
// The tensor-core decode kernel also holds x in registers (H <= 3072).
bool decode_tc_ok(int k, int H, int I) { return tc_shape_ok(k, H, I) && H <= 3072; }

// Reads the device-side error word of the tensor-core kernels after a synchronization; on error the workspace's
// counters are cleared so the next call starts clean.
void check_tc_error(void* ws, const gpt::DecodeTcLayout& L) {
    int h = 0;
    GPT_CHECK(cudaMemcpy(&h, static_cast<char*>(ws) + L.off_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        GPT_CHECK(cudaMemset(static_cast<char*>(ws) + L.zero_bytes_from, 0, L.zero_bytes_to - L.zero_bytes_from));
        if (h == kNanScaleCode)
            throw std::runtime_error("moe: an E8M0 scale of a selected expert is 0xFF (NaN); refusing to use it");
        throw std::runtime_error("moe (tensor cores): a bounded wait gave up (site " + std::to_string(h) + ")");
    }
}

// Tensor-core MoE on raw checkpoint-layout experts whose count is unknown: the scales of the k selected experts
// are gathered and repacked per call, then the fused kernel runs with the given ids (router off).
void moe_tc_raw(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias, const uint8_t* dn_blocks,
                const uint8_t* dn_scales, const float* dn_bias, const float* x_norm, const int* ids,
                const float* weights, float* x_resid, int k, int H, int I, float alpha, float limit, void* ws,
                const gpt::DecodeTcLayout& L, cudaStream_t s) {
    char* w = static_cast<char*>(ws);
    int* err = reinterpret_cast<int*>(w + L.off_err);      // a NaN scale is reported through the error word
    gpt::launch_repack_sf(gu_scales, reinterpret_cast<uint8_t*>(w + L.off_sfa_gu), k, 2 * I, H / 32, s, ids,
                          gpt::kDecodeTileRows, err, kNanScaleCode);
    gpt::launch_repack_sf(dn_scales, reinterpret_cast<uint8_t*>(w + L.off_sfa_dn), k, H, I / 32, s, ids,
                          gpt::kDecodeTileRows, err, kNanScaleCode);
    // The expert count is not part of this ABI: the maps span the 32 experts the format allows; only the selected
    // experts' rows are ever read.
    const CUtensorMap tg = gpt::make_tmap_u8_sw128_3d(gu_blocks, H / 2, 2 * I, 32, 128, gpt::kDecodeTileRows);
    const CUtensorMap td = gpt::make_tmap_u8_sw128_3d(dn_blocks, I / 2, H, 32, 128, gpt::kDecodeTileRows);
    const CUtensorMap td64 = gpt::make_tmap_u8_swz_3d(dn_blocks, I / 2, H, 32, 64, gpt::kDecodeTileRows, 64);
    gpt::DecodeTcArgs a{};
    a.tmap_gu = &tg;
    a.tmap_dn = &td;
    a.tmap_dn64 = &td64;
    a.plan = decode_plan();
    a.sfa_gu = reinterpret_cast<uint8_t*>(w + L.off_sfa_gu);
    a.sfa_dn = reinterpret_cast<uint8_t*>(w + L.off_sfa_dn);
    a.sfa_by_slot = 1;
    a.gu_bias = gu_bias;
    a.dn_bias = dn_bias;
    a.x = x_norm;
    a.ids = ids;
    a.weights = weights;
    a.x_resid = x_resid;
    a.k = k;
    a.H = H;
    a.I = I;
    a.alpha = alpha;
    a.limit = limit;
    a.workspace = ws;
    gpt::launch_moe_decode_tc(a, s);
}

std::atomic<int> g_prefill_terms{8};   // e2m1 terms per activation in the batched MoE
std::atomic<int> g_prefill_pack{-1};   // -1: by batch size, 0: stacked, 1: packed

// The batched MoE's term plan: the packed plan (16 tokens a tile, one MMA per K step) where experts average at most
// kPackRowsPerExpert rows, the stacked plan (128 tokens a tile, one MMA per term) above.
constexpr long long kPackRowsPerExpert = 64;    // measured: packed faster at T = 512, slower at 1024 (k 4, E 32)
void set_term_plan(gpt::PrefillArgs& a) {
    a.terms = g_prefill_terms.load();
    const int pk = g_prefill_pack.load();
    a.pack = pk >= 0 ? pk : ((long long)a.T * a.k <= kPackRowsPerExpert * a.E ? 1 : 0);
}
long long* g_trace = nullptr;          // device buffer for pipeline traces, installed by gptoss_trace_enable

[[noreturn]] void not_built(const char* what) {
    throw std::runtime_error(std::string(what) + ": not part of this build (the B200 MoE path); see gptoss.h");
}

}  // namespace

struct gptoss_moe_layer {
    const float* norm_w;
    float eps;
    const void* router_w;
    const float* router_b;
    const float* gu_bias;
    const float* dn_bias;
    int E, k, H, I;
    float alpha, limit;
    uint8_t* sfa_gu = nullptr;
    uint8_t* sfa_dn = nullptr;
    double* w64 = nullptr;                     // router weights as fp64 [H][32] for the batched router
    CUtensorMap tg, td;
    CUtensorMap td64;                          // down blocks in 64-byte boxes (the row-job decode kernel)
    uint8_t* dn_img = nullptr;                 // the row-job kernel's pre-packed down stages
    ~gptoss_moe_layer() {
        if (dn_img) cudaFree(dn_img);
        if (sfa_gu) cudaFree(sfa_gu);
        if (sfa_dn) cudaFree(sfa_dn);
        if (w64) cudaFree(w64);
    }
};

namespace gpt {

size_t moe_layer_workspace_bytes(int k, int H, int I) { return decode_tc_layout(k, H, I).bytes; }

// The fused decode kernel of a prepared layer with the given workspace (decode_tc_layout(k, H, I).bytes, zero-filled
// before its first use, used by one stream at a time).
void moe_layer_forward_ws(gptoss_moe_layer* l, const float* x, float* x_resid, cudaStream_t s, void* const* events,
                          void* workspace) {
    const DecodeTcLayout L = decode_tc_layout(l->k, l->H, l->I);
    char* w = static_cast<char*>(workspace);
    int* ids = reinterpret_cast<int*>(w + L.off_misc + ((size_t(l->H) * 4 + 127) & ~size_t(127)));
    float* gw = reinterpret_cast<float*>(ids + 32);
    auto rec = [&](int i) {
        if (events) GPT_CHECK(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(events[i]), s, cudaEventRecordExternal));
    };
    rec(0);
    rec(1);
    rec(2);
    DecodeTcArgs a{};
    a.tmap_gu = &l->tg;
    a.tmap_dn = &l->td;
    a.tmap_dn64 = &l->td64;
    a.plan = decode_plan();
    a.dn_img = l->dn_img;
    a.sfa_gu = l->sfa_gu;
    a.sfa_dn = l->sfa_dn;
    a.sfa_by_slot = 0;
    a.gu_bias = l->gu_bias;
    a.dn_bias = l->dn_bias;
    a.router_w = l->router_w;
    a.router_b = l->router_b;
    a.norm_w = l->norm_w;
    a.eps = l->eps;
    a.E = l->E;
    a.x = x;
    a.ids_out = ids;
    a.w_out = gw;
    a.x_resid = x_resid;
    a.k = l->k;
    a.H = l->H;
    a.I = l->I;
    a.alpha = l->alpha;
    a.limit = l->limit;
    a.workspace = w;
    a.trace = g_trace;
    launch_moe_decode_tc(a, s);
    rec(3);
}

}  // namespace gpt

namespace {
// Workspace of the batched path, owned by the calling thread, one per device (grow-only).
thread_local Scratch g_pws;
thread_local Scratch g_pws_sf;

// Private workspace of the expert-parallel path (per calling thread and device, grow-only).
thread_local Scratch g_ews;

void check_prefill_error(char* ws, const gpt::PrefillLayout& L) {
    int h = 0;
    GPT_CHECK(cudaMemcpy(&h, ws + L.off_misc + 256, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) throw std::runtime_error("moe_batched: device-side check failed (code " + std::to_string(h) + ")");
}
}  // namespace

extern "C" {

const char* gptoss_last_error(void) { return g_error.c_str(); }

// ---- engine (runtime/include/gptoss/gptoss.h:14-42): gpt::Engine in engine.cu
struct gptoss_engine {
    gpt::Engine impl;
    gptoss_engine(const char* dir, int max_ctx, long long budget) : impl(dir, max_ctx, budget) {}
};

gptoss_engine* gptoss_create(const char* model_dir, int max_ctx, long long vram_budget_bytes) {
    gptoss_engine* e = nullptr;
    guard([&] {
        if (!model_dir) throw std::runtime_error("create: null model_dir");
        e = new gptoss_engine(model_dir, max_ctx, vram_budget_bytes);
    });
    return e;
}
void gptoss_destroy(gptoss_engine* e) { delete e; }
int gptoss_vocab(const gptoss_engine* e) { return e ? e->impl.vocab() : -1; }
int gptoss_position(const gptoss_engine* e) { return e ? e->impl.position() : -1; }
long long gptoss_device_bytes(const gptoss_engine* e) { return e ? e->impl.device_bytes() : -1; }

namespace {
gpt::Engine& eng(gptoss_engine* e) {
    if (!e) throw std::runtime_error("null engine");
    return e->impl;
}
}  // namespace

int gptoss_reset(gptoss_engine* e) { return guard([&] { eng(e).reset(); }); }
int gptoss_use_graph(gptoss_engine* e, int on) { return guard([&] { eng(e).use_graph(on != 0); }); }
int gptoss_step(gptoss_engine* e, int token) { return guard([&] { eng(e).step(token); }); }
int gptoss_logits(gptoss_engine* e, float* out) {
    return guard([&] {
        if (!out) throw std::runtime_error("logits: null output");
        eng(e).copy_logits(out);
    });
}
int gptoss_prefill(gptoss_engine* e, const int32_t* tokens, int n, const int32_t* ids, int k, float* lp,
                   int32_t* argmax, float* target_lp) {
    return guard([&] {
        if (!tokens) throw std::runtime_error("prefill: null tokens");
        if (ids && (k < 0 || !lp || !argmax || !target_lp)) throw std::runtime_error("prefill: bad scoring arguments");
        eng(e).prefill(tokens, n, ids, k, lp, argmax, target_lp);
    });
}
int gptoss_score(gptoss_engine* e, const int32_t* ids, int k, int target, float* lp, int32_t* argmax,
                 float* target_lp, float* lse) {
    return guard([&] { eng(e).score(ids, k, target, lp, argmax, target_lp, lse); });
}
int gptoss_set_position(gptoss_engine* e, int pos) { return guard([&] { eng(e).set_position(pos); }); }
int gptoss_bench_steps(gptoss_engine* e, int token, int n) { return guard([&] { eng(e).bench_steps(token, n); }); }
int gptoss_generate_greedy(gptoss_engine* e, int token, int n, int32_t* out_tokens) {
    return guard([&] { eng(e).greedy(token, n, out_tokens); });
}
int gptoss_kv_fill_random(gptoss_engine* e, int positions, unsigned long long seed) {
    return guard([&] { eng(e).kv_fill_random(positions, seed); });
}

int gptoss_kernel_gemv_bf16(const void* W, const float* x, const float* bias, const float* resid, float* y, int N,
                            int K) {
    return guard([&] {
        gpt::launch_gemv_bf16(W, x, nullptr, 0.f, bias, resid, y, N, K, nullptr, false);
        sync_check("gemv_bf16");
    });
}

int gptoss_kernel_rope_append(float* qkv, const float* cos_t, const float* sin_t, int pos, void* k_cache,
                              void* v_cache, int window) {
    return guard([&] {
        if (pos < 0 || window < 0) throw std::runtime_error("rope_append: pos and window must be >= 0");
        gpt::launch_rope_append(qkv, cos_t, sin_t, nullptr, pos, k_cache, v_cache, window, nullptr, false);
        sync_check("rope_append");
    });
}

int gptoss_kernel_attention(const float* q, const void* k_cache, const void* v_cache, const float* sinks, int pos,
                            int window, int max_ctx, float* out) {
    return guard([&] {
        if (pos < 0 || window < 0) throw std::runtime_error("attention: pos and window must be >= 0");
        if (window == 0 && pos >= max_ctx) throw std::runtime_error("attention: pos must be below max_ctx");
        float* part = static_cast<float*>(g_scratch.get(gpt::attention_workspace_floats() * sizeof(float)));
        gpt::launch_attention(q, k_cache, v_cache, sinks, nullptr, pos, window, part, out, nullptr, false);
        sync_check("attention");
    });
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
        if (moe_impl_tc() && decode_tc_ok(k, H, I)) {
            const gpt::DecodeTcLayout L = gpt::decode_tc_layout(k, H, I);
            void* ws = g_dws.for_layout(L, k, H, I, nullptr);
            moe_tc_raw(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, x_norm, ids, weights, x_resid, k,
                       H, I, alpha, limit, ws, L, nullptr);
            sync_check("moe");
            check_tc_error(ws, L);
            return;
        }
        void* scratch = g_scratch.get(gpt::moe_decode_scratch_bytes(k, I));
        gpt::launch_moe_decode_simt(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, x_norm, ids,
                                    weights, x_resid, k, H, I, alpha, limit, scratch, nullptr);
        sync_check("moe");
    });
}

// ---- gptoss_kernel_moe_static_scratch: the CUDA-core MoE with its scratch in a fixed device array
//
// The only scratch of the CUDA-core path is the SwiGLU output a[k][I] (fp32), written in full by the gate/up kernel
// before the down kernel reads it, so it needs no zeroing between calls. Here it lives in one file-scope device
// array per device (kStaticScratchFloats floats = 96 KiB: k <= 8 experts of I <= 3072) instead of memory obtained
// from cudaMalloc. Its device address comes from cudaGetSymbolAddress, looked up once per device on the first call
// made with that device current, and is then passed to the kernels like any scratch pointer.
constexpr size_t kStaticScratchFloats = size_t(8) * 3072;
static __device__ __align__(256) float g_moe_static_scratch[kStaticScratchFloats];

namespace {
std::mutex g_static_mu;
void* g_static_addr[64] = {};

void* static_scratch_address() {
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("moe_static_scratch: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_moe_static_scratch);
        if (e != cudaSuccess || !p)
            throw std::runtime_error(std::string("moe_static_scratch: cudaGetSymbolAddress failed: ") +
                                     cudaGetErrorString(e));
        g_static_addr[dev] = p;
    }
    return g_static_addr[dev];
}
}  // namespace

int gptoss_kernel_moe_static_scratch(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                                     const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                                     const float* x_norm, const int32_t* ids, const float* weights, float* x_resid,
                                     int k, int H, int I, float alpha, float limit) {
    return guard([&] {
        if (k < 1 || k > 8) throw std::runtime_error("moe_static_scratch: k must be in 1..8");
        if (I < 1 || size_t(k) * size_t(I) > kStaticScratchFloats)
            throw std::runtime_error("moe_static_scratch: k * I = " + std::to_string(size_t(k) * size_t(I)) +
                                     " exceeds the fixed scratch of " + std::to_string(kStaticScratchFloats) +
                                     " floats (k <= 8 with I <= 3072)");
        void* scratch = static_scratch_address();
        gpt::launch_moe_decode_simt(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, x_norm, ids,
                                    weights, x_resid, k, H, I, alpha, limit, scratch, nullptr);
        sync_check("moe_static_scratch");
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
            if (events) GPT_CHECK(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(events[i]), s, cudaEventRecordExternal));
        };
        if (moe_impl_tc() && decode_tc_ok(k, H, I)) {
            // raw scales: the router runs first (its ids select which scales to repack), then the fused kernel
            const gpt::DecodeTcLayout L = gpt::decode_tc_layout(k, H, I);
            char* tw = static_cast<char*>(g_dws.for_layout(L, k, H, I, s));
            float* th = reinterpret_cast<float*>(tw + L.off_misc);
            int* tids = reinterpret_cast<int*>(tw + L.off_misc + ((size_t(H) * 4 + 127) & ~size_t(127)));
            float* tgw = reinterpret_cast<float*>(tids + 32);
            rec(0);
            gpt::launch_router_decode(static_cast<const __nv_bfloat16*>(router_w), router_b, x, E, H, k, tids, tgw, s,
                                      nullptr, nullptr, norm_w, eps, th);
            rec(1);
            rec(2);
            moe_tc_raw(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, th, tids, tgw, x_resid, k, H, I,
                       alpha, limit, tw, L, s);
            rec(3);
            return;
        }
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

int gptoss_selftest_mxf4_gemm_swizzle(const uint8_t* a_blocks, const uint8_t* a_scales, const uint8_t* b_blocks,
                                      const uint8_t* b_scales, float* d, int N, int K, int a_swizzle) {
    return guard([&] {
        const size_t bytes = size_t(1) << 22;
        void* scratch = g_scratch.get(bytes);
        gpt::selftest_mxf4_gemm(a_blocks, a_scales, b_blocks, b_scales, d, N, K, scratch, bytes, nullptr, a_swizzle);
    });
}

gptoss_moe_layer* gptoss_moe_layer_create(const float* norm_w, float eps, const void* router_w, const float* router_b,
                                          const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                                          const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                                          int E, int k, int H, int I, float alpha, float limit) {
    gptoss_moe_layer* L = nullptr;
    guard([&] {
        if (!tc_shape_ok(k, H, I) || E < k || E > 32)
            throw std::runtime_error("moe_layer_create: need 1 <= k <= 8, k <= E <= 32, H % 64 == 0, I % 64 == 0");
        auto* l = new gptoss_moe_layer{norm_w, eps, router_w, router_b, gu_bias, dn_bias, E, k, H, I, alpha, limit};
        try {
            GPT_CHECK(cudaMalloc(&l->sfa_gu, gpt::sf_repacked_bytes(E, 2 * I, H / 32, gpt::kDecodeTileRows)));
            GPT_CHECK(cudaMalloc(&l->sfa_dn, gpt::sf_repacked_bytes(E, H, I / 32, gpt::kDecodeTileRows)));
            // every scale byte of every expert passes through the repack once, which also refuses 0xFF (NaN)
            with_nan_scale_check("moe_layer_create", [&](int* flag) {
                gpt::launch_repack_sf(gu_scales, l->sfa_gu, E, 2 * I, H / 32, nullptr, nullptr, gpt::kDecodeTileRows,
                                      flag, kNanScaleCode);
                gpt::launch_repack_sf(dn_scales, l->sfa_dn, E, H, I / 32, nullptr, nullptr, gpt::kDecodeTileRows,
                                      flag, kNanScaleCode);
            });
            l->tg = gpt::make_tmap_u8_sw128_3d(gu_blocks, H / 2, 2 * I, E, 128, gpt::kDecodeTileRows);
            l->td = gpt::make_tmap_u8_sw128_3d(dn_blocks, I / 2, H, E, 128, gpt::kDecodeTileRows);
            l->td64 = gpt::make_tmap_u8_swz_3d(dn_blocks, I / 2, H, E, 64, gpt::kDecodeTileRows, 64);
            if (gpt::decode_rows_ok(k, H, I, E)) {    // the row-job kernel's down stages, one bulk copy each
                GPT_CHECK(cudaMalloc(&l->dn_img, gpt::down_jobs_bytes(E, H, I)));
                gpt::launch_pack_down_jobs(dn_blocks, l->sfa_dn, l->dn_img, E, H, I, nullptr);
            }
            GPT_CHECK(cudaMalloc(&l->w64, size_t(H) * 32 * sizeof(double)));
            gpt::launch_router_w64(router_w, E, H, l->w64, nullptr);
            sync_check("moe_layer_create");
        } catch (...) {
            delete l;
            throw;
        }
        L = l;
    });
    return L;
}

int gptoss_kernel_router_batched(const void* W, const float* b, const float* x, int E, int H, int k, int T,
                                 int32_t* ids, float* weights) {
    return guard([&] {
        // shapes are checked before any device work (the batched router repeats the checks)
        if (T < 1 || E < 1 || E > 32 || k < 1 || k > 8 || k > E || H < 8 || H % 8)
            throw std::runtime_error("router_batched: need T >= 1, 1 <= k <= 8, k <= E <= 32, H % 8 == 0");
        double* w64 = static_cast<double*>(g_scratch.get(size_t(H) * 32 * sizeof(double)));
        gpt::launch_router_w64(W, E, H, w64, nullptr);
        gpt::launch_router_batched(w64, b, x, nullptr, 0.f, T, E, H, k, nullptr, ids, weights, nullptr);
        sync_check("router_batched");
    });
}

int gptoss_moe_route_batched(const void* W, const float* b, const float* x, const float* norm_w, float eps, int E,
                             int H, int k, int T, float* h_out, int32_t* ids, float* weights, void* stream) {
    return guard([&] {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        double* w64 = static_cast<double*>(g_scratch.get(size_t(H) * 32 * sizeof(double)));
        gpt::launch_router_w64(W, E, H, w64, s);
        gpt::launch_router_batched(w64, b, x, norm_w, eps, T, E, H, k, h_out, ids, weights, s);
    });
}

int gptoss_kernel_moe_batched(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                              const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                              const float* x_norm, const int32_t* ids, const float* weights, float* x_resid, int T,
                              int k, int H, int I, float alpha, float limit) {
    return guard([&] {
        if (T < 1 || k < 1 || k > 8) throw std::runtime_error("moe_batched: need T >= 1 and 1 <= k <= 8");
        if (!tc_shape_ok(k, H, I)) throw std::runtime_error("moe_batched: H and I must be multiples of 64");
        // The expert count is not part of this ABI: the largest id in use bounds the experts read.
        std::vector<int32_t> hid(size_t(T) * k);
        GPT_CHECK(cudaMemcpy(hid.data(), ids, hid.size() * sizeof(int32_t), cudaMemcpyDeviceToHost));
        int E = 0;
        for (int32_t v : hid) {
            if (v < 0 || v >= 32) throw std::runtime_error("moe_batched: expert ids must be in 0..31");
            E = std::max(E, int(v) + 1);
        }
        E = std::max(E, k);
        const size_t sgu = gpt::sf_repacked_bytes(E, 2 * I, H / 32, gpt::kDecodeTileRows);
        const size_t sdn = gpt::sf_repacked_bytes(E, H, I / 32, gpt::kDecodeTileRows);
        uint8_t* sf = static_cast<uint8_t*>(g_pws_sf.get(sgu + sdn));
        with_nan_scale_check("moe_batched", [&](int* flag) {
            gpt::launch_repack_sf(gu_scales, sf, E, 2 * I, H / 32, nullptr, nullptr, gpt::kDecodeTileRows, flag,
                                  kNanScaleCode);
            gpt::launch_repack_sf(dn_scales, sf + sgu, E, H, I / 32, nullptr, nullptr, gpt::kDecodeTileRows, flag,
                                  kNanScaleCode);
        });
        const CUtensorMap tg = gpt::make_tmap_u8_sw128_3d(gu_blocks, H / 2, 2 * I, E, 128, gpt::kDecodeTileRows);
        const CUtensorMap td = gpt::make_tmap_u8_sw128_3d(dn_blocks, I / 2, H, E, 128, gpt::kDecodeTileRows);
        const gpt::PrefillLayout L = gpt::prefill_layout(T, k, E, H, I);
        char* ws = static_cast<char*>(g_pws.get(L.bytes));
        GPT_CHECK(cudaMemset(ws + L.off_misc, 0, 1024));
        gpt::PrefillArgs a{};
        a.tmap_gu = &tg;
        a.tmap_dn = &td;
        a.sf_gu = sf;
        a.sf_dn = sf + sgu;
        a.gu_bias = gu_bias;
        a.dn_bias = dn_bias;
        a.h = x_norm;
        a.ids = ids;
        a.weights = weights;
        a.x_resid = x_resid;
        a.T = T;
        a.k = k;
        a.E = E;
        a.H = H;
        a.I = I;
        a.alpha = alpha;
        a.limit = limit;
        a.workspace = ws;
        a.trace = g_trace;
        set_term_plan(a);
        gpt::launch_moe_batched(a, nullptr);
        sync_check("moe_batched");
        check_prefill_error(ws, L);
    });
}

int gptoss_moe_layer_forward_batched(gptoss_moe_layer* l, const float* x, float* x_resid, int T, void* stream,
                                     void* const* events) {
    return guard([&] {
        if (!l) throw std::runtime_error("moe_layer_forward_batched: null layer");
        if (T < 1) throw std::runtime_error("moe_layer_forward_batched: T must be positive");
        const gpt::PrefillLayout L = gpt::prefill_layout(T, l->k, l->E, l->H, l->I);
        char* ws = static_cast<char*>(g_pws.get(L.bytes));
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        GPT_CHECK(cudaMemsetAsync(ws + L.off_misc, 0, 1024, s));
        float* h = reinterpret_cast<float*>(ws + L.off_h);
        int* ids = reinterpret_cast<int*>(ws + L.off_ids);
        float* wts = reinterpret_cast<float*>(ws + L.off_w);
        gpt::launch_router_batched(l->w64, l->router_b, x, l->norm_w, l->eps, T, l->E, l->H, l->k, h, ids, wts, s);
        gpt::PrefillArgs a{};
        a.tmap_gu = &l->tg;
        a.tmap_dn = &l->td;
        a.sf_gu = l->sfa_gu;
        a.sf_dn = l->sfa_dn;
        a.gu_bias = l->gu_bias;
        a.dn_bias = l->dn_bias;
        a.h = h;
        a.ids = ids;
        a.weights = wts;
        a.x_resid = x_resid;
        a.T = T;
        a.k = l->k;
        a.E = l->E;
        a.H = l->H;
        a.I = l->I;
        a.alpha = l->alpha;
        a.limit = l->limit;
        a.workspace = ws;
        a.trace = g_trace;
        a.events = events;
        set_term_plan(a);
        gpt::launch_moe_batched(a, s);
    });
}

int gptoss_moe_layer_experts_batched(gptoss_moe_layer* l, const float* h, const int32_t* ids, const float* weights,
                                     float* x_resid, int T, int k, void* stream) {
    return guard([&] {
        if (!l) throw std::runtime_error("moe_layer_experts_batched: null layer");
        if (T < 1 || k < 1 || k > 8 || k > l->E)
            throw std::runtime_error("moe_layer_experts_batched: need T >= 1 and 1 <= k <= min(8, E)");
        const gpt::PrefillLayout L = gpt::prefill_layout(T, k, l->E, l->H, l->I);
        char* ws = static_cast<char*>(g_pws.get(L.bytes));
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        GPT_CHECK(cudaMemsetAsync(ws + L.off_misc, 0, 1024, s));
        gpt::PrefillArgs a{};
        a.tmap_gu = &l->tg;
        a.tmap_dn = &l->td;
        a.sf_gu = l->sfa_gu;
        a.sf_dn = l->sfa_dn;
        a.gu_bias = l->gu_bias;
        a.dn_bias = l->dn_bias;
        a.h = h;
        a.ids = ids;
        a.weights = weights;
        a.x_resid = x_resid;
        a.T = T;
        a.k = k;
        a.E = l->E;
        a.H = l->H;
        a.I = l->I;
        a.alpha = l->alpha;
        a.limit = l->limit;
        a.workspace = ws;
        a.trace = g_trace;
        set_term_plan(a);
        gpt::launch_moe_batched(a, s);
    });
}

void gptoss_moe_layer_destroy(gptoss_moe_layer* layer) { delete layer; }

int gptoss_moe_layer_forward(gptoss_moe_layer* l, const float* x, float* x_resid, void* stream, void* const* events) {
    return guard([&] {
        if (!l) throw std::runtime_error("moe_layer_forward: null layer");
        const gpt::DecodeTcLayout L = gpt::decode_tc_layout(l->k, l->H, l->I);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        gpt::moe_layer_forward_ws(l, x, x_resid, s, events, g_dws.for_layout(L, l->k, l->H, l->I, s));
    });
}

int gptoss_selftest_mxf4_mma_ns(int n, double* ns) {
    return guard([&] {
        if (!ns) throw std::runtime_error("selftest_mxf4_mma_ns: null output");
        int* err = static_cast<int*>(g_flag.get(sizeof(int)));
        GPT_CHECK(cudaMemset(err, 0, sizeof(int)));
        const double t = gpt::selftest_mxf4_mma_ns(n, err);
        sync_check("selftest_mxf4_mma_ns");
        int h = 0;
        GPT_CHECK(cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (h) throw std::runtime_error("selftest_mxf4_mma_ns: a wait gave up");
        *ns = t;
    });
}

int gptoss_selftest_mxf4_peak(double* tflops) {
    return guard([&] {
        if (!tflops) throw std::runtime_error("selftest_mxf4_peak: null output");
        int* err = static_cast<int*>(g_flag.get(sizeof(int)));
        GPT_CHECK(cudaMemset(err, 0, sizeof(int)));
        const double t = gpt::selftest_mxf4_peak(err);
        sync_check("selftest_mxf4_peak");
        int h = 0;
        GPT_CHECK(cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (h) throw std::runtime_error("selftest_mxf4_peak: a wait gave up");
        *tflops = t;
    });
}

int gptoss_selftest_terms(const float* x, int n, float* out, float* per_term, int which) {
    return guard([&] {
        const size_t bytes = size_t(n / 256 + 1) * gpt::kDecodeTerms * 128 + size_t(n / 128 + 1) * 512;
        gpt::selftest_terms(x, n, out, per_term, which, g_scratch.get(bytes), bytes, nullptr);
    });
}

int gptoss_trace_enable(void* device_buffer, long long bytes) {
    return guard([&] {
        if (device_buffer && bytes < 160LL * 160 * 8)
            throw std::runtime_error("trace buffer too small: need 160 * 160 * 8 bytes");
        g_trace = static_cast<long long*>(device_buffer);
    });
}

int gptoss_router_w64(const void* W, int E, int H, double* w64, void* stream) {
    return guard([&] {
        if (E < 1 || E > 32 || H < 1) throw std::runtime_error("router_w64: need 1 <= E <= 32, H >= 1");
        gpt::launch_router_w64(W, E, H, w64, static_cast<cudaStream_t>(stream));
    });
}

int gptoss_ep_region_bytes(int E, int k, int H, int I, int world, int T_max, long long* bytes) {
    return guard([&] {
        if (!bytes) throw std::runtime_error("ep_region_bytes: null output");
        *bytes = (long long)gpt::ep_layout(T_max, k, E, world, H, I).region_bytes;
    });
}

int gptoss_ep_region_alloc(long long bytes, void** region) {
    return guard([&] {
        if (!region || bytes <= 0) throw std::runtime_error("ep_region_alloc: bad arguments");
        *region = nullptr;
        GPT_CHECK(cudaMalloc(region, size_t(bytes)));
        GPT_CHECK(cudaMemset(*region, 0, size_t(bytes)));
    });
}

int gptoss_ep_region_free(void* region) {
    return guard([&] { GPT_CHECK(cudaFree(region)); });
}

int gptoss_ipc_handle(void* device_ptr, void* handle_out) {
    return guard([&] {
        static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
        cudaIpcMemHandle_t hd;
        GPT_CHECK(cudaIpcGetMemHandle(&hd, device_ptr));
        std::memcpy(handle_out, &hd, sizeof(hd));
    });
}

int gptoss_ipc_open(const void* handle, void** device_ptr) {
    return guard([&] {
        cudaIpcMemHandle_t hd;
        std::memcpy(&hd, handle, sizeof(hd));
        GPT_CHECK(cudaIpcOpenMemHandle(device_ptr, hd, cudaIpcMemLazyEnablePeerAccess));
    });
}

int gptoss_ipc_close(void* device_ptr) {
    return guard([&] { GPT_CHECK(cudaIpcCloseMemHandle(device_ptr)); });
}

int gptoss_ep_layer_forward(gptoss_moe_layer* l, const double* router_w64, const float* router_b, const float* norm_w,
                            float eps, int E, int rank, int world, const float* x, float* x_resid, int T, int T_max,
                            void* const* peers, unsigned epoch, void* stream) {
    return guard([&] {
        if (!l || !peers) throw std::runtime_error("ep_layer_forward: null layer or peer table");
        if (world < 1 || world > 8 || E % world || l->E != E / world)
            throw std::runtime_error("ep_layer_forward: the layer must hold E / world experts, 1 <= world <= 8");
        if (epoch == 0) throw std::runtime_error("ep_layer_forward: epochs start at 1");
        const gpt::EpLayout L = gpt::ep_layout(T_max, l->k, E, world, l->H, l->I);
        gpt::EpArgs a{};
        a.tmap_gu = &l->tg;
        a.tmap_dn = &l->td;
        a.sf_gu = l->sfa_gu;
        a.sf_dn = l->sfa_dn;
        a.gu_bias = l->gu_bias;
        a.dn_bias = l->dn_bias;
        a.w64 = router_w64;
        a.router_b = router_b;
        a.norm_w = norm_w;
        a.eps = eps;
        a.x = x;
        a.x_resid = x_resid;
        a.T = T;
        a.T_max = T_max;
        a.k = l->k;
        a.E = E;
        a.H = l->H;
        a.I = l->I;
        a.rank = rank;
        a.world = world;
        a.alpha = l->alpha;
        a.limit = l->limit;
        a.peers = peers;
        a.epoch = epoch;
        a.local_ws = g_ews.get(L.local_bytes);
        a.trace = g_trace;
        a.terms = g_prefill_terms.load();
        gpt::launch_ep_layer(a, static_cast<cudaStream_t>(stream));
    });
}

int gptoss_ep_status(int E, int k, int H, int I, int world, int T_max, int* code) {
    return guard([&] {
        const gpt::EpLayout L = gpt::ep_layout(T_max, k, E, world, H, I);
        char* ws = static_cast<char*>(g_ews.get(L.local_bytes));
        GPT_CHECK(cudaDeviceSynchronize());
        int h = 0;
        GPT_CHECK(cudaMemcpy(&h, ws + L.off_misc + 256, sizeof(int), cudaMemcpyDeviceToHost));
        *code = h;
    });
}

int gptoss_test_decode_epoch(int k, int H, int I, unsigned set_to, unsigned* previous) {
    return guard([&] {
        if (!tc_shape_ok(k, H, I)) throw std::runtime_error("test_decode_epoch: not a tensor-core decode shape");
        const gpt::DecodeTcLayout L = gpt::decode_tc_layout(k, H, I);
        char* w = static_cast<char*>(g_dws.for_layout(L, k, H, I, nullptr));
        unsigned* word = reinterpret_cast<unsigned*>(w + L.off_err + 256) + 4;   // grid-barrier word 4: the epoch
        GPT_CHECK(cudaDeviceSynchronize());
        unsigned prev = 0;
        GPT_CHECK(cudaMemcpy(&prev, word, sizeof(prev), cudaMemcpyDeviceToHost));
        GPT_CHECK(cudaMemcpy(word, &set_to, sizeof(set_to), cudaMemcpyHostToDevice));
        if (previous) *previous = prev;
    });
}

int gptoss_set_prefill_terms(int terms) {
    if (terms < 1 || terms > 8) {
        g_error = "gptoss_set_prefill_terms: terms must be 1 .. 8";
        return -1;
    }
    return g_prefill_terms.exchange(terms);
}

int gptoss_set_prefill_packing(int mode) {
    if (mode < -1 || mode > 1) {
        g_error = "gptoss_set_prefill_packing: mode must be -1 (by batch size), 0 (stacked) or 1 (packed)";
        return -2;
    }
    return g_prefill_pack.exchange(mode);
}

int gptoss_set_attention_impl(int impl) {
    if (impl < 0 || impl > 1) {
        g_error = "gptoss_set_attention_impl: impl must be 0 (three launches) or 1 (one cooperative launch)";
        return -1;
    }
    return gpt::g_attn_impl.exchange(impl);
}

int gptoss_set_moe_impl(int impl) {
    if (impl < 0 || impl > 2) {
        g_error = "gptoss_set_moe_impl: impl must be 0 (SIMT), 1 (tensor cores) or 2 (tensor cores, stream-K kernel)";
        return -1;
    }
    const int prev = g_moe_impl;
    g_moe_impl = impl;
    return prev;
}

}  // extern "C"
