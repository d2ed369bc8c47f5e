/* C ABI of the B200-native gpt-oss MXFP4 MoE path.
 *
 * Drop-in for openvang/gptoss-infer's runtime/include/gptoss/gptoss.h: every function of that header is declared
 * here with the same signature, the same argument meaning and the same error convention (0 on success, -1 on
 * failure with the message in gptoss_last_error(), a thread-local string; exceptions never cross the ABI). Kernel
 * entry points take caller-owned DEVICE pointers and synchronize the device before returning, as the reference's
 * do (reference capi.cpp:34-37). Not thread-safe: use one engine per thread.
 *
 * Functions marked [extension] do not exist in the reference; they are additive.
 */
#ifndef GPTOSS_H
#define GPTOSS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gptoss_engine gptoss_engine;

/* ---- Engine lifecycle and decode (reference gptoss.h:14-42) ------------------------------------------------ */

/* Loads the checkpoint in model_dir (config.json, optional generation_config.json, safetensors with Hugging Face
 * names, MXFP4 experts) onto the current CUDA device; returns NULL on failure (reference gptoss.h:14-17).
 * vram_budget_bytes > 0 caps the engine's own device allocations. Geometry: 64 query heads, 8 key/value heads, head
 * dim 64, hidden and intermediate multiples of 64 with hidden <= 3072, k <= E <= 32, k <= 8 (gpt-oss-20b and -120b).
 * A step runs embed, 24 x (RMSNorm + QKV GEMV, RoPE + fp16 KV append, split-K attention with sinks and sliding
 * window, O GEMV + residual, the fused tensor-core MoE), final RMSNorm + LM head, captured once as a CUDA graph. */
gptoss_engine* gptoss_create(const char* model_dir, int max_ctx, long long vram_budget_bytes);
void gptoss_destroy(gptoss_engine* e);                                   /* reference gptoss.h:18 */
const char* gptoss_last_error(void);                                     /* reference gptoss.h:19 */
int gptoss_vocab(const gptoss_engine* e);                                /* reference gptoss.h:21 */
int gptoss_position(const gptoss_engine* e);                             /* reference gptoss.h:22 */
long long gptoss_device_bytes(const gptoss_engine* e);                   /* reference gptoss.h:23 */
int gptoss_reset(gptoss_engine* e);                                      /* reference gptoss.h:25 */
int gptoss_use_graph(gptoss_engine* e, int on);                          /* reference gptoss.h:26 */
int gptoss_step(gptoss_engine* e, int token);                            /* reference gptoss.h:27-28 */
int gptoss_logits(gptoss_engine* e, float* out);                         /* reference gptoss.h:29 */
int gptoss_prefill(gptoss_engine* e, const int32_t* tokens, int n, const int32_t* ids, int k, float* lp,
                   int32_t* argmax, float* target_lp);                   /* reference gptoss.h:30-35 */
int gptoss_score(gptoss_engine* e, const int32_t* ids, int k, int target, float* lp, int32_t* argmax,
                 float* target_lp, float* lse);                          /* reference gptoss.h:36-38 */
int gptoss_set_position(gptoss_engine* e, int pos);                      /* reference gptoss.h:40-41 */
int gptoss_bench_steps(gptoss_engine* e, int token, int n);              /* reference gptoss.h:42 */
/* [extension] Greedy decode of n tokens from `token`: each step's argmax is found on the device and fed to the next
 * step without a host round trip; out_tokens (host, n entries, may be NULL) receives the generated tokens. Advances
 * the position by n. */
int gptoss_generate_greedy(gptoss_engine* e, int token, int n, int32_t* out_tokens);
/* [extension] Benchmarking: fills every layer's fp16 KV cache for positions 0 .. positions-1 with deterministic
 * N(0, 1) values (seeded) and sets the position to `positions`, standing in for a prefilled context. */
int gptoss_kv_fill_random(gptoss_engine* e, int positions, unsigned long long seed);

/* ---- Kernel entry points (reference gptoss.h:44-58). Device pointers; each call synchronizes. ------------- */

int gptoss_kernel_gemv_bf16(const void* W, const float* x, const float* bias, const float* resid, float* y, int N,
                            int K);                                      /* reference gptoss.h:45-46 */
/* y = x * rsqrt(mean(x^2) + eps) * w over n floats (reference gptoss.h:47). */
int gptoss_kernel_rmsnorm(const float* x, const float* w, float* y, int n, float eps);
int gptoss_kernel_rope_append(float* qkv, const float* cos_t, const float* sin_t, int pos, void* k_cache,
                              void* v_cache, int window);                /* reference gptoss.h:48-49 */
int gptoss_kernel_attention(const float* q, const void* k_cache, const void* v_cache, const float* sinks, int pos,
                            int window, int max_ctx, float* out);        /* reference gptoss.h:50-51 */
/* Router for one token (reference gptoss.h:52-53): logits = W[E,H] (bf16) x + b; ids = top-k sorted by logit
 * descending, ties to the lower expert id; weights = softmax over the k selected logits. 1 <= k <= 8, k <= E <= 32,
 * H % 8 == 0; anything else returns -1 (k > E included). */
int gptoss_kernel_router(const void* W, const float* b, const float* x, int E, int H, int k, int32_t* ids,
                         float* weights);
/* x_resid += sum_e w[e] * (W2[ids[e]] swiglu(W1[ids[e]] x_norm + b1) + b2)   (reference gptoss.h:54-58)
 * gu_blocks uint8 [E, 2I, H/32, 16], gu_scales uint8 [E, 2I, H/32], gu_bias fp32 [E, 2I],
 * dn_blocks uint8 [E, H, I/32, 16], dn_scales uint8 [E, H, I/32], dn_bias fp32 [E, H]; gate/up rows interleaved
 * (even = glu, clamped above at limit; odd = linear, clamped to [-limit, limit]). On the tensor-core path (the
 * default, for H % 64 == 0 and I % 64 == 0) an E8M0 scale byte 0xFF (NaN) of a selected expert returns -1. */
int gptoss_kernel_moe(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                      const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias, const float* x_norm,
                      const int32_t* ids, const float* weights, float* x_resid, int k, int H, int I, float alpha,
                      float limit);

/* ---- [extension] MoE-path entry points with no counterpart in the reference ------------------------------- */

/* [extension] No counterpart in the reference. gptoss_kernel_moe for callers that must not allocate device memory
 * during the call: for example an engine whose device memory is all handed to its own budgeted allocator, or a
 * decode loop where an allocation (and the device synchronization cudaMalloc may imply) is not acceptable. Same
 * arguments, semantics, layouts and synchronization as gptoss_kernel_moe, always on the CUDA-core path. Its only
 * scratch (the SwiGLU output, k * I floats) lives in a fixed device array of 8 * 3072 floats (96 KiB) per device, so
 * k * I must be at most 24576 (k <= 8 with I <= 3072); larger shapes return -1 with a message. Nothing in that array
 * needs to start at zero. The first call on each device looks up the array's address (with that device current)
 * and should come before any stream capture on that device. Calls that overlap on the same device (several host
 * threads) share the one array and race: serialize them. */
int gptoss_kernel_moe_static_scratch(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                                     const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                                     const float* x_norm, const int32_t* ids, const float* weights, float* x_resid,
                                     int k, int H, int I, float alpha, float limit);

/* [extension] Bit-exact MXFP4 decode of n_blocks blocks (16 bytes + 1 E8M0 scale each) into out[n_blocks * 32]
 * fp32, element 2j from the low nibble of byte j. Restates reference/gptoss_ref/mxfp4.py:17-31 on the GPU: returns
 * -1 if any scale is 0xFF (NaN in the OCP MX spec), as the reference's dequant raises. */
int gptoss_kernel_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, float* out, long long n_blocks);

/* [extension] One MoE block for one token, asynchronous: h = RMSNorm(x; norm_w, eps), router (W bf16 [E,H],
 * b fp32 [E]) as gptoss_kernel_router, then x_resid += MoE(h) as gptoss_kernel_moe. x_resid may alias x (the
 * residual stream). Runs on `stream` (a cudaStream_t; NULL = legacy default stream) and returns without
 * synchronizing; launch errors are reported, device faults surface at the caller's next synchronization.
 * `events`, if not NULL, points to 4 cudaEvent_t recorded before the router, before the gate/up GEMV, before the
 * down GEMV and after it (for per-kernel timing). Uses the calling thread's workspace: calls from one thread on
 * different streams must not overlap. Same expert layouts as gptoss_kernel_moe. */
int gptoss_moe_block_async(const float* x, const float* norm_w, float eps, const void* router_w,
                           const float* router_b, const uint8_t* gu_blocks, const uint8_t* gu_scales,
                           const float* gu_bias, const uint8_t* dn_blocks, const uint8_t* dn_scales,
                           const float* dn_bias, float* x_resid, int E, int k, int H, int I, float alpha, float limit,
                           void* stream, void* const* events);

/* [extension] A prepared MoE layer for the tensor-core decode path. Creation keeps the caller's device pointers
 * (they must stay valid for the handle's lifetime), repacks the E8M0 scales once into the tcgen05 scale-factor
 * layout (device memory owned by the handle, 24.9 MB for gpt-oss-20b's 32 experts) and builds the TMA descriptors;
 * returns NULL on failure (gptoss_last_error). Needs H % 64 == 0, I % 64 == 0, 1 <= k <= 8, k <= E <= 32.
 * An E8M0 scale byte 0xFF (NaN) in any expert fails the creation, as the reference's loader refuses it
 * (runtime/src/engine.cu:119-122). norm_w fp32 [H]; router_w bf16 [E,H]; router_b fp32 [E]; expert layouts as
 * gptoss_kernel_moe. Synchronizes. */
typedef struct gptoss_moe_layer gptoss_moe_layer;
gptoss_moe_layer* gptoss_moe_layer_create(const float* norm_w, float eps, const void* router_w, const float* router_b,
                                          const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                                          const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                                          int E, int k, int H, int I, float alpha, float limit);
void gptoss_moe_layer_destroy(gptoss_moe_layer* layer);
/* [extension] x_resid += MoE(RMSNorm(x)) for one token with a prepared layer, asynchronous on `stream` (a
 * cudaStream_t; NULL = legacy default stream): one persistent cooperative kernel (RMSNorm, router, top-k, softmax,
 * gate/up with SwiGLU, down with the weighted combine, all on tensor cores). x_resid may alias x. `events`, if not
 * NULL, points to 4 cudaEvent_t: [0], [1], [2] are recorded before the kernel and [3] after it. Calls from one
 * thread share its workspace and must not overlap on the GPU; the first call after a change of shape (k, H, I) on
 * that thread also clears the workspace's state words, on `stream`. */
int gptoss_moe_layer_forward(gptoss_moe_layer* layer, const float* x, float* x_resid, void* stream,
                             void* const* events);

/* [extension] Router for T tokens: ids[T][k] and weights[T][k] as gptoss_kernel_router computes them for each row
 * of x [T][H] (already normalized). fp64 logits from exact products; ties to the lower expert id. Device pointers;
 * synchronizes. */
int gptoss_kernel_router_batched(const void* W, const float* b, const float* x, int E, int H, int k, int T,
                                 int32_t* ids, float* weights);

/* [extension] Routing for T tokens, asynchronous on `stream`: h_out[T][H] = RMSNorm(x; norm_w, eps) (norm_w NULL:
 * h_out = x), ids[T][k] and weights[T][k] as gptoss_kernel_router_batched. Uses the calling thread's scratch for the
 * router weights in fp64: calls from one thread must not overlap on the GPU. */
int gptoss_moe_route_batched(const void* W, const float* b, const float* x, const float* norm_w, float eps, int E,
                             int H, int k, int T, float* h_out, int32_t* ids, float* weights, void* stream);

/* [extension] Batched (prefill) MoE on tensor cores: x_resid[t] += sum_s w[t][s] (W2[e] swiglu(W1[e] x_norm[t] + b1)
 * + b2) with e = ids[t][s], for T tokens (grouped GEMM over the experts: permute, tcgen05 block-scaled FP4 MMAs with
 * the activations split into e2m1 terms - 8 unless gptoss_set_prefill_terms says otherwise - unpermute,
 * slot-ordered combine). Layouts as gptoss_kernel_moe
 * with x_norm, ids, weights, x_resid of T rows; expert ids in 0..31; H and I multiples of 64; T <= 32768. An E8M0
 * scale byte 0xFF (NaN) in the experts up to the largest id used returns -1. Device pointers; synchronizes. */
int gptoss_kernel_moe_batched(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                              const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                              const float* x_norm, const int32_t* ids, const float* weights, float* x_resid, int T,
                              int k, int H, int I, float alpha, float limit);

/* [extension] x_resid[t] += MoE(RMSNorm(x[t])) for T tokens with a prepared layer (batched router, then the batched
 * MoE above), asynchronous on `stream`. x_resid may alias x. Uses the calling thread's batched-path workspace: calls
 * from one thread must not overlap on the GPU. events: NULL, or 4 cudaEvent_t recorded (external, so capturable)
 * before and after the gate/up grouped GEMM and before and after the down grouped GEMM. */
int gptoss_moe_layer_forward_batched(gptoss_moe_layer* layer, const float* x, float* x_resid, int T, void* stream,
                                     void* const* events);

/* [extension] The experts of a prepared layer applied to T given rows, asynchronous on `stream`: x_resid[t] +=
 * sum_s w[t][s] (W2[e] swiglu(W1[e] h[t] + b1) + b2) with e = ids[t][s] < the layer's E (the router is not used).
 * The building block of expert parallelism: a rank's layer holds only its own experts and gets the rows routed to
 * them. Same workspace rule as gptoss_moe_layer_forward_batched. */
int gptoss_moe_layer_experts_batched(gptoss_moe_layer* layer, const float* h, const int32_t* ids, const float* weights,
                                     float* x_resid, int T, int k, void* stream);

/* [extension] Expert parallelism with dispatch and combine in the kernels over NVLink peer memory (no counterpart in
 * the reference, which runs every expert on one device: an EP layer call that takes one rank's shard of the tokens).
 *
 * Every rank (one GPU each) allocates one zeroed region of gptoss_ep_region_bytes() with gptoss_ep_region_alloc(),
 * exports it with gptoss_ipc_handle() (64 bytes), receives every other rank's handle (any host channel) and maps
 * them with gptoss_ipc_open(). gptoss_ep_layer_forward() then runs one MoE layer for this rank's T <= T_max tokens:
 * routing over all E experts, each (token, slot) row's activation terms written straight into the owning rank's
 * region, the grouped GEMMs over the rows this rank received (its `layer` holds experts [rank E/world, (rank + 1)
 * E/world) and the full k), each result row written straight back into its source rank's region, and the combine
 * into x_resid in slot order: bit-identical to gptoss_moe_layer_forward_batched over all tokens on one GPU.
 * peers: host array of `world` device addresses (every rank's region as mapped on this device; peers[rank] is the
 * own region). epoch: the same value on every rank for one layer call, increasing from 1. All ranks must make the
 * same sequence of calls; a rank that stops makes the others' bounded waits (about a second) fail, reported by
 * gptoss_ep_status(). router_w64: the router as fp64 [H][32] (gptoss_router_w64). Asynchronous on `stream`. */
int gptoss_router_w64(const void* W /* bf16 [E,H] */, int E, int H, double* w64, void* stream);
int gptoss_ep_region_bytes(int E, int k, int H, int I, int world, int T_max, long long* bytes);
int gptoss_ep_region_alloc(long long bytes, void** region);
int gptoss_ep_region_free(void* region);
int gptoss_ipc_handle(void* device_ptr, void* handle_out /* 64 bytes */);
int gptoss_ipc_open(const void* handle /* 64 bytes */, void** device_ptr);
int gptoss_ipc_close(void* device_ptr);
int gptoss_ep_layer_forward(gptoss_moe_layer* layer, const double* router_w64, const float* router_b,
                            const float* norm_w, float eps, int E, int rank, int world, const float* x,
                            float* x_resid, int T, int T_max, void* const* peers, unsigned epoch, void* stream);
/* Synchronizes the device and returns in *code the calling thread's expert-parallel error word (0: none; 20 bad id,
 * 60-62 a cross-rank wait gave up, 31-36 a pipeline wait gave up). */
int gptoss_ep_status(int E, int k, int H, int I, int world, int T_max, int* code);

/* [extension] Self-test of the tensor-core block-scaled MMA path: D[128, N] (fp32, row-major) =
 * dequant(a_blocks [128, K/32, 16], a_scales [128, K/32]) . dequant(b_blocks [N, K/32, 16], b_scales [N, K/32])^T
 * computed by one CTA with TMA, tcgen05.cp scale factors and tcgen05.mma kind::mxf4. N % 8 == 0, 8 <= N <= 256,
 * K % 64 == 0, 64 <= K <= 1024. Device pointers; synchronizes. */
int gptoss_selftest_mxf4_gemm(const uint8_t* a_blocks, const uint8_t* a_scales, const uint8_t* b_blocks,
                              const uint8_t* b_scales, float* d, int N, int K);
/* [extension] The same with A loaded by TMA in the 64-byte swizzled layout (64-byte boxes of K, a_swizzle = 64; the
 * layout of the decode kernel's down-projection slices) or the 128-byte one (a_swizzle = 128). */
int gptoss_selftest_mxf4_gemm_swizzle(const uint8_t* a_blocks, const uint8_t* a_scales, const uint8_t* b_blocks,
                                      const uint8_t* b_scales, float* d, int N, int K, int a_swizzle);

/* [extension] Measures this GPU's dense block-scaled FP4 tensor rate (tcgen05.mma kind::mxf4, M = 128, N = 256,
 * K = 64, back to back on every SM, timed with CUDA events on the legacy default stream) and stores it in *tflops
 * (TFLOP/s). The denominator of the batched path's roofline. Synchronizes. */
int gptoss_selftest_mxf4_peak(double* tflops);

/* [extension] The same measurement for M = 128, N = n, K = 64 (n a multiple of 8 in 8..256): nanoseconds per MMA
 * issued back to back on one SM, every SM busy. How the MMA's cost depends on N (the decode kernels' operand choice).
 * Synchronizes. */
int gptoss_selftest_mxf4_mma_ns(int n, double* ns);

/* [extension] Pipeline tracing of the tensor-core decode kernel (profiling aid). With a device buffer of at least
 * 160 * 160 int64 installed, every later gptoss_moe_layer_forward stores, per CTA, up to 160 clock64 stamps of its
 * phases (the slot list is at the trace stamp helper in decode_tc.cu; unused slots keep their old contents). NULL
 * turns tracing off. A process-wide setting; not for concurrent use. */
int gptoss_trace_enable(void* device_buffer, long long bytes);

/* [extension] Self-test of the activation quantizer of the tensor-core path: splits x[n] (n % 256 == 0) into e2m1
 * residual terms with per-32 E8M0 scales (which = 0: comparison rounding, 1: the hardware converters, 2: the
 * fixed scale schedule with fp32 rounding, 3: the same computed by a whole warp per block, 4: the integer digit
 * split - one rounding, then the remainder's balanced octal digits - computed by a whole warp per block, as the
 * decode kernel's activations use it), decodes the terms back into out[n], and, if per_term is not NULL, stores the
 * first two terms into per_term[2][n]. Device pointers; synchronizes. */
int gptoss_selftest_terms(const float* x, int n, float* out, float* per_term, int which);

/* [extension] Test hook of the tensor-core decode path: on the current device, sets the launch-epoch word of the
 * calling thread's decode workspace for shape (k, H, I) to set_to (storing the old value in *previous if not NULL).
 * The next launch of that shape uses the epoch that follows set_to, which skips 0 when the count wraps. Synchronizes.
 * For tests of the wrap-around; a decode loop never needs it. */
int gptoss_test_decode_epoch(int k, int H, int I, unsigned set_to, unsigned* previous);

/* [extension] Which decode MoE implementation gptoss_kernel_moe, the prepared layers and the engine use: 0 = SIMT
 * (CUDA cores), 1 = tensor cores (tcgen05 block-scaled MMA) where the shape allows it: the row-job kernel (one CTA
 * per 256 gate/up rows of a selected expert, k * ceil(2I / 256) CTAs, at most the SM count) and otherwise the stream-K
 * kernel (one CTA per SM); 2 = tensor cores with the stream-K kernel only. Returns the previous setting, or -1. */
int gptoss_set_moe_impl(int impl);

/* [extension] How an engine's bs=1 decode step runs the attention block (RMSNorm, QKV projection, RoPE and cache
 * append, attention with sinks and window, O projection and residual): 0 (default) = three launches per layer (QKV
 * GEMV, attention, O GEMV), 1 = one cooperative launch per layer (three phases separated by grid-wide barriers; the
 * same logits to the engine's tolerance, measured slower on B200: 623 against 677 tok/s on configs[1]). Read when an
 * engine captures its step graph (its first step); returns the previous setting, or -1. */
int gptoss_set_attention_impl(int impl);

/* [extension] Activation terms of the batched (prefill) MoE, for every later batched and expert-parallel call in the
 * process: each 32-value block of the tensor-core operand is the sum of `terms` e2m1 terms under E8M0 scales, the
 * nearest such sum. 8 (the default) is exact to 2^-21 of each block's scale and meets the float64 bound of the
 * reference's tests; fewer terms run fewer MMAs at a larger error (measured per count in the tests and the bench).
 * Returns the previous count, or -1 (terms outside 1 .. 8). */
int gptoss_set_prefill_terms(int terms);

/* [extension] Tile plan of the batched MoE: 1 = packed (a token's terms are 8 rows of a 128-row tile, 16 tokens per
 * tile: one MMA per K step for experts with few rows), 0 = stacked (128 tokens per tile, one MMA per term), -1 (the
 * default) = packed while the experts average at most 64 rows (T * k <= 64 * E). Both give the same results within
 * the float64 bound. Returns the previous mode, or -2 (mode outside -1 .. 1). */
int gptoss_set_prefill_packing(int mode);

#ifdef __cplusplus
}
#endif

#endif /* GPTOSS_H */
