// Host-side launchers of the MoE-path kernels. Every launcher takes the stream to run on and throws
// std::runtime_error on invalid shapes or launch failure; the C ABI (capi.cu) turns that into -1.
#pragma once
#include <atomic>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

struct gptoss_moe_layer;

namespace gpt {

int num_sms();

// Residual e2m1 terms per activation value in the tensor-core decode path (the MMA's N).
constexpr int kDecodeTerms = 16;

// y[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w for T rows of n.
void launch_rmsnorm(const float* x, const float* w, float* y, int T, int n, float eps, cudaStream_t s);

// Bit-exact MXFP4 decode of n_blocks blocks (16 code bytes + 1 E8M0 byte each) into 32 floats per block.
// *bad is set to 1 if any scale byte is 0xFF (caller clears it first).
void launch_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, float* out, long long n_blocks, int* bad,
                          cudaStream_t s);

// Decode router for one token: logits = W[E,H] x + b accumulated exactly in fp64, top-k by (logit desc, id asc)
// with NaN never selected ahead of a number, softmax over the k selected fp32 logits.
// With xq_img != nullptr the router also writes its input as e2m1 residual terms (the tensor-core gate/up's B
// operand). With norm_w != nullptr the input is RMSNorm(x; norm_w, eps) computed in the kernel (and stored to h_out
// if given) instead of x itself.
void launch_router_decode(const __nv_bfloat16* W, const float* b, const float* x, int E, int H, int k, int* ids,
                          float* weights, cudaStream_t s, uint8_t* xq_img = nullptr, uint8_t* xq_sf = nullptr,
                          const float* norm_w = nullptr, float eps = 0.f, float* h_out = nullptr);

// Decode MoE for one token on raw checkpoint-layout MXFP4 experts (SIMT path).
//   a[slot][j] = swiglu(W1[ids[slot]] x + b1)          gate/up rows interleaved (even glu, odd linear)
//   x_resid[i] += sum_slot w[slot] (W2[ids[slot]] a[slot] + b2)[i]   summed in slot order
size_t moe_decode_scratch_bytes(int k, int I);
void launch_moe_decode_simt(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                            const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                            const float* x_norm, const int* ids, const float* weights, float* x_resid, int k,
                            int H, int I, float alpha, float limit, void* scratch, cudaStream_t s,
                            void* mid_event = nullptr);

// Scale-factor repack: raw E8M0 bytes [mats][rows][G] -> tcgen05 chunks of 512 bytes, chunk byte
// (r % 32) * 16 + (r / 32) * 4 + kb for row r (within its 128 rows) and k-block kb; zero padded. tile_rows = 128:
// [mats][ceil(rows/128)][ceil(G/4)][512]; tile_rows = 192 or 256: [mats][ceil(rows/tile_rows)][ceil(G/4)][2][512]
// (the tile's two 128-row parts side by side for each K chunk of 128; a 192-row tile's second part holds 64 rows).
size_t sf_repacked_bytes(long long mats, int rows, int G, int tile_rows = 128);
// With ids != nullptr, output matrix m is gathered from raw matrix ids[m] (m < mats). With nan_flag != nullptr, a
// scale byte 0xFF (E8M0 NaN) stores nan_code into *nan_flag (device int, if it still holds 0).
void launch_repack_sf(const uint8_t* raw, uint8_t* out, long long mats, int rows, int G, cudaStream_t s,
                      const int* ids = nullptr, int tile_rows = 128, int* nan_flag = nullptr, int nan_code = 1);

// Tensor-core decode MoE (decode_tc.cu): one persistent cooperative kernel per MoE layer. Weights are read in tiles
// of kDecodeTileRows rows (TMA boxes of kDecodeTileRows rows x 128 bytes; scales repacked with that tile size).
constexpr int kDecodeTileRows = 256;
// Tensor-core decode MoE (decode_tc.cu): one persistent cooperative kernel per MoE layer. The workspace layout
// depends only on (k, H, I); the byte range [zero_bytes_from, zero_bytes_to) must be zero before the first launch
// (the partial-sum words carry the launch epoch and the grid barrier resets itself afterwards).
struct DecodeTcLayout {
    int SPS_gu, KT_gu, SPS_dn, KT_dn, RT_gu, RT_dn;
    size_t off_logits, off_xq_img, off_xq_sf, off_aq_img, off_aq_sf, off_part_gu, off_part_dn, off_err;
    size_t off_sfa_gu, off_sfa_dn, off_misc, bytes, zero_bytes_from, zero_bytes_to;
    size_t off_rows, rows_bytes;   // the row-job kernel's partial output vectors [k * RT_gu][H] (64-bit words)
};
DecodeTcLayout decode_tc_layout(int k, int H, int I);

struct DecodeTcArgs {
    const CUtensorMap* tmap_gu;   // gate/up blocks viewed as [E][2I][H/2] bytes
    const CUtensorMap* tmap_dn;   // down blocks viewed as [E][H][I/2] bytes
    const uint8_t* sfa_gu;        // repacked scales, [mat][RT_gu][KT_gu][512]
    const uint8_t* sfa_dn;        // repacked scales, [mat][RT_dn][KT_dn][512]
    int sfa_by_slot;              // 1: mat = slot (scales gathered for the selected experts); 0: mat = expert id
    const float* gu_bias;
    const float* dn_bias;
    const void* router_w;         // bf16 [E][H]; null: ids/weights below give the experts
    const float* router_b;
    const float* norm_w;          // null: x is already normalized
    float eps;
    int E;
    const float* x;               // [H]
    const int* ids;               // [k] when router_w is null
    const float* weights;         // [k] when router_w is null
    int* ids_out;                 // optional: the router's choice
    float* w_out;
    float* x_resid;
    int k, H, I;
    float alpha, limit;
    void* workspace;              // decode_tc_layout(k, H, I).bytes
    long long* trace = nullptr;   // optional pipeline trace: [num_sms][160] clock64 stamps
    const CUtensorMap* tmap_dn64 = nullptr;   // down blocks [E][H][I/2] bytes in boxes of 256 rows x 64 bytes (64-byte
                                              // swizzle): enables the row-job kernel
    int plan = 0;                 // 0: the row-job kernel where it applies, else stream-K; 1: stream-K only
    const uint8_t* dn_img = nullptr;   // the row-job kernel's pre-packed down stages (launch_pack_down_jobs), or null
};
// Launches the row-job kernel (decode_rows.cu) when a.tmap_dn64 is set, a.plan == 0 and decode_rows_ok holds, else
// the stream-K kernel (decode_tc.cu).
void launch_moe_decode_tc(const DecodeTcArgs& a, cudaStream_t s);

// Row-job decode MoE (decode_rows.cu): G = k * ceil(2I / 256) CTAs, CTA c owns 256 gate/up rows of one selected expert
// over all of K and the down K-slice of their 128 activations; one reduction of the G partial vectors at the end.
// Needs G <= the SM count (and G >= E when the kernel runs the router).
int decode_rows_jobs(int k, int I);
bool decode_rows_ok(int k, int H, int I, int E_router);
void launch_moe_decode_rows(const DecodeTcArgs& a, cudaStream_t s);
// The row-job kernel's down weights pre-packed per (expert, job, stage): each stage's two 256-row x 64-byte boxes in
// their 64-byte-swizzled shared-memory image and their scale chunks (from the layer's repacked down scales), so one
// contiguous bulk copy brings a stage. down_jobs_bytes(E, H, I) bytes.
size_t down_jobs_bytes(int E, int H, int I);
void launch_pack_down_jobs(const uint8_t* dn_blocks, const uint8_t* sf_dn_repacked, uint8_t* out, int E, int H, int I,
                           cudaStream_t s);

// Batched (prefill) MoE on tensor cores (prefill_tc.cu). Workspace layout for T tokens.
struct PrefillLayout {
    int max_tiles, KB_gu, KB_dn;
    size_t off_h, off_ids, off_w, off_pos_of, off_tok_of, off_slot_of, off_tiles, off_misc, off_img_gu, off_img_dn,
        off_out, off_w64, bytes;
};
PrefillLayout prefill_layout(int T, int k, int E, int H, int I);

// Router weights bf16 [E][H] -> fp64 [H][32] (zero columns for experts >= E).
void launch_router_w64(const void* W, int E, int H, double* W64, cudaStream_t s);
// RMSNorm (norm_w != null) and router for T tokens: h_out (optional) = normalized x, ids / wts [T][k].
void launch_router_batched(const double* W64, const float* b, const float* x, const float* norm_w, float eps, int T,
                           int E, int H, int k, float* h_out, int* ids, float* wts, cudaStream_t s);

struct PrefillArgs {
    const CUtensorMap* tmap_gu;   // gate/up blocks [E][2I][H/2] bytes, boxes of kDecodeTileRows rows x 128 bytes
    const CUtensorMap* tmap_dn;
    const uint8_t* sf_gu;         // scales repacked with kDecodeTileRows-row tiles for all E experts
    const uint8_t* sf_dn;
    const float* gu_bias;         // [E][2I]
    const float* dn_bias;         // [E][H]
    const float* h;               // normalized tokens [T][H]
    const int* ids;               // [T][k]
    const float* weights;         // [T][k]
    float* x_resid;               // [T][H], += the MoE output
    int T, k, E, H, I;
    float alpha, limit;
    void* workspace;              // prefill_layout(T, k, E, H, I).bytes
    long long* trace = nullptr;   // optional: grouped GEMM wait totals per CTA, [160][160], slots 64 * mode + i
    void* const* events = nullptr;   // optional: 4 cudaEvent_t around the gate/up and the down grouped GEMM
    int terms = 8;                // e2m1 terms per activation (8: exact to 2^-21 of each block's scale)
    int pack = 0;                 // 0: terms stacked as MMAs on 128-token tiles; 1: packed as rows, 16 tokens a tile
};
void launch_moe_batched(const PrefillArgs& a, cudaStream_t s);

// Expert parallelism over `world` ranks (one GPU each): the shared region (allocated zeroed, mapped on every rank) and
// this rank's private workspace, for at most T_max tokens per rank.
struct EpLayout {
    long long max_rows;
    int max_tiles, KB_gu, KB_dn;
    size_t off_flags, off_counts, off_meta, off_img, off_out, region_bytes;
    size_t off_h, off_ids, off_w, off_pos, off_dest, off_tiles, off_misc, off_img_dn, off_act, local_bytes;
};
EpLayout ep_layout(int T_max, int k, int E, int world, int H, int I);

struct EpArgs {
    const CUtensorMap* tmap_gu;   // this rank's experts (E / world of them), as PrefillArgs
    const CUtensorMap* tmap_dn;
    const uint8_t* sf_gu;
    const uint8_t* sf_dn;
    const float* gu_bias;
    const float* dn_bias;
    const double* w64;            // the full router (E experts) as fp64 [H][32]
    const float* router_b;        // [E]
    const float* norm_w;          // [H]
    float eps;
    const float* x;               // this rank's tokens [T][H]
    float* x_resid;               // [T][H], += the MoE output
    int T, T_max, k, E, H, I, rank, world;
    float alpha, limit;
    void* const* peers;           // host array [world]: every rank's region as mapped here (peers[rank] = own)
    unsigned epoch;               // the same on every rank for one layer call; increases from 1
    void* local_ws;               // ep_layout(...).local_bytes
    long long* trace = nullptr;
    int terms = 8;                // as PrefillArgs (always stacked)
};
void launch_ep_layer(const EpArgs& a, cudaStream_t s);

// Single-CTA tcgen05 kind::mxf4 GEMM, D[128][N] = dequant(A)[128][K] . dequant(B)[N][K]^T, from raw MXFP4 arrays
// (checkpoint layout). Pins the layout conventions of the tensor-core kernels. A is loaded by TMA with the 128-byte
// swizzle (128-byte boxes of K) or the 64-byte swizzle (64-byte boxes, a_swizzle = 64). Synchronizes.
void selftest_mxf4_gemm(const uint8_t* a_blocks, const uint8_t* a_scales, const uint8_t* b_blocks,
                        const uint8_t* b_scales, float* d, int N, int K, void* scratch, size_t scratch_bytes,
                        cudaStream_t s, int a_swizzle = 128);

// Quantizes x [n] into kDecodeTerms e2m1 residual terms (which = 0: comparison quantizer, 1: converter quantizer,
// 2: fixed scale schedule with fp32 rounding, 3: the same with one warp per block)
// and decodes them back into out [n]; per_term (optional, [2][n]) receives the first two terms. Synchronizes.
void selftest_terms(const float* x, int n, float* out, float* per_term, int which, void* scratch, size_t bytes,
                    cudaStream_t s);

// Decode step around the MoE (decode_step.cu). pdl: launch with programmatic dependent launch (the kernels wait for
// the previous kernel's memory before reading their inputs). d_pos (device int) overrides pos when not null.
void launch_gemv_bf16(const void* W, const float* x, const float* norm_w, float eps, const float* bias,
                      const float* resid, float* y, int N, int K, cudaStream_t s, bool pdl);
// The attention block of a bs=1 decode step in one cooperative launch (attn_block.cu): x += Wo attention(RoPE(Wqkv
// RMSNorm(x) + bqkv)) + bo, the new position's key and value appended to the fp16 cache. work: attn_block_
// workspace_bytes(), zero-filled before the first use; err: device error word (bounded waits, codes 41-45). Returns
// false (nothing launched) when the shape does not fit the kernel's shared-memory ring.
size_t attn_block_workspace_bytes();
extern std::atomic<int> g_attn_impl;   // 1: the engine's step uses launch_attn_block, 0: three launches per layer
bool launch_attn_block(float* x, const float* ln, float eps, const void* wqkv, const float* bqkv, const void* wo,
                       const float* bo, const float* cos_t, const float* sin_t, void* k_cache, void* v_cache,
                       const float* sinks, const int* d_pos, int window, int H, void* work, int* err, cudaStream_t s,
                       bool pdl);
void launch_rope_append(float* qkv, const float* cos_t, const float* sin_t, const int* d_pos, int pos, void* k_cache,
                        void* v_cache, int window, cudaStream_t s, bool pdl);
size_t attention_workspace_floats();   // zero-filled before the first use of launch_attention_step
// RoPE of the raw QKV output, the new position's key and value into the cache, attention and the merge of the
// split partials, in one launch (qkv is not modified).
void launch_attention_step(const float* qkv, const float* cos_t, const float* sin_t, void* k_cache, void* v_cache,
                           const float* sinks, const int* d_pos, int window, float* part, float* out, cudaStream_t s,
                           bool pdl);
void launch_attention(const float* q, const void* k_cache, const void* v_cache, const float* sinks, const int* d_pos,
                      int pos, int window, float* part, float* out, cudaStream_t s, bool pdl);
void launch_embed(const void* table, const int* d_token, float* x, int H, cudaStream_t s, bool pdl);
void launch_increment(int* p, cudaStream_t s, bool pdl);
size_t score_workspace_bytes();   // zero-filled before the first use (its counter resets itself)
void launch_score(const float* logits, int V, void* work, const int* ids, int k, int target, float* lp, int* argmax,
                  float* target_lp, float* lse, int* next_token, cudaStream_t s, bool pdl);

// The fused decode kernel of a prepared layer (capi.cu) with a caller-owned workspace of
// moe_layer_workspace_bytes(k, H, I), zero-filled before its first use and used by one stream at a time.
size_t moe_layer_workspace_bytes(int k, int H, int I);
void moe_layer_forward_ws(gptoss_moe_layer* l, const float* x, float* x_resid, cudaStream_t s, void* const* events,
                          void* workspace);

// Measured dense kind::mxf4 tensor rate of the current device in TFLOP/s (tc_common.cu; err_dev: a zeroed device
// int that records a wait that gave up).
double selftest_mxf4_peak(int* err_dev);
double selftest_mxf4_mma_ns(int n, int* err_dev);

// Batched prefill of n consecutive positions p0.. of one sequence (decode_step.cu): QKV bias + RoPE in place and the
// rotated k / v rounded to fp16 into kvb [n][2][8][64]; attention of every row (older positions from the cache, the
// batch's own from kvb; part holds prefill_attention_floats(part_rows)); the batch appended to the cache afterwards;
// row splits into bf16 hi + lo (after an optional RMSNorm) for the tensor-core projections.
size_t prefill_attention_floats(int rows);
void launch_prefill_qkv_rope(float* qkv, const float* bias, const float* cos_t, const float* sin_t, int p0, int n,
                             void* kvb, cudaStream_t s);
void launch_prefill_attention(const float* qkv, const void* kvb, const void* k_cache, const void* v_cache,
                              const float* sinks, int p0, int n, int window, float* part, int part_rows, float* out,
                              cudaStream_t s);
void launch_prefill_append(const void* kvb, int p0, int n, int window, void* k_cache, void* v_cache, cudaStream_t s);
void launch_split_rows(const float* x, int n, int K, const float* norm_w, float eps, void* hi, void* lo, cudaStream_t s);
void launch_add_bias_rows(float* x, const float* b, int n, int K, cudaStream_t s);
void launch_embed_rows(const void* table, const int* tokens, float* x, int n, int H, cudaStream_t s);

}  // namespace gpt
