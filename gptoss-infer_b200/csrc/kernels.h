// Host-side launchers of the MoE-path kernels. Every launcher takes the stream to run on and throws
// std::runtime_error on invalid shapes or launch failure; the C ABI (capi.cu) turns that into -1.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace gpt {

int num_sms();

// y[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w for T rows of n.
void launch_rmsnorm(const float* x, const float* w, float* y, int T, int n, float eps, cudaStream_t s);

// Bit-exact MXFP4 decode of n_blocks blocks (16 code bytes + 1 E8M0 byte each) into 32 floats per block.
// *bad is set to 1 if any scale byte is 0xFF (caller clears it first).
void launch_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, float* out, long long n_blocks, int* bad,
                          cudaStream_t s);

// Decode router for one token: logits = W[E,H] x + b accumulated exactly in fp64, top-k by (logit desc, id asc)
// with NaN never selected ahead of a number, softmax over the k selected fp32 logits.
void launch_router_decode(const __nv_bfloat16* W, const float* b, const float* x, int E, int H, int k, int* ids,
                          float* weights, cudaStream_t s);

// Decode MoE for one token on raw checkpoint-layout MXFP4 experts (SIMT path).
//   a[slot][j] = swiglu(W1[ids[slot]] x + b1)          gate/up rows interleaved (even glu, odd linear)
//   x_resid[i] += sum_slot w[slot] (W2[ids[slot]] a[slot] + b2)[i]   summed in slot order
size_t moe_decode_scratch_bytes(int k, int I);
void launch_moe_decode_simt(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                            const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                            const float* x_norm, const int* ids, const float* weights, float* x_resid, int k,
                            int H, int I, float alpha, float limit, void* scratch, cudaStream_t s,
                            void* mid_event = nullptr);

// Scale-factor repack: raw E8M0 bytes [mats][rows][G] -> tcgen05 chunks [mats][ceil(rows/128)][ceil(G/4)][512],
// chunk byte (r % 32) * 16 + (r / 32) * 4 + kb for row r and k-block kb of the chunk; zero padded.
size_t sf_repacked_bytes(long long mats, int rows, int G);
void launch_repack_sf(const uint8_t* raw, uint8_t* out, long long mats, int rows, int G, cudaStream_t s);

// Single-CTA tcgen05 kind::mxf4 GEMM, D[128][N] = dequant(A)[128][K] . dequant(B)[N][K]^T, from raw MXFP4 arrays
// (checkpoint layout). Pins the layout conventions of the tensor-core kernels. Synchronizes.
void selftest_mxf4_gemm(const uint8_t* a_blocks, const uint8_t* a_scales, const uint8_t* b_blocks,
                        const uint8_t* b_scales, float* d, int N, int K, void* scratch, size_t scratch_bytes,
                        cudaStream_t s);

}  // namespace gpt
