// Decode-path kernels that run on the CUDA cores: RMSNorm, the MXFP4 decoder, the router, and the SIMT MXFP4
// GEMV pair (gate/up + clamped SwiGLU, down + weighted combine). The tensor-core decode path lives in
// decode_tc.cu; this one is the correctness baseline and handles every shape the C ABI accepts.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <mutex>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"
#include "terms.cuh"

namespace gpt {

// SM count of the current device, cached per device ordinal (a process may drive GPUs of different sizes).
int num_sms() {
    static std::mutex mu;
    static int count[64] = {};
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("device ordinal out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!count[dev]) GPT_CHECK(cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev));
    return count[dev];
}

namespace {

// ---------------------------------------------------------------------------------------------------------------
// RMSNorm, one CTA of kNormThreads per row. Each warp adds the squares of a strided set of the row's float4 chunks
// (scalars when the row is not 16-byte aligned); the eight warp sums meet in shared memory and every thread adds
// them in warp order, so all threads hold the same total without a second reduction round; then each thread scales
// the chunks it read.
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               float* __restrict__ y, int n, float eps) {
    __shared__ float warp_ss[kNormThreads / 32];
    const float* xr = x + size_t(blockIdx.x) * n;
    float* yr = y + size_t(blockIdx.x) * n;
    const bool vec = (n & 3) == 0 && ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(yr) |
                                       reinterpret_cast<uintptr_t>(w)) & 15) == 0;
    float ss = 0.f;
    if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int c = threadIdx.x; c < (n >> 2); c += kNormThreads) {
            const float4 v = x4[c];
            ss = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, ss))));
        }
    } else {
        for (int i = threadIdx.x; i < n; i += kNormThreads) ss = fmaf(xr[i], xr[i], ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) warp_ss[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int q = 0; q < kNormThreads / 32; ++q) total += warp_ss[q];
    const float r = rms_scale(total, n, eps);
    if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        const float4* w4 = reinterpret_cast<const float4*>(w);
        float4* y4 = reinterpret_cast<float4*>(yr);
        for (int c = threadIdx.x; c < (n >> 2); c += kNormThreads) {
            const float4 v = x4[c], g = w4[c];
            y4[c] = make_float4(v.x * r * g.x, v.y * r * g.y, v.z * r * g.z, v.w * r * g.w);
        }
    } else {
        for (int i = threadIdx.x; i < n; i += kNormThreads) yr[i] = xr[i] * r * w[i];
    }
}

// ---------------------------------------------------------------------------------------------------------------
// MXFP4 decode: one thread per block. value = e2m1 * 2^(s-127) is one IEEE multiply of two exact values, so the
// result is bit-identical to the CPU decoder (subnormal 2^-127 for s == 0, inf for 6 * 2^127).
__global__ void mxfp4_dequant_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                                     float* __restrict__ out, long long n_blocks, int* bad) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= n_blocks) return;
    const uint32_t s = scales[i];
    if (s == 0xFFu) atomicExch(bad, 1);
    const float sc = e8m0_to_f32(s);
    const uint4 u = *reinterpret_cast<const uint4*>(blocks + i * 16);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float4* o = reinterpret_cast<float4*>(out + i * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = e2m1_exact(w[q] >> (4 * j)) * sc;
        o[2 * q] = make_float4(v[0], v[1], v[2], v[3]);
        o[2 * q + 1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// Router for one token. A cluster of 8 CTAs splits the experts (CTA r owns experts r, r+8, r+16, r+24); each CTA
// reduces its logits and stores them straight into CTA 0's shared memory over DSMEM, then one warp of CTA 0 picks
// the top k. Products bf16 x fp32 are exact in fp64 and the sum is kept in fp64, so the selected ids are the exact
// ranking of the true logits: they agree with any float64 reference except for exact ties, which go to the lower
// id (runtime/src/kernels.cu:307-324 states the same rule).
constexpr int kRouterCluster = 8, kRouterThreads = 256, kRouterPerCta = 4;

__device__ __forceinline__ double bf16_lo_d(uint32_t w) { return double(__uint_as_float(w << 16)); }
__device__ __forceinline__ double bf16_hi_d(uint32_t w) { return double(__uint_as_float(w & 0xffff0000u)); }

__global__ void __cluster_dims__(kRouterCluster, 1, 1) __launch_bounds__(kRouterThreads)
    router_decode_kernel(const __nv_bfloat16* __restrict__ W, const float* __restrict__ b,
                         const float* __restrict__ x_in, int E, int H, int k, int* __restrict__ ids,
                         float* __restrict__ weights, uint8_t* xq_img, uint8_t* xq_sf,
                         const float* __restrict__ norm_w, float eps, float* h_out) {
    __shared__ double red[kRouterThreads / 32][kRouterPerCta];
    __shared__ double logits[32];
    __shared__ float ssum[kRouterThreads / 32];
    extern __shared__ float hs[];                          // [H] when norm_w is given
    const unsigned r = cluster_rank();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, H8 = H >> 3;
    pdl_launch_dependents();                               // let the tensor-core gate/up CTAs become resident
    const float* x = x_in;
    if (norm_w) {
        // Fused RMSNorm (every CTA of the cluster normalizes the whole row into its shared memory).
        float ss = 0.f;
        for (int i = tid; i < H; i += kRouterThreads) ss = fmaf(x_in[i], x_in[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) ssum[warp] = ss;
        __syncthreads();
        float tot = 0.f;
        for (int w = 0; w < kRouterThreads / 32; ++w) tot += ssum[w];
        const float rn = rms_scale(tot, H, eps);
        for (int i = tid; i < H; i += kRouterThreads) {
            const float v = x_in[i] * rn * norm_w[i];
            hs[i] = v;
            if (h_out && r == 0) h_out[i] = v;
        }
        __syncthreads();
        x = hs;
    }
    const uint4* Wv = reinterpret_cast<const uint4*>(W);
    const float4* xv = reinterpret_cast<const float4*>(x);
    double acc[kRouterPerCta] = {0.0, 0.0, 0.0, 0.0};
    for (int c = tid; c < H8; c += kRouterThreads) {
        const float4 xa = xv[2 * c], xb = xv[2 * c + 1];
#pragma unroll
        for (int q = 0; q < kRouterPerCta; ++q) {
            const int e = int(r) + kRouterCluster * q;
            if (e < E) {
                const uint4 u = __ldg(Wv + size_t(e) * H8 + c);
                double s = bf16_lo_d(u.x) * double(xa.x);
                s = fma(bf16_hi_d(u.x), double(xa.y), s);
                s = fma(bf16_lo_d(u.y), double(xa.z), s);
                s = fma(bf16_hi_d(u.y), double(xa.w), s);
                s = fma(bf16_lo_d(u.z), double(xb.x), s);
                s = fma(bf16_hi_d(u.z), double(xb.y), s);
                s = fma(bf16_lo_d(u.w), double(xb.z), s);
                s = fma(bf16_hi_d(u.w), double(xb.w), s);
                acc[q] += s;
            }
        }
    }
#pragma unroll
    for (int q = 0; q < kRouterPerCta; ++q) {
        const double v = warp_sum(acc[q]);
        if (lane == 0) red[warp][q] = v;
    }
    __syncthreads();
    if (tid < kRouterPerCta) {
        const int e = int(r) + kRouterCluster * tid;
        if (e < E) {
            double t = 0.0;
            for (int w = 0; w < kRouterThreads / 32; ++w) t += red[w][tid];
            dsmem_store_f64(&logits[e], 0, t + double(b[e]));
        }
    }
    // Fused for the tensor-core path: the cluster's 64 warps split x into e2m1 residual terms (gate/up's B operand).
    if (xq_img) quantize_vector_terms_warp(x, H, xq_img, xq_sf, int(r) * (kRouterThreads / 32) + warp,
                                           kRouterCluster * (kRouterThreads / 32));
    cluster_sync_all();
    if (r != 0 || warp != 0) return;

    // warp 0 of CTA 0: top k of the E logits and the softmax over the picks (shared selection code)
    int pick = 0;
    double pick_logit = 0.0;
    warp_topk_logits(lane < E ? logits[lane] : 0.0, lane < E, k, pick, pick_logit);
    const float gate = warp_pick_softmax(pick_logit, k);
    if (lane < k) {
        ids[lane] = pick;
        weights[lane] = gate;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// SIMT MXFP4 GEMV. Lane l of a warp owns blocks g = l, l+32, ... of every row it touches; the activation vector is
// staged in shared memory transposed (element e of block g at [e][g]) so the 32 lanes read 32 consecutive words,
// and each activation read is reused across the rows a warp processes together.
constexpr int kSimtThreads = 256;

template <int NB>
__device__ __forceinline__ void stage_transposed(float* xs, const float* __restrict__ x, int n) {
    constexpr int Gp = 32 * NB;
    for (int i = threadIdx.x; i < 32 * Gp; i += blockDim.x) {
        const int e = i / Gp, g = i % Gp;
        const int src = g * 32 + e;
        xs[i] = src < n ? x[src] : 0.f;
    }
}

// Dot of one 16-byte MXFP4 block with 32 activations held in registers, unscaled.
__device__ __forceinline__ float block_dot(const uint4 u, const float* xr) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float v[8];
        e2m1x8_to_f32(w[q], v);
#pragma unroll
        for (int t = 0; t < 4; ++t)
            acc = ffma2(make_float2(v[2 * t], v[2 * t + 1]), make_float2(xr[q * 8 + 2 * t], xr[q * 8 + 2 * t + 1]), acc);
    }
    return acc.x + acc.y;
}

template <int NB>
__global__ void __launch_bounds__(kSimtThreads) gateup_simt_kernel(const uint8_t* __restrict__ blocks,
                                                                   const uint8_t* __restrict__ scales,
                                                                   const float* __restrict__ bias,
                                                                   const float* __restrict__ x,
                                                                   const int* __restrict__ ids, float* __restrict__ a,
                                                                   int k, int H, int I, float alpha, float limit) {
    constexpr int Gp = 32 * NB;
    extern __shared__ float xs[];                       // [32][Gp]
    stage_transposed<NB>(xs, x, H);
    __syncthreads();
    const int G = H >> 5, lane = threadIdx.x & 31;
    const int warp_g = blockIdx.x * (kSimtThreads / 32) + (threadIdx.x >> 5);
    const int warp_n = gridDim.x * (kSimtThreads / 32);
    const int half = I >> 1;                            // units of two outputs j = 2u, 2u+1 (four rows)
    for (int u = warp_g; u < k * half; u += warp_n) {
        const int slot = u / half, jp = u % half;
        const int e = ids[slot];
        const size_t row0 = size_t(e) * 2 * I + 4 * size_t(jp);
        uint4 wv[4][NB];
        uint32_t sv[4][NB];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                const int g = lane + 32 * i;
                if (g < G) {
                    wv[r][i] = ldg_stream(blocks + ((row0 + r) * G + g) * 16);
                    sv[r][i] = scales[(row0 + r) * G + g];
                }
            }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < NB; ++i) {
            const int g = lane + 32 * i;
            if (g < G) {
                float xr[32];
#pragma unroll
                for (int q = 0; q < 32; ++q) xr[q] = xs[q * Gp + g];
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[r] = fmaf(block_dot(wv[r][i], xr), e8m0_to_f32(sv[r][i]), acc[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r] = warp_sum(acc[r]);
        if (lane == 0) {
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                float gv = acc[2 * p] + bias[row0 + 2 * p], lv = acc[2 * p + 1] + bias[row0 + 2 * p + 1];
                gv = fminf(gv, limit);                                   // glu: clamped from above only
                lv = fminf(fmaxf(lv, -limit), limit);
                a[size_t(slot) * I + 2 * jp + p] = gv / (1.f + expf(-alpha * gv)) * (lv + 1.f);
            }
        }
    }
    pdl_launch_dependents();
}

template <int NB, int KC>
__global__ void __launch_bounds__(kSimtThreads) down_simt_kernel(const uint8_t* __restrict__ blocks,
                                                                 const uint8_t* __restrict__ scales,
                                                                 const float* __restrict__ bias,
                                                                 const float* __restrict__ a,
                                                                 const int* __restrict__ ids,
                                                                 const float* __restrict__ weights,
                                                                 float* __restrict__ x_resid, int k, int H, int I) {
    constexpr int Gp = 32 * NB;
    extern __shared__ float as[];                       // [k][32][Gp]
    pdl_wait();                                         // a[] comes from the gate/up kernel
    for (int s = 0; s < k; ++s) stage_transposed<NB>(as + size_t(s) * 32 * Gp, a + size_t(s) * I, I);
    __syncthreads();
    const int G = I >> 5, lane = threadIdx.x & 31;
    const int warp_g = blockIdx.x * (kSimtThreads / 32) + (threadIdx.x >> 5);
    const int warp_n = gridDim.x * (kSimtThreads / 32);
    for (int rp = warp_g; rp < (H >> 1); rp += warp_n) {
        float add[2] = {0.f, 0.f};
        for (int s0 = 0; s0 < k; s0 += KC) {
            uint4 wv[KC][2][NB];
            uint32_t sv[KC][2][NB];
#pragma unroll
            for (int c = 0; c < KC; ++c) {
                if (s0 + c < k) {
                    const size_t row0 = size_t(ids[s0 + c]) * H + 2 * size_t(rp);
#pragma unroll
                    for (int r = 0; r < 2; ++r)
#pragma unroll
                        for (int i = 0; i < NB; ++i) {
                            const int g = lane + 32 * i;
                            if (g < G) {
                                wv[c][r][i] = ldg_stream(blocks + ((row0 + r) * G + g) * 16);
                                sv[c][r][i] = scales[(row0 + r) * G + g];
                            }
                        }
                }
            }
            float acc[KC][2];
#pragma unroll
            for (int c = 0; c < KC; ++c) acc[c][0] = acc[c][1] = 0.f;
#pragma unroll
            for (int c = 0; c < KC; ++c) {
                if (s0 + c < k) {
                    const float* asl = as + size_t(s0 + c) * 32 * Gp;
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        const int g = lane + 32 * i;
                        if (g < G) {
                            float xr[32];
#pragma unroll
                            for (int q = 0; q < 32; ++q) xr[q] = asl[q * Gp + g];
#pragma unroll
                            for (int r = 0; r < 2; ++r)
                                acc[c][r] = fmaf(block_dot(wv[c][r][i], xr), e8m0_to_f32(sv[c][r][i]), acc[c][r]);
                        }
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < KC; ++c) {
                const float y0 = warp_sum(acc[c][0]), y1 = warp_sum(acc[c][1]);
                if (s0 + c < k && lane == 0) {
                    const size_t rb = size_t(ids[s0 + c]) * H + 2 * size_t(rp);
                    const float w = weights[s0 + c];
                    add[0] += w * (y0 + bias[rb]);                       // slot order, as the reference combines
                    add[1] += w * (y1 + bias[rb + 1]);
                }
            }
        }
        if (lane == 0) {
            x_resid[2 * rp] += add[0];
            x_resid[2 * rp + 1] += add[1];
        }
    }
}

template <class... KArgs, class... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    GPT_CHECK(cudaLaunchKernelEx(&cfg, kernel, args...));
}

template <int NB>
void moe_simt_nb(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias, const uint8_t* dn_blocks,
                 const uint8_t* dn_scales, const float* dn_bias, const float* x_norm, const int* ids,
                 const float* weights, float* x_resid, int k, int H, int I, float alpha, float limit, float* a,
                 cudaStream_t s, void* mid_event) {
    constexpr int Gp = 32 * NB;
    const int sms = num_sms();
    const size_t smem_gu = size_t(32) * Gp * sizeof(float);
    const int units = k * (I / 2);
    const int grid_gu = std::max(1, std::min(sms * 4, (units + 7) / 8));
    gateup_simt_kernel<NB><<<grid_gu, kSimtThreads, smem_gu, s>>>(gu_blocks, gu_scales, gu_bias, x_norm, ids, a, k,
                                                                   H, I, alpha, limit);
    check_launch("moe gate/up (simt)");
    if (mid_event) GPT_CHECK(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(mid_event), s, cudaEventRecordExternal));
    const size_t smem_dn = size_t(k) * 32 * Gp * sizeof(float);
    const int grid_dn = std::max(1, std::min(sms * 2, (H / 2 + 7) / 8));
    auto kern = down_simt_kernel<NB, 4>;
    // The attribute is per device and set only when a larger plan first needs it (attribute calls stay out of
    // CUDA-graph captures after the first eager call of a shape).
    static std::mutex mu;
    static int smem_set[64] = {};
    {
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        if (dev < 0 || dev >= 64) throw std::runtime_error("moe down (simt): device ordinal out of range");
        std::lock_guard<std::mutex> lock(mu);
        if (int(smem_dn) > smem_set[dev]) {
            GPT_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_dn)));
            smem_set[dev] = int(smem_dn);
        }
    }
    launch_pdl(kern, dim3(grid_dn), dim3(kSimtThreads), smem_dn, s, true, dn_blocks, dn_scales, dn_bias,
               (const float*)a, ids, weights, x_resid, k, H, I);
    check_launch("moe down (simt)");
}

}  // namespace

void launch_rmsnorm(const float* x, const float* w, float* y, int T, int n, float eps, cudaStream_t s) {
    require(T >= 1 && n >= 1, "rmsnorm: T and n must be positive");
    rmsnorm_kernel<<<T, kNormThreads, 0, s>>>(x, w, y, n, eps);
    check_launch("rmsnorm");
}

void launch_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, float* out, long long n_blocks, int* bad,
                          cudaStream_t s) {
    require(n_blocks >= 0, "mxfp4_dequant: n_blocks must be >= 0");
    if (n_blocks == 0) return;
    const long long grid = (n_blocks + 255) / 256;
    require(grid < (1LL << 31), "mxfp4_dequant: too many blocks");
    mxfp4_dequant_kernel<<<unsigned(grid), 256, 0, s>>>(blocks, scales, out, n_blocks, bad);
    check_launch("mxfp4_dequant");
}

void launch_router_decode(const __nv_bfloat16* W, const float* b, const float* x, int E, int H, int k, int* ids,
                          float* weights, cudaStream_t s, uint8_t* xq_img, uint8_t* xq_sf, const float* norm_w,
                          float eps, float* h_out) {
    if (E < 1 || E > 32 || k < 1 || k > 8 || k > E || H % 8 || H < 8)
        throw std::runtime_error("router: unsupported shape (need 1 <= k <= 8, k <= E <= 32, H % 8 == 0)");
    if (xq_img && H % 32) throw std::runtime_error("router: fused quantization needs H % 32 == 0");
    const size_t smem = norm_w ? size_t(H) * sizeof(float) : 0;
    if (smem > 48 * 1024)
        GPT_CHECK(cudaFuncSetAttribute(router_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    router_decode_kernel<<<kRouterCluster, kRouterThreads, smem, s>>>(W, b, x, E, H, k, ids, weights, xq_img, xq_sf,
                                                                       norm_w, eps, h_out);
    check_launch("router");
}

size_t moe_decode_scratch_bytes(int k, int I) { return size_t(k) * size_t(I) * sizeof(float); }

void launch_moe_decode_simt(const uint8_t* gu_blocks, const uint8_t* gu_scales, const float* gu_bias,
                            const uint8_t* dn_blocks, const uint8_t* dn_scales, const float* dn_bias,
                            const float* x_norm, const int* ids, const float* weights, float* x_resid, int k,
                            int H, int I, float alpha, float limit, void* scratch, cudaStream_t s,
                            void* mid_event) {
    if (k < 1 || k > 8) throw std::runtime_error("moe: k must be in 1..8");
    if (H % 32 || I % 32 || H < 32 || I < 32) throw std::runtime_error("moe: H and I must be positive multiples of 32");
    const int G = std::max(H, I) / 32;
    float* a = static_cast<float*>(scratch);
    if (G <= 32)
        moe_simt_nb<1>(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, x_norm, ids, weights, x_resid, k,
                       H, I, alpha, limit, a, s, mid_event);
    else if (G <= 64)
        moe_simt_nb<2>(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, x_norm, ids, weights, x_resid, k,
                       H, I, alpha, limit, a, s, mid_event);
    else if (G <= 96)
        moe_simt_nb<3>(gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales, dn_bias, x_norm, ids, weights, x_resid, k,
                       H, I, alpha, limit, a, s, mid_event);
    else
        throw std::runtime_error("moe: H and I must be at most 3072");
}

}  // namespace gpt
