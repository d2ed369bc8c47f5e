// Shared device helpers for the gpt-oss MXFP4 MoE path on B200 (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace gpt {

#define GPT_CHECK(x)                                                                                    \
    do {                                                                                                \
        cudaError_t e_ = (x);                                                                           \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

inline void check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

inline void require(bool ok, const char* what) {
    if (!ok) throw std::runtime_error(what);
}

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// E8M0 byte -> 2^(s-127) built from the bit pattern; s == 0 is the fp32 subnormal 2^-127. (0xFF is rejected by the
// callers that can see it.) Exact on every input, unlike exp2f.
__device__ __forceinline__ float e8m0_to_f32(uint32_t s) {
    return s == 0 ? __uint_as_float(0x00400000u) : __uint_as_float(s << 23);
}

// One 32-bit word of eight e2m1 codes (byte j: low nibble = element 2j) -> eight floats, via the sm_100 e2m1x2
// converter. The word is unpacked inside the asm from a full 32-bit register: feeding a 16-bit view of a wider
// register (e.g. (unsigned short)(w >> 16)) was miscompiled into reading the wrong byte. Every e2m1 value is exact in
// f16 and f32, so this is lossless.
__device__ __forceinline__ void e2m1x8_to_f32(uint32_t word, float* out8) {
    uint32_t h[4];
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(word));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<__half2*>(&h[i]));
        out8[2 * i] = f.x;
        out8[2 * i + 1] = f.y;
    }
}

// Exact e2m1 decode by bit construction, no converter involved: the 3 magnitude bits placed at fp32 bits 22-24 give
// 2^-126 * value (code 1 lands on the subnormal 2^-127 = 2^-126 * 0.5), the sign bit goes to bit 31, and one multiply
// by 2^126 rescales exactly. Needs IEEE subnormals (no flush-to-zero), which this build keeps.
__device__ __forceinline__ float e2m1_exact(uint32_t nib) {
    return __uint_as_float(((nib & 7u) << 22) | ((nib & 8u) << 28)) * 0x1p126f;
}

// Packed fp32x2 FMA (sm_100): d = a * b + c, two lanes at once.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// 16-byte read-only global load that does not allocate in L1 (weights are streamed once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Reciprocal root-mean-square of a row from its sum of squares: the RMSNorm scale 1 / sqrt(mean(x^2) + eps) of
// gptoss_ref/model.py:21-22. Every RMSNorm in this library (the stand-alone kernel, the routers, the fused decode
// kernel) takes its scale from here, so they agree bit for bit given the same sum.
__device__ __forceinline__ float rms_scale(float sum_sq, int n, float eps) {
    return 1.0f / sqrtf(sum_sq / float(n) + eps);
}

// ---- Expert selection, shared by every router (stand-alone decode, fused decode, batched).
//
// Logits are fp64 and compared through a 64-bit unsigned key that preserves their order: a non-negative value keeps
// its bits with the top bit set, a negative one is bit-inverted. NaN and lanes that hold no expert get key 0, which
// no real logit reaches (-inf maps to 0x000FFFFFFFFFFFFF), so they can only be picked once every real logit is.
__device__ __forceinline__ unsigned long long logit_order_key(double v, bool valid) {
    const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(v));
    if (!valid || (bits << 1) > 0xFFE0000000000000ull) return 0ull;          // NaN: exponent all ones, mantissa != 0
    return (bits >> 63) ? ~bits : (bits | 0x8000000000000000ull);
}

// Top k of the 32 lane-held logits (lane e holds expert e; lanes with valid == false hold none). Each round the warp
// takes the largest key with two 32-bit max reductions (high word, then low word among the lanes that hold that high
// word) and the smallest expert id among the lanes holding the full key, so equal logits go to the lower id; the
// winner leaves the race. Lane q < k receives the q-th pick (descending logit): its expert id and logit.
__device__ __forceinline__ void warp_topk_logits(double v, bool valid, int k, int& pick_id, double& pick_logit) {
    const int lane = threadIdx.x & 31;
    unsigned long long key = logit_order_key(v, valid);
    unsigned id = valid ? unsigned(lane) : 32u + unsigned(lane);
    pick_id = 0;
    pick_logit = 0.0;
    for (int q = 0; q < k; ++q) {
        const unsigned hi = unsigned(key >> 32), lo = unsigned(key);
        const unsigned best_hi = __reduce_max_sync(kFull, hi);
        const unsigned best_lo = __reduce_max_sync(kFull, hi == best_hi ? lo : 0u);
        const unsigned winner = __reduce_min_sync(kFull, hi == best_hi && lo == best_lo ? id : 0xFFFFFFFFu);
        const double wv = __shfl_sync(kFull, v, int(winner & 31u));
        if (lane == q) {
            pick_id = int(winner);
            pick_logit = wv;
        }
        if (id == winner) {
            key = 0ull;
            id = 32u + unsigned(lane);
        }
    }
}

// Gate weights of the k picks held in lanes 0..k-1 (descending, so lane 0 holds the largest): the softmax over the k
// selected logits in fp32, as gptoss_ref/model.py:97-98 computes it. Lanes >= k return 0.
__device__ __forceinline__ float warp_pick_softmax(double pick_logit, int k) {
    const int lane = threadIdx.x & 31;
    const float l = float(pick_logit);
    const float lmax = __shfl_sync(kFull, l, 0);
    const float e = lane < k ? expf(l - lmax) : 0.f;
    return e / warp_sum(e);
}

// Thread-block clusters: this CTA's rank, a barrier over every thread of the cluster (release / acquire, so shared
// memory written before it is visible to the other CTAs after it), and distributed shared memory accesses to the
// same variable in CTA `cta` of the cluster.
__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* local_ptr, unsigned cta) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local_ptr));
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(cta));
    return ra;
}
__device__ __forceinline__ void dsmem_store_f64(double* local_ptr, unsigned cta, double v) {
    asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(dsmem_addr(local_ptr, cta)), "d"(v) : "memory");
}
__device__ __forceinline__ double dsmem_load_f64(const double* local_ptr, unsigned cta) {
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(dsmem_addr(local_ptr, cta)) : "memory");
    return v;
}
__device__ __forceinline__ float dsmem_load_f32(const float* local_ptr, unsigned cta) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(dsmem_addr(local_ptr, cta)) : "memory");
    return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue, and wait for the previous
// kernel's memory to be visible. Both are no-ops when the launch did not opt in.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace gpt
