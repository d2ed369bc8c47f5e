// The decode step around the MoE (gpt-oss attention block, LM head, scoring), for one token at a time:
//   * bf16 GEMV y = W x (+ bias) (+ residual), optionally with the RMSNorm of x fused in front (QKV, O, LM head);
//   * RoPE (YaRN cos/sin tables, NeoX half-split rotation) and the fp16 KV-cache append;
//   * split-K attention over the cached keys with per-head sinks and an optional sliding window (GQA: 8 query heads
//     per key/value head);
//   * embedding lookup, and the score of the logits (log-sum-exp, argmax, log-probabilities of given ids).
// All of it is HBM-bound streaming (weights, cache) or latency-bound small work: CUDA cores with 16-byte loads that
// bypass L1, enough bytes in flight per SM, and grids that cover every SM. Device-side positions (`d_pos`) let a
// whole step be captured once in a CUDA graph.
#include <algorithm>
#include <cfloat>
#include <climits>
#include <cmath>
#include <mutex>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace gpt {
namespace ds {

constexpr int kHeads = 64, kKvHeads = 8, kHeadDim = 64, kGroup = kHeads / kKvHeads, kPairs = kHeadDim / 2;
constexpr int kQkv = (kHeads + 2 * kKvHeads) * kHeadDim;     // 5120

__device__ __forceinline__ float bf16_lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi_f(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ---------------------------------------------------------------------------------------------------- GEMV
// y[n] = sum_k W[n][k] x'[k] (+ bias[n]) (+ resid[n]), W bf16 [N][K] (K % 8 == 0), x' = x or RMSNorm(x; g, eps).
// Every CTA stages x' (fp32) in shared memory (computing the norm itself when g is given: g is staged before the
// dependency wait, then x is read from L2; 1374 -> 1348 us per configs[1] token against reading g after the wait).
// A warp takes kRows rows at a time; lane l reads the rows' 16-byte chunks l, l + 32, ... with streaming loads (all
// loads of a row group issued before the FMAs) and accumulates in packed fp32 pairs; warp_sum ends each row.
// The weights do not depend on the previous kernel, so before the dependency wait every warp asks L2 for its first
// pf_groups row groups (one bulk prefetch per row) and the next kernel's launch is released: a CTA that is resident
// while the previous kernel still runs (programmatic dependent launch) streams its rows into L2 meanwhile.
// One row per warp at a time with 8 chunks in flight per lane and 4 CTAs per SM (64 registers): more warps in flight
// measured faster per configs[1] token than two rows per warp at 2 CTAs per SM (1470 -> 1372 us; 12 chunks at 3 CTAs
// 1414 us, 6 chunks at 5 CTAs 1371 us, 4 rows per warp 1689 us).
constexpr int kGemvThreads = 256, kRows = 1, kChunksInFlight = 8, kGemvCtasPerSm = 4;
// x' in shared memory as two float4 arrays (elements 8c..8c+3 at 4c, elements 8c+4..8c+7 at K/2 + 4c), so that the
// lanes' reads of consecutive chunks are consecutive 16-byte words (no bank conflict; 1485 -> 1463 us per configs[1]
// token measured against the plain layout, whose 32-byte lane stride is a two-way conflict)
__device__ __forceinline__ int xs_index(int i, int K) {     // float index i (a multiple of 4) of x' -> staging index
    return ((i >> 2) & 1) * (K >> 1) + ((i >> 3) << 2);
}

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm) gemv_bf16_kernel(const __nv_bfloat16* __restrict__ W,
                                                                    const float* __restrict__ x,
                                                                    const float* __restrict__ g, float eps,
                                                                    const float* __restrict__ bias,
                                                                    const float* resid, float* y, int N, int K,
                                                                    int pf_groups) {
    extern __shared__ float xs[];                               // [K]
    __shared__ float part[kGemvThreads / 32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gw = blockIdx.x * (kGemvThreads / 32) + warp, nw = gridDim.x * (kGemvThreads / 32);
    {
        // K % 8 == 0: every row starts on a 16-byte boundary and is a multiple of 16 bytes long
        int g = 0;
        for (int row0 = gw * kRows; row0 < N && g < pf_groups; row0 += nw * kRows, ++g)
            if (lane < kRows && row0 + lane < N)
                prefetch_l2_bulk(W + size_t(row0 + lane) * K, uint32_t(K) * 2u);
    }
    if (g)                                                      // the norm weight does not depend on x
        for (int i = tid * 4; i < K; i += kGemvThreads * 4)
            *reinterpret_cast<float4*>(xs + xs_index(i, K)) = __ldg(reinterpret_cast<const float4*>(g + i));
    pdl_launch_dependents();
    pdl_wait();                                                 // x comes from the previous kernel
    if (g) {
        float ss = 0.f;
        for (int i = tid * 4; i < K; i += kGemvThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(x + i);
            ss = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, ss))));
        }
        ss = warp_sum(ss);
        if (lane == 0) part[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvThreads / 32; ++w) tot += part[w];
        const float r = rms_scale(tot, K, eps);
        for (int i = tid * 4; i < K; i += kGemvThreads * 4) {   // (this thread staged g at the same places)
            float4& gg = *reinterpret_cast<float4*>(xs + xs_index(i, K));
            const float4 v = *reinterpret_cast<const float4*>(x + i);
            gg = make_float4(v.x * r * gg.x, v.y * r * gg.y, v.z * r * gg.z, v.w * r * gg.w);
        }
    } else {
        for (int i = tid * 4; i < K; i += kGemvThreads * 4)
            *reinterpret_cast<float4*>(xs + xs_index(i, K)) = *reinterpret_cast<const float4*>(x + i);
    }
    __syncthreads();
    const int K8 = K >> 3;
    const uint4* Wv = reinterpret_cast<const uint4*>(W);
    for (int row0 = gw * kRows; row0 < N; row0 += nw * kRows) {
        float2 acc[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r) acc[r] = make_float2(0.f, 0.f);
        for (int c0 = 0; c0 < K8; c0 += 32 * kChunksInFlight) {
            uint4 u[kRows][kChunksInFlight];
#pragma unroll
            for (int r = 0; r < kRows; ++r)
#pragma unroll
                for (int q = 0; q < kChunksInFlight; ++q) {
                    const int c = c0 + lane + 32 * q;
                    u[r][q] = row0 + r < N && c < K8 ? ldg_stream(Wv + size_t(row0 + r) * K8 + c)
                                                     : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
            for (int q = 0; q < kChunksInFlight; ++q) {
                const int c = c0 + lane + 32 * q;
                if (c < K8) {
                    const float4 xa = *reinterpret_cast<const float4*>(xs + xs_index(8 * c, K));
                    const float4 xb = *reinterpret_cast<const float4*>(xs + xs_index(8 * c + 4, K));
#pragma unroll
                    for (int r = 0; r < kRows; ++r) {
                        const uint4 w = u[r][q];
                        acc[r] = ffma2(make_float2(bf16_lo_f(w.x), bf16_hi_f(w.x)), make_float2(xa.x, xa.y), acc[r]);
                        acc[r] = ffma2(make_float2(bf16_lo_f(w.y), bf16_hi_f(w.y)), make_float2(xa.z, xa.w), acc[r]);
                        acc[r] = ffma2(make_float2(bf16_lo_f(w.z), bf16_hi_f(w.z)), make_float2(xb.x, xb.y), acc[r]);
                        acc[r] = ffma2(make_float2(bf16_lo_f(w.w), bf16_hi_f(w.w)), make_float2(xb.z, xb.w), acc[r]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const float v = warp_sum(acc[r].x + acc[r].y);
            const int row = row0 + r;
            if (lane == 0 && row < N) {
                float o = v;
                if (bias) o += bias[row];
                if (resid) o += resid[row];                     // resid may alias y: read before the write
                y[row] = o;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------- RoPE
// qkv [5120]: q heads 0..63, k heads 64..71, v heads 72..79 (64 dims each). The q and k heads are rotated in place
// with the NeoX half-split (x1, x2) -> (x1 cos - x2 sin, x2 cos + x1 sin) from the fp32 tables cos_t / sin_t
// [position][32]; the rotated k and the v of the position go to the fp16 caches ([slot][8][64], round to nearest)
// at slot pos (window 0) or pos % window. One thread per rotary pair of the 72 rotated heads.
__global__ void __launch_bounds__(256) rope_append_kernel(float* qkv, const float* __restrict__ cos_t,
                                                          const float* __restrict__ sin_t, const int* d_pos,
                                                          int pos_arg, __half* kc, __half* vc, int window) {
    pdl_wait();
    pdl_launch_dependents();
    const int pos = d_pos ? *d_pos : pos_arg;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < (kHeads + kKvHeads) * kPairs; p += gridDim.x * blockDim.x) {
        const int head = p / kPairs, i = p % kPairs;
        const float c = cos_t[size_t(pos) * kPairs + i], s = sin_t[size_t(pos) * kPairs + i];
        float* base = qkv + head * kHeadDim;
        const float x1 = base[i], x2 = base[i + kPairs];
        const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        base[i] = o1;
        base[i + kPairs] = o2;
        if (head >= kHeads) {
            const int kh = head - kHeads;
            const size_t slot = window > 0 ? size_t(pos % window) : size_t(pos);
            const size_t off = (slot * kKvHeads + kh) * kHeadDim;
            const float* v = qkv + (kHeads + kKvHeads + kh) * kHeadDim;
            kc[off + i] = __float2half_rn(o1);
            kc[off + i + kPairs] = __float2half_rn(o2);
            vc[off + i] = __float2half_rn(v[i]);
            vc[off + i + kPairs] = __float2half_rn(v[i + kPairs]);
        }
    }
}

// ---------------------------------------------------------------------------------------------------- attention
// Keys visible to the query at `pos`: positions first .. pos, n = min(pos + 1, window) with a window, pos + 1
// without; position p lives in cache slot p % window (window) or p. A CTA owns one key/value head (8 query heads,
// GQA) and a contiguous range [k0, k1) of the visible keys (split-K over kSplits ranges), walks it in chunks of
// kChunk keys staged in shared memory (keys and values, fp16, 16-byte loads) and keeps a running softmax per query
// head: m (max score), l (sum of exp(score - m)) and acc[64] (sum of exp(score - m) v). Scores are q . k / 8 in
// fp32. The partials (m, l, acc) of all ranges are merged with the head's sink logit (one more softmax column that
// carries no value): M = max(sink, m_s), l = exp(sink - M) + sum l_s exp(m_s - M), out = sum acc_s exp(m_s - M) / l.
constexpr int kSplits = 18, kChunk = 128, kAttnThreads = 256;
constexpr int kKvRow = kHeadDim * 2 + 16;                       // staged key/value row: 128 bytes + 16 of padding

struct AttnShared {
    __align__(16) uint8_t ks[kChunk * kKvRow];
    __align__(16) uint8_t vs[kChunk * kKvRow];
    float qs[kGroup][kHeadDim];                                 // the 8 query heads (rotated)
    float ps[kGroup][kChunk];                                   // scores, then exp(score - m_new) of the chunk
    float cm[kGroup], cl[kGroup], scale_old[kGroup];
};

// Running softmax over visible keys [k0, k1) for the 8 query heads in sh.qs (all kAttnThreads threads call; sh.qs
// written and visible). load_kv(kk, part16, kw, vw) returns the 16-byte pieces part16 of the key and value at
// visible index kk. Thread (query head = warp, lane) ends with acc = dims 2 lane, 2 lane + 1 of that head.
template <class LoadKV>
__device__ __forceinline__ float2 attend_keys(AttnShared& sh, int k0, int k1, LoadKV&& load_kv) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, qh = warp;
    if (tid < kGroup) {
        sh.cm[tid] = -INFINITY;
        sh.cl[tid] = 0.f;
    }
    float2 acc = make_float2(0.f, 0.f);
    __syncthreads();
    for (int c0 = k0; c0 < k1; c0 += kChunk) {
        const int len = min(kChunk, k1 - c0);
        for (int i = tid; i < len * 8; i += kAttnThreads) {       // 8 threads per 128-byte row
            const int kk = i >> 3, part16 = i & 7;
            uint4 kw, vw;
            load_kv(c0 + kk, part16, kw, vw);
            *reinterpret_cast<uint4*>(sh.ks + kk * kKvRow + part16 * 16) = kw;
            *reinterpret_cast<uint4*>(sh.vs + kk * kKvRow + part16 * 16) = vw;
        }
        __syncthreads();
        // scores: an 8-lane group per key (each lane 8 dims), 4 keys per warp pass; the group's partial dots for the
        // 8 query heads are reduced so that lane j of the group ends with head j's dot (bit 2 of the lane picks heads
        // 4-7, bit 1 the upper pair, bit 0 the upper head)
        for (int kb = warp * 4; kb < len; kb += (kAttnThreads / 32) * 4) {
            const int kk = kb + (lane >> 3), sub = lane & 7;
            float d[kGroup];
            if (kk < len) {
                const uint4 u = *reinterpret_cast<const uint4*>(sh.ks + kk * kKvRow + sub * 16);
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
                float kv[8];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[t]));
                    kv[2 * t] = f.x;
                    kv[2 * t + 1] = f.y;
                }
#pragma unroll
                for (int g = 0; g < kGroup; ++g) {
                    float t = 0.f;
#pragma unroll
                    for (int e = 0; e < 8; ++e) t = fmaf(sh.qs[g][sub * 8 + e], kv[e], t);
                    d[g] = t;
                }
            } else {
#pragma unroll
                for (int g = 0; g < kGroup; ++g) d[g] = 0.f;
            }
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const bool up = sub & 4;
                const float recv = __shfl_xor_sync(kFull, up ? d[g] : d[g + 4], 4);
                d[g] = (up ? d[g + 4] : d[g]) + recv;
            }
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                const bool up = sub & 2;
                const float recv = __shfl_xor_sync(kFull, up ? d[g] : d[g + 2], 2);
                d[g] = (up ? d[g + 2] : d[g]) + recv;
            }
            {
                const bool up = sub & 1;
                const float recv = __shfl_xor_sync(kFull, up ? d[0] : d[1], 1);
                d[0] = (up ? d[1] : d[0]) + recv;
            }
            if (kk < len) sh.ps[sub][kk] = d[0] * 0.125f;          // scale 1 / sqrt(64)
        }
        __syncthreads();
        // per query head (warp qh): chunk max, new running max, exp, chunk sum
        {
            float m = -INFINITY;
            for (int kk = lane; kk < len; kk += 32) m = fmaxf(m, sh.ps[qh][kk]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
            const float m_old = sh.cm[qh], m_new = fmaxf(m_old, m);
            float ssum = 0.f;
            for (int kk = lane; kk < len; kk += 32) {
                const float e = expf(sh.ps[qh][kk] - m_new);
                sh.ps[qh][kk] = e;
                ssum += e;
            }
            ssum = warp_sum(ssum);
            __syncwarp();
            if (lane == 0) {
                const float a = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                sh.scale_old[qh] = a;
                sh.cl[qh] = sh.cl[qh] * a + ssum;
                sh.cm[qh] = m_new;
            }
        }
        __syncwarp();
        // acc = acc exp(m_old - m_new) + sum_k p v
        {
            const float a = sh.scale_old[qh];
            acc.x *= a;
            acc.y *= a;
            for (int kk = 0; kk < len; ++kk) {
                const float p = sh.ps[qh][kk];
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(sh.vs + kk * kKvRow + lane * 4));
                acc.x = fmaf(p, v.x, acc.x);
                acc.y = fmaf(p, v.y, acc.y);
            }
        }
        __syncthreads();                                        // the chunk buffers are refilled next
    }
    return acc;
}

// Partials of `kSplits` ranges for (query row r, kv head h): m, l at [(r * 8 + h) * kSplits + s][8], acc after them.
struct AttnPartials {
    float* base;
    size_t rows;                                                 // query rows the buffer holds
    __device__ __forceinline__ size_t idx(int r, int h, int s) const {
        return ((size_t(r) * kKvHeads + h) * kSplits + s) * kGroup;
    }
    __device__ __forceinline__ float* m() const { return base; }
    __device__ __forceinline__ float* l() const { return base + rows * kKvHeads * kSplits * kGroup; }
    __device__ __forceinline__ float* acc() const { return base + 2 * rows * kKvHeads * kSplits * kGroup; }
};

__device__ __forceinline__ void store_partials(const AttnShared& sh, const AttnPartials& P, int r, int h, int s,
                                               float2 acc) {
    const int qh = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t b = P.idx(r, h, s) + qh;
    if (lane == 0) {
        P.m()[b] = sh.cm[qh];
        P.l()[b] = sh.cl[qh];
    }
    *reinterpret_cast<float2*>(P.acc() + b * kHeadDim + 2 * lane) = acc;
}

// Warp qh of the calling CTA merges row r / head h's partials with the sink into out (the 64 query heads' rows).
__device__ __forceinline__ void merge_partials(const AttnPartials& P, int r, int h, const float* sinks, float* out) {
    const int qh = threadIdx.x >> 5, lane = threadIdx.x & 31, head = h * kGroup + qh;
    const float sink = sinks[head];
    float M = sink;
    for (int s = 0; s < kSplits; ++s) M = fmaxf(M, __ldcg(P.m() + P.idx(r, h, s) + qh));
    float l = expf(sink - M);
    float2 o = make_float2(0.f, 0.f);
    for (int s = 0; s < kSplits; ++s) {
        const size_t b = P.idx(r, h, s) + qh;
        const float m = __ldcg(P.m() + b);
        if (m == -INFINITY) continue;                           // a range with no keys
        const float a = expf(m - M);
        l = fmaf(__ldcg(P.l() + b), a, l);
        const float2 v = __ldcg(reinterpret_cast<const float2*>(P.acc() + b * kHeadDim + 2 * lane));
        o.x = fmaf(v.x, a, o.x);
        o.y = fmaf(v.y, a, o.y);
    }
    const float inv = 1.f / l;
    *reinterpret_cast<float2*>(out + size_t(head) * kHeadDim + 2 * lane) = make_float2(o.x * inv, o.y * inv);
}

__device__ __forceinline__ void visible_range(int pos, int window, int sp, int& first, int& n, int& k0, int& k1) {
    n = window > 0 ? min(pos + 1, window) : pos + 1;
    first = pos + 1 - n;
    const int L = (n + kSplits - 1) / kSplits;
    k0 = min(n, sp * L);
    k1 = min(n, k0 + L);
}

__device__ __forceinline__ void load_cache_kv(const __half* kc, const __half* vc, int h, int p, int window, int part16,
                                              uint4& kw, uint4& vw) {
    const size_t slot = window > 0 ? size_t(p % window) : size_t(p);
    const size_t off = (slot * kKvHeads + h) * kHeadDim * 2 + part16 * 16;
    kw = ldg_stream(reinterpret_cast<const uint8_t*>(kc) + off);
    vw = ldg_stream(reinterpret_cast<const uint8_t*>(vc) + off);
}

// The ABI's attention for one query whose key and value are already in the cache: grid (8 kv heads, kSplits).
__global__ void __launch_bounds__(kAttnThreads) attention_partial_kernel(const float* __restrict__ q,
                                                                         const __half* __restrict__ kc,
                                                                         const __half* __restrict__ vc,
                                                                         const int* d_pos, int pos_arg, int window,
                                                                         float* __restrict__ part) {
    __shared__ AttnShared sh;
    const int h = blockIdx.x, sp = blockIdx.y, tid = threadIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    const int pos = d_pos ? *d_pos : pos_arg;
    int first, n, k0, k1;
    visible_range(pos, window, sp, first, n, k0, k1);
    for (int i = tid; i < kGroup * kHeadDim; i += kAttnThreads) sh.qs[i / kHeadDim][i % kHeadDim] = q[h * kGroup * kHeadDim + i];
    const float2 acc = attend_keys(sh, k0, k1, [&](int kk, int part16, uint4& kw, uint4& vw) {
        load_cache_kv(kc, vc, h, first + kk, window, part16, kw, vw);
    });
    store_partials(sh, AttnPartials{part, 1}, 0, h, sp, acc);
}

// One CTA per key/value head, one warp per query head: merges the partials with the sinks.
__global__ void __launch_bounds__(kAttnThreads) attention_combine_kernel(const float* __restrict__ part,
                                                                         const float* __restrict__ sinks,
                                                                         float* __restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    merge_partials(AttnPartials{const_cast<float*>(part), 1}, 0, blockIdx.x, sinks, out);
}

// RoPE pair i of a head row x (in registers of the caller): (x1, x2) -> (x1 c - x2 s, x2 c + x1 s), rounded per op.
__device__ __forceinline__ float2 rotate_pair(float x1, float x2, float c, float s) {
    return make_float2(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)), __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
}

// The attention of one decode step in one launch (the engine's path), grid (8 key/value heads, nsplit):
//   * before the dependency wait (the cache of older positions and the device position were written by kernels that
//     completed before this one was launched: every kernel of the step waits for its predecessor before it ends),
//     CTA (h, s) computes its range of visible keys and starts asynchronous copies of their keys and values into
//     shared memory (up to kStepCap keys per pass), then releases the next kernel's launch;
//   * after the wait it rotates its 8 query heads from the raw QKV output (query in registers, 8 dims of the 8 heads
//     per lane); the CTA whose range holds the new position rotates that position's key, rounds key and value to
//     fp16, appends them to the cache and uses those values for the position;
//   * scores (an 8-lane group per key), the running softmax per query head (warp) and p·v (a lane per 2 dims);
//   * the last CTA of each key/value head to finish (a per-head counter, reset by that CTA) merges the head's
//     partials with the sinks.
// nsplit (<= kStepMaxSplits) is chosen per launch: many splits for a full-context layer, few for a window layer.
constexpr int kStepCap = 144, kStepMaxSplits = 32;

struct StepShared {
    __align__(16) uint8_t ks[kStepCap * 128];                   // keys of the pass, 128 bytes (64 fp16) each
    __align__(16) uint8_t vs[kStepCap * 128];
    __align__(16) float ps[kGroup][kStepCap];                   // scores, then exp(score - m_new)
    __align__(16) __half newkv[2][kHeadDim];                    // the new position's key and value (fp16)
    float cm[kGroup], cl[kGroup], scale_old[kGroup];
};

// m, l at [(h * kStepMaxSplits + s) * 8 + g] (two arrays), acc [.. * 64] after them; counters after the partials
struct StepPartials {
    float* base;
    __device__ __forceinline__ size_t idx(int h, int s) const { return (size_t(h) * kStepMaxSplits + s) * kGroup; }
    __device__ __forceinline__ float* m() const { return base; }
    __device__ __forceinline__ float* l() const { return base + kKvHeads * kStepMaxSplits * kGroup; }
    __device__ __forceinline__ float* acc() const { return base + 2 * kKvHeads * kStepMaxSplits * kGroup; }
};

__device__ __forceinline__ void cp_async16_cg(void* smem_dst, const void* gsrc) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__global__ void __launch_bounds__(kAttnThreads, 2) attention_step_kernel(const float* __restrict__ qkv,
                                                                         const float* __restrict__ cos_t,
                                                                         const float* __restrict__ sin_t,
                                                                         __half* kc, __half* vc,
                                                                         const float* __restrict__ sinks,
                                                                         const int* d_pos, int window, int nsplit,
                                                                         float* part, unsigned* counters,
                                                                         float* out) {
    __shared__ StepShared sh;
    __shared__ bool last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, qh = warp, sub = lane & 7;
    const int h = blockIdx.x, sp = blockIdx.y;
    const int pos = *d_pos;
    const int n = window > 0 ? min(pos + 1, window) : pos + 1, first = pos + 1 - n;
    const int L = (n + nsplit - 1) / nsplit, k0 = min(n, sp * L), k1 = min(n, k0 + L);
    const bool holds_new = k0 <= n - 1 && n - 1 < k1;
    const uint8_t* kcb = reinterpret_cast<const uint8_t*>(kc);
    const uint8_t* vcb = reinterpret_cast<const uint8_t*>(vc);
    // keys [c0, c0 + len) of the range into shared memory (all but the new position's), asynchronously
    auto stage = [&](int c0, int len) {
        for (int i = tid; i < len * 8; i += kAttnThreads) {
            const int kk = i >> 3, part16 = i & 7;
            if (c0 + kk == n - 1) continue;
            const int p = first + c0 + kk;
            const size_t slot = window > 0 ? size_t(p % window) : size_t(p);
            const size_t off = (slot * kKvHeads + h) * kHeadDim * 2 + part16 * 16;
            cp_async16_cg(sh.ks + kk * 128 + part16 * 16, kcb + off);
            cp_async16_cg(sh.vs + kk * 128 + part16 * 16, vcb + off);
        }
    };
    stage(k0, min(kStepCap, k1 - k0));
    if (tid < kGroup) {
        sh.cm[tid] = -INFINITY;
        sh.cl[tid] = 0.f;
    }
    pdl_launch_dependents();
    pdl_wait();
    // query heads: lane (sub = lane % 8) keeps dims 8 sub .. 8 sub + 7 of all 8 heads; warp j rotates head j's pairs
    // into the score buffer first (as a staging area), the new key / value go to newkv
    float qr[kGroup][8];
    {
        const float c = cos_t[size_t(pos) * kPairs + lane], sn = sin_t[size_t(pos) * kPairs + lane];
        const float* base = qkv + (h * kGroup + warp) * kHeadDim;
        const float2 r = rotate_pair(base[lane], base[lane + kPairs], c, sn);
        sh.ps[warp][lane] = r.x;
        sh.ps[warp][lane + kPairs] = r.y;
        if (holds_new && warp == 0) {
            const float* kb = qkv + (kHeads + h) * kHeadDim;
            const float2 rk = rotate_pair(kb[lane], kb[lane + kPairs], c, sn);
            sh.newkv[0][lane] = __float2half_rn(rk.x);
            sh.newkv[0][lane + kPairs] = __float2half_rn(rk.y);
        } else if (holds_new && warp == 1) {
            const float* vb = qkv + (kHeads + kKvHeads + h) * kHeadDim;
            sh.newkv[1][lane] = __float2half_rn(vb[lane]);
            sh.newkv[1][lane + kPairs] = __float2half_rn(vb[lane + kPairs]);
        }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kGroup; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) qr[g][e] = sh.ps[g][sub * 8 + e];
    if (holds_new && tid < 16) {                                // the new position's key and value into the cache
        const size_t slot = window > 0 ? size_t(pos % window) : size_t(pos);
        const size_t off = (slot * kKvHeads + h) * kHeadDim * 2 + (tid & 7) * 16;
        uint8_t* dst = reinterpret_cast<uint8_t*>(tid < 8 ? kc : vc) + off;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(
            reinterpret_cast<const uint8_t*>(sh.newkv[tid >> 3]) + (tid & 7) * 16);
    }
    float2 acc = make_float2(0.f, 0.f);
    for (int c0 = k0; c0 < k1; c0 += kStepCap) {
        const int len = min(kStepCap, k1 - c0);
        if (c0 != k0) stage(c0, len);
        cp_async_commit_wait_all();
        __syncthreads();                                        // every copy landed; qr read before ps is reused
        if (c0 <= n - 1 && n - 1 < c0 + len && tid < 16)        // the new position from this kernel's own rotation
            *reinterpret_cast<uint4*>((tid < 8 ? sh.ks : sh.vs) + (n - 1 - c0) * 128 + (tid & 7) * 16) =
                *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(sh.newkv[tid >> 3]) + (tid & 7) * 16);
        __syncthreads();
        // scores: an 8-lane group per key (each lane 8 dims of the 8 heads), 4 keys per warp pass; the group's partial
        // dots are reduced so that lane j of the group ends with head j's dot
        for (int kb = warp * 4; kb < len; kb += (kAttnThreads / 32) * 4) {
            const int kk = kb + (lane >> 3);
            float d[kGroup];
            {
                const uint4 u = kk < len ? *reinterpret_cast<const uint4*>(sh.ks + kk * 128 + sub * 16)
                                         : make_uint4(0u, 0u, 0u, 0u);
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
                float kv[8];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[t]));
                    kv[2 * t] = f.x;
                    kv[2 * t + 1] = f.y;
                }
#pragma unroll
                for (int g = 0; g < kGroup; ++g) {
                    float t = 0.f;
#pragma unroll
                    for (int e = 0; e < 8; ++e) t = fmaf(qr[g][e], kv[e], t);
                    d[g] = t;
                }
            }
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const bool up = sub & 4;
                const float recv = __shfl_xor_sync(kFull, up ? d[g] : d[g + 4], 4);
                d[g] = (up ? d[g + 4] : d[g]) + recv;
            }
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                const bool up = sub & 2;
                const float recv = __shfl_xor_sync(kFull, up ? d[g] : d[g + 2], 2);
                d[g] = (up ? d[g + 2] : d[g]) + recv;
            }
            {
                const bool up = sub & 1;
                const float recv = __shfl_xor_sync(kFull, up ? d[0] : d[1], 1);
                d[0] = (up ? d[1] : d[0]) + recv;
            }
            if (kk < len) sh.ps[sub][kk] = d[0] * 0.125f;          // scale 1 / sqrt(64)
        }
        __syncthreads();
        // per query head (warp qh): chunk max, new running max, exp, chunk sum
        {
            float m = -INFINITY;
            for (int kk = lane; kk < len; kk += 32) m = fmaxf(m, sh.ps[qh][kk]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
            const float m_old = sh.cm[qh], m_new = fmaxf(m_old, m);
            float ssum = 0.f;
            for (int kk = lane; kk < len; kk += 32) {
                const float e = expf(sh.ps[qh][kk] - m_new);
                sh.ps[qh][kk] = e;
                ssum += e;
            }
            ssum = warp_sum(ssum);
            const float a = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
            __syncwarp();
            if (lane == 0) {
                sh.cl[qh] = sh.cl[qh] * a + ssum;
                sh.cm[qh] = m_new;
            }
            // acc = acc exp(m_old - m_new) + sum_k p v (two accumulator pairs, keys in fours)
            float2 acc2 = make_float2(0.f, 0.f);
            acc.x *= a;
            acc.y *= a;
            const uint8_t* vrow = sh.vs + lane * 4;
            int kk = 0;
            for (; kk + 4 <= len; kk += 4) {
                const float4 p4 = *reinterpret_cast<const float4*>(&sh.ps[qh][kk]);
                const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(vrow + (kk + 0) * 128));
                const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(vrow + (kk + 1) * 128));
                const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(vrow + (kk + 2) * 128));
                const float2 v3 = __half22float2(*reinterpret_cast<const __half2*>(vrow + (kk + 3) * 128));
                acc.x = fmaf(p4.x, v0.x, acc.x);
                acc.y = fmaf(p4.x, v0.y, acc.y);
                acc2.x = fmaf(p4.y, v1.x, acc2.x);
                acc2.y = fmaf(p4.y, v1.y, acc2.y);
                acc.x = fmaf(p4.z, v2.x, acc.x);
                acc.y = fmaf(p4.z, v2.y, acc.y);
                acc2.x = fmaf(p4.w, v3.x, acc2.x);
                acc2.y = fmaf(p4.w, v3.y, acc2.y);
            }
            for (; kk < len; ++kk) {
                const float p = sh.ps[qh][kk];
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(vrow + kk * 128));
                acc.x = fmaf(p, v.x, acc.x);
                acc.y = fmaf(p, v.y, acc.y);
            }
            acc.x += acc2.x;
            acc.y += acc2.y;
        }
        __syncthreads();                                        // the pass's buffers are refilled next
    }
    const StepPartials P{part};
    {
        const size_t b = P.idx(h, sp) + qh;
        if (lane == 0) {
            P.m()[b] = sh.cm[qh];
            P.l()[b] = sh.cl[qh];
        }
        *reinterpret_cast<float2*>(P.acc() + b * kHeadDim + 2 * lane) = acc;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(counters + h, 1u) == unsigned(nsplit - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    {
        const int head = h * kGroup + qh;
        const float sink = sinks[head];
        float M = sink;
        for (int s2 = 0; s2 < nsplit; ++s2) M = fmaxf(M, __ldcg(P.m() + P.idx(h, s2) + qh));
        float l = expf(sink - M);
        float2 o = make_float2(0.f, 0.f);
        for (int s2 = 0; s2 < nsplit; ++s2) {
            const size_t b = P.idx(h, s2) + qh;
            const float m = __ldcg(P.m() + b);
            if (m == -INFINITY) continue;                       // a range with no keys
            const float a = expf(m - M);
            l = fmaf(__ldcg(P.l() + b), a, l);
            const float2 v = __ldcg(reinterpret_cast<const float2*>(P.acc() + b * kHeadDim + 2 * lane));
            o.x = fmaf(v.x, a, o.x);
            o.y = fmaf(v.y, a, o.y);
        }
        const float inv = 1.f / l;
        *reinterpret_cast<float2*>(out + size_t(head) * kHeadDim + 2 * lane) = make_float2(o.x * inv, o.y * inv);
    }
    if (tid == 0) counters[h] = 0;
}

// ---------------------------------------------------------------------------------------------------- prefill
// Attention of a batch of n consecutive positions p0 .. p0 + n - 1 of one sequence (prefill), grid (8 kv heads,
// kSplits, rows of this chunk). Query row r (position p0 + r0 + r) was rotated in place in qkv; the batch's own keys
// and values (rotated, rounded to fp16) are in kvb [n][2][8][64] and are read from there, older positions from the
// cache (a sliding-window cache may already have been overwritten by the batch's later positions, so the batch is
// appended to the cache only after its attention).
__global__ void __launch_bounds__(kAttnThreads) attention_prefill_kernel(const float* __restrict__ qkv, int r0,
                                                                         const __half* __restrict__ kvb,
                                                                         const __half* __restrict__ kc,
                                                                         const __half* __restrict__ vc, int p0,
                                                                         int window, float* __restrict__ part,
                                                                         size_t part_rows) {
    __shared__ AttnShared sh;
    const int h = blockIdx.x, sp = blockIdx.y, r = blockIdx.z, tid = threadIdx.x;
    const int row = r0 + r, pos = p0 + row;
    int first, n, k0, k1;
    visible_range(pos, window, sp, first, n, k0, k1);
    for (int i = tid; i < kGroup * kHeadDim; i += kAttnThreads)
        sh.qs[i / kHeadDim][i % kHeadDim] = qkv[size_t(row) * kQkv + h * kGroup * kHeadDim + i];
    const float2 acc = attend_keys(sh, k0, k1, [&](int kk, int part16, uint4& kw, uint4& vw) {
        const int p = first + kk;
        if (p >= p0) {
            const uint8_t* b = reinterpret_cast<const uint8_t*>(kvb) + (size_t(p - p0) * 2 * kKvHeads + h) * kHeadDim * 2;
            kw = *reinterpret_cast<const uint4*>(b + part16 * 16);
            vw = *reinterpret_cast<const uint4*>(b + kKvHeads * kHeadDim * 2 + part16 * 16);
        } else {
            load_cache_kv(kc, vc, h, p, window, part16, kw, vw);
        }
    });
    store_partials(sh, AttnPartials{part, part_rows}, r, h, sp, acc);
}

// grid (8 kv heads, rows of the chunk): merges each row's partials into out[r0 + r][4096].
__global__ void __launch_bounds__(kAttnThreads) attention_prefill_merge_kernel(const float* part, size_t part_rows,
                                                                               int r0, const float* __restrict__ sinks,
                                                                               float* out) {
    const int r = blockIdx.y;
    merge_partials(AttnPartials{const_cast<float*>(part), part_rows}, r, blockIdx.x, sinks,
                   out + size_t(r0 + r) * kHeads * kHeadDim);
}

// Per batch row t (position p0 + t): qkv += bias; q and k rotated in place; the rotated k and the v rounded to fp16
// into kvb[t] ([2][8][64]). One CTA per row, one thread per rotary pair (72 heads x 32 pairs) and per v pair.
__global__ void __launch_bounds__(256) prefill_qkv_rope_kernel(float* qkv, const float* __restrict__ bias,
                                                               const float* __restrict__ cos_t,
                                                               const float* __restrict__ sin_t, int p0, __half* kvb) {
    const int t = blockIdx.x, pos = p0 + t;
    float* row = qkv + size_t(t) * kQkv;
    __half* kv = kvb + size_t(t) * 2 * kKvHeads * kHeadDim;
    for (int p = threadIdx.x; p < (kHeads + kKvHeads) * kPairs; p += blockDim.x) {
        const int head = p / kPairs, i = p % kPairs;
        float* base = row + head * kHeadDim;
        const float x1 = base[i] + bias[head * kHeadDim + i], x2 = base[i + kPairs] + bias[head * kHeadDim + i + kPairs];
        const float2 r = rotate_pair(x1, x2, cos_t[size_t(pos) * kPairs + i], sin_t[size_t(pos) * kPairs + i]);
        base[i] = r.x;
        base[i + kPairs] = r.y;
        if (head >= kHeads) {
            const int kh = head - kHeads;
            kv[kh * kHeadDim + i] = __float2half_rn(r.x);
            kv[kh * kHeadDim + i + kPairs] = __float2half_rn(r.y);
        }
    }
    for (int i = threadIdx.x; i < kKvHeads * kHeadDim; i += blockDim.x) {
        const int c = (kHeads + kKvHeads) * kHeadDim + i;
        const float v = row[c] + bias[c];
        row[c] = v;
        kv[kKvHeads * kHeadDim + i] = __float2half_rn(v);
    }
}

// Appends batch rows [t0, n) of kvb to the cache (positions p0 + t; slot p % window or p). One thread per 16 bytes.
__global__ void prefill_append_kernel(const __half* __restrict__ kvb, int t0, int n, int p0, int window, __half* kc,
                                      __half* vc) {
    const size_t per_row = 2 * kKvHeads * kHeadDim * 2 / 16;    // 16-byte pieces per row (k then v)
    const size_t total = size_t(n - t0) * per_row;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int t = t0 + int(i / per_row), piece = int(i % per_row);
        const int p = p0 + t;
        const size_t slot = window > 0 ? size_t(p % window) : size_t(p);
        const bool is_v = piece >= int(per_row / 2);
        const int pp = is_v ? piece - int(per_row / 2) : piece;
        const uint4 w = reinterpret_cast<const uint4*>(kvb + size_t(t) * 2 * kKvHeads * kHeadDim)[piece];
        reinterpret_cast<uint4*>((is_v ? vc : kc) + slot * kKvHeads * kHeadDim)[pp] = w;
    }
}

// Row-wise split for the tensor-core projections: y = RMSNorm(x; g) (g null: y = x), hi = bf16(y), lo = bf16(y -
// hi), so hi + lo carries 16 significant bits of y. One CTA per row.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int K, const float* __restrict__ g,
                                                         float eps, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    __shared__ float part[8];
    const float* xr = x + size_t(blockIdx.x) * K;
    float r = 1.f;
    if (g) {
        float ss = 0.f;
        for (int i = threadIdx.x * 4; i < K; i += 1024) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            ss = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, ss))));
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) tot += part[w];
        r = rms_scale(tot, K, eps);
    }
    for (int i = threadIdx.x; i < K; i += 256) {
        const float y = g ? xr[i] * r * g[i] : xr[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(y);
        hi[size_t(blockIdx.x) * K + i] = h;
        lo[size_t(blockIdx.x) * K + i] = __float2bfloat16_rn(y - __bfloat162float(h));
    }
}

// x[t][i] += b[i] for n rows.
__global__ void add_bias_rows_kernel(float* x, const float* __restrict__ b, int n, int K) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < size_t(n) * K; i += size_t(gridDim.x) * blockDim.x)
        x[i] += b[i % K];
}

// x[t] = embed[tokens[t]] for n tokens.
__global__ void embed_rows_kernel(const __nv_bfloat16* __restrict__ table, const int* __restrict__ tokens, float* x,
                                  int H) {
    const size_t t = size_t(tokens[blockIdx.x]);
    for (int i = threadIdx.x; i < H; i += blockDim.x) x[size_t(blockIdx.x) * H + i] = __bfloat162float(table[t * H + i]);
}

// ---------------------------------------------------------------------------------------------------- misc
// x = embed[token] (bf16 row, widened exactly); the token comes from device memory.
__global__ void embed_kernel(const __nv_bfloat16* __restrict__ table, const int* d_token, float* x, int H) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t t = size_t(*d_token);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
        x[i] = __bfloat162float(table[t * H + i]);
}

__global__ void increment_kernel(int* p) {
    pdl_wait();
    pdl_launch_dependents();
    *p += 1;
}

// Score of the logits [V]: every CTA folds its range into (max, sum of exp(l - max), best value, best index, ties to
// the lower index); the last CTA to finish (counter) folds the partials in CTA order and writes lse = max + log(sum),
// argmax, lp[i] = logits[ids[i]] - lse, target_lp (target >= 0) and, if `next_token` is given, argmax there too (the
// next token of a greedy decode). The counter is reset by that CTA.
constexpr int kScoreThreads = 512;

__global__ void __launch_bounds__(kScoreThreads) score_kernel(const float* __restrict__ logits, int V,
                                                              float4* __restrict__ work, unsigned* counter,
                                                              const int* __restrict__ ids, int k, int target,
                                                              float* lp, int* argmax, float* target_lp, float* lse,
                                                              int* next_token) {
    __shared__ float s_m[kScoreThreads / 32], s_s[kScoreThreads / 32], s_b[kScoreThreads / 32];
    __shared__ int s_i[kScoreThreads / 32];
    __shared__ bool last;
    __shared__ float lse_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait();
    pdl_launch_dependents();
    const int per = (V + gridDim.x - 1) / gridDim.x;
    const int b0 = min(V, int(blockIdx.x) * per), b1 = min(V, b0 + per);
    // one pass with a running (max, sum): s is kept relative to m
    float m = -INFINITY, s = 0.f, best = -INFINITY;
    int bi = INT_MAX;
    for (int i = b0 + tid; i < b1; i += kScoreThreads) {
        const float v = logits[i];
        if (v > m) {
            s = (m == -INFINITY ? 0.f : s * expf(m - v)) + 1.f;
            m = v;
        } else {
            s += expf(v - m);
        }
        if (v > best) {                                         // i ascends within a thread: first max kept
            best = v;
            bi = i;
        }
    }
    auto merge = [](float& m1, float& s1, float m2, float s2) {
        if (m2 == -INFINITY) return;
        if (m1 == -INFINITY) { m1 = m2; s1 = s2; return; }
        const float mm = fmaxf(m1, m2);
        s1 = s1 * expf(m1 - mm) + s2 * expf(m2 - mm);
        m1 = mm;
    };
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(kFull, m, o), os = __shfl_xor_sync(kFull, s, o);
        const float ob = __shfl_xor_sync(kFull, best, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        merge(m, s, om, os);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) { s_m[warp] = m; s_s[warp] = s; s_b[warp] = best; s_i[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        float M = -INFINITY, S = 0.f, B = -INFINITY;
        int BI = INT_MAX;
        for (int w = 0; w < kScoreThreads / 32; ++w) {
            merge(M, S, s_m[w], s_s[w]);
            if (s_b[w] > B || (s_b[w] == B && s_i[w] < BI)) { B = s_b[w]; BI = s_i[w]; }
        }
        work[blockIdx.x] = make_float4(M, S, B, __int_as_float(BI));
        __threadfence();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) {
        float M = -INFINITY, S = 0.f, B = -INFINITY;
        int BI = INT_MAX;
        for (int b = 0; b < int(gridDim.x); ++b) {
            const float4 w = __ldcg(work + b);
            merge(M, S, w.x, w.y);
            const int wi = __float_as_int(w.w);
            if (w.z > B || (w.z == B && wi < BI)) { B = w.z; BI = wi; }
        }
        lse_s = M + logf(S);
        if (argmax) *argmax = BI;
        if (lse) *lse = lse_s;
        if (next_token) *next_token = BI;
        if (target_lp && target >= 0) *target_lp = logits[target] - lse_s;
        *counter = 0;
    }
    __syncthreads();
    for (int i = tid; i < k; i += kScoreThreads) lp[i] = logits[ids[i]] - lse_s;
}

template <class... KArgs, class... Args>
void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
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

}  // namespace ds

// ---------------------------------------------------------------------------------------------------- host API
void launch_gemv_bf16(const void* W, const float* x, const float* norm_w, float eps, const float* bias,
                      const float* resid, float* y, int N, int K, cudaStream_t s, bool pdl) {
    require(N >= 1 && K >= 8 && K % 8 == 0, "gemv_bf16: need N >= 1 and K a positive multiple of 8");
    require(size_t(K) * 4 <= 200 * 1024, "gemv_bf16: K too large for the staged x");
    const size_t smem = size_t(K) * 4;
    static std::mutex mu;
    static int set[64] = {};
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    require(dev >= 0 && dev < 64, "gemv_bf16: device ordinal out of range");
    {
        std::lock_guard<std::mutex> lock(mu);
        if (int(smem) > set[dev] && smem > 48 * 1024) {
            GPT_CHECK(cudaFuncSetAttribute(ds::gemv_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            set[dev] = int(smem);
        }
    }
    const int warps_needed = (N + ds::kRows - 1) / ds::kRows;
    const int grid = std::max(1, std::min(num_sms() * ds::kGemvCtasPerSm, (warps_needed + 7) / 8));
    // matrices that fit in a half of L2 are prefetched whole, larger ones (the LM head) one row group per warp
    const int pf_groups = size_t(N) * K * 2 <= (size_t(64) << 20) ? INT_MAX : 1;
    ds::launch(ds::gemv_bf16_kernel, dim3(grid), dim3(ds::kGemvThreads), smem, s, pdl,
               static_cast<const __nv_bfloat16*>(W), x, norm_w, eps, bias, resid, y, N, K, pf_groups);
}

void launch_rope_append(float* qkv, const float* cos_t, const float* sin_t, const int* d_pos, int pos, void* k_cache,
                        void* v_cache, int window, cudaStream_t s, bool pdl) {
    require(window >= 0, "rope_append: window must be >= 0");
    ds::launch(ds::rope_append_kernel, dim3(9), dim3(256), 0, s, pdl, qkv, cos_t, sin_t, d_pos, pos,
               static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), window);
}

// partials (m, l, acc) of every (head, split), then 8 per-head counters (zero-filled before the first use); sized
// for the larger of the step kernel's and the two-kernel attention's split counts
size_t attention_workspace_floats() {
    return size_t(ds::kKvHeads) * std::max(ds::kSplits, ds::kStepMaxSplits) * ds::kGroup * (2 + ds::kHeadDim) + 16;
}

void launch_attention_step(const float* qkv, const float* cos_t, const float* sin_t, void* k_cache, void* v_cache,
                           const float* sinks, const int* d_pos, int window, float* part, float* out, cudaStream_t s,
                           bool pdl) {
    require(window >= 0, "attention: window must be >= 0");
    unsigned* counters = reinterpret_cast<unsigned*>(part + (attention_workspace_floats() - 16));
    // a window layer's keys (<= window) in few ranges, a full layer's in kStepMaxSplits ranges (one pass each up to
    // kStepMaxSplits * kStepCap = 4608 visible keys)
    const int nsplit = window > 0 ? std::min(ds::kStepMaxSplits, std::max(1, (window + 31) / 32)) : ds::kStepMaxSplits;
    ds::launch(ds::attention_step_kernel, dim3(ds::kKvHeads, nsplit), dim3(ds::kAttnThreads), 0, s, pdl, qkv, cos_t,
               sin_t, static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), sinks, d_pos, window, nsplit,
               part, counters, out);
}

void launch_attention(const float* q, const void* k_cache, const void* v_cache, const float* sinks, const int* d_pos,
                      int pos, int window, float* part, float* out, cudaStream_t s, bool pdl) {
    require(window >= 0, "attention: window must be >= 0");
    ds::launch(ds::attention_partial_kernel, dim3(ds::kKvHeads, ds::kSplits), dim3(ds::kAttnThreads), 0, s, pdl, q,
               static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache), d_pos, pos, window, part);
    ds::launch(ds::attention_combine_kernel, dim3(ds::kKvHeads), dim3(ds::kAttnThreads), 0, s, pdl,
               static_cast<const float*>(part), sinks, out);
}

size_t prefill_attention_floats(int rows) {
    return size_t(rows) * ds::kKvHeads * ds::kSplits * ds::kGroup * (2 + ds::kHeadDim);
}

void launch_prefill_qkv_rope(float* qkv, const float* bias, const float* cos_t, const float* sin_t, int p0, int n,
                             void* kvb, cudaStream_t s) {
    ds::prefill_qkv_rope_kernel<<<n, 256, 0, s>>>(qkv, bias, cos_t, sin_t, p0, static_cast<__half*>(kvb));
    check_launch("prefill qkv rope");
}

void launch_prefill_attention(const float* qkv, const void* kvb, const void* k_cache, const void* v_cache,
                              const float* sinks, int p0, int n, int window, float* part, int part_rows, float* out,
                              cudaStream_t s) {
    for (int r0 = 0; r0 < n; r0 += part_rows) {
        const int rows = std::min(part_rows, n - r0);
        ds::attention_prefill_kernel<<<dim3(ds::kKvHeads, ds::kSplits, rows), ds::kAttnThreads, 0, s>>>(
            qkv, r0, static_cast<const __half*>(kvb), static_cast<const __half*>(k_cache),
            static_cast<const __half*>(v_cache), p0, window, part, size_t(part_rows));
        check_launch("prefill attention");
        ds::attention_prefill_merge_kernel<<<dim3(ds::kKvHeads, rows), ds::kAttnThreads, 0, s>>>(
            part, size_t(part_rows), r0, sinks, out);
        check_launch("prefill attention merge");
    }
}

void launch_prefill_append(const void* kvb, int p0, int n, int window, void* k_cache, void* v_cache, cudaStream_t s) {
    const int t0 = window > 0 ? std::max(0, n - window) : 0;  // a window cache keeps only the last `window`
    if (t0 >= n) return;
    const size_t pieces = size_t(n - t0) * 2 * ds::kKvHeads * ds::kHeadDim * 2 / 16;
    const int grid = int(std::min<size_t>((pieces + 255) / 256, size_t(num_sms()) * 8));
    ds::prefill_append_kernel<<<std::max(1, grid), 256, 0, s>>>(static_cast<const __half*>(kvb), t0, n, p0, window,
                                                               static_cast<__half*>(k_cache), static_cast<__half*>(v_cache));
    check_launch("prefill append");
}

void launch_split_rows(const float* x, int n, int K, const float* norm_w, float eps, void* hi, void* lo, cudaStream_t s) {
    require(K % 4 == 0, "split_rows: K must be a multiple of 4");
    ds::split_rows_kernel<<<n, 256, 0, s>>>(x, K, norm_w, eps, static_cast<__nv_bfloat16*>(hi),
                                            static_cast<__nv_bfloat16*>(lo));
    check_launch("split rows");
}

void launch_add_bias_rows(float* x, const float* b, int n, int K, cudaStream_t s) {
    const size_t total = size_t(n) * K;
    const int grid = int(std::min<size_t>((total + 255) / 256, size_t(num_sms()) * 8));
    ds::add_bias_rows_kernel<<<std::max(1, grid), 256, 0, s>>>(x, b, n, K);
    check_launch("add bias rows");
}

void launch_embed_rows(const void* table, const int* tokens, float* x, int n, int H, cudaStream_t s) {
    ds::embed_rows_kernel<<<n, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(table), tokens, x, H);
    check_launch("embed rows");
}

void launch_embed(const void* table, const int* d_token, float* x, int H, cudaStream_t s, bool pdl) {
    ds::launch(ds::embed_kernel, dim3((H + 255) / 256), dim3(256), 0, s, pdl, static_cast<const __nv_bfloat16*>(table),
               d_token, x, H);
}

void launch_increment(int* p, cudaStream_t s, bool pdl) { ds::launch(ds::increment_kernel, dim3(1), dim3(1), 0, s, pdl, p); }

size_t score_workspace_bytes() { return size_t(num_sms()) * sizeof(float4) + 256; }

void launch_score(const float* logits, int V, void* work, const int* ids, int k, int target, float* lp, int* argmax,
                  float* target_lp, float* lse, int* next_token, cudaStream_t s, bool pdl) {
    require(V >= 1, "score: V must be positive");
    const int grid = std::min(num_sms(), std::max(1, (V + ds::kScoreThreads - 1) / ds::kScoreThreads));
    float4* w = static_cast<float4*>(work);
    unsigned* counter = reinterpret_cast<unsigned*>(static_cast<char*>(work) + size_t(num_sms()) * sizeof(float4));
    ds::launch(ds::score_kernel, dim3(grid), dim3(ds::kScoreThreads), 0, s, pdl, logits, V, w, counter, ids, k, target,
               lp, argmax, target_lp, lse, next_token);
}

}  // namespace gpt
