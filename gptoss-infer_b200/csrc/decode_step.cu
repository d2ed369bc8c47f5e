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
// Every CTA stages x' (fp32) in shared memory (computing the norm itself when g is given: one read of x from L2).
// A warp takes kRows rows at a time; lane l reads the rows' 16-byte chunks l, l + 32, ... with streaming loads (all
// loads of a row group issued before the FMAs) and accumulates in packed fp32 pairs; warp_sum ends each row.
constexpr int kGemvThreads = 256, kRows = 2, kChunksInFlight = 8;

__global__ void __launch_bounds__(kGemvThreads, 2) gemv_bf16_kernel(const __nv_bfloat16* __restrict__ W,
                                                                    const float* __restrict__ x,
                                                                    const float* __restrict__ g, float eps,
                                                                    const float* __restrict__ bias,
                                                                    const float* resid, float* y, int N, int K) {
    extern __shared__ float xs[];                               // [K]
    __shared__ float part[kGemvThreads / 32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
        for (int i = tid * 4; i < K; i += kGemvThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(x + i), gg = *reinterpret_cast<const float4*>(g + i);
            *reinterpret_cast<float4*>(xs + i) = make_float4(v.x * r * gg.x, v.y * r * gg.y, v.z * r * gg.z,
                                                             v.w * r * gg.w);
        }
    } else {
        for (int i = tid * 4; i < K; i += kGemvThreads * 4)
            *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(x + i);
    }
    __syncthreads();
    pdl_launch_dependents();
    const int K8 = K >> 3;
    const uint4* Wv = reinterpret_cast<const uint4*>(W);
    const int gw = blockIdx.x * (kGemvThreads / 32) + warp, nw = gridDim.x * (kGemvThreads / 32);
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
                    const float4 xa = *reinterpret_cast<const float4*>(xs + 8 * c);
                    const float4 xb = *reinterpret_cast<const float4*>(xs + 8 * c + 4);
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
// without; position p lives in cache slot p % window (window) or p. Grid (8 key/value heads, kSplits): CTA (h, s)
// takes positions [first + s L, first + (s + 1) L), L = ceil(n / kSplits), in chunks of kChunk keys staged in shared
// memory (keys and values, fp16, 16-byte loads), and keeps a running softmax for its 8 query heads: m (max score),
// l (sum of exp(score - m)) and acc[8][64] (sum of exp(score - m) v). Scores are q . k / 8 in fp32. The partials
// (m, l, acc) go to `part`; attention_combine_kernel merges the splits with the head's sink logit (one more
// softmax column that carries no value) and writes out = acc / l.
constexpr int kSplits = 18, kChunk = 128, kAttnThreads = 256;
constexpr int kKvRow = kHeadDim * 2 + 16;                       // staged key/value row: 128 bytes + 16 of padding

__global__ void __launch_bounds__(kAttnThreads) attention_partial_kernel(const float* __restrict__ q,
                                                                         const __half* __restrict__ kc,
                                                                         const __half* __restrict__ vc,
                                                                         const int* d_pos, int pos_arg, int window,
                                                                         float* __restrict__ part) {
    __shared__ __align__(16) uint8_t ks[kChunk * kKvRow];
    __shared__ __align__(16) uint8_t vs[kChunk * kKvRow];
    __shared__ float qs[kGroup][kHeadDim];
    __shared__ float ps[kGroup][kChunk];                        // exp(score - m_new) of the chunk
    __shared__ float cm[kGroup], cl[kGroup], scale_old[kGroup];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, sp = blockIdx.y;
    pdl_wait();
    pdl_launch_dependents();
    const int pos = d_pos ? *d_pos : pos_arg;
    const int n = window > 0 ? min(pos + 1, window) : pos + 1;
    const int first = pos + 1 - n;
    const int L = (n + kSplits - 1) / kSplits;
    const int k0 = min(n, sp * L), k1 = min(n, k0 + L);
    for (int i = tid; i < kGroup * kHeadDim; i += kAttnThreads) qs[i / kHeadDim][i % kHeadDim] = q[h * kGroup * kHeadDim + i];
    if (tid < kGroup) {
        cm[tid] = -INFINITY;
        cl[tid] = 0.f;
    }
    // thread (qh = tid / 32, d pair = lane) owns acc[qh][2 lane .. 2 lane + 1]
    const int qh = warp;
    float2 acc = make_float2(0.f, 0.f);
    __syncthreads();
    for (int c0 = k0; c0 < k1; c0 += kChunk) {
        const int len = min(kChunk, k1 - c0);
        // stage the chunk's keys and values: 8 threads per 128-byte row
        for (int i = tid; i < len * 8; i += kAttnThreads) {
            const int kk = i >> 3, part16 = i & 7;
            const int p = first + c0 + kk;
            const size_t slot = window > 0 ? size_t(p % window) : size_t(p);
            const size_t off = (slot * kKvHeads + h) * kHeadDim * 2 + part16 * 16;
            *reinterpret_cast<uint4*>(ks + kk * kKvRow + part16 * 16) =
                ldg_stream(reinterpret_cast<const uint8_t*>(kc) + off);
            *reinterpret_cast<uint4*>(vs + kk * kKvRow + part16 * 16) =
                ldg_stream(reinterpret_cast<const uint8_t*>(vc) + off);
        }
        __syncthreads();
        // scores: an 8-lane group per key (each lane 8 dims), 4 keys per warp pass; the group's partial dots for the
        // 8 query heads are reduced so that lane j of the group ends with head j's score
        for (int kb = warp * 4; kb < len; kb += (kAttnThreads / 32) * 4) {
            const int kk = kb + (lane >> 3), sub = lane & 7;
            float d[kGroup];
            if (kk < len) {
                const uint4 u = *reinterpret_cast<const uint4*>(ks + kk * kKvRow + sub * 16);
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
                    for (int e = 0; e < 8; ++e) t = fmaf(qs[g][sub * 8 + e], kv[e], t);
                    d[g] = t;
                }
            } else {
#pragma unroll
                for (int g = 0; g < kGroup; ++g) d[g] = 0.f;
            }
            // reduce-scatter over the 8 lanes: after the three steps lane `sub` holds the full dot of head `sub`
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const bool up = sub & 4;
                const float send = up ? d[g] : d[g + 4];
                const float recv = __shfl_xor_sync(kFull, send, 4);
                d[g] = (up ? d[g + 4] : d[g]) + recv;
            }
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                const bool up = sub & 2;
                const float send = up ? d[g] : d[g + 2];
                const float recv = __shfl_xor_sync(kFull, send, 2);
                d[g] = (up ? d[g + 2] : d[g]) + recv;
            }
            {
                const bool up = sub & 1;
                const float send = up ? d[0] : d[1];
                const float recv = __shfl_xor_sync(kFull, send, 1);
                d[0] = (up ? d[1] : d[0]) + recv;
            }
            // lane sub now holds the full dot of query head sub (bit 2 picked heads 4-7, bit 1 the upper pair, bit 0
            // the upper head); the score is the dot scaled by 1 / sqrt(64)
            if (kk < len) ps[sub][kk] = d[0] * 0.125f;
        }
        __syncthreads();
        // per query head (warp qh): chunk max, new running max, exp, chunk sum
        {
            float m = -INFINITY;
            for (int kk = lane; kk < len; kk += 32) m = fmaxf(m, ps[qh][kk]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
            const float m_old = cm[qh], m_new = fmaxf(m_old, m);
            float s = 0.f;
            for (int kk = lane; kk < len; kk += 32) {
                const float e = expf(ps[qh][kk] - m_new);
                ps[qh][kk] = e;
                s += e;
            }
            s = warp_sum(s);
            __syncwarp();
            if (lane == 0) {
                const float a = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                scale_old[qh] = a;
                cl[qh] = cl[qh] * a + s;
                cm[qh] = m_new;
            }
        }
        __syncwarp();
        // acc = acc * exp(m_old - m_new) + sum_k p v (thread: head qh, dims 2 lane .. 2 lane + 1)
        {
            const float a = scale_old[qh];
            acc.x *= a;
            acc.y *= a;
            for (int kk = 0; kk < len; ++kk) {
                const float p = ps[qh][kk];
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(vs + kk * kKvRow + lane * 4));
                acc.x = fmaf(p, v.x, acc.x);
                acc.y = fmaf(p, v.y, acc.y);
            }
        }
        __syncthreads();                                        // the chunk buffers are refilled next
    }
    const size_t base = (size_t(h) * kSplits + sp) * kGroup;
    float* pm = part;
    float* pl = part + kKvHeads * kSplits * kGroup;
    float* pa = part + 2 * kKvHeads * kSplits * kGroup;
    if (lane == 0) {
        pm[base + qh] = cm[qh];
        pl[base + qh] = cl[qh];
    }
    *reinterpret_cast<float2*>(pa + (base + qh) * kHeadDim + 2 * lane) = acc;
}

// One CTA per key/value head, one warp per query head: merges the kSplits partials with the sink column.
__global__ void __launch_bounds__(kAttnThreads) attention_combine_kernel(const float* __restrict__ part,
                                                                         const float* __restrict__ sinks,
                                                                         float* __restrict__ out) {
    const int h = blockIdx.x, qh = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    const int head = h * kGroup + qh;
    const float* pm = part;
    const float* pl = part + kKvHeads * kSplits * kGroup;
    const float* pa = part + 2 * kKvHeads * kSplits * kGroup;
    const float sink = sinks[head];
    float M = sink;
    for (int s = 0; s < kSplits; ++s) M = fmaxf(M, pm[(size_t(h) * kSplits + s) * kGroup + qh]);
    float l = expf(sink - M);
    float2 o = make_float2(0.f, 0.f);
    for (int s = 0; s < kSplits; ++s) {
        const size_t b = (size_t(h) * kSplits + s) * kGroup + qh;
        const float m = pm[b];
        if (m == -INFINITY) continue;                           // a split with no keys
        const float a = expf(m - M);
        l = fmaf(pl[b], a, l);
        const float2 v = *reinterpret_cast<const float2*>(pa + b * kHeadDim + 2 * lane);
        o.x = fmaf(v.x, a, o.x);
        o.y = fmaf(v.y, a, o.y);
    }
    const float inv = 1.f / l;
    *reinterpret_cast<float2*>(out + size_t(head) * kHeadDim + 2 * lane) = make_float2(o.x * inv, o.y * inv);
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
    const int grid = std::max(1, std::min(num_sms() * 2, (warps_needed + 7) / 8));
    ds::launch(ds::gemv_bf16_kernel, dim3(grid), dim3(ds::kGemvThreads), smem, s, pdl,
               static_cast<const __nv_bfloat16*>(W), x, norm_w, eps, bias, resid, y, N, K);
}

void launch_rope_append(float* qkv, const float* cos_t, const float* sin_t, const int* d_pos, int pos, void* k_cache,
                        void* v_cache, int window, cudaStream_t s, bool pdl) {
    require(window >= 0, "rope_append: window must be >= 0");
    ds::launch(ds::rope_append_kernel, dim3(9), dim3(256), 0, s, pdl, qkv, cos_t, sin_t, d_pos, pos,
               static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), window);
}

size_t attention_workspace_floats() { return size_t(ds::kKvHeads) * ds::kSplits * ds::kGroup * (2 + ds::kHeadDim); }

void launch_attention(const float* q, const void* k_cache, const void* v_cache, const float* sinks, const int* d_pos,
                      int pos, int window, float* part, float* out, cudaStream_t s, bool pdl) {
    require(window >= 0, "attention: window must be >= 0");
    ds::launch(ds::attention_partial_kernel, dim3(ds::kKvHeads, ds::kSplits), dim3(ds::kAttnThreads), 0, s, pdl, q,
               static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache), d_pos, pos, window, part);
    ds::launch(ds::attention_combine_kernel, dim3(ds::kKvHeads), dim3(ds::kAttnThreads), 0, s, pdl,
               static_cast<const float*>(part), sinks, out);
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
