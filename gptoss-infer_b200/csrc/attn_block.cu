// The attention block of one bs=1 decode step in one cooperative launch (one CTA per SM):
//   phase A  qkv = Wqkv RMSNorm(x) + bqkv          (CTA c: rows [RA c, RA c + RA) of the 5120)
//   barrier
//   phase B  attention of the new position          (CTA i < 8 * nsplit: key/value head i / nsplit, key range
//            i % nsplit; RoPE of q and of the new key, the new key and value rounded to fp16 into the cache, running
//            softmax with the per-head sink, split partials merged by the last CTA of each head)
//   barrier
//   phase C  x = Wo attn + bo + x                    (CTA c: rows [RC c, RC c + RC) of the H)
// Three dependent steps in one launch instead of three launches (the engine's default is the three launches, which
// measured faster: see gptoss_set_attention_impl).
// Nothing but x depends on the previous kernel, so before the dependency wait every CTA puts all of its QKV rows in
// flight into shared memory (one bulk copy and one mbarrier per row), reads the RMSNorm weight, and asks L2 for its O
// rows and for its share of the cached keys and values of its attention range. After the wait, x is read once: the
// rows are dotted with x * g and the RMSNorm scale (a scalar) is applied to each dot product. The shared memory the
// QKV rows used then holds the staged keys and values of the attention, and after that the CTA's O rows (bulk copies
// from L2, issued as soon as the attention no longer needs the space, so they land during the second barrier). Every
// wait is bounded (error codes 41-45 in the error word; a wait that ran out leaves NaN in what depends on it).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace gpt {
namespace ab {

constexpr int kHeads = 64, kKvHeads = 8, kHeadDim = 64, kGroup = kHeads / kKvHeads, kPairs = kHeadDim / 2;
constexpr int kQD = kHeads * kHeadDim, kKVD = kKvHeads * kHeadDim, kQkv = kQD + 2 * kKVD;   // 4096, 512, 5120
constexpr int kThreads = 256, kWarps = kThreads / 32;
constexpr int kCap = 256;                        // keys staged per pass
constexpr int kMaxSplits = 32;                   // key ranges per head (the partials' layout)
constexpr int kMaxRowsA = 48, kMaxRowsC = 32;    // rows per CTA of phases A and C (one mbarrier each)
constexpr int kRingBytes = 1576 * 128;           // 201,728 bytes: 35 QKV rows of H = 2880, 20 O rows, the staging
constexpr int kFullSplits = 18, kWindowSplits = 4;
constexpr int kMaxH = 3072;                      // x's chunks per lane in registers: phase A H / 256, phase C 4096 / 256
constexpr int kChA = kMaxH / 256, kChC = kQD / 256;

struct Args {
    float* x;                                    // [H] residual stream: read in phase A, updated in phase C
    const float* ln;                             // [H] RMSNorm weight
    float eps;
    const __nv_bfloat16* wqkv;                   // [5120][H]
    const float* bqkv;                           // [5120]
    const __nv_bfloat16* wo;                     // [H][4096]
    const float* bo;                             // [H]
    const float* cos_t;                          // [positions][32]
    const float* sin_t;
    __half* kc;                                  // [slots][8][64]
    __half* vc;
    const float* sinks;                          // [64]
    const int* d_pos;
    int window, nsplit, H;
    int RA, RC;                                  // rows per CTA of phases A and C
    float* qkv;                                  // [5120] workspace
    float* part;                                 // split partials: m, l [8][kMaxSplits][8], acc [8][kMaxSplits][8][64]
    unsigned* counters;                          // [8] per head, zero between launches
    float* attn;                                 // [4096] workspace
    unsigned* gbar;                              // grid barrier word (zero-filled once)
    int* err;
};

struct Smem {
    uint64_t barA[kMaxRowsA], barC[kMaxRowsC];
    __align__(16) float xs[kQD];                 // x * g (phase A), attn (phase C)
    __align__(128) uint8_t ring[kRingBytes];     // QKV rows (A), keys and values of a pass (B), O rows (C)
    __align__(16) float ps[kGroup][kCap];        // scores, then exp(score - m)
    __align__(16) __half newkv[2][kHeadDim];
    float bA[kMaxRowsA], bC[kMaxRowsC], xr[kMaxRowsC];   // the rows' biases, phase C's residuals
    float cm[kGroup], cl[kGroup], red[kWarps];
    int flag;
};

__device__ __forceinline__ float bf16_lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi_f(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float2 rotate_pair(float x1, float x2, float c, float s) {
    return make_float2(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)), __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier on one word that is never reset: every CTA adds 1 except CTA 0, which adds 2^31 - (G - 1), so
// the word gains exactly 2^31 per barrier and its top bit flips when the last CTA arrives; a CTA waits for the flip
// relative to the value its own arrival returned. Split in two so that a CTA can issue copies between its arrival and
// its wait. Thread 0 arrives and waits (warp 0 issues no asynchronous copies, so its fences wait for nothing else).
// Bounded: after tc::kSpinLimit polls the CTA records `code` and goes on (the host then re-zeroes the word).
__device__ __forceinline__ unsigned grid_arrive(unsigned* word) {
    __syncthreads();
    unsigned old = 0;
    if (threadIdx.x == 0) {
        const unsigned add = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1u) : 1u;
        __threadfence();
        old = atomicAdd(word, add);
    }
    return old;
}
__device__ bool grid_wait(unsigned* word, unsigned old, int* err, int code, int* flag) {
    if (threadIdx.x == 0) {
        bool ok = false;
        for (uint32_t i = 0; i < tc::kSpinLimit; ++i) {
            if (((old ^ ld_acquire(word)) & 0x80000000u) != 0) {
                ok = true;
                break;
            }
            __nanosleep(32);
        }
        if (!ok) atomicCAS(err, 0, code);
        __threadfence();
        *flag = ok ? 1 : 0;
    }
    __syncthreads();
    return *flag != 0;
}

// Dot products of the CTA's nr rows (K bf16 values each, row r at ring + r * 2K, landing on bar[r]) with xs; warp w
// takes rows w, w + 8, ...; row r -> out(r, value). Lane l owns the 16-byte chunks l, l + 32, ... of every row, so it
// holds x's values for them in registers (NCH chunks, K <= 256 NCH) and reads only weights from shared memory.
template <int NCH, class F>
__device__ __forceinline__ void rows_dot(Smem& sh, uint64_t* bar, int nr, int K, int* err, int code, F&& out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, K8 = K >> 3;
    const uint32_t rb = uint32_t(K) * 2u;
    float2 xv[NCH][4];
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = lane + 32 * i;
        const float4 xa = c < K8 ? *reinterpret_cast<const float4*>(sh.xs + 8 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 xb = c < K8 ? *reinterpret_cast<const float4*>(sh.xs + 8 * c + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
        xv[i][0] = make_float2(xa.x, xa.y);
        xv[i][1] = make_float2(xa.z, xa.w);
        xv[i][2] = make_float2(xb.x, xb.y);
        xv[i][3] = make_float2(xb.z, xb.w);
    }
    bool alive = true;
    for (int r = warp; r < nr; r += kWarps) {
        const bool ok = alive && __all_sync(kFull, tc::mbar_wait(&bar[r], 0u, err, code));
        alive = ok;
        float v = __int_as_float(0x7fc00000);
        if (ok) {
            const uint4* wr = reinterpret_cast<const uint4*>(sh.ring + size_t(r) * rb);
            float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < NCH; ++i) {
                const int c = lane + 32 * i;
                if (c < K8) {
                    const uint4 w = wr[c];
                    acc0 = ffma2(make_float2(bf16_lo_f(w.x), bf16_hi_f(w.x)), xv[i][0], acc0);
                    acc1 = ffma2(make_float2(bf16_lo_f(w.y), bf16_hi_f(w.y)), xv[i][1], acc1);
                    acc0 = ffma2(make_float2(bf16_lo_f(w.z), bf16_hi_f(w.z)), xv[i][2], acc0);
                    acc1 = ffma2(make_float2(bf16_lo_f(w.w), bf16_hi_f(w.w)), xv[i][3], acc1);
                }
            }
            v = warp_sum((acc0.x + acc0.y) + (acc1.x + acc1.y));
        }
        if (lane == 0) out(r, v);
    }
}

// All nr rows of W starting at row0 into the ring, one bulk copy per row completing on bar[r] (the last warp's lanes).
__device__ __forceinline__ void issue_rows(Smem& sh, uint64_t* bar, const __nv_bfloat16* W, int row0, int nr, int K) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rb = uint32_t(K) * 2u;
    if (warp == kWarps - 1)
        for (int r = lane; r < nr; r += 32) {
            tc::mbar_arrive_expect_tx(&bar[r], rb);
            tc::bulk_g2s(sh.ring + size_t(r) * rb, W + size_t(row0 + r) * K, rb, &bar[r]);
        }
}

__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {   // 16-byte aligned, pieces of 64 KB
    const uint8_t* b = static_cast<const uint8_t*>(p);
    for (size_t o = 0; o < bytes; o += 65536) {
        const uint32_t n = uint32_t(bytes - o < 65536 ? bytes - o : size_t(65536));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b + o), "r"(n) : "memory");
    }
}

struct Partials {
    float* base;
    __device__ __forceinline__ size_t idx(int h, int s) const { return (size_t(h) * kMaxSplits + s) * kGroup; }
    __device__ __forceinline__ float* m() const { return base; }
    __device__ __forceinline__ float* l() const { return base + kKvHeads * kMaxSplits * kGroup; }
    __device__ __forceinline__ float* acc() const { return base + 2 * kKvHeads * kMaxSplits * kGroup; }
};

__global__ void __launch_bounds__(kThreads, 1) attn_block_kernel(const __grid_constant__ Args a) {
    extern __shared__ uint8_t ab_smem_raw[];
    Smem& sh = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(ab_smem_raw) + 127) & ~uintptr_t(127));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, sub = lane & 7;
    const int c = blockIdx.x, H = a.H;
    const int rA0 = c * a.RA, nA = max(0, min(a.RA, kQkv - rA0));
    const int rC0 = c * a.RC, nC = max(0, min(a.RC, H - rC0));
    // ---- before the dependency wait: barriers, the QKV rows, the RMSNorm weight, L2 prefetches
    if (tid == 0) {
        for (int i = 0; i < nA; ++i) tc::mbar_init(&sh.barA[i], 1);
        for (int i = 0; i < nC; ++i) tc::mbar_init(&sh.barC[i], 1);
        tc::fence_barrier_init();
    }
    if (tid < kGroup) {
        sh.cm[tid] = -INFINITY;
        sh.cl[tid] = 0.f;
    }
    __syncthreads();
    issue_rows(sh, sh.barA, a.wqkv, rA0, nA, H);
    for (int i = tid * 4; i < H; i += kThreads * 4)                  // g first; x * g after the wait
        *reinterpret_cast<float4*>(sh.xs + i) = __ldg(reinterpret_cast<const float4*>(a.ln + i));
    if (tid < nA) sh.bA[tid] = __ldg(a.bqkv + rA0 + tid);
    if (tid >= 64 && tid - 64 < nC) sh.bC[tid - 64] = __ldg(a.bo + rC0 + tid - 64);
    const bool has_item = c < kKvHeads * a.nsplit;
    const int h = has_item ? c / a.nsplit : 0, sp = has_item ? c % a.nsplit : 0;
    // The device position and the cache of older positions were written by kernels that completed before this one
    // was launched (the position advances between steps; every kernel of a step waits for its predecessor).
    const int pos = *a.d_pos;
    const int window = a.window;
    const int n = window > 0 ? min(pos + 1, window) : pos + 1, first = pos + 1 - n;
    const int L = (n + a.nsplit - 1) / a.nsplit, k0 = min(n, sp * L), k1 = has_item ? min(n, k0 + L) : k0;
    const bool holds_new = k0 <= n - 1 && n - 1 < k1;
    if (warp == 1 && lane == 0) {
        if (window == 0 && k1 > k0) {
            // the range's cache rows (all 8 heads, 1 KB per position), an eighth per head's CTA, keys and values
            const size_t lo = size_t(first + k0) * kKVD * 2, hi = size_t(first + k1) * kKVD * 2;
            const size_t piece = ((hi - lo) / kKvHeads + 15) / 16 * 16, b0 = lo + piece * h;
            const size_t b1 = b0 + piece < hi ? b0 + piece : hi;
            if (b1 > b0) {
                prefetch_l2(reinterpret_cast<const uint8_t*>(a.kc) + b0, b1 - b0);
                prefetch_l2(reinterpret_cast<const uint8_t*>(a.vc) + b0, b1 - b0);
            }
        }
    }
    const float cs = __ldg(a.cos_t + size_t(pos) * kPairs + lane), sn = __ldg(a.sin_t + size_t(pos) * kPairs + lane);
    const float sink = has_item ? __ldg(a.sinks + h * kGroup + warp) : 0.f;
    uint8_t* ks = sh.ring;                            // phase B: keys and values of a pass in the ring
    uint8_t* vs = sh.ring + kCap * 128;
    auto stage = [&](int c0, int len) {
        const uint8_t* kcb = reinterpret_cast<const uint8_t*>(a.kc);
        const uint8_t* vcb = reinterpret_cast<const uint8_t*>(a.vc);
        for (int i = tid; i < len * 8; i += kThreads) {
            const int kk = i >> 3, part16 = i & 7;
            if (c0 + kk == n - 1) continue;
            const int p = first + c0 + kk;
            const size_t slot = window > 0 ? size_t(p % window) : size_t(p);
            const size_t off = (slot * kKvHeads + h) * kHeadDim * 2 + part16 * 16;
            cp_async16(ks + kk * 128 + part16 * 16, kcb + off);
            cp_async16(vs + kk * 128 + part16 * 16, vcb + off);
        }
    };
    pdl_launch_dependents();
    pdl_wait();                                      // x comes from the previous kernel

    // ---- phase A: qkv rows of this CTA = r * (Wqkv (x * g)) + bqkv, r the RMSNorm scale
    float rn;
    {
        if (tid >= 128 && tid - 128 < nC) sh.xr[tid - 128] = a.x[rC0 + tid - 128];
        float ss = 0.f;
        for (int i = tid * 4; i < H; i += kThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(a.x + i);
            float4& g = *reinterpret_cast<float4*>(sh.xs + i);
            g = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
            ss = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, ss))));
        }
        ss = warp_sum(ss);
        if (lane == 0) sh.red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += sh.red[w];
        rn = rms_scale(tot, H, a.eps);
        rows_dot<kChA>(sh, sh.barA, nA, H, a.err, 41, [&](int r, float v) { a.qkv[rA0 + r] = v * rn + sh.bA[r]; });
    }
    // the QKV rows are consumed (the arrival's barrier): the ring is free for the keys and values of the attention
    // or, in a CTA without keys, for its O rows at once; the others ask L2 for their O rows, which the attention's
    // end brings into the ring
    const bool staged = has_item && k1 > k0;
    const unsigned arrivedA = grid_arrive(a.gbar);
    if (staged) {
        stage(k0, min(kCap, k1 - k0));
        if (warp == 1 && lane == 0 && nC > 0) prefetch_l2(a.wo + size_t(rC0) * kQD, size_t(nC) * kQD * 2);
    } else {
        if (warp == kWarps - 1) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_rows(sh, sh.barC, a.wo, rC0, nC, kQD);
    }
    const bool okA = grid_wait(a.gbar, arrivedA, a.err, 42, &sh.flag);

    // ---- phase B: attention of key/value head h over key range [k0, k1)
    if (has_item) {
        float qr[kGroup][8];
        {
                const float* base = a.qkv + (h * kGroup + warp) * kHeadDim;
            const float2 r = rotate_pair(__ldcg(base + lane), __ldcg(base + lane + kPairs), cs, sn);
            sh.ps[warp][lane] = r.x;
            sh.ps[warp][lane + kPairs] = r.y;
            if (holds_new && warp == 0) {
                const float* kb = a.qkv + kQD + h * kHeadDim;
                const float2 rk = rotate_pair(__ldcg(kb + lane), __ldcg(kb + lane + kPairs), cs, sn);
                sh.newkv[0][lane] = __float2half_rn(rk.x);
                sh.newkv[0][lane + kPairs] = __float2half_rn(rk.y);
            } else if (holds_new && warp == 1) {
                const float* vb = a.qkv + kQD + kKVD + h * kHeadDim;
                sh.newkv[1][lane] = __float2half_rn(__ldcg(vb + lane));
                sh.newkv[1][lane + kPairs] = __float2half_rn(__ldcg(vb + lane + kPairs));
            }
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < kGroup; ++g)
#pragma unroll
            for (int e = 0; e < 8; ++e) qr[g][e] = sh.ps[g][sub * 8 + e];
        if (holds_new && tid < 16) {                 // the new position's key and value into the cache
            const size_t slot = window > 0 ? size_t(pos % window) : size_t(pos);
            const size_t off = (slot * kKvHeads + h) * kHeadDim * 2 + (tid & 7) * 16;
            uint8_t* dst = reinterpret_cast<uint8_t*>(tid < 8 ? a.kc : a.vc) + off;
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(
                reinterpret_cast<const uint8_t*>(sh.newkv[tid >> 3]) + (tid & 7) * 16);
        }
        const int qh = warp;
        float2 acc = make_float2(0.f, 0.f);
        for (int c0 = k0; c0 < k1; c0 += kCap) {
            const int len = min(kCap, k1 - c0);
            if (c0 != k0) stage(c0, len);
            cp_async_wait_all();
            __syncthreads();                         // every copy landed; qr read before ps is reused
            if (c0 <= n - 1 && n - 1 < c0 + len && tid < 16)
                *reinterpret_cast<uint4*>((tid < 8 ? ks : vs) + (n - 1 - c0) * 128 + (tid & 7) * 16) =
                    *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(sh.newkv[tid >> 3]) + (tid & 7) * 16);
            __syncthreads();
            // scores: an 8-lane group per key (each lane 8 dims of the 8 heads), 4 keys per warp pass
            for (int kb = warp * 4; kb < len; kb += kWarps * 4) {
                const int kk = kb + (lane >> 3);
                float d[kGroup];
                {
                    const uint4 u = kk < len ? *reinterpret_cast<const uint4*>(ks + kk * 128 + sub * 16)
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
                if (kk < len) sh.ps[sub][kk] = d[0] * 0.125f;      // scale 1 / sqrt(64)
            }
            __syncthreads();
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
                const float al = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                __syncwarp();
                if (lane == 0) {
                    sh.cl[qh] = sh.cl[qh] * al + ssum;
                    sh.cm[qh] = m_new;
                }
                float2 acc2 = make_float2(0.f, 0.f);
                acc.x *= al;
                acc.y *= al;
                const uint8_t* vrow = vs + lane * 4;
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
            __syncthreads();                         // the pass's buffers are refilled next
        }
        if (staged) {   // the staged keys and values are no longer read (the loop ended on a barrier): O rows in
            if (warp == kWarps - 1) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_rows(sh, sh.barC, a.wo, rC0, nC, kQD);
        }
        const Partials P{a.part};
        {
            const size_t b = P.idx(h, sp) + qh;
            if (lane == 0) {
                P.m()[b] = sh.cm[qh];
                P.l()[b] = sh.cl[qh];
            }
            *reinterpret_cast<float2*>(P.acc() + b * kHeadDim + 2 * lane) = acc;
        }
        __syncthreads();
        if (tid == 0) {                              // the CTA's partials are ordered before the count (cumulative)
            __threadfence();
            sh.flag = atomicAdd(a.counters + h, 1u) == unsigned(a.nsplit - 1);
            __threadfence();
        }
        __syncthreads();
        if (sh.flag) {                               // the last range of head h merges the ranges with the sink
            const int head = h * kGroup + qh;
            float M = sink;
            for (int s2 = 0; s2 < a.nsplit; ++s2) M = fmaxf(M, __ldcg(P.m() + P.idx(h, s2) + qh));
            float l = expf(sink - M);
            float2 o = make_float2(0.f, 0.f);
            for (int s2 = 0; s2 < a.nsplit; ++s2) {
                const size_t b = P.idx(h, s2) + qh;
                const float m = __ldcg(P.m() + b);
                if (m == -INFINITY) continue;        // a range with no keys
                const float al = expf(m - M);
                l = fmaf(__ldcg(P.l() + b), al, l);
                const float2 v = __ldcg(reinterpret_cast<const float2*>(P.acc() + b * kHeadDim + 2 * lane));
                o.x = fmaf(v.x, al, o.x);
                o.y = fmaf(v.y, al, o.y);
            }
            const float inv = 1.f / l;
            *reinterpret_cast<float2*>(a.attn + size_t(head) * kHeadDim + 2 * lane) = make_float2(o.x * inv, o.y * inv);
            if (tid == 0) a.counters[h] = 0;
        }
    }
    const bool okB = grid_wait(a.gbar, grid_arrive(a.gbar), a.err, 43, &sh.flag);

    // ---- phase C: x rows of this CTA = Wo attn + bo + x
    if (nC > 0) {
        for (int i = tid * 4; i < kQD; i += kThreads * 4)
            *reinterpret_cast<float4*>(sh.xs + i) = __ldcg(reinterpret_cast<const float4*>(a.attn + i));
        __syncthreads();
        const bool ok = okA && okB;
        rows_dot<kChC>(sh, sh.barC, nC, kQD, a.err, 44, [&](int r, float v) {
            const int row = rC0 + r;
            a.x[row] = ok ? v + sh.bC[r] + sh.xr[r] : __int_as_float(0x7fc00000);
        });
    }
}

}  // namespace ab

std::atomic<int> g_attn_impl{0};

size_t attn_block_workspace_bytes() {
    // qkv [5120] + attn [4096] floats, the partials, 8 counters and the barrier word (own 256-byte lines)
    return size_t(ab::kQkv + ab::kQD) * 4 + size_t(ab::kKvHeads) * ab::kMaxSplits * ab::kGroup * (2 + ab::kHeadDim) * 4 +
           512;
}

bool launch_attn_block(float* x, const float* ln, float eps, const void* wqkv, const float* bqkv, const void* wo,
                       const float* bo, const float* cos_t, const float* sin_t, void* k_cache, void* v_cache,
                       const float* sinks, const int* d_pos, int window, int H, void* work, int* err, cudaStream_t s,
                       bool pdl) {
    require(H >= 8 && H % 8 == 0, "attn block: H must be a positive multiple of 8");
    if (H > ab::kMaxH) return false;
    require((reinterpret_cast<uintptr_t>(wqkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(wo) & 15) == 0,
            "attn block: weights must be 16-byte aligned");
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    require(dev >= 0 && dev < 64, "attn block: device ordinal out of range");
    const int G = num_sms();
    ab::Args a{};
    a.x = x;
    a.ln = ln;
    a.eps = eps;
    a.wqkv = static_cast<const __nv_bfloat16*>(wqkv);
    a.bqkv = bqkv;
    a.wo = static_cast<const __nv_bfloat16*>(wo);
    a.bo = bo;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.kc = static_cast<__half*>(k_cache);
    a.vc = static_cast<__half*>(v_cache);
    a.sinks = sinks;
    a.d_pos = d_pos;
    a.window = window;
    a.nsplit = std::min(window > 0 ? ab::kWindowSplits : ab::kFullSplits, G / ab::kKvHeads);
    a.H = H;
    a.RA = (ab::kQkv + G - 1) / G;
    a.RC = (H + G - 1) / G;
    // every row of a phase in the ring at once; the staged keys and values of a pass fit as well
    if (a.RA > ab::kMaxRowsA || a.RC > ab::kMaxRowsC || size_t(a.RA) * H * 2 > size_t(ab::kRingBytes) ||
        size_t(a.RC) * ab::kQD * 2 > size_t(ab::kRingBytes) || 2 * ab::kCap * 128 > ab::kRingBytes)
        return false;
    float* w = static_cast<float*>(work);
    a.qkv = w;
    a.attn = w + ab::kQkv;
    a.part = w + ab::kQkv + ab::kQD;
    unsigned* words = reinterpret_cast<unsigned*>(a.part + size_t(ab::kKvHeads) * ab::kMaxSplits * ab::kGroup *
                                                                (2 + ab::kHeadDim));
    a.counters = words;
    a.gbar = words + 64;
    a.err = err;

    const size_t smem = sizeof(ab::Smem) + 128;      // + the alignment of the base
    static std::mutex mu;
    static bool smem_set[64] = {};
    static std::atomic<int> pdl_ok[64] = {};         // 0 unknown, 1 accepted, -1 refused
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!smem_set[dev]) {
            GPT_CHECK(cudaFuncSetAttribute(ab::attn_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            smem_set[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(ab::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_ok[dev].load() >= 0 ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, ab::attn_block_kernel, a);
    if (e != cudaSuccess && cfg.numAttrs == 2 && pdl_ok[dev].load() == 0) {
        (void)cudaGetLastError();
        pdl_ok[dev].store(-1);
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, ab::attn_block_kernel, a);
    } else if (e == cudaSuccess && cfg.numAttrs == 2) {
        pdl_ok[dev].store(1);
    }
    GPT_CHECK(e);
    check_launch("attention block");
    return true;
}

}  // namespace gpt
