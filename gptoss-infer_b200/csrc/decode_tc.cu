// Tensor-core decode MoE for one token: one persistent, cooperatively launched kernel per MoE layer.
//
// Operands. A = expert weights straight from the checkpoint layout (TMA boxes of 128 rows x 128 bytes of K, 128-byte
// swizzle); their E8M0 scales repacked into 512-byte tcgen05 chunks. B = the activation vector split into R = 16
// e2m1 residual terms, each with its own E8M0 scale per 32 elements, so x equals the sum of the terms to about
// 2^-30 of each block's maximum: the MMA's N = 16 columns hold the terms, the tensor core performs the MXFP4
// dequantization (tcgen05.mma kind::mxf4 block32) and the epilogue adds the 16 columns.
//
// Phases of every CTA (all 148 resident, one per SM):
//   0. RMSNorm of x (every CTA, into shared memory) and the router split over the grid: each CTA computes the
//      router's partial dot products over its slice of K (fp64, exact products) and publishes them; after a
//      counting barrier every CTA adds all partial sums in the same fixed order (so all CTAs pick the same experts),
//      takes the top k (ties to the lower id) and the softmax over the k.
//   1. Gate/up stream-K GEMV; the CTA finishing a 128-row tile applies bias, the clamped SwiGLU (rows 2j glu, 2j+1
//      linear) and the slot's gate weight, and writes the result as down's B terms (global memory).
//   2. Down stream-K GEMV over K' = k * I: the k experts' rows form one long GEMV because B carries the gate
//      weights; the CTA finishing a tile adds sum_slot w b2 and the residual.
// Roles: warp 0 streams the weights (TMA, one 16 KB box per stage, gate/up and down through one ring, so down's
// weights arrive while the grid finishes gate/up); warp 1 issues the MMAs (every scale factor is copied into TMEM
// once, up front, and one commit releases two ring slots: a tcgen05.commit costs about ten MMAs to issue); warps
// 2-5 split h into x's terms in shared memory and load the weight scale chunks with asynchronous 16-byte copies,
// run the tile epilogues, and after the grid barrier (all gate/up epilogues done) load down's B terms. Every wait is bounded:
// the launch is cooperative, so all CTAs are resident and every barrier completes; a timeout records an error
// instead of hanging. Split tiles are reduced by their last contributor (deterministic order), never by spinning.
// The per-CTA stage lists are computed on the host once per shape (stream-K partition, segment boundaries and
// which CTAs share each tile) and read by each CTA at start.
#include <algorithm>
#include <map>
#include <mutex>
#include <stdexcept>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "streamk.cuh"
#include "tc.cuh"
#include "terms.cuh"
#include "tma.h"

namespace gpt {
namespace fz {

using sk::Part;
using sk::Stage;
static_assert(sizeof(Stage) % 4 == 0, "stage entries are copied as 32-bit words");
constexpr int R = kDecodeTerms;
constexpr int kThreads = 192;                 // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kA = 16384, kB = R * 128;       // one weight stage (128 rows x 128 bytes of K), one B stage
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSF = 2 * R;            // accumulators in columns [0, 2R), scale factors from 2R on
constexpr int kTraceSlots = 160;
constexpr int kMaxK = 8;
constexpr int kMaxX4 = 8;                     // x is held as kMaxX4 float4 per thread: H <= 4 * kThreads * kMaxX4

struct Layout {
    int NS, cap;                              // weight ring depth (even), stage-list capacity
    int ringA, regBgu, regSFBgu, regSFA, regBdn, regSFBdn, hs, bars, misc, bytes;
};

struct Job {
    int k, H, I, E;
    const __nv_bfloat16* router_w;            // null: ids_in / w_in give the experts
    const float* router_b;
    const float* norm_w;                      // null: x is already normalized
    float eps;
    const float* x;
    const int* ids_in;
    const float* w_in;
    int* ids_out;                             // written by the publishing CTA when not null
    float* w_out;
    const uint8_t* sfa_gu;                    // [mat][RT][KT][512]
    const uint8_t* sfa_dn;
    int sfa_by_slot;                          // mat = slot (1) or expert id (0)
    const float* gu_bias;                     // [E][2I]
    const float* dn_bias;                     // [E][H]
    float alpha, limit;
    Part gu, dn;
    const Stage* stab;                        // host-built stage lists of all CTAs
    const int* shdr;                          // [grid][4]: first entry, entries, gate/up entries
    int sf_upfront;                           // 1: every scale chunk of the CTA fits in TMEM at once
    uint8_t* aq_img;                          // down's B terms [k][SPS_dn][R*128]
    uint8_t* aq_sf;                           // down's B scales [k][KT_dn][512]
    float* x_resid;
    unsigned* gbar;                           // [3]: gate/up done, exits, router partials published
    double* partials;                         // [grid][32] router partial sums
    int* err;
    long long* trace;                         // optional [grid][kTraceSlots] clock64 stamps
    Layout L;
};

// Trace slots per CTA: 0 start, 84 h in shared memory, 85 router partials published, 86 all partials published, 87
// logits, 88 ids known, 1 phase 0 done, 89 producer start, 2+i producer issues stage i, 80 small operands in shared memory, 90 scale
// factors in TMEM, 34+i MMA warp sees stage i landed, 96+i its MMAs issued, 66+g epilogue finished segment g, 81 grid
// barrier passed, 83 down's B terms in shared memory, 82 end.
__device__ __forceinline__ void stamp(const Job& j, int slot) {
    if (j.trace) j.trace[size_t(blockIdx.x) * kTraceSlots + slot] = clock64();
}

__device__ __forceinline__ bool epi_all(bool p) {            // AND over the 128 epilogue threads (barrier 1)
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r)
                 : "r"(uint32_t(p))
                 : "memory");
    return r != 0;
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ double bf16lo(uint32_t w) { return double(__uint_as_float(w << 16)); }
__device__ __forceinline__ double bf16hi(uint32_t w) { return double(__uint_as_float(w & 0xffff0000u)); }

__global__ void __launch_bounds__(kThreads, 1) moe_fused_kernel(const __grid_constant__ CUtensorMap tm_gu,
                                                                const __grid_constant__ CUtensorMap tm_dn,
                                                                const __grid_constant__ Job j) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NS = j.L.NS, cap = j.L.cap, NP = NS / 2;
    uint8_t* ringA = smem + j.L.ringA;
    uint8_t* regBgu = smem + j.L.regBgu;
    uint8_t* regSFBgu = smem + j.L.regSFBgu;
    uint8_t* regSFA = smem + j.L.regSFA;
    uint8_t* regBdn = smem + j.L.regBdn;
    uint8_t* regSFBdn = smem + j.L.regSFBdn;
    uint64_t* fullA = reinterpret_cast<uint64_t*>(smem + j.L.bars);   // [NS] weight stage landed
    uint64_t* emptyP = fullA + NS;            // [NS/2] both slots of a pair consumed by the MMAs
    uint64_t* fullS = emptyP + NP;            // [0] gate/up's small operands, [1] down's B terms and scales
    uint64_t* accF = fullS + 2;               // [2] accumulator buffer complete
    uint64_t* accE = accF + 2;                // [2] accumulator buffer read out
    float* hs = reinterpret_cast<float*>(smem + j.L.hs);     // h = RMSNorm(x) [H]
    uint32_t* holder = reinterpret_cast<uint32_t*>(smem + j.L.misc);
    int* cnts = reinterpret_cast<int*>(holder + 2);          // [2] partials barrier result, [3] grid barrier result
    double* red = reinterpret_cast<double*>(cnts + 6);       // [6][32] router sums
    int* ids_s = reinterpret_cast<int*>(red + 7 * 32);       // [8]
    float* w_s = reinterpret_cast<float*>(ids_s + kMaxK);    // [8]
    float* aval = w_s + kMaxK;                               // [64]
    Stage* stages = reinterpret_cast<Stage*>(aval + 64);     // [cap]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, nc = gridDim.x;
    if (tid == 0) stamp(j, 0);
    // this CTA's slice of the router weights: thread (expert = lane, o = warp) takes chunks cs0 + o, cs0 + o + 6, ...
    // of 8 weights; the first is loaded before anything else (it does not depend on x)
    const int H8 = j.H >> 3;
    const int cs0 = int((long long)c * H8 / nc), cs1 = int((long long)(c + 1) * H8 / nc);
    uint4 w_first = make_uint4(0u, 0u, 0u, 0u);
    if (j.router_w && lane < j.E && cs0 + warp < cs1)
        w_first = __ldg(reinterpret_cast<const uint4*>(j.router_w) + size_t(lane) * H8 + cs0 + warp);
    const float bias = j.router_w && warp == 0 && lane < j.E ? __ldg(j.router_b + lane) : 0.f;
    // x and the norm weights, kept in registers: thread t holds float4 chunks t, t + kThreads, ...
    float4 xv[kMaxX4], gv[kMaxX4];
#pragma unroll
    for (int r = 0; r < kMaxX4; ++r) {
        const int i = (tid + r * kThreads) * 4;
        xv[r] = i < j.H ? *reinterpret_cast<const float4*>(j.x + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        gv[r] = i < j.H && j.norm_w ? __ldg(reinterpret_cast<const float4*>(j.norm_w + i))
                                    : make_float4(1.f, 1.f, 1.f, 1.f);
    }
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) tc::mbar_init(&fullA[i], 1);
        for (int i = 0; i < NP; ++i) tc::mbar_init(&emptyP[i], 1);
        tc::mbar_init(&fullS[0], 128);                       // one arrival per epilogue thread after its copies
        tc::mbar_init(&fullS[1], 128);
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&accF[i], 1);
            tc::mbar_init(&accE[i], 128);
        }
        tc::fence_barrier_init();
    }
    const int s_first = __ldg(j.shdr + 4 * c), s_n = __ldg(j.shdr + 4 * c + 1), s_ngu = __ldg(j.shdr + 4 * c + 2);
    const int nst = min(s_n, cap), ngu = min(s_ngu, nst);
    {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(j.stab + s_first);
        uint32_t* dst = reinterpret_cast<uint32_t*>(stages);
        const int nw = nst * int(sizeof(Stage) / 4);
        for (int i = tid; i < nw; i += kThreads) dst[i] = __ldg(src + i);
    }
    if (tid == 0 && s_n > cap) atomicCAS(j.err, 0, 100);    // host sized the stage list too small
    if (tid == 0) stamp(j, 123);
    if (warp == 1) {
        tc::tmem_alloc(holder, kTmemCols);
        tc::tmem_relinquish();
    }

    // ---------------------------------------------------------------- phase 0: RMSNorm, router, expert ids
    {
        const int H = j.H;
        float ss = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxX4; ++r)
            ss = fmaf(xv[r].x, xv[r].x, fmaf(xv[r].y, xv[r].y, fmaf(xv[r].z, xv[r].z, fmaf(xv[r].w, xv[r].w, ss))));
        ss = warp_sum(ss);
        if (lane == 0) aval[warp] = ss;
        if (tid == 0) stamp(j, 124);
        __syncthreads();
        if (tid == 0) stamp(j, 125);
        float rn = 1.f;
        if (j.norm_w) {
            float tot = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) tot += aval[w];
            rn = 1.0f / sqrtf(tot / float(H) + j.eps);
        }
#pragma unroll
        for (int r = 0; r < kMaxX4; ++r) {
            const int i = (tid + r * kThreads) * 4;
            if (i < H) {
                float4 v = xv[r];
                if (j.norm_w) {
                    v.x = v.x * rn * gv[r].x; v.y = v.y * rn * gv[r].y; v.z = v.z * rn * gv[r].z; v.w = v.w * rn * gv[r].w;
                }
                *reinterpret_cast<float4*>(hs + i) = v;
            }
        }
        __syncthreads();
        if (tid == 0) stamp(j, 84);
        if (j.router_w) {
            double acc = 0.0;
            for (int cc = cs0 + warp; cc < cs1; cc += kThreads / 32) {
                if (lane < j.E) {
                    const uint4 u = cc == cs0 + warp
                                        ? w_first
                                        : __ldg(reinterpret_cast<const uint4*>(j.router_w) + size_t(lane) * H8 + cc);
                    const float4 h0 = *reinterpret_cast<const float4*>(hs + cc * 8);
                    const float4 h1 = *reinterpret_cast<const float4*>(hs + cc * 8 + 4);
                    acc = fma(bf16lo(u.x), double(h0.x), acc); acc = fma(bf16hi(u.x), double(h0.y), acc);
                    acc = fma(bf16lo(u.y), double(h0.z), acc); acc = fma(bf16hi(u.y), double(h0.w), acc);
                    acc = fma(bf16lo(u.z), double(h1.x), acc); acc = fma(bf16hi(u.z), double(h1.y), acc);
                    acc = fma(bf16lo(u.w), double(h1.z), acc); acc = fma(bf16hi(u.w), double(h1.w), acc);
                }
            }
            red[warp * 32 + lane] = acc;
            __syncthreads();
            if (warp == 0) {
                double t = 0.0;
                for (int w = 0; w < kThreads / 32; ++w) t += red[w * 32 + lane];
                j.partials[size_t(c) * 32 + lane] = t;
                __threadfence();
                __syncwarp();
                if (lane == 0) {
                    atomicAdd(&j.gbar[2], 1u);
                    stamp(j, 85);
                }
                // every CTA's partial sums published (bounded wait; the launch is cooperative)
                bool done = false;
                for (uint32_t i = 0; i < tc::kSpinLimit && !done; ++i) {
                    done = __shfl_sync(kFull, lane == 0 ? ld_acquire(&j.gbar[2]) >= unsigned(nc) : false, 0);
                    if (!done) __nanosleep(20);
                }
                if (lane == 0) {
                    if (!done) atomicCAS(j.err, 0, 10);
                    cnts[2] = done;
                    stamp(j, 86);
                }
            }
            __syncthreads();
            // every CTA adds all partial sums in the same order: thread (w, e) takes CTAs w, w + 6, ... (loads
            // issued eight at a time), then warp 0 adds the six sums
            double t = 0.0;
            if (cnts[2]) {
                for (int c0 = warp; c0 < nc; c0 += 8 * (kThreads / 32)) {
                    double v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int cc = c0 + u * (kThreads / 32);
                        v[u] = cc < nc ? __ldcg(&j.partials[size_t(cc) * 32 + lane]) : 0.0;
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u) t += v[u];
                }
            }
            red[warp * 32 + lane] = t;
            __syncthreads();
            if (tid == 0) stamp(j, 87);
            if (warp == 0) {
                // top k on order-preserving 64-bit keys of the fp64 logits (integer warp reductions; ties to the
                // lower id; NaN, picked experts and lanes >= E get key 0 and never win while a real logit is left)
                double v = 0.0;
                if (lane < j.E) {
                    double tt = 0.0;
                    for (int w = 0; w < kThreads / 32; ++w) tt += red[w * 32 + lane];
                    v = tt + double(bias);
                }
                const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(v));
                unsigned long long key = (bits >> 63) ? ~bits : (bits | (1ull << 63));
                if ((bits & 0x7FFFFFFFFFFFFFFFull) > 0x7FF0000000000000ull || lane >= j.E) key = 0;   // NaN / unused
                if (lane == 0) stamp(j, 120);
                unsigned id = lane < j.E ? unsigned(lane) : 32u + lane;
                float sel = -INFINITY;
                int sel_id = 0;
                for (int q = 0; q < j.k; ++q) {
                    const unsigned hi = unsigned(key >> 32), lo = unsigned(key);
                    const unsigned m1 = __reduce_max_sync(kFull, hi);
                    const unsigned m2 = __reduce_max_sync(kFull, hi == m1 ? lo : 0u);
                    const unsigned win = __reduce_min_sync(kFull, hi == m1 && lo == m2 ? id : 0xFFFFFFFFu);
                    const double wv = __shfl_sync(kFull, v, int(win & 31u));
                    if (lane == q) { sel = float(wv); sel_id = int(win); }
                    if (id == win) { key = 0; id = 32u + lane; }
                }
                if (lane == 0) stamp(j, 121);
                const float top = __shfl_sync(kFull, sel, 0);
                const float pz = lane < j.k ? expf(sel - top) : 0.f;
                const float sum = warp_sum(pz);
                if (lane == 0) stamp(j, 122);
                if (lane < j.k) {
                    ids_s[lane] = sel_id;
                    w_s[lane] = pz / sum;
                    if (j.ids_out && c == 0) { j.ids_out[lane] = sel_id; j.w_out[lane] = pz / sum; }
                }
            }
        } else if (tid < j.k) {
            ids_s[tid] = j.ids_in[tid];
            w_s[tid] = j.w_in[tid];
        }
        if (tid == 0) stamp(j, 88);
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (tid == 0) stamp(j, 1);
    const uint32_t tmem = *holder;
    const bool upfront = j.sf_upfront != 0;
    // TMEM columns of the scale factors. Up front: stage i's weight scales at kColSF + 8i, x's scale chunk kt at
    // sfb_gu0 + 4kt, down stage i's B scales at sfb_dn0 + 8(i - ngu). Otherwise copied per stage to kColSF (A) and
    // kColSF + 8 (B).
    const uint32_t sfb_gu0 = kColSF + 8u * uint32_t(nst), sfb_dn0 = sfb_gu0 + 4u * uint32_t(j.gu.KT);

    auto part_of = [&](const Stage& st) -> const Part& { return st.mode == sk::kGateUp ? j.gu : j.dn; };

    if (warp == 0) {
        // ---------------------------------------------------------------- producer (converged warp, elected lane)
        if (tc::elect_one()) {
            stamp(j, 89);
            tc::prefetch_tmap(&tm_gu);
            tc::prefetch_tmap(&tm_dn);
        }
        __syncwarp();
        // Stages 2p and 2p+1 share slot pair p % NP; the MMA warp releases a pair with one commit.
        auto wait_pair = [&](int it) -> bool {
            const int p = (it - NS) >> 1;
            return __all_sync(kFull, tc::mbar_wait(&emptyP[p % NP], uint32_t(p / NP) & 1u, j.err, 1));
        };
        // The tensor map is a compile-time operand of each loop: selecting it at run time made every TMA issue wait
        // for a descriptor fetch.
        bool ok = true;
        for (int it = 0; it < ngu && ok; ++it) {
            if (it >= NS && (it & 1) == 0) ok = wait_pair(it);
            if (ok && tc::elect_one()) {
                if (it < 32) stamp(j, 2 + it);
                const Stage& st = stages[it];
                tc::mbar_arrive_expect_tx(&fullA[it % NS], kA);
                tc::tma_load_3d(ringA + (it % NS) * kA, &tm_gu, (st.ku0 / 4) * 128, (st.tile % j.gu.RT) * 128,
                                ids_s[st.s], &fullA[it % NS]);
            }
            __syncwarp();
        }
        for (int it = ngu; it < nst && ok; ++it) {
            if (it >= NS && (it & 1) == 0) ok = wait_pair(it);
            if (ok && tc::elect_one()) {
                if (it < 32) stamp(j, 2 + it);
                const Stage& st = stages[it];
                tc::mbar_arrive_expect_tx(&fullA[it % NS], kA);
                tc::tma_load_3d(ringA + (it % NS) * kA, &tm_dn, (st.ku0 / 4) * 128, st.tile * 128, ids_s[st.s],
                                &fullA[it % NS]);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (converged warp, one lane)
        // One fixed lane issues every tcgen05 operation, so scale copies and MMAs are ordered. With the scales up
        // front, each stage's scale chunks are copied into their own TMEM columns before the stage's data is waited
        // for (the copies overlap that wait); x's scale chunks are copied the first time a stage needs them.
        const bool leader = tc::elect_one();
        bool ok = nst == 0 || tc::mbar_wait(&fullS[0], 0, j.err, 6);
        ok = __all_sync(kFull, ok);
        unsigned long long x_sf_done = 0;                    // x's scale chunks in TMEM (leader's copy)
        for (int it = 0; it < nst && ok; ++it) {
            const Stage& st = stages[it];
            const int slot = it % NS, ph = (it / NS) & 1;
            const int buf = st.seg & 1;
            const int kt0 = st.ku0 / 2, nkt = sk::nkt_of(st);
            const bool gu = st.mode == sk::kGateUp;
            if (it == ngu) ok = __all_sync(kFull, tc::mbar_wait(&fullS[1], 0, j.err, 9));   // down's B terms
            if (ok && upfront) {
                tc::tc_fence_after();
                if (leader) {
                    for (int q = 0; q < nkt; ++q)
                        tc::tmem_cp_sf(tmem + kColSF + 8 * it + 4 * q,
                                       tc::desc_sf_chunk(tc::smem_u32(regSFA + it * 1024 + q * 512)));
                    if (gu) {
                        for (int q = 0; q < nkt; ++q) {
                            const int kt = kt0 + q;
                            if (!((x_sf_done >> kt) & 1ull)) {
                                tc::tmem_cp_sf(tmem + sfb_gu0 + 4 * kt,
                                               tc::desc_sf_chunk(tc::smem_u32(regSFBgu + kt * 512)));
                                x_sf_done |= 1ull << kt;
                            }
                        }
                    } else {
                        for (int q = 0; q < nkt; ++q)
                            tc::tmem_cp_sf(tmem + sfb_dn0 + 8 * (it - ngu) + 4 * q,
                                           tc::desc_sf_chunk(tc::smem_u32(regSFBdn + (it - ngu) * 1024 + q * 512)));
                    }
                }
                __syncwarp();
            }
            if (st.first && st.seg >= 2) ok = ok && tc::mbar_wait(&accE[buf], ((st.seg >> 1) - 1) & 1, j.err, 2);
            ok = ok && tc::mbar_wait(&fullA[slot], ph, j.err, 3);
            ok = __all_sync(kFull, ok);
            if (!ok) break;
            tc::tc_fence_after();
            if (leader) {
                if (it < 32) stamp(j, 34 + it);
                const uint8_t* bst = gu ? regBgu + (st.ku0 / 4) * kB : regBdn + (it - ngu) * kB;
                uint32_t sfa_c, sfb_c;
                if (upfront) {
                    sfa_c = kColSF + 8u * uint32_t(it);
                    sfb_c = gu ? sfb_gu0 + 4u * uint32_t(kt0) : sfb_dn0 + 8u * uint32_t(it - ngu);
                } else {
                    sfa_c = kColSF;
                    sfb_c = kColSF + 8;
                    const uint8_t* sfb = gu ? regSFBgu + kt0 * 512 : regSFBdn + (it - ngu) * 1024;
                    for (int q = 0; q < nkt; ++q) {
                        tc::tmem_cp_sf(tmem + sfa_c + 4 * q, tc::desc_sf_chunk(tc::smem_u32(regSFA + it * 1024 + q * 512)));
                        tc::tmem_cp_sf(tmem + sfb_c + 4 * q, tc::desc_sf_chunk(tc::smem_u32(sfb + q * 512)));
                    }
                }
                for (int u = 0; u < st.nu; ++u) {
                    const int ku = st.ku0 + u;
                    const uint32_t sf_id = 2u * (ku & 1);
                    const uint32_t q = uint32_t(ku / 2 - kt0);
                    const uint64_t ad = tc::desc_sw128(tc::smem_u32(ringA + slot * kA + u * 32));
                    const uint64_t bd = tc::desc_sw128(tc::smem_u32(bst + u * 32));
                    tc::mma_mxf4(tmem + buf * R, ad, bd, tc::idesc_mxf4(128, R, sf_id, sf_id),
                                 (tmem + sfa_c + 4 * q) | (sf_id << 30), (tmem + sfb_c + 4 * q) | (sf_id << 30),
                                 !(st.first && u == 0));
                }
                if ((it & 1) || it == nst - 1) tc::mma_commit(&emptyP[(it >> 1) % NP]);
                if (st.last) tc::mma_commit(&accF[buf]);
                if (it < 32) stamp(j, 96 + it);
            }
            __syncwarp();
        }
    } else {
        // ---------------------------------------------------------------- epilogue warps 2..5
        const int quad = warp & 3;                  // TMEM lane quadrant this warp may read
        const int row = quad * 32 + lane;           // row within the 128-row tile
        const int et = tid - 64;                    // 0..127

        // Small operands of gate/up: the weight scale chunks of every stage (asynchronous 16-byte copies, in flight
        // while x is quantized) and x's B terms and scales, split from h straight into shared memory (warp w - 2
        // takes 8 blocks per pass, 4 lanes per block).
        {
            const int n3 = nst * 64;
            for (int x = et; x < n3; x += 128) {
                const int i = x >> 6, q16 = x & 63;
                const Stage& st = stages[i];
                if (q16 < sk::nkt_of(st) * 32) {
                    const Part& p = part_of(st);
                    const bool gu = st.mode == sk::kGateUp;
                    const int mat = j.sfa_by_slot ? int(st.s) : ids_s[st.s];
                    const int rt = gu ? st.tile % p.RT : st.tile;
                    const uint8_t* base = gu ? j.sfa_gu : j.sfa_dn;
                    tc::cp_async16(regSFA + i * 1024 + 16 * q16,
                                   base + ((size_t(mat) * p.RT + rt) * p.KT + st.ku0 / 2) * 512 + 16 * q16);
                }
            }
            if (et == 0) stamp(j, 126);
            const int nb = j.H / 32, sub = lane & 3;
            for (int g0 = (warp - 2) * 8; g0 < nb; g0 += 32) {
                const int g = g0 + (lane >> 2);
                const bool active = g < nb;
                const int gg = active ? g : 0;
                const float4 h0 = *reinterpret_cast<const float4*>(hs + gg * 32 + sub * 8);
                const float4 h1 = *reinterpret_cast<const float4*>(hs + gg * 32 + sub * 8 + 4);
                float v8[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                if (!active)
#pragma unroll
                    for (int i = 0; i < 8; ++i) v8[i] = 0.f;
                quantize_block_terms_fixed(v8, regBgu + (gg / 8) * kB, gg % 8, regSFBgu + (gg / 4) * 512, gg % 4,
                                           sub, active);
                if (et == 0 && g0 < 96) stamp(j, 127 + g0 / 32);
            }
            if (et == 0) stamp(j, 130);
            tc::cp_async_wait_all();
            tc::fence_proxy_async_smem();
            tc::mbar_arrive(&fullS[0]);
            if (et == 0) stamp(j, 80);
        }
        // After the CTA's last gate/up epilogue: count it on the grid barrier, wait for all CTAs, then load down's B
        // terms and scales for the down stages.
        auto gate_up_done_then_load_down_b = [&]() {
            __threadfence();                        // this thread's down-B terms and partial sums are published
            epi_sync();
            if (et == 0) {
                __threadfence();
                atomicAdd(&j.gbar[0], 1u);
            }
            if (ngu == nst) return;                 // no down stages here
            if (et == 0) {
                bool done = false;
                for (uint32_t i = 0; i < tc::kSpinLimit && !done; ++i) {
                    done = ld_acquire(&j.gbar[0]) >= unsigned(nc);
                    if (!done) __nanosleep(32);
                }
                if (!done) atomicCAS(j.err, 0, 8);
                cnts[3] = done;
                stamp(j, 81);
            }
            epi_sync();
            if (cnts[3]) {
                const int nd = (nst - ngu) * 192;
                for (int x = et; x < nd; x += 128) {
                    const int i = ngu + x / 192, q = x % 192;
                    const Stage& st = stages[i];
                    if (q < 128) {
                        tc::cp_async16(regBdn + (i - ngu) * kB + 16 * q,
                                       j.aq_img + (size_t(st.s) * j.dn.SPS + st.ku0 / 4) * kB + 16 * q);
                    } else if (q - 128 < sk::nkt_of(st) * 32) {
                        tc::cp_async16(regSFBdn + (i - ngu) * 1024 + 16 * (q - 128),
                                       j.aq_sf + (size_t(st.s) * j.dn.KT + st.ku0 / 2) * 512 + 16 * (q - 128));
                    }
                }
                tc::cp_async_wait_all();
                tc::fence_proxy_async_smem();
            }
            tc::mbar_arrive(&fullS[1]);
            if (et == 0) stamp(j, 83);
        };
        if (ngu == 0) gate_up_done_then_load_down_b();
        bool ok = true;
        for (int it = 0; it < nst; ++it) {
            const Stage& st = stages[it];
            if (!st.last) continue;
            const int buf = st.seg & 1;
            ok = ok && tc::mbar_wait_sleepy(&accF[buf], (st.seg >> 1) & 1, j.err, 5, 64);
            ok = epi_all(ok);                        // uniform over the 4 epilogue warps before any named barrier
            float v = 0.f;
            if (ok) {
                tc::tc_fence_after();
                float t0[8], t1[8];
                tc::tmem_ld_32x32b_x8(tmem + buf * R + (uint32_t(quad * 32) << 16), t0);
                tc::tmem_ld_32x32b_x8(tmem + buf * R + 8 + (uint32_t(quad * 32) << 16), t1);
                tc::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 8; ++i) v += t0[i];
#pragma unroll
                for (int i = 0; i < 8; ++i) v += t1[i];
            }
            tc::tc_fence_before();
            tc::mbar_arrive(&accE[buf]);
            if (et == 0 && st.seg < 14) stamp(j, 66 + st.seg);
            if (ok) {
                const Part& p = part_of(st);
                const int t = st.tile;
                float total = v;
                bool mine = true;                    // this CTA applies the tile's epilogue
                if (st.whole < 0) {                  // more CTAs share the tile than there are partial slots
                    if (et == 0) atomicCAS(j.err, 0, 101);
                    mine = false;
                } else if (!st.whole) {
                    p.partial[(size_t(t) * sk::kMaxContrib + (c - st.cf)) * 128 + row] = v;
                    __threadfence();
                    epi_sync();
                    if (et == 0) {
                        __threadfence();
                        const unsigned old = atomicAdd(&p.cnt[t], unsigned(st.units));
                        const bool last = old + unsigned(st.units) == unsigned(p.UT);
                        if (last) p.cnt[t] = 0;      // every contributor has arrived: reset for the next launch
                        __threadfence();
                        cnts[2] = last;
                    }
                    epi_sync();
                    mine = cnts[2] != 0;
                    if (mine) {
                        // contributors in CTA order; the loads are independent and issue together
                        total = 0.f;
                        const float* pp = p.partial + size_t(t) * sk::kMaxContrib * 128 + row;
                        const unsigned m = st.mask;
                        float pv[sk::kMaxContrib];
#pragma unroll
                        for (int b = 0; b < sk::kMaxContrib; ++b) pv[b] = (m >> b) & 1u ? __ldcg(pp + b * 128) : 0.f;
#pragma unroll
                        for (int b = 0; b < sk::kMaxContrib; ++b)
                            if ((m >> b) & 1u) total += pv[b];
                    }
                }
                if (mine && st.mode == sk::kGateUp) {
                    const int s = t / p.RT, rt = t % p.RT;
                    const int e = ids_s[s];
                    const int grow = rt * 128 + row;
                    const float y = grow < 2 * j.I ? total + j.gu_bias[size_t(e) * 2 * j.I + grow] : 0.f;
                    const float lin = __shfl_down_sync(kFull, y, 1);
                    if ((lane & 1) == 0) {
                        const float gv = fminf(y, j.limit);
                        const float lv = fminf(fmaxf(lin, -j.limit), j.limit);
                        aval[row >> 1] = gv / (1.f + expf(-j.alpha * gv)) * (lv + 1.f) * w_s[s];
                    }
                    epi_sync();
                    if (quad == 0) {                 // one warp: the tile's two 32-element blocks, 4 lanes each
                        const int grp = lane >> 2, sub = lane & 3;
                        const int gb = rt * 2 + (grp & 1);
                        const bool active = grp < 2 && gb * 32 < j.I;
                        float v8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) v8[i] = aval[(grp & 1) * 32 + sub * 8 + i];
                        uint8_t* img = j.aq_img + (size_t(s) * j.dn.SPS + gb / 8) * kB;
                        uint8_t* sf = j.aq_sf + (size_t(s) * j.dn.KT + gb / 4) * 512;
                        quantize_block_terms_fixed(v8, img, gb % 8, sf, gb % 4, sub, active);
                    }
                    epi_sync();
                } else if (mine) {
                    const int grow = t * 128 + row;
                    if (grow < j.H) {
                        float add = total;
                        for (int s = 0; s < j.k; ++s) add += w_s[s] * j.dn_bias[size_t(ids_s[s]) * j.H + grow];
                        j.x_resid[grow] += add;
                    }
                }
            }
            // after the last gate/up segment (also when a wait gave up, so other CTAs are not held up)
            if (st.mode == sk::kGateUp && it == ngu - 1) gate_up_done_then_load_down_b();
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        stamp(j, 82);
        __threadfence();
        if (atomicAdd(&j.gbar[1], 1u) == unsigned(nc - 1)) {   // last CTA out resets the grid barriers
            j.gbar[0] = 0;
            j.gbar[2] = 0;
            j.gbar[1] = 0;
        }
    }
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// Shared-memory plan: NS weight stages, the x image and its scales, per-entry weight-scale chunks (1 KB each),
// per-down-entry B stages and scale chunks, h (fp32; in the down-B region when it fits there: h is consumed before
// down's B terms arrive), barriers, and the small per-CTA state.
Layout make_layout(int NS, int cap, int cap_dn, const Part& gu, int H) {
    Layout L{};
    L.NS = NS;
    L.cap = cap;
    int o = 0;
    L.ringA = o; o += NS * kA;
    L.regBgu = o; o += gu.SPS * kB;
    L.regSFBgu = o; o += (gu.KT * 512 + 1023) & ~1023;
    L.regSFA = o; o += cap * 1024;
    L.regBdn = o; o += cap_dn * kB;
    L.regSFBdn = o; o += cap_dn * 1024;
    if (H * 4 <= o - L.regBdn) {
        L.hs = L.regBdn;
    } else {
        L.hs = o;
        o += (H * 4 + 15) & ~15;
    }
    L.bars = o; o += (NS + NS / 2 + 6) * 8;
    o = (o + 15) & ~15;
    L.misc = o; o += 8 + 24 + 7 * 32 * 8 + 2 * kMaxK * 4 + 64 * 4 + cap * int(sizeof(Stage));
    L.bytes = 1024 + o;
    return L;
}

// Stage lists of every CTA for one shape and grid, built once on the host and kept on the device for the life of
// the process (one table per device and shape).
struct StageTable {
    Stage* st = nullptr;
    int* hdr = nullptr;
    int cap = 1, cap_dn = 1;
    int cols = 0;                             // TMEM columns needed to hold every scale chunk of the busiest CTA
};

const StageTable& stage_table(const Part& g, const Part& d, int nc, int k, int H, int I) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int, int>, StageTable> cache;
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev, k, H, I, nc);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    StageTable T;
    std::vector<Stage> all;
    std::vector<int> hdr(size_t(nc) * 4, 0);
    for (int c = 0; c < nc; ++c) {
        int seg = 0;
        const int ngu = sk::build_stages(g, c, nc, nullptr, 0, 0, 0, &seg);
        const int n = sk::build_stages(d, c, nc, nullptr, ngu, 0, seg, nullptr);
        const size_t n0 = all.size();
        all.resize(n0 + size_t(n));
        Stage* o = all.data() + n0;
        seg = 0;
        sk::build_stages(g, c, nc, o, 0, n, 0, &seg);
        sk::build_stages(d, c, nc, o, ngu, n, seg, nullptr);
        sk::fill_tile_info(g, c, nc, o, 0, ngu);
        sk::fill_tile_info(d, c, nc, o, ngu, n);
        hdr[size_t(c) * 4 + 0] = int(n0);
        hdr[size_t(c) * 4 + 1] = n;
        hdr[size_t(c) * 4 + 2] = ngu;
        T.cap = std::max(T.cap, n);
        T.cap_dn = std::max(T.cap_dn, n - ngu);
        T.cols = std::max(T.cols, int(kColSF) + 8 * n + 4 * g.KT + 8 * (n - ngu));
    }
    if (all.empty()) all.resize(1);
    GPT_CHECK(cudaMalloc(&T.st, all.size() * sizeof(Stage)));
    GPT_CHECK(cudaMalloc(&T.hdr, hdr.size() * sizeof(int)));
    GPT_CHECK(cudaMemcpy(T.st, all.data(), all.size() * sizeof(Stage), cudaMemcpyHostToDevice));
    GPT_CHECK(cudaMemcpy(T.hdr, hdr.data(), hdr.size() * sizeof(int), cudaMemcpyHostToDevice));
    return cache.emplace(key, T).first->second;
}

}  // namespace fz

// ---------------------------------------------------------------------------------------------------- host API
DecodeTcLayout decode_tc_layout(int k, int H, int I) {
    DecodeTcLayout L{};
    const int R = kDecodeTerms;
    auto al = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    const int UKd = (I + 63) / 64;
    L.SPS_dn = (UKd + 3) / 4;
    L.KT_dn = (I + 127) / 128;
    L.SPS_gu = ((H + 63) / 64 + 3) / 4;
    L.KT_gu = (H + 127) / 128;
    L.RT_gu = (2 * I + 127) / 128;
    L.RT_dn = (H + 127) / 128;
    size_t o = 0;
    L.off_partials = o; o += al(size_t(256) * 32 * 8);
    L.off_aq_img = o; o += al(size_t(k) * L.SPS_dn * R * 128);
    L.off_aq_sf = o; o += al(size_t(k) * L.KT_dn * 512);
    L.off_part_gu = o; o += al(size_t(k) * L.RT_gu * sk::kMaxContrib * 128 * 4);
    L.off_part_dn = o; o += al(size_t(L.RT_dn) * sk::kMaxContrib * 128 * 4);
    L.off_cnt_gu = o; o += al(size_t(k) * L.RT_gu * 4);
    L.off_cnt_dn = o; o += al(size_t(L.RT_dn) * 4);
    L.off_err = o; o += 1024;                                // error word, then the grid barrier at +256
    L.off_sfa_gu = o; o += al(sf_repacked_bytes(k, 2 * I, H / 32));
    L.off_sfa_dn = o; o += al(sf_repacked_bytes(k, H, I / 32));
    L.off_misc = o; o += al(size_t(H) * 4 + 256);
    L.bytes = o;
    L.zero_bytes_from = L.off_cnt_gu;                        // counters, error word and grid barrier start at zero
    L.zero_bytes_to = L.off_err + 1024;
    return L;
}

namespace {
void set_fused_smem(int bytes) {
    static std::mutex mu;
    static std::map<int, int> current;                       // per device
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (bytes > current[dev]) {
        require(bytes <= 227 * 1024, "moe (tc): shared-memory plan exceeds 227 KB");
        GPT_CHECK(cudaFuncSetAttribute(fz::moe_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        current[dev] = bytes;
    }
}
}  // namespace

void launch_moe_decode_tc(const DecodeTcArgs& a, cudaStream_t s) {
    using namespace fz;
    require(a.k >= 1 && a.k <= kMaxK, "moe (tc): k must be in 1..8");
    require(a.H % 64 == 0 && a.I % 64 == 0, "moe (tc): H and I must be multiples of 64");
    require(a.H <= 4 * kThreads * kMaxX4, "moe (tc): H too large for the register-held x");
    require(!a.router_w || (a.E >= a.k && a.E <= 32), "moe (tc): router needs k <= E <= 32");
    require(num_sms() <= 256, "moe (tc): more than 256 SMs");            // router partial-sum buffer
    const DecodeTcLayout W = decode_tc_layout(a.k, a.H, a.I);
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    Job j{};
    j.k = a.k;
    j.H = a.H;
    j.I = a.I;
    j.E = a.E;
    j.router_w = static_cast<const __nv_bfloat16*>(a.router_w);
    j.router_b = a.router_b;
    j.norm_w = a.norm_w;
    j.eps = a.eps;
    j.x = a.x;
    j.ids_in = a.ids;
    j.w_in = a.weights;
    j.ids_out = a.ids_out;
    j.w_out = a.w_out;
    j.sfa_gu = a.sfa_gu;
    j.sfa_dn = a.sfa_dn;
    j.sfa_by_slot = a.sfa_by_slot;
    j.gu_bias = a.gu_bias;
    j.dn_bias = a.dn_bias;
    j.alpha = a.alpha;
    j.limit = a.limit;
    Part& g = j.gu;
    g.mode = sk::kGateUp;
    g.RT = W.RT_gu;
    g.n_tiles = a.k * g.RT;
    g.UK = a.H / 64;
    g.KT = W.KT_gu;
    g.SPS = W.SPS_gu;
    g.UT = g.UK;
    g.total = (long long)g.n_tiles * g.UT;
    g.partial = reinterpret_cast<float*>(ws + W.off_part_gu);
    g.cnt = reinterpret_cast<unsigned*>(ws + W.off_cnt_gu);
    Part& d = j.dn;
    d.mode = sk::kDown;
    d.RT = W.RT_dn;
    d.n_tiles = d.RT;
    d.UK = a.I / 64;
    d.KT = W.KT_dn;
    d.SPS = W.SPS_dn;
    d.UT = a.k * d.UK;
    d.total = (long long)d.n_tiles * d.UT;
    d.partial = reinterpret_cast<float*>(ws + W.off_part_dn);
    d.cnt = reinterpret_cast<unsigned*>(ws + W.off_cnt_dn);
    j.aq_img = ws + W.off_aq_img;
    j.aq_sf = ws + W.off_aq_sf;
    j.x_resid = a.x_resid;
    j.err = reinterpret_cast<int*>(ws + W.off_err);
    j.gbar = reinterpret_cast<unsigned*>(ws + W.off_err + 256);
    j.partials = reinterpret_cast<double*>(ws + W.off_partials);
    j.trace = a.trace;

    // One CTA per SM, all resident (cooperative launch); the stage lists come from the per-shape table.
    const int nc = num_sms();
    const StageTable& T = stage_table(g, d, nc, a.k, a.H, a.I);
    j.stab = T.st;
    j.shdr = T.hdr;
    j.sf_upfront = T.cols <= int(kTmemCols);
    int NS = 8;
    Layout L = make_layout(NS, T.cap, T.cap_dn, g, a.H);
    while (L.bytes > 227 * 1024 && NS > 2) L = make_layout(NS -= 2, T.cap, T.cap_dn, g, a.H);
    require(L.bytes <= 227 * 1024, "moe (tc): shapes too large for one CTA's shared memory");
    j.L = L;
    set_fused_smem(L.bytes);

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nc);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = size_t(L.bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GPT_CHECK(cudaLaunchKernelEx(&cfg, moe_fused_kernel, *a.tmap_gu, *a.tmap_dn, j));
    check_launch("moe (tensor cores, fused)");
}

}  // namespace gpt
