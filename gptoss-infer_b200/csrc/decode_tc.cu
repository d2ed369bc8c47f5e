// Tensor-core decode MoE for one token: one persistent, cooperatively launched kernel per MoE layer.
//
// Operands. A = expert weights straight from the checkpoint layout (TMA boxes of 128 rows x 128 bytes of K, 128-byte
// swizzle); their E8M0 scales repacked into 512-byte tcgen05 chunks. B = the activation vector split into R = 16
// e2m1 residual terms, each with its own E8M0 scale per 32 elements, so x equals the sum of the terms to about
// 2^-30 of each block's maximum: the MMA's N = 16 columns hold the terms, the tensor core performs the MXFP4
// dequantization (tcgen05.mma kind::mxf4 block32) and the epilogue adds the 16 columns.
//
// Phases of every CTA (all 148 resident, one per SM):
//   0. RMSNorm of x and the router (logits = W h + b accumulated exactly in fp64, top-k with ties to the lower id,
//      softmax over the k) computed redundantly in every CTA; the weight stream starts as soon as the ids are known,
//      while the epilogue warps split h into e2m1 terms in shared memory.
//   1. Gate/up stream-K GEMV; the CTA finishing a 128-row tile applies bias, the clamped SwiGLU (rows 2j glu, 2j+1
//      linear) and the slot's gate weight, and writes the result as down's B terms (global memory).
//   2. Down stream-K GEMV over K' = k * I: the k experts' rows form one long GEMV because B carries the gate
//      weights; the CTA finishing a tile adds sum_slot w b2 and the residual.
// Gate/up and down stages flow through one TMA ring, so down's weights stream right behind gate/up's; only down's
// B operand waits, on a grid barrier counting CTAs whose gate/up epilogues are done (a bounded wait: the launch is
// cooperative, so every CTA is resident and the barrier always completes; a timeout records an error instead of
// hanging). Split tiles are reduced by their last contributor (deterministic order), never by spinning.
#include <algorithm>
#include <stdexcept>

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
constexpr int R = kDecodeTerms;
constexpr int kThreads = 192;                 // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kA = 16384, kB = R * 128;       // one weight stage (128 rows x 128 bytes of K), one B stage
constexpr uint32_t kTmemCols = 64;            // 2 x R accumulator columns + 8 SFA + 8 SFB
constexpr int kTraceSlots = 160;
constexpr int kMaxK = 8;

struct Layout {
    int NS, cap;                              // weight ring depth, stage-list capacity
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
    int* ids_out;                             // written by CTA 0 when not null
    float* w_out;
    const uint8_t* sfa_gu;                    // [mat][RT][KT][512]
    const uint8_t* sfa_dn;
    int sfa_by_slot;                          // mat = slot (1) or expert id (0)
    const float* gu_bias;                     // [E][2I]
    const float* dn_bias;                     // [E][H]
    float alpha, limit;
    Part gu, dn;
    uint8_t* aq_img;                          // down's B terms [k][SPS_dn][R*128]
    uint8_t* aq_sf;                           // down's B scales [k][KT_dn][512]
    float* x_resid;
    unsigned* gbar;                           // [4]: gate/up done, exits, phase-0 arrivals, ids published
    double* partials;                         // [grid][32] router partial sums
    int* ids_g;                               // [8] published expert ids
    float* w_g;                               // [8] published gate weights
    uint8_t* xq_img;                          // x as B terms [SPS_gu][R*128] (global)
    uint8_t* xq_sf;                           // their scales [KT_gu][512]
    int* err;
    long long* trace;                         // optional [grid][kTraceSlots] clock64 stamps
    Layout L;
};

// Trace slots per CTA: 0 start, 1 router done, 2+i producer issues stage i, 34+i MMA warp sees stage i landed,
// 66+g epilogue finished segment g, 80 x terms ready, 81 grid barrier passed (producer), 82 end.
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
    const int NS = j.L.NS, cap = j.L.cap;
    uint8_t* ringA = smem + j.L.ringA;
    uint8_t* regBgu = smem + j.L.regBgu;
    uint8_t* regSFBgu = smem + j.L.regSFBgu;
    uint8_t* regSFA = smem + j.L.regSFA;
    uint8_t* regBdn = smem + j.L.regBdn;
    uint8_t* regSFBdn = smem + j.L.regSFBdn;
    uint64_t* fullA = reinterpret_cast<uint64_t*>(smem + j.L.bars);
    uint64_t* empty = fullA + NS;
    uint64_t* fullS = empty + NS;             // [0] weight scales, [1] x terms (written here), [2] down's B terms
    uint64_t* accF = fullS + 3;               // [2]
    uint64_t* accE = accF + 2;                // [2]
    uint32_t* holder = reinterpret_cast<uint32_t*>(smem + j.L.misc);
    int* cnts = reinterpret_cast<int*>(holder + 2);          // [0] stages, [1] gate/up stages, [2] flag
    double* red = reinterpret_cast<double*>(cnts + 6);       // [6][32] router partial sums, then logits [32]
    int* ids_s = reinterpret_cast<int*>(red + 7 * 32);       // [8]
    float* w_s = reinterpret_cast<float*>(ids_s + kMaxK);    // [8]
    float* aval = w_s + kMaxK;                               // [64]
    Stage* stages = reinterpret_cast<Stage*>(aval + 64);     // [cap]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, nc = gridDim.x;
    if (tid == 0) stamp(j, 0);
    if (tid == 0) {
        int seg = 0;
        int n = sk::build_stages(j.gu, c, nc, stages, 0, cap, 0, &seg);
        const int ngu = n;
        n = sk::build_stages(j.dn, c, nc, stages, n, cap, seg, nullptr);
        if (n > cap) {
            atomicCAS(j.err, 0, 100);                        // host sized the stage list too small
            n = 0;
        }
        cnts[0] = n;
        cnts[1] = min(ngu, n);
        for (int i = 0; i < NS; ++i) {
            tc::mbar_init(&fullA[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        tc::mbar_init(&fullS[0], 1);
        tc::mbar_init(&fullS[1], 1);                         // x terms: bulk copies from global
        tc::mbar_init(&fullS[2], 1);
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&accF[i], 1);
            tc::mbar_init(&accE[i], 128);
        }
        tc::fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(holder, kTmemCols);
        tc::tmem_relinquish();
    }

    // ---------------------------------------------------------------- phase 0: RMSNorm, router, expert ids
    // Split across the grid: every CTA computes the RMSNorm factor (all of x), the router's partial dot products over
    // its slice of K for all experts (fp64, exact products) and the e2m1 terms of its share of x's 32-blocks (to
    // global memory). The last CTA to arrive adds the partial sums in CTA order, picks the top k, publishes the ids
    // and raises a release flag; every CTA waits for it (bounded wait; the launch is cooperative).
    {
        const int H = j.H, H8 = H >> 3;
        float ss = 0.f;
        if (j.norm_w) {
            for (int i = tid * 4; i < H; i += kThreads * 4) {
                const float4 v = *reinterpret_cast<const float4*>(j.x + i);
                ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
            }
            ss = warp_sum(ss);
            if (lane == 0) aval[warp] = ss;
        }
        __syncthreads();
        if (tid == 0) stamp(j, 84);
        float rn = 1.f;
        if (j.norm_w) {
            float tot = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) tot += aval[w];
            rn = 1.0f / sqrtf(tot / float(H) + j.eps);
        }
        auto hval = [&](int i) { return j.norm_w ? j.x[i] * rn * j.norm_w[i] : j.x[i]; };
        if (j.router_w) {
            // thread (e = tid % 32, o = tid / 32) takes chunk cs0 + o of expert e (8 bf16 weights)
            const int cs0 = int((long long)c * H8 / nc), cs1 = int((long long)(c + 1) * H8 / nc);
            const int e = tid & 31, o = tid >> 5;
            double acc = 0.0;
            for (int cc = cs0 + o; cc < cs1; cc += kThreads / 32) {
                if (e < j.E) {
                    const uint4 u = __ldg(reinterpret_cast<const uint4*>(j.router_w) + size_t(e) * H8 + cc);
                    const int b = cc * 8;
                    acc = fma(bf16lo(u.x), double(hval(b + 0)), acc); acc = fma(bf16hi(u.x), double(hval(b + 1)), acc);
                    acc = fma(bf16lo(u.y), double(hval(b + 2)), acc); acc = fma(bf16hi(u.y), double(hval(b + 3)), acc);
                    acc = fma(bf16lo(u.z), double(hval(b + 4)), acc); acc = fma(bf16hi(u.z), double(hval(b + 5)), acc);
                    acc = fma(bf16lo(u.w), double(hval(b + 6)), acc); acc = fma(bf16hi(u.w), double(hval(b + 7)), acc);
                }
            }
            red[o * 32 + e] = acc;
        }
        if (tid == 0) stamp(j, 85);
        // this CTA's x blocks -> e2m1 terms in global memory (warp 1; 4 lanes per block, up to 8 blocks per pass)
        const int nb = H / 32, b0 = int((long long)c * nb / nc), b1 = int((long long)(c + 1) * nb / nc);
        if (warp == 1) {
            for (int g0 = b0; g0 < b1; g0 += 8) {
                const int g = g0 + (lane >> 2), sub = lane & 3;
                const bool active = g < b1;
                const int gg = active ? g : b0;
                float v8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v8[i] = active ? hval(gg * 32 + sub * 8 + i) : 0.f;
                quantize_block_terms_cvt(v8, j.xq_img + (gg / 8) * kB, gg % 8, j.xq_sf + (gg / 4) * 512, gg % 4, sub,
                                         active);
            }
            __threadfence();
            if (lane == 0) stamp(j, 86);
        }
        __syncthreads();
        if (warp == 0) {
            bool last = false;
            if (lane == 0) {
                if (j.router_w)
                    for (int q = 0; q < 32; ++q) {
                        double t = 0.0;
                        for (int w = 0; w < kThreads / 32; ++w) t += red[w * 32 + q];
                        j.partials[size_t(c) * 32 + q] = t;
                    }
                __threadfence();
                last = atomicAdd(&j.gbar[2], 1u) == unsigned(nc - 1);
                stamp(j, 87);
            }
            last = __shfl_sync(kFull, last, 0);
            if (last) {
                __threadfence();
                if (j.router_w) {
                    // lane i sums expert i's partials in CTA order, then the top k (ties to the lower id; picked
                    // experts and lanes >= E carry -inf and an id >= 32; NaN never wins) and the softmax
                    double v = -INFINITY;
                    if (lane < j.E) {
                        double t = 0.0;
                        for (int cc = 0; cc < nc; ++cc) t += __ldcg(&j.partials[size_t(cc) * 32 + lane]);
                        v = t + double(j.router_b[lane]);
                    }
                    if (v != v) v = -INFINITY;
                    int id = lane < j.E ? lane : 32 + lane;
                    float sel = -INFINITY;
                    int sel_id = 0;
                    for (int q = 0; q < j.k; ++q) {
                        double best = v;
                        int besti = id;
#pragma unroll
                        for (int o2 = 16; o2 > 0; o2 >>= 1) {
                            const double ob = __shfl_xor_sync(kFull, best, o2);
                            const int oi = __shfl_xor_sync(kFull, besti, o2);
                            if (ob > best || (ob == best && oi < besti)) { best = ob; besti = oi; }
                        }
                        if (lane == q) { sel = float(best); sel_id = besti; }
                        if (id == besti) { v = -INFINITY; id = 32 + lane; }
                    }
                    const float top = __shfl_sync(kFull, sel, 0);
                    const float pz = lane < j.k ? expf(sel - top) : 0.f;
                    const float sum = warp_sum(pz);
                    if (lane < j.k) {
                        j.ids_g[lane] = sel_id;
                        j.w_g[lane] = pz / sum;
                        if (j.ids_out) { j.ids_out[lane] = sel_id; j.w_out[lane] = pz / sum; }
                    }
                } else if (lane < j.k) {
                    j.ids_g[lane] = j.ids_in[lane];
                    j.w_g[lane] = j.w_in[lane];
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&j.gbar[3]), "r"(1u) : "memory");
            }
            // every CTA: wait for the published ids (bounded)
            bool ready = false;
            for (uint32_t i = 0; i < tc::kSpinLimit && !ready; ++i) {
                ready = __shfl_sync(kFull, lane == 0 ? ld_acquire(&j.gbar[3]) != 0u : false, 0);
                if (!ready) __nanosleep(32);
            }
            if (lane == 0) stamp(j, 88);
            if (!ready) {
                if (lane == 0) atomicCAS(j.err, 0, 10);
                if (lane < j.k) { ids_s[lane] = 0; w_s[lane] = 0.f; }
            } else if (lane < j.k) {
                ids_s[lane] = __ldcg(&j.ids_g[lane]);
                w_s[lane] = __ldcg(&j.w_g[lane]);
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (tid == 0) stamp(j, 1);
    const int nst = cnts[0], ngu = cnts[1];
    const uint32_t tmem = *holder;
    const uint32_t tm_acc = tmem, tm_sfa = tmem + 2 * R, tm_sfb = tmem + 2 * R + 8;

    auto part_of = [&](const Stage& st) -> const Part& { return st.mode == sk::kGateUp ? j.gu : j.dn; };
    auto rt_of = [&](const Stage& st) { return st.mode == sk::kGateUp ? st.tile % j.gu.RT : st.tile; };

    if (warp == 0) {
        // ---------------------------------------------------------------- producer (converged warp, elected lane)
        // Per stage one 16 KB TMA box of weights; the scales of the whole range and down's B terms in a few large
        // copies (every copy instruction costs hundreds of cycles to issue regardless of its size).
        bool dn_b_issued = nst == ngu;
        auto issue_dn_b = [&]() {
            uint32_t bytes = 0;
            sk::for_each_run(stages, ngu, nst, [&](int a, int b, int chunks) { bytes += (b - a) * kB + chunks * 512; });
            tc::mbar_arrive_expect_tx(&fullS[2], bytes);
            sk::for_each_run(stages, ngu, nst, [&](int a, int b, int chunks) {
                const Stage& st = stages[a];
                tc::bulk_g2s(regBdn + (a - ngu) * kB, j.aq_img + (size_t(st.s) * j.dn.SPS + st.ku0 / 4) * kB,
                             (b - a) * kB, &fullS[2]);
                tc::bulk_g2s(regSFBdn + (a - ngu) * 1024, j.aq_sf + (size_t(st.s) * j.dn.KT + st.ku0 / 2) * 512,
                             chunks * 512, &fullS[2]);
            });
        };
        auto gate_up_done = [&]() { return ld_acquire(&j.gbar[0]) >= unsigned(nc); };
        auto after_barrier = [&]() {
            stamp(j, 81);
            asm volatile("fence.proxy.async.global;" ::: "memory");   // others' generic writes -> our bulk reads
            issue_dn_b();
            dn_b_issued = true;
        };
        if (tc::elect_one()) {
            stamp(j, 89);
            tc::prefetch_tmap(&tm_gu);
            tc::prefetch_tmap(&tm_dn);
            stamp(j, 90);
            // x terms written by all CTAs in phase 0 (generic stores, published by the release flag)
            asm volatile("fence.proxy.async.global;" ::: "memory");
            stamp(j, 91);
            tc::mbar_arrive_expect_tx(&fullS[1], j.gu.SPS * kB + j.gu.KT * 512);
            tc::bulk_g2s(regBgu, j.xq_img, j.gu.SPS * kB, &fullS[1]);
            tc::bulk_g2s(regSFBgu, j.xq_sf, j.gu.KT * 512, &fullS[1]);
            stamp(j, 92);
            uint32_t bytes = 0;
            sk::for_each_run(stages, 0, nst, [&](int a, int b, int chunks) { bytes += chunks * 512; });
            tc::mbar_arrive_expect_tx(&fullS[0], bytes);
            sk::for_each_run(stages, 0, nst, [&](int a, int b, int chunks) {
                const Stage& st = stages[a];
                const Part& p = part_of(st);
                const int mat = j.sfa_by_slot ? int(st.s) : ids_s[st.s];
                const uint8_t* base = st.mode == sk::kGateUp ? j.sfa_gu : j.sfa_dn;
                tc::bulk_g2s(regSFA + a * 1024, base + ((size_t(mat) * p.RT + rt_of(st)) * p.KT + st.ku0 / 2) * 512,
                             chunks * 512, &fullS[0]);
            });
            stamp(j, 93);
        }
        __syncwarp();
        // The tensor map is a compile-time parameter of each loop: selecting it at run time made every TMA issue
        // wait for a descriptor fetch.
        auto wait_slot = [&](int it) -> bool {
            // wait for the slot; meanwhile issue down's B terms as soon as every CTA finished gate/up
            const int slot = it % NS;
            bool got = false;
            for (uint32_t i = 0; i < tc::kSpinLimit && !got; ++i) {
                got = __all_sync(kFull, tc::mbar_try_wait(&empty[slot], ((it / NS) - 1) & 1));
                if (!got && !dn_b_issued && (i & 15) == 0) {
                    const bool done = __shfl_sync(kFull, lane == 0 ? gate_up_done() : false, 0);
                    if (done) {
                        if (tc::elect_one()) after_barrier();
                        dn_b_issued = true;
                        __syncwarp();
                    }
                }
            }
            if (!got && lane == 0) atomicCAS(j.err, 0, 1);
            return got;
        };
        bool ok = true;
        for (int it = 0; it < ngu && ok; ++it) {
            if (it >= NS) ok = wait_slot(it);
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
            if (it >= NS) ok = wait_slot(it);
            if (ok && tc::elect_one()) {
                if (it < 32) stamp(j, 2 + it);
                const Stage& st = stages[it];
                tc::mbar_arrive_expect_tx(&fullA[it % NS], kA);
                tc::tma_load_3d(ringA + (it % NS) * kA, &tm_dn, (st.ku0 / 4) * 128, st.tile * 128, ids_s[st.s],
                                &fullA[it % NS]);
            }
            __syncwarp();
        }
        if (!dn_b_issued) {                                  // every weight stage issued; wait for gate/up
            bool done = false;
            for (uint32_t i = 0; i < tc::kSpinLimit && !done; ++i) {
                done = __shfl_sync(kFull, lane == 0 ? gate_up_done() : false, 0);
                if (!done) __nanosleep(64);
            }
            if (done) {
                if (tc::elect_one()) after_barrier();
            } else if (lane == 0) {
                atomicCAS(j.err, 0, 8);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (converged warp, one lane)
        bool ok = nst == 0 || (tc::mbar_wait(&fullS[0], 0, j.err, 6) && tc::mbar_wait(&fullS[1], 0, j.err, 7));
        ok = __all_sync(kFull, ok);
        for (int it = 0; it < nst && ok; ++it) {
            const Stage& st = stages[it];
            const int slot = it % NS, ph = (it / NS) & 1;
            const int buf = st.seg & 1;
            if (it == ngu) ok = tc::mbar_wait(&fullS[2], 0, j.err, 9);     // down's B terms
            if (st.first && st.seg >= 2) ok = ok && tc::mbar_wait(&accE[buf], ((st.seg >> 1) - 1) & 1, j.err, 2);
            ok = ok && tc::mbar_wait(&fullA[slot], ph, j.err, 3);
            ok = __all_sync(kFull, ok);
            if (!ok) break;
            tc::tc_fence_after();
            if (tc::elect_one()) {
                if (it < 32) stamp(j, 34 + it);
                const int kt0 = st.ku0 / 2, nkt = sk::nkt_of(st);
                const bool gu = st.mode == sk::kGateUp;
                const uint8_t* sfb = gu ? regSFBgu + kt0 * 512 : regSFBdn + (it - ngu) * 1024;
                const uint8_t* bst = gu ? regBgu + (st.ku0 / 4) * kB : regBdn + (it - ngu) * kB;
                for (int q = 0; q < nkt; ++q) {
                    tc::tmem_cp_sf(tm_sfa + 4 * q, tc::desc_sf_chunk(tc::smem_u32(regSFA + it * 1024 + q * 512)));
                    tc::tmem_cp_sf(tm_sfb + 4 * q, tc::desc_sf_chunk(tc::smem_u32(sfb + q * 512)));
                }
                for (int u = 0; u < st.nu; ++u) {
                    const int ku = st.ku0 + u;
                    const uint32_t sf_id = 2u * (ku & 1);
                    const uint32_t q = uint32_t(ku / 2 - kt0);
                    const uint64_t ad = tc::desc_sw128(tc::smem_u32(ringA + slot * kA + u * 32));
                    const uint64_t bd = tc::desc_sw128(tc::smem_u32(bst + u * 32));
                    tc::mma_mxf4(tm_acc + buf * R, ad, bd, tc::idesc_mxf4(128, R, sf_id, sf_id),
                                 (tm_sfa + 4 * q) | (sf_id << 30), (tm_sfb + 4 * q) | (sf_id << 30),
                                 !(st.first && u == 0));
                }
                tc::mma_commit(&empty[slot]);
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
        if (et == 0) stamp(j, 80);
        auto arrive_gate_up_done = [&]() {
            __threadfence();                        // this thread's down-B terms and partial sums are published
            epi_sync();
            if (et == 0) {
                __threadfence();
                atomicAdd(&j.gbar[0], 1u);
            }
        };
        if (ngu == 0) arrive_gate_up_done();
        bool ok = true;
        for (int it = 0; it < nst; ++it) {
            const Stage& st = stages[it];
            if (!st.last) continue;
            const int buf = st.seg & 1;
            ok = ok && tc::mbar_wait_sleepy(&accF[buf], (st.seg >> 1) & 1, j.err, 5, 128);
            ok = epi_all(ok);                        // uniform over the 4 epilogue warps before any named barrier
            float v = 0.f;
            if (ok) {
                tc::tc_fence_after();
                float t0[8], t1[8];
                tc::tmem_ld_32x32b_x8(tm_acc + buf * R + (uint32_t(quad * 32) << 16), t0);
                tc::tmem_ld_32x32b_x8(tm_acc + buf * R + 8 + (uint32_t(quad * 32) << 16), t1);
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
                const long long T0 = (long long)t * p.UT, T1 = T0 + p.UT;
                const bool whole = sk::cta_begin(p, c, nc) <= T0 && sk::cta_begin(p, c + 1, nc) >= T1;
                float total = v;
                bool mine = true;                    // this CTA applies the tile's epilogue
                if (!whole) {
                    int cf, cl;
                    sk::tile_contributors(p, t, nc, cf, cl);
                    if (c - cf >= sk::kMaxContrib) {
                        if (et == 0) atomicCAS(j.err, 0, 101);
                        mine = false;
                    } else {
                        p.partial[(size_t(t) * sk::kMaxContrib + (c - cf)) * 128 + row] = v;
                        __threadfence();
                        epi_sync();
                        if (et == 0) {
                            long long s0 = sk::cta_begin(p, c, nc), s1 = sk::cta_begin(p, c + 1, nc);
                            s0 = s0 > T0 ? s0 : T0;
                            s1 = s1 < T1 ? s1 : T1;
                            __threadfence();
                            const unsigned old = atomicAdd(&p.cnt[t], unsigned(s1 - s0));
                            const bool last = old + unsigned(s1 - s0) == unsigned(p.UT);
                            if (last) p.cnt[t] = 0;      // every contributor has arrived: reset for the next launch
                            __threadfence();
                            cnts[2] = last;
                        }
                        epi_sync();
                        mine = cnts[2] != 0;
                        if (mine) {
                            total = 0.f;
                            for (int cc = cf; cc <= cl && cc - cf < sk::kMaxContrib; ++cc) {
                                long long a0 = sk::cta_begin(p, cc, nc), a1 = sk::cta_begin(p, cc + 1, nc);
                                if ((a0 > T0 ? a0 : T0) >= (a1 < T1 ? a1 : T1)) continue;   // no work in this tile
                                total += __ldcg(&p.partial[(size_t(t) * sk::kMaxContrib + (cc - cf)) * 128 + row]);
                            }
                        }
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
                        quantize_block_terms_cvt(v8, img, gb % 8, sf, gb % 4, sub, active);
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
            if (st.mode == sk::kGateUp && it == ngu - 1) arrive_gate_up_done();
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
            j.gbar[3] = 0;
            j.gbar[1] = 0;
        }
    }
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// Shared-memory plan: NS weight stages, the x image and its scales, per-entry weight-scale chunks (1 KB each),
// per-down-entry B stages and scale chunks, h (fp32), barriers, and the small per-CTA state.
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
    L.hs = o;
    L.bars = o; o += (2 * NS + 7) * 8;
    o = (o + 15) & ~15;
    L.misc = o; o += 8 + 24 + 7 * 32 * 8 + 2 * kMaxK * 4 + 64 * 4 + cap * int(sizeof(Stage));
    L.bytes = 1024 + o;
    return L;
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
    L.off_xq_img = o; o += al(size_t(L.SPS_gu) * R * 128);
    L.off_xq_sf = o; o += al(size_t(L.KT_gu) * 512);
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
    static int current = 0;
    if (bytes > current) {
        require(bytes <= 227 * 1024, "moe (tc): shared-memory plan exceeds 227 KB");
        GPT_CHECK(cudaFuncSetAttribute(fz::moe_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        current = bytes;
    }
}
}  // namespace

void launch_moe_decode_tc(const DecodeTcArgs& a, cudaStream_t s) {
    using namespace fz;
    require(a.k >= 1 && a.k <= kMaxK, "moe (tc): k must be in 1..8");
    require(a.H % 64 == 0 && a.I % 64 == 0, "moe (tc): H and I must be multiples of 64");
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
    j.ids_g = reinterpret_cast<int*>(ws + W.off_err + 512);
    j.w_g = reinterpret_cast<float*>(ws + W.off_err + 640);
    j.xq_img = ws + W.off_xq_img;
    j.xq_sf = ws + W.off_xq_sf;
    j.trace = a.trace;

    // One CTA per SM, all resident (cooperative launch). The stage-list capacity comes from running the same
    // partition code the kernel runs.
    const int nc = num_sms();
    int cap = 1, cap_dn = 1;
    for (int cta = 0; cta < nc; ++cta) {
        int seg = 0;
        const int ngu = sk::build_stages(g, cta, nc, nullptr, 0, 0, 0, &seg);
        const int n = sk::build_stages(d, cta, nc, nullptr, ngu, 0, seg, nullptr);
        cap = std::max(cap, n);
        cap_dn = std::max(cap_dn, n - ngu);
    }
    int NS = 8;
    Layout L = make_layout(NS, cap, cap_dn, g, a.H);
    while (L.bytes > 227 * 1024 && NS > 2) L = make_layout(--NS, cap, cap_dn, g, a.H);
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
