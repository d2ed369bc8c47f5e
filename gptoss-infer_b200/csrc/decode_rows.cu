// Tensor-core decode MoE for one token, one job per CTA: a persistent cooperative kernel of G = k * ceil(2I / 256)
// CTAs per MoE layer. CTA c owns job (slot s, row tile rt) = (c / RT, c % RT):
//   gate/up: the 256 interleaved gate/up rows [256 rt, 256 rt + 256) of expert ids[s] over the whole of K = H, so the
//            tile's 128 activations [128 rt, 128 rt + 128) are finished inside the CTA (no partial sums cross CTAs);
//   down:    the K-slice of those 128 activations (64 bytes of every down row) against all H rows, giving a partial
//            output vector of H values (already weighted by the slot's gate weight);
//   end:     one grid-wide count of finished partial vectors, then CTA c adds the G partial vectors of its 32-row
//            groups in job order, the weighted down biases and the residual.
// The activations never leave the CTA: the gate/up epilogue quantizes them into down's operand in shared memory. The
// only exchanges between CTAs are the router logits (phase 0), x's terms and the final partial vectors.
//
// Operands (tcgen05.mma kind::mxf4, M = 128, N = 8, K = 64, measured at the same ~56-cycle cost as any N <= 64):
//   A = 128 weight rows straight from the checkpoint layout by TMA: gate/up boxes of 256 rows x 128 bytes of K (the
//       128-byte swizzle), down boxes of 256 rows x 64 bytes of K (the 64-byte swizzle: exactly the job's slice);
//       their E8M0 scales come from the layer's repacked chunks (tiles of 256 rows: [tile][K chunk][half][512]).
//   B = the activation vector as NT = 8 e2m1 residual terms with their own E8M0 scale per 32 elements (the integer
//       digit split of terms.cuh: their sum equals the vector to 2^-21 of each block's scale); the 8 terms are the
//       MMA's 8 columns, so accumulator lane r holds weight row r's dot product with each term, and the epilogue adds
//       the 8 columns in a fixed order.
// Roles: warp 0 streams the weights (TMA; gate/up stages, then the down stages, through one ring); warp 1 issues the
// tcgen05 operations; warps 2-3 make x's terms (see there); warps 2-5 run the gate/up epilogue (bias, clamped SwiGLU,
// gate weight, quantization into down's operand) and the down epilogue (partial vector to global memory), then the
// final reduction. Phase 0 (RMSNorm, router) is the same as in the stream-K decode kernel. Every wait is
// bounded: the launch is cooperative, so all CTAs are resident; a timeout records an error code and the kernel
// drains instead of hanging.
#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"
#include "terms.cuh"

namespace gpt {
namespace rj {

constexpr int NT = 8;                         // activation terms (the MMA's N)
constexpr int kThreads = 192;                 // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kRows = 256;                    // weight rows per TMA box (two M = 128 halves)
constexpr int kGu = kRows * 128;              // gate/up stage: 256 rows x 128 bytes of K (32 KB)
constexpr int kDn = kRows * 64;               // down box: 256 rows x 64 bytes of K (16 KB)
constexpr int kSlot = kGu + 2048;             // ring slot: a gate/up box and its scale chunks (2 K chunks x 2 halves
                                              // x 512), or two down boxes and theirs (2 x 1 KB)
constexpr int kMaxPairs = 8;                  // down stages (pairs of row boxes): H <= 4096
constexpr int kMaxStages = 12;                // gate/up stages of 256 values of K: H <= 3072
constexpr int kA = NT * 128;                  // terms of 256 values of K (8 rows x 128 bytes)
constexpr int kSF8 = 128;                     // terms' scale chunk (rows 0-7 of a 512-byte chunk)
constexpr int kMaxK = 8;
constexpr int kMaxX4 = 4;                     // x is held as kMaxX4 float4 per thread: H <= 4 * kThreads * kMaxX4
constexpr int kTraceSlots = 160;
constexpr uint32_t kTmemCols = 512;
#ifndef GPTOSS_LOGIT_POLL_NS
#define GPTOSS_LOGIT_POLL_NS 200
#endif
constexpr unsigned kLogitPollNs = GPTOSS_LOGIT_POLL_NS;   // pause between two polls of the router logits
#ifndef GPTOSS_X_PLAN
#define GPTOSS_X_PLAN 0
#endif
// Where x's terms are made: 0 in phase 0 from the registers that hold h (each CTA its blocks), counted after phase 0;
// 1 right after phase 0 by one epilogue warp from h recomputed from global memory; 2 the same after the expert ids.
constexpr int kXPlan = GPTOSS_X_PLAN;
#ifndef GPTOSS_STAGE_COUNTS
#define GPTOSS_STAGE_COUNTS 0
#endif
// 1: the partial sums are counted per down stage (reductions of early rows start before the last stage is done);
// 0: one count after the whole down phase.
constexpr bool kStageCounts = GPTOSS_STAGE_COUNTS != 0;
#ifndef GPTOSS_TAGGED_PARTIALS
#define GPTOSS_TAGGED_PARTIALS 1
#endif
// 1: partial sums travel as 64-bit words (launch epoch << 32) | fp32 bits, which the reducing CTAs poll directly (no
// count, no release fence); 0: fp32 words behind one grid-wide count.
constexpr bool kTagged = GPTOSS_TAGGED_PARTIALS != 0;
constexpr uint32_t kColGu = 0;                // gate/up accumulator: 2 halves x 8 columns
constexpr uint32_t kColDn = 16;               // down accumulators: row box d, half h at 16 d + 8 h

struct Layout {
    int NS, NSF;                              // ring depth, weight-scale TMEM ring depth
    uint32_t colXs, colDs, colW;              // TMEM columns: x's scale chunks, down operand's scale chunk, ring
    int ring, xA, xSF, dA, dSF, act, red4, bars, misc, bytes;
};

struct Job {
    int k, H, I, E, RT, G;                    // RT jobs per slot, G jobs
    int SPS, UK, KT_gu, RD, KT_dn, RT_dn;     // gate/up stages and units, down row boxes
    int NP;                                   // down stages: pairs of row boxes, (RD + 1) / 2
    const __nv_bfloat16* router_w;            // null: ids_in / w_in give the experts
    const float* router_b;
    const float* norm_w;                      // null: x is already normalized
    float eps;
    const float* x;
    const int* ids_in;
    const float* w_in;
    int* ids_out;                             // written by CTA 0 when not null
    float* w_out;
    const uint8_t* sf_gu;                     // [mat][RT_gu256][KT_gu][2][512]
    const uint8_t* sf_dn;                     // [mat][RT_dn][KT_dn][2][512]
    int sf_by_slot;                           // mat = slot (1) or expert id (0)
    const float* gu_bias;                     // [E][2I]
    const float* dn_bias;                     // [E][H]
    float alpha, limit;
    float* part;                              // [G][H] partial output vectors (fp32, or 64-bit tagged words)
    const uint8_t* dn_img;                    // pre-packed down stages [E][RT][NP][kSlot], or null (TMA boxes)
    uint8_t* xq_img;                          // x's terms [SPS][NT*128]
    uint8_t* xq_sf;                           // their scales [KT_gu][128]
    float* x_resid;
    unsigned* gbar;                           // [16]: -, exits, -, x blocks written, last epoch, -, -, -, then per down
                                              // stage p at [8 + p] the CTAs whose partial sums of its rows are stored
    unsigned long long* logit_words;          // [32][2] router logit e as (epoch << 32) | high and low 32 bits
    int* err;
    long long* trace;                         // optional [grid][kTraceSlots] clock64 stamps
    Layout L;
};

// Trace slots (cycles from each CTA's start): 0 start, 123 previous layer complete, 85 router logit published, 120
// logits read, 121 top k, 122 softmax, 88 ids released, 2+i producer issues stage i (i < 32), 34+i MMA warp sees stage
// i landed, 131 gate/up epilogue done (down operand ready), 140+p down stage p's accumulators read out, 133 partial
// vector stored, 81 all partial vectors counted, 134 partial vectors of the first row group added, 82 end.
template <bool kTrace>
__device__ __forceinline__ void stamp(const Job& j, int slot) {
    if constexpr (kTrace) j.trace[size_t(blockIdx.x) * kTraceSlots + slot] = clock64();
}
// Slot 159: the global timer (ns) at the CTA's start, which places the CTAs' clock64 stamps on one time axis.
template <bool kTrace>
__device__ __forceinline__ void stamp_global_start(const Job& j) {
    if constexpr (kTrace) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        j.trace[size_t(blockIdx.x) * kTraceSlots + 159] = static_cast<long long>(t);
    }
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
__device__ __forceinline__ void red_add_release(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// The launch epoch that follows prev, skipping 0 (a zero-filled logit word must never read as current).
__device__ __forceinline__ unsigned next_epoch(unsigned prev) { return prev == 0xFFFFFFFFu ? 1u : prev + 1u; }

__device__ __forceinline__ double bf16lo(uint32_t w) { return double(__uint_as_float(w << 16)); }
__device__ __forceinline__ double bf16hi(uint32_t w) { return double(__uint_as_float(w & 0xffff0000u)); }

// One accumulator row (M = 128, N = 8) as read by tcgen05.ld: its 8 term columns added in column order.
__device__ __forceinline__ float term_sum(const uint32_t* v) {
    float s = __uint_as_float(v[0]);
#pragma unroll
    for (int t = 1; t < NT; ++t) s += __uint_as_float(v[t]);
    return s;
}

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1) moe_rows_kernel(const __grid_constant__ CUtensorMap tm_gu,
                                                               const __grid_constant__ CUtensorMap tm_dn,
                                                               const __grid_constant__ Job j) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NS = j.L.NS, NSF = j.L.NSF;
    uint8_t* ring = smem + j.L.ring;          // [NS][kSlot]
    uint8_t* xA = smem + j.L.xA;              // [SPS][kA] x's terms
    uint8_t* xSF = smem + j.L.xSF;            // [KT_gu][kSF8] their scales
    uint8_t* dA = smem + j.L.dA;              // [kA] down's operand: the job's activations as terms
    uint8_t* dSF = smem + j.L.dSF;            // [kSF8] their scales
    float* act_s = reinterpret_cast<float*>(smem + j.L.act);     // [128] the job's activations
    float* red16 = reinterpret_cast<float*>(smem + j.L.red4);    // [16][32] reduction partials
    uint64_t* fullB = reinterpret_cast<uint64_t*>(smem + j.L.bars);   // [NS] stage landed
    uint64_t* emptyB = fullB + NS;            // [NS] stage consumed by the MMAs
    uint64_t* fullS = emptyB + NS;            // x's terms copied into shared memory (bulk copies)
    uint64_t* accF = fullS + 1;               // gate/up accumulator complete
    uint64_t* dReady = accF + 1;              // down's operand written (128 arrivals)
    uint64_t* accD = dReady + 1;              // [NP] down stage p's accumulators complete
    uint64_t* pDone = accD + kMaxPairs;       // [NP] down stage p's partial sums stored (128 arrivals)
    uint32_t* holder = reinterpret_cast<uint32_t*>(smem + j.L.misc);
    double* red = reinterpret_cast<double*>(holder + 8);     // [8] router sums
    int* ids_s = reinterpret_cast<int*>(red + 8);            // [8]
    float* w_s = reinterpret_cast<float*>(ids_s + kMaxK);    // [8]
    float* aval = w_s + kMaxK;                               // [8] per-warp sums of squares
    int* flag_s = reinterpret_cast<int*>(aval + 8);          // [1] final count reached

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, nc = gridDim.x;
    const int s_job = c / j.RT, rt = c - s_job * j.RT;
    if (tid == 0) {
        stamp<kTrace>(j, 0);
        stamp_global_start<kTrace>(j);
    }
    // Router CTAs: CTA c < E computes expert c's logit over all of K; thread t holds the same elements of the router
    // row as of x (float4 chunks t, t + kThreads, ...), widened to fp64 before the previous layer has finished.
    const bool router_cta = j.router_w != nullptr && c < j.E;
    double wd[kMaxX4][4];
    double rbias = 0.0;
#pragma unroll
    for (int r = 0; r < kMaxX4; ++r) {
        const int i = (tid + r * kThreads) * 4;
        uint2 u = make_uint2(0u, 0u);
        if (router_cta && i < j.H) u = __ldg(reinterpret_cast<const uint2*>(j.router_w + size_t(c) * j.H + i));
        wd[r][0] = bf16lo(u.x);
        wd[r][1] = bf16hi(u.x);
        wd[r][2] = bf16lo(u.y);
        wd[r][3] = bf16hi(u.y);
    }
    if (router_cta) rbias = double(__ldg(j.router_b + c));
    float4 xv[kMaxX4], gv[kMaxX4];
#pragma unroll
    for (int r = 0; r < kMaxX4; ++r) {
        const int i = (tid + r * kThreads) * 4;
        gv[r] = i < j.H && j.norm_w ? __ldg(reinterpret_cast<const float4*>(j.norm_w + i))
                                    : make_float4(1.f, 1.f, 1.f, 1.f);
    }
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            tc::mbar_init(&fullB[i], 1);
            tc::mbar_init(&emptyB[i], 1);
        }
        tc::mbar_init(fullS, 1);
        tc::mbar_init(accF, 1);
        tc::mbar_init(dReady, 128);
        for (int p = 0; p < j.NP; ++p) {
            tc::mbar_init(&accD[p], 1);
            tc::mbar_init(&pDone[p], 128);
        }
        tc::fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(holder, kTmemCols);
        tc::tmem_relinquish();
    }
    // Everything above reads only what no earlier kernel writes. With programmatic dependent launch the next
    // layer's kernel is released now and this one waits for the previous layer's kernel to finish.
    pdl_launch_dependents();
    pdl_wait();
    const unsigned ep = next_epoch(__ldcg(&j.gbar[4]));
    if (tid == 0) stamp<kTrace>(j, 123);
#pragma unroll
    for (int r = 0; r < kMaxX4; ++r) {
        const int i = (tid + r * kThreads) * 4;
        xv[r] = i < j.H ? *reinterpret_cast<const float4*>(j.x + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // ---------------------------------------------------------------- phase 0: RMSNorm, router
    // Router CTA c publishes logit c (fp64, exact bf16 x fp32 products summed in a fixed order) as two epoch-tagged
    // 64-bit words that warp 0 of every CTA polls. x's terms are made afterwards (see the epilogue warps).
    float rn = 1.f;
    {
        const int H = j.H;
        float ss = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxX4; ++r)
            ss = fmaf(xv[r].x, xv[r].x, fmaf(xv[r].y, xv[r].y, fmaf(xv[r].z, xv[r].z, fmaf(xv[r].w, xv[r].w, ss))));
        ss = warp_sum(ss);
        if (lane == 0) aval[warp] = ss;
        __syncthreads();
        if (j.norm_w) {
            float tot = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) tot += aval[w];
            rn = rms_scale(tot, H, j.eps);
        }
#pragma unroll
        for (int r = 0; r < kMaxX4; ++r)
            if (j.norm_w) {
                xv[r].x = xv[r].x * rn * gv[r].x; xv[r].y = xv[r].y * rn * gv[r].y;
                xv[r].z = xv[r].z * rn * gv[r].z; xv[r].w = xv[r].w * rn * gv[r].w;
            }
        if (router_cta) {
            double acc = 0.0;
#pragma unroll
            for (int r = 0; r < kMaxX4; ++r) {
                acc = fma(wd[r][0], double(xv[r].x), acc);
                acc = fma(wd[r][1], double(xv[r].y), acc);
                acc = fma(wd[r][2], double(xv[r].z), acc);
                acc = fma(wd[r][3], double(xv[r].w), acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) red[warp] = acc;
            __syncthreads();
            if (tid == 0) {
                double t = 0.0;
                for (int w = 0; w < kThreads / 32; ++w) t += red[w];
                const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(t + rbias));
                st_relaxed64(j.logit_words + 2 * c, (static_cast<unsigned long long>(ep) << 32) | (bits >> 32));
                st_relaxed64(j.logit_words + 2 * c + 1,
                             (static_cast<unsigned long long>(ep) << 32) | (bits & 0xFFFFFFFFull));
                stamp<kTrace>(j, 85);
            }
        }
        if constexpr (kXPlan == 0) {
            // x's block g (g = nc - 1 - c mod nc) in the 8 lanes whose registers hold it (float4 round g / 24,
            // threads 8 (g % 24) .. + 7), into global memory; counted after phase 0
            const int nb = H / 32, per_round = kThreads / 8;
#pragma unroll
            for (int r = 0; r < kMaxX4; ++r) {
                const int g = r * per_round + tid / 8;
                if (g < nb && nc - 1 - (g % nc) == c) {          // uniform over the 8 lanes of the group
                    const int sub8 = tid & 7;
                    const float v[4] = {xv[r].x, xv[r].y, xv[r].z, xv[r].w};
                    uint8_t* img = j.xq_img + size_t(g / 8) * kA + 2 * sub8;
                    uint8_t* sf = j.xq_sf + size_t(g / 4) * kSF8 + (g & 3);
                    const int q = g & 7;
                    const unsigned grp = 0xFFu << (lane & 24);
                    quantize_block_digits_lanes8_masked(v, grp, [&](int t, uint32_t half, uint32_t scale) {
                        *reinterpret_cast<uint16_t*>(img + t * 128 + ((q ^ (t & 7)) << 4)) = uint16_t(half);
                        if (sub8 < 4) sf[t * 16 + sub8 * 4] = uint8_t(scale);
                    });
                }
            }
        }
    }
    tc::fence_proxy_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *holder;

    if (warp == 0) {
        // ---------------------------------------------------------------- expert ids, then the TMA producer
        int sel_id = 0;
        double sel_logit = 0.0;
        if (j.router_w) {
            unsigned long long w0 = 0, w1 = 0;
            bool done = false;
            for (uint32_t i = 0; i < tc::kSpinLimit && !done; ++i) {
                if (lane < j.E) {
                    w0 = ld_relaxed64(j.logit_words + 2 * lane);
                    w1 = ld_relaxed64(j.logit_words + 2 * lane + 1);
                }
                done = __all_sync(kFull, lane >= j.E || (unsigned(w0 >> 32) == ep && unsigned(w1 >> 32) == ep));
                if (!done) __nanosleep(kLogitPollNs);
            }
            if (!done && lane == 0) atomicCAS(j.err, 0, 10);
            const double v = __longlong_as_double(static_cast<long long>((w0 << 32) | (w1 & 0xFFFFFFFFull)));
            if (lane == 0) stamp<kTrace>(j, 120);
            warp_topk_logits(v, lane < j.E, j.k, sel_id, sel_logit);
            if (lane == 0) stamp<kTrace>(j, 121);
        }
        // The job's expert is known: the loads start now; the gate weights (the softmax over the k picks), which
        // only the epilogue needs, are computed after the ring's first loads are issued (publish below).
        const int e = j.router_w ? __shfl_sync(kFull, sel_id, s_job) : __ldg(j.ids_in + s_job);
        bool published = false;
        auto publish = [&]() {
            if (j.router_w) {
                const float gate = warp_pick_softmax(sel_logit, j.k);
                if (lane == 0) stamp<kTrace>(j, 122);
                if (lane < j.k) {
                    ids_s[lane] = sel_id;
                    w_s[lane] = gate;
                    if (j.ids_out && c == 0) { j.ids_out[lane] = sel_id; j.w_out[lane] = gate; }
                }
            } else if (lane < j.k) {
                ids_s[lane] = j.ids_in[lane];
                w_s[lane] = j.w_in[lane];
            }
            __syncwarp();
            asm volatile("bar.arrive 3, 160;" ::: "memory");   // ids and gate weights known: release the epilogue
            if (lane == 0) stamp<kTrace>(j, 88);
            published = true;
        };
        if (tc::elect_one()) {
            tc::prefetch_tmap(&tm_gu);
            tc::prefetch_tmap(&tm_dn);
        }
        __syncwarp();
        const int mat = j.sf_by_slot ? s_job : e;
        int slot = 0;
        uint32_t ph = 0;
        bool ok = true;
        auto next_slot = [&]() {
            if (++slot == NS) {
                slot = 0;
                ph ^= 1u;
            }
        };
        const int nst = j.SPS + j.NP;
        for (int it = 0; it < nst && ok; ++it, next_slot()) {
            if (it >= NS) ok = __all_sync(kFull, tc::mbar_wait(&emptyB[slot], ph ^ 1u, j.err, 1));
            __syncwarp();
            if (ok && tc::elect_one()) {
                if (it < 32) stamp<kTrace>(j, 2 + it);
                uint8_t* dst = ring + slot * kSlot;
                if (it < j.SPS) {                      // gate/up: rows [256 rt, +256), K bytes [128 it, +128)
                    const int nkt = min(2, j.KT_gu - 2 * it);
                    tc::mbar_arrive_expect_tx(&fullB[slot], uint32_t(kGu + nkt * 1024));
                    tc::tma_load_3d(dst, &tm_gu, it * 128, rt * kRows, e, &fullB[slot]);
                    tc::bulk_g2s(dst + kGu, j.sf_gu + ((size_t(mat) * j.RT + rt) * j.KT_gu + 2 * it) * 1024,
                                 uint32_t(nkt * 1024), &fullB[slot]);
                } else if (j.dn_img) {                  // down, pre-packed: the stage's two boxes and scales at once
                    const int p = it - j.SPS;
                    tc::mbar_arrive_expect_tx(&fullB[slot], uint32_t(kSlot));
                    tc::bulk_g2s(dst, j.dn_img + ((size_t(e) * j.RT + rt) * j.NP + p) * kSlot, uint32_t(kSlot),
                                 &fullB[slot]);
                } else {                                // down: row boxes d0, d0 + 1, K bytes [64 rt, +64)
                    const int d0 = 2 * (it - j.SPS), nb = min(2, j.RD - d0);
                    tc::mbar_arrive_expect_tx(&fullB[slot], uint32_t(nb * (kDn + 1024)));
                    for (int b = 0; b < nb; ++b) {
                        tc::tma_load_3d(dst + b * kDn, &tm_dn, rt * 64, (d0 + b) * kRows, e, &fullB[slot]);
                        tc::bulk_g2s(dst + 2 * kDn + b * 1024,
                                     j.sf_dn + ((size_t(mat) * j.RT_dn + d0 + b) * j.KT_dn + rt) * 1024, 1024u,
                                     &fullB[slot]);
                    }
                }
            }
            __syncwarp();
            if (!published) publish();               // after the first stage's loads (measured best)
        }
        if (!published) publish();                   // no stage issued: the epilogue warps are released all the same
        // Then, per down stage p, once the epilogue warps have stored this CTA's partial sums of its rows: one
        // release of gbar[8 + p] (the CTAs that reduce those rows wait for the count to reach G). The epilogue warps
        // arrive on pDone[p] also when a wait gave up, so this never blocks them.
        // (The mbarrier wait acquires the epilogue threads' stores at CTA scope; the GPU-scope release that follows
        // is cumulative, so a CTA that acquires the count sees them.)
        if constexpr (kStageCounts) {
            for (int p = 0; p < j.NP; ++p) {
                __all_sync(kFull, tc::mbar_wait(&pDone[p], 0, j.err, 15));
                if (lane == 0) red_add_release(&j.gbar[8 + p], 1u);
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (one lane of warp 1)
        // One thread issues every tcgen05 operation; its cost per operation bounds the stage rate (the tensor pipe
        // itself needs ~55 cycles per M = 128, N = 8 MMA and ~47 per scale copy), so every descriptor is a base
        // computed once plus a byte offset / 16 (shared-memory addresses stay below 256 KB: the 14-bit start field
        // never carries), and the common stages are fully unrolled.
        if (tc::elect_one()) {
            bool ok = true;
            int slot = 0, f = 0;
            uint32_t ph = 0, so = 0;                 // ring slot, its phase, its byte offset
            auto advance = [&]() {
                so += kSlot;
                if (++slot == NS) {
                    slot = 0;
                    so = 0;
                    ph ^= 1u;
                }
                if (++f == NSF) f = 0;
            };
            const uint64_t dA128 = tc::desc_sw128(tc::smem_u32(ring)), dA64 = tc::desc_sw64(tc::smem_u32(ring));
            const uint64_t dBx = tc::desc_sw128(tc::smem_u32(xA)), dBd = tc::desc_sw128(tc::smem_u32(dA));
            const uint64_t dSFw = tc::desc_sf_chunk(tc::smem_u32(ring)), dSFx = tc::desc_sf_chunk8(tc::smem_u32(xSF));
            constexpr uint32_t id0 = tc::idesc_mxf4(128, NT, 0, 0), id2 = tc::idesc_mxf4(128, NT, 2, 2);
            const uint32_t colXs = tmem + j.L.colXs;
            // gate/up: per stage x's and the weights' scale chunks, then per unit of K = 64 one MMA per 128-row half
            for (int it = 0; it < j.SPS && ok; ++it, advance()) {
                const int nu = min(4, j.UK - 4 * it), nkt = (nu + 1) / 2;
                if (it == 0) ok = tc::mbar_wait(fullS, 0, j.err, 6);
                ok = ok && tc::mbar_wait(&fullB[slot], ph, j.err, 3);
                if (!ok) break;
                tc::tc_fence_after();
                if (it < 32) stamp<kTrace>(j, 34 + it);
                const uint32_t col = tmem + j.L.colW + 16u * uint32_t(f);
                const uint64_t aB = dA128 + (so >> 4), bB = dBx + uint64_t(it) * (kA >> 4),
                               sfw = dSFw + ((so + kGu) >> 4), sfx = dSFx + uint64_t(2 * it) * (kSF8 >> 4);
                const uint32_t cx = colXs + 8u * uint32_t(it);
                if (nu == 4) {
                    tc::tmem_cp_sf(cx, sfx);
                    tc::tmem_cp_sf(cx + 4, sfx + (kSF8 >> 4));
#pragma unroll
                    for (int x = 0; x < 4; ++x) tc::tmem_cp_sf(col + 4 * x, sfw + 32 * x);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint32_t sfb = (cx + 4u * (u >> 1)) | ((u & 1) ? (2u << 30) : 0u);
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            tc::mma_mxf4(tmem + kColGu + 8u * h, aB + 1024 * h + 2 * u, bB + 2 * u, (u & 1) ? id2 : id0,
                                         (col + 4u * (2u * (u >> 1) + h)) | ((u & 1) ? (2u << 30) : 0u), sfb,
                                         it > 0 || u > 0);
                    }
                } else {
                    for (int q = 0; q < nkt; ++q) tc::tmem_cp_sf(cx + 4 * q, sfx + q * (kSF8 >> 4));
                    for (int x = 0; x < 2 * nkt; ++x) tc::tmem_cp_sf(col + 4 * x, sfw + 32 * x);
                    for (int u = 0; u < nu; ++u) {
                        const uint32_t sfhi = (u & 1) ? (2u << 30) : 0u;
                        for (int h = 0; h < 2; ++h)
                            tc::mma_mxf4(tmem + kColGu + 8u * h, aB + 1024 * h + 2 * u, bB + 2 * u, (u & 1) ? id2 : id0,
                                         (col + 4u * (2u * (u >> 1) + h)) | sfhi, (cx + 4u * (u >> 1)) | sfhi,
                                         it > 0 || u > 0);
                    }
                }
                tc::mma_commit(&emptyB[slot]);
            }
            tc::mma_commit(accF);                    // (also when a wait gave up: the epilogue is not held)
            // down: the job's activations (down's operand, written by the epilogue warps) against every row box
            ok = ok && tc::mbar_wait(dReady, 0, j.err, 9);
            const uint32_t cds = tmem + j.L.colDs;
            if (ok) {
                tc::tc_fence_after();
                tc::tmem_cp_sf(cds, tc::desc_sf_chunk8(tc::smem_u32(dSF)));
            }
            // Down stage p: row boxes 2p, 2p + 1 (rows [512 p, +512)); its accumulators are committed to accD[p] so the
            // epilogue reads them out while the next stages stream.
            const int nu_dn = min(2, (j.I - 128 * rt) / 64);
            int p = 0;
            for (; p < j.NP && ok; ++p, advance()) {
                ok = tc::mbar_wait(&fullB[slot], ph, j.err, 3);
                if (!ok) break;
                tc::tc_fence_after();
                if (j.SPS + p < 32) stamp<kTrace>(j, 34 + j.SPS + p);
                const uint32_t col = tmem + j.L.colW + 16u * uint32_t(f);
                const uint64_t aB = dA64 + (so >> 4), sfw = dSFw + ((so + 2 * kDn) >> 4);
                const uint32_t acc = tmem + kColDn + 32u * uint32_t(p);
                const int nb = min(2, j.RD - 2 * p);
                if (nb == 2 && (2 * p + 1) * kRows + 128 < j.H && nu_dn == 2) {   // the common stage, unrolled
#pragma unroll
                    for (int x = 0; x < 4; ++x) tc::tmem_cp_sf(col + 4 * x, sfw + 32 * x);
#pragma unroll
                    for (int b = 0; b < 2; ++b)
#pragma unroll
                        for (int u = 0; u < 2; ++u)
#pragma unroll
                            for (int h = 0; h < 2; ++h)
                                tc::mma_mxf4(acc + 16u * b + 8u * h, aB + (b * kDn + h * 8192) / 16 + 2 * u, dBd + 2 * u,
                                             u ? id2 : id0, (col + 4u * (2 * b + h)) | (u ? (2u << 30) : 0u),
                                             cds | (u ? (2u << 30) : 0u), u > 0);
                } else {
                    for (int b = 0; b < nb; ++b) {
                        const int d = 2 * p + b, nh = d * kRows + 128 < j.H ? 2 : 1;
                        for (int h = 0; h < nh; ++h) tc::tmem_cp_sf(col + 4 * (2 * b + h), sfw + 64 * b + 32 * h);
                        for (int u = 0; u < nu_dn; ++u)
                            for (int h = 0; h < nh; ++h)
                                tc::mma_mxf4(acc + 16u * b + 8u * h, aB + (b * kDn + h * 8192) / 16 + 2 * u, dBd + 2 * u,
                                             u ? id2 : id0, (col + 4u * (2 * b + h)) | (u ? (2u << 30) : 0u),
                                             cds | (u ? (2u << 30) : 0u), u > 0);
                    }
                }
                tc::mma_commit(&emptyB[slot]);
                tc::mma_commit(&accD[p]);
            }
            for (; p < j.NP; ++p) tc::mma_commit(&accD[p]);   // a wait gave up: release the epilogue's waits
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue warps 2..5
        const int et = tid - 64;                     // 0..127
        const int quad = warp & 3;                   // the TMEM lane quadrant this warp may read
        // x's terms (gate/up's B operand) are made once per launch, spread over the CTAs: CTA c quantizes x's
        // 32-element blocks g = nc - 1 - c (mod nc) into global memory (plan 0: in phase 0; plans 1, 2: warp 2 from
        // h = RMSNorm(x) recomputed from global memory exactly as phase 0 computes it) and counts them on gbar[3];
        // warp 3 waits for all blocks and brings the image into shared memory with two bulk copies completing on
        // fullS, which the MMA warp awaits.
        auto x_exchange = [&]() {
            const int nb = j.H / 32;
            if (warp == 2) {
                unsigned mine = 0;
                for (int g = nc - 1 - c; g < nb; g += nc, ++mine) {
                    if constexpr (kXPlan != 0) {
                        const int idx = 32 * g + lane;
                        const float h = j.norm_w ? j.x[idx] * rn * __ldg(j.norm_w + idx) : j.x[idx];
                        quantize_block_digits_warp32(h, j.xq_img + size_t(g / 8) * kA, g % 8,
                                                     j.xq_sf + size_t(g / 4) * kSF8, g % 4, true);
                    }
                }
                __syncwarp();
                if (lane == 0 && mine) red_add_release(&j.gbar[3], mine);
            } else if (warp == 3 && lane == 0) {
                bool done = false;
                for (uint32_t w = 0; w < tc::kSpinLimit && !done; ++w) {
                    done = ld_acquire(&j.gbar[3]) >= unsigned(nb);
                    if (!done) __nanosleep(32);
                }
                if (done) {
                    asm volatile("fence.proxy.async.global;" ::: "memory");   // generic writes -> bulk-copy reads
                    const uint32_t b1 = uint32_t(j.SPS * kA), b2 = uint32_t(j.KT_gu * kSF8);
                    tc::mbar_arrive_expect_tx(fullS, b1 + b2);
                    tc::bulk_g2s(xA, j.xq_img, b1, fullS);
                    tc::bulk_g2s(xSF, j.xq_sf, b2, fullS);
                } else {
                    atomicCAS(j.err, 0, 13);
                    tc::mbar_arrive(fullS);             // gave up: release the MMA warp's wait
                }
                stamp<kTrace>(j, 80);
            }
        };
        if constexpr (kXPlan != 2) x_exchange();
        asm volatile("bar.sync 3, 160;" ::: "memory");   // expert ids known (warp 0)
        if constexpr (kXPlan == 2) x_exchange();
        const int e = ids_s[s_job];
        const float gate = w_s[s_job];
        // the first row group's weighted down biases and residual for the final reduction, read early
        float pre_b = 0.f, pre_x = 0.f;
        if (et < 32 && c * 32 + et < j.H) {
            const int row = c * 32 + et;
            for (int s2 = 0; s2 < j.k; ++s2) pre_b = fmaf(w_s[s2], __ldg(j.dn_bias + size_t(ids_s[s2]) * j.H + row), pre_b);
            pre_x = j.x_resid[row];
        }
        // gate/up: this thread's rows of the job's tile are r_h = 128 h + 32 quad + lane (h = 0, 1); an even row is a
        // glu row, the odd row after it (the next lane) its linear row.
        float bias[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int R = rt * kRows + 128 * h + 32 * quad + lane;
            bias[h] = R < 2 * j.I ? __ldg(j.gu_bias + size_t(e) * 2 * j.I + R) : 0.f;
        }
        bool ok = true;
        if (warp == 4) ok = __all_sync(kFull, tc::mbar_wait(accF, 0, j.err, 5));
        ok = epi_all(ok);
        if (ok) {
            tc::tc_fence_after();
            uint32_t v[16];
            tc::tmem_ld_32x32b_x16(tmem + (uint32_t(quad * 32) << 16) + kColGu, v);
            tc::tmem_ld_wait();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float y = term_sum(v + 8 * h) + bias[h];
                const float lin = __shfl_xor_sync(kFull, y, 1);
                const int a = 64 * h + 16 * quad + (lane >> 1);           // activation within the job
                if (!(lane & 1)) {
                    float act = 0.f;
                    if (rt * 128 + a < j.I) {
                        const float gv2 = fminf(y, j.limit);
                        const float lv = fminf(fmaxf(lin, -j.limit), j.limit);
                        act = __fdividef(gv2, 1.f + __expf(-j.alpha * gv2)) * (lv + 1.f) * gate;
                    }
                    act_s[a] = act;
                }
            }
        }
        tc::tc_fence_before();
        epi_sync();
        // the job's 4 blocks of 32 activations, one per epilogue warp, into down's operand (terms and their scales)
        if (ok) quantize_block_digits_warp32(act_s[32 * quad + lane], dA, quad, dSF, quad, true);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(dReady);
        if (et == 0) stamp<kTrace>(j, 131);
        // down: this thread's rows are 256 d + 128 h + 32 quad + lane; each accumulator's 8 term columns are added.
        // Stage p's four accumulators (row boxes 2p, 2p + 1) are read out as soon as its MMAs complete.
        {
            const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
            float* prow = j.part + size_t(c) * j.H * (kTagged ? 2 : 1);
            for (int p = 0; p < j.NP; ++p) {
                ok = __all_sync(kFull, ok && tc::mbar_wait(&accD[p], 0, j.err, 14));
                if (ok) {
                    tc::tc_fence_after();
                    uint32_t v[32];
                    tc::tmem_ld_32x32b_x32(lane_base + kColDn + 32u * p, v);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int d = 2 * p + i / 2, r0 = d * kRows + 128 * (i & 1) + 32 * quad;   // warp-uniform
                        if (d < j.RD && r0 < j.H) {
                            if constexpr (kTagged)
                                st_relaxed64(reinterpret_cast<unsigned long long*>(prow) + r0 + lane,
                                             (static_cast<unsigned long long>(ep) << 32) |
                                                 __float_as_uint(term_sum(v + 8 * i)));
                            else
                                prow[r0 + lane] = term_sum(v + 8 * i);
                        }
                    }
                }
                if constexpr (kStageCounts) tc::mbar_arrive(&pDone[p]);   // the stores above precede warp 0's count
                if (et == 0 && p < 8) stamp<kTrace>(j, 140 + p);
            }
        }
        ok = epi_all(ok);
        tc::tc_fence_before();
        if (et == 0) stamp<kTrace>(j, 133);
        if constexpr (!kStageCounts && !kTagged) {   // one count of the CTAs whose partial vectors are complete
            epi_sync();
            if (et == 0) red_add_release(&j.gbar[8], 1u);
        }
        if (ok) {
            // 32-row group g (g = c, c + G, ...), in down stage g / 16: once every CTA has stored its partial sums of
            // that stage (gbar[8 + g / 16] = G), thread et reads rows 32 g + 4 (et % 8) .. + 3 (one 16-byte load per
            // job) of jobs et / 8, et / 8 + 16, ..., all loads issued before any addition; the 16 job-lane sums are
            // then added in job-lane order with the weighted biases and the residual.
            const int rq = et & 7, jl = et >> 3;
            for (int g = c; g * 32 < j.H; g += nc) {
                if (!kTagged && et == 0) {
                    bool done = false;
                    for (uint32_t w = 0; w < tc::kSpinLimit && !done; ++w) {
                        done = ld_acquire(&j.gbar[kStageCounts ? 8 + g / 16 : 8]) >= unsigned(nc);
                        if (!done) __nanosleep(32);
                    }
                    if (!done) atomicCAS(j.err, 0, 8);
                    *flag_s = done ? 1 : 0;
                    if (g == c) stamp<kTrace>(j, 81);
                }
                if constexpr (kTagged) {
                    // the 4 rows of this thread from jobs jl, jl + 16, ...: every word is loaded, then the ones not
                    // yet tagged with this launch's epoch are loaded again (bounded) until all are current
                    const int row4 = g * 32 + 4 * rq;
                    constexpr int kMaxLoads = (160 + 15) / 16;
                    unsigned long long w[kMaxLoads][4];
                    const unsigned long long* base = reinterpret_cast<const unsigned long long*>(j.part) + row4;
                    const unsigned long long cur = static_cast<unsigned long long>(ep);
#pragma unroll
                    for (int i = 0; i < kMaxLoads; ++i)
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int jb = jl + 16 * i;
                            w[i][q] = (jb < nc && row4 < j.H) ? ld_relaxed64(base + size_t(jb) * j.H + q) : (cur << 32);
                        }
                    bool done = false;
                    for (uint32_t t = 0; t < tc::kSpinLimit; ++t) {
                        done = true;
#pragma unroll
                        for (int i = 0; i < kMaxLoads; ++i)
#pragma unroll
                            for (int q = 0; q < 4; ++q) done = done && (w[i][q] >> 32) == cur;
                        if (done) break;
                        __nanosleep(32);
#pragma unroll
                        for (int i = 0; i < kMaxLoads; ++i)
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if ((w[i][q] >> 32) != cur) w[i][q] = ld_relaxed64(base + size_t(jl + 16 * i) * j.H + q);
                    }
                    done = epi_all(done);
                    if (!done) {
                        if (et == 0) atomicCAS(j.err, 0, 8);
                        break;                       // (uniform) gave up: the error word says so
                    }
                    if (et == 0 && g == c) stamp<kTrace>(j, 81);
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < kMaxLoads; ++i) {
                        acc.x += __uint_as_float(unsigned(w[i][0]));
                        acc.y += __uint_as_float(unsigned(w[i][1]));
                        acc.z += __uint_as_float(unsigned(w[i][2]));
                        acc.w += __uint_as_float(unsigned(w[i][3]));
                    }
                    *reinterpret_cast<float4*>(red16 + jl * 32 + 4 * rq) = acc;
                } else {
                epi_sync();
                if (!*flag_s) break;                 // (uniform) gave up: the error word says so
                const int row4 = g * 32 + 4 * rq;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                if (row4 < j.H) {
                    constexpr int kMaxLoads = (160 + 15) / 16;
                    float4 vals[kMaxLoads];
#pragma unroll
                    for (int i = 0; i < kMaxLoads; ++i) {
                        const int jb = jl + 16 * i;
                        vals[i] = jb < nc ? __ldcg(reinterpret_cast<const float4*>(j.part + size_t(jb) * j.H + row4))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int i = 0; i < kMaxLoads; ++i) {
                        acc.x += vals[i].x;
                        acc.y += vals[i].y;
                        acc.z += vals[i].z;
                        acc.w += vals[i].w;
                    }
                }
                *reinterpret_cast<float4*>(red16 + jl * 32 + 4 * rq) = acc;
                }
                epi_sync();
                if (et == 0 && g == c) stamp<kTrace>(j, 134);
                const int row = g * 32 + et;
                if (et < 32 && row < j.H) {
                    float b = pre_b, xr = pre_x;
                    if (g != c) {
                        b = 0.f;
                        for (int s2 = 0; s2 < j.k; ++s2)
                            b = fmaf(w_s[s2], __ldg(j.dn_bias + size_t(ids_s[s2]) * j.H + row), b);
                        xr = j.x_resid[row];
                    }
                    float tot = red16[et];
#pragma unroll
                    for (int q = 1; q < 16; ++q) tot += red16[q * 32 + et];
                    j.x_resid[row] = xr + (tot + b);
                }
                epi_sync();
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        stamp<kTrace>(j, 82);
        __threadfence();
        if (atomicAdd(&j.gbar[1], 1u) == unsigned(nc - 1)) {   // last CTA out resets the counters
            j.gbar[3] = 0;
            for (int p = 0; p < j.NP; ++p) j.gbar[8 + p] = 0;
            j.gbar[4] = ep;                                  // the next launch's epoch is this + 1
            j.gbar[1] = 0;
        }
    }
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// Shared memory: NS ring slots, x's terms and scales, down's operand and its scales, the activations, the reduction
// partials, barriers and small per-CTA state. TMEM: accumulators in [0, 16 + 16 RD), x's scale chunks, down's scale
// chunk, then a ring of NSF weight-scale slots of 16 columns.
Layout make_layout(int NS, int SPS, int KT_gu, int RD) {
    Layout L{};
    L.NS = NS;
    L.colXs = kColDn + 16u * uint32_t(RD);
    L.colDs = L.colXs + 4u * uint32_t(KT_gu);
    L.colW = L.colDs + 4u;
    L.NSF = std::min(8, int(kTmemCols - L.colW) / 16);
    int o = 0;
    L.ring = o; o += NS * kSlot;
    L.xA = o; o += SPS * kA;
    L.xSF = o; o += (KT_gu * kSF8 + 1023) & ~1023;
    L.dA = o; o += kA;
    L.dSF = o; o += kSF8;
    L.act = o; o += 128 * 4;
    L.red4 = o; o += 16 * 32 * 4;
    L.bars = o; o += (2 * NS + 3 + 2 * kMaxPairs) * 8;
    o = (o + 15) & ~15;
    L.misc = o; o += 32 + 8 * 8 + 2 * kMaxK * 4 + 8 * 4 + 16;
    L.bytes = 1024 + o;
    return L;
}


// Pre-packed down stages: for expert e, job rt (activations [128 rt, +128)) and stage p (row boxes 2p, 2p + 1), the
// shared-memory image of the stage exactly as the TMA path lands it: box b (256 rows x 64 bytes, the 64-byte swizzle:
// 16-byte chunk ch of row r at chunk position ch ^ ((r / 2) % 4)) at b * 16 KB, then box b's two scale chunks (the
// layer's repacked chunks of row tile 2p + b, K chunk rt) at 32 KB + b * 1 KB. Rows past H and bytes past I / 2 are
// zero. One thread per 16 bytes of output.
__global__ void pack_down_jobs_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ sf_rep,
                                      uint8_t* __restrict__ out, int E, int H, int I, int RT, int NP, int RT_dn,
                                      int KT_dn) {
    const long long per_stage = kSlot / 16, total = (long long)E * RT * NP * per_stage;
    const int row_bytes = I / 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int w = int(i % per_stage);
        long long st = i / per_stage;
        const int p = int(st % NP);
        st /= NP;
        const int rt = int(st % RT);
        const int e = int(st / RT);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (w < 2 * kDn / 16) {                              // weight bytes
            const int b = w / (kDn / 16), o = (w % (kDn / 16)) * 16;
            const int r = o / 64, pos = (o % 64) / 16, ch = pos ^ ((r >> 1) & 3);
            const int row = (2 * p + b) * kRows + r, col = 64 * rt + 16 * ch;
            if (row < H && col < row_bytes)
                v = *reinterpret_cast<const uint4*>(blocks + ((size_t(e) * H + row) * row_bytes + col));
        } else {                                             // scale chunks
            const int o = (w - 2 * kDn / 16) * 16, b = o / 1024, d = 2 * p + b;
            if (d < RT_dn)
                v = *reinterpret_cast<const uint4*>(sf_rep + ((size_t(e) * RT_dn + d) * KT_dn + rt) * 1024 + o % 1024);
        }
        reinterpret_cast<uint4*>(out)[i] = v;
    }
}

}  // namespace rj

// ---------------------------------------------------------------------------------------------------- host API
int decode_rows_jobs(int k, int I) { return k * ((2 * I + rj::kRows - 1) / rj::kRows); }

size_t down_jobs_bytes(int E, int H, int I) {
    const int RT = (2 * I + rj::kRows - 1) / rj::kRows, RD = (H + rj::kRows - 1) / rj::kRows;
    return size_t(E) * RT * ((RD + 1) / 2) * rj::kSlot;
}

void launch_pack_down_jobs(const uint8_t* dn_blocks, const uint8_t* sf_dn_repacked, uint8_t* out, int E, int H, int I,
                           cudaStream_t s) {
    require(H % 64 == 0 && I % 64 == 0, "pack_down_jobs: H and I must be multiples of 64");
    const int RT = (2 * I + rj::kRows - 1) / rj::kRows, RD = (H + rj::kRows - 1) / rj::kRows;
    const int RT_dn = (H + kDecodeTileRows - 1) / kDecodeTileRows, KT_dn = (I / 32 + 3) / 4;
    const long long n16 = (long long)down_jobs_bytes(E, H, I) / 16;
    const int grid = int(std::min<long long>((n16 + 255) / 256, num_sms() * 16LL));
    rj::pack_down_jobs_kernel<<<std::max(1, grid), 256, 0, s>>>(dn_blocks, sf_dn_repacked, out, E, H, I, RT,
                                                                (RD + 1) / 2, RT_dn, KT_dn);
    check_launch("pack_down_jobs");
}

bool decode_rows_ok(int k, int H, int I, int E_router) {
    const int G = decode_rows_jobs(k, I);
    if (k < 1 || k > rj::kMaxK || H % 64 || I % 64 || H > 4 * rj::kThreads * rj::kMaxX4) return false;
    if (G > num_sms() || (E_router > 0 && G < E_router) || G > 160) return false;
    const int SPS = (H + 255) / 256, KT = (H + 127) / 128, RD = (H + 255) / 256;
    if ((RD + 1) / 2 > rj::kMaxPairs || SPS > rj::kMaxStages) return false;
    const rj::Layout L = rj::make_layout(2, SPS, KT, RD);
    return L.NSF >= 2 && L.bytes <= 227 * 1024;
}

namespace {
void set_rows_smem(int bytes) {
    static std::mutex mu;
    static std::map<int, int> current;                       // per device
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (bytes > current[dev]) {
        require(bytes <= 227 * 1024, "moe (rows): shared-memory plan exceeds 227 KB");
        GPT_CHECK(cudaFuncSetAttribute(rj::moe_rows_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        GPT_CHECK(cudaFuncSetAttribute(rj::moe_rows_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        current[dev] = bytes;
    }
}
}  // namespace

void launch_moe_decode_rows(const DecodeTcArgs& a, cudaStream_t s) {
    using namespace rj;
    require(a.tmap_dn64 != nullptr, "moe (rows): needs the 64-byte-box map of the down blocks");
    require(decode_rows_ok(a.k, a.H, a.I, a.router_w ? a.E : 0), "moe (rows): shape not supported");
    const DecodeTcLayout W = decode_tc_layout(a.k, a.H, a.I);
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    Job j{};
    j.k = a.k;
    j.H = a.H;
    j.I = a.I;
    j.E = a.E;
    j.RT = (2 * a.I + kRows - 1) / kRows;
    j.G = decode_rows_jobs(a.k, a.I);
    j.SPS = (a.H + 255) / 256;
    j.UK = a.H / 64;
    j.KT_gu = (a.H + 127) / 128;
    j.RD = (a.H + kRows - 1) / kRows;
    j.NP = (j.RD + 1) / 2;
    j.RT_dn = W.RT_dn;
    j.KT_dn = W.KT_dn;
    j.router_w = static_cast<const __nv_bfloat16*>(a.router_w);
    j.router_b = a.router_b;
    j.norm_w = a.norm_w;
    j.eps = a.eps;
    j.x = a.x;
    j.ids_in = a.ids;
    j.w_in = a.weights;
    j.ids_out = a.ids_out;
    j.w_out = a.w_out;
    j.sf_gu = a.sfa_gu;
    j.sf_dn = a.sfa_dn;
    j.sf_by_slot = a.sfa_by_slot;
    j.gu_bias = a.gu_bias;
    j.dn_bias = a.dn_bias;
    j.alpha = a.alpha;
    j.limit = a.limit;
    j.part = reinterpret_cast<float*>(ws + W.off_rows);
#ifdef GPTOSS_NO_DOWN_IMAGE
    j.dn_img = nullptr;                     // (A/B builds: the TMA path of the down stages)
#else
    j.dn_img = a.dn_img;
#endif
    j.xq_img = ws + W.off_xq_img;
    j.xq_sf = ws + W.off_xq_sf;
    j.x_resid = a.x_resid;
    j.err = reinterpret_cast<int*>(ws + W.off_err);
    j.gbar = reinterpret_cast<unsigned*>(ws + W.off_err + 256);
    j.logit_words = reinterpret_cast<unsigned long long*>(ws + W.off_logits);
    j.trace = a.trace;
    require(j.RT == W.RT_gu && size_t(j.G) * a.H * 8 <= W.rows_bytes, "moe (rows): workspace layout mismatch");
    int NS = 6;
    Layout L = make_layout(NS, j.SPS, j.KT_gu, j.RD);
    while (L.bytes > 227 * 1024 && NS > 2) L = make_layout(--NS, j.SPS, j.KT_gu, j.RD);
    require(L.bytes <= 227 * 1024 && L.NSF >= 2, "moe (rows): shapes too large for one CTA");
    j.L = L;
    set_rows_smem(L.bytes);

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(j.G);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = size_t(L.bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    // As the stream-K kernel: programmatic dependent launch unless this runtime refuses it with a cooperative launch.
    static std::atomic<int> pdl_ok[64] = {};                 // 0 unknown, 1 accepted, -1 refused
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    require(dev >= 0 && dev < 64, "moe (rows): device ordinal out of range");
    cfg.numAttrs = pdl_ok[dev].load() >= 0 ? 2 : 1;
    auto kernel = a.trace ? moe_rows_kernel<true> : moe_rows_kernel<false>;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, *a.tmap_gu, *a.tmap_dn64, j);
    if (e != cudaSuccess && cfg.numAttrs == 2 && pdl_ok[dev].load() == 0) {
        (void)cudaGetLastError();
        pdl_ok[dev].store(-1);
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kernel, *a.tmap_gu, *a.tmap_dn64, j);
    } else if (e == cudaSuccess && cfg.numAttrs == 2) {
        pdl_ok[dev].store(1);
    }
    GPT_CHECK(e);
    check_launch("moe (tensor cores, row jobs)");
}

}  // namespace gpt
