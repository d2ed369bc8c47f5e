// Tensor-core decode MoE for one token: one persistent, cooperatively launched kernel per MoE layer.
//
// Operands. B = expert weights straight from the checkpoint layout: TMA boxes of 256 rows x 128 bytes of K (256
// e2m1 values) with the 128-byte swizzle, one 32 KB box per pipeline stage; their E8M0 scales repacked once into
// 512-byte tcgen05 chunks ([tile][K chunk][half]). A = the activation vector split into NT = 8 e2m1 terms, each
// with its own E8M0 scale per 32 elements (the integer digit split of terms.cuh: the vector equals their sum to
// 2^-21 of each block's scale, below 2^-22 of the block's maximum): 8 rows of
// 128 bytes per 256 values of K, read as M = 128 rows through a descriptor whose 8-row groups all start at the same
// address. One tcgen05.mma kind::mxf4 (M = 128, N = 256, K = 64) therefore consumes 8 KB of weights; the tensor core
// performs the MXFP4 dequantization, accumulator rows 0..7 hold the 8 terms' dot products and the epilogue adds them.
//
// Phases of every CTA (all 148 resident, one per SM):
//   0. RMSNorm of x (every CTA, in registers); router CTA c < E computes logit c over all of K (fp64, exact products
//      summed in a fixed order) and publishes it; warp 0 of every CTA reads the E logits, takes the top k (ties to
//      the lower id) and the softmax over the k, so all CTAs pick the same experts. The last CTAs quantize x's
//      32-value blocks into its terms in global memory (gate/up's A operand), counted on a grid-wide word.
//   1. Gate/up stream-K GEMV; the CTA finishing a 256-row tile applies bias, the clamped SwiGLU (rows 2j glu, 2j+1
//      linear) and the slot's gate weight, and writes the tile's 128 activations as down's A terms (global memory).
//   2. Down stream-K GEMV over K' = k * I: the k experts' rows form one long GEMV because A carries the gate
//      weights; the CTA finishing a tile adds sum_slot w b2 and the residual.
// Roles: warp 0 streams the weights (TMA, gate/up and down through one ring, so down's weights arrive while the grid
// finishes gate/up); warp 1 issues the tcgen05 operations (per stage: the activation scales, the weight scales into
// a ring of TMEM columns, 4 MMAs, commits); warps 2-5 copy x's terms (written to global memory by all CTAs in phase 0)
// into shared memory, run the tile epilogues (each reads a quarter of the accumulator's columns from its own TMEM lane
// quadrant) and, after the grid barrier (all gate/up epilogues done), load down's A terms. A tile split between CTAs
// is finished by one designated contributor, which adds the others' published partial sums in a fixed order. Every
// wait is bounded: the launch is cooperative, so all CTAs are resident and every barrier completes; a timeout records
// an error instead of hanging. The per-CTA stage lists are computed on the host once per shape (stream-K partition,
// segment boundaries and which CTAs share each tile) and read by each CTA at start.
#include <algorithm>
#include <atomic>
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
constexpr int NT = 8;                         // activation terms (A rows)
constexpr int kRows = kDecodeTileRows;        // weight rows per tile (the MMA's N)
constexpr int kThreads = 192;                 // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kB = kRows * 128;               // one weight stage: 256 rows x 128 bytes of K (32 KB)
constexpr int kA = NT * 128;                  // one activation stage: 8 terms x 128 bytes (1 KB)
constexpr int kSFB = 2 * 1024;                // a stage's weight scales: 2 K chunks x 2 halves x 512 bytes
constexpr int kSlot = kB + kSFB;              // ring slot: the weight box, then its scales
constexpr int kSF8 = 128;                     // an activation scale chunk: rows 0-7 of a 512-byte chunk
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColX = kRows;             // accumulator in columns [0, 256); x's scale chunks from 256 on
constexpr int kTraceSlots = 160;
constexpr int kMaxK = 8;
constexpr int kMaxX4 = 4;                     // x is held as kMaxX4 float4 per thread: H <= 4 * kThreads * kMaxX4
constexpr int kMaxGrid = 160;                 // CTAs (SMs) the stage tables and traces are sized for

struct Layout {
    int NS, NSF, cap;                         // weight ring depth, TMEM scale ring depth, stage-list capacity
    uint32_t colSFB, colDSF;                  // TMEM columns of the weight-scale ring and of down's A-scale ring
    int ring, xA, xSF, dA, dSF, red, bars, misc, bytes;
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
    const uint8_t* sf_gu;                     // [mat][RT][KT][2][512]
    const uint8_t* sf_dn;
    int sf_by_slot;                           // mat = slot (1) or expert id (0)
    const float* gu_bias;                     // [E][2I]
    const float* dn_bias;                     // [E][H]
    float alpha, limit;
    Part gu, dn;
    const Stage* stab;                        // host-built stage lists of all CTAs
    const int* shdr;                          // [grid][4]: first entry, entries, gate/up entries
    uint8_t* aq_img;                          // down's A terms [k][SPS_dn][NT*128]
    uint8_t* aq_sf;                           // down's A scales [k][KT_dn][128]
    float* x_resid;
    unsigned* gbar;                           // [5]: gate/up done, exits, router partials published, x blocks written,
                                              // the last launch's epoch
    unsigned long long* logit_words;          // [32][2] router logit e as (epoch << 32) | high and low 32 bits
    uint8_t* xq_img;                          // x's A terms [SPS_gu][NT*128] (quantized by the last CTAs in phase 0)
    uint8_t* xq_sf;                           // their scales [KT_gu][128] (rows 0-7 of each chunk)
    int* err;
    long long* trace;                         // optional [grid][kTraceSlots] clock64 stamps
    Layout L;
};

// Trace slots per CTA: 0 start, 123 previous layer complete, 124 sum of squares, 84 h, 85 router logit published,
// 126 x blocks quantized, 1 phase 0 done, 120 logits read, 121 top k, 122 softmax, 127 ids in shared memory, 88 ids
// released to the other warps, 89 producer start, 2+i producer issues stage i, 80 x's terms in shared memory, 78
// epilogue warps see the ids, 34+i MMA warp sees stage i landed, 96+i its MMAs issued, 66+g epilogue read segment g,
// 132+g its split partial sums added, 140+g its down terms written, 131 gate/up done (counted on the grid barrier),
// 81 grid barrier passed, 83 down's A terms loaded, 82 end.
// Tracing is a compile-time choice: the untraced kernel carries no stamp code at all (branches over it in the
// single-thread issue loops measurably slowed them).
template <bool kTrace>
__device__ __forceinline__ void stamp(const Job& j, int slot) {
    if constexpr (kTrace) j.trace[size_t(blockIdx.x) * kTraceSlots + slot] = clock64();
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

// Atomic add with acquire-release semantics at GPU scope: the CTA's stores before a bar.sync are released with it,
// and the returning thread acquires the other contributors' (other threads read after the next bar.sync).
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Split-tile partial sums travel as one 64-bit word each, (launch epoch << 32) | fp32 bits: a single-copy-atomic
// relaxed store and load, so a word read with the current epoch carries the current value and no fence or counter is
// needed between the contributor's store and the finalizer's read.
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long tag_sum(float v, unsigned ep) {
    return (static_cast<unsigned long long>(ep) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void red_add_release(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The launch epoch that follows prev, skipping 0 (the tag of a zero-filled partial-sum word, which must never read
// as current).
__host__ __device__ __forceinline__ unsigned next_epoch(unsigned prev) { return prev == 0xFFFFFFFFu ? 1u : prev + 1u; }

__device__ __forceinline__ double bf16lo(uint32_t w) { return double(__uint_as_float(w << 16)); }
__device__ __forceinline__ double bf16hi(uint32_t w) { return double(__uint_as_float(w & 0xffff0000u)); }

// Warp reads 32 lanes (its quadrant) x 32 consecutive fp32 columns: thread t gets lane (quadrant * 32 + t).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1) moe_fused_kernel(const __grid_constant__ CUtensorMap tm_gu,
                                                                const __grid_constant__ CUtensorMap tm_dn,
                                                                const __grid_constant__ Job j) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NS = j.L.NS, NSF = j.L.NSF, cap = j.L.cap;
    uint8_t* ring = smem + j.L.ring;          // [NS][kSlot] weight stages and their scales
    uint8_t* xA = smem + j.L.xA;              // [SPS_gu][kA] x's terms
    uint8_t* xSF = smem + j.L.xSF;            // [KT_gu][kSF8] x's scales
    uint8_t* dA = smem + j.L.dA;              // [cap_dn][kA] down's A terms
    uint8_t* dSF = smem + j.L.dSF;            // [cap_dn][2][kSF8] their scales
    float* red_s = reinterpret_cast<float*>(smem + j.L.red);                // [NT][kRows] accumulator rows 0..7
    uint64_t* fullB = reinterpret_cast<uint64_t*>(smem + j.L.bars);        // [NS] weight stage landed
    uint64_t* emptyB = fullB + NS;            // [NS] weight stage consumed by the MMAs
    uint64_t* fullS = emptyB + NS;            // [0] x's terms in shared memory
    uint64_t* accF = fullS + 2;               // accumulator complete (one phase per segment)
    uint64_t* accE = accF + 1;                // accumulator read out (one phase per segment)
    uint64_t* fullD = accE + 1;               // [cap] down stage's A terms and scales loaded
    uint32_t* holder = reinterpret_cast<uint32_t*>(smem + j.L.misc);
    double* red = reinterpret_cast<double*>(holder + 8);     // [6][32] router sums
    int* ids_s = reinterpret_cast<int*>(red + 7 * 32);       // [8]
    float* w_s = reinterpret_cast<float*>(ids_s + kMaxK);    // [8]
    float* aval = w_s + kMaxK;                               // [kRows / 2] phase 0's per-warp sums of squares
    Stage* stages = reinterpret_cast<Stage*>(aval + kRows / 2);   // [cap]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, nc = gridDim.x;
    if (tid == 0) stamp<kTrace>(j, 0);
    // Router CTAs: CTA c < E computes expert c's logit over all of K. Thread t holds the same elements of the router
    // row as of x (float4 chunks t, t + kThreads, ...), widened to fp64 before the previous layer has finished (they
    // do not depend on it).
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
    // the norm weights and x, kept in registers: thread t holds float4 chunks t, t + kThreads, ...
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
        tc::mbar_init(&fullS[0], 128);                       // one arrival per epilogue thread after its copies
        tc::mbar_init(accF, 1);
        tc::mbar_init(accE, 4);                              // one arrival per epilogue warp after its TMEM reads
        for (int i = 0; i < cap; ++i) tc::mbar_init(&fullD[i], 1);
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
    if (warp == 1) {
        tc::tmem_alloc(holder, kTmemCols);
        tc::tmem_relinquish();
    }
    // Everything above reads only what no earlier kernel writes (stage table, weights, biases). With programmatic
    // dependent launch the next layer's kernel is released now and this one waits here for the previous layer's
    // kernel to finish (x, the residual stream, and the shared workspace are written there).
    pdl_launch_dependents();
    pdl_wait();
    // This launch's epoch (tags its split-tile partial sums): one more than the previous launch's, which that
    // launch's last CTA out stored; never 0, the value of a zeroed word: after 2^32 - 1 launches the count wraps to 1.
    const unsigned ep = next_epoch(__ldcg(&j.gbar[4]));
    if (tid == 0 && s_n > cap) atomicCAS(j.err, 0, 100);    // host sized the stage list too small
    if (tid == 0) stamp<kTrace>(j, 123);
#pragma unroll
    for (int r = 0; r < kMaxX4; ++r) {
        const int i = (tid + r * kThreads) * 4;
        xv[r] = i < j.H ? *reinterpret_cast<const float4*>(j.x + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // ---------------------------------------------------------------- phase 0: RMSNorm, router, x's terms
    // Two publications between CTAs, made at the same time and awaited by different warps: router CTA c publishes
    // logit c (fp64, exact bf16 x fp32 products summed in a fixed order, so every CTA reads the same values and
    // picks the same experts) as two epoch-tagged 64-bit words that warp 0 of every CTA polls directly; and the 32-
    // element blocks of x's 8 activation terms (gate/up's A operand) are quantized by the last CTAs, one block each,
    // into global memory, counted on gbar[3], which the epilogue warps await and copy into shared memory. h =
    // RMSNorm(x) and the router products stay in registers.
    {
        const int H = j.H;
        float ss = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxX4; ++r)
            ss = fmaf(xv[r].x, xv[r].x, fmaf(xv[r].y, xv[r].y, fmaf(xv[r].z, xv[r].z, fmaf(xv[r].w, xv[r].w, ss))));
        ss = warp_sum(ss);
        if (lane == 0) aval[warp] = ss;
        if (tid == 0) stamp<kTrace>(j, 124);
        __syncthreads();
        float rn = 1.f;
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
        if (tid == 0) stamp<kTrace>(j, 84);
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
                st_relaxed64(j.logit_words + 2 * c + 1, (static_cast<unsigned long long>(ep) << 32) | (bits & 0xFFFFFFFFull));
                stamp<kTrace>(j, 85);
            }
        }
        // x's blocks: block g is quantized by CTA nc - 1 - (g % nc), in the 8 lanes whose registers hold it (float4
        // round r = g / (kThreads / 8), threads 8 (g % (kThreads / 8)) ..+7), which write its terms into global memory.
        // The CTA counts its blocks on gbar[3] with one release after the barrier that ends phase 0 (an epilogue
        // thread, below): a release per block here would hold that barrier, and warp 0's wait for the expert ids
        // behind it, until the stores were acknowledged.
        {
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
                        // the scale byte goes to all four lane-quadrant copies of the term's row (lane sub8 < 4:
                        // copy sub8)
                        if (sub8 < 4) sf[t * 16 + sub8 * 4] = uint8_t(scale);
                    });
                }
            }
        }
        if (tid == 0) stamp<kTrace>(j, 126);
    }
    tc::fence_proxy_async_smem();             // phase 0's generic shared-memory accesses before the TMA's writes
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (tid == 0) stamp<kTrace>(j, 1);
    const uint32_t tmem = *holder;

    auto part_of = [&](const Stage& st) -> const Part& { return st.mode == sk::kGateUp ? j.gu : j.dn; };

    if (warp == 0) {
        // ---------------------------------------------------------------- expert ids, then the TMA producer
        if (j.router_w) {
            // lane e polls logit e's two words until both carry this launch's epoch (bounded)
            unsigned long long w0 = 0, w1 = 0;
            bool done = false;
            for (uint32_t i = 0; i < tc::kSpinLimit && !done; ++i) {
                if (lane < j.E) {
                    w0 = ld_relaxed64(j.logit_words + 2 * lane);
                    w1 = ld_relaxed64(j.logit_words + 2 * lane + 1);
                }
                done = __all_sync(kFull, lane >= j.E || (unsigned(w0 >> 32) == ep && unsigned(w1 >> 32) == ep));
                if (!done) __nanosleep(20);
            }
            if (!done && lane == 0) atomicCAS(j.err, 0, 10);
            const double v = __longlong_as_double(static_cast<long long>((w0 << 32) | (w1 & 0xFFFFFFFFull)));
            if (lane == 0) stamp<kTrace>(j, 120);
            int sel_id = 0;
            double sel_logit = 0.0;
            warp_topk_logits(v, lane < j.E, j.k, sel_id, sel_logit);
            if (lane == 0) stamp<kTrace>(j, 121);
            const float gate = warp_pick_softmax(sel_logit, j.k);
            if (lane == 0) stamp<kTrace>(j, 122);
            if (lane < j.k) {
                ids_s[lane] = sel_id;
                w_s[lane] = gate;
                if (j.ids_out && c == 0) { j.ids_out[lane] = sel_id; j.w_out[lane] = gate; }
            }
            if (lane == 0) stamp<kTrace>(j, 127);
        } else if (lane < j.k) {
            ids_s[lane] = j.ids_in[lane];
            w_s[lane] = j.w_in[lane];
        }
        // ids and gate weights are in shared memory: release the MMA and epilogue warps, which sleep in named
        // barrier 3 meanwhile (a spinning wait there would compete with this warp's shuffles and reductions)
        __syncwarp();
        asm volatile("bar.arrive 3, %0;" ::"n"(kThreads) : "memory");
        if (lane == 0) stamp<kTrace>(j, 88);
        if (tc::elect_one()) {
            stamp<kTrace>(j, 89);
            tc::prefetch_tmap(&tm_gu);
            tc::prefetch_tmap(&tm_dn);
        }
        __syncwarp();
        // Ring position of stage it: slot = it % NS, phase = (it / NS) & 1, kept as counters (a division by the
        // run-time ring depth per stage is measurable on a single issuing thread). Stage it - NS, which used the slot
        // in the previous phase, must have released it.
        int slot = 0;
        uint32_t ph = 0;
        auto next_slot = [&]() {
            if (++slot == NS) {
                slot = 0;
                ph ^= 1u;
            }
        };
        auto wait_slot = [&]() -> bool {
            return __all_sync(kFull, tc::mbar_wait(&emptyB[slot], ph ^ 1u, j.err, 1));
        };
        // The tensor map is a compile-time operand of each loop: selecting it at run time made every TMA issue wait
        // for a descriptor fetch.
        bool ok = true;
        // Each stage: the weight box (TMA) and its scale chunks (one bulk copy of nkt KB, contiguous in the repacked
        // layout) complete on the slot's barrier.
        auto scales_of = [&](const Stage& st, const Part& p, const uint8_t* base, int rt) {
            const int mat = j.sf_by_slot ? int(st.s) : ids_s[st.s];
            return base + ((size_t(mat) * p.RT + rt) * p.KT + st.ku0 / 2) * 1024;
        };
        for (int it = 0; it < ngu && ok; ++it, next_slot()) {
            if (it >= NS) ok = wait_slot();
            if (ok && tc::elect_one()) {
                if (it < 32) stamp<kTrace>(j, 2 + it);
                const Stage& st = stages[it];
                const int rt = st.tile - st.s * j.gu.RT;     // gate/up tiles are numbered slot * RT + row tile
                const uint32_t sb = uint32_t(sk::nkt_of(st)) * 1024u;
                uint8_t* dst = ring + slot * kSlot;
                tc::mbar_arrive_expect_tx(&fullB[slot], kB + sb);
                tc::tma_load_3d(dst, &tm_gu, (st.ku0 / 4) * 128, rt * kRows, ids_s[st.s], &fullB[slot]);
                tc::bulk_g2s(dst + kB, scales_of(st, j.gu, j.sf_gu, rt), sb, &fullB[slot]);
            }
            __syncwarp();
        }
        for (int it = ngu; it < nst && ok; ++it, next_slot()) {
            if (it >= NS) ok = wait_slot();
            if (ok && tc::elect_one()) {
                if (it < 32) stamp<kTrace>(j, 2 + it);
                const Stage& st = stages[it];
                const uint32_t sb = uint32_t(sk::nkt_of(st)) * 1024u;
                uint8_t* dst = ring + slot * kSlot;
                tc::mbar_arrive_expect_tx(&fullB[slot], kB + sb);
                tc::tma_load_3d(dst, &tm_dn, (st.ku0 / 4) * 128, st.tile * kRows, ids_s[st.s], &fullB[slot]);
                tc::bulk_g2s(dst + kB, scales_of(st, j.dn, j.sf_dn, st.tile), sb, &fullB[slot]);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (one lane of warp 1)
        // One fixed lane issues every tcgen05 operation, so scale copies and MMAs execute in issue order. Per stage:
        // the activation scales (x's chunk the first time a stage needs it, or down's chunks into the A-scale ring
        // slot it % NSF) before the stage's data is waited for, then the weight scales (4 chunks from the ring slot:
        // 2 K chunks x 2 row halves, 8 TMEM columns per K chunk) into weight-scale slot it % NSF, up to 4 MMAs and
        // one commit.
        asm volatile("bar.sync 3, %0;" ::"n"(kThreads) : "memory");   // expert ids known (warp 0)
        if (tc::elect_one()) {
            bool ok = nst == 0 || tc::mbar_wait(&fullS[0], 0, j.err, 6);
            // Gate/up stages: x's scale chunks (first use of each K chunk), the weight scales, 4 MMAs, commits.
            unsigned long long x_sf_done = 0;                // x's scale chunks in TMEM
            // ring slot, its phase and the TMEM scale slot of stage it (it % NS, (it / NS) & 1, it % NSF) as counters
            int slot = 0, f = 0;
            uint32_t ph = 0;
            auto advance = [&]() {
                if (++slot == NS) {
                    slot = 0;
                    ph ^= 1u;
                }
                if (++f == NSF) f = 0;
            };
            // A stage's MMAs. Stages start on 4-unit boundaries, so unit u uses scale id 2 (u & 1) of K chunk u / 2;
            // sfa / sfb are the TMEM columns of the stage's first activation / weight scale chunk. A full stage (the
            // common case) is issued fully unrolled.
            auto issue_mmas = [&](const uint8_t* ast, const uint8_t* wslot, uint32_t sfa, uint32_t sfb, int nu,
                                  bool first) {
                auto one = [&](int u) {
                    const uint32_t sf_id = 2u * uint32_t(u & 1), q = uint32_t(u >> 1);
                    tc::mma_mxf4(tmem, tc::desc_sw128_rows8(tc::smem_u32(ast + u * 32)),
                                 tc::desc_sw128(tc::smem_u32(wslot + u * 32)), tc::idesc_mxf4(128, kRows, sf_id, sf_id),
                                 (sfa + 4 * q) | (sf_id << 30), (sfb + 8 * q) | (sf_id << 30), !(first && u == 0));
                };
                if (nu == 4) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) one(u);
                } else {
                    for (int u = 0; u < nu; ++u) one(u);
                }
            };
            // the weight scales of a stage (2 chunks of a full stage unrolled)
            auto copy_wsf = [&](const uint8_t* wslot, int nkt) {
                const uint32_t col = tmem + j.L.colSFB + 16 * f;
                if (nkt == 2) {
#pragma unroll
                    for (int x = 0; x < 4; ++x)
                        tc::tmem_cp_sf(col + 4 * x, tc::desc_sf_chunk(tc::smem_u32(wslot + kB + x * 512)));
                } else {
                    for (int x = 0; x < 2 * nkt; ++x)
                        tc::tmem_cp_sf(col + 4 * x, tc::desc_sf_chunk(tc::smem_u32(wslot + kB + x * 512)));
                }
            };
            for (int it = 0; it < ngu && ok; ++it, advance()) {
                const Stage& st = stages[it];
                const int kt0 = st.ku0 / 2, nkt = sk::nkt_of(st);
                tc::tc_fence_after();
                for (int q = 0; q < nkt; ++q) {
                    const int kt = kt0 + q;
                    if (!((x_sf_done >> kt) & 1ull)) {
                        tc::tmem_cp_sf(tmem + kColX + 4 * kt, tc::desc_sf_chunk8(tc::smem_u32(xSF + kt * kSF8)));
                        x_sf_done |= 1ull << kt;
                    }
                }
                // one accumulator: a segment's first MMA waits until the previous segment has been read out
                if (st.first && st.seg >= 1) ok = tc::mbar_wait(accE, uint32_t(st.seg - 1) & 1u, j.err, 2);
                ok = ok && tc::mbar_wait(&fullB[slot], ph, j.err, 3);
                if (!ok) break;
                tc::tc_fence_after();
                if (it < 32) stamp<kTrace>(j, 34 + it);
                const uint8_t* wslot = ring + slot * kSlot;
                copy_wsf(wslot, nkt);
                issue_mmas(xA + (st.ku0 / 4) * kA, wslot, tmem + kColX + 4 * kt0, tmem + j.L.colSFB + 16 * f, st.nu,
                           st.first);
                tc::mma_commit(&emptyB[slot]);
                if (st.last) tc::mma_commit(accF);
                if (it < 32) stamp<kTrace>(j, 96 + it);
            }
            // Down stages: wait for the stage's A terms, their scales and the weight scales, 4 MMAs, commits.
            for (int it = ngu; it < nst && ok; ++it, advance()) {
                const Stage& st = stages[it];
                const int d = it - ngu;
                const int nkt = sk::nkt_of(st);
                ok = tc::mbar_wait(&fullD[d], 0, j.err, 9);
                if (!ok) break;
                tc::tc_fence_after();
                for (int q = 0; q < nkt; ++q)
                    tc::tmem_cp_sf(tmem + j.L.colDSF + 8 * f + 4 * q,
                                   tc::desc_sf_chunk8(tc::smem_u32(dSF + d * 2 * kSF8 + q * kSF8)));
                if (st.first && st.seg >= 1) ok = tc::mbar_wait(accE, uint32_t(st.seg - 1) & 1u, j.err, 2);
                ok = ok && tc::mbar_wait(&fullB[slot], ph, j.err, 3);
                if (!ok) break;
                tc::tc_fence_after();
                if (it < 32) stamp<kTrace>(j, 34 + it);
                const uint8_t* wslot = ring + slot * kSlot;
                copy_wsf(wslot, nkt);
                issue_mmas(dA + d * kA, wslot, tmem + j.L.colDSF + 8 * f, tmem + j.L.colSFB + 16 * f, st.nu, st.first);
                tc::mma_commit(&emptyB[slot]);
                if (st.last) tc::mma_commit(accF);
                if (it < 32) stamp<kTrace>(j, 96 + it);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue warps 2..5
        const int et = tid - 64;                    // 0..127

        // x's terms and scales (quantized by the last CTAs in phase 0, counted on gbar[3]), with asynchronous 16-byte
        // copies; then the expert ids from warp 0
        {
            if (et == 0) {
                // this CTA's x blocks (every thread's stores precede the phase-0 barrier): nc - 1 - c = g % nc
                const int nb = j.H / 32, r0 = nc - 1 - c;
                if (r0 < nb) red_add_release(&j.gbar[3], unsigned((nb - r0 + nc - 1) / nc));
                bool done = false;
                for (uint32_t w = 0; w < tc::kSpinLimit && !done; ++w) {
                    done = ld_acquire(&j.gbar[3]) >= unsigned(j.H / 32);
                    if (!done) __nanosleep(32);
                }
                if (!done) atomicCAS(j.err, 0, 13);
            }
            epi_sync();
            const int n1 = j.gu.SPS * (kA / 16), n2 = j.gu.KT * (kSF8 / 16);
            for (int x = et; x < n1 + n2; x += 128) {
                if (x < n1) tc::cp_async16(xA + 16 * x, j.xq_img + 16 * x);
                else tc::cp_async16(xSF + 16 * (x - n1), j.xq_sf + 16 * (x - n1));
            }
            tc::cp_async_wait_all();
            tc::fence_proxy_async_smem();
            tc::mbar_arrive(&fullS[0]);
            if (et == 0) stamp<kTrace>(j, 80);
            asm volatile("bar.sync 3, %0;" ::"n"(kThreads) : "memory");   // expert ids known (warp 0)
            if (et == 0) stamp<kTrace>(j, 78);
        }
        // After the CTA's last gate/up epilogue: count it on the grid barrier; once every CTA has finished gate/up
        // (bounded wait), one thread loads each down stage's A terms and scales with two bulk copies completing on
        // the stage's barrier.
        auto load_down_stages = [&]() {
            epi_sync();                             // every thread's down-A terms and partial sums are written
            if (et != 0) return;
            red_add_release(&j.gbar[0], 1u);        // ... and released to the CTAs that acquire the count
            stamp<kTrace>(j, 131);
            if (ngu == nst) return;
            bool done = false;
            for (uint32_t w = 0; w < tc::kSpinLimit && !done; ++w) done = ld_acquire(&j.gbar[0]) >= unsigned(nc);
            stamp<kTrace>(j, 81);
            if (done) asm volatile("fence.proxy.async.global;" ::: "memory");   // generic writes -> bulk reads
            else atomicCAS(j.err, 0, 8);
            for (int i = ngu; i < nst; ++i) {
                const Stage& st = stages[i];
                if (!done) {                          // gave up: release the MMA warp's wait
                    tc::mbar_arrive(&fullD[i - ngu]);
                    continue;
                }
                const uint32_t sfb8 = uint32_t(sk::nkt_of(st) * kSF8);
                tc::mbar_arrive_expect_tx(&fullD[i - ngu], uint32_t(kA) + sfb8);
                tc::bulk_g2s(dA + (i - ngu) * kA, j.aq_img + (size_t(st.s) * j.dn.SPS + st.ku0 / 4) * kA, kA,
                             &fullD[i - ngu]);
                tc::bulk_g2s(dSF + (i - ngu) * 2 * kSF8, j.aq_sf + (size_t(st.s) * j.dn.KT + st.ku0 / 2) * kSF8, sfb8,
                             &fullD[i - ngu]);
            }
            stamp<kTrace>(j, 83);
        };
        if (ngu == 0) load_down_stages();
        bool ok = true;
        for (int it = 0; it < nst; ++it) {
            const Stage& st = stages[it];
            if (!st.last) continue;
            // The thread's two rows of the tile are r0 = 2 et and r0 + 1: for gate/up that is one activation's glu and
            // linear rows, so thread et computes activation et and epilogue warp w holds the tile's 32-element block w.
            // Their biases are loaded before the accumulator is waited for.
            const int r0 = 2 * et;
            float b0 = 0.f, b1 = 0.f;
            if (st.mode == sk::kGateUp) {
                const int rt = st.tile - st.s * j.gu.RT;
                const float* bb = j.gu_bias + size_t(ids_s[st.tile / j.gu.RT]) * 2 * j.I + rt * kRows;
                if (rt * kRows + r0 < 2 * j.I) b0 = __ldg(bb + r0);
                if (rt * kRows + r0 + 1 < 2 * j.I) b1 = __ldg(bb + r0 + 1);
            } else {
                const int g0 = st.tile * kRows + r0;
                for (int s2 = 0; s2 < j.k; ++s2) {
                    const float* bb = j.dn_bias + size_t(ids_s[s2]) * j.H;
                    if (g0 < j.H) b0 = fmaf(w_s[s2], __ldg(bb + g0), b0);
                    if (g0 + 1 < j.H) b1 = fmaf(w_s[s2], __ldg(bb + g0 + 1), b1);
                }
            }
            // Each epilogue warp moves a quarter of the columns of accumulator rows 0..7 (the 8 terms) into shared
            // memory and releases its part of TMEM. A's 8-row groups all alias the same 8 rows, so accumulator row
            // 8g + r equals row r and every TMEM lane quadrant holds the 8 terms in its first 8 lanes: warp w reads
            // columns 64 (w - 2) .. + 63 of lanes 32 (w % 4) .. + 31, which it may access.
            // Warp 4 alone polls the accumulator barrier (warp 5 shares a scheduler with the MMA warp, whose issue
            // rate it would take); the others sleep in the named barrier until it reports.
            {
                if (warp == 4) {
                    ok = ok && tc::mbar_wait(accF, uint32_t(st.seg) & 1u, j.err, 5);
                    ok = __all_sync(kFull, ok);
                }
                ok = epi_all(ok);
                if (ok) {
                    tc::tc_fence_after();
                    const int c0 = 64 * (warp - 2);
                    const uint32_t ta = tmem + (uint32_t((warp & 3) * 32) << 16) + uint32_t(c0);
                    uint32_t v[32], w[32];
                    tmem_ld_32x32b_x32(ta, v);
                    tmem_ld_32x32b_x32(ta + 32, w);
                    tc::tmem_ld_wait();
                    if (lane < NT) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            *reinterpret_cast<float4*>(red_s + lane * kRows + c0 + i) =
                                make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]),
                                            __uint_as_float(v[i + 3]));
                            *reinterpret_cast<float4*>(red_s + lane * kRows + c0 + 32 + i) =
                                make_float4(__uint_as_float(w[i]), __uint_as_float(w[i + 1]), __uint_as_float(w[i + 2]),
                                            __uint_as_float(w[i + 3]));
                        }
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(accE);
            }
            ok = epi_all(ok);                        // uniform over the 4 epilogue warps; red_s written
            if (et == 0 && st.seg < 14) stamp<kTrace>(j, 66 + st.seg);
            float v0 = 0.f, v1 = 0.f;                // rows r0 and r0 + 1 of the tile
            if (ok) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const float2 q = *reinterpret_cast<const float2*>(red_s + t * kRows + r0);
                    v0 += q.x;
                    v1 += q.y;
                }
            }
            epi_sync();                              // red_s may be overwritten from here on
            if (ok) {
                const Part& p = part_of(st);
                const int t = st.tile;
                bool mine = true;                    // this CTA applies the tile's epilogue
                if (st.whole < 0) {                  // more CTAs share the tile than there are partial slots
                    if (et == 0) atomicCAS(j.err, 0, 101);
                    mine = false;
                } else if (!st.whole) {
                    // Split tile. Its first contributor (the CTA whose range ends inside it: the tile is that CTA's
                    // last segment of the part) finalizes it; the others (for whom it is a first or only segment)
                    // store their partial sums, tagged with the launch's epoch, and the finalizer polls the words
                    // themselves until each carries this epoch (bounded; usually already the case).
                    mine = c == st.cf;
                    unsigned long long* pb = p.partial + size_t(t) * sk::kMaxContrib * kRows;
                    if (!mine) {
                        unsigned long long* pp = pb + size_t(c - st.cf) * kRows;
                        st_relaxed64(pp + r0, tag_sum(v0, ep));
                        st_relaxed64(pp + r0 + 1, tag_sum(v1, ep));
                    } else {
                        const unsigned m = st.mask;
                        const unsigned long long none = static_cast<unsigned long long>(ep) << 32;
                        unsigned long long w0[sk::kMaxContrib], w1[sk::kMaxContrib];
#pragma unroll
                        for (int b = 1; b < sk::kMaxContrib; ++b) {   // all loads issued together
                            const bool on = (m >> b) & 1u;
                            w0[b] = on ? ld_relaxed64(pb + b * kRows + r0) : none;
                            w1[b] = on ? ld_relaxed64(pb + b * kRows + r0 + 1) : none;
                        }
                        bool done = false;
                        for (uint32_t w = 0; w < tc::kSpinLimit; ++w) {
                            done = true;
#pragma unroll
                            for (int b = 1; b < sk::kMaxContrib; ++b)
                                done = done && unsigned(w0[b] >> 32) == ep && unsigned(w1[b] >> 32) == ep;
                            if (done) break;
                            __nanosleep(32);
#pragma unroll
                            for (int b = 1; b < sk::kMaxContrib; ++b) {
                                if (unsigned(w0[b] >> 32) != ep) w0[b] = ld_relaxed64(pb + b * kRows + r0);
                                if (unsigned(w1[b] >> 32) != ep) w1[b] = ld_relaxed64(pb + b * kRows + r0 + 1);
                            }
                        }
                        mine = epi_all(done);
                        if (!mine && et == 0) atomicCAS(j.err, 0, 12);
                        if (mine) {                  // own sums first, then the other contributors in CTA order
#pragma unroll
                            for (int b = 1; b < sk::kMaxContrib; ++b)
                                if ((m >> b) & 1u) {
                                    v0 += __uint_as_float(unsigned(w0[b]));
                                    v1 += __uint_as_float(unsigned(w1[b]));
                                }
                        }
                    }
                    if (et == 0 && st.seg < 8) stamp<kTrace>(j, 132 + st.seg);
                }
                if (mine && st.mode == sk::kGateUp) {
                    const int s = t / p.RT, rt = t % p.RT;
                    const int grow = rt * kRows + r0;
                    const float y = grow < 2 * j.I ? v0 + b0 : 0.f;          // glu row
                    const float lin = grow + 1 < 2 * j.I ? v1 + b1 : 0.f;    // linear row
                    const float gv = fminf(y, j.limit);
                    const float lv = fminf(fmaxf(lin, -j.limit), j.limit);
                    const float act = __fdividef(gv, 1.f + __expf(-j.alpha * gv)) * (lv + 1.f) * w_s[s];
                    {                                // the tile's four 32-element blocks, one per epilogue warp
                        static_assert(NT == 8, "the digit split makes 8 terms");
                        const int gb = rt * (kRows / 64) + (warp - 2);
                        quantize_block_digits_warp32(act, j.aq_img + (size_t(s) * j.dn.SPS + gb / 8) * kA, gb % 8,
                                                     j.aq_sf + (size_t(s) * j.dn.KT + gb / 4) * kSF8, gb % 4,
                                                     gb * 32 < j.I);
                    }

                    if (et == 0 && st.seg < 8) stamp<kTrace>(j, 140 + st.seg);
                } else if (mine) {
                    const int grow = t * kRows + r0;
                    if (grow < j.H) j.x_resid[grow] += v0 + b0;
                    if (grow + 1 < j.H) j.x_resid[grow + 1] += v1 + b1;
                }
            }
            // after the last gate/up segment (also when a wait gave up, so other CTAs are not held up)
            if (st.mode == sk::kGateUp && it == ngu - 1) load_down_stages();
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        stamp<kTrace>(j, 82);
        __threadfence();
        if (atomicAdd(&j.gbar[1], 1u) == unsigned(nc - 1)) {   // last CTA out resets the counters and flags
            j.gbar[0] = 0;
            j.gbar[2] = 0;
            j.gbar[3] = 0;
            j.gbar[4] = ep;                                  // the next launch's epoch is this + 1
            j.gbar[1] = 0;
        }
    }
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// Shared-memory plan: NS ring slots (a 32 KB weight box and its 2 KB of scales each), x's terms and scales, down's A
// terms and scales per down stage, the accumulator's 8 term rows, barriers, and the small per-CTA state. TMEM: the accumulator in columns [0, 256), x's scale chunks, then
// a ring of NSF weight-scale slots (16 columns each) and of down's A-scale slots (8 columns each).
Layout make_layout(int NS, int cap, int cap_dn, const Part& gu, int H) {
    Layout L{};
    L.NS = NS;
    L.cap = cap;
    const int free_cols = int(kTmemCols) - int(kColX) - 4 * gu.KT;
    L.NSF = std::min(6, free_cols / 24);
    L.colSFB = kColX + 4u * uint32_t(gu.KT);
    L.colDSF = L.colSFB + 16u * uint32_t(L.NSF);
    int o = 0;
    L.ring = o; o += NS * kSlot;
    L.xA = o; o += gu.SPS * kA;
    L.xSF = o; o += (gu.KT * kSF8 + 1023) & ~1023;
    L.dA = o; o += cap_dn * kA;
    L.dSF = o; o += cap_dn * 2 * kSF8;
    L.red = o; o += NT * kRows * 4;
    L.bars = o; o += (2 * NS + 4 + cap) * 8;
    o = (o + 15) & ~15;
    L.misc = o; o += 8 + 24 + 7 * 32 * 8 + 2 * kMaxK * 4 + (kRows / 2) * 4 + cap * int(sizeof(Stage));
    L.bytes = 1024 + o;
    return L;
}

// Stage lists of every CTA for one shape and grid, built once on the host and kept on the device for the life of
// the process (one table per device and shape).
struct StageTable {
    Stage* st = nullptr;
    int* hdr = nullptr;
    int cap = 1, cap_dn = 1;
    bool crowded = false;                     // some tile is shared by more CTAs than there are partial slots
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
    // Gate/up streams from HBM, a resource all CTAs share, so its ranges hold equal unit counts. Down's weights are
    // resident by the time its stages run, which are then bound by each CTA's issue rate: its ranges balance the
    // per-CTA cost model sk::kDownCost.
    const std::vector<long long> Bg = sk::equal_bounds(g, nc);
    const std::vector<long long> Bd = sk::balanced_bounds(d, nc, sk::kDownCost);
    for (int c = 0; c < nc; ++c) {
        int seg = 0;
        const int ngu = sk::build_stages(g, Bg.data(), c, nullptr, 0, 0, 0, &seg);
        const int n = sk::build_stages(d, Bd.data(), c, nullptr, ngu, 0, seg, nullptr);
        const size_t n0 = all.size();
        all.resize(n0 + size_t(n));
        Stage* o = all.data() + n0;
        seg = 0;
        sk::build_stages(g, Bg.data(), c, o, 0, n, 0, &seg);
        sk::build_stages(d, Bd.data(), c, o, ngu, n, seg, nullptr);
        sk::fill_tile_info(g, Bg.data(), nc, c, o, 0, ngu);
        sk::fill_tile_info(d, Bd.data(), nc, c, o, ngu, n);
        hdr[size_t(c) * 4 + 0] = int(n0);
        hdr[size_t(c) * 4 + 1] = n;
        hdr[size_t(c) * 4 + 2] = ngu;
        T.cap = std::max(T.cap, n);
        T.cap_dn = std::max(T.cap_dn, n - ngu);
        for (int i = 0; i < n; ++i) T.crowded = T.crowded || (o[i].last && o[i].whole < 0);
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
    const int NT = fz::NT, TR = kDecodeTileRows;
    auto al = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    const int UKd = (I + 63) / 64;
    L.SPS_dn = (UKd + 3) / 4;
    L.KT_dn = (I + 127) / 128;
    L.SPS_gu = ((H + 63) / 64 + 3) / 4;
    L.KT_gu = (H + 127) / 128;
    L.RT_gu = (2 * I + TR - 1) / TR;
    L.RT_dn = (H + TR - 1) / TR;
    size_t o = 0;
    L.off_xq_img = o; o += al(size_t(L.SPS_gu) * NT * 128);
    L.off_xq_sf = o; o += al(size_t(L.KT_gu) * fz::kSF8);
    L.off_aq_img = o; o += al(size_t(k) * L.SPS_dn * NT * 128);
    L.off_aq_sf = o; o += al(size_t(k) * L.KT_dn * fz::kSF8);
    L.off_part_gu = o; o += al(size_t(k) * L.RT_gu * sk::kMaxContrib * TR * 8);
    L.off_part_dn = o; o += al(size_t(L.RT_dn) * sk::kMaxContrib * TR * 8);
    L.off_logits = o; o += al(size_t(32) * 16);              // epoch-tagged router logits
    L.off_err = o; o += 1024;                                // error word, then the grid barrier at +256
    L.off_sfa_gu = o; o += al(sf_repacked_bytes(k, 2 * I, H / 32, TR));
    L.off_sfa_dn = o; o += al(sf_repacked_bytes(k, H, I / 32, TR));
    L.off_misc = o; o += al(size_t(H) * 4 + 256);
    L.off_rows = o;
    L.rows_bytes = size_t(k) * L.RT_gu * H * 8;
    o += al(L.rows_bytes);
    L.bytes = o;
    L.zero_bytes_from = L.off_part_gu;                        // tagged partial sums and logits, error word, barrier
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
        GPT_CHECK(cudaFuncSetAttribute(fz::moe_fused_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        GPT_CHECK(cudaFuncSetAttribute(fz::moe_fused_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        current[dev] = bytes;
    }
}
}  // namespace

void launch_moe_decode_tc(const DecodeTcArgs& a, cudaStream_t s) {
    using namespace fz;
    if (a.tmap_dn64 && a.plan == 0 && decode_rows_ok(a.k, a.H, a.I, a.router_w ? a.E : 0)) {
        launch_moe_decode_rows(a, s);
        return;
    }
    require(a.k >= 1 && a.k <= kMaxK, "moe (tc): k must be in 1..8");
    require(a.H % 64 == 0 && a.I % 64 == 0, "moe (tc): H and I must be multiples of 64");
    require(a.H <= 4 * kThreads * kMaxX4, "moe (tc): H must be at most 3072 (x is held in registers)");
    require(!a.router_w || (a.E >= a.k && a.E <= 32), "moe (tc): router needs k <= E <= 32");
    require(num_sms() <= kMaxGrid, "moe (tc): more SMs than the stage tables are written for");
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
    j.sf_gu = a.sfa_gu;
    j.sf_dn = a.sfa_dn;
    j.sf_by_slot = a.sfa_by_slot;
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
    g.partial = reinterpret_cast<unsigned long long*>(ws + W.off_part_gu);
    Part& d = j.dn;
    d.mode = sk::kDown;
    d.RT = W.RT_dn;
    d.n_tiles = d.RT;
    d.UK = a.I / 64;
    d.KT = W.KT_dn;
    d.SPS = W.SPS_dn;
    d.UT = a.k * d.UK;
    d.total = (long long)d.n_tiles * d.UT;
    d.partial = reinterpret_cast<unsigned long long*>(ws + W.off_part_dn);
    j.aq_img = ws + W.off_aq_img;
    j.aq_sf = ws + W.off_aq_sf;
    j.x_resid = a.x_resid;
    j.err = reinterpret_cast<int*>(ws + W.off_err);
    j.gbar = reinterpret_cast<unsigned*>(ws + W.off_err + 256);
    j.logit_words = reinterpret_cast<unsigned long long*>(ws + W.off_logits);
    j.xq_img = ws + W.off_xq_img;
    j.xq_sf = ws + W.off_xq_sf;
    j.trace = a.trace;

    // One CTA per SM, all resident (cooperative launch); the stage lists come from the per-shape table.
    const int nc = num_sms();
    const StageTable& T = stage_table(g, d, nc, a.k, a.H, a.I);
    require(!T.crowded, "moe (tc): a tile would be shared by more CTAs than there are partial-sum slots");
    j.stab = T.st;
    j.shdr = T.hdr;
    int NS = 6;
    Layout L = make_layout(NS, T.cap, T.cap_dn, g, a.H);
    while (L.bytes > 227 * 1024 && NS > 2) L = make_layout(--NS, T.cap, T.cap_dn, g, a.H);
    require(L.bytes <= 227 * 1024, "moe (tc): shapes too large for one CTA's shared memory");
    require(L.NSF >= 2, "moe (tc): H too large for the TMEM scale-factor plan");
    j.L = L;
    set_fused_smem(L.bytes);

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nc);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = size_t(L.bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    // Programmatic dependent launch lets the next kernel on the stream start as this one's CTAs exit. If this
    // runtime refuses it together with a cooperative launch, the first launch on this device finds out and every
    // later one goes without it.
    static std::atomic<int> pdl_ok[64] = {};                 // 0 unknown, 1 accepted, -1 refused
    int dev = 0;
    GPT_CHECK(cudaGetDevice(&dev));
    require(dev >= 0 && dev < 64, "moe (tc): device ordinal out of range");
    cfg.numAttrs = pdl_ok[dev].load() >= 0 ? 2 : 1;
    auto kernel = a.trace ? moe_fused_kernel<true> : moe_fused_kernel<false>;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, *a.tmap_gu, *a.tmap_dn, j);
    if (e != cudaSuccess && cfg.numAttrs == 2 && pdl_ok[dev].load() == 0) {
        (void)cudaGetLastError();
        pdl_ok[dev].store(-1);
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kernel, *a.tmap_gu, *a.tmap_dn, j);
    } else if (e == cudaSuccess && cfg.numAttrs == 2) {
        pdl_ok[dev].store(1);
    }
    GPT_CHECK(e);
    check_launch("moe (tensor cores, fused)");
}

}  // namespace gpt
