// Batched (prefill) MoE for T tokens on tensor cores: the grouped-GEMM form of the reference's batched expert
// semantics (reference gptoss_ref/model.py:100-104: each expert gathers the rows that selected it, runs its two
// GEMMs, and the weighted results are added back into the residual stream).
//
// Pipeline (stream-ordered kernels):
//   1. router_batched_kernel: RMSNorm (optional) and the router for 8 tokens per CTA; logits accumulated in fp64
//      from exact products in a fixed order, top k with ties to the lower id, softmax over the k. Writes h (fp32).
//   2. permute_kernel (one CTA): the (token, slot) pairs sorted by expert, then token, into "rows"; the rows of each
//      expert cut into M tiles of 16 tokens.
//   3. quantize_tiles_kernel: every token of an M tile split into NT = 8 e2m1 residual terms with E8M0 scales per 32
//      values (exact to 2^-24 of each block's maximum) - A operand images laid out exactly as shared memory wants them
//      (128 rows = 16 tokens x 8 terms, 128-byte swizzle) and scale chunks.
//   4. grouped_gemm_kernel (persistent, one CTA per SM): tiles of (M tile, 256 weight rows); the weights are the MMA's B
//      operand straight from the checkpoint layout (TMA boxes of 256 rows x 128 bytes), tcgen05.mma kind::mxf4 with
//      M = 128, N = 256, K = 64, the accumulator in TMEM. Gate/up epilogue: the 8 term rows of each token added
//      (fixed butterfly), bias, clamped SwiGLU -> activations (fp32). Down epilogue: bias, times the gate weight ->
//      the (token, slot) result row.
//   5. quantize_tiles_kernel again on the activations, then the down GEMM.
//   6. combine_kernel: x_resid[t] += sum over slots in slot order (deterministic).
#include <algorithm>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"
#include "terms.cuh"
#include "tma.h"

namespace gpt {
namespace pf {

constexpr int NT = 8;                          // terms per token
constexpr int kTok = 16;                       // tokens per M tile (16 x 8 = 128 A rows)
constexpr int kRows = kDecodeTileRows;         // weight rows per N tile (the MMA's N)
constexpr int kThreads = 192;                  // warp 0 producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kAst = 128 * 128;                // A stage: 128 rows x 128 bytes of K (16 KB)
constexpr int kBst = kRows * 128;              // B stage: 256 rows x 128 bytes (32 KB)
constexpr int kSFAst = 2 * 512;                // A scales of a stage: 2 K chunks
constexpr int kSFBst = 2 * 1024;               // B scales of a stage: 2 K chunks x 2 row halves
constexpr int kSlot = kAst + kBst + kSFAst + kSFBst;
constexpr uint32_t kTmemCols = 512;
constexpr int kNSF = 8;                        // TMEM scale slots (8 A-scale + 16 B-scale columns each)
constexpr uint32_t kColSFA = kRows, kColSFB = kRows + 8 * kNSF;
constexpr int kRtTok = 8;                      // tokens per router CTA

// ------------------------------------------------------------------------------------------------ router (batched)
// W bf16 [E][H] -> W64 [H][32] fp64 (experts >= E zero): the router's weights once per layer (or call).
__global__ void router_w64_kernel(const __nv_bfloat16* __restrict__ W, int E, int H, double* __restrict__ W64) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H * 32; i += gridDim.x * blockDim.x) {
        const int e = i & 31, kk = i >> 5;
        W64[i] = e < E ? double(__bfloat162float(W[size_t(e) * H + kk])) : 0.0;
    }
}

// 8 tokens per CTA, 512 threads: RMSNorm (warp w < 8 on token w), h in shared memory as fp64, then thread
// (e = tid % 32, kp = tid / 32) accumulates expert e over k = kp, kp + 16, ... for the 8 tokens (the weight loads of
// four k issued ahead of their FMAs); the 16 partial sums are added in order and warp w picks token w's top k on
// order-preserving integer keys of the fp64 logits.
constexpr int kRtParts = 16;
__global__ void __launch_bounds__(512) router_batched_kernel(const double* __restrict__ W64, const float* __restrict__ b,
                                                             const float* __restrict__ x, const float* __restrict__ g,
                                                             float eps, int T, int E, int H, int k,
                                                             float* __restrict__ h_out, int* __restrict__ ids,
                                                             float* __restrict__ wts) {
    extern __shared__ double h64[];                          // [kRtTok][H]
    __shared__ double red[kRtParts][kRtTok][32];
    __shared__ float rn_s[kRtTok];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * kRtTok, nt = min(kRtTok, T - t0);
    if (warp < nt) {
        float ss = 0.f;
        const float* xr = x + size_t(t0 + warp) * H;
        for (int i = lane * 4; i < H; i += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
        ss = warp_sum(ss);
        if (lane == 0) rn_s[warp] = g ? 1.0f / sqrtf(ss / float(H) + eps) : 1.f;
    }
    __syncthreads();
    for (int i = tid * 4; i < nt * H; i += 512 * 4) {
        const int tb = i / H, kk = i - tb * H;
        float4 v = *reinterpret_cast<const float4*>(x + size_t(t0) * H + i);
        if (g) {
            const float4 gg = *reinterpret_cast<const float4*>(g + kk);
            const float r = rn_s[tb];
            v.x = v.x * r * gg.x; v.y = v.y * r * gg.y; v.z = v.z * r * gg.z; v.w = v.w * r * gg.w;
        }
        if (h_out) *reinterpret_cast<float4*>(h_out + size_t(t0) * H + i) = v;
        h64[i] = v.x; h64[i + 1] = v.y; h64[i + 2] = v.z; h64[i + 3] = v.w;
    }
    for (int i = nt * H + tid; i < kRtTok * H; i += 512) h64[i] = 0.0;
    __syncthreads();
    const int e = lane, kp = warp;
    double acc[kRtTok];
#pragma unroll
    for (int tb = 0; tb < kRtTok; ++tb) acc[tb] = 0.0;
    for (int kk0 = kp; kk0 < H; kk0 += 4 * kRtParts) {
        double wk[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int kk = kk0 + u * kRtParts;
            wk[u] = kk < H ? W64[size_t(kk) * 32 + e] : 0.0;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int kk = kk0 + u * kRtParts;
            if (kk < H) {
#pragma unroll
                for (int tb = 0; tb < kRtTok; ++tb) acc[tb] = fma(wk[u], h64[tb * H + kk], acc[tb]);
            }
        }
    }
#pragma unroll
    for (int tb = 0; tb < kRtTok; ++tb) red[kp][tb][e] = acc[tb];
    __syncthreads();
    if (warp < nt) {
        const int t = t0 + warp;
        double v = 0.0;
        if (lane < E) {
            for (int p = 0; p < kRtParts; ++p) v += red[p][warp][lane];
            v += double(b[lane]);
        }
        const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(v));
        unsigned long long key = (bits >> 63) ? ~bits : (bits | (1ull << 63));
        if ((bits & 0x7FFFFFFFFFFFFFFFull) > 0x7FF0000000000000ull || lane >= E) key = 0;   // NaN / unused
        unsigned id = lane < E ? unsigned(lane) : 32u + lane;
        float sel = -INFINITY;
        int sel_id = 0;
        for (int q = 0; q < k; ++q) {
            const unsigned hi = unsigned(key >> 32), lo = unsigned(key);
            const unsigned m1 = __reduce_max_sync(kFull, hi);
            const unsigned m2 = __reduce_max_sync(kFull, hi == m1 ? lo : 0u);
            const unsigned win = __reduce_min_sync(kFull, hi == m1 && lo == m2 ? id : 0xFFFFFFFFu);
            const double wv = __shfl_sync(kFull, v, int(win & 31u));
            if (lane == q) { sel = float(wv); sel_id = int(win); }
            if (id == win) { key = 0; id = 32u + lane; }
        }
        const float top = __shfl_sync(kFull, sel, 0);
        const float pz = lane < k ? expf(sel - top) : 0.f;
        const float sum = warp_sum(pz);
        if (lane < k) {
            ids[size_t(t) * k + lane] = sel_id;
            wts[size_t(t) * k + lane] = pz / sum;
        }
    }
}

// ------------------------------------------------------------------------------------------------ permute
// One CTA of 1024 threads. Thread i owns tokens [i * per, (i + 1) * per); its per-expert counts are scanned over the
// threads (expert e by warp e), giving every (token, slot) its row: experts in id order, tokens ascending within an
// expert. Rows of expert e are cut into M tiles of kTok rows: tiles[m] = (expert, first row, rows).
__global__ void __launch_bounds__(1024) permute_kernel(const int* __restrict__ ids, int T, int k, int E,
                                                       int* __restrict__ row_of, int* __restrict__ tok_of,
                                                       int* __restrict__ slot_of, int4* __restrict__ tiles,
                                                       int* __restrict__ n_tiles, int* __restrict__ err) {
    extern __shared__ unsigned short cnt_raw[];
    unsigned short (*cnt)[1024] = reinterpret_cast<unsigned short (*)[1024]>(cnt_raw);   // [32][1024]
    __shared__ int total[32], base[33];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int per = (T + 1023) / 1024, tb = min(T, tid * per), te = min(T, tb + per);
    for (int e = 0; e < 32; ++e) cnt[e][tid] = 0;
    bool bad = false;
    for (int t = tb; t < te; ++t)
        for (int s = 0; s < k; ++s) {
            const int e = ids[size_t(t) * k + s];
            if (e < 0 || e >= E) bad = true;
            else ++cnt[e][tid];
        }
    if (bad) atomicCAS(err, 0, 20);
    __syncthreads();
    {
        // warp e: exclusive scan of cnt[e][0..1023], lane l owning entries 32l .. 32l + 31
        const int e = warp;
        int local = 0;
        for (int i = 0; i < 32; ++i) local += cnt[e][lane * 32 + i];
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < 32; ++i) {
            const int c = cnt[e][lane * 32 + i];
            cnt[e][lane * 32 + i] = (unsigned short)run;
            run += c;
        }
        if (lane == 31) total[e] = incl;
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0, m = 0;
        for (int e = 0; e < 32; ++e) {
            base[e] = acc;
            for (int r = 0; r < total[e]; r += kTok) tiles[m++] = make_int4(e, acc + r, min(kTok, total[e] - r), 0);
            acc += total[e];
        }
        base[32] = acc;
        *n_tiles = m;
    }
    __syncthreads();
    for (int t = tb; t < te; ++t)
        for (int s = 0; s < k; ++s) {
            const int e = ids[size_t(t) * k + s];
            if (e < 0 || e >= E) continue;
            const int row = base[e] + cnt[e][tid];
            cnt[e][tid] = (unsigned short)(cnt[e][tid] + 1);
            row_of[size_t(t) * k + s] = row;
            tok_of[row] = t;
            slot_of[row] = s;
        }
}

// ------------------------------------------------------------------------------------------------ A images
// Work item (M tile m, stage st, token slot j): one warp quantizes the token's 8 blocks of the stage (4 lanes per
// block) into rows 8j .. 8j + 7 of the stage image and its scale bytes; slots past the tile's rows get zero terms.
// src row of slot j: tok_of[first row + j] (by_token) or first row + j.
__global__ void __launch_bounds__(256) quantize_tiles_kernel(const float* __restrict__ src, int by_token,
                                                             const int* __restrict__ tok_of,
                                                             const int4* __restrict__ tiles,
                                                             const int* __restrict__ n_tiles, int K, int SPS, int KT,
                                                             uint8_t* __restrict__ img, uint8_t* __restrict__ sf) {
    const int lane = threadIdx.x & 31, sub = lane & 3, gl = lane >> 2;
    const long long items = (long long)(*n_tiles) * SPS * kTok;
    const long long warps = (long long)gridDim.x * (blockDim.x / 32);
    for (long long w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; w < items; w += warps) {
        const int j = int(w % kTok);
        const long long ms = w / kTok;
        const int st = int(ms % SPS), m = int(ms / SPS);
        const int4 tl = tiles[m];
        const int g = st * 8 + gl;                       // block (32 values) along K
        float v8[8];
        if (j < tl.z && g * 32 < K) {
            const int row = tl.y + j;
            const float* sr = src + size_t(by_token ? tok_of[row] : row) * K + g * 32 + sub * 8;
            const float4 a = *reinterpret_cast<const float4*>(sr);
            const float4 c = *reinterpret_cast<const float4*>(sr + 4);
            v8[0] = a.x; v8[1] = a.y; v8[2] = a.z; v8[3] = a.w; v8[4] = c.x; v8[5] = c.y; v8[6] = c.z; v8[7] = c.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v8[i] = 0.f;
        }
        uint8_t* stage_img = img + (size_t(m) * SPS + st) * kAst + j * (NT * 128);
        const int kt = st * 2 + (gl >> 2);
        uint8_t* chunk = sf + (size_t(m) * KT + min(kt, KT - 1)) * 512 + 128 * (j & 3) + 4 * (j >> 2);
        quantize_block_terms_fixed_n<NT>(v8, stage_img, gl, chunk, gl & 3, sub, kt < KT);
    }
}

// ------------------------------------------------------------------------------------------------ grouped GEMM
struct GemmJob {
    int mode;                                  // 0: gate/up (SwiGLU -> act), 1: down (gate weight -> out_ts)
    int K, N;                                  // reduction length, weight rows of one expert
    int UK, SPS, KT, RT;                       // K / 64, stages of 256, chunks of 128, 256-row tiles of N
    const uint8_t* a_img;                      // [tiles][SPS][kAst]
    const uint8_t* a_sf;                       // [tiles][KT][512]
    const uint8_t* b_sf;                       // [E][RT][KT][2][512]
    const int4* tiles;
    const int* n_tiles;
    const float* bias;                         // [E][N]
    float alpha, limit;
    float* act;                                // gate/up: [rows][N / 2]
    const int* tok_of;                         // down
    const int* slot_of;
    const float* wts;                          // [T][k]
    int k;
    float* out_ts;                             // down: [T][k][N]
    int* err;
};

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

// Persistent: CTA c takes output tiles c, c + grid, ... of (M tile m, N tile nt) = (tau / RT, tau % RT), so the CTAs
// working at one time share an expert's weights (and each M tile's A image) through L2. Per stage one 51 KB ring slot:
// A (bulk copy), B (TMA box), A and B scales (bulk copies), all completing on the slot's barrier.
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_b,
                                                                   const __grid_constant__ GemmJob j, int NS) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * kSlot);
    uint64_t* empty = full + NS;
    uint64_t* accF = empty + NS;
    uint64_t* accE = accF + 1;
    uint32_t* holder = reinterpret_cast<uint32_t*>(accE + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        tc::mbar_init(accF, 1);
        tc::mbar_init(accE, 128);
        tc::fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(holder, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *holder;
    const int n_tiles = *j.n_tiles * j.RT;
    const int c = blockIdx.x, nc = gridDim.x;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (tc::elect_one()) {
            tc::prefetch_tmap(&tm_b);
            bool ok = true;
            int it = 0;
            for (int tau = c; tau < n_tiles && ok; tau += nc) {
                const int m = tau / j.RT, nt = tau % j.RT;
                const int e = j.tiles[m].x;
                for (int st = 0; st < j.SPS && ok; ++st, ++it) {
                    const int slot = it % NS;
                    if (it >= NS) ok = tc::mbar_wait(&empty[slot], uint32_t((it - NS) / NS) & 1u, j.err, 31);
                    if (!ok) break;
                    const int ku0 = 4 * st, nu = min(4, j.UK - ku0);
                    const int nkt = (ku0 + nu - 1) / 2 - ku0 / 2 + 1;
                    uint8_t* d = smem + slot * kSlot;
                    tc::mbar_arrive_expect_tx(&full[slot], uint32_t(kAst + kBst + nkt * 512 + nkt * 1024));
                    tc::bulk_g2s(d, j.a_img + (size_t(m) * j.SPS + st) * kAst, kAst, &full[slot]);
                    tc::tma_load_3d(d + kAst, &tm_b, st * 128, nt * kRows, e, &full[slot]);
                    tc::bulk_g2s(d + kAst + kBst, j.a_sf + (size_t(m) * j.KT + 2 * st) * 512, nkt * 512, &full[slot]);
                    tc::bulk_g2s(d + kAst + kBst + kSFAst, j.b_sf + ((size_t(e) * j.RT + nt) * j.KT + 2 * st) * 1024,
                                 nkt * 1024, &full[slot]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (one lane)
        if (tc::elect_one()) {
            bool ok = true;
            int it = 0, nt_done = 0;
            for (int tau = c; tau < n_tiles && ok; tau += nc, ++nt_done) {
                for (int st = 0; st < j.SPS && ok; ++st, ++it) {
                    const int slot = it % NS, f = it % kNSF;
                    const int ku0 = 4 * st, nu = min(4, j.UK - ku0);
                    const int nkt = (ku0 + nu - 1) / 2 - ku0 / 2 + 1;
                    if (st == 0 && nt_done > 0) ok = tc::mbar_wait(accE, uint32_t(nt_done - 1) & 1u, j.err, 32);
                    ok = ok && tc::mbar_wait(&full[slot], uint32_t(it / NS) & 1u, j.err, 33);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint8_t* d = smem + slot * kSlot;
                    for (int q = 0; q < nkt; ++q) {
                        tc::tmem_cp_sf(tmem + kColSFA + 8 * f + 4 * q,
                                       tc::desc_sf_chunk(tc::smem_u32(d + kAst + kBst + q * 512)));
                        for (int h = 0; h < 2; ++h)
                            tc::tmem_cp_sf(tmem + kColSFB + 16 * f + 8 * q + 4 * h,
                                           tc::desc_sf_chunk(tc::smem_u32(d + kAst + kBst + kSFAst + (2 * q + h) * 512)));
                    }
                    for (int u = 0; u < nu; ++u) {
                        const int ku = ku0 + u, q = ku / 2 - ku0 / 2;
                        const uint32_t sf_id = 2u * (ku & 1);
                        tc::mma_mxf4(tmem, tc::desc_sw128(tc::smem_u32(d + u * 32)),
                                     tc::desc_sw128(tc::smem_u32(d + kAst + u * 32)),
                                     tc::idesc_mxf4(128, kRows, sf_id, sf_id),
                                     (tmem + kColSFA + 8 * f + 4 * q) | (sf_id << 30),
                                     (tmem + kColSFB + 16 * f + 8 * q) | (sf_id << 30), !(st == 0 && u == 0));
                    }
                    tc::mma_commit(&empty[slot]);
                    if (st == j.SPS - 1) tc::mma_commit(accF);
                }
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue warps 2..5
        // Warp w reads TMEM lanes 32 (w % 4) .. + 31 = token slots 4 (w % 4) .. + 3, 8 term rows each. Per 32
        // columns: the 8 terms of each token added by a fixed butterfly over lanes, lane i of a token group keeping
        // columns 4i .. 4i + 3.
        const int quad = warp & 3, jslot = quad * 4 + (lane >> 3), i8 = lane & 7;
        int nt_done = 0;
        for (int tau = c; tau < n_tiles; tau += nc, ++nt_done) {
            const int m = tau / j.RT, nt = tau % j.RT;
            const int4 tl = j.tiles[m];
            bool ok = tc::mbar_wait(accF, uint32_t(nt_done) & 1u, j.err, 34);
            ok = __all_sync(kFull, ok);
            float vals[8][4];
            if (ok) {
                tc::tc_fence_after();
#pragma unroll
                for (int r = 0; r < kRows / 32; ++r) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tmem + (uint32_t(quad * 32) << 16) + 32 * r, v);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        float s = __uint_as_float(v[i]);
                        s += __shfl_xor_sync(kFull, s, 1);
                        s += __shfl_xor_sync(kFull, s, 2);
                        s += __shfl_xor_sync(kFull, s, 4);
                        if ((i >> 2) == i8) vals[r][i & 3] = s;
                    }
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(accE);
            if (!ok || jslot >= tl.z) continue;
            const int row = tl.y + jslot, e = tl.x;
            if (j.mode == 0) {
                const float* bb = j.bias + size_t(e) * j.N;
                float* ar = j.act + size_t(row) * (j.N / 2);
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const int n0 = nt * kRows + 32 * r + 4 * i8;
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        const int n = n0 + 2 * pr;
                        if (n + 1 < j.N) {
                            const float gv = fminf(vals[r][2 * pr] + bb[n], j.limit);
                            const float lv = fminf(fmaxf(vals[r][2 * pr + 1] + bb[n + 1], -j.limit), j.limit);
                            ar[n / 2] = gv / (1.f + expf(-j.alpha * gv)) * (lv + 1.f);
                        }
                    }
                }
            } else {
                const int t = j.tok_of[row], s = j.slot_of[row];
                const float w = j.wts[size_t(t) * j.k + s];
                const float* bb = j.bias + size_t(e) * j.N;
                float* orow = j.out_ts + (size_t(t) * j.k + s) * j.N;
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const int n0 = nt * kRows + 32 * r + 4 * i8;
#pragma unroll
                    for (int d = 0; d < 4; ++d)
                        if (n0 + d < j.N) orow[n0 + d] = w * (vals[r][d] + bb[n0 + d]);
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------------------------------------ combine
__global__ void combine_kernel(const float* __restrict__ out_ts, int T, int k, int H, float* __restrict__ x_resid) {
    const long long n = (long long)T * H;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / H, h = i - t * H;
        float acc = x_resid[i];
        for (int s = 0; s < k; ++s) acc += out_ts[(t * k + s) * H + h];
        x_resid[i] = acc;
    }
}

int gemm_smem_bytes(int NS) { return 1024 + NS * kSlot + (2 * NS + 2) * 8 + 16; }

}  // namespace pf

// ---------------------------------------------------------------------------------------------------- host API
PrefillLayout prefill_layout(int T, int k, int E, int H, int I) {
    PrefillLayout L{};
    auto al = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    const long long rows = (long long)T * k;
    L.max_tiles = int((rows + pf::kTok - 1) / pf::kTok) + E;
    L.SPS_gu = ((H + 63) / 64 + 3) / 4;
    L.KT_gu = (H + 127) / 128;
    L.SPS_dn = ((I + 63) / 64 + 3) / 4;
    L.KT_dn = (I + 127) / 128;
    size_t o = 0;
    L.off_h = o; o += al(size_t(T) * H * 4);
    L.off_ids = o; o += al(size_t(rows) * 4);
    L.off_w = o; o += al(size_t(rows) * 4);
    L.off_row_of = o; o += al(size_t(rows) * 4);
    L.off_tok_of = o; o += al(size_t(rows) * 4);
    L.off_slot_of = o; o += al(size_t(rows) * 4);
    L.off_tiles = o; o += al(size_t(L.max_tiles) * 16);
    L.off_misc = o; o += 1024;                              // [0] tile count, [64] error word
    const size_t img = size_t(L.max_tiles) * std::max(L.SPS_gu, L.SPS_dn) * pf::kAst;
    L.off_img = o; o += al(img);
    L.off_sf = o; o += al(size_t(L.max_tiles) * std::max(L.KT_gu, L.KT_dn) * 512);
    L.off_act = o; o += al(size_t(rows) * std::max(H, I) * 4);   // activations, then the (token, slot) results
    L.off_w64 = o; o += al(size_t(H) * 32 * 8);
    L.bytes = o;
    return L;
}

void launch_router_w64(const void* W, int E, int H, double* W64, cudaStream_t s) {
    const int grid = std::min((H * 32 + 255) / 256, num_sms() * 4);
    pf::router_w64_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(W), E, H, W64);
    check_launch("router_w64");
}

void launch_router_batched(const double* W64, const float* b, const float* x, const float* norm_w, float eps, int T,
                           int E, int H, int k, float* h_out, int* ids, float* wts, cudaStream_t s) {
    require(T >= 1, "router_batched: T must be positive");
    require(H % 8 == 0 && H >= 8, "router_batched: H must be a positive multiple of 8");
    require(k >= 1 && k <= 8 && k <= E && E <= 32, "router_batched: needs 1 <= k <= 8 and k <= E <= 32");
    const int smem = pf::kRtTok * H * 8;
    require(smem <= 200 * 1024, "router_batched: H too large");
    static std::mutex mu;
    static std::map<int, int> done;
    {
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lock(mu);
        if (done[dev] < smem) {
            GPT_CHECK(cudaFuncSetAttribute(pf::router_batched_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            done[dev] = smem;
        }
    }
    pf::router_batched_kernel<<<(T + pf::kRtTok - 1) / pf::kRtTok, 512, smem, s>>>(W64, b, x, norm_w, eps, T, E, H, k,
                                                                                   h_out, ids, wts);
    check_launch("router_batched");
}

void launch_moe_batched(const PrefillArgs& a, cudaStream_t s) {
    using namespace pf;
    require(a.T >= 1, "moe_batched: T must be positive");
    require(a.k >= 1 && a.k <= 8 && a.k <= a.E && a.E <= 32, "moe_batched: needs 1 <= k <= 8 and k <= E <= 32");
    require(a.H % 64 == 0 && a.I % 64 == 0, "moe_batched: H and I must be multiples of 64");
    const PrefillLayout L = prefill_layout(a.T, a.k, a.E, a.H, a.I);
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    int* tok_of = reinterpret_cast<int*>(ws + L.off_tok_of);
    int* slot_of = reinterpret_cast<int*>(ws + L.off_slot_of);
    int4* tiles = reinterpret_cast<int4*>(ws + L.off_tiles);
    int* n_tiles = reinterpret_cast<int*>(ws + L.off_misc);
    int* err = reinterpret_cast<int*>(ws + L.off_misc + 64 * 4);
    uint8_t* img = ws + L.off_img;
    uint8_t* sf = ws + L.off_sf;
    float* act = reinterpret_cast<float*>(ws + L.off_act);
    const int sms = num_sms();

    require(a.T <= 32768, "moe_batched: at most 32768 tokens per call");
    static std::mutex pmu;
    static std::map<int, bool> pdone;
    {
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lock(pmu);
        if (!pdone[dev]) {
            GPT_CHECK(cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 32 * 1024 * 2));
            pdone[dev] = true;
        }
    }
    permute_kernel<<<1, 1024, 32 * 1024 * 2, s>>>(a.ids, a.T, a.k, a.E, reinterpret_cast<int*>(ws + L.off_row_of),
                                                   tok_of, slot_of, tiles, n_tiles, err);
    check_launch("moe_batched permute");

    int NS = 4;
    while (gemm_smem_bytes(NS) > 227 * 1024 && NS > 2) --NS;
    const int smem = gemm_smem_bytes(NS);
    static std::mutex mu;
    static std::map<int, int> done;
    {
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lock(mu);
        if (done[dev] < smem) {
            GPT_CHECK(cudaFuncSetAttribute(grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            done[dev] = smem;
        }
    }
    for (int pass = 0; pass < 2; ++pass) {
        const bool gu = pass == 0;
        const int K = gu ? a.H : a.I, N = gu ? 2 * a.I : a.H;
        const int SPS = gu ? L.SPS_gu : L.SPS_dn, KT = gu ? L.KT_gu : L.KT_dn;
        quantize_tiles_kernel<<<sms * 8, 256, 0, s>>>(gu ? a.h : act, gu ? 1 : 0, tok_of, tiles, n_tiles, K, SPS, KT,
                                                      img, sf);
        check_launch("moe_batched quantize");
        GemmJob g{};
        g.mode = gu ? 0 : 1;
        g.K = K;
        g.N = N;
        g.UK = K / 64;
        g.SPS = SPS;
        g.KT = KT;
        g.RT = (N + kRows - 1) / kRows;
        g.a_img = img;
        g.a_sf = sf;
        g.b_sf = gu ? a.sf_gu : a.sf_dn;
        g.tiles = tiles;
        g.n_tiles = n_tiles;
        g.bias = gu ? a.gu_bias : a.dn_bias;
        g.alpha = a.alpha;
        g.limit = a.limit;
        g.act = act;
        g.tok_of = tok_of;
        g.slot_of = slot_of;
        g.wts = a.weights;
        g.k = a.k;
        g.out_ts = act;                                    // the activations are consumed by then
        g.err = err;
        grouped_gemm_kernel<<<sms, kThreads, smem, s>>>(gu ? *a.tmap_gu : *a.tmap_dn, g, NS);
        check_launch("moe_batched grouped gemm");
    }
    combine_kernel<<<sms * 8, 256, 0, s>>>(act, a.T, a.k, a.H, a.x_resid);
    check_launch("moe_batched combine");
}

}  // namespace gpt
