// Batched (prefill) MoE for T tokens on tensor cores: the grouped-GEMM form of the reference's batched expert
// semantics (reference gptoss_ref/model.py:100-104: each expert gathers the rows that selected it, runs its two
// GEMMs, and the weighted results are added back into the residual stream).
//
// Pipeline (stream-ordered kernels):
//   1. router_batched_kernel: RMSNorm (optional) and the router for 8 tokens per CTA; logits accumulated in fp64
//      from exact products in a fixed order, top k with ties to the lower id, softmax over the k. Writes h (fp32).
//   2. permute_kernel (one CTA): the (token, slot) pairs sorted by expert, then token, into "rows"; the rows of each
//      expert cut into M tiles of 128 / P rows; pos_of[(token, slot)] = 128 * tile + P * (row in the tile).
//   3. quantize_h_kernel: every token's h split once into nt (default NT = 8) e2m1 terms with E8M0 scales per 32
//      values (8 terms: exact to 2^-21 of each block's scale) and written into the A images of the k tiles that hold
//      it. An A "slot" is 128 rows x 128 bytes of one 256-wide K block of one M tile, in the 128-byte-swizzled layout
//      shared memory wants, followed by its scale chunks - one bulk copy.
//   4. grouped_gemm_kernel (persistent, one CTA per SM), gate/up: tiles of (M tile, 256 weight rows); the weights
//      are the MMA's B operand straight from the checkpoint layout (TMA boxes of 256 rows x 128 bytes). Per K block
//      the S slots are S MMAs of M = 128 rows, N = 256, K = 64 x 4 (tcgen05.mma kind::mxf4) into the SAME TMEM
//      accumulator. Epilogue: bias, clamped SwiGLU -> activations.
//   5. quantize_act_kernel: the activations into the down projection's A slots, as step 3.
//   6. grouped_gemm_kernel, down: the same mainloop; epilogue w * (y + b2) -> the (token, slot) result row.
//   7. combine_kernel: x_resid[t] += sum over slots in slot order (deterministic).
//
// Term plan (nt terms, S slots, P rows per token; S P >= nt). Stacked (P = 1, S = nt): row r of a tile is one token,
// slot i holds its term S - 1 - i, and the tensor core adds the terms in the accumulator; one B tile serves
// nt x 128 token-terms. Packed (P = 8, S = 1): row P j + t holds term t of the tile's token j (rows t >= nt zero),
// 16 tokens per tile, and the epilogue adds each token's P rows (lanes) - an expert with few rows (small batches)
// then costs one MMA per K step instead of nt on a mostly empty tile.
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

constexpr int NT = 8;                          // most terms per token (the exact default)
constexpr int kPackRows = 8;                   // rows per token in the packed plan
constexpr int kTileM = 128;                    // tokens (rows of one expert) per M tile = the MMA's M
constexpr int kRows = kDecodeTileRows;         // weight rows per N tile (the MMA's N)
constexpr int kEpiWarps = 8;                   // two per TMEM lane quadrant, 128 columns each
constexpr int kThreads = 64 + 32 * kEpiWarps;  // warp 0 producer, warp 1 MMA issuer, warps 2.. epilogue
constexpr int kImg = kTileM * 128;             // one term's A image for a 256-wide K block (16 KB)
constexpr int kSFA = 4096;                     // its scales, replicated per lane quadrant (tcgen05.cp 128x256b source)
constexpr int kTermA = kImg + kSFA;            // 20 KB
constexpr int kPT = 2;                         // slots per A piece (one barrier wait per 8 MMAs)
constexpr int kPieceA = kPT * kTermA;
constexpr int kBImg = kRows * 128;             // B tile for a 256-wide K block (32 KB)
constexpr int kPieceB = kBImg + 4 * 512;       // + its scale chunks (2 K chunks x 2 row halves)
constexpr int kSeg = 2;                        // K blocks per accumulation segment (stacked plan)
constexpr int NSA = 3, NSB = kSeg + 1;         // ring slots: A pieces, B pieces
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSFA = kRows;            // 8 columns per term, 16 per A slot
constexpr uint32_t kColSFB = kRows + 16 * NSA; // 16 columns per B slot
static_assert(kColSFB + 16 * NSB <= kTmemCols, "TMEM budget");
constexpr int kRtTok = 14;                     // tokens per router CTA (2048 tokens: 147 CTAs, one wave)

// ------------------------------------------------------------------------------------------------ router (batched)
// W bf16 [E][H] -> W64 [H][32] fp64 (experts >= E zero): the router's weights once per layer (or call).
__global__ void router_w64_kernel(const __nv_bfloat16* __restrict__ W, int E, int H, double* __restrict__ W64) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H * 32; i += gridDim.x * blockDim.x) {
        const int e = i & 31, kk = i >> 5;
        W64[i] = e < E ? double(__bfloat162float(W[size_t(e) * H + kk])) : 0.0;
    }
}

// kRtTok tokens per cluster of KS CTAs (KS = 1, 2, 4 or 8: the grid is token groups x KS, cluster dims (KS, 1, 1)),
// 512 threads per CTA. CTA q of a cluster owns the K slice [q SW, (q + 1) SW), SW = router_slice(H, KS):
//   1. the sums of squares of its tokens over the slice (warp w < kRtTok on token w); the cluster's KS partial sums
//      are added in rank order (distributed shared memory), so every CTA of the cluster has the same RMSNorm scale;
//   2. h over the slice (fp32, x * rn * g as RMSNorm computes it) into shared memory and h_out;
//   3. thread (e = tid % 32, kp = tid / 32) accumulates expert e over k = kp, kp + 16, ... of the slice, chunk by
//      chunk of K: the chunk's twelve weight loads per thread are issued first, the CTA widens the chunk's h values to
//      fp64 once (exact; widening at every FMA kept the conversion pipe saturated), then each load serves all tokens;
//   4. the 16 partial sums (stored over h, which is dead by then) are added in order; CTA 0 of the cluster adds the
//      KS slices' sums in rank order and warp w picks token w's top k on order-preserving integer keys of the fp64
//      logits.
// Small batches use several CTAs per token group (KS > 1), so that the router is spread over the GPU instead of
// running through K on a few SMs; KS = 1 is one CTA per group over all of K.
constexpr int kRtParts = 16;
static_assert(kRtTok <= 16, "one top-k warp per token");
constexpr int kRtAhead = 12;                   // weight loads in flight per router thread
constexpr int kRtChunk = kRtAhead * kRtParts;  // K values widened to fp64 at a time (192)
constexpr int kRtMaxSplit = 8;                 // CTAs per token group at most (a portable cluster size)
// Router shared memory: h (fp32, [kRtTok][SW]; the partial sums go over it after the FMAs), one chunk of h widened to
// fp64 ([kRtTok][kRtChunk]), the slice's logit sums ([kRtTok][32] fp64) and sums of squares ([kRtTok] fp32).
__host__ __device__ constexpr int router_slice(int H, int KS) { return ((H / 4 + KS - 1) / KS) * 4; }
__host__ __device__ constexpr int router_chunk_off(int H, int KS) {
    return ((kRtTok * router_slice(H, KS) * 4 > kRtParts * kRtTok * 32 * 8 ? kRtTok * router_slice(H, KS) * 4
                                                                             : kRtParts * kRtTok * 32 * 8) + 15) & ~15;
}
__host__ __device__ constexpr int router_sum_off(int H, int KS) { return router_chunk_off(H, KS) + kRtTok * kRtChunk * 8; }
__host__ __device__ constexpr int router_smem_bytes(int H, int KS) {
    return router_sum_off(H, KS) + kRtTok * 32 * 8 + kRtTok * 4;
}
__global__ void __launch_bounds__(512, 1) router_batched_kernel(const double* __restrict__ W64, const float* __restrict__ b,
                                                             const float* __restrict__ x, const float* __restrict__ g,
                                                             float eps, int T, int E, int H, int k, int KS,
                                                             float* __restrict__ h_out, int* __restrict__ ids,
                                                             float* __restrict__ wts) {
    extern __shared__ __align__(16) uint8_t rt_smem[];
    const int SW = router_slice(H, KS);
    float* hs = reinterpret_cast<float*>(rt_smem);           // [kRtTok][SW]
    double (*red)[kRtTok][32] = reinterpret_cast<double (*)[kRtTok][32]>(rt_smem);   // [kRtParts]: after the FMAs
    double* hc = reinterpret_cast<double*>(rt_smem + router_chunk_off(H, KS));       // [kRtTok][kRtChunk]
    double (*csum)[32] = reinterpret_cast<double (*)[32]>(rt_smem + router_sum_off(H, KS));   // [kRtTok][32]
    float* ssp = reinterpret_cast<float*>(rt_smem + router_sum_off(H, KS) + kRtTok * 32 * 8);   // [kRtTok]
    __shared__ float rn_s[kRtTok];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const unsigned q = KS > 1 ? cluster_rank() : 0u;
    const int t0 = (blockIdx.x / KS) * kRtTok, nt = min(kRtTok, T - t0);
    const int k0 = min(H, int(q) * SW), k1 = min(H, k0 + SW), w = k1 - k0;
    if (warp < nt) {
        float ss = 0.f;
        const float* xr = x + size_t(t0 + warp) * H;
        for (int i = k0 + lane * 4; i < k1; i += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
        ss = warp_sum(ss);
        if (lane == 0) ssp[warp] = ss;
    }
    if (KS > 1) cluster_sync_all();
    else __syncthreads();
    if (warp < nt && lane == 0) {
        float tot = 0.f;
        for (int r = 0; r < KS; ++r) tot += KS > 1 ? dsmem_load_f32(ssp + warp, unsigned(r)) : ssp[warp];
        rn_s[warp] = g ? rms_scale(tot, H, eps) : 1.f;
    }
    __syncthreads();
    for (int i = tid * 4; i < nt * w; i += 512 * 4) {        // w % 4 == 0: a float4 never crosses a token
        const int tb = i / w, kk = k0 + (i - tb * w);
        float4 v = *reinterpret_cast<const float4*>(x + size_t(t0 + tb) * H + kk);
        if (g) {
            const float4 gg = *reinterpret_cast<const float4*>(g + kk);
            const float r = rn_s[tb];
            v.x = v.x * r * gg.x; v.y = v.y * r * gg.y; v.z = v.z * r * gg.z; v.w = v.w * r * gg.w;
        }
        if (h_out) *reinterpret_cast<float4*>(h_out + size_t(t0 + tb) * H + kk) = v;
        *reinterpret_cast<float4*>(hs + tb * SW + (kk - k0)) = v;
    }
    for (int i = nt * SW + tid; i < kRtTok * SW; i += 512) hs[i] = 0.f;
    __syncthreads();
    const int e = lane, kp = warp;
    double acc[kRtTok];
#pragma unroll
    for (int tb = 0; tb < kRtTok; ++tb) acc[tb] = 0.0;
    for (int c0 = k0; c0 < k1; c0 += kRtChunk) {
        double wk[kRtAhead];
#pragma unroll
        for (int u = 0; u < kRtAhead; ++u) {
            const int kk = c0 + kp + u * kRtParts;
            wk[u] = kk < k1 ? W64[size_t(kk) * 32 + e] : 0.0;
        }
        for (int i = tid; i < kRtTok * kRtChunk; i += 512) {
            const int tb = i / kRtChunk, jj = i - tb * kRtChunk;
            hc[i] = c0 + jj < k1 ? double(hs[tb * SW + (c0 - k0) + jj]) : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < kRtAhead; ++u) {
            const int jj = kp + u * kRtParts;
            if (c0 + jj < k1) {
#pragma unroll
                for (int tb = 0; tb < kRtTok; ++tb) acc[tb] = fma(wk[u], hc[tb * kRtChunk + jj], acc[tb]);
            }
        }
        __syncthreads();                                     // the chunk buffer is refilled next
    }
    __syncthreads();                                         // h is dead: the partial sums go over it
#pragma unroll
    for (int tb = 0; tb < kRtTok; ++tb) red[kp][tb][e] = acc[tb];
    __syncthreads();
    if (warp < nt) {
        double v = 0.0;
        for (int p = 0; p < kRtParts; ++p) v += red[p][warp][lane];
        csum[warp][lane] = v;
    }
    if (KS > 1) cluster_sync_all();
    else __syncthreads();
    if (q == 0 && warp < nt) {
        const int t = t0 + warp;
        double v = 0.0;
        if (lane < E) {
            for (int r = 0; r < KS; ++r) v += KS > 1 ? dsmem_load_f64(&csum[warp][lane], unsigned(r)) : csum[warp][lane];
            v += double(b[lane]);
        }
        int sel_id = 0;
        double sel_logit = 0.0;
        warp_topk_logits(v, lane < E, k, sel_id, sel_logit);
        const float gate = warp_pick_softmax(sel_logit, k);
        if (lane < k) {
            ids[size_t(t) * k + lane] = sel_id;
            wts[size_t(t) * k + lane] = gate;
        }
    }
    if (KS > 1) cluster_sync_all();                          // the slices' sums stay until CTA 0 has read them
}

// ------------------------------------------------------------------------------------------------ permute
// One CTA of 1024 threads. Thread i owns tokens [i * per, (i + 1) * per); its per-expert counts are scanned over the
// threads (expert e by warp e), giving every (token, slot) its row: experts in id order, tokens ascending within an
// expert. Rows of expert e are cut into M tiles of kTileM / P rows: tiles[m] = (expert, first row, rows), and
// pos_of[t * k + s] = kTileM * (tile) + P * (row within the tile), or -1 for an invalid id.
__global__ void __launch_bounds__(1024) permute_kernel(const int* __restrict__ ids, int T, int k, int E, int P,
                                                       int* __restrict__ pos_of, int* __restrict__ tok_of,
                                                       int* __restrict__ slot_of, int4* __restrict__ tiles,
                                                       int* __restrict__ n_tiles, int* __restrict__ err) {
    const int TM = kTileM / P;
    extern __shared__ unsigned short cnt_raw[];
    unsigned short (*cnt)[1024] = reinterpret_cast<unsigned short (*)[1024]>(cnt_raw);   // [32][1024]
    __shared__ int total[32], base[33], tile0[32];
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
            tile0[e] = m;
            for (int r = 0; r < total[e]; r += TM) tiles[m++] = make_int4(e, acc + r, min(TM, total[e] - r), 0);
            acc += total[e];
        }
        base[32] = acc;
        *n_tiles = m;
    }
    __syncthreads();
    for (int t = tb; t < te; ++t)
        for (int s = 0; s < k; ++s) {
            const int e = ids[size_t(t) * k + s];
            if (e < 0 || e >= E) {
                pos_of[size_t(t) * k + s] = -1;
                continue;
            }
            const int r = cnt[e][tid];
            const int row = base[e] + r;
            cnt[e][tid] = (unsigned short)(r + 1);
            pos_of[size_t(t) * k + s] = (tile0[e] + r / TM) * kTileM + (r % TM) * P;
            tok_of[row] = t;
            slot_of[row] = s;
        }
}

// ------------------------------------------------------------------------------------------------ A images
// A images: per (M tile, K block) S slots of kTermA bytes each: the 128 x 128-byte image in the 128-byte swizzle,
// then its scales. Slot i holds the rows' terms P (S - 1 - i) .. P (S - 1 - i) + P - 1 (DESCENDING: the smallest
// first). A piece of up to kPT consecutive slots is one bulk copy.
__device__ __forceinline__ uint8_t* a_slot(uint8_t* img, int m, int KB, int kb, int S, int i) {
    return img + ((size_t(m) * KB + kb) * S + i) * kTermA;
}

// Term t's 16-byte unit of block g (0..7 within the K block) in row r (128-byte swizzle).
__device__ __forceinline__ int a_unit_off(int r, int g) { return r * 128 + ((g ^ (r & 7)) << 4); }

// The scales of a term as the source of one tcgen05.cp 128x256b (128 rows x 32 bytes in 8-row x 16-byte core
// matrices: row L byte b at (L / 8) 256 + (b / 16) 128 + (L % 8) 16 + b % 16): row L holds what the 32x128b.warpx4
// copy of the term's two 512-byte chunks would put in TMEM lane L, i.e. chunk c's 16-byte row L % 32 at bytes
// 16 c .. 16 c + 15, where byte 4 j + kk of chunk row i is the scale of token row i + 32 j, block 4 c + kk. Each
// scale therefore appears in the 4 rows L = r % 32 + 32 q. Offset of the copy for quadrant q of row r, block g:
__device__ __forceinline__ int a_sf_off(int r, int g, int q) {
    const int L = (r & 31) + 32 * q, b = (g >> 2) * 16 + (r >> 5) * 4 + (g & 3);
    return kImg + (L >> 3) * 256 + (b >> 4) * 128 + (L & 7) * 16 + (b & 15);
}

__device__ __forceinline__ uint64_t desc_sfa_128x256b(uint32_t saddr) { return tc::smem_desc(saddr, 128, 256, 0); }

__device__ __forceinline__ void tmem_cp_128x256b(uint32_t tmem_col, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(tmem_col), "l"(sdesc) : "memory");
}

struct TermPlan {
    int nt;                                    // terms per token (1 .. NT)
    int S;                                     // A slots per (M tile, K block)
    int P;                                     // rows per token (1 or kPackRows); tokens per tile = kTileM / P
};

// One warp quantizes 8 blocks (K block kb, 4 lanes per 32-value block) of the source row `src` once and writes the
// terms into the A slots of `nd` destination tokens (pos = 128 * tile + P * (token in the tile); negative = none):
// term t to row pos % 128 + t % P of slot S - 1 - t / P.
template <int MaxD>                                 // destinations the caller may pass (nd <= MaxD <= 8)
__device__ __forceinline__ void quantize_row_kblock(const float* __restrict__ src, int K, int kb, const int (&pos)[8],
                                                    int nd, int KB, uint8_t* const (&img)[8], const TermPlan tp) {
    const int lane = threadIdx.x & 31, sub = lane & 3, gl = lane >> 2;
    const int g = kb * 8 + gl;
    const bool valid = g * 32 < K;
    float v8[8];
    if (valid) {
        const float* sr = src + g * 32 + sub * 8;
        const float4 a = *reinterpret_cast<const float4*>(sr);
        const float4 c = *reinterpret_cast<const float4*>(sr + 4);
        v8[0] = a.x; v8[1] = a.y; v8[2] = a.z; v8[3] = a.w; v8[4] = c.x; v8[5] = c.y; v8[6] = c.z; v8[7] = c.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v8[i] = 0.f;
    }
    // The scale bytes of the 8 blocks as two words per (row, quadrant copy): lane l < 8 stores word (l >> 2) of
    // quadrant copy l & 3, covering blocks 4 (l >> 2) .. + 3. A term's scale follows from its block's k (term 0
    // carries k + 127; term 1 k - 1; term t >= 2 k + 2 - 3t; clamped at 0), so the four blocks' term-0 scales are
    // gathered once and every later word is a bytewise saturating subtraction (saturating step by step equals
    // clamping the total, the amounts only grow).
    const int wsel = (lane >> 2) & 1, qsel = lane & 3;
    // Per destination, once: its (M tile, K block) slot 0 and first row.
    uint8_t* base[MaxD];
    int row0[MaxD];
#pragma unroll
    for (int s = 0; s < MaxD; ++s) {
        const bool on = s < nd && pos[s] >= 0;
        const int ps_ = on ? pos[s] : 0;
        base[s] = on ? a_slot(img[s], ps_ / kTileM, KB, kb, tp.S, 0) : nullptr;
        row0[s] = ps_ % kTileM;
    }
    const int n_emit = tp.S * tp.P;
    uint32_t sw0 = 0, sw = 0;
    quantize_block_digits_lanes4(v8, [&](int term, uint32_t word, uint32_t scale) {
        if (term == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) sw0 |= (__shfl_sync(kFull, scale, 4 * (4 * wsel + kk)) & 0xFFu) << (8 * kk);
            sw = sw0;
        } else if (term == 1) {
            sw = __vsubus4(sw0, 0x01010101u);
        } else if (term == 2) {
            sw = __vsubus4(sw0, 0x04040404u);
        } else {
            sw = __vsubus4(sw, 0x03030303u);
        }
        if (term >= n_emit) return;
        const int slot = tp.S - 1 - term / tp.P, dr = term % tp.P;
#pragma unroll
        for (int s = 0; s < MaxD; ++s) {
            if (!base[s]) continue;
            uint8_t* piece = base[s] + size_t(slot) * kTermA;
            const int r = row0[s] + dr;
            if (valid) *reinterpret_cast<uint32_t*>(piece + a_unit_off(r, gl) + sub * 4) = word;
            if (lane < 8) *reinterpret_cast<uint32_t*>(piece + a_sf_off(r, 4 * wsel, qsel)) = sw;
        }
    }, tp.nt);
}

// Image bases by rank (expert parallelism: index = the rank that owns the row's expert, the peer's mapping of its
// region); one rank: all equal.
struct ImgBases {
    uint8_t* p[8];
};

// Gate/up A terms from h: work item (token t, K block kb) per warp; the token's terms are computed once and written
// to the k tiles that hold it (pos_of; dest_of = the owning rank, or null for one rank).
__global__ void __launch_bounds__(256) quantize_h_kernel(const float* __restrict__ h, int T, int H, int k,
                                                         const int* __restrict__ pos_of, const int* __restrict__ dest_of,
                                                         int KB, const __grid_constant__ ImgBases imgs,
                                                         const TermPlan tp) {
    const long long items = (long long)T * KB;
    const long long warps = (long long)gridDim.x * (blockDim.x / 32);
    for (long long w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; w < items; w += warps) {
        const int t = int(w / KB), kb = int(w % KB);
        int pos[8];
        uint8_t* img[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            pos[s] = s < k ? pos_of[size_t(t) * k + s] : -1;
            img[s] = imgs.p[(s < k && dest_of) ? (dest_of[size_t(t) * k + s] & 7) : 0];
        }
        quantize_row_kblock<8>(h + size_t(t) * H, H, kb, pos, k, KB, img, tp);
    }
    if (dest_of) __threadfence_system();                    // expert parallel: stores into peers' regions
}

// Down A terms from the activations act [rows][I] (rows in tile order): work item (tile m, token j, K block kb).
__global__ void __launch_bounds__(256) quantize_act_kernel(const float* __restrict__ act, int I,
                                                           const int4* __restrict__ tiles,
                                                           const int* __restrict__ n_tiles, int KB,
                                                           uint8_t* __restrict__ img, const TermPlan tp) {
    const int TM = kTileM / tp.P;
    const long long items = (long long)(*n_tiles) * TM * KB;
    const long long warps = (long long)gridDim.x * (blockDim.x / 32);
    for (long long w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; w < items; w += warps) {
        const int kb = int(w % KB);
        const int jm = int(w / KB), j = jm % TM, m = jm / TM;
        const int4 tl = tiles[m];
        if (j >= tl.z) continue;
        int pos[8];
        uint8_t* im[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            pos[s] = s == 0 ? m * kTileM + j * tp.P : -1;
            im[s] = img;
        }
        quantize_row_kblock<1>(act + size_t(tl.y + j) * I, I, kb, pos, 1, KB, im, tp);
    }
}

// ------------------------------------------------------------------------------------------------ grouped GEMM
struct GemmJob {
    int mode;                                  // 0: gate/up (SwiGLU -> down A pieces), 1: down (w (y + b) -> out_ts)
    int K, N;                                  // reduction length, weight rows of one expert
    int UK, KB, KT, RT;                        // K / 64, 256-wide K blocks, 128-wide K chunks, 256-row N tiles
    const uint8_t* a_img;                      // [tiles][KB][S] slots, descending terms
    int S, P;                                  // term plan: slots per (tile, K block), rows per token
    int seg;                                   // K blocks per accumulation segment (kSeg; KB when S == 1)
    const uint8_t* b_sf;                       // [E][RT][KT][2][512]
    const int4* tiles;
    const int* n_tiles;
    const float* bias;                         // [E][N]
    float alpha, limit;
    float* act;                                // gate/up: activations [rows][I]
    int I;
    const int* tok_of;                         // down
    const int* slot_of;
    const float* wts;                          // [T][k]
    int k;
    float* out_ts;                             // down: [T][k][N]
    const int4* meta;                          // expert parallel: per row (pos) source rank, token, slot, weight bits
    float* out_rank[8];                        // expert parallel: each source rank's result rows as mapped here
    int* err;
    long long* trace;                          // optional: per CTA (< 160) 160 stamps, slots 64 mode + i
};

// Named barrier 1 over the epilogue warps (warps 2 ..), so that only one of their threads polls an mbarrier.
__device__ __forceinline__ void epi_bar_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
}

// Timed wait: adds the cycles spent in the wait to *acc when tracing.
__device__ __forceinline__ bool twait(uint64_t* bar, uint32_t parity, int* err, int where, long long* acc) {
    if (!acc) return tc::mbar_wait(bar, parity, err, where);
    const long long t0 = clock64();
    const bool ok = tc::mbar_wait(bar, parity, err, where);
    *acc += clock64() - t0;
    return ok;
}

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

// Packed plan: a token's kPackRows term rows are 8 aligned lanes (q = lane % 8 = the term). A reduce-scatter over
// the three lane bits leaves lane q with the token's sums of columns 16 q .. 16 q + 15 (112 shuffles; every column is
// added once, in an order fixed by the lanes, so the result is deterministic).
__device__ __forceinline__ void pack_reduce_scatter(const float (&sums)[128], int q, float (&out)[16]) {
    static_assert(kPackRows == 8, "three lane bits");
    float r1[64], r2[32];
    const bool b2 = q & 4, b1 = q & 2, b0 = q & 1;
#pragma unroll
    for (int i = 0; i < 64; ++i) {                 // r1[i] = column 64 b2 + i
        const float keep = b2 ? sums[64 + i] : sums[i], send = b2 ? sums[i] : sums[64 + i];
        r1[i] = keep + __shfl_xor_sync(kFull, send, 4);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {                 // r2[i] = column 64 b2 + 32 b1 + i
        const float keep = b1 ? r1[32 + i] : r1[i], send = b1 ? r1[i] : r1[32 + i];
        r2[i] = keep + __shfl_xor_sync(kFull, send, 2);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {                 // out[i] = column 16 q + i
        const float keep = b0 ? r2[16 + i] : r2[i], send = b0 ? r2[i] : r2[16 + i];
        out[i] = keep + __shfl_xor_sync(kFull, send, 1);
    }
}

// Persistent: CTA c takes output tiles c, c + grid, ... of (M tile m, N tile nt) = (tau / RT, tau % RT), so the CTAs
// working at one time share an expert's weights (and each M tile's A pieces) through L2. Two rings: B pieces (TMA box +
// scale chunks, one per K block) and A pieces (one bulk copy per (K block, term)); the producer and the MMA issuer are
// single threads.
//
// Accumulation order. The tensor core adds each MMA's result into D with an error that scales with |D| (about one
// unit in the last place of fp32 per MMA), so the number of MMAs added into a large accumulator decides the
// precision. The K blocks of a tile are processed in segments of kSeg: within a segment the terms go from the
// smallest (NT - 1) to the largest (0), each over the segment's K blocks (whose B pieces stay resident), so the small
// terms are added while D is still small; after each segment the epilogue warps add D into fp32 registers and D
// restarts from zero. Term 0, the only term of full magnitude, then meets at most 4 kSeg MMAs per accumulator.
// In the packed plan every accumulator row holds one term of one token, as in the decode kernel, and its B pieces are
// used once each (one slot per K block): the whole K range is one segment (j.seg = KB), so the MMAs stop for the
// epilogue's read of TMEM once per tile instead of every kSeg K blocks.
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_b,
                                                                   const __grid_constant__ GemmJob j) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ringA = smem;
    uint8_t* ringB = smem + NSA * kPieceA;
    uint64_t* fullA = reinterpret_cast<uint64_t*>(ringB + NSB * kPieceB);
    uint64_t* emptyA = fullA + NSA;
    uint64_t* fullB = emptyA + NSA;
    uint64_t* emptyB = fullB + NSB;
    uint64_t* accF = emptyB + NSB;
    uint64_t* accE = accF + 1;
    uint32_t* holder = reinterpret_cast<uint32_t*>(accE + 1);
    int* epi_flag = reinterpret_cast<int*>(holder + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < NSA; ++i) {
            tc::mbar_init(&fullA[i], 1);
            tc::mbar_init(&emptyA[i], 1);
        }
        for (int i = 0; i < NSB; ++i) {
            tc::mbar_init(&fullB[i], 1);
            tc::mbar_init(&emptyB[i], 1);
        }
        tc::mbar_init(accF, 1);
        tc::mbar_init(accE, kEpiWarps);
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
        // ---------------------------------------------------------------- producer (one thread)
        if (lane == 0) {
            tc::prefetch_tmap(&tm_b);
            bool ok = true;
            int ia = 0, ib = 0;
            const int npc = (j.S + kPT - 1) / kPT;
            long long wA = 0, wB = 0;
            long long* twA = j.trace && c < 160 ? &wA : nullptr;
            long long* twB = j.trace && c < 160 ? &wB : nullptr;
            for (int tau = c; tau < n_tiles && ok; tau += nc) {
                const int m = tau / j.RT, nt = tau % j.RT;
                const int e = j.tiles[m].x;
                for (int s0 = 0; s0 < j.KB && ok; s0 += j.seg) {
                    const int s1 = min(j.KB, s0 + j.seg);
                    for (int pc = 0; pc < npc && ok; ++pc)
                        for (int kb = s0; kb < s1; ++kb) {
                            if (pc == 0) {
                                const int nkq = min(2, j.KT - 2 * kb);
                                const int sb = ib % NSB;
                                if (ib >= NSB) ok = twait(&emptyB[sb], uint32_t(ib / NSB - 1) & 1u, j.err, 31, twB);
                                if (!ok) break;
                                uint8_t* pb = ringB + sb * kPieceB;
                                tc::mbar_arrive_expect_tx(&fullB[sb], uint32_t(kBImg + nkq * 1024));
                                tc::tma_load_3d(pb, &tm_b, kb * 128, nt * kRows, e, &fullB[sb]);
                                tc::bulk_g2s(pb + kBImg, j.b_sf + ((size_t(e) * j.RT + nt) * j.KT + 2 * kb) * 1024,
                                             nkq * 1024, &fullB[sb]);
                                ++ib;
                            }
                            const int sa = ia % NSA, nw = min(kPT, j.S - kPT * pc);
                            if (ia >= NSA) ok = twait(&emptyA[sa], uint32_t(ia / NSA - 1) & 1u, j.err, 32, twA);
                            if (!ok) break;
                            tc::mbar_arrive_expect_tx(&fullA[sa], uint32_t(nw * kTermA));
                            tc::bulk_g2s(ringA + sa * kPieceA,
                                         a_slot(const_cast<uint8_t*>(j.a_img), m, j.KB, kb, j.S, kPT * pc),
                                         nw * kTermA, &fullA[sa]);
                            ++ia;
                        }
                }
            }
            if (twA) {
                long long* tr = j.trace + c * 160 + 64 * j.mode;
                tr[6] = wA;
                tr[7] = wB;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (one thread)
        if (lane == 0) {
            bool ok = true;
            int ia = 0, ib = 0, seg = 0;
            const int npc = (j.S + kPT - 1) / kPT;
            long long wA = 0, wB = 0, wE = 0, t_start = clock64();
            const bool trc = j.trace && c < 160;
            const uint32_t idesc0 = tc::idesc_mxf4(128, kRows, 0, 0), idesc2 = tc::idesc_mxf4(128, kRows, 2, 2);
            for (int tau = c; tau < n_tiles && ok; tau += nc) {
                for (int s0 = 0; s0 < j.KB && ok; s0 += j.seg, ++seg) {
                    const int s1 = min(j.KB, s0 + j.seg);
                    if (seg > 0) ok = twait(accE, uint32_t(seg - 1) & 1u, j.err, 33, trc ? &wE : nullptr);
                    for (int pc = 0; pc < npc && ok; ++pc)
                        for (int kb = s0; kb < s1; ++kb) {
                            const int nw = min(kPT, j.S - kPT * pc);
                            const int nu = min(4, j.UK - 4 * kb), nkq = (nu + 1) / 2;
                            const int sb = (ib + kb - s0) % NSB;
                            const uint8_t* pb = ringB + sb * kPieceB;
                            const uint32_t csfb = tmem + kColSFB + 16 * sb;
                            if (pc == 0) {
                                ok = twait(&fullB[sb], uint32_t((ib + kb - s0) / NSB) & 1u, j.err, 34, trc ? &wB : nullptr);
                                if (!ok) break;
                                tc::tc_fence_after();
                                for (int q = 0; q < nkq; ++q)
                                    for (int hh = 0; hh < 2; ++hh)
                                        tc::tmem_cp_sf(csfb + 8 * q + 4 * hh,
                                                       tc::desc_sf_chunk(tc::smem_u32(pb + kBImg + (2 * q + hh) * 512)));
                            }
                            const int sa = ia % NSA;
                            ok = twait(&fullA[sa], uint32_t(ia / NSA) & 1u, j.err, 35, trc ? &wA : nullptr);
                            if (!ok) break;
                            tc::tc_fence_after();
                            auto slot_mmas = [&](int w) {
                                const uint8_t* pa = ringA + sa * kPieceA + w * kTermA;
                                const uint32_t csfa = tmem + kColSFA + 16 * sa + 8 * w;
                                tmem_cp_128x256b(csfa, desc_sfa_128x256b(tc::smem_u32(pa + kImg)));
                                for (int u = 0; u < nu; ++u) {
                                    const uint32_t sfid = 2u * (u & 1), q = u >> 1;
                                    tc::mma_mxf4(tmem, tc::desc_sw128(tc::smem_u32(pa + u * 32)),
                                                 tc::desc_sw128(tc::smem_u32(pb + u * 32)), (u & 1) ? idesc2 : idesc0,
                                                 (csfa + 4 * q) | (sfid << 30), (csfb + 8 * q) | (sfid << 30),
                                                 !(pc == 0 && w == 0 && kb == s0 && u == 0));
                                }
                            };
                            if (nw == kPT) {                     // a full piece (the common case), unrolled
#pragma unroll
                                for (int w = 0; w < kPT; ++w) slot_mmas(w);
                            } else {
                                for (int w = 0; w < nw; ++w) slot_mmas(w);
                            }
                            tc::mma_commit(&emptyA[sa]);
                            ++ia;
                            if (pc == npc - 1) tc::mma_commit(&emptyB[sb]);
                        }
                    ib += s1 - s0;
                    if (ok) tc::mma_commit(accF);
                }
            }
            if (trc) {
                long long* tr = j.trace + c * 160 + 64 * j.mode;
                tr[0] = t_start;
                tr[1] = wA;
                tr[2] = wB;
                tr[3] = wE;
                tr[4] = seg;
                tr[5] = clock64();
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue warps
        // Thread = one token row of the tile and 128 of the 256 columns: warp w reads TMEM lanes 32 (w % 4) .. + 31,
        // columns 128 hc .. + 127 (hc = 0 for warps 2..5, 1 for warps 6..9). Per segment: D added into sums.
        const int quad = warp & 3, hc = (warp - 2) >> 2, row_t = quad * 32 + lane;
        const uint32_t tl_base = tmem + (uint32_t(quad * 32) << 16) + 128 * hc;
        int seg = 0;
        const bool trc = j.trace && c < 160 && warp == 2 && lane == 0;
        long long wF = 0, tEpi = 0;
        for (int tau = c; tau < n_tiles; tau += nc) {
            const int m = tau / j.RT, nt = tau % j.RT;
            const int4 tl = j.tiles[m];
            float sums[128];
#pragma unroll
            for (int i = 0; i < 128; ++i) sums[i] = 0.f;
            bool ok = true;
            for (int s0 = 0; s0 < j.KB; s0 += j.seg, ++seg) {
                // One thread polls the accumulator barrier; the other epilogue warps sleep in a named barrier.
                if (warp == 2 && lane == 0)
                    epi_flag[seg & 1] = (ok && twait(accF, uint32_t(seg) & 1u, j.err, 36, trc ? &wF : nullptr)) ? 1 : 0;
                epi_bar_sync();
                const bool got = reinterpret_cast<volatile int*>(epi_flag)[seg & 1] != 0;   // two flags: no reuse race
                if (got) {
                    tc::tc_fence_after();
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t v[32];
                        tmem_ld_32x32b_x32(tl_base + 32 * cc, v);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) sums[32 * cc + i] += __uint_as_float(v[i]);
                    }
                }
                ok = got;
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(accE);
            }
            if (!ok) continue;
            const long long te0 = clock64();
            const int e = tl.x;
            const float* bb = j.bias + size_t(e) * j.N;
            const int n0 = nt * kRows + 128 * hc;
            if (j.P > 1) {
                // packed plan: lane q (= row % 8, the term) of the token's 8 lanes ends with the token's sums of
                // columns 16 q .. 16 q + 15 and stores them
                const int tok_t = row_t / kPackRows, q = row_t % kPackRows;
                float r[16];
                pack_reduce_scatter(sums, q, r);
                const int nb = n0 + 16 * q;
                if (tok_t < tl.z && j.mode == 0) {
                    const int ab = nt * (kRows / 2) + 64 * hc + 8 * q;     // activations ab .. ab + 7
                    float* arow = j.act + size_t(tl.y + tok_t) * j.I;
                    if (ab < j.I) {
                        float o[8];
#pragma unroll
                        for (int d = 0; d < 8; ++d) {
                            const int n = min(nb + 2 * d, j.N - 2);           // I % 64 == 0: never clamped
                            const float gv = fminf(r[2 * d] + __ldg(bb + n), j.limit);
                            const float lv = fminf(fmaxf(r[2 * d + 1] + __ldg(bb + (n + 1)), -j.limit), j.limit);
                            o[d] = __fdividef(gv, 1.f + __expf(-j.alpha * gv)) * (lv + 1.f);
                        }
                        if (ab + 7 < j.I) {
                            *reinterpret_cast<float4*>(arow + ab) = make_float4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<float4*>(arow + ab + 4) = make_float4(o[4], o[5], o[6], o[7]);
                        } else {
                            for (int d = 0; d < 8; ++d)
                                if (ab + d < j.I) arow[ab + d] = o[d];
                        }
                    }
                } else if (tok_t < tl.z && j.mode == 1 && nb < j.N) {
                    const int row = tl.y + tok_t, t = j.tok_of[row], s = j.slot_of[row];
                    const float w = j.wts[size_t(t) * j.k + s];
                    float* orow = j.out_ts + (size_t(t) * j.k + s) * j.N;
                    if (nb + 16 <= j.N) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4) {
                            float4 o;
                            o.x = w * (r[i] + __ldg(bb + (nb + i)));
                            o.y = w * (r[i + 1] + __ldg(bb + (nb + i + 1)));
                            o.z = w * (r[i + 2] + __ldg(bb + (nb + i + 2)));
                            o.w = w * (r[i + 3] + __ldg(bb + (nb + i + 3)));
                            *reinterpret_cast<float4*>(orow + nb + i) = o;
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (nb + i < j.N) orow[nb + i] = w * (r[i] + __ldg(bb + (nb + i)));
                    }
                }
            } else if (j.mode == 0 && row_t < tl.z) {
                // columns n0 .. n0 + 127 = 64 (gate, up) pairs = activations 64 (2 nt + hc) .. + 63
                const int a0 = nt * (kRows / 2) + 64 * hc;
                float* arow = j.act + size_t(tl.y + row_t) * j.I + a0;
                if (a0 < j.I) {
#pragma unroll
                    for (int i = 0; i < 64; i += 4) {
                        float o[4];
#pragma unroll
                        for (int d = 0; d < 4; ++d) {
                            const int n = min(n0 + 2 * (i + d), j.N - 2);     // I % 64 == 0: never clamped
                            const float gv = fminf(sums[2 * (i + d)] + __ldg(bb + (n)), j.limit);
                            const float lv = fminf(fmaxf(sums[2 * (i + d) + 1] + __ldg(bb + (n + 1)), -j.limit), j.limit);
                            o[d] = __fdividef(gv, 1.f + __expf(-j.alpha * gv)) * (lv + 1.f);
                        }
                        if (a0 + i + 3 < j.I) *reinterpret_cast<float4*>(arow + i) = make_float4(o[0], o[1], o[2], o[3]);
                        else
                            for (int d = 0; d < 4; ++d)
                                if (a0 + i + d < j.I) arow[i + d] = o[d];
                    }
                }
            } else if (j.mode == 1 && row_t < tl.z && n0 < j.N) {
                const int row = tl.y + row_t;
                float w;
                float* orow;
                if (j.meta) {                        // the row came from rank src: its result goes back there
                    const int4 mt = j.meta[row];
                    w = __int_as_float(mt.w);
                    orow = j.out_rank[mt.x & 7] + (size_t(mt.y) * j.k + mt.z) * j.N;
                } else {
                    const int t = j.tok_of[row], s = j.slot_of[row];
                    w = j.wts[size_t(t) * j.k + s];
                    orow = j.out_ts + (size_t(t) * j.k + s) * j.N;
                }
                if (n0 + 128 <= j.N) {
#pragma unroll
                    for (int i = 0; i < 128; i += 4) {
                        float4 o;
                        o.x = w * (sums[i] + __ldg(bb + (n0 + i)));
                        o.y = w * (sums[i + 1] + __ldg(bb + (n0 + i + 1)));
                        o.z = w * (sums[i + 2] + __ldg(bb + (n0 + i + 2)));
                        o.w = w * (sums[i + 3] + __ldg(bb + (n0 + i + 3)));
                        *reinterpret_cast<float4*>(orow + n0 + i) = o;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 128; ++i)
                        if (n0 + i < j.N) orow[n0 + i] = w * (sums[i] + __ldg(bb + (n0 + i)));
                }
            }
            if (trc) tEpi += clock64() - te0;
        }
        if (j.meta) __threadfence_system();                  // expert parallel: result rows went to peers
        if (trc) {
            long long* tr = j.trace + c * 160 + 64 * j.mode;
            tr[8] = wF;
            tr[9] = tEpi;
            tr[10] = clock64();
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

// The same four values per thread (H % 4 == 0, both arrays 16-byte aligned); each value's additions in the same order.
__global__ void combine4_kernel(const float4* __restrict__ out_ts, int T, int k, int H4, float4* __restrict__ x_resid) {
    const long long n = (long long)T * H4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / H4, h = i - t * H4;
        float4 acc = x_resid[i];
        for (int s = 0; s < k; ++s) {
            const float4 o = out_ts[(t * k + s) * H4 + h];
            acc.x += o.x;
            acc.y += o.y;
            acc.z += o.z;
            acc.w += o.w;
        }
        x_resid[i] = acc;
    }
}

// x_resid[t] += the k result rows of token t, slot by slot.
void launch_combine(const float* out_ts, int T, int k, int H, float* x_resid, int grid, cudaStream_t s) {
    if (H % 4 == 0 && ((reinterpret_cast<uintptr_t>(out_ts) | reinterpret_cast<uintptr_t>(x_resid)) & 15) == 0)
        combine4_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(out_ts), T, k, H / 4,
                                             reinterpret_cast<float4*>(x_resid));
    else
        combine_kernel<<<grid, 256, 0, s>>>(out_ts, T, k, H, x_resid);
}

// ------------------------------------------------------------------------------------------------ expert parallel
// The batched MoE with the experts spread over G ranks (one GPU each), tokens split over the ranks. Every rank
// allocates one zero-initialised "region" (cudaMalloc, shared with the others through CUDA IPC) and gets every
// peer's region mapped into its address space (NVLink peer memory). Per layer call:
//   counts:   each rank counts its (token, slot) pairs per expert and writes its row of the count matrix into every
//             region; barrier 0;
//   permute:  from the full count matrix every rank knows where each of its pairs goes: rows of an expert on its
//             owner are ordered by source rank, then by the source's token order, cut into 128-row tiles; the pair's
//             (source rank, token, slot, gate weight) is written to the owner's row metadata;
//   dispatch: the h quantizer writes each token's A terms straight into the owners' A images (the data crosses
//             NVLink once, as e2m1 terms); barrier 1;
//   compute:  each rank runs the grouped GEMMs over the rows it received; the down epilogue writes every row's
//             w (y + b2) straight into its source rank's result rows; barrier 2;
//   combine:  each rank adds its result rows into its residual stream in slot order.
// Every row's computation and the combine order are those of the single-GPU batched forward, so the result is
// bit-identical to it. Barriers are epoch flags (release / acquire at system scope) with bounded waits.
constexpr int kMaxRanks = 8;

struct EpDev {
    uint8_t* base[kMaxRanks];                  // every rank's region as mapped on this device (base[rank] = own)
    int rank, G, E, El;
    size_t off_flags, off_counts, off_meta;
    unsigned epoch;
    int* err;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread: tells every rank (flag `which` of its region, slot = this rank) that this rank reached the barrier in
// layer call `epoch`, after a system-scope fence that orders everything this rank's earlier kernels wrote; then waits
// (bounded: about a second) until every rank did the same. Epochs only grow, so a flag at or past `epoch` counts.
__device__ void ep_barrier(const EpDev& d, int which) {
    __threadfence_system();
    for (int r = 0; r < d.G; ++r)
        st_release_sys(reinterpret_cast<unsigned*>(d.base[r] + d.off_flags) + which * kMaxRanks + d.rank, d.epoch);
    const unsigned* own = reinterpret_cast<const unsigned*>(d.base[d.rank] + d.off_flags) + which * kMaxRanks;
    for (int r = 0; r < d.G; ++r) {
        bool ok = false;
        for (uint32_t i = 0; i < (1u << 24) && !ok; ++i) {
            ok = ld_acquire_sys(own + r) >= d.epoch;
            if (!ok) __nanosleep(64);
        }
        if (!ok) {
            atomicCAS(d.err, 0, 60 + which);
            return;
        }
    }
}

__global__ void ep_barrier_kernel(const __grid_constant__ EpDev d, int which) {
    if (threadIdx.x == 0) ep_barrier(d, which);
}

// Counts of this rank's (token, slot) pairs per expert -> row `rank` of every region's count matrix; barrier 0.
__global__ void __launch_bounds__(256) ep_counts_kernel(const int* __restrict__ ids, int T, int k,
                                                        const __grid_constant__ EpDev d) {
    __shared__ int cnt[32];
    const int tid = threadIdx.x;
    if (tid < 32) cnt[tid] = 0;
    __syncthreads();
    bool bad = false;
    for (int i = tid; i < T * k; i += blockDim.x) {
        const int e = ids[i];
        if (e < 0 || e >= d.E) bad = true;
        else atomicAdd(&cnt[e], 1);
    }
    if (bad) atomicCAS(d.err, 0, 20);
    __syncthreads();
    if (tid < 32) {
        for (int r = 0; r < d.G; ++r)
            reinterpret_cast<int*>(d.base[r] + d.off_counts)[d.rank * 32 + tid] = tid < d.E ? cnt[tid] : 0;
        __threadfence_system();                              // peer stores ordered before the barrier's flags
    }
    __syncthreads();
    if (tid == 0) ep_barrier(d, 0);
}

// One CTA of 1024 threads. Local tiles: this rank's experts' received rows in 128-row tiles, tiles[m] = (local
// expert, 128 m, rows). Own pairs: pos_of / dest_of (tile row on the owner, owner rank), and the owner's metadata
// row = (this rank, token, slot, gate weight). Thread i owns tokens [i * per, (i + 1) * per); per-expert counts are
// scanned over the threads (expert e by warp e), as in permute_kernel.
__global__ void __launch_bounds__(1024) ep_permute_kernel(const int* __restrict__ ids, const float* __restrict__ wts,
                                                          int T, int k, const __grid_constant__ EpDev d,
                                                          int* __restrict__ pos_of, int* __restrict__ dest_of,
                                                          int4* __restrict__ tiles, int* __restrict__ n_tiles) {
    extern __shared__ unsigned short cnt_raw[];
    unsigned short (*cnt)[1024] = reinterpret_cast<unsigned short (*)[1024]>(cnt_raw);   // [32][1024]
    __shared__ int before[32], tile0[32], total[32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int* C = reinterpret_cast<const int*>(d.base[d.rank] + d.off_counts);          // [G][32]
    if (tid < 32) {
        int tot = 0, bef = 0;
        for (int r = 0; r < d.G; ++r) {
            const int c = tid < d.E ? C[r * 32 + tid] : 0;
            tot += c;
            if (r < d.rank) bef += c;
        }
        total[tid] = tot;
        before[tid] = bef;
    }
    __syncthreads();
    if (tid == 0) {
        int m = 0;
        for (int e = 0; e < d.E; ++e) {
            if (e % d.El == 0) m = 0;                       // tile numbers restart on every owner
            tile0[e] = m;
            const bool mine = e / d.El == d.rank;
            for (int r = 0; r < total[e]; r += kTileM) {
                if (mine) tiles[m] = make_int4(e - d.rank * d.El, m * kTileM, min(kTileM, total[e] - r), 0);
                ++m;
            }
            if (mine && (e + 1) % d.El == 0) *n_tiles = m;
        }
    }
    const int per = (T + 1023) / 1024, tb = min(T, tid * per), te = min(T, tb + per);
    for (int e = 0; e < 32; ++e) cnt[e][tid] = 0;
    for (int t = tb; t < te; ++t)
        for (int s = 0; s < k; ++s) {
            const int e = ids[size_t(t) * k + s];
            if (e >= 0 && e < d.E) ++cnt[e][tid];
        }
    __syncthreads();
    {
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
    }
    __syncthreads();
    for (int t = tb; t < te; ++t)
        for (int s = 0; s < k; ++s) {
            const size_t i = size_t(t) * k + s;
            const int e = ids[i];
            if (e < 0 || e >= d.E) {
                pos_of[i] = -1;
                dest_of[i] = 0;
                continue;
            }
            const int r = before[e] + cnt[e][tid];
            cnt[e][tid] = (unsigned short)(cnt[e][tid] + 1);
            const int owner = e / d.El;
            const int pos = (tile0[e] + r / kTileM) * kTileM + r % kTileM;
            pos_of[i] = pos;
            dest_of[i] = owner;
            reinterpret_cast<int4*>(d.base[owner] + d.off_meta)[pos] = make_int4(d.rank, t, s, __float_as_int(wts[i]));
        }
    __threadfence_system();
}

constexpr int kGemmSmem = 1024 + NSA * kPieceA + NSB * kPieceB + (2 * NSA + 2 * NSB + 2) * 8 + 32;
static_assert(kGemmSmem <= 227 * 1024, "shared memory budget");

}  // namespace pf

// ---------------------------------------------------------------------------------------------------- host API
PrefillLayout prefill_layout(int T, int k, int E, int H, int I) {
    PrefillLayout L{};
    auto al = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    const long long rows = (long long)T * k;
    // Sized for either term plan: tiles of 16 rows (packed) and, per (tile, K block), NT slots of 128-row tiles
    // (stacked; at least the packed plan's tiles x 1 slot).
    const int tiles_stacked = int((rows + pf::kTileM - 1) / pf::kTileM) + E;
    L.max_tiles = int((rows + pf::kTileM / pf::kPackRows - 1) / (pf::kTileM / pf::kPackRows)) + E;
    const size_t img_slots = size_t(tiles_stacked) * pf::NT;
    L.KB_gu = (H + 255) / 256;
    L.KB_dn = (I + 255) / 256;
    size_t o = 0;
    L.off_h = o; o += al(size_t(T) * H * 4);
    L.off_ids = o; o += al(size_t(rows) * 4);
    L.off_w = o; o += al(size_t(rows) * 4);
    L.off_pos_of = o; o += al(size_t(rows) * 4);
    L.off_tok_of = o; o += al(size_t(rows) * 4);
    L.off_slot_of = o; o += al(size_t(rows) * 4);
    L.off_tiles = o; o += al(size_t(L.max_tiles) * 16);
    L.off_misc = o; o += 1024;                              // [0] tile count, [64] error word
    L.off_img_gu = o; o += al(img_slots * L.KB_gu * pf::kTermA);
    L.off_img_dn = o; o += al(img_slots * L.KB_dn * pf::kTermA);
    L.off_out = o; o += al(size_t(rows) * std::max(H, I) * 4);   // activations, then the (token, slot) results
    L.off_w64 = o; o += al(size_t(H) * 32 * 8);
    L.bytes = o;
    return L;
}

void launch_router_w64(const void* W, int E, int H, double* W64, cudaStream_t s) {
    const int grid = std::min((H * 32 + 255) / 256, num_sms() * 4);
    pf::router_w64_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(W), E, H, W64);
    check_launch("router_w64");
}

// CTAs per token group of the batched router: as many (up to kRtMaxSplit, a power of two) as keep the grid within one
// wave of SMs.
static int router_split(int T) {
    const int groups = (T + pf::kRtTok - 1) / pf::kRtTok, sms = num_sms();
    int KS = 1;
    while (KS < pf::kRtMaxSplit && groups * KS * 2 <= sms) KS *= 2;
    return KS;
}

void launch_router_batched(const double* W64, const float* b, const float* x, const float* norm_w, float eps, int T,
                           int E, int H, int k, float* h_out, int* ids, float* wts, cudaStream_t s) {
    require(T >= 1, "router_batched: T must be positive");
    require(H % 8 == 0 && H >= 8, "router_batched: H must be a positive multiple of 8");
    require(k >= 1 && k <= 8 && k <= E && E <= 32, "router_batched: needs 1 <= k <= 8 and k <= E <= 32");
    const int KS = router_split(T);
    const int smem = pf::router_smem_bytes(H, KS);
    require(smem <= 220 * 1024, "router_batched: H too large");
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
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((T + pf::kRtTok - 1) / pf::kRtTok) * KS);
    cfg.blockDim = dim3(512);
    cfg.dynamicSmemBytes = size_t(smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(KS);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = KS > 1 ? 1 : 0;
    GPT_CHECK(cudaLaunchKernelEx(&cfg, pf::router_batched_kernel, W64, b, x, norm_w, eps, T, E, H, k, KS, h_out, ids,
                                 wts));
    check_launch("router_batched");
}

void launch_moe_batched(const PrefillArgs& a, cudaStream_t s) {
    using namespace pf;
    require(a.T >= 1, "moe_batched: T must be positive");
    require(a.k >= 1 && a.k <= 8 && a.k <= a.E && a.E <= 32, "moe_batched: needs 1 <= k <= 8 and k <= E <= 32");
    require(a.H % 64 == 0 && a.I % 64 == 0, "moe_batched: H and I must be multiples of 64");
    require(a.T <= 32768, "moe_batched: at most 32768 tokens per call");
    require(a.terms >= 1 && a.terms <= NT && (a.pack == 0 || a.pack == 1), "moe_batched: bad term plan");
    const TermPlan tp = a.pack ? TermPlan{a.terms, 1, kPackRows} : TermPlan{a.terms, a.terms, 1};
    const PrefillLayout L = prefill_layout(a.T, a.k, a.E, a.H, a.I);
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    int* pos_of = reinterpret_cast<int*>(ws + L.off_pos_of);
    int* tok_of = reinterpret_cast<int*>(ws + L.off_tok_of);
    int* slot_of = reinterpret_cast<int*>(ws + L.off_slot_of);
    int4* tiles = reinterpret_cast<int4*>(ws + L.off_tiles);
    int* n_tiles = reinterpret_cast<int*>(ws + L.off_misc);
    int* err = reinterpret_cast<int*>(ws + L.off_misc + 64 * 4);
    uint8_t* img_gu = ws + L.off_img_gu;
    uint8_t* img_dn = ws + L.off_img_dn;
    float* out = reinterpret_cast<float*>(ws + L.off_out);
    const int sms = num_sms();

    static std::mutex mu;
    static std::map<int, bool> done;
    {
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lock(mu);
        if (!done[dev]) {
            GPT_CHECK(cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 32 * 1024 * 2));
            GPT_CHECK(cudaFuncSetAttribute(grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
            done[dev] = true;
        }
    }
    permute_kernel<<<1, 1024, 32 * 1024 * 2, s>>>(a.ids, a.T, a.k, a.E, tp.P, pos_of, tok_of, slot_of, tiles, n_tiles,
                                                  err);
    check_launch("moe_batched permute");
    ImgBases ib{};
    for (int r = 0; r < 8; ++r) ib.p[r] = img_gu;
    quantize_h_kernel<<<sms * 8, 256, 0, s>>>(a.h, a.T, a.H, a.k, pos_of, nullptr, L.KB_gu, ib, tp);
    check_launch("moe_batched quantize");
    for (int pass = 0; pass < 2; ++pass) {
        const bool gu = pass == 0;
        const int K = gu ? a.H : a.I, N = gu ? 2 * a.I : a.H;
        GemmJob g{};
        g.mode = gu ? 0 : 1;
        g.K = K;
        g.N = N;
        g.UK = K / 64;
        g.KB = gu ? L.KB_gu : L.KB_dn;
        g.KT = (K + 127) / 128;
        g.RT = (N + kRows - 1) / kRows;
        g.a_img = gu ? img_gu : img_dn;
        g.S = tp.S;
        g.P = tp.P;
        g.seg = tp.S == 1 ? g.KB : kSeg;          // one slot per K block: B pieces are used once, any segment fits
        g.b_sf = gu ? a.sf_gu : a.sf_dn;
        g.tiles = tiles;
        g.n_tiles = n_tiles;
        g.bias = gu ? a.gu_bias : a.dn_bias;
        g.alpha = a.alpha;
        g.limit = a.limit;
        g.act = out;                                       // consumed by quantize_act before the down GEMM
        g.I = a.I;
        g.tok_of = tok_of;
        g.slot_of = slot_of;
        g.wts = a.weights;
        g.k = a.k;
        g.out_ts = out;
        g.err = err;
        g.trace = a.trace;
        auto rec = [&](int i) {
            if (a.events)
                GPT_CHECK(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(a.events[i]), s, cudaEventRecordExternal));
        };
        rec(2 * pass);
        grouped_gemm_kernel<<<sms, kThreads, kGemmSmem, s>>>(gu ? *a.tmap_gu : *a.tmap_dn, g);
        check_launch("moe_batched grouped gemm");
        rec(2 * pass + 1);
        if (gu) {
            quantize_act_kernel<<<sms * 8, 256, 0, s>>>(out, a.I, tiles, n_tiles, L.KB_dn, img_dn, tp);
            check_launch("moe_batched quantize act");
        }
    }
    launch_combine(out, a.T, a.k, a.H, a.x_resid, sms * 8, s);
    check_launch("moe_batched combine");
}


EpLayout ep_layout(int T_max, int k, int E, int world, int H, int I) {
    EpLayout L{};
    auto al = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    require(world >= 1 && world <= pf::kMaxRanks && E % world == 0, "ep: 1 <= world <= 8 and E % world == 0");
    const int El = E / world;
    L.max_rows = (long long)world * T_max * k;
    L.max_tiles = int((L.max_rows + pf::kTileM - 1) / pf::kTileM) + El;
    L.KB_gu = (H + 255) / 256;
    L.KB_dn = (I + 255) / 256;
    size_t o = 0;                                            // the shared region
    L.off_flags = o; o += 1024;                              // [3][8] epoch flags
    L.off_counts = o; o += al(size_t(pf::kMaxRanks) * 32 * 4);
    L.off_meta = o; o += al(size_t(L.max_tiles) * pf::kTileM * 16);
    L.off_img = o; o += al(size_t(L.max_tiles) * L.KB_gu * pf::NT * pf::kTermA);
    L.off_out = o; o += al(size_t(T_max) * k * H * 4);
    L.region_bytes = o;
    o = 0;                                                   // this rank's private workspace
    L.off_h = o; o += al(size_t(T_max) * H * 4);
    L.off_ids = o; o += al(size_t(T_max) * k * 4);
    L.off_w = o; o += al(size_t(T_max) * k * 4);
    L.off_pos = o; o += al(size_t(T_max) * k * 4);
    L.off_dest = o; o += al(size_t(T_max) * k * 4);
    L.off_tiles = o; o += al(size_t(L.max_tiles) * 16);
    L.off_misc = o; o += 1024;                               // [0] tile count, [64] error word
    L.off_img_dn = o; o += al(size_t(L.max_tiles) * L.KB_dn * pf::NT * pf::kTermA);
    L.off_act = o; o += al(size_t(L.max_tiles) * pf::kTileM * I * 4);
    L.local_bytes = o;
    return L;
}

void launch_ep_layer(const EpArgs& a, cudaStream_t s) {
    using namespace pf;
    require(a.T >= 0 && a.T <= a.T_max && a.T_max <= 32768, "ep: 0 <= T <= T_max <= 32768");
    require(a.k >= 1 && a.k <= 8 && a.E <= 32 && a.rank >= 0 && a.rank < a.world, "ep: bad k, E or rank");
    require(a.H % 64 == 0 && a.I % 64 == 0, "ep: H and I must be multiples of 64");
    require(a.terms >= 1 && a.terms <= NT, "ep: terms must be 1 .. 8");
    const TermPlan tp{a.terms, a.terms, 1};                  // stacked: the peers' row metadata is per row
    const EpLayout L = ep_layout(a.T_max, a.k, a.E, a.world, a.H, a.I);
    uint8_t* ws = static_cast<uint8_t*>(a.local_ws);
    float* h = reinterpret_cast<float*>(ws + L.off_h);
    int* ids = reinterpret_cast<int*>(ws + L.off_ids);
    float* wts = reinterpret_cast<float*>(ws + L.off_w);
    int* pos_of = reinterpret_cast<int*>(ws + L.off_pos);
    int* dest_of = reinterpret_cast<int*>(ws + L.off_dest);
    int4* tiles = reinterpret_cast<int4*>(ws + L.off_tiles);
    int* n_tiles = reinterpret_cast<int*>(ws + L.off_misc);
    int* err = reinterpret_cast<int*>(ws + L.off_misc + 64 * 4);
    uint8_t* img_dn = ws + L.off_img_dn;
    float* act = reinterpret_cast<float*>(ws + L.off_act);
    uint8_t* own = static_cast<uint8_t*>(a.peers[a.rank]);
    const int sms = num_sms();

    EpDev d{};
    for (int r = 0; r < a.world; ++r) d.base[r] = static_cast<uint8_t*>(a.peers[r]);
    d.rank = a.rank;
    d.G = a.world;
    d.E = a.E;
    d.El = a.E / a.world;
    d.off_flags = L.off_flags;
    d.off_counts = L.off_counts;
    d.off_meta = L.off_meta;
    d.epoch = a.epoch;
    d.err = err;

    static std::mutex mu;
    static std::map<int, bool> done;
    {
        int dev = 0;
        GPT_CHECK(cudaGetDevice(&dev));
        std::lock_guard<std::mutex> lock(mu);
        if (!done[dev]) {
            GPT_CHECK(cudaFuncSetAttribute(ep_permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 32 * 1024 * 2));
            GPT_CHECK(cudaFuncSetAttribute(grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
            done[dev] = true;
        }
    }
    GPT_CHECK(cudaMemsetAsync(ws + L.off_misc, 0, 1024, s));
    if (a.T > 0)
        launch_router_batched(a.w64, a.router_b, a.x, a.norm_w, a.eps, a.T, a.E, a.H, a.k, h, ids, wts, s);
    ep_counts_kernel<<<1, 256, 0, s>>>(ids, a.T, a.k, d);
    check_launch("ep counts");
    ep_permute_kernel<<<1, 1024, 32 * 1024 * 2, s>>>(ids, wts, a.T, a.k, d, pos_of, dest_of, tiles, n_tiles);
    check_launch("ep permute");
    if (a.T > 0) {
        ImgBases ib{};
        for (int r = 0; r < kMaxRanks; ++r) ib.p[r] = r < a.world ? d.base[r] + L.off_img : nullptr;
        quantize_h_kernel<<<sms * 8, 256, 0, s>>>(h, a.T, a.H, a.k, pos_of, dest_of, L.KB_gu, ib, tp);
        check_launch("ep dispatch");
    }
    ep_barrier_kernel<<<1, 32, 0, s>>>(d, 1);
    check_launch("ep barrier 1");
    for (int pass = 0; pass < 2; ++pass) {
        const bool gu = pass == 0;
        const int K = gu ? a.H : a.I, N = gu ? 2 * a.I : a.H;
        GemmJob g{};
        g.mode = gu ? 0 : 1;
        g.K = K;
        g.N = N;
        g.UK = K / 64;
        g.KB = gu ? L.KB_gu : L.KB_dn;
        g.KT = (K + 127) / 128;
        g.RT = (N + kRows - 1) / kRows;
        g.a_img = gu ? own + L.off_img : img_dn;
        g.S = tp.S;
        g.P = tp.P;
        g.seg = tp.S == 1 ? g.KB : kSeg;          // one slot per K block: B pieces are used once, any segment fits
        g.b_sf = gu ? a.sf_gu : a.sf_dn;
        g.tiles = tiles;
        g.n_tiles = n_tiles;
        g.bias = gu ? a.gu_bias : a.dn_bias;
        g.alpha = a.alpha;
        g.limit = a.limit;
        g.act = act;
        g.I = a.I;
        g.k = a.k;
        g.meta = reinterpret_cast<const int4*>(own + L.off_meta);
        for (int r = 0; r < a.world; ++r) g.out_rank[r] = reinterpret_cast<float*>(d.base[r] + L.off_out);
        g.err = err;
        g.trace = a.trace;
        grouped_gemm_kernel<<<sms, kThreads, kGemmSmem, s>>>(gu ? *a.tmap_gu : *a.tmap_dn, g);
        check_launch("ep grouped gemm");
        if (gu) {
            quantize_act_kernel<<<sms * 8, 256, 0, s>>>(act, a.I, tiles, n_tiles, L.KB_dn, img_dn, tp);
            check_launch("ep quantize act");
        }
    }
    ep_barrier_kernel<<<1, 32, 0, s>>>(d, 2);
    check_launch("ep barrier 2");
    if (a.T > 0) {
        launch_combine(reinterpret_cast<const float*>(own + L.off_out), a.T, a.k, a.H, a.x_resid, sms * 8, s);
        check_launch("ep combine");
    }
}

}  // namespace gpt
