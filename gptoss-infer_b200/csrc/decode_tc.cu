// Tensor-core decode MoE (one token): the MXFP4 expert GEMVs on tcgen05 kind::mxf4.
//
// Operands. A = expert weights straight from the checkpoint layout (128 rows x 128 bytes of K per TMA box, 128-byte
// swizzle), scales repacked into 512-byte tcgen05 chunks. B = the activation vector split into R = 16 e2m1 residual
// terms, each with its own E8M0 scale per 32 elements (x = sum of terms to about 2^-30 of each block's maximum), so
// the MMA's N = 16 columns hold the terms and the tensor core performs the MXFP4 dequantization; the epilogue sums
// the 16 columns. B tiles are written pre-swizzled by the kernel that produces them and copied with bulk copies.
//
// Work split ("stream-K"). The MMA unit is K = 64 of one 128-row tile. Units are laid out tile by tile; every CTA
// takes a contiguous range rounded to 4-unit stages (one TMA box), so each CTA streams the same number of bytes
// within one stage. A tile split between CTAs is reduced by the last CTA to finish it (an atomic unit count; partial
// sums stored per contributor and added in CTA order, so the result is deterministic); nothing ever spins on
// another CTA.
//
// Gate/up: tile = (slot, 128 rows of W1[ids[slot]]); the finishing CTA applies bias, the clamped SwiGLU (rows 2j glu,
// 2j+1 linear), multiplies by the slot's gate weight and writes the result directly as the down kernel's B terms.
// Down: tile = 128 rows of the output, K' = k * I: the k experts' rows are one long GEMV because B already carries
// the gate weights, so one accumulator holds sum_slot W2[e] (w a); the finishing CTA adds sum_slot w b2 and the
// residual. Gate/up -> down uses programmatic dependent launch: down CTAs start early and stream their weights
// while gate/up drains.
#include <algorithm>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"
#include "terms.cuh"
#include "tma.h"

namespace gpt {
namespace dtc {

constexpr int R = kDecodeTerms;               // residual terms = MMA N
constexpr int kThreads = 192;                 // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kMaxContrib = 16;               // CTAs that may share one tile
constexpr int kMaxStages = 96;                // per-CTA stage list capacity
constexpr int kA = 16384, kB = R * 128, kSF = 1024;
constexpr int kStageBytes = kA + kB + 2 * kSF;
constexpr uint32_t kTmemCols = 64;            // 2 x R accumulator columns + 8 SFA + 8 SFB

enum Mode { kGateUp = 0, kDown = 1 };

struct Job {
    int mode;
    int n_tiles;            // gate/up: k * RT; down: RT
    int RT;                 // 128-row tiles per expert matrix
    int UK;                 // MMA units (K = 64) per slot
    int KT;                 // scale chunks per row (K = 128 each)
    int SPS;                // stages per slot
    int k;                  // slots (selected experts)
    int UT;                 // units per tile: gate/up UK, down k * UK
    long long total;        // n_tiles * UT
    const uint8_t* sfa;     // [mat][RT][KT][512]
    int sfa_by_slot;        // mat = slot (1) or ids[slot] (0)
    const uint8_t* bimg;    // B terms: gate/up [SPS][R*128]; down [k][SPS][R*128]
    const uint8_t* bsf;     // B scale chunks: gate/up [KT][512]; down [k][KT][512]
    const float* bias;      // gate/up [E][2I]; down [E][H]
    const int* ids;
    const float* gate_w;
    float* partial;         // [n_tiles][kMaxContrib][128]
    unsigned* cnt;          // [n_tiles], zero between launches
    uint8_t* out_img;       // gate/up: down's B terms [k][SPS_dn][R*128]
    uint8_t* out_sf;        // gate/up: down's B scales [k][KT_dn][512]
    int out_SPS, out_KT;
    float* x_resid;         // down: residual stream [H]
    int rows;               // rows per expert matrix (gate/up 2I, down H)
    float alpha, limit;
    int* err;
};

struct Stage {
    int tile;
    short s, ku0, nu;       // slot, first unit in the slot, units in this stage
    short first, last;      // first / last stage of this CTA's segment of the tile
    int seg;                // segment index within this CTA
};

__device__ __forceinline__ long long stage_round(const Job& j, long long u) {
    const long long t = u / j.UT;
    const int m = int(u - t * j.UT);
    const int s = m / j.UK, ku = m - s * j.UK;
    const int ku2 = min(j.UK, (ku + 3) & ~3);
    return t * j.UT + (long long)s * j.UK + ku2;
}

__device__ __forceinline__ long long cta_begin(const Job& j, int c) {
    return stage_round(j, (long long)c * j.total / gridDim.x);
}

// CTAs whose ranges intersect tile t: [c_first, c_last].
__device__ void tile_contributors(const Job& j, int t, int& c_first, int& c_last) {
    const long long T0 = (long long)t * j.UT, T1 = T0 + j.UT;
    const int nc = gridDim.x;
    int c = int(T0 * nc / j.total);
    c = min(max(c, 0), nc - 1);
    while (c > 0 && cta_begin(j, c) > T0) --c;
    while (c + 1 < nc && cta_begin(j, c + 1) <= T0) ++c;
    c_first = c;
    int d = int((T1 - 1) * nc / j.total);
    d = min(max(d, c_first), nc - 1);
    while (d > c_first && cta_begin(j, d) > T1 - 1) --d;
    while (d + 1 < nc && cta_begin(j, d + 1) <= T1 - 1) ++d;
    c_last = d;
}

// AND of a predicate over the 128 epilogue threads (named barrier 1).
__device__ __forceinline__ bool epi_all(bool p) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r)
                 : "r"(uint32_t(p))
                 : "memory");
    return r != 0;
}

}  // namespace dtc

namespace dtc {

__global__ void quantize_terms_kernel(const float* __restrict__ x, int n, uint8_t* img, uint8_t* sf) {
    const int warps = blockDim.x / 32;
    quantize_vector_terms_warp(x, n, img, sf, blockIdx.x * warps + threadIdx.x / 32, gridDim.x * warps);
}

// ---------------------------------------------------------------------------------------------------- GEMV
__global__ void __launch_bounds__(kThreads, 1) moe_gemv_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                  const __grid_constant__ Job j, int NS) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ringA = smem;                                   // NS x 16 KB
    uint8_t* ringB = ringA + NS * kA;                         // NS x R*128
    uint8_t* ringSFA = ringB + NS * kB;                       // NS x 1 KB
    uint8_t* ringSFB = ringSFA + NS * kSF;                    // NS x 1 KB
    uint64_t* fullA = reinterpret_cast<uint64_t*>(ringSFB + NS * kSF);
    uint64_t* fullB = fullA + NS;
    uint64_t* empty = fullB + NS;
    uint64_t* accF = empty + NS;                             // [2]
    uint64_t* accE = accF + 2;                               // [2]
    uint32_t* holder = reinterpret_cast<uint32_t*>(accE + 2);
    int* nst_s = reinterpret_cast<int*>(holder + 2);
    int* flag = nst_s + 1;
    float* aval = reinterpret_cast<float*>(flag + 3);        // [64]
    Stage* stages = reinterpret_cast<Stage*>(aval + 64);     // [kMaxStages]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x;

    if (tid == 0) {
        // This CTA's stage list: its unit range [B0, B1) cut at tile boundaries into segments, each cut into
        // 4-unit stages that never cross a slot boundary.
        const long long B0 = cta_begin(j, c), B1 = cta_begin(j, c + 1);
        int n = 0, seg = 0;
        for (long long u = B0; u < B1;) {
            const int t = int(u / j.UT);
            const long long Tend = (long long)(t + 1) * j.UT;
            const long long e = B1 < Tend ? B1 : Tend;
            int m = int(u - (long long)t * j.UT);
            const int m_end = int(e - (long long)t * j.UT);
            const int first_idx = n;
            while (m < m_end && n < kMaxStages) {
                const int s = j.mode == kGateUp ? t / j.RT : m / j.UK;
                const int ku = j.mode == kGateUp ? m : m - s * j.UK;
                const int nu = min(4, min(j.UK - ku, m_end - m));
                stages[n] = Stage{t, short(s), short(ku), short(nu), short(n == first_idx), 0, seg};
                m += nu;
                ++n;
            }
            if (n > first_idx) stages[n - 1].last = 1;
            ++seg;
            u = e;
        }
        if (n >= kMaxStages && cta_begin(j, c) < cta_begin(j, c + 1) && stages[n - 1].last == 0)
            atomicCAS(j.err, 0, 100);                        // stage list overflow: host sizing bug
        *nst_s = n;
        for (int i = 0; i < NS; ++i) {
            tc::mbar_init(&fullA[i], 1);
            tc::mbar_init(&fullB[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
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
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const int nst = *nst_s;
    const uint32_t tmem = *holder;
    if (j.mode == kGateUp) {              // ids, gate weights and B terms come from the router
        pdl_wait();
        pdl_launch_dependents();
    }
    const uint32_t tm_acc = tmem, tm_sfa = tmem + 2 * R, tm_sfb = tmem + 2 * R + 8;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            tc::prefetch_tmap(&tmA);
            const bool split = j.mode == kDown;            // down's B comes from the previous kernel
            auto issueA = [&](int it) {
                const Stage& st = stages[it];
                const int slot = it % NS;
                const int e = j.ids[st.s];
                const int rt = j.mode == kGateUp ? st.tile % j.RT : st.tile;
                const int kt0 = st.ku0 / 2, nkt = (st.ku0 + st.nu - 1) / 2 - kt0 + 1;
                const int mat = j.sfa_by_slot ? st.s : e;
                tc::mbar_arrive_expect_tx(&fullA[slot], kA + nkt * 512);
                tc::tma_load_3d(ringA + slot * kA, &tmA, (st.ku0 / 4) * 128, rt * 128, e, &fullA[slot]);
                tc::bulk_g2s(ringSFA + slot * kSF, j.sfa + ((size_t(mat) * j.RT + rt) * j.KT + kt0) * 512, nkt * 512,
                             &fullA[slot]);
            };
            auto issueB = [&](int it) {
                const Stage& st = stages[it];
                const int slot = it % NS;
                const int kt0 = st.ku0 / 2, nkt = (st.ku0 + st.nu - 1) / 2 - kt0 + 1;
                const size_t sb = j.mode == kDown ? size_t(st.s) : 0;
                tc::mbar_arrive_expect_tx(&fullB[slot], kB + nkt * 512);
                tc::bulk_g2s(ringB + slot * kB, j.bimg + (sb * j.SPS + st.ku0 / 4) * kB, kB, &fullB[slot]);
                tc::bulk_g2s(ringSFB + slot * kSF, j.bsf + (sb * j.KT + kt0) * 512, nkt * 512, &fullB[slot]);
            };
            const int pre = split ? min(NS, nst) : 0;
            for (int it = 0; it < pre; ++it) issueA(it);
            if (split) pdl_wait();
            for (int it = 0; it < pre; ++it) issueB(it);
            bool ok = true;
            for (int it = pre; it < nst && ok; ++it) {
                if (it >= NS) ok = tc::mbar_wait(&empty[it % NS], ((it / NS) - 1) & 1, j.err, 1);
                if (!ok) break;
                issueA(it);
                issueB(it);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        bool ok = true;
        for (int it = 0; it < nst && ok; ++it) {
            const Stage& st = stages[it];
            const int slot = it % NS, ph = (it / NS) & 1;
            const int buf = st.seg & 1;
            if (st.first && st.seg >= 2) ok = tc::mbar_wait(&accE[buf], ((st.seg >> 1) - 1) & 1, j.err, 2);
            ok = ok && tc::mbar_wait(&fullA[slot], ph, j.err, 3) && tc::mbar_wait(&fullB[slot], ph, j.err, 4);
            ok = __all_sync(kFull, ok);
            if (!ok) break;
            tc::tc_fence_after();
            if (lane == 0) {
                const int kt0 = st.ku0 / 2, nkt = (st.ku0 + st.nu - 1) / 2 - kt0 + 1;
                for (int q = 0; q < nkt; ++q) {
                    tc::tmem_cp_sf(tm_sfa + 4 * q, tc::desc_sf_chunk(tc::smem_u32(ringSFA + slot * kSF + q * 512)));
                    tc::tmem_cp_sf(tm_sfb + 4 * q, tc::desc_sf_chunk(tc::smem_u32(ringSFB + slot * kSF + q * 512)));
                }
                for (int u = 0; u < st.nu; ++u) {
                    const int ku = st.ku0 + u;
                    const uint32_t sf_id = 2u * (ku & 1);
                    const uint32_t q = uint32_t(ku / 2 - kt0);
                    const uint64_t ad = tc::desc_sw128(tc::smem_u32(ringA + slot * kA + u * 32));
                    const uint64_t bd = tc::desc_sw128(tc::smem_u32(ringB + slot * kB + u * 32));
                    tc::mma_mxf4(tm_acc + buf * R, ad, bd, tc::idesc_mxf4(128, R, sf_id, sf_id),
                                 (tm_sfa + 4 * q) | (sf_id << 30), (tm_sfb + 4 * q) | (sf_id << 30),
                                 !(st.first && u == 0));
                }
                tc::mma_commit(&empty[slot]);
                if (st.last) tc::mma_commit(&accF[buf]);
            }
            __syncwarp();
        }
    } else {
        // ---------------------------------------------------------------- epilogue (warps 2..5)
        const int quad = warp & 3;                  // TMEM lane quadrant this warp may read
        const int row = quad * 32 + lane;           // row within the 128-row tile
        const int et = tid - 64;                    // 0..127
        bool ok = true;
        for (int it = 0; it < nst; ++it) {
            const Stage& st = stages[it];
            if (!st.last) continue;
            const int buf = st.seg & 1;
            ok = ok && tc::mbar_wait(&accF[buf], (st.seg >> 1) & 1, j.err, 5);
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
            if (!ok) continue;

            // Which CTAs share this tile; the whole tile in one segment needs no reduction.
            const int t = st.tile;
            int cf = c, cl = c;
            const bool whole = cta_begin(j, c) <= (long long)t * j.UT && cta_begin(j, c + 1) >= (long long)(t + 1) * j.UT;
            float total = v;
            if (!whole) {
                tile_contributors(j, t, cf, cl);
                const int my = c - cf;
                if (my >= kMaxContrib) {
                    if (et == 0) atomicCAS(j.err, 0, 101);
                    continue;
                }
                j.partial[(size_t(t) * kMaxContrib + my) * 128 + row] = v;
                __threadfence();                             // each thread publishes its own partial
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (et == 0) {
                    const long long T0 = (long long)t * j.UT;
                    long long s0 = cta_begin(j, c), s1 = cta_begin(j, c + 1);
                    s0 = s0 > T0 ? s0 : T0;
                    s1 = s1 < T0 + j.UT ? s1 : T0 + j.UT;
                    __threadfence();
                    const unsigned old = atomicAdd(&j.cnt[t], unsigned(s1 - s0));
                    const bool last = old + unsigned(s1 - s0) == unsigned(j.UT);
                    if (last) j.cnt[t] = 0;                  // every contributor has arrived: reset for next launch
                    __threadfence();
                    *flag = last;
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (!*flag) continue;
                total = 0.f;
                const long long T0 = (long long)t * j.UT;
                for (int cc = cf; cc <= cl && cc - cf < kMaxContrib; ++cc) {
                    const long long a0 = cta_begin(j, cc), a1 = cta_begin(j, cc + 1);
                    if ((a0 > T0 ? a0 : T0) >= (a1 < T0 + j.UT ? a1 : T0 + j.UT)) continue;   // no work in tile
                    total += __ldcg(&j.partial[(size_t(t) * kMaxContrib + (cc - cf)) * 128 + row]);
                }
            }

            if (j.mode == kGateUp) {
                // rows 2m (glu) and 2m+1 (linear) of this tile -> a[m] of slot s, times the slot's gate weight
                const int s = t / j.RT, rt = t % j.RT;
                const int e = j.ids[s];
                const int grow = rt * 128 + row;
                const float y = grow < j.rows ? total + j.bias[size_t(e) * j.rows + grow] : 0.f;
                const float lin = __shfl_down_sync(kFull, y, 1);
                if ((lane & 1) == 0) {
                    const float gv = fminf(y, j.limit);
                    const float lv = fminf(fmaxf(lin, -j.limit), j.limit);
                    aval[row >> 1] = gv / (1.f + expf(-j.alpha * gv)) * (lv + 1.f) * j.gate_w[s];
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                // warps with quad 0 and 1 quantize the tile's two 32-element blocks (block index rt*2 + quad)
                if (quad < 2) {
                    const int gb = rt * 2 + quad;            // block of I
                    if (gb * 32 < j.rows / 2) {
                        uint8_t* img = j.out_img + (size_t(s) * j.out_SPS + gb / 8) * (R * 128);
                        uint8_t* sf = j.out_sf + (size_t(s) * j.out_KT + gb / 4) * 512;
                        quantize_block_terms(aval[quad * 32 + lane], img, gb % 8, sf, gb % 4);
                    }
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
            } else {
                const int grow = t * 128 + row;
                if (grow < j.rows) {
                    float add = total;
                    for (int s = 0; s < j.k; ++s) add += j.gate_w[s] * j.bias[size_t(j.ids[s]) * j.rows + grow];
                    j.x_resid[grow] += add;
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

size_t smem_bytes(int NS) {
    return 1024 + size_t(NS) * kStageBytes + size_t(3 * NS + 4) * 8 + 16 + 64 * 4 + kMaxStages * sizeof(Stage) + 64;
}

template <class... KArgs, class... Args>
void launch_ex(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    GPT_CHECK(cudaLaunchKernelEx(&cfg, kernel, args...));
}

int grid_for(long long total, int UT) {
    // At least max(8, UT/8) units per CTA keeps every tile within kMaxContrib contributors.
    const long long min_units = std::max<long long>(8, (UT + 7) / 8);
    const long long g = std::max<long long>(1, total / min_units);
    return int(std::min<long long>(g, num_sms()));
}

}  // namespace dtc

// ---------------------------------------------------------------------------------------------------- host API
DecodeTcLayout decode_tc_layout(int k, int H, int I) {
    DecodeTcLayout L{};
    const int R = kDecodeTerms;
    auto al = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    const int UKg = (H + 63) / 64, UKd = (I + 63) / 64;
    L.SPS_gu = (UKg + 3) / 4;
    L.KT_gu = (H + 127) / 128;
    L.SPS_dn = (UKd + 3) / 4;
    L.KT_dn = (I + 127) / 128;
    L.RT_gu = (2 * I + 127) / 128;
    L.RT_dn = (H + 127) / 128;
    size_t o = 0;
    L.off_xq_img = o; o += al(size_t(L.SPS_gu) * R * 128);
    L.off_xq_sf = o; o += al(size_t(L.KT_gu) * 512);
    L.off_aq_img = o; o += al(size_t(k) * L.SPS_dn * R * 128);
    L.off_aq_sf = o; o += al(size_t(k) * L.KT_dn * 512);
    L.off_part_gu = o; o += al(size_t(k) * L.RT_gu * dtc::kMaxContrib * 128 * 4);
    L.off_part_dn = o; o += al(size_t(L.RT_dn) * dtc::kMaxContrib * 128 * 4);
    L.off_cnt_gu = o; o += al(size_t(k) * L.RT_gu * 4);
    L.off_cnt_dn = o; o += al(size_t(L.RT_dn) * 4);
    L.off_err = o; o += 1024;
    L.off_sfa_gu = o; o += al(sf_repacked_bytes(k, 2 * I, H / 32));
    L.off_sfa_dn = o; o += al(sf_repacked_bytes(k, H, I / 32));
    L.off_misc = o; o += al(size_t(H) * 4 + 256);
    L.bytes = o;
    L.zero_bytes_from = L.off_cnt_gu;                        // counters and error word must start at zero
    L.zero_bytes_to = L.off_err + 1024;
    return L;
}

void launch_quantize_terms(const float* x, int n, uint8_t* img, uint8_t* sf, cudaStream_t s) {
    require(n % 32 == 0, "quantize_terms: n must be a multiple of 32");
    const int blocks = n / 32;
    dtc::quantize_terms_kernel<<<std::max(1, (blocks + 7) / 8), 256, 0, s>>>(x, n, img, sf);
    check_launch("quantize_terms");
}

void launch_moe_decode_tc(const DecodeTcArgs& a, cudaStream_t s) {
    using namespace dtc;
    require(a.k >= 1 && a.k <= 8, "moe (tc): k must be in 1..8");
    require(a.H % 64 == 0 && a.I % 64 == 0, "moe (tc): H and I must be multiples of 64");
    const DecodeTcLayout L = decode_tc_layout(a.k, a.H, a.I);
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    int* err = reinterpret_cast<int*>(ws + L.off_err);
    const int NS = 5;
    const size_t smem = smem_bytes(NS);
    static bool attr_set = false;
    if (!attr_set) {
        GPT_CHECK(cudaFuncSetAttribute(moe_gemv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        attr_set = true;
    }
    // gate/up
    Job g{};
    g.mode = kGateUp;
    g.RT = L.RT_gu;
    g.n_tiles = a.k * g.RT;
    g.UK = a.H / 64;
    g.KT = L.KT_gu;
    g.SPS = L.SPS_gu;
    g.k = a.k;
    g.UT = g.UK;
    g.total = (long long)g.n_tiles * g.UT;
    g.sfa = a.sfa_gu;
    g.sfa_by_slot = a.sfa_by_slot;
    g.bimg = ws + L.off_xq_img;
    g.bsf = ws + L.off_xq_sf;
    g.bias = a.gu_bias;
    g.ids = a.ids;
    g.gate_w = a.weights;
    g.partial = reinterpret_cast<float*>(ws + L.off_part_gu);
    g.cnt = reinterpret_cast<unsigned*>(ws + L.off_cnt_gu);
    g.out_img = ws + L.off_aq_img;
    g.out_sf = ws + L.off_aq_sf;
    g.out_SPS = L.SPS_dn;
    g.out_KT = L.KT_dn;
    g.rows = 2 * a.I;
    g.alpha = a.alpha;
    g.limit = a.limit;
    g.err = err;
    const int grid_g = grid_for(g.total, g.UT);
    launch_ex(moe_gemv_tc_kernel, grid_g, kThreads, smem, s, a.pdl_gateup, *a.tmap_gu, g, NS);
    check_launch("moe gate/up (tc)");
    if (a.mid_event) GPT_CHECK(cudaEventRecord(static_cast<cudaEvent_t>(a.mid_event), s));
    // down
    Job d{};
    d.mode = kDown;
    d.RT = L.RT_dn;
    d.n_tiles = d.RT;
    d.UK = a.I / 64;
    d.KT = L.KT_dn;
    d.SPS = L.SPS_dn;
    d.k = a.k;
    d.UT = a.k * d.UK;
    d.total = (long long)d.n_tiles * d.UT;
    d.sfa = a.sfa_dn;
    d.sfa_by_slot = a.sfa_by_slot;
    d.bimg = ws + L.off_aq_img;
    d.bsf = ws + L.off_aq_sf;
    d.bias = a.dn_bias;
    d.ids = a.ids;
    d.gate_w = a.weights;
    d.partial = reinterpret_cast<float*>(ws + L.off_part_dn);
    d.cnt = reinterpret_cast<unsigned*>(ws + L.off_cnt_dn);
    d.x_resid = a.x_resid;
    d.rows = a.H;
    d.err = err;
    const int grid_d = grid_for(d.total, d.UT);
    launch_ex(moe_gemv_tc_kernel, grid_d, kThreads, smem, s, a.mid_event == nullptr, *a.tmap_dn, d, NS);
    check_launch("moe down (tc)");
}

}  // namespace gpt
