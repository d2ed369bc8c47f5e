// Tensor-core support shared by the decode and prefill paths: TMA tensor maps, the scale-factor repack into the
// tcgen05 chunk layout, and a single-CTA block-scaled GEMM self-test that pins every layout convention the real
// kernels rely on (operand swizzle, descriptor fields, scale-factor placement, accumulator readback).
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <stdexcept>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"
#include "terms.cuh"
#include "tma.h"

namespace gpt {

// ---------------------------------------------------------------------------------------------------- TMA maps
namespace {
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    return fn;
}
}  // namespace

namespace {
CUtensorMapSwizzle swizzle_mode(uint32_t swizzle_bytes) {
    require(swizzle_bytes == 64 || swizzle_bytes == 128, "TMA swizzle must be 64 or 128 bytes");
    return swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
}
}  // namespace

CUtensorMap make_tmap_u8_swz(const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                             uint32_t box_rows, uint32_t swizzle_bytes) {
    require(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
    require(row_bytes % 16 == 0, "TMA row pitch must be a multiple of 16 bytes");
    require(box_bytes <= swizzle_bytes && box_bytes % 16 == 0 && box_rows >= 1 && box_rows <= 256, "bad TMA box");
    CUtensorMap m;
    std::memset(&m, 0, sizeof(m));
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_bytes, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_mode(swizzle_bytes),
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
    return m;
}

CUtensorMap make_tmap_u8_sw128(const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                               uint32_t box_rows) {
    return make_tmap_u8_swz(base, row_bytes, rows, box_bytes, box_rows, 128);
}

CUtensorMap make_tmap_u8_swz_3d(const void* base, uint64_t row_bytes, uint64_t rows, uint64_t mats,
                                uint32_t box_bytes, uint32_t box_rows, uint32_t swizzle_bytes) {
    require(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
    require(row_bytes % 16 == 0, "TMA row pitch must be a multiple of 16 bytes");
    require(box_bytes <= swizzle_bytes && box_bytes % 16 == 0 && box_rows >= 1 && box_rows <= 256, "bad TMA box");
    CUtensorMap m;
    std::memset(&m, 0, sizeof(m));
    const cuuint64_t dims[3] = {row_bytes, rows, mats};
    const cuuint64_t strides[2] = {row_bytes, row_bytes * rows};
    const cuuint32_t box[3] = {box_bytes, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_mode(swizzle_bytes),
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3d) failed: " + std::to_string(int(r)));
    return m;
}

CUtensorMap make_tmap_u8_sw128_3d(const void* base, uint64_t row_bytes, uint64_t rows, uint64_t mats,
                                  uint32_t box_bytes, uint32_t box_rows) {
    return make_tmap_u8_swz_3d(base, row_bytes, rows, mats, box_bytes, box_rows, 128);
}

// ---------------------------------------------------------------------------------------------------- SF repack
namespace {
// raw [mats][rows][G] E8M0 bytes -> [mats][RT][KT][halves][512] tcgen05 chunks (tiles of 128 * halves rows,
// RT = ceil(rows / tile), KT = ceil(G/4)), zero padded. One thread per output word of 4 bytes (one row's 4 k-blocks).
// A scale byte 0xFF (E8M0's NaN encoding) sets *nan_flag to nan_code when a flag is given (the first code set stays).
__global__ void repack_sf_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ out, long long mats, int rows,
                                 int G, int RT, int KT, int halves, int tile_rows, const int* __restrict__ ids,
                                 int* nan_flag, int nan_code) {
    const long long words = mats * RT * KT * halves * 128;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < words;
         i += (long long)gridDim.x * blockDim.x) {
        const int w = int(i % 128);                  // word within the chunk: (row % 32) * 4 + row / 32
        long long c = i / 128;
        const int h = int(c % halves);               // 128-row part of the tile (the last one may be partial)
        c /= halves;
        const int kt = int(c % KT);
        c /= KT;
        const int rt = int(c % RT);
        const long long mat = ids ? (long long)ids[c / RT] : c / RT;
        const int in_tile = h * 128 + (w & 3) * 32 + (w >> 2);
        const int row = rt * tile_rows + in_tile;
        uint32_t v = 0;
        if (in_tile < tile_rows && row < rows) {
            const uint8_t* src = raw + (mat * rows + row) * G;
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
                const int g = kt * 4 + kb;
                if (g < G) v |= uint32_t(src[g]) << (8 * kb);
            }
            if (nan_flag && __vcmpeq4(v, 0xFFFFFFFFu)) atomicCAS(nan_flag, 0, nan_code);
        }
        reinterpret_cast<uint32_t*>(out)[i] = v;
    }
}
}  // namespace

size_t sf_repacked_bytes(long long mats, int rows, int G, int tile_rows) {
    return size_t(mats) * size_t((rows + tile_rows - 1) / tile_rows) * size_t((G + 3) / 4) *
           size_t((tile_rows + 127) / 128) * 512;
}

void launch_repack_sf(const uint8_t* raw, uint8_t* out, long long mats, int rows, int G, cudaStream_t s,
                      const int* ids, int tile_rows, int* nan_flag, int nan_code) {
    require(tile_rows == 128 || tile_rows == 192 || tile_rows == 256, "repack_sf: tiles of 128, 192 or 256 rows");
    const int halves = (tile_rows + 127) / 128, RT = (rows + tile_rows - 1) / tile_rows, KT = (G + 3) / 4;
    const long long words = mats * RT * KT * halves * 128;
    const int grid = int(std::min<long long>((words + 255) / 256, num_sms() * 8LL));
    repack_sf_kernel<<<std::max(1, grid), 256, 0, s>>>(raw, out, mats, rows, G, RT, KT, halves, tile_rows, ids,
                                                        nan_flag, nan_code);
    check_launch("repack_sf");
}

// ---------------------------------------------------------------------------------------------------- self-test
namespace {
__global__ void __launch_bounds__(128) mxf4_selftest_kernel(const __grid_constant__ CUtensorMap tmA,
                                                            const uint8_t* __restrict__ sfa,
                                                            const uint8_t* __restrict__ bimg,
                                                            const uint8_t* __restrict__ sfb, float* __restrict__ out,
                                                            int N, int K, int a64, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = (K + 255) / 256, KT = (K + 127) / 128, nB = N > 128 ? 2 : 1;
    uint8_t* sA = smem;                                      // S x 16384
    uint8_t* sB = sA + S * 16384;                            // S x N*128
    uint8_t* sSFA = sB + S * N * 128;                        // KT x 512
    uint8_t* sSFB = sSFA + KT * 512;                         // KT x nB x 512
    uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + KT * nB * 512);   // S full + 1 done
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + S + 1);
    const int tid = threadIdx.x, warp = tid >> 5;

    if (tid == 0) {
        for (int s = 0; s <= S; ++s) tc::mbar_init(&bars[s], 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(holder, 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tm = *holder;
    const uint32_t tm_d = tm, tm_sfa = tm + 256, tm_sfb = tm + 256 + 4 * KT;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            const int kt0 = 2 * s, nkt = min(2, KT - kt0);
            const uint32_t bytes = 16384 + N * 128 + nkt * 512 + nkt * nB * 512;
            tc::mbar_arrive_expect_tx(&bars[s], bytes);
            if (a64) {                           // two 64-byte-wide boxes per stage, one per K chunk of 128
                tc::tma_load_2d(sA + s * 16384, &tmA, s * 128, 0, &bars[s]);
                tc::tma_load_2d(sA + s * 16384 + 8192, &tmA, s * 128 + 64, 0, &bars[s]);
            } else {
                tc::tma_load_2d(sA + s * 16384, &tmA, s * 128, 0, &bars[s]);
            }
            tc::bulk_g2s(sB + s * N * 128, bimg + size_t(s) * N * 128, N * 128, &bars[s]);
            tc::bulk_g2s(sSFA + kt0 * 512, sfa + size_t(kt0) * 512, nkt * 512, &bars[s]);
            tc::bulk_g2s(sSFB + kt0 * nB * 512, sfb + size_t(kt0) * nB * 512, nkt * nB * 512, &bars[s]);
        }
        bool ok = true;
        for (int s = 0; s < S && ok; ++s) {
            ok = tc::mbar_wait(&bars[s], 0, err, 1);
            if (!ok) break;
            tc::tc_fence_after();
            for (int kt2 = 0; kt2 < 2; ++kt2) {
                const int kt = 2 * s + kt2;
                if (kt >= KT) break;
                tc::tmem_cp_sf(tm_sfa + 4 * kt, tc::desc_sf_chunk(tc::smem_u32(sSFA + kt * 512)));
                for (int b = 0; b < nB; ++b)
                    tc::tmem_cp_sf(tm_sfb + 4 * (kt * nB + b), tc::desc_sf_chunk(tc::smem_u32(sSFB + (kt * nB + b) * 512)));
                for (int j = 0; j < 2; ++j) {
                    const int kk = kt * 128 + j * 64;
                    if (kk >= K) break;
                    const uint64_t ad = a64 ? tc::desc_sw64(tc::smem_u32(sA + s * 16384 + kt2 * 8192 + j * 32))
                                            : tc::desc_sw128(tc::smem_u32(sA + s * 16384 + (kt2 * 2 + j) * 32));
                    const uint64_t bd = tc::desc_sw128(tc::smem_u32(sB + s * N * 128 + (kt2 * 2 + j) * 32));
                    const uint32_t sf_id = 2u * j;
                    tc::mma_mxf4(tm_d, ad, bd, tc::idesc_mxf4(128, N, sf_id, sf_id), (tm_sfa + 4 * kt) | (sf_id << 30),
                                 (tm_sfb + 4 * kt * nB) | (sf_id << 30), kk > 0);
                }
            }
        }
        tc::mma_commit(&bars[S]);                // arrives once all issued MMAs (possibly none) completed
    }
    __syncwarp();
    const bool done = __all_sync(kFull, tc::mbar_wait(&bars[S], 0, err, 2));   // warp-uniform for tcgen05.ld
    tc::tc_fence_after();
    if (done) {
        const int row = warp * 32 + (tid & 31);
        for (int c = 0; c < N; c += 8) {
            float v[8];
            tc::tmem_ld_32x32b_x8(tm_d + (uint32_t(warp * 32) << 16) + c, v);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 8; ++i) out[size_t(row) * N + c + i] = v[i];
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tm, 512);
}
}  // namespace

// Dense kind::mxf4 tensor rate of this GPU: every CTA (one per SM) issues `iters` x 4 back-to-back M = 128, N = n,
// K = 64 block-scaled MMAs into one TMEM accumulator from shared-memory operands (zero e2m1 codes, every E8M0 scale
// 2^0: the operands' values do not change the rate) and commits once; the host times the launch with events.
__global__ void __launch_bounds__(128) mxf4_peak_kernel(int iters, int n, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                                      // 128 rows x 128 bytes (256 values of K)
    uint8_t* sB = sA + 128 * 128;                            // 256 rows x 128 bytes
    uint8_t* sSF = sB + 256 * 128;                           // 6 scale chunks of 512 bytes: A (2), B (2 x 2)
    uint64_t* bar = reinterpret_cast<uint64_t*>(sSF + 6 * 512);
    uint32_t* holder = reinterpret_cast<uint32_t*>(bar + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < (128 + 256) * 128 / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sA)[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid; i < 6 * 512 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sSF)[i] = 0x7F7F7F7Fu;
    if (tid == 0) {
        tc::mbar_init(bar, 1);
        tc::fence_barrier_init();
    }
    tc::fence_proxy_async_smem();
    if (warp == 0) {
        tc::tmem_alloc(holder, 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tm = *holder, tm_sfa = tm + 256, tm_sfb = tm + 264;
    if (tid == 0) {
        for (int kt = 0; kt < 2; ++kt) {
            tc::tmem_cp_sf(tm_sfa + 4 * kt, tc::desc_sf_chunk(tc::smem_u32(sSF + kt * 512)));
            for (int hh = 0; hh < 2; ++hh)
                tc::tmem_cp_sf(tm_sfb + 8 * kt + 4 * hh, tc::desc_sf_chunk(tc::smem_u32(sSF + (2 + 2 * kt + hh) * 512)));
        }
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t sf_id = 2u * uint32_t(u & 1), q = uint32_t(u >> 1);
                tc::mma_mxf4(tm, tc::desc_sw128(tc::smem_u32(sA + u * 32)), tc::desc_sw128(tc::smem_u32(sB + u * 32)),
                             tc::idesc_mxf4(128, n, sf_id, sf_id), (tm_sfa + 4 * q) | (sf_id << 30),
                             (tm_sfb + 8 * q) | (sf_id << 30), it > 0 || u > 0);
            }
        }
        tc::mma_commit(bar);
    }
    __syncwarp();
    tc::mbar_wait(bar, 0, err, 1);
    tc::tc_fence_after();
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tm, 512);
}

// Nanoseconds per M = 128, N = n, K = 64 kind::mxf4 MMA issued back to back on one SM (every SM busy).
double selftest_mxf4_mma_ns(int n, int* err_dev) {
    require(n % 8 == 0 && n >= 8 && n <= 256, "selftest_mxf4_mma_ns: n must be a multiple of 8 in 8..256");
    const int sms = num_sms();
    const int smem = 1024 + (128 + 256) * 128 + 6 * 512 + 64;
    GPT_CHECK(cudaFuncSetAttribute(mxf4_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaEvent_t e0, e1;
    GPT_CHECK(cudaEventCreate(&e0));
    GPT_CHECK(cudaEventCreate(&e1));
    const int iters = 4096;
    mxf4_peak_kernel<<<sms, 128, smem>>>(64, n, err_dev);          // warm-up
    check_launch("mxf4_peak");
    GPT_CHECK(cudaEventRecord(e0));
    mxf4_peak_kernel<<<sms, 128, smem>>>(iters, n, err_dev);
    check_launch("mxf4_peak");
    GPT_CHECK(cudaEventRecord(e1));
    GPT_CHECK(cudaEventSynchronize(e1));
    float ms = 0.f;
    GPT_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return double(ms) * 1e6 / (4.0 * iters);
}

double selftest_mxf4_peak(int* err_dev) {
    const double ns = selftest_mxf4_mma_ns(256, err_dev);
    return 2.0 * 128 * 256 * 64 * num_sms() / (ns * 1e-9) / 1e12;
}

void selftest_mxf4_gemm(const uint8_t* a_blocks, const uint8_t* a_scales, const uint8_t* b_blocks,
                        const uint8_t* b_scales, float* d, int N, int K, void* scratch, size_t scratch_bytes,
                        cudaStream_t s, int a_swizzle) {
    require(a_swizzle == 64 || a_swizzle == 128, "selftest: A's swizzle must be 64 or 128 bytes");
    require(N % 8 == 0 && N >= 8 && N <= 256, "selftest: N must be a multiple of 8 in 8..256");
    require(K % 64 == 0 && K >= 64 && K <= 1024, "selftest: K must be a multiple of 64 in 64..1024");
    const int S = (K + 255) / 256, KT = (K + 127) / 128, nB = N > 128 ? 2 : 1, G = K / 32;
    // B operand images (swizzled, zero beyond K) and SFB chunks, built on the host from the raw device arrays.
    std::vector<uint8_t> hb(size_t(N) * K / 2), hs(size_t(N) * G);
    GPT_CHECK(cudaMemcpy(hb.data(), b_blocks, hb.size(), cudaMemcpyDeviceToHost));
    GPT_CHECK(cudaMemcpy(hs.data(), b_scales, hs.size(), cudaMemcpyDeviceToHost));
    std::vector<uint8_t> img(size_t(S) * N * 128, 0), sfb(size_t(KT) * nB * 512, 0);
    for (int st = 0; st < S; ++st)
        for (int n = 0; n < N; ++n)
            for (int kb = 0; kb < 128; ++kb) {
                const int src = st * 128 + kb;
                if (src < K / 2) img[size_t(st) * N * 128 + tc::sw128_offset(n, kb)] = hb[size_t(n) * K / 2 + src];
            }
    for (int kt = 0; kt < KT; ++kt)
        for (int n = 0; n < N; ++n)
            for (int kb = 0; kb < 4; ++kb) {
                const int g = kt * 4 + kb;
                if (g < G) sfb[(size_t(kt) * nB + n / 128) * 512 + tc::sf_offset(n % 128, kb)] = hs[size_t(n) * G + g];
            }
    const size_t sfa_bytes = sf_repacked_bytes(1, 128, G);
    const size_t need = img.size() + sfb.size() + sfa_bytes + 64;
    require(scratch_bytes >= need, "selftest: scratch too small");
    uint8_t* base = static_cast<uint8_t*>(scratch);
    uint8_t* d_img = base;
    uint8_t* d_sfb = d_img + ((img.size() + 1023) & ~size_t(1023));
    uint8_t* d_sfa = d_sfb + ((sfb.size() + 1023) & ~size_t(1023));
    int* d_err = reinterpret_cast<int*>(d_sfa + ((sfa_bytes + 1023) & ~size_t(1023)));
    GPT_CHECK(cudaMemcpy(d_img, img.data(), img.size(), cudaMemcpyHostToDevice));
    GPT_CHECK(cudaMemcpy(d_sfb, sfb.data(), sfb.size(), cudaMemcpyHostToDevice));
    GPT_CHECK(cudaMemset(d_err, 0, sizeof(int)));
    launch_repack_sf(a_scales, d_sfa, 1, 128, G, s);
    const CUtensorMap tmA = make_tmap_u8_swz(a_blocks, K / 2, 128, uint32_t(a_swizzle), 128, uint32_t(a_swizzle));
    const size_t smem = 1024 + size_t(S) * 16384 + size_t(S) * N * 128 + KT * 512 + KT * nB * 512 + (S + 1) * 8 + 16;
    GPT_CHECK(cudaFuncSetAttribute(mxf4_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    mxf4_selftest_kernel<<<1, 128, smem, s>>>(tmA, d_sfa, d_img, d_sfb, d, N, K, a_swizzle == 64 ? 1 : 0, d_err);
    check_launch("mxf4 selftest");
    GPT_CHECK(cudaStreamSynchronize(s));
    int herr = 0;
    GPT_CHECK(cudaMemcpy(&herr, d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) throw std::runtime_error("mxf4 selftest: a bounded wait timed out at site " + std::to_string(herr));
}

namespace {
// One warp per 8 blocks: quantize x into residual terms with the chosen quantizer (0 = comparisons, 1 = converters,
// 2 = fixed scale schedule with fp32 rounding, 3 = the same computed by a whole warp per block, 4 = the integer digit
// split computed by a whole warp per block).
__global__ void terms_quantize_kernel(const float* x, int n, uint8_t* img, uint8_t* sf, int which) {
    const int lane = threadIdx.x & 31, sub = lane & 3;
    if (which == 3 || which == 4) {                          // one block per warp, one element per lane
        const int warps = gridDim.x * (blockDim.x / 32), w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
        for (int g = w; g < n / 32; g += warps) {
            if (which == 3)
                quantize_block_terms_warp32<kDecodeTerms>(x[g * 32 + lane], img + (g / 8) * (kDecodeTerms * 128),
                                                          g % 8, sf + (g / 4) * 512, g % 4, true);
            else
                quantize_block_digits_warp32(x[g * 32 + lane], img + (g / 8) * (kDecodeTerms * 128), g % 8,
                                             sf + (g / 4) * 512, g % 4, true);
        }
        return;
    }
    const int g = (blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * 8 + (lane >> 2);
    const bool active = g < n / 32;
    const int gg = active ? g : 0;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = active ? x[gg * 32 + sub * 8 + i] : 0.f;
    uint8_t* im = img + (gg / 8) * (kDecodeTerms * 128);
    uint8_t* sc = sf + (gg / 4) * 512;
    if (which == 2) quantize_block_terms_fixed(v, im, gg % 8, sc, gg % 4, sub, active);
    else if (which == 1) quantize_block_terms_cvt(v, im, gg % 8, sc, gg % 4, sub, active);
    else quantize_block_terms(v, im, gg % 8, sc, gg % 4, sub, active);
}

// Reference decoder of the term images: out[i] = sum_t e2m1(code_t[i]) * 2^(scale_t - 127), in fp64 then rounded.
__global__ void terms_decode_kernel(const uint8_t* img, const uint8_t* sf, int n, float* out, float* per_term) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int g = i / 32, e = i % 32;
    double acc = 0.0;
    for (int t = 0; t < kDecodeTerms; ++t) {
        const uint8_t* row = img + (g / 8) * (kDecodeTerms * 128) + t * 128;
        const int q = g % 8;
        const uint8_t byte = row[((q ^ (t & 7)) << 4) + e / 2];
        const uint32_t code = (e & 1) ? (byte >> 4) : (byte & 15);
        const uint32_t s = sf[(g / 4) * 512 + (t & 31) * 16 + (t >> 5) * 4 + (g % 4)];
        const double v = double(e2m1_exact(code)) * ldexp(1.0, int(s) - 127);
        if (per_term && t < 2) per_term[size_t(t) * n + i] = float(v);
        acc += v;
    }
    out[i] = float(acc);
}
}  // namespace

void selftest_terms(const float* x, int n, float* out, float* per_term, int which, void* scratch, size_t bytes,
                    cudaStream_t s) {
    require(n % 256 == 0 && n > 0, "selftest_terms: n must be a positive multiple of 256");
    require(which >= 0 && which <= 4, "selftest_terms: which must be 0 .. 4");
    const size_t img_bytes = size_t(n / 256) * kDecodeTerms * 128, sf_bytes = size_t(n / 128) * 512;
    require(bytes >= img_bytes + sf_bytes, "selftest_terms: scratch too small");
    uint8_t* img = static_cast<uint8_t*>(scratch);
    uint8_t* sf = img + img_bytes;
    GPT_CHECK(cudaMemsetAsync(scratch, 0, img_bytes + sf_bytes, s));
    const int warps = (n / 32 + 7) / 8;
    terms_quantize_kernel<<<(warps + 3) / 4, 128, 0, s>>>(x, n, img, sf, which);
    check_launch("terms quantize");
    terms_decode_kernel<<<(n + 255) / 256, 256, 0, s>>>(img, sf, n, out, per_term);
    check_launch("terms decode");
    GPT_CHECK(cudaStreamSynchronize(s));
}

}  // namespace gpt
