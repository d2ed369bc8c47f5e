// Activation quantization into e2m1 residual terms: the B operand of the tensor-core decode GEMVs.
#pragma once
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace gpt {

__device__ __forceinline__ float exp2i_exact(int n) {         // exact 2^n for n in [-127, 127]
    return n <= -127 ? __uint_as_float(0x00400000u) : __uint_as_float(uint32_t(n + 127) << 23);
}

// Warp-cooperative: lane i holds element i of one 32-element block. Writes kDecodeTerms e2m1 residual terms of the
// block: term t's 16 code bytes at img_stage + t*128 + ((q ^ (t & 7)) << 4) (q = the block's 16-byte chunk within
// the 128-byte stage row, pre-swizzled) and its E8M0 scale at sf_chunk[(t % 32) * 16 + (t / 32) * 4 + kb].
// Each term's scale is the smallest power of two keeping the remaining block maximum within 6; codes round to
// nearest, ties to even; the subtraction of each term is exact, so the terms sum to the input up to the last
// term's rounding.
__device__ __forceinline__ void quantize_block_terms(float v, uint8_t* img_stage, int q, uint8_t* sf_chunk, int kb) {
    const int lane = threadIdx.x & 31;
    float r = v;
#pragma unroll 1
    for (int t = 0; t < kDecodeTerms; ++t) {
        float amax = fabsf(r);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
        int k = -127;
        const uint32_t bits = __float_as_uint(amax);
        const int e = int((bits >> 23) & 0xFF);
        if (e != 0) {
            const int k0 = e - 127;
            k = ((bits & 0x7FFFFFu) <= 0x400000u) ? k0 - 2 : k0 - 1;
            k = max(-127, min(127, k));
        }
        const float y = fabsf(r) * exp2i_exact(-k);
        uint32_t c = (y > 0.25f) + (y >= 0.75f) + (y > 1.25f) + (y >= 1.75f) + (y > 2.5f) + (y >= 3.5f) + (y > 5.0f);
        const float mag = e2m1_exact(c) * exp2i_exact(k);
        if (signbit(r)) {
            c |= 8u;
            r += mag;
        } else {
            r -= mag;
        }
        uint32_t w = c << (4 * (lane & 7));
        w |= __shfl_xor_sync(kFull, w, 1);
        w |= __shfl_xor_sync(kFull, w, 2);
        w |= __shfl_xor_sync(kFull, w, 4);
        if ((lane & 7) == 0)
            *reinterpret_cast<uint32_t*>(img_stage + t * 128 + (((q ^ (t & 7)) << 4) | ((lane >> 3) * 4))) = w;
        if (lane == 0) sf_chunk[(t & 31) * 16 + (t >> 5) * 4 + kb] = uint8_t(k + 127);
    }
}

// Quantize a whole vector (n elements, n % 32 == 0) into B terms: img [n/256 stages][R*128], sf [n/128 chunks][512].
__device__ __forceinline__ void quantize_vector_terms_warp(const float* x, int n, uint8_t* img, uint8_t* sf, int warp_id, int n_warps) {
    const int lane = threadIdx.x & 31;
    for (int g = warp_id; g < n / 32; g += n_warps) {
        const float v = x[g * 32 + lane];
        quantize_block_terms(v, img + (g / 8) * (kDecodeTerms * 128), g % 8, sf + (g / 4) * 512, g % 4);
    }
}

}  // namespace gpt
