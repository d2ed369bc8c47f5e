// Activation quantization into e2m1 residual terms: the B operand of the tensor-core decode GEMVs.
#pragma once
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace gpt {

__device__ __forceinline__ float exp2i_exact(int n) {         // exact 2^n for n in [-127, 127]
    return n <= -127 ? __uint_as_float(0x00400000u) : __uint_as_float(uint32_t(n + 127) << 23);
}

// Quantization of 32-element blocks into kDecodeTerms e2m1 residual terms, four lanes per block: lane `sub` (0..3)
// of a 4-lane group holds elements 8*sub .. 8*sub+7 in v[], which become one 32-bit word (bytes 4*sub..4*sub+3) of
// the block's 16 code bytes. Term t's codes go to img_stage + t*128 + ((q ^ (t & 7)) << 4) + 4*sub (the B-operand
// image, pre-swizzled; q = the block's 16-byte chunk within its 128-byte stage row) and its E8M0 scale to
// sf_chunk[(t % 32) * 16 + (t / 32) * 4 + kb]. Each term's scale is the smallest power of two keeping the remaining
// block maximum within 6; codes round to nearest, ties to even; each term's subtraction is exact, so the terms sum
// to the input up to the last term's rounding. All 32 lanes must call (the group max uses shuffles); `active`
// false only suppresses a group's stores.
__device__ __forceinline__ void quantize_block_terms(float (&v)[8], uint8_t* img_stage, int q, uint8_t* sf_chunk, int kb,
                                                     int sub, bool active) {
#pragma unroll 1
    for (int t = 0; t < kDecodeTerms; ++t) {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
        int k = -127;
        const uint32_t bits = __float_as_uint(amax);
        const int e = int((bits >> 23) & 0xFF);
        if (e != 0) {
            const int k0 = e - 127;
            k = ((bits & 0x7FFFFFu) <= 0x400000u) ? k0 - 2 : k0 - 1;
            k = max(-127, min(127, k));
        }
        const float inv = exp2i_exact(-k), sc = exp2i_exact(k);
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float y = fabsf(v[i]) * inv;
            uint32_t c = (y > 0.25f) + (y >= 0.75f) + (y > 1.25f) + (y >= 1.75f) + (y > 2.5f) + (y >= 3.5f) + (y > 5.0f);
            const float mag = e2m1_exact(c) * sc;
            if (signbit(v[i])) {
                c |= 8u;
                v[i] += mag;
            } else {
                v[i] -= mag;
            }
            word |= c << (4 * i);
        }
        if (active) {
            *reinterpret_cast<uint32_t*>(img_stage + t * 128 + (((q ^ (t & 7)) << 4) | (sub * 4))) = word;
            if (sub == 0) sf_chunk[(t & 31) * 16 + (t >> 5) * 4 + kb] = uint8_t(k + 127);
        }
    }
}

// Same contract as quantize_block_terms, computed with the sm_100 converters: cvt.rn.satfinite.e2m1x2.f32 rounds
// pairs to e2m1 (nearest, ties to even) and cvt.rn.f16x2.e2m1x2 decodes them back exactly for the residual. About a
// quarter of the instructions of the comparison form. The bytes are packed from and unpacked to whole 32-bit
// registers inside the asm (16-bit views of wider registers were miscompiled into wrong bytes).
// `reps` copies of the output are written, the r-th at img_stage + r * img_rs and sf_chunk + r * sf_rs.
__device__ __forceinline__ void quantize_block_terms_cvt(float (&v)[8], uint8_t* img_stage, int q, uint8_t* sf_chunk,
                                                         int kb, int sub, bool active, int reps = 1,
                                                         size_t img_rs = 0, size_t sf_rs = 0) {
#pragma unroll 1
    for (int t = 0; t < kDecodeTerms; ++t) {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
        int k = -127;
        const uint32_t bits = __float_as_uint(amax);
        const int e = int((bits >> 23) & 0xFF);
        if (e != 0) {
            const int k0 = e - 127;
            k = ((bits & 0x7FFFFFu) <= 0x400000u) ? k0 - 2 : k0 - 1;
            k = max(-127, min(127, k));
        }
        const float inv = exp2i_exact(-k), sc = exp2i_exact(k);
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = v[i] * inv;
        // each pair is rounded to e2m1 and decoded back from the same 8-bit register; the four bytes are packed
        // into the output word once at the end
        uint32_t word, h[4];
        asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b0, %6, %5;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b1, %8, %7;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b2, %10, %9;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b3, %12, %11;\n\t"
            "cvt.rn.f16x2.e2m1x2 %1, b0;\n\t"
            "cvt.rn.f16x2.e2m1x2 %2, b1;\n\t"
            "cvt.rn.f16x2.e2m1x2 %3, b2;\n\t"
            "cvt.rn.f16x2.e2m1x2 %4, b3;\n\t"
            "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
            : "=r"(word), "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
            : "f"(y[0]), "f"(y[1]), "f"(y[2]), "f"(y[3]), "f"(y[4]), "f"(y[5]), "f"(y[6]), "f"(y[7]));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<__half2*>(&h[i]));
            v[2 * i] = fmaf(-f.x, sc, v[2 * i]);
            v[2 * i + 1] = fmaf(-f.y, sc, v[2 * i + 1]);
        }
        if (active) {
            for (int r = 0; r < reps; ++r) {
                *reinterpret_cast<uint32_t*>(img_stage + r * img_rs + t * 128 + (((q ^ (t & 7)) << 4) | (sub * 4))) =
                    word;
                if (sub == 0) sf_chunk[r * sf_rs + (t & 31) * 16 + (t >> 5) * 4 + kb] = uint8_t(k + 127);
            }
        }
    }
}

// Nearest e2m1 value of y for |y| <= 6, ties to even, in plain fp32 arithmetic: adding and subtracting 1.5 * 2^23 *
// step rounds y to a multiple of the grid step (0.5 below 2, 1 below 4, 2 up to 6) with the hardware's
// round-to-nearest-even, and an even multiple of the step is exactly an e2m1 value with an even mantissa bit. Short
// latency (two adds after a select), unlike the converter instructions.
__device__ __forceinline__ float round_e2m1(float y) {
    const float a = fabsf(y);
    const float c = a < 2.f ? 0x1.8p22f : (a < 4.f ? 0x1.8p23f : 0x1.8p24f);   // 1.5 * 2^23 * (0.5, 1, 2)
    return __fsub_rn(__fadd_rn(y, c), c);
}

// round_e2m1 that also returns the e2m1 code (sign in bit 3): after the magic add the integer difference of the float
// bits is the rounded multiple of the grid step (0.5, 1 or 2), and the code is that multiple's magnitude plus 0, 2 or
// 4 for the three step ranges (2.0 = code 4, 4.0 = code 6, 6.0 = code 7).
__device__ __forceinline__ float round_e2m1_code(float y, uint32_t& code) {
    const float a = fabsf(y);
    const bool lo = a < 2.f, mid = a < 4.f;
    const float c = lo ? 0x1.8p22f : (mid ? 0x1.8p23f : 0x1.8p24f);
    const float sm = __fadd_rn(y, c);
    const int m = __float_as_int(sm) - __float_as_int(c);
    code = (uint32_t(abs(m) + (lo ? 0 : (mid ? 2 : 4))) & 7u) | ((__float_as_uint(y) >> 28) & 8u);
    return __fsub_rn(sm, c);
}

// e2m1 code (sign in bit 3) of a value q that is exactly an e2m1 value (other inputs give some code, never more
// than 4 bits).
__device__ __forceinline__ uint32_t e2m1_code(float q) {
    const uint32_t u = __float_as_uint(q);
    const float a = fabsf(q);
    const uint32_t mag = a < 1.f ? (a > 0.f ? 1u : 0u) : ((((u & 0x7FFFFFFFu) >> 22) - 252u) & 7u);
    return mag | ((u >> 28) & 8u);
}

constexpr int kActiveTerms = 10;              // terms quantize_block_terms_fixed computes; the rest are zero

// First scale exponent of the fixed schedule for a block whose largest magnitude is amax: the block maximum fits
// within 6 * 2^k (k = floor(log2 amax) - 2, or - 1 when the mantissa is above 1.5), clamped to E8M0's range.
__device__ __forceinline__ int fixed_schedule_k0(float amax) {
    int k = -127;
    const uint32_t bits = __float_as_uint(amax);
    const int e = int((bits >> 23) & 0xFF);
    if (e != 0) {
        const int k0 = e - 127;
        k = ((bits & 0x7FFFFFu) <= 0x400000u) ? k0 - 2 : k0 - 1;
        k = max(-127, min(127, k));
    }
    return k;
}

// Eight terms per 32-value block from one round and an integer split (the prefill path's A operand), four lanes per
// block (lane `sub` holds elements 8 sub .. 8 sub + 7): term 0 is the RNE e2m1 value of v / 2^k (k from the block
// maximum as in fixed_schedule_k0, so |v / 2^k| <= 6 and the remainder r satisfies |r| <= 2^k); then
// R = rint(r 2^(20 - k)) (|R| <= 2^20, the only rounding after term 0) is written in balanced base 8, digits in
// [-4, 3] for 8^0 .. 8^5 and the top one in [-4, 4]: adding 4 (8^7 - 1) / 7 makes every digit the plain octal digit
// plus 4, so each is a 3-bit field. A digit d in units of 2^(k_t - 1) is the e2m1 value d / 2 (0, 0.5, 1, 1.5, 2)
// with scale 2^k_t: term 1 (top digit) has k_1 = k - 1 and term t = 2..7 has k_t = k + 2 - 3t (digit 7 - t). The
// represented value is exact up to the rint: |error| <= 2^(k - 21). Terms whose scale would fall below 2^-127 (blocks
// under about 2^-105) are left zero. emit(t, word, scale) as quantize_block_terms_lanes4.
//
// Fewer terms: with `nt` < 8 the remainder is rounded once to the grid of the last kept digit (R = rint(r 2^(20 - s))
// 2^s, s = 3 (8 - nt); nt = 1 keeps term 0 alone), so terms 0 .. nt - 1 are the nearest nt-term value (|error| <=
// 2^(k + 3 - 3 nt) for nt >= 2, 2^k for nt = 1) and the later terms' codes are all zero.
__device__ __forceinline__ uint32_t balanced_digit_code(uint32_t u) {     // u = digit + 4 in 0..7 -> e2m1 code
    return (0x32109ABCu >> (4 * u)) & 0xFu;
}

template <class Emit>
__device__ __forceinline__ void quantize_block_digits_lanes4(const float (&v)[8], Emit&& emit, int nt = 8) {
    constexpr int kOff = 4 * 299593;                            // 4 (8^7 - 1) / 7
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
    const int k = fixed_schedule_k0(amax);
    const float inv = exp2i_exact(-k), sc = exp2i_exact(k);
    // grid of the last kept digit: 2^s units of 2^(k - 20); nt = 1 keeps no digit (scale 0 makes R = 0)
    const int sh = 3 * (8 - max(2, min(8, nt)));
    const float gscale = nt <= 1 ? 0.f : exp2i_exact(20 - sh);
    uint32_t w0 = 0, w1 = 0;
    int Rp[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t code;
        const float q0 = round_e2m1_code(v[i] * inv, code);
        w0 |= code << (4 * i);
        const float r = fmaf(-q0, sc, v[i]);                    // exact
        Rp[i] = __float2int_rn((r * inv) * gscale) * (1 << sh) + kOff;   // in 0 .. 2^20 + kOff
        const uint32_t u1 = uint32_t(Rp[i]) >> 18;               // top digit + 4, 0..8
        w1 |= (u1 < 4 ? 12u - u1 : u1 - 4u) << (4 * i);
    }
    emit(0, w0, uint32_t(k + 127));
    emit(1, (k - 1 >= -127) ? w1 : 0u, uint32_t(max(k - 1 + 127, 0)));
#pragma unroll
    for (int t = 2; t < 8; ++t) {
        const int kt = k + 2 - 3 * t, j = 7 - t;
        uint32_t u = 0;                                         // the 8 elements' digit fields, one per nibble
#pragma unroll
        for (int i = 0; i < 8; ++i) u |= ((uint32_t(Rp[i]) >> (3 * j)) & 7u) << (4 * i);
        // balanced_digit_code of all 8 nibbles at once: u >= 4 -> u - 4 = u & 3; u < 4 -> 8 | (4 - u) = 8 | ((~u & 3)
        // + 1) (no carry leaves a nibble)
        const uint32_t hi = ((u >> 2) & 0x11111111u) * 0xFu;
        const uint32_t w = (u & 0x33333333u & hi) | ((0x88888888u | ((~u & 0x33333333u) + 0x11111111u)) & ~hi);
        emit(t, kt >= -127 ? w : 0u, uint32_t(max(kt + 127, 0)));
    }
}

// quantize_block_digits_lanes4 with eight lanes per block, four elements each (lane `sub8` = 0..7 of an aligned
// 8-lane group holds elements 4 sub8 .. 4 sub8 + 3): the same terms, scales and digits, so the same bits. emit(t,
// half, scale) receives the lane's 16 bits of term t's codes (element 4 sub8 + i in bits 4i..4i+3), which are bytes
// 2 sub8 and 2 sub8 + 1 of the block's 16 code bytes. `mask` names the lanes that call (whole aligned 8-lane groups).
template <class Emit>
__device__ __forceinline__ void quantize_block_digits_lanes8_masked(const float (&v)[4], unsigned mask, Emit&& emit) {
    constexpr int kOff = 4 * 299593;                            // 4 (8^7 - 1) / 7
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 4));
    const int k = fixed_schedule_k0(amax);
    const float inv = exp2i_exact(-k), sc = exp2i_exact(k);
    uint32_t w0 = 0, w1 = 0;
    int Rp[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t code;
        const float q0 = round_e2m1_code(v[i] * inv, code);
        w0 |= code << (4 * i);
        const float r = fmaf(-q0, sc, v[i]);                    // exact
        Rp[i] = __float2int_rn((r * inv) * 1048576.f) + kOff;    // in 0 .. 2^20 + kOff
        const uint32_t u1 = uint32_t(Rp[i]) >> 18;               // top digit + 4, 0..8
        w1 |= (u1 < 4 ? 12u - u1 : u1 - 4u) << (4 * i);
    }
    emit(0, w0, uint32_t(k + 127));
    emit(1, (k - 1 >= -127) ? w1 : 0u, uint32_t(max(k - 1 + 127, 0)));
#pragma unroll
    for (int t = 2; t < 8; ++t) {
        const int kt = k + 2 - 3 * t, j = 7 - t;
        uint32_t u = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) u |= ((uint32_t(Rp[i]) >> (3 * j)) & 7u) << (4 * i);
        const uint32_t hi = ((u >> 2) & 0x1111u) * 0xFu;
        const uint32_t w = (u & 0x3333u & hi) | ((0x8888u | ((~u & 0x3333u) + 0x1111u)) & ~hi & 0xFFFFu);
        emit(t, kt >= -127 ? w : 0u, uint32_t(max(kt + 127, 0)));
    }
}

// One 32-element block, one element per lane (lane l holds element l), into the 8 terms of
// quantize_block_digits_lanes4 (the same codes and scales) in the image format of quantize_block_terms_warp32<8>.
// Each lane builds its element's 8 codes as one 32-bit word (term t in nibble t), then three shuffle-and-select
// steps transpose the 8 x 8 nibble matrix of each aligned 8-lane group, after which lane l holds term (l % 8)'s codes
// of elements 8 (l / 8) .. + 7: every lane stores one code word and one scale byte. There is no per-term dependency
// chain (the digits come from one integer), unlike the residual form.
__device__ __forceinline__ void quantize_block_digits_warp32(float v, uint8_t* img_stage, int q, uint8_t* sf_chunk,
                                                            int kb, bool active) {
    constexpr int kOff = 4 * 299593;                            // 4 (8^7 - 1) / 7
    const int lane = threadIdx.x & 31;
    const float amax = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(fabsf(v))));
    const int k = fixed_schedule_k0(amax);
    const float inv = exp2i_exact(-k), sc = exp2i_exact(k);
    uint32_t code0;
    const float q0 = round_e2m1_code(v * inv, code0);
    const float r = fmaf(-q0, sc, v);                           // exact
    const uint32_t R = uint32_t(__float2int_rn((r * inv) * 1048576.f) + kOff);
    const uint32_t u1 = R >> 18;                                // top digit + 4, 0..8
    uint32_t w = code0 | ((u1 < 4 ? 12u - u1 : u1 - 4u) << 4);
    uint32_t keep = 0xFu | (k - 1 >= -127 ? 0xF0u : 0u);       // terms whose scale would fall below 2^-127: zero
#pragma unroll
    for (int t = 2; t < 8; ++t) {
        w |= balanced_digit_code((R >> (3 * (7 - t))) & 7u) << (4 * t);
        if (k + 2 - 3 * t >= -127) keep |= 0xFu << (4 * t);
    }
    w &= keep;
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) {                          // swap the off-diagonal m x m nibble blocks
        const uint32_t lo = m == 4 ? 0x0000FFFFu : (m == 2 ? 0x00FF00FFu : 0x0F0F0F0Fu);
        const uint32_t y = __shfl_xor_sync(kFull, w, m);
        w = (lane & m) ? ((w & ~lo) | ((y & ~lo) >> (4 * m))) : ((w & lo) | ((y & lo) << (4 * m)));
    }
    const int t = lane & 7;
    const int kt = t == 0 ? k : (t == 1 ? k - 1 : k + 2 - 3 * t);
    if (active) {
        *reinterpret_cast<uint32_t*>(img_stage + t * 128 + (((q ^ t) << 4) | ((lane >> 3) * 4))) = w;
        // the scale byte in all four 4-byte groups of the term's 16-byte row, as quantize_block_terms_warp32
        sf_chunk[t * 16 + (lane >> 3) * 4 + kb] = uint8_t(max(kt + 127, 0));
    }
}

// Same image format and first term as quantize_block_terms_cvt, with the later terms' scales fixed instead of
// taken from each residual's maximum: term 0 keeps the block's maximum within 6 * 2^k0, so its rounding error is at
// most 2^k0 (the e2m1 grid step is 2 between 4 and 6); term 1 uses k0 - 2 (|y| <= 4), and from then on every
// rounding error is at most half a grid step of 1, i.e. 2^(k-1), so k drops by 3 per term and |y| stays <= 4.
// After n terms the remainder is at most 2^(k0 - 3n + 3) (the subtractions are exact): below 2^-24 of the block's
// maximum after 8 terms and 2^-27 after 10. NT term rows are written (image row stride 128 bytes, NT rows per stage),
// the first min(NT, kActiveTerms) computed and the rest zero. There is no per-term maximum (no lane shuffles), and
// the rounding is round_e2m1: each term is a short chain of full-rate fp32 operations per element. Scales below
// 2^-127 are clamped there (the terms of such tiny remainders are then merely close, never NaN).
template <int NT>
__device__ __forceinline__ void quantize_block_terms_fixed_n(float (&v)[8], uint8_t* img_stage, int q,
                                                             uint8_t* sf_chunk, int kb, int sub, bool active) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
    int k = fixed_schedule_k0(amax);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        uint32_t word = 0, scale = 0;
        if (t < kActiveTerms) {
            const int kc = max(-127, k);
            const float inv = exp2i_exact(-kc), sc = exp2i_exact(kc);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t code;
                const float qv = round_e2m1_code(v[i] * inv, code);
                v[i] = fmaf(-qv, sc, v[i]);
                word |= code << (4 * i);
            }
            scale = uint32_t(kc + 127);
            k -= t == 0 ? 2 : 3;
        }
        if (active) {
            *reinterpret_cast<uint32_t*>(img_stage + t * 128 + (((q ^ (t & 7)) << 4) | (sub * 4))) = word;
            if (sub == 0) sf_chunk[(t & 31) * 16 + (t >> 5) * 4 + kb] = uint8_t(scale);
        }
    }
}

__device__ __forceinline__ void quantize_block_terms_fixed(float (&v)[8], uint8_t* img_stage, int q, uint8_t* sf_chunk,
                                                           int kb, int sub, bool active) {
    quantize_block_terms_fixed_n<kDecodeTerms>(v, img_stage, q, sf_chunk, kb, sub, active);
}

// One 32-element block quantized by a whole warp, one element per lane (lane l holds element l), for latency: the
// same terms, scales and image format as quantize_block_terms_fixed_n<NT>. The block maximum is one warp reduction;
// each term's 4-bit codes are gathered into 32-bit words (8 lanes per word) by three shuffles and stored by lanes
// 0, 8, 16 and 24. `active` must be the same in all lanes (it only suppresses the stores).
template <int NT>
__device__ __forceinline__ void quantize_block_terms_warp32(float v, uint8_t* img_stage, int q, uint8_t* sf_chunk,
                                                            int kb, bool active) {
    static_assert(NT <= 32, "one 16-byte scale row per term in a 512-byte chunk");
    const int lane = threadIdx.x & 31;
    const float amax = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(fabsf(v))));
    int k = -127;
    {
        const uint32_t bits = __float_as_uint(amax);
        const int e = int((bits >> 23) & 0xFF);
        if (e != 0) {
            const int k0 = e - 127;
            k = ((bits & 0x7FFFFFu) <= 0x400000u) ? k0 - 2 : k0 - 1;
            k = max(-127, min(127, k));
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        uint32_t nib = 0, scale = 0;
        if (t < kActiveTerms) {
            const int kc = max(-127, k);
            const float qv = round_e2m1_code(v * exp2i_exact(-kc), nib);
            v = fmaf(-qv, exp2i_exact(kc), v);
            scale = uint32_t(kc + 127);
            k -= t == 0 ? 2 : 3;
        }
        uint32_t word = nib << (4 * (lane & 7));
        word |= __shfl_xor_sync(kFull, word, 1);
        word |= __shfl_xor_sync(kFull, word, 2);
        word |= __shfl_xor_sync(kFull, word, 4);
        if (active && (lane & 7) == 0)
            *reinterpret_cast<uint32_t*>(img_stage + t * 128 + (((q ^ (t & 7)) << 4) | ((lane >> 3) * 4))) = word;
        // The scale byte goes to all four 4-byte groups of the term's 16-byte row (lanes 0-3 one each): an M = 128
        // operand whose 8-row groups alias these rows then finds term t's scale in every TMEM lane quadrant (row r
        // reads byte (r / 32) * 4 + kb of row r % 8), so every quadrant's first 8 accumulator lanes hold the terms.
        if (active && lane < 4) sf_chunk[t * 16 + lane * 4 + kb] = uint8_t(scale);
    }
}

// Quantize a whole vector (n elements, n % 32 == 0) into B terms: img [n/256 stages][terms*128],
// sf [n/128 chunks][512]. Each warp handles 8 blocks at a time; warp_id/n_warps enumerate the participating warps.
__device__ __forceinline__ void quantize_vector_terms_warp(const float* x, int n, uint8_t* img, uint8_t* sf,
                                                           int warp_id, int n_warps) {
    const int lane = threadIdx.x & 31, sub = lane & 3;
    const int nb = n / 32;
    for (int g0 = warp_id * 8; g0 < nb; g0 += n_warps * 8) {
        const int g = g0 + (lane >> 2);
        const bool active = g < nb;
        float v[8];
        if (active) {
            const float4 a = *reinterpret_cast<const float4*>(x + g * 32 + sub * 8);
            const float4 b = *reinterpret_cast<const float4*>(x + g * 32 + sub * 8 + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.f;
        }
        const int gg = active ? g : 0;
        quantize_block_terms_cvt(v, img + (gg / 8) * (kDecodeTerms * 128), gg % 8, sf + (gg / 4) * 512, gg % 4,
                                 sub, active);
    }
}

// Quantize a vector (n % 32 == 0, n <= 32 * 8 * n_warps * 3) into B terms like quantize_vector_terms_warp, with
// each warp working on up to three groups of 8 blocks at once: the three independent dependency chains (group
// maximum, scale, rounding, residual per term) overlap, so the warp takes about as long as for one group.
__device__ __forceinline__ void quantize_vector_terms_multi(const float* x, int n, uint8_t* img, uint8_t* sf,
                                                            int warp_id, int n_warps) {
    const int lane = threadIdx.x & 31, sub = lane & 3;
    const int nb = n / 32;
    float v[3][8];
    int gg[3];
    bool act[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        const int g = (warp_id + r * n_warps) * 8 + (lane >> 2);
        act[r] = g < nb;
        gg[r] = act[r] ? g : 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[r][i] = act[r] ? x[gg[r] * 32 + sub * 8 + i] : 0.f;
    }
#pragma unroll 1
    for (int t = 0; t < kDecodeTerms; ++t) {
        float amax[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            amax[r] = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax[r] = fmaxf(amax[r], fabsf(v[r][i]));
        }
#pragma unroll
        for (int r = 0; r < 3; ++r) amax[r] = fmaxf(amax[r], __shfl_xor_sync(kFull, amax[r], 1));
#pragma unroll
        for (int r = 0; r < 3; ++r) amax[r] = fmaxf(amax[r], __shfl_xor_sync(kFull, amax[r], 2));
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            int k = -127;
            const uint32_t bits = __float_as_uint(amax[r]);
            const int e = int((bits >> 23) & 0xFF);
            if (e != 0) {
                const int k0 = e - 127;
                k = ((bits & 0x7FFFFFu) <= 0x400000u) ? k0 - 2 : k0 - 1;
                k = max(-127, min(127, k));
            }
            const float inv = exp2i_exact(-k), sc = exp2i_exact(k);
            float y[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = v[r][i] * inv;
            uint32_t word, h[4];
            asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
                "cvt.rn.satfinite.e2m1x2.f32 b0, %6, %5;\n\t"
                "cvt.rn.satfinite.e2m1x2.f32 b1, %8, %7;\n\t"
                "cvt.rn.satfinite.e2m1x2.f32 b2, %10, %9;\n\t"
                "cvt.rn.satfinite.e2m1x2.f32 b3, %12, %11;\n\t"
                "cvt.rn.f16x2.e2m1x2 %1, b0;\n\t"
                "cvt.rn.f16x2.e2m1x2 %2, b1;\n\t"
                "cvt.rn.f16x2.e2m1x2 %3, b2;\n\t"
                "cvt.rn.f16x2.e2m1x2 %4, b3;\n\t"
                "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
                : "=r"(word), "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
                : "f"(y[0]), "f"(y[1]), "f"(y[2]), "f"(y[3]), "f"(y[4]), "f"(y[5]), "f"(y[6]), "f"(y[7]));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<__half2*>(&h[i]));
                v[r][2 * i] = fmaf(-f.x, sc, v[r][2 * i]);
                v[r][2 * i + 1] = fmaf(-f.y, sc, v[r][2 * i + 1]);
            }
            if (act[r]) {
                const int g = gg[r];
                uint8_t* im = img + (g / 8) * (kDecodeTerms * 128);
                *reinterpret_cast<uint32_t*>(im + t * 128 + ((((g % 8) ^ (t & 7)) << 4) | (sub * 4))) = word;
                if (sub == 0) sf[(g / 4) * 512 + (t & 31) * 16 + (t >> 5) * 4 + (g % 4)] = uint8_t(k + 127);
            }
        }
    }
}

}  // namespace gpt
