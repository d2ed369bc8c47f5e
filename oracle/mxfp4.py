"""CPU oracle (test infrastructure only): MXFP4 decoding restated in numpy.

This module is a checker. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it; the
product path (the CUDA library) never imports or calls it.

Restates reference/gptoss_ref/mxfp4.py of openvang/gptoss-infer:
  * FP4_VALUES               mxfp4.py:11-12   e2m1 code -> value, codes 8..15 negate 0..7 (code 8 is -0.0)
  * dequant(blocks, scales)  mxfp4.py:17-31   byte j of a block: element 2j = LOW nibble, 2j+1 = HIGH nibble;
                                              value = e2m1 * 2**(scale - 127); scale 0xFF (NaN) is rejected
  * e8m0_to_float(scales)    mxfp4.py:34-39   exact power of two from the bit pattern; s == 0 is 2**-127
  * quantize(weights)        mxfp4.py:47-67   test helper: smallest power-of-two scale with max|w| <= 6, then
                                              nearest e2m1 code (ties to the lower code, like argmin)
Parity is pinned by tests/test_oracle.py against the reference's own known-answer tests
(reference/tests/test_mxfp4.py:7-62) and against golden vectors produced by the reference itself
(tests/golden/make_golden.py).
"""
import numpy as np

FP4_VALUES = (+0.0, +0.5, +1.0, +1.5, +2.0, +3.0, +4.0, +6.0,
              -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)
BLOCK = 32
BYTES_PER_BLOCK = 16

# byte -> (value of the low nibble, value of the high nibble), fp32
_BYTE_LUT = np.array([[FP4_VALUES[b & 0x0F], FP4_VALUES[b >> 4]] for b in range(256)], dtype=np.float32)


def e8m0_to_float(scales):
    """uint8 E8M0 -> float32 2**(s-127), built from the bit pattern (mxfp4.py:34-39)."""
    s = np.asarray(scales)
    bits = s.astype(np.uint32) << np.uint32(23)
    bits = np.where(s == 0, np.uint32(0x00400000), bits).astype(np.uint32)
    return bits.view(np.float32)


def dequant(blocks, scales):
    """blocks uint8 [..., G, 16], scales uint8 [..., G] -> float32 [..., G*32] (mxfp4.py:17-31)."""
    blocks, scales = np.asarray(blocks), np.asarray(scales)
    if blocks.dtype != np.uint8 or scales.dtype != np.uint8:
        raise TypeError("blocks and scales must be uint8")
    if blocks.shape[-1] != BYTES_PER_BLOCK or blocks.shape[:-1] != scales.shape:
        raise ValueError(f"shape mismatch: blocks {blocks.shape} scales {scales.shape}")
    if (scales == 255).any():
        raise ValueError("E8M0 scale 0xFF encodes NaN in the OCP MX spec; refusing to decode it")
    vals = _BYTE_LUT[blocks]                                   # [..., G, 16, 2]
    vals = vals.reshape(*blocks.shape[:-1], BLOCK)             # [..., G, 32]: low nibble first per byte
    with np.errstate(over="ignore"):                   # 6 * 2**127 overflows to inf, as in the reference
        out = vals * e8m0_to_float(scales)[..., None]
    return out.reshape(*scales.shape[:-1], scales.shape[-1] * BLOCK)


def quantize(weights):
    """fp32 [..., K] -> (blocks uint8 [..., K/32, 16], scales uint8 [..., K/32]) (mxfp4.py:47-67)."""
    w = np.asarray(weights, dtype=np.float32)
    *lead, k = w.shape
    if k % BLOCK:
        raise ValueError("last dim must be a multiple of 32")
    w = w.reshape(*lead, k // BLOCK, BLOCK)
    amax = np.maximum(np.abs(w).max(axis=-1), np.float32(2.0 ** -120))
    exp = np.clip(np.ceil(np.log2(amax / np.float32(6.0))), -127, 127)
    scales = (exp + 127).astype(np.uint8)
    scaled = w / np.exp2(exp).astype(np.float32)[..., None]
    grid = np.array(FP4_VALUES[:8], dtype=np.float32)
    code = np.abs(np.abs(scaled)[..., None] - grid).argmin(axis=-1)      # 0..7, first minimum wins
    code = (code + 8 * (scaled < 0)).astype(np.uint8)
    blocks = code[..., 0::2] | (code[..., 1::2] << 4)
    return np.ascontiguousarray(blocks), np.ascontiguousarray(scales)
