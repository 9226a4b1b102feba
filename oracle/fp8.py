"""Oracle for the block-FP8 linear (TEST INFRASTRUCTURE; numpy).

Restates qwen3_8/fp8_triton.py of yz29528/tokenFactory:
  quantize_act        - fp8_triton.py:124-130   amax in the activation dtype, clamp(min=1e-12) and
                                                 / 448 in that dtype, then x / x_scale in fp32,
                                                 clamp to +-448, round to e4m3 (nearest even)
  block_fp8_linear    - fp8_triton.py:17-98     out = sum over K of q * w * (x_scale * w_scale
                                                 [n // bh, k // bw]) + bias, in float64 here (the
                                                 kernel's fp32 tile sums are compared within a
                                                 tolerance)
e4m3 ("fn" variant: no infinities, 0x7f / 0xff NaN, largest finite 448): 1 sign, 4 exponent
bits (bias 7), 3 mantissa bits, subnormals below 2^-6 in steps of 2^-9.
"""

from typing import Optional

import numpy as np

from . import bf16 as _bf


def e4m3_decode(bits: np.ndarray) -> np.ndarray:
    b = bits.astype(np.int32)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * np.exp2(e.astype(np.float64) - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Round to nearest, ties to even, of finite values with |x| <= 448."""
    x = x.astype(np.float64)
    sign = (np.signbit(x)).astype(np.uint8) << 7
    a = np.abs(x)
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)                      # subnormal range shares the 2^-6 exponent
    step = np.exp2(e - 3)                        # spacing of representable values there
    k = a / step
    r = np.floor(k)
    frac = k - r
    r = np.where((frac > 0.5) | ((frac == 0.5) & (r % 2 == 1)), r + 1, r)
    v = r * step                                 # the rounded magnitude (may reach the next binade)
    ev = np.floor(np.log2(np.where(v > 0, v, 1.0)))
    normal = v >= 2.0 ** -6
    exp_bits = np.where(normal, ev + 7, 0).astype(np.int64)
    man = np.where(normal, np.round((v / np.exp2(ev) - 1.0) * 8), np.round(v / 2.0 ** -9)).astype(np.int64)
    bits = (exp_bits << 3) | man
    bits = np.where(v == 0, 0, bits)
    return (bits.astype(np.uint8) | sign).astype(np.uint8)


def quantize_act(x: np.ndarray, dtype: str):
    """(e4m3 bits [M, K], x_scale float32) of the wrapper's activation quantization."""
    xf = _bf.as_f32(x, dtype)
    amax = np.float32(np.max(np.abs(xf))) if xf.size else np.float32(0)
    c = np.maximum(amax, np.float32(1e-12))
    if dtype == "bf16":
        c = _bf.round_f32(np.asarray([c], np.float32))[0]
        s = _bf.round_f32(np.asarray([np.float32(c) / np.float32(448.0)], np.float32))[0]
    else:
        s = np.float32(c) / np.float32(448.0)
    s = np.float32(s)
    q = np.clip(xf / s, np.float32(-448.0), np.float32(448.0)).astype(np.float32)
    return e4m3_encode(q), s


def block_fp8_linear(q_bits: np.ndarray, x_scale: float, w_bits: np.ndarray,
                     w_scale: Optional[np.ndarray], bias: Optional[np.ndarray],
                     block_h: int = 128, block_w: int = 128) -> np.ndarray:
    """float64 value of the kernel's output before the cast to the output dtype."""
    q = e4m3_decode(q_bits).astype(np.float64)
    w = e4m3_decode(w_bits).astype(np.float64)
    N, K = w.shape
    if w_scale is not None:
        sc = np.repeat(np.repeat(w_scale.astype(np.float64), block_h, 0)[:N], block_w, 1)[:, :K]
        w = w * sc
    out = (q @ w.T) * float(x_scale)
    if bias is not None:
        out = out + bias.astype(np.float64)[None, :]
    return out
