"""numpy restatement of the e4m3 (float8_e4m3fn) linears of both FP8 recipes.

Test infrastructure only (see oracle/__init__.py).  The reference quantises every
nn.Linear except lm_head with torchao 0.17.0 at load time (bench/model_loader.py:46-58,
applied at :82-88); torchao is a third-party dependency (uv.lock:1779-1780) that is not
vendored, so its published recipes are restated here:

* "fp8", Float8WeightOnlyConfig: per output channel n, s[n] = max_k |W[n, k]| / 448,
  q[n, k] = e4m3(W[n, k] / s[n]) with round-to-nearest-even, and the matmul is
  y = x @ (q * s)^T computed in wide precision and rounded to bf16 by the caller.
* "fp8-dynamic", Float8DynamicActivationFloat8WeightConfig (:53-55; granularity PerTensor
  by default, PerRow optional): weights at load time and activations on every forward get
  s = amax / 448 (fp32) over the tensor or the row and q = e4m3(clamp(x / s, +-448)); the
  product is s_x * s_w * (q_x @ q_w^T) (torch._scaled_mm), rounded to the activations'
  dtype.  The rounding of that rule is pinned by tests/golden/fp8_dynamic_golden.npz,
  written by torch's own e4m3 cast and _scaled_mm; torchao itself is absent, so parity with
  its exact code is unpinned.  An all-zero tensor or row gives 0 / 0 there (NaN codes and
  outputs); this restatement, like the kernels, uses s = 1 and zero codes instead.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def _code_values() -> np.ndarray:
    """Values of the 127 finite non-negative e4m3fn codes 0x00..0x7E."""
    vals = np.empty(127, dtype=np.float64)
    for code in range(127):
        exp, mant = code >> 3, code & 7
        vals[code] = mant * 2.0 ** -9 if exp == 0 else (1.0 + mant / 8.0) * 2.0 ** (exp - 7)
    return vals


_VALUES = _code_values()


def e4m3_decode(codes) -> np.ndarray:
    """uint8 e4m3fn codes -> float32 (0x7F / 0xFF are NaN)."""
    codes = np.asarray(codes, dtype=np.uint8)
    mag = codes & 0x7F
    out = np.where(mag == 0x7F, np.nan, _VALUES[np.minimum(mag, 126)])
    out = np.where(codes & 0x80, -out, out)
    return out.astype(np.float32)


def e4m3_encode(x) -> np.ndarray:
    """float32 -> uint8 e4m3fn code, round to nearest, ties to the even code.

    Finite inputs are saturated to +-448 first (inputs produced by quantize_per_channel
    never exceed 448 in magnitude by more than a rounding error).  NaN maps to 0x7F.
    """
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = np.signbit(x)
    a = np.minimum(np.abs(x), E4M3_MAX)
    hi = np.clip(np.searchsorted(_VALUES, a, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    d_hi = np.abs(_VALUES[hi] - a)
    d_lo = np.abs(a - _VALUES[lo])
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & (lo % 2 == 0))
    code = np.where(pick_lo, lo, hi).astype(np.uint8)
    code = np.where(sign, code | 0x80, code).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def quantize_per_channel(w):
    """W [N, K] (float32 view of bf16 weights) -> (q uint8 [N, K], s float32 [N]).

    s = absmax / 448 in float32; an all-zero row gets s = 1 (its codes are all zero).
    q = e4m3(float32(W / s)), the division rounded to float32 first.
    """
    w = np.asarray(w, dtype=np.float32)
    amax = np.max(np.abs(w), axis=1)
    s = (amax / np.float32(E4M3_MAX)).astype(np.float32)
    s = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
    scaled = (w / s[:, None]).astype(np.float32)
    return e4m3_encode(scaled), s


def fp8_linear(x, q, s):
    """y = x @ (dequant(q) * s)^T in float64 (returned as float64; the kernel's output is
    bf16, so callers round or compare with a bf16-sized tolerance)."""
    x = np.asarray(x, dtype=np.float64)
    w = e4m3_decode(q).astype(np.float64) * np.asarray(s, dtype=np.float64)[:, None]
    return x @ w.T


def quantize_dynamic(x, granularity: str = "tensor"):
    """x [rows, K] float32 (a view of bf16 / fp16 / fp32 values) -> (q uint8 [rows, K],
    s float32 [rows]): s = amax / 448 over the tensor (every row the same s) or per row,
    1 when amax is 0; q = e4m3(float32(x / s)), saturating."""
    x = np.asarray(x, dtype=np.float32)
    if granularity == "tensor":
        amax = np.full(x.shape[0], np.max(np.abs(x)) if x.size else 0.0, dtype=np.float32)
    elif granularity == "row":
        amax = np.max(np.abs(x), axis=1).astype(np.float32)
    else:
        raise ValueError(f"unknown granularity {granularity!r}")
    s = (amax / np.float32(E4M3_MAX)).astype(np.float32)
    s = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
    return e4m3_encode((x / s[:, None]).astype(np.float32)), s


def fp8_dynamic_linear(qx, sx, qw, sw):
    """y = s_x[m] * s_w[n] * sum_k q_x[m, k] q_w[n, k] in float64 (the kernel rounds to bf16)."""
    a = e4m3_decode(qx).astype(np.float64)
    b = e4m3_decode(qw).astype(np.float64)
    return (a @ b.T) * np.asarray(sx, np.float64)[:, None] * np.asarray(sw, np.float64)[None, :]
