"""CPU restatement of the reference's decode-step sampling -- TEST INFRASTRUCTURE ONLY.

nucleus_probs follows core/spec_decode.py:14-31 step by step in float32: logits / T,
softmax, descending sort, inclusive cumsum, zero the entries whose exclusive cumulative
mass exceeds top_p (`cumulative - sorted_probs > top_p`, :26), scatter back, renormalise.
T <= 0 gives a one-hot row at the argmax (:18-21).  The reference sorts with torch.sort,
whose order among equal probabilities is unspecified; this restatement uses a stable
descending order (equal probabilities in index order), one valid instance of it.

sample_from (core/spec_decode.py:34-35) is torch.multinomial; its draws cannot be
reproduced, so the kernels are checked in two ways: the exact inverse-CDF rule below
(given the same random bits, the same token) and the distribution of many draws.

The fixed-point helpers state the kernels' exact arithmetic: the top-p select sums
round(p * 2^31) integers and the draw round(p * 2^52) integers (unnormalised weights first
scaled by a power of two, see weight_scale), so the kept set and the sampled token depend
on no summation order.  philox4x32_10 is the counter-based generator of Salmon, Moraes, Dror
and Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC 2011), which the sampling
kernels use for their per-row random bits.
"""

from __future__ import annotations

import numpy as np

FIXED_ONE = 1 << 52  # fixed-point scale of probability masses


def nucleus_probs(logits, temperature: float, top_p: float) -> np.ndarray:
    """Row-wise probs [..., V] (float32) after temperature and top-p, as the reference."""
    x = np.asarray(logits, dtype=np.float32)
    squeeze = x.ndim == 1
    x = np.atleast_2d(x)
    out = np.zeros_like(x, dtype=np.float32)
    for r in range(x.shape[0]):
        row = x[r]
        if temperature <= 0:
            out[r, int(np.argmax(row))] = 1.0
            continue
        y = (row / np.float32(temperature)).astype(np.float32)
        e = np.exp(y - y.max()).astype(np.float32)
        p = (e / e.sum(dtype=np.float32)).astype(np.float32)
        if top_p < 1.0:
            order = np.argsort(-p, kind="stable")
            sp = p[order]
            cum = np.cumsum(sp, dtype=np.float32)
            sp = np.where(cum - sp > np.float32(top_p), np.float32(0.0), sp).astype(np.float32)
            p = np.zeros_like(p)
            p[order] = sp
        out[r] = (p / p.sum(dtype=np.float32)).astype(np.float32)
    return out[0] if squeeze else out


def to_fixed(p) -> np.ndarray:
    """round(p * 2^52) as uint64 (p float32 >= 0; the product is exact before rounding)."""
    return np.rint(np.asarray(p, dtype=np.float32).astype(np.float64) * FIXED_ONE).astype(np.uint64)


SELECT_ONE = 1 << 31  # fixed-point scale of the masses in the top-p select


def kept_mask_fixed(p, top_p: float) -> np.ndarray:
    """The kernels' top-p rule on one row of float32 probabilities p: keep, in descending
    order with ties in index order, every entry whose exclusive cumulative mass, in
    multiples of 2^-31 (each entry rounded), is <= round(top_p * 2^31)."""
    p = np.asarray(p, dtype=np.float32)
    if top_p >= 1.0:
        return np.ones(p.shape, dtype=bool)
    q = np.rint(p.astype(np.float64) * SELECT_ONE).astype(np.uint64)
    limit = int(np.rint(np.float64(np.float32(top_p)) * SELECT_ONE))
    order = np.argsort(-p, kind="stable")
    excl = np.concatenate([[0], np.cumsum(q[order].astype(object))[:-1]])
    keep = np.zeros(p.shape, dtype=bool)
    keep[order] = np.array([int(c) <= limit for c in excl], dtype=bool)
    return keep


def weight_scale(weights) -> np.float32:
    """The power of two 2^(52 - k), 2^k >= vocab * max weight, by which the draw from
    unnormalised weights turns them into integers (the total stays <= 2^52)."""
    w = np.asarray(weights, dtype=np.float32)
    wmax = float(w.max()) if w.size else 0.0
    ex = int(np.frexp(np.float32(wmax))[1])
    lv = int(w.size - 1).bit_length() if w.size > 1 else 0
    return np.float32(2.0 ** (52 - max(0, ex + lv)))


def sample_fixed(weights, rand64: int) -> int:
    """Inverse-CDF draw over float32 weights w >= 0 in index order (sample_from): weights
    scaled by weight_scale and rounded to integers; the first index whose inclusive prefix
    exceeds floor(rand64 * total / 2^64); -1 if the total is 0."""
    w = np.asarray(weights, dtype=np.float32)
    scaled = (w * weight_scale(w)).astype(np.float32)  # exact: a power of two
    q = [int(v) for v in np.rint(scaled.astype(np.float64)).astype(np.uint64)]
    total = sum(q)
    if total == 0:
        return -1
    target = (int(rand64) * total) >> 64
    acc = 0
    for i, v in enumerate(q):
        acc += v
        if acc > target:
            return i
    return len(q) - 1


_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32_10(counter, key) -> list[int]:
    """Philox4x32 with 10 rounds: counter (4 x uint32), key (2 x uint32) -> 4 x uint32."""
    c = [int(v) & _MASK for v in counter]
    k0, k1 = int(key[0]) & _MASK, int(key[1]) & _MASK
    for r in range(10):
        p0 = _M0 * c[0]
        p1 = _M1 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & _MASK, p1 & _MASK,
             ((p0 >> 32) ^ c[3] ^ k1) & _MASK, p0 & _MASK]
        if r < 9:
            k0 = (k0 + _W0) & _MASK
            k1 = (k1 + _W1) & _MASK
    return c


def row_random64(seed: int, offset: int, row: int) -> int:
    """The 64 random bits the sampling kernels draw for `row`: Philox4x32-10 with key =
    seed (low, high words) and counter = (offset + row (low, high words), 0, 0); the first
    two output words, word 0 high."""
    n = int(offset) + int(row)
    out = philox4x32_10([n & _MASK, (n >> 32) & _MASK, 0, 0], [seed & _MASK, (seed >> 32) & _MASK])
    return (out[0] << 32) | out[1]


def row_uniform(seed: int, offset: int, row: int, stream: int) -> np.float32:
    """The uniform in [0, 1) the accept step draws for `row` on `stream` (1 + draft index):
    Philox4x32-10, key = seed, counter = (offset + row (low, high words), stream, 0); the
    top 24 bits of output word 0 times 2^-24 (the float32 grid torch.rand draws from)."""
    n = int(offset) + int(row)
    out = philox4x32_10([n & _MASK, (n >> 32) & _MASK, int(stream) & _MASK, 0],
                        [seed & _MASK, (seed >> 32) & _MASK])
    return np.float32((out[0] >> 8) * 2.0 ** -24)


def accept_resample(p, q, proposals, seed: int, offset: int, row: int):
    """core/spec_decode.py:145-161 for one sequence.  p [gamma + 1, V] are the target's
    probabilities (p[k] verifies draft token k, p[gamma] is the bonus distribution), q
    [gamma, V] the draft's, proposals [gamma] the drafted tokens.  Draft token k is accepted
    when u_k <= p[k][x_k] / q[k][x_k] (float32 division, u_k = row_uniform(.., 1 + k)); at the
    first rejection one token is drawn from clamp(p[k] - q[k], 0) (from p[k] when that is all
    zero) and the round ends; if every draft is accepted the bonus token is drawn from
    p[gamma].  Draws use sample_fixed with row_random64(seed, offset, row).  Returns
    (number accepted, emitted tokens), the tokens being the accepted drafts then the draw."""
    p = np.asarray(p, dtype=np.float32)
    q = np.asarray(q, dtype=np.float32)
    gamma = q.shape[0]
    emitted = []
    for k in range(gamma):
        x = int(proposals[k])
        with np.errstate(divide="ignore", invalid="ignore"):
            ratio = np.float32(p[k, x]) / np.float32(q[k, x])
        if row_uniform(seed, offset, row, 1 + k) <= ratio:
            emitted.append(x)
            continue
        w = np.maximum(p[k] - q[k], np.float32(0.0)).astype(np.float32)
        if not np.any(w > 0):
            w = p[k]
        emitted.append(sample_fixed(w, row_random64(seed, offset, row)))
        return k, emitted
    emitted.append(sample_fixed(p[gamma], row_random64(seed, offset, row)))
    return gamma, emitted
