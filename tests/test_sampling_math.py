"""CPU checks of the arithmetic the 16-bit sampling kernel relies on (no GPU needed).

* Markstein's division (P. Markstein, IBM J. Res. Dev. 34(1), 1990): with r = RN(1/d) and
  q0 = RN(x r), RN(q0 + r RN(x - d q0)) equals RN(x / d).  Checked with exact rational
  arithmetic for every bf16 value x in the range the kernel uses it for ([2^-60, 2^60] in
  magnitude) and several temperatures d, and for random (e, z) pairs of the p = e / z
  division.
* The candidate bound: with q = round(p 2^31) and L = round(top_p 2^31), every kept entry
  has p >= p_min = ((2^31 (1 - 2^-12) - V / 2 - L) / V - 1) / 2^31; the kept set computed
  over the entries with p >= p_min alone equals the kept set over the whole row; and the
  kernel's threshold on x (from p_min with its margin) admits every entry with p >= p_min.
"""

from __future__ import annotations

import math
from fractions import Fraction

import numpy as np
import pytest
import torch

import oracle


def _rn32(fr: Fraction) -> np.float32:
    """Fraction -> float32, round to nearest even (normal and subnormal range)."""
    if fr == 0:
        return np.float32(0.0)
    sign = -1 if fr < 0 else 1
    a = abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    e = max(e, -126)
    ulp = Fraction(2) ** (e - 23)
    q, rem = divmod(a, ulp)
    q = int(q)
    if rem > ulp / 2 or (rem == ulp / 2 and q % 2 == 1):
        q += 1
    return np.float32(sign * float(q * ulp))


def _markstein(x: np.float32, d: np.float32) -> np.float32:
    fx, fd = Fraction(float(x)), Fraction(float(d))
    r = _rn32(1 / fd)
    q0 = _rn32(fx * Fraction(float(r)))
    rem = _rn32(fx - fd * Fraction(float(q0)))          # fma(-q0, d, x), exact in the kernel
    return _rn32(Fraction(float(q0)) + Fraction(float(rem)) * Fraction(float(r)))  # fma(rem, r, q0)


@pytest.mark.parametrize("temp", [0.7, 1.3, 1.0 / 3.0])
def test_markstein_division_is_correctly_rounded_on_every_bf16_value(temp):
    bits = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    xs = bits[np.isfinite(bits) & (np.abs(bits) >= 2.0 ** -60) & (np.abs(bits) <= 2.0 ** 60)]
    d = np.float32(temp)
    fd = Fraction(float(d))
    bad = [float(x) for x in xs[::3] if _markstein(x, d) != _rn32(Fraction(float(x)) / fd)]
    assert not bad, bad[:5]


def test_markstein_division_of_p_by_z():
    rng = np.random.default_rng(1)
    es = (2.0 ** rng.uniform(-60, 0, 3000)).astype(np.float32)
    zs = (2.0 ** rng.uniform(0, 19, 3000)).astype(np.float32)
    for e, z in zip(es, zs):
        assert _markstein(e, z) == _rn32(Fraction(float(e)) / Fraction(float(z)))


def _pmin(vocab: int, top_p: float) -> float:
    limit = round(float(np.float32(top_p)) * 2 ** 31)
    return ((2 ** 31 * (1 - 1 / 4096) - 0.5 * vocab - limit) / vocab - 1) / 2 ** 31


def test_candidate_bound_keeps_the_kept_set():
    rng = np.random.default_rng(0)
    for trial in range(120):
        vocab = int(rng.choice([7, 100, 5000, 32785, 151936]))
        scale = float(rng.choice([0.01, 0.5, 1, 3, 8, 30]))
        t = float(rng.choice([0.3, 0.7, 1.0, 1.3, 2.0]))
        top_p = float(rng.choice([0.05, 0.3, 0.5, 0.9, 0.95, 0.99, 0.999]))
        x = (torch.from_numpy(rng.standard_normal(vocab).astype(np.float32)) * scale
             ).to(torch.bfloat16).float().numpy()
        if trial % 7 == 0:
            x = np.round(x)  # many equal logits
        y = (x / np.float32(t)).astype(np.float32)
        e = np.exp(y - y.max()).astype(np.float32)
        z = e.sum(dtype=np.float32)
        p = (e / z).astype(np.float32)
        pmin = _pmin(vocab, top_p)
        keep = oracle.kept_mask_fixed(p, np.float32(top_p))
        if pmin <= 0:
            continue
        assert np.all(p[keep] >= pmin)
        # the kernel's threshold on x: ymax + ln(p_min) + ln(z), less its margin, times T
        th = float(y.max()) + math.log(pmin) + math.log(float(z))
        th -= 1e-3 + 1e-5 * abs(th)
        xt = th * t
        xt -= 1e-5 * abs(xt)
        cand = x >= np.float32(xt)
        assert np.all(cand[p >= pmin]), "the threshold drops an entry that could be kept"
        kc = oracle.kept_mask_fixed(p[cand], np.float32(top_p))
        keep_c = np.zeros(vocab, bool)
        keep_c[np.nonzero(cand)[0][kc]] = True
        assert np.array_equal(keep_c, keep), (vocab, scale, t, top_p)
