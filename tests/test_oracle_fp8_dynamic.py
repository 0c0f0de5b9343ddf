"""The fp8-dynamic restatement (oracle.quantize_dynamic / fp8_dynamic_linear) against
torch's own float8_e4m3fn cast and _scaled_mm run on torchao's dynamic-scaling rule
(tests/golden/fp8_dynamic_golden.npz, written by tests/golden/make_golden.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "fp8_dynamic_golden.npz"


def _cases():
    g = np.load(GOLDEN)
    return [(i, "tensor" if c[0] == 0 else "row") for i, c in enumerate(g["dyn_cases"])]


def _bf16(v: np.ndarray) -> np.ndarray:
    """float64 -> nearest bf16 (ties to even), returned as float32."""
    f = np.asarray(v, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("i,gran", _cases())
def test_quantize_dynamic_matches_torch(i, gran):
    g = np.load(GOLDEN)
    for t in ("w", "x"):
        src, q_ref, s_ref = g[f"dyn_{i}_{t}"], g[f"dyn_{i}_q{t}"], g[f"dyn_{i}_s{t}"]
        q, s = oracle.quantize_dynamic(src, gran)
        live = np.abs(src).max(axis=1) > 0 if gran == "row" else np.ones(src.shape[0], bool)
        if gran == "tensor":
            assert np.all(s == s_ref[0])
        else:
            assert np.array_equal(s[live], s_ref[live])
        assert np.array_equal(q[live], q_ref[live]), f"{t}: e4m3 codes differ"
        # an all-zero row: torch divides 0 by 0 (NaN codes); the restatement keeps s = 1, q = 0
        if (~live).any():
            assert np.all(s_ref[~live] == 0) and np.all((q_ref[~live] & 0x7F) == 0x7F)
            assert np.all(s[~live] == 1) and np.all(q[~live] == 0)


@pytest.mark.parametrize("i,gran", _cases())
def test_dynamic_linear_matches_scaled_mm(i, gran):
    g = np.load(GOLDEN)
    qx, sx = oracle.quantize_dynamic(g[f"dyn_{i}_x"], gran)
    qw, sw = oracle.quantize_dynamic(g[f"dyn_{i}_w"], gran)
    y = _bf16(oracle.fp8_dynamic_linear(qx, sx, qw, sw))
    ref = g[f"dyn_{i}_y"]
    live = ~np.isnan(ref).any(axis=0)  # the NaN columns of an all-zero weight row
    np.testing.assert_allclose(y[:, live], ref[:, live], rtol=2 ** -7, atol=1e-6)
    assert np.mean(y[:, live] == ref[:, live]) > 0.97
    assert np.all(y[:, ~live] == 0)


def test_quantize_dynamic_edge_cases():
    x = np.zeros((3, 16), np.float32)
    q, s = oracle.quantize_dynamic(x, "tensor")
    assert np.all(q == 0) and np.all(s == 1)
    x[1, 2] = -448.0 * 3
    x[2, 5] = 1e-30  # underflows to zero code under the tensor's scale
    q, s = oracle.quantize_dynamic(x, "tensor")
    assert np.all(s == np.float32(3.0)) and q[1, 2] == 0xFE and q[2, 5] == 0
    q, s = oracle.quantize_dynamic(x, "row")
    assert s[0] == 1 and s[2] == np.float32(np.float32(1e-30) / np.float32(448)) and q[2, 5] == 0x7E
    with pytest.raises(ValueError):
        oracle.quantize_dynamic(x, "block")
