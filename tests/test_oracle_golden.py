"""Pin the CPU oracle to outputs of the reference itself (tests/golden/reference_golden.npz).

The fixtures were produced by tests/golden/make_golden.py from the reference's own
core.paged_attn / core.paged_cache, from transformers' eager attention (the verify path
of core/spec_decode.py:135) and from torch's float8_e4m3fn cast.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.make_golden import CFG1, cfg1_inputs


@pytest.mark.parametrize("kv_heads,q_heads", [(2, 4), (4, 4), (2, 8)])
@pytest.mark.parametrize("seq_len", [1, 15, 16, 17, 31, 32, 33])
def test_unit_sweep(golden, kv_heads, q_heads, seq_len):
    tag = f"unit_{kv_heads}_{q_heads}_{seq_len}"
    key, value = golden[tag + "_key"], golden[tag + "_value"]
    query, table = golden[tag + "_query"], golden[tag + "_table"]
    # rebuild the pool the reference's cache held: blocks 0.. in allocation order
    nb, bs = 16, 16
    kc = np.zeros((nb, kv_heads, bs, 8), np.float32)
    vc = np.zeros_like(kc)
    slots = [int(table[p // bs]) * bs + p % bs for p in range(seq_len)]
    oracle.reshape_and_cache(kc, vc, key, value, slots)
    out = oracle.paged_attention(query, kc, vc, table, seq_len)
    np.testing.assert_allclose(out, golden[tag + "_paged"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out, golden[tag + "_sdpa"], rtol=1e-4, atol=1e-5)
    ind = oracle.sdpa_attention(query, key, value)
    np.testing.assert_allclose(ind, golden[tag + "_sdpa"], rtol=1e-4, atol=1e-5)


def test_cfg1_matches_reference(golden):
    inp = cfg1_inputs()
    for b, L in enumerate(CFG1["lens"]):
        out = oracle.paged_attention(inp["query"][b], inp["key_cache"], inp["value_cache"],
                                     inp["tables"][b], L)
        np.testing.assert_allclose(out, golden[f"cfg1_out_fp32_{b}"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(out, golden[f"cfg1_sdpa_fp32_{b}"], rtol=1e-4, atol=1e-5)


def test_cfg1_append_bit_exact(golden):
    inp = cfg1_inputs()
    kc, vc = inp["key_cache"].copy(), inp["value_cache"].copy()
    slots = golden["cfg1_append_slots"]
    oracle.reshape_and_cache(kc, vc, inp["new_k"], inp["new_v"], slots)
    assert kc.view(np.uint32).astype(np.uint64).sum() == golden["cfg1_pool_k_after_sum"][0]
    assert vc.view(np.uint32).astype(np.uint64).sum() == golden["cfg1_pool_v_after_sum"][0]


@pytest.mark.parametrize("case", range(4))
def test_verify_matches_hf_eager(golden, case):
    out = oracle.verify_attention(golden[f"verify_{case}_query"], golden[f"verify_{case}_key"],
                                  golden[f"verify_{case}_value"])
    np.testing.assert_allclose(out, golden[f"verify_{case}_out"], rtol=1e-4, atol=1e-5)


def test_verify_single_query_equals_decode(golden):
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 16, 32), dtype=np.float32)
    k = rng.standard_normal((50, 4, 32), dtype=np.float32)
    v = rng.standard_normal((50, 4, 32), dtype=np.float32)
    np.testing.assert_allclose(oracle.verify_attention(q, k, v)[0],
                               oracle.dense_attention(q[0], k, v), rtol=1e-6, atol=1e-7)


def test_e4m3_codes_match_torch(golden):
    assert np.array_equal(oracle.e4m3_encode(golden["e4m3_in"]), golden["e4m3_code"])
    vals = golden["e4m3_all_codes_value"]
    dec = oracle.e4m3_decode(np.arange(256, dtype=np.uint8))
    finite = np.isfinite(vals)
    assert np.array_equal(np.isnan(dec), ~finite)
    assert np.array_equal(dec[finite], vals[finite])


def test_quantize_and_linear_match_torch(golden):
    q, s = oracle.quantize_per_channel(golden["fp8_w"])
    assert np.array_equal(s, golden["fp8_scale"])
    assert np.array_equal(q, golden["fp8_q"])
    y = oracle.fp8_linear(golden["fp8_x"], q, s)
    np.testing.assert_allclose(y, golden["fp8_y"], rtol=1e-12, atol=1e-12)


def test_gather_errors_match_reference():
    kc = np.zeros((4, 2, 16, 8), np.float32)
    with pytest.raises(ValueError):
        oracle.gather_paged_kv(kc, kc, np.array([0]), 20)
    with pytest.raises(ValueError):
        oracle.gather_paged_kv(kc, kc, np.array([0]), -1)
    with pytest.raises(ValueError):
        oracle.gather_paged_kv(kc, kc[:3], np.array([0]), 1)
    with pytest.raises(IndexError):
        oracle.gather_paged_kv(kc, kc, np.array([0, 7]), 20)
    k, v = oracle.gather_paged_kv(kc, kc, np.array([], dtype=np.int64), 0)
    assert k.shape == (0, 2, 8)
