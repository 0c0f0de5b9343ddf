"""GPU parity of the fp8-dynamic recipe (torchao Float8DynamicActivationFloat8WeightConfig,
bench/model_loader.py:53-55): dynamic e4m3 quantisation and the one-plane tcgen05 linear.

Quantisation (scales and codes) must be bit-exact with torch's float8 cast on torchao's
rule (the golden file) and with the oracle.  The linear must equal the oracle's float64
s_x * s_w * (q_x @ q_w^T) rounded to bf16 within fp32 accumulation error:
|y - y_ref| <= 2^-7 |y_ref| + 2^-14 max |y_ref| everywhere, and >= 90 % of entries
bit-identical.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from inferd_b200 import _lib
from inferd_b200.fp8_linear import (
    Fp8DynamicLinear,
    fp8_dynamic_linear,
    pack_fp8_weight,
    quantize_fp8_dynamic,
    quantize_model_fp8,
)

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "fp8_dynamic_golden.npz"


def _bf16(v: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.asarray(v, dtype=np.float64)).to(torch.bfloat16).float().numpy()


def assert_gemm_exact(y: np.ndarray, ref64: np.ndarray, what: str) -> None:
    ref = _bf16(ref64)
    bound = 2.0 ** -7 * np.abs(ref) + 2.0 ** -14 * float(np.abs(ref).max())
    bad = np.abs(y - ref) > bound
    assert not bad.any(), f"{what}: {int(bad.sum())} entries outside the bound"
    assert np.mean(y == ref) >= 0.9, f"{what}: only {np.mean(y == ref):.3f} bit-identical"


def _quant(t: torch.Tensor, gran: str):
    q, s = quantize_fp8_dynamic(t, gran)
    return q.view(torch.uint8).cpu().numpy(), s.cpu().numpy()


@pytest.mark.parametrize("i", range(3))
def test_quantize_dynamic_matches_golden(cuda_device, i):
    g = np.load(GOLDEN)
    gran = "tensor" if g["dyn_cases"][i][0] == 0 else "row"
    for t in ("w", "x"):
        src = torch.from_numpy(g[f"dyn_{i}_{t}"]).to(torch.bfloat16).to(cuda_device)
        q, s = _quant(src, gran)
        q_ref, s_ref = g[f"dyn_{i}_q{t}"], g[f"dyn_{i}_s{t}"]
        live = s_ref > 0 if gran == "row" else np.ones(q.shape[0], bool)
        assert np.array_equal(s[live], np.broadcast_to(s_ref, s.shape)[live] if gran == "tensor" else s_ref[live])
        assert np.array_equal(q[live], q_ref[live])
        assert np.all(s[~live] == 1) and np.all(q[~live] == 0)  # all-zero row: s = 1, zero codes


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("gran", ["tensor", "row"])
def test_quantize_dynamic_matches_oracle(cuda_device, dtype, gran):
    g = torch.Generator().manual_seed(21)
    x = (torch.randn(300, 1000, generator=g) * 2.0)
    x[3, 4] = 5e3
    x[7] = 0.0
    x[9, :7] = torch.tensor([1e-6, -1e-7, 3e-8, 1.0, -1.0, 0.5, 2.0])  # subnormal codes under the tensor's scale
    x = x.to(dtype)
    q, s = _quant(x.to(cuda_device), gran)
    q_ref, s_ref = oracle.quantize_dynamic(x.float().numpy(), gran)
    assert np.array_equal(s, s_ref)
    assert np.array_equal(q, q_ref)


@pytest.mark.parametrize("i", range(3))
def test_dynamic_linear_matches_golden(cuda_device, i):
    g = np.load(GOLDEN)
    gran = "tensor" if g["dyn_cases"][i][0] == 0 else "row"
    w = torch.from_numpy(g[f"dyn_{i}_w"]).to(torch.bfloat16).to(cuda_device)
    x = torch.from_numpy(g[f"dyn_{i}_x"]).to(torch.bfloat16).to(cuda_device)
    qw, sw = quantize_fp8_dynamic(w, gran)
    n, k = w.shape
    for packed in (False, True):
        wt = pack_fp8_weight(qw) if packed else qw
        y = fp8_dynamic_linear(x, wt, sw, granularity=gran, packed_shape=(n, k) if packed else None)
        y = y.float().cpu().numpy()
        ref = g[f"dyn_{i}_y"]
        live = ~np.isnan(ref).any(axis=0)  # torch's 0/0 columns of an all-zero weight row
        np.testing.assert_allclose(y[:, live], ref[:, live], rtol=2 ** -7, atol=1e-6)
        assert np.all(y[:, ~live] == 0)


@pytest.mark.parametrize("gran", ["tensor", "row"])
@pytest.mark.parametrize("m", [1, 3, 16, 40, 128, 200, 256, 300])
def test_dynamic_linear_matches_oracle(cuda_device, gran, m):
    g = torch.Generator().manual_seed(100 + m)
    n, k = 1000, 640  # a partial last weight tile
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g)
    x[m // 2, 11] = 40.0
    x = x.to(torch.bfloat16).to(cuda_device)
    qw, sw = quantize_fp8_dynamic(w.to(cuda_device), gran)
    y = fp8_dynamic_linear(x, qw, sw, granularity=gran).float().cpu().numpy()
    qx, sx = _quant(x, gran)
    ref = oracle.fp8_dynamic_linear(qx, sx, qw.view(torch.uint8).cpu().numpy(), sw.cpu().numpy())
    assert_gemm_exact(y, ref, f"m={m} {gran}")


@pytest.fixture(scope="module")
def config4_dynamic_weight(cuda_device):
    # config-4 weight: N = 17408, K = 5120, N(0, 0.02), per-tensor scales, packed tiles
    g = torch.Generator().manual_seed(4)
    n, k = 17408, 5120
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    qw, sw = quantize_fp8_dynamic(w)
    packed = pack_fp8_weight(qw)
    yield n, k, qw.view(torch.uint8).cpu().numpy(), sw.cpu().numpy(), packed, sw
    del w, qw, packed
    torch.cuda.empty_cache()


@pytest.mark.parametrize("m", [1, 8, 32, 128, 256])
def test_dynamic_linear_config4_all_rows(cuda_device, config4_dynamic_weight, m):
    # every benchmarked token count over all 17408 output channels
    n, k, qw, sw_host, packed, sw = config4_dynamic_weight
    g = torch.Generator().manual_seed(400 + m)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(cuda_device)
    y = fp8_dynamic_linear(x, packed, sw, packed_shape=(n, k)).float().cpu().numpy()
    qx, sx = _quant(x, "tensor")
    ref = oracle.fp8_dynamic_linear(qx, sx, qw, sw_host)
    assert_gemm_exact(y, ref, f"config 4, m={m}")


def test_per_tensor_scale_spans_the_batch(cuda_device):
    # one row's outlier sets every row's scale (torchao's PerTensor): row 0 alone differs
    g = torch.Generator().manual_seed(8)
    w = (torch.randn(256, 512, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    x = torch.randn(4, 512, generator=g).to(torch.bfloat16).to(cuda_device)
    x[3, 0] = 300.0
    qw, sw = quantize_fp8_dynamic(w)
    batch = fp8_dynamic_linear(x, qw, sw)
    alone = fp8_dynamic_linear(x[:1], qw, sw)
    assert not torch.equal(batch[:1], alone)
    by_row = fp8_dynamic_linear(x, qw, sw, granularity="row")
    assert torch.equal(by_row[:1], fp8_dynamic_linear(x[:1], qw, sw, granularity="row"))


def test_leading_dims_bias_zero_input_and_model_helper(cuda_device):
    g = torch.Generator().manual_seed(6)
    w = (torch.randn(256, 512, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    bias = torch.randn(256, generator=g).to(torch.bfloat16).to(cuda_device)
    qw, sw = quantize_fp8_dynamic(w)
    x = torch.randn(2, 3, 512, generator=g).to(torch.bfloat16).to(cuda_device)
    y = fp8_dynamic_linear(x, qw, sw, bias)
    flat = fp8_dynamic_linear(x.reshape(6, 512), qw, sw) + bias
    assert y.shape == (2, 3, 256) and torch.equal(y.reshape(6, 256), flat)
    zero = fp8_dynamic_linear(torch.zeros(5, 512, dtype=torch.bfloat16, device=cuda_device), qw, sw)
    assert torch.all(zero == 0)

    model = torch.nn.Sequential()
    model.add_module("proj", torch.nn.Linear(128, 256, bias=True))
    model.add_module("lm_head", torch.nn.Linear(256, 64, bias=False))
    model = model.to(cuda_device).to(torch.bfloat16)
    xin = torch.randn(4, 128, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad():
        ref = model(xin).float()
        quantize_model_fp8(model, recipe="fp8-dynamic")
        assert isinstance(model.proj, Fp8DynamicLinear)
        assert isinstance(model.lm_head, torch.nn.Linear)
        out = model(xin).float()
    assert float((out - ref).norm() / ref.norm()) < 8e-2  # e4m3 activations and weights
    with pytest.raises(ValueError, match="unknown fp8 recipe"):
        quantize_model_fp8(model, recipe="fp8-blockwise")
    with pytest.raises(ValueError):
        fp8_dynamic_linear(xin, qw, sw, granularity="block")


def test_c_abi_rejects_bad_granularity(cuda_device):
    lib = _lib.load()
    x = torch.zeros(2, 32, dtype=torch.bfloat16, device=cuda_device)
    q = torch.empty(2, 32, dtype=torch.uint8, device=cuda_device)
    s = torch.empty(2, dtype=torch.float32, device=cuda_device)
    st = lib.inferd_fp8_quantize_dynamic(x.data_ptr(), 2, q.data_ptr(), s.data_ptr(), 2, 32, 7, None,
                                         _lib.stream_of(cuda_device))
    assert st == _lib.ERR_INVALID_ARGUMENT
    st = lib.inferd_fp8_quantize_dynamic(x.data_ptr(), 2, q.data_ptr(), s.data_ptr(), 2, 32, 0, None,
                                         _lib.stream_of(cuda_device))
    assert st == _lib.ERR_INVALID_ARGUMENT  # per tensor needs the row_amax scratch
    st = lib.inferd_fp8_dynamic_linear(None, None, None, None, 1, 1, 16, 0, 3, None, ctypes.c_size_t(0),
                                       _lib.stream_of(cuda_device))
    assert st == _lib.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("n,k", [(200, 144), (130, 5136), (17408 - 128, 272)])
@pytest.mark.parametrize("gran", ["tensor", "row"])
def test_dynamic_linear_ragged_shapes(cuda_device, n, k, gran):
    # K not a multiple of the 128-byte K step (TMA zero-fills the tail), N ending in a half
    # empty tile pair, and a config-4-wide N whose last pair holds one tile (whole-tile plan)
    g = torch.Generator().manual_seed(n + k)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    for m in (3, 40):
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(cuda_device)
        qw, sw = quantize_fp8_dynamic(w, gran)
        for packed in (False, True):
            wt = pack_fp8_weight(qw) if packed else qw
            y = fp8_dynamic_linear(x, wt, sw, granularity=gran, packed_shape=(n, k) if packed else None)
            qx, sx = _quant(x, gran)
            cols = slice(0, n) if n <= 2048 else slice(n - 1536, n)
            ref = oracle.fp8_dynamic_linear(qx, sx, qw.view(torch.uint8).cpu().numpy()[cols], sw.cpu().numpy()[cols])
            assert_gemm_exact(y.float().cpu().numpy()[:, cols], ref, f"n={n} k={k} m={m} packed={packed}")
