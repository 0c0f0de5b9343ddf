"""GPU parity of the FP8 weight-only linear (tcgen05) and its load-time quantiser.

Quantisation (scales and e4m3 codes) must be bit-exact with the oracle, which is pinned to
torch's float8_e4m3fn cast.  The linear must be within 1e-2 relative of the oracle's
dequant-then-matmul, read normwise (an element-wise relative bound is undefined where the
exact output crosses zero): max |y - y_ref| <= 1e-2 * max |y_ref|, and for every token row
||y_m - y_ref_m||_2 <= 1e-2 * ||y_ref_m||_2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from inferd_b200.fp8_linear import (
    Fp8Linear,
    fp8_linear,
    pack_fp8_weight,
    quantize_fp8_per_channel,
    quantize_model_fp8,
)

pytestmark = pytest.mark.gpu

RTOL = 1e-2


def assert_linear_close(y: np.ndarray, ref: np.ndarray, what: str) -> None:
    err = np.abs(y - ref)
    scale = float(np.abs(ref).max())
    assert float(err.max()) <= RTOL * scale, f"{what}: max err {err.max()} vs max |ref| {scale}"
    y2, r2 = y.reshape(-1, y.shape[-1]), ref.reshape(-1, ref.shape[-1])
    row = np.linalg.norm(y2 - r2, axis=1) / np.maximum(np.linalg.norm(r2, axis=1), 1e-30)
    live = np.linalg.norm(r2, axis=1) > 0
    assert float(row[live].max(initial=0.0)) <= RTOL, \
        f"{what}: worst row relative error {row[live].max()}"


def test_quantize_matches_golden_and_oracle(cuda_device, golden):
    w = torch.from_numpy(golden["fp8_w"]).to(torch.bfloat16).to(cuda_device)
    q, s = quantize_fp8_per_channel(w)
    assert np.array_equal(s.cpu().numpy(), golden["fp8_scale"])
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), golden["fp8_q"])
    g = torch.Generator().manual_seed(3)
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        w = (torch.randn(300, 1000, generator=g) * 0.02).to(dtype)
        w[7] = 0
        q, s = quantize_fp8_per_channel(w.to(cuda_device))
        q_ref, s_ref = oracle.quantize_per_channel(w.float().numpy())
        assert np.array_equal(s.cpu().numpy(), s_ref)
        assert np.array_equal(q.view(torch.uint8).cpu().numpy(), q_ref)


@pytest.mark.parametrize("m", [1, 3, 8, 16, 32, 100, 128, 256, 300])
def test_fp8_linear_matches_dequant_matmul(cuda_device, m):
    g = torch.Generator().manual_seed(10 + m)
    n, k = 1000, 640   # partial last weight tile (1000 = 7 * 128 + 104)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    q, s = quantize_fp8_per_channel(w.to(cuda_device))
    y = fp8_linear(x.to(cuda_device), q, s)
    torch.cuda.synchronize()
    ref = oracle.fp8_linear(x.float().numpy(), q.view(torch.uint8).cpu().numpy(), s.cpu().numpy())
    assert y.shape == (m, n) and y.dtype == torch.bfloat16
    assert_linear_close(y.float().cpu().numpy(), ref, f"m={m}")


def _pack_reference(q: np.ndarray) -> np.ndarray:
    """numpy statement of the packed tile layout (zero padding to whole 256-row tile pairs,
    16-byte chunk swizzle)."""
    n, k = q.shape
    nt, kt = 2 * -(-n // 256), -(-k // 128)
    padded = np.zeros((nt * 128, kt * 128), np.uint8)
    padded[:n, :k] = q
    tiles = padded.reshape(nt, 128, kt, 8, 16).transpose(0, 2, 1, 3, 4)  # [nt, kt, r, c16, b]
    out = np.empty_like(tiles)
    r = np.arange(128)[:, None]
    c = np.arange(8)[None, :]
    out[:, :, r, c ^ (r & 7), :] = tiles[:, :, r, c, :]
    return out.reshape(-1)


# (384, 256): three weight tiles, so the second tile pair has one tile past N (padded band)
@pytest.mark.parametrize("n,k", [(256, 512), (1000, 640), (130, 144), (384, 256)])
def test_pack_layout_and_packed_linear(cuda_device, n, k):
    g = torch.Generator().manual_seed(n + k)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    q, s = quantize_fp8_per_channel(w.to(cuda_device))
    packed = pack_fp8_weight(q)
    assert np.array_equal(packed.cpu().numpy(), _pack_reference(q.view(torch.uint8).cpu().numpy()))
    x = torch.randn(37, k, generator=g).to(torch.bfloat16).to(cuda_device)
    y_row = fp8_linear(x, q, s)
    y_packed = fp8_linear(x, packed, s, packed_shape=(n, k))
    torch.cuda.synchronize()
    assert torch.equal(y_row, y_packed)  # same MMAs in the same order


@pytest.fixture(scope="module")
def config4_weight(cuda_device):
    # config-4 weight: N = 17408, K = 5120, N(0, 0.02) bf16, quantised per channel, packed
    g = torch.Generator().manual_seed(4)
    n, k = 17408, 5120
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    q, s = quantize_fp8_per_channel(w.to(cuda_device))
    packed = pack_fp8_weight(q)
    deq = (oracle.e4m3_decode(q.view(torch.uint8).cpu().numpy()).astype(np.float64)
           * s.cpu().numpy().astype(np.float64)[:, None])
    yield n, k, q, s, packed, deq
    del q, packed
    torch.cuda.empty_cache()


@pytest.mark.parametrize("m", [1, 8, 32, 128, 256])
def test_fp8_linear_config4_all_rows(cuda_device, config4_weight, m):
    # every benchmarked token count, all 17408 output channels, packed and row-major weights
    n, k, q, s, packed, deq = config4_weight
    g = torch.Generator().manual_seed(40 + m)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    ref = x.double().numpy() @ deq.T
    y = fp8_linear(x.to(cuda_device), packed, s, packed_shape=(n, k))
    y_row = fp8_linear(x.to(cuda_device), q, s)
    torch.cuda.synchronize()
    assert torch.equal(y, y_row)
    assert_linear_close(y.float().cpu().numpy(), ref, f"config 4, m={m}")


def test_fp8_linear_leading_dims_bias_and_outliers(cuda_device):
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(256, 512, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.randn(2, 3, 512, generator=g)
    x[0, 1, 17] = 900.0     # activation outlier: the per-row power-of-two scale absorbs it
    x[1, 2] = 0.0           # an all-zero row
    x = x.to(torch.bfloat16)
    bias = torch.randn(256, generator=g).to(torch.bfloat16)
    q, s = quantize_fp8_per_channel(w.to(cuda_device))
    y = fp8_linear(x.to(cuda_device), q, s, bias.to(cuda_device))
    ref = oracle.fp8_linear(x.reshape(6, 512).float().numpy(), q.view(torch.uint8).cpu().numpy(),
                            s.cpu().numpy()) + bias.float().numpy()
    assert y.shape == (2, 3, 256)
    assert_linear_close(y.reshape(6, 256).float().cpu().numpy(), ref, "leading dims")
    assert torch.all(y[1, 2] == bias.to(cuda_device))


def test_quantize_model_keeps_lm_head(cuda_device):
    model = torch.nn.Sequential()
    model.add_module("proj", torch.nn.Linear(128, 256, bias=False))
    model.add_module("lm_head", torch.nn.Linear(256, 64, bias=False))
    model = model.to(cuda_device).to(torch.bfloat16)
    x = torch.randn(4, 128, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad():
        ref = model(x).float()
        quantize_model_fp8(model)
        assert isinstance(model.proj, Fp8Linear)
        assert isinstance(model.lm_head, torch.nn.Linear)
        out = model(x).float()
    rel = float((out - ref).norm() / ref.norm())
    assert rel < 5e-2  # weight quantisation error, not a kernel tolerance


@pytest.mark.parametrize("n,k", [(200, 144), (130, 5136), (17408 - 128, 272)])
def test_fp8_linear_ragged_shapes(cuda_device, n, k):
    # K tails inside a 128-byte step, a half-empty last tile pair, and the whole-tile plan
    g = torch.Generator().manual_seed(7 * n + k)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    q, s = quantize_fp8_per_channel(w.to(cuda_device))
    for m in (5, 64, 130):
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        for packed in (False, True):
            wt = pack_fp8_weight(q) if packed else q
            y = fp8_linear(x.to(cuda_device), wt, s, packed_shape=(n, k) if packed else None)
            rows = slice(0, n) if n <= 2048 else slice(n - 1536, n)
            ref = oracle.fp8_linear(x.float().numpy(), q.view(torch.uint8).cpu().numpy()[rows], s.cpu().numpy()[rows])
            assert_linear_close(y.float().cpu().numpy()[:, rows], ref, f"n={n} k={k} m={m} packed={packed}")


@pytest.mark.parametrize("m", [1, 3, 13, 16])
def test_fp8_linear_decode_tile_equals_rows_of_a_wider_tile(cuda_device, m):
    # decode token counts on the whole-tile plan: a 16-token tile (MMA N = 32) and the
    # 32-token tile of a 17-token call (N = 64) give the same rows bit for bit (same codes,
    # scales and K order; rows past M and the K tail zero), within tolerance of the oracle
    n, k = 17408 - 128, 272   # 68 tile pairs; K = 2 * 128 + 16
    g = torch.Generator().manual_seed(90 + m)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    q, s = quantize_fp8_per_channel(w.to(cuda_device))
    packed = pack_fp8_weight(q)
    x = (torch.randn(17, k, generator=g) * torch.logspace(-3, 2, 17)[:, None]).to(torch.bfloat16)
    xd = x.to(cuda_device)
    for wt, shape in ((packed, (n, k)), (q, None)):
        y17 = fp8_linear(xd, wt, s, packed_shape=shape)
        y = fp8_linear(xd[:m], wt, s, packed_shape=shape)
        torch.cuda.synchronize()
        assert torch.equal(y, y17[:m])
    rows = slice(n - 1536, n)
    ref = oracle.fp8_linear(x[:m].float().numpy(), q.view(torch.uint8).cpu().numpy()[rows],
                            s.cpu().numpy()[rows])
    assert_linear_close(y.float().cpu().numpy()[:, rows], ref, f"m={m}")


def test_fp8_linear_out_must_be_on_device(cuda_device):
    # the GEMM writes `out` through its raw pointer: host tensors and wrong dtypes or sizes
    # are refused before anything is launched
    w = torch.zeros(384, 512, dtype=torch.bfloat16, device=cuda_device)
    q, s = quantize_fp8_per_channel(w)
    x = torch.zeros(2, 512, dtype=torch.bfloat16, device=cuda_device)
    bad = [torch.empty(2, 384, dtype=torch.bfloat16),
           torch.empty(2, 384, dtype=torch.bfloat16, pin_memory=True),
           torch.empty(2, 384, dtype=torch.float32, device=cuda_device),
           torch.empty(2, 383, dtype=torch.bfloat16, device=cuda_device)]
    for out in bad:
        with pytest.raises(ValueError):
            fp8_linear(x, q, s, out=out)
    good = torch.empty(2, 384, dtype=torch.bfloat16, device=cuda_device)
    assert fp8_linear(x, q, s, out=good).data_ptr() == good.data_ptr()
