"""GPU decode-step sampling (inferd_b200.sampling) against the reference's own
nucleus_probs outputs and the CPU oracle."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from inferd_b200 import _lib
from inferd_b200.sampling import nucleus_probs, sample_from, sample_nucleus

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "sampling_golden.npz"
CASES = [
    (4096, 1.0, 1.0, 1), (4096, 0.7, 0.9, 1), (4096, 1.3, 0.5, 1), (4096, 0.7, 0.05, 1),
    (4096, 0.0, 0.9, 1), (1000, 1.0, 0.95, 4), (32000, 0.7, 0.9, 1), (32000, 1.0, 0.99, 1),
    (7, 0.5, 0.3, 3),
]


@pytest.mark.parametrize("i", range(len(CASES)))
def test_nucleus_probs_matches_reference_outputs(cuda_device, i):
    golden = np.load(GOLDEN)
    v, t, p, rows = CASES[i]
    logits = torch.from_numpy(golden[f"samp_{i}_logits"]).to(cuda_device)
    ref = golden[f"samp_{i}_probs"]
    got = nucleus_probs(logits, t, p).cpu().numpy()
    assert got.shape == ref.shape and got.dtype == np.float32
    assert np.array_equal(got > 0, ref > 0), "kept sets differ from the reference"
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-9)


def _boundary_ok(got: np.ndarray, logits: np.ndarray, t: float, p: float) -> None:
    """Kept sets equal to the oracle's, except entries whose exclusive cumulative mass is
    within 5e-4 of top_p: the reference decides those with an fp32 cumsum over up to 262k
    sorted entries, whose rounding drifts by ~1e-5 .. 1e-4 that deep (the kernel sums
    exactly in fixed point)."""
    ref = oracle.nucleus_probs(logits, t, p)
    for r in range(ref.shape[0]):
        diff = np.nonzero((got[r] > 0) != (ref[r] > 0))[0]
        if diff.size:
            x = logits[r] / np.float32(t)
            e = np.exp(x - x.max())
            pr = e / e.sum()
            order = np.argsort(-pr, kind="stable")
            excl = np.concatenate([[0.0], np.cumsum(pr[order])[:-1]])
            pos = np.empty_like(order)
            pos[order] = np.arange(order.size)
            assert np.all(np.abs(excl[pos[diff]] - p) < 5e-4), f"row {r}: {diff.size} entries differ"
        # an entry the two rules decide differently changes the renormalisation; compare the
        # distributions renormalised over the entries both keep
        keep = (got[r] > 0) & (ref[r] > 0)
        a, b = got[r][keep].astype(np.float64), ref[r][keep].astype(np.float64)
        np.testing.assert_allclose(a / a.sum(), b / b.sum(), rtol=1e-4)


@pytest.mark.parametrize("vocab", [7, 5000, 32768 + 17, 100000, 151936, 262144])
def test_nucleus_probs_cluster_sizes(cuda_device, vocab):
    # 1, 2, 4 and 8 CTAs per row (32768 entries per CTA at most)
    g = torch.Generator().manual_seed(vocab)
    logits = torch.randn(3, vocab, generator=g) * 3.0
    got = nucleus_probs(logits.to(cuda_device), 0.8, 0.9).cpu().numpy()
    _boundary_ok(got, logits.numpy(), 0.8, 0.9)
    np.testing.assert_allclose(got.sum(axis=1), 1.0, rtol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_nucleus_probs_half_logits(cuda_device, dtype):
    # bf16 logits of a 151936 vocabulary: many equal values, including at the cut
    g = torch.Generator().manual_seed(5)
    logits = (torch.randn(4, 151936, generator=g) * 2.0).to(dtype)
    got = nucleus_probs(logits.to(cuda_device), 0.7, 0.95).cpu().numpy()
    _boundary_ok(got, logits.float().numpy(), 0.7, 0.95)


@pytest.mark.parametrize("vocab", [4096, 65536])
def test_ties_cut_in_index_order(cuda_device, vocab):
    # equal logits: p = 1/vocab exactly; entry j is kept iff j / vocab <= top_p, so the first
    # floor(top_p * vocab) + 1 indices are kept -- across CTAs when vocab = 65536
    logits = torch.zeros(2, vocab, device=cuda_device)
    got = nucleus_probs(logits, 1.0, 0.3).cpu().numpy()
    n_keep = int(np.floor(np.float32(0.3) * vocab)) + 1
    expect = np.zeros(vocab, np.float32)
    expect[:n_keep] = 1.0 / n_keep
    for r in range(2):
        assert np.count_nonzero(got[r]) == n_keep
        np.testing.assert_allclose(got[r], expect, rtol=1e-6)


def test_greedy_rows(cuda_device):
    logits = torch.randn(4, 5000, device=cuda_device)
    logits[1, 10] = logits[1, 20] = 50.0  # a tie at the max: the first index wins
    got = nucleus_probs(logits, 0.0, 0.9)
    idx = logits.argmax(dim=-1)
    idx[1] = 10
    assert torch.equal(got.argmax(dim=-1), idx) and torch.all(got.sum(dim=-1) == 1)
    tok = sample_nucleus(logits, 0.0, 0.5)
    assert tok.view(-1).tolist() == idx.tolist()


def test_per_row_temperature_and_top_p(cuda_device):
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(4, 3000, generator=g) * 3.0
    temps = torch.tensor([0.5, 1.0, 0.0, 1.5])
    tops = torch.tensor([0.9, 1.0, 0.5, 0.2])
    got = nucleus_probs(logits.to(cuda_device), temps.to(cuda_device), tops.to(cuda_device)).cpu().numpy()
    for r in range(4):
        ref = oracle.nucleus_probs(logits[r].numpy(), float(temps[r]), float(tops[r]))
        assert np.array_equal(got[r] > 0, ref > 0)
        np.testing.assert_allclose(got[r], ref, rtol=1e-5, atol=1e-9)


def test_sample_probs_exact_draws_through_c_abi(cuda_device):
    # given the same 64 random bits (Philox4x32-10, seed, counter = row) the same token
    lib = _lib.load()
    g = torch.Generator().manual_seed(3)
    rows, vocab = 64, 50000
    w = torch.rand(rows, vocab, generator=g) ** 8
    w[5, :] = 0.0
    w[5, 123] = 2.0  # a single non-zero weight
    wd = w.to(cuda_device)
    tokens = torch.empty(rows, dtype=torch.int64, device=cuda_device)
    seed = 0x1234_5678_9ABC
    err = _lib.error_word(cuda_device)
    st = lib.inferd_sample_probs(tokens.data_ptr(), wd.data_ptr(), vocab, rows, vocab, seed, 7,
                                 err.data_ptr(), _lib.stream_of(cuda_device))
    assert st == 0
    torch.cuda.synchronize()
    _lib.raise_device_errors(cuda_device)
    expect = [oracle.sample_fixed(w[r].numpy(), oracle.row_random64(seed, 7, r)) for r in range(rows)]
    assert tokens.cpu().tolist() == expect
    assert expect[5] == 123


def test_sample_from_distribution(cuda_device):
    p = torch.tensor([0.05, 0.0, 0.4, 0.25, 0.3], dtype=torch.float32)
    n = 200_000
    tok = sample_from(p.to(cuda_device).expand(n, 5).contiguous()).view(-1).cpu()
    assert tok.shape == (n,) and tok.min() >= 0 and tok.max() <= 4
    freq = torch.bincount(tok, minlength=5).double() / n
    assert freq[1] == 0.0
    assert torch.all((freq - p.double()).abs() < 5 * torch.sqrt(p.double() * (1 - p.double()) / n) + 1e-9)


def test_sample_nucleus_distribution_and_support(cuda_device):
    logits = torch.tensor([3.0, 2.5, 0.0, -1.0, 2.0, 1.0, -3.0, 0.5])
    ref = torch.from_numpy(oracle.nucleus_probs(logits.numpy(), 0.9, 0.8)).double()
    n = 200_000
    tok, probs = sample_nucleus(logits.to(cuda_device).expand(n, 8).contiguous(), 0.9, 0.8,
                                return_probs=True)
    np.testing.assert_allclose(probs[0].cpu().numpy(), ref.numpy(), rtol=1e-5)
    freq = torch.bincount(tok.view(-1).cpu(), minlength=8).double() / n
    assert torch.all(freq[ref == 0] == 0), "drew a token outside the nucleus"
    assert torch.all((freq - ref).abs() < 5 * torch.sqrt(ref * (1 - ref) / n) + 1e-9)


def test_seeded_draws_repeat_under_manual_seed(cuda_device):
    logits = torch.randn(32, 20000, device=cuda_device)
    torch.manual_seed(123)
    a = sample_nucleus(logits, 1.0, 0.95)
    torch.manual_seed(123)
    b = sample_nucleus(logits, 1.0, 0.95)
    assert torch.equal(a, b)


def test_zero_row_is_an_error(cuda_device):
    p = torch.zeros(2, 100, device=cuda_device)
    p[0, 3] = 1.0
    with pytest.raises(ValueError):
        sample_from(p)


# ------------------------------------------------------------------ 16-bit logits
# bf16 / f16 logits take the candidate kernel: the top-p select runs over the entries whose
# p can reach the cut (a bound from top_p and the vocabulary size), or over every entry when
# the candidates overflow the per-CTA lists.  Both must follow the same rule.

@pytest.mark.parametrize("scale,t,top_p", [(3.0, 0.7, 0.9), (5.0, 1.0, 0.8), (3.0, 1.3, 0.5),
                                           (8.0, 0.5, 0.99), (2.0, 0.7, 0.95)])
def test_nucleus_probs_bf16_rows(cuda_device, scale, t, top_p):
    # (3.0, 0.7, 0.9) is the sampling benchmark's row; (2.0, 0.7, 0.95) overflows the lists
    g = torch.Generator().manual_seed(int(scale * 100 + t * 10))
    logits = (torch.randn(6, 151936, generator=g) * scale).to(torch.bfloat16)
    got = nucleus_probs(logits.to(cuda_device), t, top_p).cpu().numpy()
    _boundary_ok(got, logits.float().numpy(), t, top_p)
    np.testing.assert_allclose(got.sum(axis=1), 1.0, rtol=1e-5)
    # the fp32 kernel on the same values: the same kept entries (its z is summed in another
    # order, which may move an entry sitting exactly on the cut) and the same values
    ref32 = nucleus_probs(logits.float().to(cuda_device), t, top_p).cpu().numpy()
    for r in range(got.shape[0]):
        assert np.count_nonzero((got[r] > 0) != (ref32[r] > 0)) <= 2
        both = (got[r] > 0) & (ref32[r] > 0)
        a, b = got[r][both].astype(np.float64), ref32[r][both].astype(np.float64)
        np.testing.assert_allclose(a / a.sum(), b / b.sum(), rtol=1e-5)


@pytest.mark.parametrize("n_ties,n_expect", [(256, 77), (32, 10)])
def test_bf16_tied_group_cut_across_ctas_in_index_order(cuda_device, n_ties, n_expect):
    # n_ties equal logits scattered over a 151936 vocabulary (four CTAs), everything else so
    # far below that z rounds to n_ties exactly: each tied p is 1/n_ties, so top_p = 0.3 keeps
    # the first floor(0.3 * 2^31 / q) + 1 of them in index order (256 ties: q = 2^23, 77
    # kept; 32 ties: 10 kept).  32 ties share the threshold's 16-bit prefix with nothing else,
    # so the select finishes by sorting them; 256 are too many and it runs all four passes.
    vocab = 151936
    logits = torch.full((2, vocab), -40.0)
    g = torch.Generator().manual_seed(11)
    pos = torch.randperm(vocab, generator=g)[:n_ties].sort().values
    logits[:, pos] = 10.0
    logits = logits.to(torch.bfloat16)
    got = nucleus_probs(logits.to(cuda_device), 1.0, 0.3).cpu().numpy()
    p = oracle.nucleus_probs(logits[0].float().numpy(), 1.0, 1.0)
    assert np.all(p[pos.numpy()] == np.float32(1.0 / n_ties))
    n_keep = int(oracle.kept_mask_fixed(p, 0.3).sum())
    assert n_keep == n_expect
    for r in range(2):
        kept = np.nonzero(got[r])[0]
        assert kept.tolist() == pos[:n_keep].tolist()
        np.testing.assert_allclose(got[r][kept], 1.0 / n_keep, rtol=1e-6)


@pytest.mark.parametrize("cta,tied", [(0, True), (1, False), (3, True)])
def test_bf16_one_cta_overflows_its_candidate_list(cuda_device, cta, tied):
    # 6000 high entries inside one CTA's slice (four CTAs per 151936-entry row) overflow that
    # CTA's 4096-entry candidate list: it takes the full path while the other CTAs keep
    # their lists, and the kept set still follows the one rule (ties in index order)
    vocab = 151936
    per = ((vocab + 3) // 4 + 7) // 8 * 8
    g = torch.Generator().manual_seed(40 + cta)
    logits = torch.randn(2, vocab, generator=g) * 3.0
    idx = per * cta + torch.randperm(per, generator=g)[:6000]
    logits[:, idx] = 7.0 if tied else 6.0 + torch.rand(2, 6000, generator=g)
    logits = logits.to(torch.bfloat16)
    got = nucleus_probs(logits.to(cuda_device), 0.7, 0.9).cpu().numpy()
    _boundary_ok(got, logits.float().numpy(), 0.7, 0.9)
    np.testing.assert_allclose(got.sum(axis=1), 1.0, rtol=1e-5)
    assert np.count_nonzero(got[:, idx.numpy()]) > 0  # the overflowing CTA holds kept entries


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_greedy_rows_half_logits(cuda_device, dtype):
    logits = torch.randn(4, 151936, device=cuda_device).to(dtype)
    logits[1, 1000] = logits[1, 120000] = 60.0  # a tie at the max across CTAs: the first wins
    got = nucleus_probs(logits, 0.0, 0.9)
    idx = logits.float().argmax(dim=-1)
    idx[1] = 1000
    assert torch.equal(got.argmax(dim=-1), idx) and torch.all(got.sum(dim=-1) == 1)
    tok = sample_nucleus(logits, 0.0, 0.5)
    assert tok.view(-1).tolist() == idx.tolist()


def test_sample_nucleus_bf16_distribution_and_support(cuda_device):
    logits = torch.tensor([3.0, 2.5, 0.0, -1.0, 2.0, 1.0, -3.0, 0.5])
    ref = torch.from_numpy(oracle.nucleus_probs(logits.numpy(), 0.9, 0.8)).double()
    n = 200_000
    tok, probs = sample_nucleus(logits.to(torch.bfloat16).to(cuda_device).expand(n, 8).contiguous(),
                                0.9, 0.8, return_probs=True)
    np.testing.assert_allclose(probs[0].cpu().numpy(), ref.numpy(), rtol=1e-5)
    freq = torch.bincount(tok.view(-1).cpu(), minlength=8).double() / n
    assert torch.all(freq[ref == 0] == 0), "drew a token outside the nucleus"
    assert torch.all((freq - ref).abs() < 5 * torch.sqrt(ref * (1 - ref) / n) + 1e-9)


def test_sample_nucleus_bf16_large_vocab_draws_from_the_kept_set(cuda_device):
    # draws over a full vocabulary land on kept entries, with the row's kept probabilities
    g = torch.Generator().manual_seed(21)
    logits = (torch.randn(64, 151936, generator=g) * 3.0).to(torch.bfloat16).to(cuda_device)
    torch.manual_seed(5)
    tok, probs = sample_nucleus(logits, 0.7, 0.9, return_probs=True)
    picked = probs.gather(1, tok.view(-1, 1)).view(-1)
    assert torch.all(picked > 0)
    torch.manual_seed(5)
    tok2 = sample_nucleus(logits, 0.7, 0.9)
    assert torch.equal(tok.view(-1), tok2.view(-1))  # same draws with or without probs
