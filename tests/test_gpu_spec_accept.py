"""Speculative accept / resample on the GPU (inferd_spec_accept, sampling.accept_resample)
against the oracle's restatement of core/spec_decode.py:145-161: given the same seed and
offset the same accept decisions and the same drawn tokens; and the rule's defining property,
that the first emitted token is distributed as the target's p whatever the draft's q."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from inferd_b200 import _lib
from inferd_b200.sampling import accept_resample

pytestmark = pytest.mark.gpu


def _dists(rng, b, n, vocab, scale=3.0):
    x = rng.standard_normal((b, n, vocab)).astype(np.float32) * scale
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def _run(p, q, props, seed, offset, device):
    lib = _lib.load()
    b, g1, vocab = p.shape
    gamma = g1 - 1
    pd = torch.from_numpy(p).to(device)
    qd = torch.from_numpy(q).to(device)
    xd = torch.from_numpy(props.astype(np.int64)).to(device)
    acc = torch.empty(b, dtype=torch.int32, device=device)
    tok = torch.empty(b, gamma + 1, dtype=torch.int64, device=device)
    err = _lib.error_word(device)
    st = lib.inferd_spec_accept(acc.data_ptr(), tok.data_ptr(), gamma + 1, pd.data_ptr(), g1 * vocab,
                                vocab, qd.data_ptr(), gamma * vocab, vocab, xd.data_ptr(), gamma, b,
                                gamma, vocab, seed, offset, err.data_ptr(), _lib.stream_of(device))
    _lib.check(st, "spec_accept")
    torch.cuda.synchronize()
    code = int(err.item())
    err.zero_()
    return acc.cpu().numpy(), tok.cpu().numpy(), code


def _expect(p, q, props, seed, offset):
    out = []
    for r in range(p.shape[0]):
        k, emitted = oracle.accept_resample(p[r], q[r], props[r], seed, offset, r)
        out.append((k, emitted + [-1] * (p.shape[1] - len(emitted))))
    return out


@pytest.mark.parametrize("vocab,b,gamma", [(5000, 32, 4), (151936, 16, 4), (777, 40, 1), (64, 8, 6)])
def test_matches_oracle_exactly(cuda_device, vocab, b, gamma):
    rng = np.random.default_rng(vocab + gamma)
    p = _dists(rng, b, gamma + 1, vocab)
    q = (0.7 * p[:, :gamma] + 0.3 * _dists(rng, b, gamma, vocab)).astype(np.float32)
    props = np.stack([[rng.choice(vocab, p=q[r, k] / q[r, k].sum()) for k in range(gamma)]
                      for r in range(b)]).astype(np.int64)
    seed, offset = 0xDEADBEEF1234, 77
    acc, tok, code = _run(p, q, props, seed, offset, cuda_device)
    assert code == 0
    for r, (k, emitted) in enumerate(_expect(p, q, props, seed, offset)):
        assert acc[r] == k and tok[r].tolist() == emitted, f"row {r}"
    assert 0 < acc.mean() < gamma  # both accepts and rejections occur


def test_edge_cases(cuda_device):
    rng = np.random.default_rng(3)
    vocab, gamma = 300, 3
    p = _dists(rng, 5, gamma + 1, vocab)
    q = _dists(rng, 5, gamma, vocab)
    props = rng.integers(0, vocab, (5, gamma))
    q[0] = p[0, :gamma]                       # q == p: every draft accepted, bonus from p[gamma]
    p[1, 0, props[1, 0]] = 0.0                # p(x) = 0: the first draft is rejected
    p[2, :gamma] = 0.5 * q[2]                 # residual clamp(p - q, 0) all zero: draw from p
    props[3, 1] = vocab + 5                   # not a token: rejected, reported
    seed, offset = 12345, 0
    acc, tok, code = _run(p, q, props, seed, offset, cuda_device)
    assert code == _lib.ERR_INVALID_ARGUMENT  # row 3's proposal
    assert acc[0] == gamma and tok[0, :gamma].tolist() == props[0].tolist()
    assert acc[1] == 0
    k3 = int(acc[3])  # draft 0 may be accepted or not; draft 1 is never a token
    assert k3 <= 1 and tok[3, k3] >= 0 and (tok[3, k3 + 1:] == -1).all()
    # rows 0, 1, 2 and 4 against the oracle
    for r in (0, 1, 2, 4):
        kk, em = oracle.accept_resample(p[r], q[r], props[r], seed, offset, r)
        assert acc[r] == kk and tok[r].tolist() == em + [-1] * (gamma + 1 - len(em)), f"row {r}"


def test_gamma_zero_draws_the_bonus_token(cuda_device):
    rng = np.random.default_rng(4)
    p = _dists(rng, 6, 1, 1000)
    q = np.zeros((6, 0, 1000), np.float32)
    props = np.zeros((6, 0), np.int64)
    acc, tok = accept_resample(torch.from_numpy(p).to(cuda_device), torch.from_numpy(q).to(cuda_device),
                               torch.from_numpy(props).to(cuda_device))
    assert acc.tolist() == [0] * 6 and bool((tok >= 0).all()) and tok.shape == (6, 1)


def test_first_token_is_distributed_as_p(cuda_device):
    # speculative sampling's guarantee: the first emitted token ~ p[0], whatever q is
    p0 = torch.tensor([0.05, 0.0, 0.4, 0.25, 0.3])
    q0 = torch.tensor([0.3, 0.2, 0.1, 0.2, 0.2])
    n = 200_000
    g = torch.Generator().manual_seed(1)
    props = torch.multinomial(q0, n, replacement=True, generator=g).view(n, 1)
    p = torch.stack([p0, p0], 0).expand(n, 2, 5).contiguous()
    q = q0.expand(n, 1, 5).contiguous()
    torch.manual_seed(7)
    acc, tok = accept_resample(p.to(cuda_device), q.to(cuda_device), props.to(cuda_device))
    first = tok[:, 0].cpu()
    freq = torch.bincount(first, minlength=5).double() / n
    assert freq[1] == 0.0
    ref = p0.double()
    assert torch.all((freq - ref).abs() < 5 * torch.sqrt(ref * (1 - ref) / n) + 1e-9), freq
    # acceptance rate sum_x min(p, q)
    assert abs(float(acc.float().mean()) - float(torch.minimum(p0, q0).sum())) < 0.01
