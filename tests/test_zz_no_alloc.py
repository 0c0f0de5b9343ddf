"""inferd_paged_attention_noalloc: paged attention for callers that cannot allocate.

Some callers of the C ABI cannot allocate device memory at call time -- FFI hosts that
have no device allocator of their own, and serving loops whose device-memory budget is
fixed at start-up.  This entry point uses the library's own static 32 MiB scratch area
instead of a caller-provided workspace.  Its results must match inferd_paged_attention
(called here through the Python API, which passes a workspace) within the bf16
tolerance of the other attention tests, on two consecutive calls that reuse the shared
scratch, and the fp32 oracle within the same tolerance.  Shapes that run on the generic
path use no scratch and must not be refused however large the batch.  The file name keeps
it last in collection order.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from inferd_b200 import _lib, paged_attention_batched

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _inputs(device, seed, b=16, hq=32, hkv=8, d=128, bs=16, q_len=1):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(512, 4097, (b,), generator=g)
    pages = (lens + bs - 1) // bs
    nb = int(pages.sum()) + 8
    kc = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16).to(device)
    vc = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16).to(device)
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(b, int(pages.max()), dtype=torch.int32)
    s = 0
    for i, p in enumerate(pages.tolist()):
        bt[i, :p] = perm[s:s + p].to(torch.int32)
        s += p
    q = torch.randn(b, q_len, hq, d, generator=g).to(torch.bfloat16).to(device)
    return q, kc, vc, bt.to(device), lens.to(torch.int32).to(device), int(lens.max())


def _noalloc(q, kc, vc, bt, cl, max_len, device):
    lib = _lib.load()
    out = torch.empty_like(q)
    b, q_len, hq, d = q.shape
    nb, hkv, bs, _ = kc.shape
    st = lib.inferd_paged_attention_noalloc(
        out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
        bt.element_size(), bt.stride(0), cl.data_ptr(), b, q_len, hq, hkv, d, bs, nb, max_len,
        1.0 / d ** 0.5, _lib.dtype_code(q.dtype), _lib.error_word(device).data_ptr(),
        _lib.stream_of(device))
    _lib.check(st, "inferd_paged_attention_noalloc")
    return out


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda_device):
    for call, (seed, q_len) in enumerate([(101, 1), (202, 5)]):
        q, kc, vc, bt, cl, mx = _inputs(cuda_device, seed, q_len=q_len)
        expect = paged_attention_batched(q, kc, vc, bt, cl, max_context_len=mx)
        got = _noalloc(q, kc, vc, bt, cl, mx, cuda_device)
        torch.cuda.synchronize()
        _lib.raise_device_errors(cuda_device)
        err = float((got.float() - expect.float()).abs().max())
        assert err <= ATOL, f"call {call}: max abs difference {err}"
        out = got.float().cpu().numpy()
        assert np.isfinite(out).all()
        ref = oracle.batched_paged_attention(q.float().cpu().numpy(), kc.float().cpu().numpy(),
                                             vc.float().cpu().numpy(), bt.cpu().numpy(),
                                             cl.cpu().numpy())
        err = float(np.abs(out - ref).max())
        assert err <= ATOL and err <= 1e-2 * float(np.abs(ref).max()), \
            f"call {call}: max abs error {err} against the oracle"


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    # 4096 sequences x 8 kv heads x 32 query rows needs far more than 32 MiB of partials
    need = lib.inferd_paged_attention_workspace_bytes(4096, 4, 64, 8, 128, 0)
    assert need > 32 << 20
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=cuda_device)
    st = lib.inferd_paged_attention_noalloc(
        dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
        4, 1, None, 4096, 4, 64, 8, 128, 16, 1, 16, 1.0, 2, None, _lib.stream_of(cuda_device))
    assert st == _lib.ERR_WORKSPACE


def test_noalloc_generic_path_needs_no_scratch(cuda_device):
    # head_dim 64 runs on the generic path: a batch whose tensor-core workspace would exceed
    # 32 MiB is still served, and equals the workspace entry point bit for bit
    b, q_len, hq, hkv, d, bs = 4096, 4, 64, 8, 64, 16
    assert _lib.load().inferd_paged_attention_workspace_bytes(b, q_len, hq, hkv, d, 0) > 32 << 20
    g = torch.Generator().manual_seed(7)
    lens = torch.randint(q_len, 3 * bs, (b,), generator=g)
    pages = (lens + bs - 1) // bs
    nb = int(pages.sum())
    kc = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16).to(cuda_device)
    vc = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16).to(cuda_device)
    bt = torch.zeros(b, int(pages.max()), dtype=torch.int32)
    s = 0
    for i, p in enumerate(pages.tolist()):
        bt[i, :p] = torch.arange(s, s + p, dtype=torch.int32)
        s += p
    q = torch.randn(b, q_len, hq, d, generator=g).to(torch.bfloat16).to(cuda_device)
    bt, cl = bt.to(cuda_device), lens.to(torch.int32).to(cuda_device)
    mx = int(lens.max())
    expect = paged_attention_batched(q, kc, vc, bt, cl, max_context_len=mx)
    got = _noalloc(q, kc, vc, bt, cl, mx, cuda_device)
    torch.cuda.synchronize()
    _lib.raise_device_errors(cuda_device)
    assert torch.equal(got, expect)
