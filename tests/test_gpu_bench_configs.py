"""Parity at the benchmarked sizes: the exact inputs bench.py times, checked against the oracle.

bench.DeviceWorkload rebuilds the timed data (same seeds, lengths, pool size and block
tables).  One step runs exactly as the benchmark runs it -- a reshape_and_cache append
through the C ABI, then one paged attention launch -- and then:

* the pool holds the appended K/V bit for bit at every slot;
* every sequence's output is within 2e-2 max-abs and 1e-2 relative (max-abs error over
  max |oracle|) of the fp32 oracle on the same bf16 pages (core/paged_attn.py:64-106,
  causal inside the window for verify);
* a second step gives bitwise the same output (the split-merge counters reset).

The oracle runs one sequence at a time on pages read back from HBM, so host memory stays
small even for the 3.5 GB pool of the long-context shard.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from inferd_b200 import _lib

pytestmark = pytest.mark.gpu


def _run_and_check(wl: "bench.DeviceWorkload", device) -> None:
    wl.append()
    wl.attend()
    torch.cuda.synchronize(device)
    _lib.raise_device_errors(device)
    assert wl.appended_bit_exact()
    first = wl.out.clone()
    q = wl.q.float().cpu().numpy()
    out = first.float().cpu().numpy()
    for i in range(wl.b):
        kp, vp = wl.sequence_pages(i)
        ref = bench._oracle_sequence(q[i], kp, vp, int(wl.ctx[i]))
        err = float(np.abs(out[i] - ref).max())
        scale = float(np.abs(ref).max())
        assert err <= bench.ATOL_BF16, f"sequence {i} (context {wl.ctx[i]}): max abs error {err}"
        assert err <= bench.RTOL_BF16 * scale, f"sequence {i}: relative error {err / scale}"
    assert np.isfinite(out).all()
    wl.append()
    wl.attend()
    torch.cuda.synchronize(device)
    assert torch.equal(wl.out, first), "a repeated step changed the output"


def test_config2_decode_all_64_sequences(cuda_device):
    # 64 sequences, L ~ U[512, 8192], 32 / 8 heads: the default bench workload
    wl = bench.DeviceWorkload("decode", 0, 1, cuda_device)
    assert wl.b == 64 and wl.q_len == 1
    _run_and_check(wl, cuda_device)


def test_config3_verify_all_32_sequences(cuda_device):
    # 32 sequences, L ~ U[1024, 4096], 4 drafts + 1 query, causal inside the window
    wl = bench.DeviceWorkload("verify", 0, 1, cuda_device)
    assert wl.b == 32 and wl.q_len == 5
    _run_and_check(wl, cuda_device)


@pytest.mark.parametrize("rank,world", [(0, 1), (7, 8)])
def test_config5_long_context_full_shard(cuda_device, rank, world):
    # one GPU's full shard of config 5: 32 sequences, L ~ U[16384, 32768]; (0, 1) is the
    # single-GPU bench line, (7, 8) the last shard of the 8-GPU run
    wl = bench.DeviceWorkload("long", rank, world, cuda_device)
    assert wl.b == 32 and wl.ctx.min() >= 16384
    _run_and_check(wl, cuda_device)
    del wl
    torch.cuda.empty_cache()
