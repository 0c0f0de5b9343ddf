"""DecodeGraph (a decode / verify step of a fixed batch as one CUDA graph replay) against
the same steps run eagerly through PagedKVCache.plan_append / commit_append and
paged_attention_batched on an identical cache: outputs, page tables and pool bytes equal."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from inferd_b200.decode_graph import DecodeGraph
from inferd_b200.paged_attn import paged_attention_batched
from inferd_b200.paged_cache import PagedKVCache

pytestmark = pytest.mark.gpu

BS, HKV, D, HQ = 16, 2, 128, 8


def _twin_caches(device, lens, num_blocks=900, seed=0):
    g = torch.Generator().manual_seed(seed)
    caches = []
    for _ in range(2):
        caches.append(PagedKVCache(num_layers=1, num_blocks=num_blocks, block_size=BS, num_kv_heads=HKV,
                                   head_dim=D, dtype=torch.bfloat16, device=device))
    pool_k = torch.randn(num_blocks, HKV, BS, D, generator=g).to(torch.bfloat16)
    pool_v = torch.randn(num_blocks, HKV, BS, D, generator=g).to(torch.bfloat16)
    for c in caches:
        c.key_cache[0].copy_(pool_k)
        c.value_cache[0].copy_(pool_v)
    for s, n in enumerate(lens):
        k = torch.randn(n, HKV, D, generator=g).to(torch.bfloat16).to(device)
        v = torch.randn(n, HKV, D, generator=g).to(torch.bfloat16).to(device)
        for c in caches:
            c.create_sequence(s)
            c.append_tokens(s, [k], [v])
    return caches, g


@pytest.mark.parametrize("q_len,max_pairs", [(1, None), (5, None), (1, 0), (5, 2)])
def test_graph_steps_equal_eager_steps(cuda_device, q_len, max_pairs):
    # max_pairs caps the table changes one step may stage: past it prepare() sends every
    # table whole before the replay (the overflow path), which a small cap forces often
    lens = [9, 40, 130, 17, 990]  # 62 pages: the table outgrows a 64-page capacity mid-run
    (a, b), g = _twin_caches(cuda_device, lens, seed=q_len)
    ids = list(range(len(lens)))
    graph = DecodeGraph(a, ids, num_q_heads=HQ, q_len=q_len, headroom_pages=2)  # small: re-captures
    if max_pairs is not None:
        graph._max_pairs = max_pairs
    dense = 0
    real_upload = graph._upload_dense

    def counted_upload():
        nonlocal dense
        dense += 1
        real_upload()

    graph._upload_dense = counted_upload
    rng = np.random.default_rng(q_len)
    caps = set()
    assert graph._host_rows is not None  # the attention writes the pinned output itself
    for step in range(60):
        q = torch.randn(len(ids), q_len, HQ, D, generator=g).to(torch.bfloat16)
        k = torch.randn(len(ids) * q_len, HKV, D, generator=g).to(torch.bfloat16)
        v = torch.randn(len(ids) * q_len, HKV, D, generator=g).to(torch.bfloat16)
        graph.prepare()
        gq, gk, gv = graph.inputs()
        gq.copy_(q)
        gk.copy_(k)
        gv.copy_(v)
        graph.launch()
        torch.cuda.synchronize()
        out_g = graph.result().clone()
        caps.add(graph._cap)

        plan = b.plan_append(ids, q_len)
        b.commit_append(plan, [k.to(cuda_device)], [v.to(cuda_device)])
        # same launch bound as the graph's, so the kernel splits the work the same way
        out_e = paged_attention_batched(q.to(cuda_device), b.key_cache[0], b.value_cache[0],
                                        plan.block_tables, plan.context_lens,
                                        max_context_len=graph._cap * BS).cpu()
        assert torch.equal(out_g, out_e), f"step {step}"
        assert [a.sequence_length(s) for s in ids] == [b.sequence_length(s) for s in ids]
        if q_len > 1:  # verify: keep 1..q_len tokens of the window, roll the rest back
            accepted = [int(rng.integers(1, q_len + 1)) for _ in ids]
            if step % 2:
                graph.rollback(accepted)
            else:
                a.truncate_batched(ids, [a.sequence_length(s) - q_len + k for s, k in zip(ids, accepted)])
            b.truncate_batched(ids, [b.sequence_length(s) - q_len + k for s, k in zip(ids, accepted)])
    assert [a.sequences[s].blocks for s in ids] == [b.sequences[s].blocks for s in ids]
    assert torch.equal(a.key_cache[0], b.key_cache[0]) and torch.equal(a.value_cache[0], b.value_cache[0])
    assert len(caps) > 1, "the capacity never grew: the re-capture path was not exercised"
    if max_pairs is not None:
        assert dense > len(caps) + 5, "the overflow path was not exercised"


def test_rollback_argument_checks(cuda_device):
    (a, _), g = _twin_caches(cuda_device, [30, 31])
    graph = DecodeGraph(a, [0, 1], num_q_heads=HQ, q_len=3)
    with pytest.raises(RuntimeError):
        graph.rollback([1, 1])  # nothing launched yet
    graph.prepare()
    graph.launch()
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        graph.rollback([1])  # one count per sequence
    with pytest.raises(ValueError):
        graph.rollback([4, 1])  # more than the window
    assert [a.sequence_length(s) for s in (0, 1)] == [33, 34]
    graph.rollback([0, 3])
    assert [a.sequence_length(s) for s in (0, 1)] == [30, 34]
    graph.prepare()
    with pytest.raises(RuntimeError):
        graph.rollback([1, 1])  # a step is prepared
    graph.abort()
    a.assert_consistent()


def test_abort_and_exhausted_pool(cuda_device):
    (a, _), g = _twin_caches(cuda_device, [30, 31], num_blocks=8)
    ids = [0, 1]
    graph = DecodeGraph(a, ids, num_q_heads=HQ, q_len=1)
    free = a.allocator.free_count
    graph.prepare()
    with pytest.raises(RuntimeError):
        graph.prepare()  # one step at a time
    graph.abort()
    assert a.allocator.free_count == free and [a.sequence_length(s) for s in ids] == [30, 31]
    with pytest.raises(RuntimeError):
        graph.launch()
    # 8 blocks: 2 + 2 in use; 4 more steps of growth fit, then the pool runs out mid-batch
    steps = 0
    with pytest.raises(MemoryError):
        while True:
            graph.prepare()
            graph.launch()
            torch.cuda.synchronize()
            steps += 1
    assert a.allocator.free_count == 0
    lens_after = [a.sequence_length(s) for s in ids]
    assert lens_after == [30 + steps, 31 + steps]
    a.assert_consistent()


def test_host_device_pointer_of_pinned_and_pageable_memory(cuda_device):
    import ctypes

    from inferd_b200 import _lib

    lib = _lib.load()
    dptr = ctypes.c_void_p()
    pinned = torch.empty(4096, dtype=torch.uint8, pin_memory=True)
    assert lib.inferd_host_device_pointer(pinned.data_ptr(), ctypes.byref(dptr)) == _lib.OK
    assert dptr.value is not None
    pageable = torch.empty(4096, dtype=torch.uint8)
    assert lib.inferd_host_device_pointer(pageable.data_ptr(), ctypes.byref(dptr)) == _lib.ERR_CUDA
    assert lib.inferd_host_device_pointer(None, ctypes.byref(dptr)) == _lib.ERR_INVALID_ARGUMENT
    x = torch.arange(10, device=cuda_device)
    assert int(x.sum()) == 45  # no error is left behind for later launches


def test_fp32_pool_copies_the_output_after_the_grid(cuda_device):
    # fp32 pools take the generic attention kernel, which has no epilogue copy: the graph
    # falls back to a device-to-host copy after the grid, with the same results
    g = torch.Generator().manual_seed(3)
    lens = [5, 40, 77]
    caches = [PagedKVCache(num_layers=1, num_blocks=64, block_size=BS, num_kv_heads=HKV, head_dim=D,
                           dtype=torch.float32, device=cuda_device) for _ in range(2)]
    for s, n in enumerate(lens):
        k = torch.randn(n, HKV, D, generator=g).to(cuda_device)
        v = torch.randn(n, HKV, D, generator=g).to(cuda_device)
        for c in caches:
            c.create_sequence(s)
            c.append_tokens(s, [k], [v])
    a, b = caches
    ids = list(range(len(lens)))
    graph = DecodeGraph(a, ids, num_q_heads=HQ, q_len=1)
    assert graph._host_rows is None
    for step in range(3):
        q = torch.randn(len(ids), 1, HQ, D, generator=g)
        k = torch.randn(len(ids), HKV, D, generator=g)
        v = torch.randn(len(ids), HKV, D, generator=g)
        graph.prepare()
        gq, gk, gv = graph.inputs()
        gq.copy_(q)
        gk.copy_(k)
        gv.copy_(v)
        graph.launch()
        torch.cuda.synchronize()
        plan = b.plan_append(ids, 1)
        b.commit_append(plan, [k.to(cuda_device)], [v.to(cuda_device)])
        out_e = paged_attention_batched(q.to(cuda_device), b.key_cache[0], b.value_cache[0],
                                        plan.block_tables, plan.context_lens,
                                        max_context_len=graph._cap * BS).cpu()
        assert torch.equal(graph.result(), out_e), f"step {step}"
