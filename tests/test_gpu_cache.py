"""GPU parity of the KV-pool kernels (reshape_and_cache, gather) -- bit-exact.

Reference behaviour: core/paged_cache.py:151-205 (append_tokens, gather_layer) and
core/paged_attn.py:20-61 (gather_paged_kv); tests mirror the reference's
tests/test_paged_equiv.py:44-69,106-125 and core/paged_cache.py:370-420 selfcheck.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from inferd_b200 import _lib, gather_paged_kv
from inferd_b200.paged_cache import PagedHybridCache, PagedKVCache

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    view = {4: torch.int32, 2: torch.int16, 1: torch.uint8}[t.element_size()]
    return t.view(view).numpy()


@pytest.mark.parametrize("dtype", DTYPES)
def test_append_gather_across_page_boundaries(cuda_device, dtype):
    # reference tests/test_paged_equiv.py:44-69 on the device, in three dtypes
    cache = PagedKVCache(num_layers=3, num_blocks=16, block_size=16, num_kv_heads=2,
                         head_dim=4, dtype=dtype, device=cuda_device)
    cache.create_sequence(7)
    layer_keys, layer_values = [], []
    for layer in range(3):
        base = torch.arange(33 * 2 * 4, dtype=torch.float32).reshape(33, 2, 4)
        layer_keys.append((base + layer * 1000).to(dtype).to(cuda_device))
        layer_values.append((base + layer * 1000 + 0.5).to(dtype).to(cuda_device))
    cache.append_tokens(7, layer_keys, layer_values)
    cache.assert_consistent()
    assert cache.sequence_length(7) == 33
    assert cache.allocator.allocated_count == 3
    for layer in range(3):
        got_k, got_v = cache.gather_layer(7, layer)
        assert np.array_equal(_bits(got_k), _bits(layer_keys[layer]))
        assert np.array_equal(_bits(got_v), _bits(layer_values[layer]))


def test_selfcheck_trace(cuda_device):
    # core/paged_cache.py:370-400 selfcheck on the device
    cache = PagedKVCache(num_layers=2, num_blocks=8, block_size=4, num_kv_heads=3, head_dim=5,
                         dtype=torch.float32, device=cuda_device)
    cache.create_sequence(10)
    keys = [torch.arange(7 * 3 * 5, dtype=torch.float32).reshape(7, 3, 5).to(cuda_device)
            + layer * 10_000 for layer in range(2)]
    values = [k + 0.25 for k in keys]
    cache.append_tokens(10, keys, values)
    cache.assert_consistent()
    assert cache.sequence_length(10) == 7 and cache.allocator.allocated_count == 2
    for layer in range(2):
        got_k, got_v = cache.gather_layer(10, layer)
        assert torch.equal(got_k, keys[layer]) and torch.equal(got_v, values[layer])
    cache.create_sequence(11)
    one = [torch.ones(1, 3, 5, device=cuda_device) for _ in range(2)]
    cache.append_tokens(11, one, one)
    cache.free_sequence(10)
    cache.free_sequence(11)
    cache.assert_consistent()
    assert cache.allocator.free_count == cache.num_blocks


@pytest.mark.parametrize("dtype", DTYPES)
def test_reshape_and_cache_matches_oracle_bit_exact(cuda_device, dtype):
    g = torch.Generator().manual_seed(11)
    nb, hkv, bs, d = 40, 4, 16, 128
    kc = torch.randn(nb, hkv, bs, d, generator=g).to(dtype)
    vc = torch.randn(nb, hkv, bs, d, generator=g).to(dtype)
    n = 77
    k = torch.randn(n, hkv, d, generator=g).to(dtype)
    v = torch.randn(n, hkv, d, generator=g).to(dtype)
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int64)
    slots[5] = -1  # padding token: skipped
    kc_d, vc_d = kc.to(cuda_device), vc.to(cuda_device)
    lib = _lib.load()
    # zero tokens is a no-op that touches no pointer
    st = lib.inferd_reshape_and_cache(None, None, 0, 0, 0, 0, None, None, None, 0,
                                      hkv, d, bs, nb, _lib.dtype_code(dtype), None, None)
    assert st == _lib.OK
    kd, vd, sd = k.to(cuda_device), v.to(cuda_device), slots.to(cuda_device)
    st = lib.inferd_reshape_and_cache(
        kd.data_ptr(), vd.data_ptr(), kd.stride(0), kd.stride(1), vd.stride(0), vd.stride(1),
        kc_d.data_ptr(), vc_d.data_ptr(), sd.data_ptr(), n, hkv, d, bs, nb,
        _lib.dtype_code(dtype), _lib.error_word(cuda_device).data_ptr(),
        _lib.stream_of(cuda_device))
    _lib.check(st, "reshape_and_cache")
    torch.cuda.synchronize()
    _lib.raise_device_errors(cuda_device)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    # oracle works on the raw bit patterns so the comparison is exact for every dtype
    kb, vb = _bits(kc_ref).copy(), _bits(vc_ref).copy()
    oracle.reshape_and_cache(kb, vb, _bits(k), _bits(v), slots.numpy())
    assert np.array_equal(_bits(kc_d), kb)
    assert np.array_equal(_bits(vc_d), vb)


def test_reshape_and_cache_strided_input(cuda_device):
    # HF K/V arrive as [1, heads, seq, dim]; the kernel reads the transposed view in place
    g = torch.Generator().manual_seed(12)
    hkv, L, d = 8, 50, 128
    k = torch.randn(1, hkv, L, d, generator=g).to(torch.bfloat16).to(cuda_device)
    v = torch.randn(1, hkv, L, d, generator=g).to(torch.bfloat16).to(cuda_device)
    cache = PagedKVCache(num_layers=1, num_blocks=8, block_size=16, num_kv_heads=hkv,
                         head_dim=d, dtype=torch.bfloat16, device=cuda_device)
    cache.create_sequence(0)
    cache.append_tokens(0, [k[0].transpose(0, 1)], [v[0].transpose(0, 1)])
    gk, gv = cache.gather_layer(0, 0)
    assert torch.equal(gk, k[0].transpose(0, 1)) and torch.equal(gv, v[0].transpose(0, 1))


def test_reshape_and_cache_out_of_pool_slot_reports_index_error(cuda_device):
    nb, hkv, bs, d = 4, 2, 16, 128
    kc = torch.zeros(nb, hkv, bs, d, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    k = torch.ones(2, hkv, d, dtype=torch.bfloat16, device=cuda_device)
    slots = torch.tensor([3, nb * bs + 5], dtype=torch.int64, device=cuda_device)
    lib = _lib.load()
    st = lib.inferd_reshape_and_cache(
        k.data_ptr(), k.data_ptr(), k.stride(0), k.stride(1), k.stride(0), k.stride(1),
        kc.data_ptr(), vc.data_ptr(), slots.data_ptr(), 2, hkv, d, bs, nb,
        _lib.dtype_code(torch.bfloat16), _lib.error_word(cuda_device).data_ptr(),
        _lib.stream_of(cuda_device))
    _lib.check(st, "reshape_and_cache")
    with pytest.raises(IndexError):
        _lib.raise_device_errors(cuda_device)
    # the in-range token was written, nothing else was touched
    assert torch.equal(kc[0, :, 3, :], k[0])
    assert int((kc != 0).sum()) == hkv * d


def test_gather_bad_block_raises_index_error(cuda_device):
    kb = torch.zeros(4, 2, 16, 8, device=cuda_device)
    with pytest.raises(IndexError):
        gather_paged_kv(kb, kb, torch.tensor([0, 9]), 20)


def test_cfg1_append_matches_reference(cuda_device, golden):
    # config 1 append: one token per sequence at slot L_i; the reference's bookkeeping
    # (tables, slots) and its pool after the append are pinned by the golden file
    from tests.golden.make_golden import CFG1, cfg1_inputs

    inp = cfg1_inputs()
    c = CFG1
    cache = PagedKVCache(num_layers=1, num_blocks=c["num_blocks"], block_size=c["block_size"],
                         num_kv_heads=c["kv_heads"], head_dim=c["head_dim"], dtype=torch.float32,
                         device=cuda_device)
    cache.key_cache[0].copy_(torch.from_numpy(inp["key_cache"]))
    cache.value_cache[0].copy_(torch.from_numpy(inp["value_cache"]))
    used = set()
    for b, L in enumerate(c["lens"]):
        t = cache.create_sequence(b)
        t.blocks = [int(x) for x in inp["tables"][b]]
        t.length = L
        used.update(t.blocks)
    cache.allocator._allocated = set(used)
    cache.allocator._free = [x for x in cache.allocator._free if x not in used]
    seq_ids = list(range(len(c["lens"])))
    nk = torch.from_numpy(inp["new_k"]).to(cuda_device)
    nv = torch.from_numpy(inp["new_v"]).to(cuda_device)
    cache.append_tokens_batched(seq_ids, [nk], [nv])
    cache.assert_consistent()
    slots = [cache.sequences[b].slots(L, 1)[0] for b, L in enumerate(c["lens"])]
    assert slots == golden["cfg1_append_slots"].tolist()
    for b in seq_ids:
        bl = cache.sequences[b].blocks
        assert bl == golden["cfg1_tables_after"][b][: len(bl)].tolist()
    ksum = cache.key_cache[0].cpu().numpy().view(np.uint32).astype(np.uint64).sum()
    vsum = cache.value_cache[0].cpu().numpy().view(np.uint32).astype(np.uint64).sum()
    assert ksum == golden["cfg1_pool_k_after_sum"][0]
    assert vsum == golden["cfg1_pool_v_after_sum"][0]


def test_hybrid_cache_roundtrip(cuda_device):
    # reference tests/test_paged_equiv.py:127-148 on the device
    class FakeQwenCache:
        pass

    fake = FakeQwenCache()
    fake.layer_types = ["linear_attention", "full_attention", "linear_attention", "full_attention"]
    fake.transformer_layers = [1, 3]
    fake.last_linear_layer = 2
    dev = cuda_device
    fake.key_cache = [None, torch.randn(1, 2, 17, 8, device=dev), None, torch.randn(1, 2, 17, 8, device=dev)]
    fake.value_cache = [None, torch.randn(1, 2, 17, 8, device=dev), None, torch.randn(1, 2, 17, 8, device=dev)]
    fake.conv_states = [torch.randn(1, 4, 3, device=dev), None, torch.randn(1, 4, 3, device=dev), None]
    fake.recurrent_states = [torch.randn(1, 4, 6, device=dev), None, torch.randn(1, 4, 6, device=dev), None]
    paged = PagedHybridCache.from_qwen_cache(fake, block_size=16)
    rt = paged.to_qwen_cache_like(fake)
    for layer in fake.transformer_layers:
        assert torch.equal(rt.key_cache[layer], fake.key_cache[layer])
        assert torch.equal(rt.value_cache[layer], fake.value_cache[layer])
    for layer in [0, 2]:
        assert torch.equal(rt.conv_states[layer], fake.conv_states[layer])
        assert torch.equal(rt.recurrent_states[layer], fake.recurrent_states[layer])


def test_decode_metadata_device_refresh_matches_rebuild(cuda_device):
    # the device-resident tables are refreshed with sparse (column, block) updates; after
    # appends, block-crossing growth, multi-sequence rollbacks, a replaced list and batch
    # reorders they must equal tables rebuilt from the host page tables
    cache = PagedKVCache(num_layers=1, num_blocks=600, block_size=4, num_kv_heads=1, head_dim=8,
                         dtype=torch.bfloat16, device=cuda_device)
    rng = np.random.default_rng(5)
    ids = list(range(7))
    for s in ids:
        cache.create_sequence(s)
        n = int(rng.integers(1, 40))
        kv = torch.zeros(n, 1, 8, dtype=torch.bfloat16, device=cuda_device)
        cache.append_tokens(s, [kv], [kv])
    for step in range(150):
        per = 1 if step % 5 else 3
        kv = torch.zeros(len(ids) * per, 1, 8, dtype=torch.bfloat16, device=cuda_device)
        cache.append_tokens_batched(ids, [kv], [kv])
        for s in ids:
            if rng.random() < 0.2:
                cache.truncate_sequence(s, int(rng.integers(0, cache.sequence_length(s) + 1)))
        if step == 60:
            cache.sequences[3].blocks = list(cache.sequences[3].blocks)
        if step == 90:  # a long sequence: the table outgrows the cached capacity
            kv = torch.zeros(400, 1, 8, dtype=torch.bfloat16, device=cuda_device)
            cache.append_tokens(2, [kv], [kv])
        order = ids if step % 13 else ids[::-1]
        bt, cl, mx = cache.decode_metadata(order, extra_tokens=step % 3)
        width = max(len(cache.sequences[s].blocks) for s in order)
        rows = [cache.sequences[s].blocks + [0] * (width - len(cache.sequences[s].blocks)) for s in order]
        assert bt.is_cuda and bt.dtype == torch.int32 and bt.shape == (len(order), width)
        assert bt.cpu().tolist() == rows, f"step {step}"
        assert cl.cpu().tolist() == [cache.sequence_length(s) + step % 3 for s in order]
        assert mx == max(cl.cpu().tolist())
