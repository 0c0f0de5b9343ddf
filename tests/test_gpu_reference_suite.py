"""The reference's paged unit tests (tests/test_paged_equiv.py:44-148 of the reference) run
against this package through the import swap a maintainer makes: the names the reference's
tests import from core.paged_attn and core.paged_cache resolve to inferd_b200's modules.

The cases are restated here (same inputs, same assertions); the only change a maintainer
makes to them is the cache device, because these kernels run on CUDA tensors only.
"""

from __future__ import annotations

import sys
import types

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def core_modules(cuda_device):
    """Alias core.paged_attn / core.paged_cache / core.paged_attn_interface to this
    package, as the import swap does, for the duration of one test."""
    from inferd_b200 import paged_attn, paged_attn_interface, paged_cache

    saved = {k: sys.modules.get(k) for k in
             ("core", "core.paged_attn", "core.paged_cache", "core.paged_attn_interface")}
    pkg = types.ModuleType("core")
    pkg.__path__ = []
    pkg.paged_attn, pkg.paged_cache, pkg.paged_attn_interface = (
        paged_attn, paged_cache, paged_attn_interface)
    sys.modules.update({"core": pkg, "core.paged_attn": paged_attn,
                        "core.paged_cache": paged_cache,
                        "core.paged_attn_interface": paged_attn_interface})
    yield cuda_device
    for k, v in saved.items():
        if v is None:
            sys.modules.pop(k, None)
        else:
            sys.modules[k] = v


def test_append_gather_across_page_boundaries(core_modules):
    from core.paged_cache import PagedKVCache

    cache = PagedKVCache(num_layers=3, num_blocks=16, block_size=16, num_kv_heads=2, head_dim=4,
                         dtype=torch.float32, device=core_modules)
    cache.create_sequence(7)
    keys, values = [], []
    for layer in range(3):
        base = torch.arange(33 * 2 * 4, dtype=torch.float32).reshape(33, 2, 4)
        keys.append((base + layer * 1000).to(core_modules))
        values.append((base + layer * 1000 + 0.5).to(core_modules))
    cache.append_tokens(7, keys, values)
    cache.assert_consistent()
    assert cache.sequence_length(7) == 33
    assert cache.allocator.allocated_count == 3
    for layer in range(3):
        got_k, got_v = cache.gather_layer(7, layer)
        torch.testing.assert_close(got_k, keys[layer])
        torch.testing.assert_close(got_v, values[layer])


def test_paged_attention_matches_independent_sdpa_reference(core_modules):
    from core.paged_attn import paged_attention, sdpa_reference
    from core.paged_cache import PagedKVCache

    torch.manual_seed(0)
    for kv_heads, q_heads in [(2, 4), (4, 4), (2, 8)]:
        for seq_len in [1, 15, 16, 17, 31, 32, 33]:
            cache = PagedKVCache(num_layers=1, num_blocks=16, block_size=16,
                                 num_kv_heads=kv_heads, head_dim=8, dtype=torch.float32,
                                 device=core_modules)
            cache.create_sequence(0)
            key = torch.randn(seq_len, kv_heads, 8).to(core_modules)
            value = torch.randn(seq_len, kv_heads, 8).to(core_modules)
            query = torch.randn(q_heads, 8).to(core_modules)
            cache.append_tokens(0, [key], [value])
            out_paged = paged_attention(query, cache.key_cache[0], cache.value_cache[0],
                                        cache.block_table(0), seq_len)
            out_ref = sdpa_reference(query, key, value)
            torch.testing.assert_close(out_paged, out_ref, rtol=1e-4, atol=1e-5,
                                       msg=f"seq_len={seq_len} kv={kv_heads} q={q_heads}")


def test_allocator_reuses_freed_blocks_without_leaks(core_modules):
    from core.paged_cache import PagedKVCache

    cache = PagedKVCache(num_layers=1, num_blocks=4, block_size=2, num_kv_heads=1, head_dim=1,
                         dtype=torch.float32, device=core_modules)
    cache.create_sequence(1)
    cache.create_sequence(2)
    one = [torch.ones(3, 1, 1, device=core_modules)]
    cache.append_tokens(1, one, one)
    first_blocks = list(cache.sequences[1].blocks)
    cache.free_sequence(1)
    cache.append_tokens(2, one, one)
    assert cache.sequences[2].blocks == first_blocks[::-1]
    cache.free_sequence(2)
    cache.assert_consistent()
    assert cache.allocator.free_count == cache.num_blocks


def test_qwen_hybrid_cache_roundtrip_preserves_attention_and_linear_state(core_modules):
    from core.paged_cache import PagedHybridCache

    class FakeQwenCache:
        pass

    dev = core_modules
    fake = FakeQwenCache()
    fake.layer_types = ["linear_attention", "full_attention", "linear_attention", "full_attention"]
    fake.transformer_layers = [1, 3]
    fake.last_linear_layer = 2
    fake.key_cache = [None, torch.randn(1, 2, 17, 8, device=dev), None,
                      torch.randn(1, 2, 17, 8, device=dev)]
    fake.value_cache = [None, torch.randn(1, 2, 17, 8, device=dev), None,
                        torch.randn(1, 2, 17, 8, device=dev)]
    fake.conv_states = [torch.randn(1, 4, 3, device=dev), None, torch.randn(1, 4, 3, device=dev),
                        None]
    fake.recurrent_states = [torch.randn(1, 4, 6, device=dev), None,
                             torch.randn(1, 4, 6, device=dev), None]
    paged = PagedHybridCache.from_qwen_cache(fake, block_size=16)
    roundtrip = paged.to_qwen_cache_like(fake)
    for layer in fake.transformer_layers:
        torch.testing.assert_close(roundtrip.key_cache[layer], fake.key_cache[layer])
        torch.testing.assert_close(roundtrip.value_cache[layer], fake.value_cache[layer])
    for layer in [0, 2]:
        torch.testing.assert_close(roundtrip.conv_states[layer], fake.conv_states[layer])
        torch.testing.assert_close(roundtrip.recurrent_states[layer],
                                   fake.recurrent_states[layer])


def test_hook_module_swap(core_modules):
    # core.paged_attn_interface resolves to the drop-in: install() patches the same global
    import core.paged_attn_interface as pai
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mm

    real = mm.eager_attention_forward
    pai.install()
    try:
        assert mm.eager_attention_forward is not real
    finally:
        pai.uninstall()
    assert mm.eager_attention_forward is real
