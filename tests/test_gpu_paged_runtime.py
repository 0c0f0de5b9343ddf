"""PagedRuntimeCache: batched decode of a (tiny, random-init) Qwen3.5 hybrid model with its
full-attention K/V in a persistent paged pool, against HF's own per-sequence DynamicCache
path with stock eager attention."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

m = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")


def _model(dtype, device):
    torch.manual_seed(0)
    cfg = m.Qwen3_5TextConfig(
        vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, linear_num_key_heads=2,
        linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
        layer_types=["linear_attention", "full_attention", "linear_attention", "full_attention"])
    cfg._attn_implementation = "eager"
    return m.Qwen3_5ForCausalLM(cfg).to(device=device, dtype=dtype).eval()


def _reference(model, prompts, steps, device):
    """Per-sequence HF decode (stock eager attention, DynamicCache): logits per step and
    the greedy tokens fed back."""
    from transformers import DynamicCache
    out = []
    with torch.no_grad():
        for p in prompts:
            kv = DynamicCache(config=model.config)
            lg = model(torch.tensor([p], device=device), past_key_values=kv, use_cache=True).logits[:, -1]
            seq = [lg[0].float().cpu()]
            toks = []
            for _ in range(steps):
                t = int(lg.argmax(-1))
                toks.append(t)
                lg = model(torch.tensor([[t]], device=device), past_key_values=kv, use_cache=True).logits[:, -1]
                seq.append(lg[0].float().cpu())
            out.append((seq, toks))
    return out


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-3), (torch.bfloat16, 6e-2)])
def test_batched_decode_matches_per_sequence_hf(cuda_device, dtype, tol):
    from inferd_b200 import paged_attn_interface
    from inferd_b200.paged_runtime import PagedRuntimeCache

    model = _model(dtype, cuda_device)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 17, 33)]
    steps = 12
    paged_attn_interface.uninstall()
    ref = _reference(model, prompts, steps, cuda_device)

    paged_attn_interface.install()
    try:
        cache = PagedRuntimeCache(model.config, num_blocks=64, max_seqs=4, dtype=dtype, device=cuda_device)
        with torch.no_grad():
            for sid, p in enumerate(prompts):
                cache.begin_prefill(sid)
                lg = model(torch.tensor([p], device=cuda_device), past_key_values=cache, use_cache=True).logits[:, -1]
                cache.end_prefill()
                assert (lg[0].float().cpu() - ref[sid][0][0]).abs().max() < tol
            for s in range(steps):
                if s == 6:
                    cache.release(0)  # row order becomes [2, 1]: the last row moves into slot 0
                rows = list(cache.rows)
                toks = torch.tensor([[ref[sid][1][s]] for sid in rows], device=cuda_device)
                lg = model(toks, past_key_values=cache, use_cache=True,
                           position_ids=cache.position_ids()).logits[:, -1]
                for r, sid in enumerate(rows):
                    err = (lg[r].float().cpu() - ref[sid][0][s + 1]).abs().max()
                    assert err < tol, f"step {s} seq {sid}: {err}"
        assert cache.rows == [2, 1]
        assert [cache.pool.sequence_length(s) for s in cache.rows] == [33 + steps, 17 + steps]
        assert cache.pool.allocator.allocated_count == sum(
            (n + steps + 15) // 16 for n in (33, 17))  # sequence 0's pages went back
    finally:
        paged_attn_interface.uninstall()


def test_speculative_window_and_rollback(cuda_device):
    # verify a 5-token window for every row, roll back, then feed 2 "accepted" tokens: the
    # logits equal a clean HF run over prompt + those tokens (the rejected ones left no trace)
    from transformers import DynamicCache

    from inferd_b200 import paged_attn_interface
    from inferd_b200.paged_runtime import PagedRuntimeCache

    model = _model(torch.float32, cuda_device)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (14, 31)]
    window = [torch.randint(0, 512, (5,), generator=g).tolist() for _ in prompts]
    keep = [w[:2] for w in window]
    paged_attn_interface.uninstall()
    with torch.no_grad():
        clean = []
        for p, k in zip(prompts, keep):
            kv = DynamicCache(config=model.config)
            model(torch.tensor([p], device=cuda_device), past_key_values=kv, use_cache=True)
            clean.append(model(torch.tensor([k], device=cuda_device), past_key_values=kv,
                               use_cache=True).logits[0].float().cpu())
    paged_attn_interface.install()
    try:
        cache = PagedRuntimeCache(model.config, num_blocks=32, max_seqs=2, dtype=torch.float32,
                                  device=cuda_device)
        with torch.no_grad():
            for sid, p in enumerate(prompts):
                cache.begin_prefill(sid)
                model(torch.tensor([p], device=cuda_device), past_key_values=cache, use_cache=True)
                cache.end_prefill()
            free_before = cache.pool.allocator.free_count
            snap = cache.snapshot()
            pos = cache.position_ids() + torch.arange(5, device=cuda_device)
            model(torch.tensor(window, device=cuda_device), past_key_values=cache, use_cache=True,
                  position_ids=pos)
            assert [cache.pool.sequence_length(s) for s in cache.rows] == [19, 36]
            cache.restore(snap)
            assert cache.pool.allocator.free_count == free_before  # the window's blocks came back
            pos = cache.position_ids() + torch.arange(2, device=cuda_device)
            lg = model(torch.tensor(keep, device=cuda_device), past_key_values=cache, use_cache=True,
                       position_ids=pos).logits.float().cpu()
        for r in range(2):
            assert (lg[r] - clean[r]).abs().max() < 2e-3
    finally:
        paged_attn_interface.uninstall()
