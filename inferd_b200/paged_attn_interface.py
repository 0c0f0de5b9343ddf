"""Route an HF Qwen3.5 model's full attention through the paged kernels
(drop-in for core/paged_attn_interface.py).

`install()` rebinds transformers.models.qwen3_5.modeling_qwen3_5.eager_attention_forward,
exactly like the reference (core/paged_attn_interface.py:78-93), so HF keeps preparing the
eager (causal) mask.  By default only the reference's route is taken: batch 1, one query
-> paged decode; everything else -> the real eager function.  `install(routes=...)` also
enables the routes the reference left to eager:

  "batched_decode"  b > 1, q_len == 1 (left-padded rows: the unmasked keys of each row
                    are appended to a paged cache, then one batched decode launch)
  "verify"          b == 1, 1 < q_len and q_len * group <= 32 (the speculative verify
                    window, causal over the cached prefix; longer prefills stay on eager)

A model driven with a PagedRuntimeCache (inferd_b200.paged_runtime) needs only install():
its full-attention layers then read K/V from the cache's persistent pool.
"""

from __future__ import annotations

import torch

from .paged_attn import paged_attention, paged_attention_batched
from .paged_cache import PagedKVCache

_BLOCK_SIZE = 16
_MAX_VERIFY_ROWS = 32

_real_eager = None
_routes: frozenset[str] = frozenset({"decode"})
# the PagedRuntimeCache (inferd_b200.paged_runtime) whose step is in progress: its
# full-attention layers attend over its pool instead of the K/V HF passes in
_runtime = None


def _paged_cache_for(k: torch.Tensor, v: torch.Tensor, lengths: list[int]) -> tuple[PagedKVCache, list[int]]:
    """Fresh single-layer paged cache holding k/v [b, kv_heads, kv_len, dim], row i's
    last lengths[i] positions (the unpadded keys of a left-padded batch)."""
    b, num_kv_heads, kv_len, head_dim = k.shape
    blocks = sum((n + _BLOCK_SIZE - 1) // _BLOCK_SIZE for n in lengths)
    cache = PagedKVCache(num_layers=1, num_blocks=max(blocks, 1), block_size=_BLOCK_SIZE,
                         num_kv_heads=num_kv_heads, head_dim=head_dim, dtype=k.dtype,
                         device=k.device)
    for i, n in enumerate(lengths):
        cache.create_sequence(i)
        if n:
            cache.append_tokens(i, [k[i, :, kv_len - n:, :].transpose(0, 1)],
                                [v[i, :, kv_len - n:, :].transpose(0, 1)])
    return cache, list(range(b))


def paged_ref_attention_forward(
    module,
    query: torch.Tensor,   # [b, num_heads, q_len, head_dim]
    key: torch.Tensor,     # [b, num_kv_heads, kv_len, head_dim]
    value: torch.Tensor,
    attention_mask,
    scaling: float,
    dropout: float = 0.0,
    **kwargs,
):
    """HF attention hook body (core/paged_attn_interface.py:25-62).

    b == 1, q_len == 1: build a fresh paged cache, append the whole K/V history with the
    reshape_and_cache kernel, run the paged decode kernel; returns
    ([b, q_len, heads, dim], None).  Other shapes go to the real eager function unless
    an extra route was installed.
    """
    b, num_heads, q_len, head_dim = query.shape
    if b == 1 and q_len == 1:
        kv_len = key.shape[2]
        cache, _ = _paged_cache_for(key, value, [kv_len])
        q = query[0, :, 0, :]
        out = paged_attention(q, cache.key_cache[0], cache.value_cache[0],
                              cache.block_table(0), kv_len, scale=scaling)
        return out.unsqueeze(0).unsqueeze(0).to(query.dtype), None
    group = num_heads // key.shape[1]
    if b > 1 and q_len == 1 and "batched_decode" in _routes:
        return _batched_decode(query, key, value, attention_mask, scaling), None
    if b == 1 and 1 < q_len and q_len * group <= _MAX_VERIFY_ROWS and "verify" in _routes \
            and key.shape[2] >= q_len:
        return _verify(query, key, value, scaling), None
    from transformers.models.qwen3_5.modeling_qwen3_5 import eager_attention_forward
    return eager_attention_forward(
        module, query, key, value, attention_mask, scaling, dropout=dropout, **kwargs)


def _row_lengths(attention_mask, b: int, kv_len: int) -> list[int]:
    """Unmasked key count per row from HF's 4-D additive eager mask (0 = visible)."""
    if attention_mask is None:
        return [kv_len] * b
    m = attention_mask[:, 0, -1, :kv_len] if attention_mask.ndim == 4 else attention_mask
    if m.dtype == torch.bool:
        visible = m
    else:
        visible = m == 0
    return [int(x) for x in visible.sum(dim=-1).tolist()]


def _batched_decode(query, key, value, attention_mask, scaling):
    b, num_heads, _, head_dim = query.shape
    lengths = _row_lengths(attention_mask, b, key.shape[2])
    cache, ids = _paged_cache_for(key, value, lengths)
    bt, cl, max_len = cache.decode_metadata(ids)
    q = query[:, :, 0, :].to(key.dtype).unsqueeze(1).contiguous()   # [b, 1, heads, dim]
    out = paged_attention_batched(q, cache.key_cache[0], cache.value_cache[0], bt, cl,
                                  scale=scaling, max_context_len=max_len)
    return out.to(query.dtype)                                       # [b, 1, heads, dim]


def _verify(query, key, value, scaling):
    _, num_heads, q_len, head_dim = query.shape
    kv_len = key.shape[2]
    cache, ids = _paged_cache_for(key, value, [kv_len])
    bt, cl, max_len = cache.decode_metadata(ids)
    q = query[0].transpose(0, 1).to(key.dtype).unsqueeze(0).contiguous()  # [1, q_len, heads, dim]
    out = paged_attention_batched(q, cache.key_cache[0], cache.value_cache[0], bt, cl,
                                  scale=scaling, max_context_len=max_len)
    return out.to(query.dtype)                                       # [1, q_len, heads, dim]


def _wrapper(module, query, key, value, attention_mask, scaling, dropout=0.0, **kwargs):
    """Dispatch on shape (core/paged_attn_interface.py:68-75); a layer of a persistent
    PagedRuntimeCache step attends over that cache's pool."""
    rt = _runtime
    if rt is not None and rt.owns_layer(getattr(module, "layer_idx", None)):
        return rt.attend(module.layer_idx, query, scaling), None
    b, _, q_len, _ = query.shape
    group = query.shape[1] // key.shape[1]
    take = (b == 1 and q_len == 1) \
        or (b > 1 and q_len == 1 and "batched_decode" in _routes) \
        or (b == 1 and 1 < q_len and q_len * group <= _MAX_VERIFY_ROWS and "verify" in _routes
            and key.shape[2] >= q_len)
    if take:
        return paged_ref_attention_forward(
            module, query, key, value, attention_mask, scaling, dropout=dropout, **kwargs)
    return _real_eager(module, query, key, value, attention_mask, scaling, dropout=dropout, **kwargs)


def install(routes=("decode",)) -> None:
    """Route the model's full-attention steps through the paged kernels by rebinding the
    module-level eager_attention_forward symbol (core/paged_attn_interface.py:78-93).

    routes: any of "decode" (always on), "batched_decode", "verify".
    """
    global _real_eager, _routes
    unknown = set(routes) - {"decode", "batched_decode", "verify"}
    if unknown:
        raise ValueError(f"unknown routes: {sorted(unknown)}")
    from transformers.models.qwen3_5 import modeling_qwen3_5 as m
    if _real_eager is None:
        _real_eager = m.eager_attention_forward
    _routes = frozenset(routes) | {"decode"}
    m.eager_attention_forward = _wrapper


def uninstall() -> None:
    """Restore the real eager function (core/paged_attn_interface.py:96-99)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as m
    if _real_eager is not None:
        m.eager_attention_forward = _real_eager


def set_impl(runner, impl: str = "eager") -> str:
    """Force `_attn_implementation` across the backbone so mask preparation is the causal
    eager one (core/paged_attn_interface.py:102-112).  Returns the previous value."""
    prev = getattr(runner.lm.config, "_attn_implementation", "eager")
    for module in runner.lm.modules():
        cfg = getattr(module, "config", None)
        if cfg is not None and hasattr(cfg, "_attn_implementation"):
            cfg._attn_implementation = impl
    if hasattr(runner.lm, "config"):
        runner.lm.config._attn_implementation = impl
    return prev
