"""numpy restatement of the reference's paged KV gather, append and attention.

Test infrastructure only (see oracle/__init__.py).  Arrays are numpy; floating-point
work is done in float32 like the reference's fp32 path, with bf16 inputs widened to
float32 exactly before they reach these functions.
"""

from __future__ import annotations

import math

import numpy as np


def gather_paged_kv(key_blocks, value_blocks, block_table, seq_len):
    """core/paged_attn.py:20-61 -- pages of one sequence back to [seq_len, kv_heads, dim].

    Same argument checks as the reference (:37-46): seq_len >= 0, identical K/V shapes,
    4-D blocks, block table long enough.  Block ids outside the pool raise IndexError,
    as torch indexing does in the reference.
    """
    key_blocks = np.asarray(key_blocks)
    value_blocks = np.asarray(value_blocks)
    block_table = np.asarray(block_table).reshape(-1)
    if seq_len < 0:
        raise ValueError("seq_len must be non-negative")
    if key_blocks.shape != value_blocks.shape:
        raise ValueError("key/value block tensors must have identical shape")
    if key_blocks.ndim != 4:
        raise ValueError("block tensors must be [blocks, heads, block_size, head_dim]")
    num_blocks, kv_heads, block_size, head_dim = key_blocks.shape
    needed = (seq_len + block_size - 1) // block_size
    if block_table.size < needed:
        raise ValueError("block_table is shorter than seq_len requires")
    if seq_len == 0:
        empty = np.empty((0, kv_heads, head_dim), dtype=key_blocks.dtype)
        return empty, empty.copy()
    ids = block_table[:needed].astype(np.int64)
    if ids.min() < 0 or ids.max() >= num_blocks:
        raise IndexError("block id outside the pool")
    # [pages, heads, bs, dim] -> [pages, bs, heads, dim] -> [pages*bs, heads, dim]
    k = key_blocks[ids].transpose(0, 2, 1, 3).reshape(needed * block_size, kv_heads, head_dim)
    v = value_blocks[ids].transpose(0, 2, 1, 3).reshape(needed * block_size, kv_heads, head_dim)
    return k[:seq_len].copy(), v[:seq_len].copy()


def _softmax_rows(x):
    m = np.max(x, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(x - m)
    s = np.sum(e, axis=-1, keepdims=True)
    return np.divide(e, s, out=np.zeros_like(e), where=s > 0)


def dense_attention(query, key, value, scale=None):
    """core/paged_attn.py:64-106 -- single-query GQA attention, no mask, in float32.

    query [q_heads, dim]; key/value [seq, kv_heads, dim] -> [q_heads, dim].  Query head h
    reads kv head h // group (repeat_interleave order, :98-100); scores = q.K * scale;
    softmax in fp32 (:104-105); out = P.V (:106).  An empty key set gives zeros, as the
    reference's einsum over a zero-length axis does.
    """
    query = np.asarray(query, dtype=np.float32)
    key = np.asarray(key, dtype=np.float32)
    value = np.asarray(value, dtype=np.float32)
    if query.ndim != 2 or key.ndim != 3 or value.ndim != 3:
        raise ValueError("expected query [q_heads, dim], key/value [seq, kv_heads, dim]")
    if key.shape != value.shape:
        raise ValueError("key/value shapes differ")
    if query.shape[-1] != key.shape[-1]:
        raise ValueError("query/key head_dim differs")
    q_heads, kv_heads = query.shape[0], key.shape[1]
    if q_heads % kv_heads != 0:
        raise ValueError("q_heads must be a multiple of kv_heads")
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    group = q_heads // kv_heads
    out = np.zeros_like(query)
    if key.shape[0] == 0:
        return out
    for h in range(kv_heads):
        q = query[h * group:(h + 1) * group]            # [group, dim]
        s = (q @ key[:, h, :].T) * np.float32(scale)     # [group, seq]
        p = _softmax_rows(s.astype(np.float32))
        out[h * group:(h + 1) * group] = p @ value[:, h, :]
    return out


def paged_attention(query, key_blocks, value_blocks, block_table, seq_len, scale=None):
    """core/paged_attn.py:134-167 -- gather then dense attention for one sequence."""
    k, v = gather_paged_kv(key_blocks, value_blocks, block_table, seq_len)
    return dense_attention(query, k, v, scale=scale)


def verify_attention(query, key, value, scale=None):
    """Causal multi-query attention of the speculative verify step.

    query [q_len, q_heads, dim] holds the last q_len positions of a sequence whose keys
    key/value [seq, kv_heads, dim] include those q_len positions.  Query i (absolute
    position seq - q_len + i) sees keys 0 .. seq - q_len + i, the causal mask HF builds
    for the verify forward of core/spec_decode.py:135; softmax in fp32 as in
    transformers' eager_attention_forward.  Returns [q_len, q_heads, dim].
    """
    query = np.asarray(query, dtype=np.float32)
    key = np.asarray(key, dtype=np.float32)
    value = np.asarray(value, dtype=np.float32)
    q_len, q_heads, dim = query.shape
    seq, kv_heads, _ = key.shape
    if q_heads % kv_heads != 0:
        raise ValueError("q_heads must be a multiple of kv_heads")
    if scale is None:
        scale = 1.0 / math.sqrt(dim)
    group = q_heads // kv_heads
    out = np.zeros_like(query)
    pos = np.arange(seq)
    for i in range(q_len):
        visible = pos <= seq - q_len + i
        if not visible.any():
            continue
        for h in range(kv_heads):
            q = query[i, h * group:(h + 1) * group]
            s = (q @ key[visible, h, :].T) * np.float32(scale)
            p = _softmax_rows(s.astype(np.float32))
            out[i, h * group:(h + 1) * group] = p @ value[visible, h, :]
    return out


def sdpa_attention(query, key, value, scale=None):
    """Independent float64 formulation (core/paged_attn.py:109-131 plays this role in
    the reference): explicit repeat of K/V per query head, max-subtracted softmax.
    query [q_heads, dim], key/value [seq, kv_heads, dim]."""
    q = np.asarray(query, dtype=np.float64)
    k = np.asarray(key, dtype=np.float64)
    v = np.asarray(value, dtype=np.float64)
    q_heads, kv_heads = q.shape[0], k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    kh = np.repeat(k, q_heads // kv_heads, axis=1)  # [seq, q_heads, dim]
    vh = np.repeat(v, q_heads // kv_heads, axis=1)
    s = np.einsum("hd,shd->hs", q, kh) * scale
    if s.shape[1] == 0:
        return np.zeros_like(q)
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return np.einsum("hs,shd->hd", p, vh)


def batched_paged_attention(query, key_cache, value_cache, block_tables, context_lens,
                            scale=None):
    """Per-sequence loop of the reference algorithm over a batch, as the reference's
    callers do (bench/runners/paged.py:120-140): query [B, q_len, q_heads, dim],
    block_tables [B, P], context_lens [B] (keys visible to the last query).  q_len == 1
    is paged_attention; q_len > 1 is verify_attention over the gathered keys."""
    query = np.asarray(query, dtype=np.float32)
    b_count, q_len = query.shape[0], query.shape[1]
    out = np.zeros_like(query)
    kc = np.asarray(key_cache, dtype=np.float32)
    vc = np.asarray(value_cache, dtype=np.float32)
    for b in range(b_count):
        L = int(context_lens[b])
        k, v = gather_paged_kv(kc, vc, block_tables[b], L)
        if q_len == 1:
            out[b, 0] = dense_attention(query[b, 0], k, v, scale=scale)
        else:
            out[b] = verify_attention(query[b], k, v, scale=scale)
    return out


def reshape_and_cache(key_cache, value_cache, key, value, slots):
    """core/paged_cache.py:177-183 -- key_cache[block, :, offset, :] = key[token] with
    (block, offset) = divmod(slot, block_size); slots < 0 are skipped.  In place, exact."""
    block_size = key_cache.shape[2]
    for t, slot in enumerate(np.asarray(slots).reshape(-1).tolist()):
        if slot < 0:
            continue
        blk, off = divmod(int(slot), block_size)
        if blk >= key_cache.shape[0]:
            raise IndexError("slot outside the pool")
        key_cache[blk, :, off, :] = key[t]
        value_cache[blk, :, off, :] = value[t]
    return key_cache, value_cache
