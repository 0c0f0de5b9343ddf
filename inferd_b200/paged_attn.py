"""Paged attention over a block-table KV pool (drop-in for the reference's core/paged_attn.py).

The single-sequence functions keep the reference's names, argument order and error
behaviour (core/paged_attn.py:20-167); their bodies call the sm_100a kernels in
libinferd_sm100a.so instead of a Python page loop plus einsum.  The batched entry
points (`paged_attention_batched`, `paged_decode`, `paged_verify`) are what a batched
runtime calls: one launch for every sequence of a step, no host synchronisation.

Tensor layouts:
    key_blocks / value_blocks : [num_blocks, kv_heads, block_size, head_dim]
    query (single sequence)   : [q_heads, head_dim]
    query (batched)           : [num_seqs, q_len, q_heads, head_dim]
    block_tables              : [num_seqs, max_pages] int32 or int64
    context_lens              : [num_seqs] int32 (keys visible to the last query)
"""

from __future__ import annotations

import math

import torch

from . import _lib

# Single-sequence compatibility calls synchronise once to turn a device-side block-id
# error into the IndexError the reference raises; the batched calls never synchronise.
_SYNC_CHECKS = True


def set_sync_checks(enabled: bool) -> bool:
    """Enable/disable the post-call device error check of the single-sequence API."""
    global _SYNC_CHECKS
    prev = _SYNC_CHECKS
    _SYNC_CHECKS = bool(enabled)
    return prev


def reserve_sms(sms: int) -> int:
    """Leave `sms` SMs out of the persistent attention grids launched from now on
    (process-wide; 0 restores full grids), for a collective that runs beside the attention
    on another stream with at most that many CTAs, so that none of the attention's
    statically assigned CTAs waits for it.  Returns the previous value."""
    lib = _lib.load()
    prev = int(lib.inferd_paged_attention_reserved_sms())
    _lib.check(lib.inferd_paged_attention_reserve_sms(int(sms)), "paged_attention_reserve_sms")
    return prev


def _check_blocks(key_blocks: torch.Tensor, value_blocks: torch.Tensor) -> None:
    if key_blocks.shape != value_blocks.shape:
        raise ValueError("key/value block tensors must have identical shape")
    if key_blocks.ndim != 4:
        raise ValueError("block tensors must be [blocks, heads, block_size, head_dim]")


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def gather_paged_kv(
    key_blocks: torch.Tensor,
    value_blocks: torch.Tensor,
    block_table: torch.Tensor,
    seq_len: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather one sequence's K/V pages into contiguous [seq_len, kv_heads, head_dim].

    Same checks as core/paged_attn.py:37-46; one gather kernel instead of a per-page
    Python loop with a host sync per page (:51-56).
    """
    if seq_len < 0:
        raise ValueError("seq_len must be non-negative")
    _check_blocks(key_blocks, value_blocks)
    num_blocks, kv_heads, block_size, head_dim = key_blocks.shape
    needed_pages = (seq_len + block_size - 1) // block_size
    if block_table.numel() < needed_pages:
        raise ValueError("block_table is shorter than seq_len requires")
    dev = _lib.require_cuda(key_blocks, value_blocks)
    k_out = key_blocks.new_empty((seq_len, kv_heads, head_dim))
    v_out = value_blocks.new_empty((seq_len, kv_heads, head_dim))
    if seq_len == 0:
        return k_out, v_out
    table = _table_on(block_table, dev)
    kb, vb = _contig(key_blocks), _contig(value_blocks)
    lib = _lib.load()
    st = lib.inferd_gather_paged_kv(
        k_out.data_ptr(), v_out.data_ptr(), kb.data_ptr(), vb.data_ptr(), table.data_ptr(),
        table.element_size(), seq_len, kv_heads, head_dim, block_size, num_blocks,
        _lib.dtype_code(key_blocks.dtype), _lib.error_word(dev).data_ptr(), _lib.stream_of(dev))
    _lib.check(st, "gather_paged_kv")
    if _SYNC_CHECKS:
        _lib.raise_device_errors(dev)
    return k_out, v_out


def _table_on(block_table: torch.Tensor, dev: torch.device) -> torch.Tensor:
    t = block_table.reshape(-1)
    if t.dtype not in (torch.int32, torch.int64):
        t = t.to(torch.int64)
    if t.device != dev:
        t = t.to(dev)
    return _contig(t)


def _check_dense(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> None:
    if query.ndim != 2 or key.ndim != 3 or value.ndim != 3:
        raise ValueError("expected query [q_heads, dim], key/value [seq, kv_heads, dim]")
    if key.shape != value.shape:
        raise ValueError("key/value shapes differ")
    if query.shape[-1] != key.shape[-1]:
        raise ValueError("query/key head_dim differs")
    if query.shape[0] % key.shape[1] != 0:
        raise ValueError("q_heads must be a multiple of kv_heads")


def dense_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    scale: float | None = None,
) -> torch.Tensor:
    """Single-query GQA decode attention over contiguous K/V (core/paged_attn.py:64-106).

    query [q_heads, head_dim], key/value [seq_len, kv_heads, head_dim] -> [q_heads, head_dim]
    in the value dtype.  No causal mask (the one query sees every key).  Computed by the
    generic fp32-accumulating CUDA kernel.
    """
    _check_dense(query, key, value)
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    dev = _lib.require_cuda(query, key, value)
    q = _contig(query.to(value.dtype))
    k, v = _contig(key), _contig(value)
    out = torch.empty(query.shape, dtype=value.dtype, device=dev)
    lib = _lib.load()
    st = lib.inferd_dense_attention(
        out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), key.shape[0], 1,
        query.shape[0], key.shape[1], query.shape[1], float(scale),
        _lib.dtype_code(value.dtype), _lib.stream_of(dev))
    _lib.check(st, "dense_attention")
    return out


def sdpa_reference(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    scale: float | None = None,
) -> torch.Tensor:
    """Independent single-query reference through torch's fused SDPA (the role of
    core/paged_attn.py:109-131): fp32 math on repeat-interleaved K/V, cast back to the
    value dtype.  Kept for callers that validate against it; it is not on the kernel path.
    """
    q_heads = query.shape[0]
    kv_heads = key.shape[1]
    group = q_heads // kv_heads
    q = query.unsqueeze(0).unsqueeze(2).float()
    k = key.repeat_interleave(group, dim=1).transpose(0, 1).unsqueeze(0).float()
    v = value.repeat_interleave(group, dim=1).transpose(0, 1).unsqueeze(0).float()
    out = torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale)
    return out.squeeze(2).squeeze(0).to(value.dtype)


def paged_attention_reference(
    query: torch.Tensor,
    key_blocks: torch.Tensor,
    value_blocks: torch.Tensor,
    block_table: torch.Tensor,
    seq_len: int,
    *,
    scale: float | None = None,
) -> torch.Tensor:
    """Gather-then-attend formulation (core/paged_attn.py:134-144), both steps as kernels."""
    key, value = gather_paged_kv(key_blocks, value_blocks, block_table, seq_len)
    return dense_attention(query, key, value, scale=scale)


def paged_attention(
    query: torch.Tensor,
    key_blocks: torch.Tensor,
    value_blocks: torch.Tensor,
    block_table: torch.Tensor,
    seq_len: int,
    *,
    scale: float | None = None,
    backend: str = "auto",
) -> torch.Tensor:
    """Stable paged-attention interface (core/paged_attn.py:147-167).

    backend "auto" runs the fused paged kernel (no materialised gather); "reference"
    runs gather + dense kernels like the reference's own path.  Any other name raises
    ValueError, as in the reference.
    """
    if backend not in {"auto", "reference"}:
        raise ValueError(f"unsupported backend: {backend}")
    if backend == "reference":
        return paged_attention_reference(
            query, key_blocks, value_blocks, block_table, seq_len, scale=scale)
    if seq_len < 0:
        raise ValueError("seq_len must be non-negative")
    _check_blocks(key_blocks, value_blocks)
    if query.ndim != 2:
        raise ValueError("expected query [q_heads, dim], key/value [seq, kv_heads, dim]")
    num_blocks, kv_heads, block_size, head_dim = key_blocks.shape
    if query.shape[-1] != head_dim:
        raise ValueError("query/key head_dim differs")
    if query.shape[0] % kv_heads != 0:
        raise ValueError("q_heads must be a multiple of kv_heads")
    needed_pages = (seq_len + block_size - 1) // block_size
    if block_table.numel() < needed_pages:
        raise ValueError("block_table is shorter than seq_len requires")
    dev = _lib.require_cuda(query, key_blocks, value_blocks)
    table = _table_on(block_table, dev)
    if table.numel() == 0:
        table = torch.zeros(1, dtype=torch.int32, device=dev)
    out = paged_attention_batched(
        query.to(key_blocks.dtype).reshape(1, 1, *query.shape), key_blocks, value_blocks,
        table.reshape(1, -1), None, scale=scale, max_context_len=seq_len)
    if _SYNC_CHECKS:
        _lib.raise_device_errors(dev)
    return out.reshape(query.shape)


_WS_BYTES: dict[tuple, int] = {}  # workspace size per launch shape (a pure function of it)


def paged_attention_batched(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor | None,
    *,
    scale: float | None = None,
    max_context_len: int | None = None,
    out: torch.Tensor | None = None,
    gather=None,
) -> torch.Tensor:
    """Batched paged attention, one launch for all sequences.

    query [B, q_len, q_heads, D].  Query i of sequence b is at position
    context_lens[b] - q_len + i and sees keys up to that position (q_len == 1: plain
    decode; q_len > 1: the causal verify window, whose K/V must already be appended).
    context_lens None means every sequence has max_context_len keys.  max_context_len is
    a host-side upper bound used only to size the launch; it defaults to the block-table
    capacity, so nothing here synchronises with the device.

    gather: an inferd_b200.sharded.PeerGather whose rows are this call's output; the kernel
    also stores them into every rank's gather slot and the step is published (call
    gather.wait() before the next gathered call, and to read the gathered rows).
    """
    if query.ndim != 4:
        raise ValueError("query must be [num_seqs, q_len, q_heads, head_dim]")
    _check_blocks(key_cache, value_cache)
    num_blocks, kv_heads, block_size, head_dim = key_cache.shape
    b, q_len, q_heads, qd = query.shape
    if qd != head_dim:
        raise ValueError("query/key head_dim differs")
    if q_heads % kv_heads != 0:
        raise ValueError("q_heads must be a multiple of kv_heads")
    if query.dtype != key_cache.dtype:
        raise ValueError(f"query dtype {query.dtype} != cache dtype {key_cache.dtype}")
    if block_tables.ndim != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must be [num_seqs, max_pages]")
    if block_tables.dtype not in (torch.int32, torch.int64):
        raise ValueError("block_tables must be int32 or int64")
    if context_lens is not None:
        if context_lens.shape != (b,) or context_lens.dtype != torch.int32:
            raise ValueError("context_lens must be an int32 tensor of shape [num_seqs]")
    dev = _lib.require_cuda(query, key_cache, value_cache, block_tables, context_lens)
    if max_context_len is None:
        max_context_len = block_tables.shape[1] * block_size
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    q = _contig(query)
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor shaped and typed like query")
    else:
        _lib.check_out(out, dev, "paged_attention")
    if b == 0:
        return out
    kc, vc = _contig(key_cache), _contig(value_cache)
    bt = block_tables if block_tables.stride(1) == 1 else block_tables.contiguous()
    lib = _lib.load()
    dev_index = dev.index if dev.index is not None else 0
    ws_key = (b, q_len, q_heads, kv_heads, head_dim, dev_index)
    ws_bytes = _WS_BYTES.get(ws_key)
    if ws_bytes is None:
        ws_bytes = lib.inferd_paged_attention_workspace_bytes(b, q_len, q_heads, kv_heads, head_dim, dev_index)
        if len(_WS_BYTES) > 256:
            _WS_BYTES.clear()
        _WS_BYTES[ws_key] = ws_bytes
    ws = _lib.workspace(dev, ws_bytes)
    if gather is not None:
        if gather.device != dev or gather.rows != b or gather.tail != (q_len, q_heads, head_dim) \
                or gather.dtype != query.dtype:
            raise ValueError("gather was built for other rows, shapes, dtype or device")
        dst, n_dst, offset = gather.begin()
        st = lib.inferd_paged_attention_gather(
            out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
            bt.element_size(), bt.stride(0), _lib.ptr(context_lens), b, q_len, q_heads, kv_heads,
            head_dim, block_size, num_blocks, int(max_context_len), float(scale),
            _lib.dtype_code(query.dtype), ws.data_ptr(), ws.numel(), dst, n_dst, offset,
            _lib.error_word(dev).data_ptr(), _lib.stream_of(dev))
        _lib.check(st, "paged_attention_gather")
        gather.publish()
        return out
    st = lib.inferd_paged_attention(
        out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
        bt.element_size(), bt.stride(0), _lib.ptr(context_lens), b, q_len, q_heads, kv_heads,
        head_dim, block_size, num_blocks, int(max_context_len), float(scale),
        _lib.dtype_code(query.dtype), ws.data_ptr(), ws.numel(),
        _lib.error_word(dev).data_ptr(), _lib.stream_of(dev))
    _lib.check(st, "paged_attention")
    return out


def paged_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    *,
    scale: float | None = None,
    max_context_len: int | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Batched single-query decode: query [B, q_heads, D] -> [B, q_heads, D]."""
    if query.ndim != 3:
        raise ValueError("query must be [num_seqs, q_heads, head_dim]")
    o = None if out is None else out.unsqueeze(1)
    res = paged_attention_batched(
        query.unsqueeze(1), key_cache, value_cache, block_tables, context_lens,
        scale=scale, max_context_len=max_context_len, out=o)
    return res.squeeze(1)


def paged_verify(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    *,
    scale: float | None = None,
    max_context_len: int | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Speculative-decoding verify attention: query [B, k+1, q_heads, D] over the paged
    KV whose last k+1 positions are the draft window (appended before the call);
    causal inside the window.  Replaces the target verify forward's attention of
    core/spec_decode.py:135."""
    return paged_attention_batched(
        query, key_cache, value_cache, block_tables, context_lens,
        scale=scale, max_context_len=max_context_len, out=out)
