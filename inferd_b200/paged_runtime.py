"""Persistent paged runtime cache for Qwen3.5's hybrid layout: an HF `Cache` whose
full-attention K/V live in a PagedKVCache pool across steps and sequences.

The reference's batched decode (core/scheduler.py:142-159 decode_batch) re-pads and
clones every sequence's whole KV history every step (core/batched_cache.py:51-104
stack_caches / split_caches), and its paged cache is a one-shot round trip
(core/paged_cache.py:255-363).  Here the cache persists:

* full-attention layers: `update()` writes the step's new K/V straight into the pool with
  the reshape_and_cache kernel, and the installed attention hook
  (inferd_b200.paged_attn_interface) attends over the pool with per-row context lengths
  -- no K/V byte moves between steps, and rows of different lengths need no padding;
* linear-attention (GatedDeltaNet) layers: their fixed-size conv / recurrent states live
  in slot-indexed pools; the active rows are always slots [0, n), handed to HF's layer
  objects as views, so HF's in-place state updates land in the pools.

    cache = PagedRuntimeCache(model.config, num_blocks=..., max_seqs=...)
    paged_attn_interface.install()               # the model runs with attn_implementation="eager"
    cache.begin_prefill(seq_id)                  # one new sequence, alone
    logits = model(prompt_ids, past_key_values=cache, use_cache=True).logits
    cache.end_prefill()
    ids = cache.rows                             # batch order of every later step
    logits = model(next_tokens[len(ids), 1], past_key_values=cache, use_cache=True,
                   position_ids=cache.position_ids()).logits
    cache.release(seq_id)                        # frees its pages, moves one state row

Speculative verify (core/spec_decode.py:117-170): `snap = cache.snapshot()`, one forward of
the gamma + 1 window (causal inside it), then `cache.restore(snap)` and a forward of the
emitted tokens -- the K/V rollback is a page-table truncation, not a cache copy.

This is the "persistent paged runtime cache" the reference plans as its next step
(core/batched_cache.py, core/scheduler.py:142-159); the page-table semantics are
PagedKVCache's (core/paged_cache.py:95-252).
"""

from __future__ import annotations

import torch
from transformers import DynamicCache

from . import paged_attn_interface
from .paged_attn import paged_attention_batched
from .paged_cache import PagedKVCache


class PagedRuntimeCache(DynamicCache):
    """HF cache backed by a paged K/V pool and slot-indexed linear-attention states."""

    def __init__(self, config, *, num_blocks: int, max_seqs: int, block_size: int = 16,
                 dtype: torch.dtype = torch.bfloat16, device: str | torch.device = "cuda") -> None:
        super().__init__(config=config)
        text = config.get_text_config() if hasattr(config, "get_text_config") else config
        types = list(text.layer_types)
        self.attn_layers = [i for i, t in enumerate(types) if t == "full_attention"]
        self.linear_layers = [i for i, t in enumerate(types) if t == "linear_attention"]
        if not self.attn_layers:
            raise ValueError("the model has no full-attention layers")
        self._pool_index = {layer: j for j, layer in enumerate(self.attn_layers)}
        self.pool = PagedKVCache(num_layers=len(self.attn_layers), num_blocks=num_blocks,
                                 block_size=block_size, num_kv_heads=text.num_key_value_heads,
                                 head_dim=text.head_dim, dtype=dtype, device=device)
        self.max_seqs = int(max_seqs)
        self.rows: list[int] = []          # active sequences in slot (= batch row) order
        self._conv: dict[int, torch.Tensor] = {}   # layer -> [max_seqs, ...] state pool
        self._rec: dict[int, torch.Tensor] = {}
        self._batch: list[int] = []        # rows of the forward in progress
        self._prefill: int | None = None
        self._step: dict | None = None     # per-forward: q_len, slots, attention metadata

    # ------------------------------------------------------------ sequences
    def begin_prefill(self, seq_id: int) -> None:
        """Next forward is the prompt of a new sequence, as a batch of one."""
        if self._prefill is not None:
            raise RuntimeError("a prefill is already open")
        if len(self.rows) >= self.max_seqs:
            raise MemoryError("all state slots are in use")
        self.pool.create_sequence(seq_id)
        self._prefill = seq_id
        self._batch = [seq_id]
        for layer in self.linear_layers:  # fresh states, lazily created by HF at batch 1
            lyr = self.layers[layer]
            lyr.conv_states = None
            lyr.recurrent_states = None
            lyr.is_conv_states_initialized = False
            lyr.is_recurrent_states_initialized = False
            lyr.has_previous_state = False

    def end_prefill(self) -> None:
        """Store the new sequence's linear states in the next slot; it joins the batch."""
        seq = self._prefill
        if seq is None:
            raise RuntimeError("no prefill is open")
        slot = len(self.rows)
        for layer in self.linear_layers:
            lyr = self.layers[layer]
            for pools, state in ((self._conv, lyr.conv_states), (self._rec, lyr.recurrent_states)):
                if state is None:
                    raise RuntimeError(f"layer {layer} produced no state during the prefill")
                if layer not in pools:
                    pools[layer] = torch.zeros((self.max_seqs,) + tuple(state.shape[1:]),
                                               dtype=state.dtype, device=state.device)
                pools[layer][slot].copy_(state[0])
        self.rows.append(seq)
        self._prefill = None
        self._use_rows()

    def release(self, seq_id: int) -> None:
        """Drop a finished sequence: its pages go back to the allocator and the last row's
        linear states move into its slot, so the active rows stay contiguous."""
        slot = self.rows.index(seq_id)
        last = len(self.rows) - 1
        if slot != last:
            for pools in (self._conv, self._rec):
                for state in pools.values():
                    state[slot].copy_(state[last])
            self.rows[slot] = self.rows[last]
        self.rows.pop()
        self.pool.free_sequence(seq_id)
        self._use_rows()

    def _use_rows(self) -> None:
        """Point HF's linear layers at the active slots and batch the active rows."""
        n = len(self.rows)
        self._batch = list(self.rows)
        for layer in self.linear_layers:
            lyr = self.layers[layer]
            if layer not in self._conv:
                continue
            lyr.conv_states = self._conv[layer][:n]
            lyr.recurrent_states = self._rec[layer][:n]
            lyr.is_conv_states_initialized = True
            lyr.is_recurrent_states_initialized = True
            lyr.has_previous_state = n > 0
            lyr.max_batch_size = n
            lyr.dtype, lyr.device = self._conv[layer].dtype, self._conv[layer].device
            lyr.conv_kernel_size = self._conv[layer].shape[-1]

    # ------------------------------------------------------------ speculative rollback
    def snapshot(self) -> dict:
        """Lengths and linear-attention states of the active rows before a speculative
        verify forward (core/spec_decode.py:118-119 _snapshot_linear).  The K/V need no
        copy: rollback only shortens the page tables."""
        n = len(self.rows)
        return {"rows": list(self.rows),
                "lengths": [self.pool.sequence_length(s) for s in self.rows],
                "conv": {k: v[:n].clone() for k, v in self._conv.items()},
                "rec": {k: v[:n].clone() for k, v in self._rec.items()}}

    def restore(self, snap: dict, lengths: list[int] | None = None) -> None:
        """Roll the active rows back to `snap` (core/spec_decode.py:48-57 _restore_to, which
        copies the whole cache): linear states are copied back and each row's K/V is cut to
        `lengths` (default: the snapshot's) by truncating its page table -- the tail blocks
        return to the allocator and no K/V byte moves."""
        if snap["rows"] != self.rows:
            raise ValueError("the active rows changed since the snapshot")
        n = len(self.rows)
        for k, v in snap["conv"].items():
            self._conv[k][:n].copy_(v)
        for k, v in snap["rec"].items():
            self._rec[k][:n].copy_(v)
        self.pool.truncate_batched(self.rows, lengths if lengths is not None else snap["lengths"])
        self._use_rows()

    def position_ids(self) -> torch.Tensor:
        """[rows, 1] positions of the next token of every active row."""
        lens = [self.pool.sequence_length(s) for s in self.rows]
        return torch.tensor(lens, dtype=torch.long, device=self.pool.device).view(-1, 1)

    # ------------------------------------------------------------ HF cache interface
    def get_seq_length(self, layer_idx: int = 0) -> int:
        lens = [self.pool.sequence_length(s) for s in self._batch]
        return max(lens) if lens else 0

    def get_mask_sizes(self, cache_position, layer_idx: int = 0):
        # the paged hook uses per-row context lengths, not HF's mask; sizes stay consistent
        q = cache_position.shape[0] if hasattr(cache_position, "shape") else int(cache_position)
        return self.get_seq_length() + q, 0

    def update(self, key_states, value_states, layer_idx: int, cache_kwargs=None):
        """Append the step's K/V [rows, kv_heads, q_len, head_dim] of one full-attention
        layer to the pool; returns them unchanged (the paged hook reads the pool)."""
        j = self._pool_index.get(layer_idx)
        if j is None:
            return super().update(key_states, value_states, layer_idx, cache_kwargs)
        b, _, q_len, _ = key_states.shape
        if b != len(self._batch):
            raise ValueError(f"batch of {b} rows for {len(self._batch)} cached sequences")
        if self._step is None or j == 0:
            self._begin_step(q_len)
        paged_attn_interface._runtime = self  # the hook attends over this cache's pool
        step = self._step
        k = key_states.transpose(1, 2).reshape(b * q_len, key_states.shape[1], -1)
        v = value_states.transpose(1, 2).reshape(b * q_len, value_states.shape[1], -1)
        self.pool._write(j, k.to(self.pool.dtype), v.to(self.pool.dtype), step["slots"])
        if j == len(self.attn_layers) - 1:  # every layer written: the rows are longer now
            for t in step["tables"]:
                t.length += q_len
        return key_states, value_states

    def _begin_step(self, q_len: int) -> None:
        tables = [self.pool._table(s) for s in self._batch]
        reserved = []
        try:
            for t in tables:
                reserved.append((t, self.pool._reserve(t, q_len)))
        except Exception:
            for t, nb in reversed(reserved):
                self.pool._rollback(t, nb)
            raise
        slots = []
        for t in tables:
            slots.extend(t.slots(t.length, q_len))
        bt, cl, mx = self.pool.decode_metadata(self._batch, extra_tokens=q_len)
        self._step = {"q_len": q_len, "slots": self.pool._slot_tensor(slots), "tables": tables,
                      "bt": bt, "cl": cl, "max": mx}

    def attend(self, layer_idx: int, query: torch.Tensor, scaling: float) -> torch.Tensor:
        """Causal attention of query [rows, heads, q_len, dim] over the pool (the step's
        tokens included) -> [rows, q_len, heads, dim]."""
        j = self._pool_index[layer_idx]
        step = self._step
        q = query.transpose(1, 2).to(self.pool.dtype).contiguous()
        out = paged_attention_batched(q, self.pool.key_cache[j], self.pool.value_cache[j],
                                      step["bt"], step["cl"], scale=scaling,
                                      max_context_len=step["max"])
        if j == len(self.attn_layers) - 1:
            self._step = None
        return out.to(query.dtype)

    def owns_layer(self, layer_idx) -> bool:
        return self._step is not None and layer_idx in self._pool_index
