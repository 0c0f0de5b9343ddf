"""Paged KV cache: block allocator, page tables and KV pools (drop-in for core/paged_cache.py).

Host bookkeeping (LIFO block allocator, per-sequence page tables, transactional
allocation with rollback) keeps the reference's exact semantics
(core/paged_cache.py:27-92,139-252), because callers and tests depend on the block
reuse order.  Every byte that moves between token tensors and the pools goes through
the sm_100a kernels: `append_tokens` computes the slot of every new token on the host
and issues one reshape_and_cache launch per layer (the reference's Python token x layer
loop of :177-183), and `gather_layer` is one gather launch (:191-205).

Pools are laid out [num_blocks, num_kv_heads, block_size, head_dim] per layer, exactly as
in the reference, so a pool written here can be read by the reference code and vice
versa.  Bookkeeping-only use (create/free sequences, page tables) works on any device;
moving K/V needs the pools on a CUDA device.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from .paged_attn import gather_paged_kv

try:  # page-table loops in C (csrc/host_ops.cpp); the Python loops below are their twins
    from . import _hostops
except ImportError:  # not built: the same bookkeeping in Python
    _hostops = None

_NATIVE = _hostops is not None  # tests switch this off to compare the two


class BlockAllocator:
    """LIFO allocator for fixed-size KV blocks (core/paged_cache.py:27-64).

    The free list starts as [num_blocks-1 .. 0], so a fresh allocator hands out
    0, 1, 2, ...; freed blocks are reused last-freed-first.
    """

    def __init__(self, num_blocks: int) -> None:
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        self._free: list[int] = list(range(num_blocks - 1, -1, -1))
        self._allocated: set[int] = set()

    @property
    def free_count(self) -> int:
        return len(self._free)

    @property
    def allocated_count(self) -> int:
        return len(self._allocated)

    def allocate(self, n: int = 1) -> list[int]:
        if n < 0:
            raise ValueError("cannot allocate a negative number of blocks")
        if n > len(self._free):
            raise MemoryError(f"requested {n} blocks, only {len(self._free)} free")
        blocks = [self._free.pop() for _ in range(n)]
        self._allocated.update(blocks)
        return blocks

    def free(self, blocks: list[int]) -> None:
        seen: set[int] = set()
        for block in blocks:
            if block in seen:
                raise ValueError(f"duplicate block in free request: {block}")
            if block not in self._allocated:
                raise ValueError(f"block is not allocated: {block}")
            seen.add(block)
        for block in blocks:
            self._allocated.remove(block)
            self._free.append(block)


@dataclass
class SequencePageTable:
    """Logical -> physical page mapping of one sequence (core/paged_cache.py:67-92)."""

    seq_id: int
    block_size: int
    blocks: list[int] = field(default_factory=list)
    length: int = 0
    # lowest page index changed since decode_metadata last packed this table (tables only
    # change at their tail: appends, rollbacks and truncations); _CLEAN when unchanged
    dirty_from: int = field(default=0, repr=False, compare=False)

    @property
    def block_count(self) -> int:
        return len(self.blocks)

    @property
    def capacity_tokens(self) -> int:
        return len(self.blocks) * self.block_size

    @property
    def free_slots(self) -> int:
        return self.capacity_tokens - self.length

    def block_for_pos(self, pos: int) -> tuple[int, int]:
        if pos < 0 or pos >= self.length:
            raise IndexError(f"position {pos} outside sequence length {self.length}")
        page_idx, offset = divmod(pos, self.block_size)
        return self.blocks[page_idx], offset

    def slots(self, start: int, n: int) -> list[int]:
        """Pool slots (block * block_size + offset) of positions start .. start+n-1."""
        bs = self.block_size
        return [self.blocks[p // bs] * bs + p % bs for p in range(start, start + n)]


_CLEAN = 1 << 62


class _MetaCache:
    """decode_metadata's state for the last batch it packed: the host copy of the batch's
    page tables [rows, capacity], each row's block count and list identity at that time,
    and (CUDA pools) the device copy the refresh kernel updates in place."""

    __slots__ = ("key", "cap", "host", "nblk", "ids", "master", "device")

    def __init__(self, key, cap, host, nblk, ids, master, device) -> None:
        self.key, self.cap, self.host, self.nblk, self.ids = key, cap, host, nblk, ids
        self.master, self.device = master, device


@dataclass
class AppendPlan:
    """Pages reserved, slots and attention metadata for an append not yet written
    (PagedKVCache.plan_append).  block_tables / context_lens / max_context_len describe the
    sequences as they will be once the append is committed."""

    seq_ids: list[int]
    tokens_per_seq: int
    slots: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    max_context_len: int
    _tables: list = field(repr=False, default_factory=list)
    _reserved: list = field(repr=False, default_factory=list)
    _open: bool = field(repr=False, default=True)


class _PinnedStaging:
    """Two reusable pinned host buffers for the small per-step uploads (slots, block tables).

    Pinning a fresh buffer per call is a host allocation of its own; these grow on demand
    and alternate, and a buffer is rewritten only after the copy that last read it has
    finished (its event)."""

    def __init__(self, dtype: torch.dtype) -> None:
        self.dtype = dtype
        self._bufs: list[torch.Tensor | None] = [None, None]
        self._events: list[torch.cuda.Event | None] = [None, None]
        self._recorded = [False, False]
        self._next = 0
        self.bytes_uploaded = 0

    def upload(self, arr: np.ndarray, device: torch.device) -> torch.Tensor:
        i = self._next
        self._next ^= 1
        n = int(arr.size)
        buf = self._bufs[i]
        if buf is None or buf.numel() < n:
            buf = torch.empty(max(n, 2 * (0 if buf is None else buf.numel()), 1024),
                              dtype=self.dtype, pin_memory=True)
            self._bufs[i] = buf
        elif self._recorded[i]:
            self._events[i].synchronize()
        buf[:n].numpy()[...] = arr.reshape(-1)
        out = buf[:n].to(device, non_blocking=True)
        self.bytes_uploaded += n * buf.element_size()
        if self._events[i] is None:
            self._events[i] = torch.cuda.Event()
        self._events[i].record(torch.cuda.current_stream(device))
        self._recorded[i] = True
        return out


class PagedKVCache:
    """Per-layer K/V block pools plus per-sequence page tables (core/paged_cache.py:95-252)."""

    def __init__(
        self,
        *,
        num_layers: int,
        num_blocks: int,
        block_size: int = 16,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype = torch.bfloat16,
        device: str | torch.device = "cpu",
    ) -> None:
        if num_layers <= 0:
            raise ValueError("num_layers must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        if num_kv_heads <= 0 or head_dim <= 0:
            raise ValueError("num_kv_heads and head_dim must be positive")

        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.allocator = BlockAllocator(num_blocks)
        self.sequences: dict[int, SequencePageTable] = {}
        self._stage_i32 = _PinnedStaging(torch.int32)
        self._stage_i64 = _PinnedStaging(torch.int64)
        # decode_metadata's last packed batch (host and device copies of its page tables)
        self._meta_cache: _MetaCache | None = None

        shape = (num_blocks, num_kv_heads, block_size, head_dim)
        self.key_cache = [
            torch.empty(shape, dtype=dtype, device=self.device) for _ in range(num_layers)
        ]
        self.value_cache = [
            torch.empty(shape, dtype=dtype, device=self.device) for _ in range(num_layers)
        ]

    # ------------------------------------------------------------ bookkeeping
    def create_sequence(self, seq_id: int) -> SequencePageTable:
        if seq_id in self.sequences:
            raise ValueError(f"sequence already exists: {seq_id}")
        table = SequencePageTable(seq_id=seq_id, block_size=self.block_size)
        self.sequences[seq_id] = table
        return table

    def free_sequence(self, seq_id: int) -> None:
        table = self._table(seq_id)
        self.allocator.free(table.blocks)
        del self.sequences[seq_id]

    def truncate_sequence(self, seq_id: int, length: int) -> list[int]:
        """Drop the tokens at positions >= length and free the blocks no longer needed.

        This is the rollback of rejected speculative drafts. The reference crops its
        contiguous cache with copies (core/spec_decode.py:48-57). Here no K/V byte moves:
        the length drops, and whole blocks past the new end go back to the allocator in
        table order. Returns the freed block ids.
        """
        table = self._table(seq_id)
        if length < 0 or length > table.length:
            raise ValueError(f"cannot truncate a sequence of length {table.length} to {length}")
        keep = (length + self.block_size - 1) // self.block_size
        freed = table.blocks[keep:]
        if freed:
            del table.blocks[keep:]
            self.allocator.free(freed)
            table.dirty_from = min(table.dirty_from, keep)
        table.length = length
        return freed

    def truncate_batched(self, seq_ids: list[int], lengths: list[int]) -> list[int]:
        """truncate_sequence for several sequences (the rollback of a batched verify step);
        all lengths are checked before any table changes.  Returns every freed block."""
        if len(seq_ids) != len(lengths):
            raise ValueError("one length per sequence")
        tables = [self._table(s) for s in seq_ids]
        if _NATIVE:
            return _hostops.truncate(tables, [int(n) for n in lengths], self.block_size,
                                     self.allocator._free, self.allocator._allocated)
        for t, n in zip(tables, lengths):
            if n < 0 or n > t.length:
                raise ValueError(f"cannot truncate a sequence of length {t.length} to {n}")
        bs = self.block_size
        freed_all: list[int] = []
        for t, n in zip(tables, lengths):
            keep = (n + bs - 1) // bs
            if keep < len(t.blocks):
                freed = t.blocks[keep:]
                del t.blocks[keep:]
                self.allocator.free(freed)
                freed_all.extend(freed)
                if keep < t.dirty_from:
                    t.dirty_from = keep
            t.length = n
        return freed_all

    def _reserve(self, table: SequencePageTable, n_tokens: int) -> list[int]:
        """Extend a page table to hold n_tokens more tokens (core/paged_cache.py:170-176)."""
        needed_capacity = table.length + n_tokens
        needed_blocks = (needed_capacity + self.block_size - 1) // self.block_size
        extra = needed_blocks - len(table.blocks)
        if extra <= 0:
            return []
        new_blocks = self.allocator.allocate(extra)
        table.dirty_from = min(table.dirty_from, len(table.blocks))
        table.blocks.extend(new_blocks)
        return new_blocks

    def _rollback(self, table: SequencePageTable, new_blocks: list[int]) -> None:
        if new_blocks:
            del table.blocks[-len(new_blocks):]
            self.allocator.free(new_blocks)
            table.dirty_from = min(table.dirty_from, len(table.blocks))

    # ------------------------------------------------------------ K/V movement
    def append_tokens(
        self,
        seq_id: int,
        layer_keys: list[torch.Tensor],
        layer_values: list[torch.Tensor],
    ) -> None:
        """Append one or more logical tokens for every layer (core/paged_cache.py:151-189).

        layer_keys / layer_values hold num_layers tensors [num_tokens, num_kv_heads,
        head_dim].  The page table is extended before any write, so an allocation
        failure (MemoryError) leaves the cache unchanged; any later failure frees the
        blocks this call allocated and re-raises.  The writes are one reshape_and_cache
        launch per layer, bit-exact.
        """
        table = self._table(seq_id)
        self._validate_layers(layer_keys, layer_values)
        n_tokens = int(layer_keys[0].shape[0])
        if n_tokens == 0:
            return
        new_blocks = self._reserve(table, n_tokens)
        try:
            slots = self._slot_tensor(table.slots(table.length, n_tokens))
            for layer in range(self.num_layers):
                self._write(layer, layer_keys[layer], layer_values[layer], slots)
            table.length += n_tokens
        except Exception:
            self._rollback(table, new_blocks)
            raise

    def append_tokens_batched(
        self,
        seq_ids: list[int],
        layer_keys: list[torch.Tensor],
        layer_values: list[torch.Tensor],
    ) -> None:
        """Append tokens_per_seq tokens to each of several sequences in one launch per layer.

        layer_keys[layer]: [len(seq_ids) * tokens_per_seq, num_kv_heads, head_dim], the
        tokens of seq_ids[0] first.  Same all-or-nothing allocation as append_tokens.
        """
        if not seq_ids:
            return
        tables = [self._table(s) for s in seq_ids]
        if len(set(seq_ids)) != len(seq_ids):
            raise ValueError("duplicate sequence in batched append")
        self._validate_layers(layer_keys, layer_values)
        total = int(layer_keys[0].shape[0])
        if total % len(seq_ids) != 0:
            raise ValueError("token count must be a multiple of the number of sequences")
        per = total // len(seq_ids)
        if per == 0:
            return
        reserved: list[tuple[SequencePageTable, list[int]]] = []
        bs = self.block_size
        try:
            slot_list: list[int] = []
            if per == 1:
                # decode: one token per sequence; a new block only when a page fills up
                for t in tables:
                    pos = t.length
                    page = pos // bs
                    if page >= len(t.blocks):
                        reserved.append((t, self._reserve(t, 1)))
                    slot_list.append(t.blocks[page] * bs + pos - page * bs)
            elif per <= bs:
                # a short window (speculative verify): its tokens span at most two pages
                for t in tables:
                    pos = t.length
                    last = pos + per - 1
                    if last // bs >= len(t.blocks):
                        reserved.append((t, self._reserve(t, per)))
                    blocks = t.blocks
                    p0, p1 = pos // bs, last // bs
                    b0, b1 = blocks[p0] * bs - p0 * bs, blocks[p1] * bs - p1 * bs
                    split = (p0 + 1) * bs  # first position on page p1 when p1 > p0
                    slot_list.extend([(b0 if q < split else b1) + q for q in range(pos, pos + per)])
            else:
                for t in tables:
                    reserved.append((t, self._reserve(t, per)))
                for t in tables:
                    slot_list.extend(t.slots(t.length, per))
            slots = self._slot_tensor(slot_list)
            for layer in range(self.num_layers):
                self._write(layer, layer_keys[layer], layer_values[layer], slots)
            for t in tables:
                t.length += per
        except Exception:
            for t, nb in reversed(reserved):
                self._rollback(t, nb)
            raise

    # ------------------------------------------------------------ planned appends
    def plan_append(self, seq_ids: list[int], tokens_per_seq: int) -> AppendPlan:
        """Reserve the pages for tokens_per_seq new tokens of every sequence, upload their
        slots and build the attention metadata of the state after the append -- everything
        but the K/V write, which commit_append does once the tokens exist.

        A decode engine plans step N + 1 while step N runs on the GPU: the pages and slots
        depend only on the lengths.  Until the plan is committed or aborted, these
        sequences must not change otherwise.  Reservation is all-or-nothing (MemoryError
        leaves the cache unchanged), as in append_tokens."""
        if len(set(seq_ids)) != len(seq_ids):
            raise ValueError("duplicate sequence in batched append")
        per = int(tokens_per_seq)
        if per <= 0:
            raise ValueError("tokens_per_seq must be positive")
        tables = [self._table(s) for s in seq_ids]
        bs = self.block_size
        if _NATIVE:
            slots_np = np.empty(len(tables) * per, dtype=np.int64)
            reserved, failed = _hostops.plan_slots(tables, per, bs, self.allocator._free,
                                                   self.allocator._allocated, slots_np)
            if failed >= 0:
                t = tables[failed]
                need = (t.length + per + bs - 1) // bs - len(t.blocks)
                msg = f"requested {need} blocks, only {self.allocator.free_count} free"
                for tt, nb in reversed(reserved):
                    self._rollback(tt, nb)
                raise MemoryError(msg)
            slots = self._slot_tensor(slots_np)
            bt, cl, mx = self._metadata(tables, seq_ids, per, None, None)
            return AppendPlan(list(seq_ids), per, slots, bt, cl, mx, tables, reserved)
        reserved: list[tuple[SequencePageTable, list[int]]] = []
        slot_list: list[int] = []
        try:
            for t in tables:
                pos = t.length
                last = pos + per - 1
                if last // bs >= len(t.blocks):
                    reserved.append((t, self._reserve(t, per)))
                blocks = t.blocks
                if per == 1:
                    page = pos // bs
                    slot_list.append(blocks[page] * bs + pos - page * bs)
                elif per <= bs:  # the window spans at most two pages
                    p0, p1 = pos // bs, last // bs
                    b0, b1 = blocks[p0] * bs - p0 * bs, blocks[p1] * bs - p1 * bs
                    split = (p0 + 1) * bs
                    slot_list.extend([(b0 if q < split else b1) + q for q in range(pos, pos + per)])
                else:
                    slot_list.extend([blocks[q // bs] * bs + q % bs for q in range(pos, pos + per)])
        except Exception:
            for t, nb in reversed(reserved):
                self._rollback(t, nb)
            raise
        slots = self._slot_tensor(slot_list)
        bt, cl, mx = self.decode_metadata(seq_ids, extra_tokens=per)
        return AppendPlan(list(seq_ids), per, slots, bt, cl, mx, tables, reserved)

    def commit_append(self, plan: AppendPlan, layer_keys: list[torch.Tensor],
                      layer_values: list[torch.Tensor]) -> None:
        """Write the planned tokens (layer_keys[layer]: [len(seq_ids) * tokens_per_seq,
        num_kv_heads, head_dim], seq_ids[0]'s tokens first) and advance the lengths.  On a
        failure the plan's pages are released (abort_append) and the error re-raised."""
        if not plan._open:
            raise ValueError("this plan was already committed or aborted")
        try:
            self._validate_layers(layer_keys, layer_values)
            if int(layer_keys[0].shape[0]) != len(plan.seq_ids) * plan.tokens_per_seq:
                raise ValueError("token count differs from the plan's")
            for layer in range(self.num_layers):
                self._write(layer, layer_keys[layer], layer_values[layer], plan.slots)
        except Exception:
            self.abort_append(plan)
            raise
        per = plan.tokens_per_seq
        if _NATIVE:
            _hostops.advance(plan._tables, per)
        else:
            for t in plan._tables:
                t.length += per
        plan._open = False

    def abort_append(self, plan: AppendPlan) -> None:
        """Release the pages an uncommitted plan reserved."""
        if not plan._open:
            return
        for t, nb in reversed(plan._reserved):
            self._rollback(t, nb)
        plan._open = False

    def _slot_tensor(self, slots: list[int]) -> torch.Tensor:
        arr = np.asarray(slots, dtype=np.int64)
        if self.device.type != "cuda":
            return torch.from_numpy(arr)
        return self._stage_i64.upload(arr, self.device)

    def _write(self, layer: int, keys: torch.Tensor, values: torch.Tensor,
               slots: torch.Tensor) -> None:
        kc, vc = self.key_cache[layer], self.value_cache[layer]
        dev = _lib.require_cuda(kc, vc, keys, values)
        if keys.dtype != self.dtype or values.dtype != self.dtype:
            raise ValueError(f"tensor dtype must be the cache dtype {self.dtype}")
        if keys.stride(2) != 1:
            keys = keys.contiguous()
        if values.stride(2) != 1:
            values = values.contiguous()
        lib = _lib.load()
        st = lib.inferd_reshape_and_cache(
            keys.data_ptr(), values.data_ptr(), keys.stride(0), keys.stride(1),
            values.stride(0), values.stride(1), kc.data_ptr(), vc.data_ptr(), slots.data_ptr(),
            slots.numel(), self.num_kv_heads, self.head_dim, self.block_size, self.num_blocks,
            _lib.dtype_code(self.dtype), _lib.error_word(dev).data_ptr(), _lib.stream_of(dev))
        _lib.check(st, "reshape_and_cache")

    def gather_layer(self, seq_id: int, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Contiguous K/V [seq_len, num_kv_heads, head_dim] of one layer (one gather launch)."""
        table = self._table(seq_id)
        self._check_layer(layer)
        if table.length == 0:
            empty = torch.empty((0, self.num_kv_heads, self.head_dim), dtype=self.dtype,
                                device=self.device)
            return empty, empty.clone()
        return gather_paged_kv(self.key_cache[layer], self.value_cache[layer],
                               self.block_table(seq_id), table.length)

    # ------------------------------------------------------------ tables
    def block_table(self, seq_id: int, *, device: str | torch.device | None = None) -> torch.Tensor:
        table = self._table(seq_id)
        out_device = self.device if device is None else device
        return torch.tensor(table.blocks, dtype=torch.int64, device=out_device)

    def decode_metadata(
        self, seq_ids: list[int], *, extra_tokens: int = 0, pad_pages: int | None = None,
        device: str | torch.device | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor, int]:
        """Packed batch metadata for the batched attention kernels.

        Returns (block_tables int32 [B, P], context_lens int32 [B], max_context_len), new
        tensors on every call, P the widest table (or pad_pages), rows zero-padded.
        extra_tokens is added to every length (for a verify window appended after this call).

        For a batch packed by the previous call (same seq_ids, same device) only the page-
        table entries changed since then travel: the tables are kept on the device and one
        refresh launch applies the (column, block) changes and writes the packed table, so a
        decode step uploads the lengths plus about one entry per block_size steps per
        sequence instead of the whole [B, P] table (core/paged_cache.py:207-213 builds a new
        tensor per sequence per call).  Page tables must change through this class (appends,
        rollbacks, truncations), which records the lowest changed index; a table whose list
        object was replaced from outside is recognised by the list's identity and re-sent
        whole.
        """
        return self._metadata([self._table(s) for s in seq_ids], seq_ids, extra_tokens, pad_pages, device)

    def _metadata(self, tables, seq_ids, extra_tokens, pad_pages, device):
        b = len(tables)
        if _NATIVE:
            lens_np = np.empty(b, dtype=np.int32)
            nblk, width, mx = _hostops.scan(tables, extra_tokens, lens_np)
            lens = lens_np
        else:
            lens = [t.length + extra_tokens for t in tables]
            nblk = [len(t.blocks) for t in tables]
            width = max(nblk + [1])
            mx = max(lens + [0])
        if pad_pages is not None:
            if pad_pages < width:
                raise ValueError("pad_pages is narrower than the widest page table")
            width = pad_pages
        dev = self.device if device is None else torch.device(device)
        key = tuple(seq_ids)
        c = self._meta_cache
        dense = c is None or c.key != key or width > c.cap or c.device != dev
        ids = [id(t.blocks) for t in tables] if (dense or not _NATIVE) else None
        if dense:
            cap = (width + 63) // 64 * 64  # room to grow without a rebuild
            host = np.zeros((b, cap), dtype=np.int32)
            for i, t in enumerate(tables):
                host[i, :nblk[i]] = t.blocks
            master = torch.empty((b, cap), dtype=torch.int32, device=dev) if dev.type == "cuda" else None
            flat = np.concatenate([np.asarray(lens, dtype=np.int32), host.reshape(-1)])
            for t in tables:
                t.dirty_from = _CLEAN
        else:
            cap, host, master = c.cap, c.host, c.master
            keep_host = master is None  # a CUDA cache's tables live on the device after the rebuild
        if not dense and _NATIVE:
            counts = np.zeros(b + 1, dtype=np.int32)
            pair_bytes, ids, _ = _hostops.pack_changes(tables, c.ids, c.nblk, _CLEAN, counts[1:])
            pairs_np = np.frombuffer(pair_bytes, dtype=np.int32)
            row_ptr = np.cumsum(counts, dtype=np.int32)
            if keep_host and pairs_np.size:
                rows = np.repeat(np.arange(b), counts[1:])
                host[rows, pairs_np[0::2]] = pairs_np[1::2]
            flat = np.concatenate([np.asarray(lens, dtype=np.int32), row_ptr, pairs_np])
        elif not dense:
            # rows to send: those changed through this class since the last call, and those
            # whose list object was replaced from outside (whole row)
            starts = {i: t.dirty_from for i, t in enumerate(tables) if t.dirty_from != _CLEAN}
            if ids != c.ids:
                for i in range(b):
                    if ids[i] != c.ids[i]:
                        starts[i] = 0
            counts = np.zeros(b + 1, dtype=np.int32)
            pairs: list[int] = []
            for i in sorted(starts):
                start, old, n = starts[i], c.nblk[i], nblk[i]
                blocks = tables[i].blocks
                for col in range(start, n):
                    pairs.append(col)
                    pairs.append(blocks[col])
                for col in range(max(n, start), old):
                    pairs.append(col)
                    pairs.append(0)
                if keep_host:
                    if start < n:
                        host[i, start:n] = blocks[start:n]
                    if n < old:
                        host[i, n:old] = 0
                counts[i + 1] = len(pairs) // 2
                tables[i].dirty_from = _CLEAN
            row_ptr = np.maximum.accumulate(counts)  # entries of rows before each row
            flat = np.concatenate([np.asarray(lens, dtype=np.int32), row_ptr,
                                   np.asarray(pairs, dtype=np.int32)])
        self._meta_cache = _MetaCache(key, cap, host, nblk, ids, master, dev)
        if dev.type != "cuda":
            return torch.from_numpy(host[:, :width].copy()), torch.as_tensor(np.asarray(lens, dtype=np.int32)), mx
        packed = self._stage_i32.upload(flat, dev)
        cl = packed[:b]
        bt = torch.empty((b, width), dtype=torch.int32, device=dev)
        if b:
            if dense:
                rp, upd = None, packed[b:]
            else:
                rp, upd = packed[b:2 * b + 1], packed[2 * b + 1:]
            upd_ptr = upd.data_ptr() if upd.numel() else packed.data_ptr()
            lib = _lib.load()
            st = lib.inferd_block_tables_refresh(master.data_ptr(), cap, _lib.ptr(rp), upd_ptr,
                                                 1 if dense else 0, b, width, bt.data_ptr(),
                                                 _lib.stream_of(dev))
            _lib.check(st, "block_tables_refresh")
        return bt, cl, mx

    def uploaded_bytes(self) -> int:
        """Host-to-device bytes this cache has copied so far (slot mappings and decode
        metadata), for end-to-end accounting."""
        return self._stage_i32.bytes_uploaded + self._stage_i64.bytes_uploaded

    def sequence_length(self, seq_id: int) -> int:
        return self._table(seq_id).length

    def _table(self, seq_id: int) -> SequencePageTable:
        table = self.sequences.get(seq_id)
        if table is None:
            raise KeyError(f"no sequence {seq_id!r} in this cache")
        return table

    def _check_layer(self, layer: int) -> None:
        if not 0 <= layer < self.num_layers:
            raise IndexError(f"layer index {layer} is not below num_layers={self.num_layers}")

    def _validate_layers(self, layer_keys: list[torch.Tensor],
                         layer_values: list[torch.Tensor]) -> None:
        """One [tokens, kv_heads, head_dim] tensor per layer for keys and for values, all of
        one shape and on the cache's device; ValueError otherwise (the reference's
        exception type for these checks, core/paged_cache.py:225-242)."""
        n_layers = self.num_layers
        if (len(layer_keys), len(layer_values)) != (n_layers, n_layers):
            raise ValueError(f"need {n_layers} key and {n_layers} value tensors, got "
                             f"{len(layer_keys)} and {len(layer_values)}")
        want_tail = (self.num_kv_heads, self.head_dim)
        shape = None
        for t in (*layer_keys, *layer_values):
            if t.ndim != 3 or tuple(t.shape[1:]) != want_tail:
                raise ValueError(f"token tensors are [tokens, {want_tail[0]}, {want_tail[1]}], "
                                 f"got {tuple(t.shape)}")
            if shape is None:
                shape = t.shape
            elif t.shape != shape:
                raise ValueError(f"token tensors differ in shape: {tuple(shape)} and {tuple(t.shape)}")
            if t.device != self.device:
                raise ValueError(f"token tensor on {t.device}, cache on {self.device}")

    def assert_consistent(self) -> None:
        """Every block is owned by at most one sequence, the owned blocks are exactly the
        allocator's allocated set, and free + allocated partition the pool."""
        owners: dict[int, int] = {}
        for seq_id, table in self.sequences.items():
            for blk in table.blocks:
                if not 0 <= blk < self.num_blocks:
                    raise AssertionError(f"sequence {seq_id} holds block {blk}, outside the pool")
                if blk in owners:
                    raise AssertionError(f"block {blk} held by sequences {owners[blk]} and {seq_id}")
                owners[blk] = seq_id
        allocated = self.allocator._allocated
        if owners.keys() != allocated:
            raise AssertionError(f"{len(owners)} blocks in page tables, "
                                 f"{len(allocated)} marked allocated")
        free = self.allocator._free
        if len(free) + len(allocated) != self.num_blocks or allocated.intersection(free):
            raise AssertionError("free and allocated blocks do not partition the pool")


def _full_attention_layers(kv) -> list[int]:
    """Indices of the layers whose K/V a Qwen3.5 hybrid cache holds: its own
    transformer_layers when it lists them, else every 4-D key tensor with tokens in it."""
    listed = list(getattr(kv, "transformer_layers", None) or [])
    if listed:
        return listed
    return [i for i, k in enumerate(kv.key_cache)
            if isinstance(k, torch.Tensor) and k.ndim == 4 and k.shape[2] > 0]


def _clone_all(states):
    """Fresh copies of a per-layer state list (None where a layer has no state)."""
    return [None if t is None else t.clone() for t in states]


@dataclass
class PagedHybridCache:
    """Paged form of Qwen3.5's hybrid cache (the API of core/paged_cache.py:255-363).

    The full-attention layers' K/V go into one PagedKVCache (`attention`, one pool layer
    per full-attention layer, `layer_to_cache` mapping model layer -> pool layer) through
    the reshape_and_cache kernel; the linear-attention conv / recurrent states have a fixed
    size per sequence, so they are kept as copies.  Batch-1 caches only.
    """

    attention: PagedKVCache
    layer_to_cache: dict[int, int]
    conv_states: list[torch.Tensor | None]
    recurrent_states: list[torch.Tensor | None]
    layer_types: list[str] | None
    transformer_layers: list[int]
    seq_id: int = 0

    @classmethod
    def from_qwen_cache(cls, kv, *, block_size: int = 16, seq_id: int = 0) -> "PagedHybridCache":
        """Page a batch-1 HF Qwen3.5 cache: every full-attention layer's [1, heads, seq,
        dim] K/V is appended to one sequence of a pool sized to hold it exactly."""
        layers = _full_attention_layers(kv)
        if not layers:
            raise ValueError("the cache holds no full-attention K/V")
        pairs = []
        for layer in layers:
            k, v = kv.key_cache[layer], kv.value_cache[layer]
            if k is None or v is None:
                raise ValueError(f"layer {layer} is listed as full attention but has no K/V")
            if k.ndim != 4 or k.shape != v.shape:
                raise ValueError(f"layer {layer}: K {tuple(k.shape)} and V {tuple(v.shape)} "
                                 "are not one [batch, heads, seq, dim] shape")
            pairs.append((k, v))
        batch, heads, tokens, dim = pairs[0][0].shape
        if batch != 1:
            raise ValueError(f"only batch-1 caches can be paged (batch is {batch})")
        for layer, (k, _) in zip(layers, pairs):
            if tuple(k.shape) != (1, heads, tokens, dim):
                raise ValueError(f"layer {layer} K/V is {tuple(k.shape)}, layer {layers[0]}'s "
                                 f"is {(1, heads, tokens, dim)}")
        first = pairs[0][0]
        pool = PagedKVCache(num_layers=len(layers),
                            num_blocks=max(1, -(-tokens // block_size)), block_size=block_size,
                            num_kv_heads=heads, head_dim=dim, dtype=first.dtype,
                            device=first.device)
        pool.create_sequence(seq_id)
        # [1, heads, seq, dim] -> strided [seq, heads, dim] views; the append kernel reads
        # token and head strides, so nothing is transposed in memory first
        pool.append_tokens(seq_id, [k[0].transpose(0, 1) for k, _ in pairs],
                           [v[0].transpose(0, 1) for _, v in pairs])
        types = getattr(kv, "layer_types", None)
        return cls(attention=pool, layer_to_cache={layer: i for i, layer in enumerate(layers)},
                   conv_states=_clone_all(kv.conv_states),
                   recurrent_states=_clone_all(kv.recurrent_states),
                   layer_types=list(types) if types else None, transformer_layers=layers,
                   seq_id=seq_id)

    def to_qwen_cache_like(self, template):
        """A shallow copy of `template` (same class, same other attributes) whose K/V come
        back out of the pool as contiguous [1, heads, seq, dim] tensors, whose state lists
        are fresh copies, and whose layer lists are its own."""
        out = copy.copy(template)
        for name in ("layer_types", "transformer_layers"):
            if hasattr(template, name):
                setattr(out, name, list(getattr(template, name)))
        out.conv_states = _clone_all(self.conv_states)
        out.recurrent_states = _clone_all(self.recurrent_states)
        n = len(template.key_cache)
        out.key_cache, out.value_cache = [None] * n, [None] * len(template.value_cache)
        for layer, pool_layer in self.layer_to_cache.items():
            k, v = self.attention.gather_layer(self.seq_id, pool_layer)
            out.key_cache[layer] = k.permute(1, 0, 2).contiguous()[None]
            out.value_cache[layer] = v.permute(1, 0, 2).contiguous()[None]
        return out
