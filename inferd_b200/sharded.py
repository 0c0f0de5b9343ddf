"""Sequence sharding across the GPUs of one node.

Decode attention needs no cross-GPU exchange: each sequence's KV pages live in one GPU's
pool, so every rank owns a slice of the batch (its own PagedKVCache, block tables and
kernels) and the only collective is gathering the per-rank attention outputs, in global
sequence order, after each step.  The reference runs one process on one GPU
(core/model_runner.py); this module is what spreads its batch over N of them.

    lo, hi = shard_range(num_seqs, world, rank)              # contiguous, equal counts
    owners = assign_by_tokens(context_lens, world)           # balanced KV bytes, ragged counts
    full = gather_outputs(local_out, counts, group=None)     # all ranks get [sum(counts), ...]

    g = OutputGather((rows, q_heads, dim), dtype, device, counts)   # a decode loop's gather
    out = g.local()          # this step's output buffer: the attention writes it
    g.start()                # all-gather it on the collective's own stream, asynchronously
    full = g.result()        # the step's gathered outputs (the current stream waits for them)

`gather_outputs` uses NCCL's all-gather into one tensor when the process group is NCCL and
every shard has the same size, else a padded all-gather (also what gloo ranks on CPU use).
`OutputGather` preallocates everything and overlaps step N's all-gather with step N + 1's
compute: local outputs alternate between two buffers, so the collective reading step N's
buffer never races the kernels writing step N + 1's.  With max_ctas=k it runs NCCL on at
most k CTAs in a process group of its own and leaves k SMs out of the persistent attention
grid (paged_attn.reserve_sms), so the overlapped all-gather never delays an attention CTA.
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def shard_range(num_items: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) slice of num_items for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_items < 0:
        raise ValueError("num_items must be >= 0")
    base, extra = divmod(num_items, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def assign_by_tokens(context_lens, world: int) -> list[list[int]]:
    """Sequence indices per rank so that each rank's total context (its KV bytes, the
    attention kernel's work) is balanced: longest sequence first onto the least-loaded rank.
    Each rank's list is sorted, so its outputs keep the global order within the shard."""
    if world <= 0:
        raise ValueError("world must be >= 1")
    lens = [int(v) for v in context_lens]
    if any(v < 0 for v in lens):
        raise ValueError("context lengths must be >= 0")
    heap = [(0, r) for r in range(world)]
    owners: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda j: (-lens[j], j)):
        load, r = heapq.heappop(heap)
        owners[r].append(i)
        heapq.heappush(heap, (load + lens[i], r))
    return [sorted(o) for o in owners]


def gather_outputs(local: torch.Tensor, counts: list[int] | None = None, *, group=None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather each rank's [count_r, ...] output along dim 0 into [sum(counts), ...], rank
    order.  counts=None means every rank holds local.shape[0] rows."""
    world = dist.get_world_size(group)
    if counts is None:
        counts = [local.shape[0]] * world
    if len(counts) != world:
        raise ValueError(f"{len(counts)} counts for a world of {world}")
    if local.shape[0] != counts[dist.get_rank(group)]:
        raise ValueError("local rows differ from this rank's count")
    total = sum(counts)
    tail = tuple(local.shape[1:])
    if out is None:
        out = torch.empty((total,) + tail, dtype=local.dtype, device=local.device)
    elif tuple(out.shape) != (total,) + tail:
        raise ValueError("out has the wrong shape")
    local = local.contiguous()
    equal = all(c == counts[0] for c in counts)
    if equal and dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
        return out
    width = max(counts)
    padded = torch.zeros((width,) + tail, dtype=local.dtype, device=local.device)
    padded[:local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    row = 0
    for c, part in zip(counts, parts):
        out[row:row + c] = part[:c]
        row += c
    return out


class OutputGather:
    """Double-buffered, asynchronous all-gather of per-step outputs (decode outputs of the
    sequences each rank owns, gathered in rank order).

    Every buffer is allocated once: two local output buffers [width, *tail] (width = the
    largest count), two gathered buffers [world * width, *tail] and, for ragged counts, the
    row index that compacts a gathered buffer to [sum(counts), *tail].  start() issues the
    collective with async_op=True, so it runs on the process group's own stream after the
    work already queued on the current stream, while the current stream goes on with the
    next step.  A local buffer is handed out again only after the collective that read it
    two steps earlier has completed on the current stream (Work.wait orders the streams;
    the host does not block).
    """

    def __init__(self, tail: tuple[int, ...], dtype: torch.dtype, device: torch.device,
                 counts: list[int] | None = None, *, group=None, max_ctas: int = 0) -> None:
        self._own_group = None
        self._prev_reserve = None
        if max_ctas and dist.get_backend(group) == "nccl":
            # NCCL on at most max_ctas CTAs, in a group of its own, and as many SMs left
            # out of the persistent attention grid: the overlapped all-gather then holds
            # no SM that a statically assigned attention CTA waits for
            from .paged_attn import reserve_sms

            opts = dist.ProcessGroupNCCL.Options()
            opts.config.max_ctas = int(max_ctas)
            opts.config.min_ctas = 1
            ranks = dist.get_process_group_ranks(group) if group is not None else None
            group = self._own_group = dist.new_group(ranks, backend="nccl", pg_options=opts)
            self._prev_reserve = reserve_sms(int(max_ctas))
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if counts is None:
            raise ValueError("counts: rows per rank (a list of world integers)")
        if len(counts) != self.world or any(c < 0 for c in counts):
            raise ValueError(f"{len(counts)} counts for a world of {self.world}")
        self.counts = [int(c) for c in counts]
        self.width = max(max(self.counts), 1)
        self.tail = tuple(int(t) for t in tail)
        self.ragged = any(c != self.width for c in self.counts)
        self._nccl = dist.get_backend(group) == "nccl"
        shape_l = (self.width,) + self.tail
        shape_g = (self.world * self.width,) + self.tail
        self._local = [torch.zeros(shape_l, dtype=dtype, device=device) for _ in range(2)]
        self._gathered = [torch.zeros(shape_g, dtype=dtype, device=device) for _ in range(2)]
        self._compact = None
        if self.ragged:
            rows = [r * self.width + i for r, c in enumerate(self.counts) for i in range(c)]
            self._index = torch.tensor(rows, dtype=torch.long, device=device)
            self._compact = [torch.empty((sum(self.counts),) + self.tail, dtype=dtype, device=device)
                             for _ in range(2)]
        self._work = [None, None]
        self._cur = 0
        self._last = None
        self._started = False

    def local(self) -> torch.Tensor:
        """This step's local output buffer, [counts[rank], *tail]; write it, then start()."""
        i = self._cur
        if self._work[i] is not None:  # the collective that read this buffer two steps ago
            self._work[i].wait()
            self._work[i] = None
        self._started = False
        return self._local[i][:self.counts[self.rank]]

    def start(self) -> None:
        """All-gather this step's local buffer, asynchronously; the next local() call hands
        out the other buffer."""
        if self._started:
            raise RuntimeError("start() once per local()")
        i = self._cur
        src, dst = self._local[i], self._gathered[i]
        if self._nccl:
            self._work[i] = dist.all_gather_into_tensor(dst, src, group=self.group, async_op=True)
        else:
            self._work[i] = dist.all_gather(list(dst.chunk(self.world)), src, group=self.group,
                                            async_op=True)
        self._started = True
        self._last = i
        self._cur = i ^ 1

    def result(self) -> torch.Tensor:
        """The last started step's gathered outputs, [sum(counts), *tail], rank order; the
        current stream waits for the collective (no host synchronisation)."""
        i = self._last
        if i is None:
            raise RuntimeError("no all-gather has been started")
        if self._work[i] is not None:
            self._work[i].wait()
            self._work[i] = None
        if not self.ragged:
            return self._gathered[i]
        torch.index_select(self._gathered[i], 0, self._index, out=self._compact[i])
        return self._compact[i]

    def wait_all(self) -> None:
        """Order every started collective before the current stream's next work."""
        for i in range(2):
            if self._work[i] is not None:
                self._work[i].wait()
                self._work[i] = None

    def close(self) -> None:
        """Order every started collective, give the attention its full grid back and
        destroy the gather's own process group (if max_ctas made one); collective, like
        the constructor."""
        self.wait_all()
        if self._prev_reserve is not None:
            from .paged_attn import reserve_sms

            reserve_sms(self._prev_reserve)
            self._prev_reserve = None
        if self._own_group is not None:
            dist.destroy_process_group(self._own_group)
            self._own_group = None


class _DeviceBytes:
    """A raw device allocation seen by torch through the CUDA array interface (no copy, no
    ownership)."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerGather:
    """Per-step gather of equal-sized per-rank outputs through NVLink peer memory, without
    a collective call on the data path (the kernels of csrc/peer.cu).

    Every rank allocates one buffer in its own HBM (flags, push counters, then two slots of
    world x rows outputs) and maps every other rank's buffer through CUDA IPC; the process group is
    used once, to exchange the IPC handles.  push(local) copies this rank's rows into the
    current slot of every rank's buffer and publishes the step's epoch; wait() orders the
    current stream after every rank's push of that epoch (a bounded device-side wait: a
    rank that stops publishing leaves INFERD_ERR_DEVICE_TIMEOUT in the error word instead
    of a hung GPU) and returns this rank's slot, [world * rows, *tail] in rank order.  Each
    push must be followed by its wait before the next push: that is what keeps a rank
    from overwriting a slot a peer may still read (the slot is rewritten two steps later,
    after every rank has pushed the step in between).
    """

    HEADER_BYTES = 512  # epoch flags [0, 256), this rank's push counters [256, 512)

    def __init__(self, tail: tuple[int, ...], dtype: torch.dtype, device: torch.device,
                 rows_per_rank: int, *, group=None, timeout_s: float = 2.0) -> None:
        import ctypes

        from . import _lib

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 64:
            raise ValueError("at most 64 ranks")
        self.device = torch.device(device)
        self.tail = tuple(int(t) for t in tail)
        self.rows = int(rows_per_rank)
        self.dtype = dtype
        elems = self.rows
        for t in self.tail:
            elems *= t
        self.bytes_per_rank = elems * torch.empty(0, dtype=dtype).element_size()
        if self.bytes_per_rank % 16 != 0:
            raise ValueError("one rank's rows must be a multiple of 16 bytes")
        self.timeout_ns = int(timeout_s * 1e9)
        slot_bytes = self.world * self.bytes_per_rank
        total = self.HEADER_BYTES + 2 * slot_bytes
        self._lib = lib = _lib.load()
        self._opened: list[int] = []
        self._own = None
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
            _lib.check(lib.inferd_peer_alloc(total, ctypes.byref(ptr), handle), "peer_alloc")
            self._own = ptr.value
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
            bases = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.inferd_peer_open(ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES),
                                                ctypes.byref(p)), "peer_open")
                self._opened.append(p.value)
                bases.append(p.value)
            self._dst = [torch.tensor([b + self.HEADER_BYTES + s * slot_bytes for b in bases],
                                      dtype=torch.int64, device=self.device) for s in range(2)]
            self._flags = torch.tensor(bases, dtype=torch.int64, device=self.device)
            own = torch.as_tensor(_DeviceBytes(self._own, total), device=self.device)
            self._slots = [own[self.HEADER_BYTES + s * slot_bytes:self.HEADER_BYTES + (s + 1) * slot_bytes]
                           .view(dtype).view((self.world * self.rows,) + self.tail) for s in range(2)]
        self._epoch = 0
        self._pending = False
        dist.barrier(group=group)  # every buffer is mapped everywhere before the first push

    def push(self, local: torch.Tensor) -> None:
        """Copy this rank's rows ([rows, *tail], contiguous, on this device) into every rank's
        current slot and publish the step; enqueued on the current stream."""
        from . import _lib

        if self._pending:
            raise RuntimeError("wait() for the previous push before the next one")
        if tuple(local.shape) != (self.rows,) + self.tail or local.dtype != self.dtype \
                or local.device != self.device or not local.is_contiguous():
            raise ValueError("local must be a contiguous [rows, *tail] tensor of this gather's "
                             "dtype on its device")
        self._epoch += 1
        st = self._lib.inferd_gather_push(
            local.data_ptr(), self.bytes_per_rank, self._dst[self._epoch & 1].data_ptr(),
            self._flags.data_ptr(), self._own + 256, self.rank, self.world,
            self._epoch & 0xFFFFFFFF, _lib.stream_of(self.device))
        _lib.check(st, "gather_push")
        self._pending = True

    def begin(self) -> tuple[int, int, int]:
        """Open the next step for a kernel that stores its outputs into every rank's slot
        itself (inferd_paged_attention_gather): returns (device array of the destinations,
        number of destinations, this rank's element offset in each).  publish() follows the
        kernel, then wait()."""
        if self._pending:
            raise RuntimeError("wait() for the previous push before the next one")
        self._epoch += 1
        elems = self.bytes_per_rank // torch.empty(0, dtype=self.dtype).element_size()
        return self._dst[self._epoch & 1].data_ptr(), self.world, self.rank * elems

    def publish(self) -> None:
        """Publish the step opened by begin() once the kernels that stored its rows are
        enqueued (a one-CTA kernel: system-scope release of this rank's flag everywhere)."""
        from . import _lib

        st = self._lib.inferd_gather_publish(self._flags.data_ptr(), self.rank, self.world,
                                             self._epoch & 0xFFFFFFFF, _lib.stream_of(self.device))
        _lib.check(st, "gather_publish")
        self._pending = True

    def wait(self) -> torch.Tensor:
        """Order the current stream after every rank's push of this step; returns this rank's
        slot, [world * rows, *tail] in rank order, valid until the push after next."""
        from . import _lib

        if not self._pending:
            raise RuntimeError("no push to wait for")
        st = self._lib.inferd_gather_wait(self._own, self.world, self._epoch & 0xFFFFFFFF,
                                          self.timeout_ns, _lib.error_word(self.device).data_ptr(),
                                          _lib.stream_of(self.device))
        _lib.check(st, "gather_wait")
        self._pending = False
        return self._slots[self._epoch & 1]

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still writes into a buffer being released
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.inferd_peer_close(p)
            self._opened = []
            self._slots = []
            self._lib.inferd_peer_free(self._own)
        self._own = None
