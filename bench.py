"""Decode hot-path benchmark: paged decode attention HBM GB/s and decode tok/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|long|verify]
                    [--impl ours|reference]
    python bench.py --workload fp8|fp8-dynamic|sampling     (one line per kernel case)

One step = one decode step of one attention layer for every sequence this GPU owns:
a one-token KV append per sequence (reshape_and_cache) followed by paged attention
over the sequence's context including that token; with N > 1 the outputs of all ranks
are gathered over NCCL inside the step.  Workloads (synthetic, seeded):

  decode  64 sequences per GPU, context lengths uniform in [512, 8192], 32 query heads
          over 8 KV heads, head_dim 128, block 16, pool = sequences + 10 % free blocks,
          block tables a random permutation of the pool, Q/K/V ~ N(0,1) in bf16
  long    32 sequences per GPU, lengths uniform in [16384, 32768], same heads
  verify  32 sequences per GPU, lengths uniform in [1024, 4096], k = 4 drafts + 1 query
          (5 queries, causal inside the window), 5-token append per sequence

`value` is algorithmic bytes (KV read + Q read + output write + block tables + the
append's read/write) of all ranks divided by the max-over-ranks device time of the K
timed steps, inputs resident in HBM; the KV pool (>= 1 GB per GPU) is larger than L2, so
no flush is needed between steps.  `e2e` repeats the step through the public Python
API with host (pinned) inputs and a device->host read of the output every step.
Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

HQ, HKV, D, BS = 32, 8, 128, 16
ELEM = 2  # bf16

WORKLOADS = {
    "decode": dict(seqs=64, lo=512, hi=8192, q_len=1,
                   label="config 2: batched paged decode"),
    "long": dict(seqs=32, lo=16384, hi=32768, q_len=1,
                 label="config 5: long-context sharded decode"),
    "verify": dict(seqs=32, lo=1024, hi=4096, q_len=5,
                   label="config 3: speculative verify"),
}
E2E_STEPS = 200            # default number of end-to-end steps
POOL_GROWTH = E2E_STEPS + 64  # spare tokens per sequence in the pool for the e2e steps


# ------------------------------------------------------------------ workload
def context_lengths(workload: str, world: int, seed: int = 0) -> np.ndarray:
    """Lengths of all sequences of the job (world * seqs); rank r owns a contiguous slice."""
    w = WORKLOADS[workload]
    rng = np.random.default_rng(seed)
    return rng.integers(w["lo"], w["hi"] + 1, size=w["seqs"] * world)


def rank_shards(workload: str, world: int) -> tuple[np.ndarray, list[list[int]]]:
    """The job's lengths and each rank's sequences: longest first onto the rank with the
    fewest tokens (inferd_b200.sharded.assign_by_tokens), so every GPU streams about the
    same KV bytes; a contiguous split of the same random lengths left one of four GPUs
    8.7 % above the mean, and every step waits for the slowest rank."""
    from inferd_b200.sharded import assign_by_tokens

    lens = context_lengths(workload, world)
    return lens, assign_by_tokens(lens.tolist(), world)


def step_bytes(ctx_lens, q_len: int) -> dict:
    """Algorithmic bytes of one step for sequences whose context (after the append) is
    ctx_lens: K and V of every visible key, query read, output write, block-table and
    context-length reads, and the append (read new K/V, write them to the pool, slots)."""
    ctx = np.asarray(ctx_lens, dtype=np.int64)
    b = ctx.size
    pages = (ctx + BS - 1) // BS
    attn = int(ctx.sum()) * HKV * D * ELEM * 2 + b * q_len * HQ * D * ELEM * 2 \
        + int(pages.sum()) * 4 + b * 4
    append = b * q_len * HKV * D * ELEM * 2 * 2 + b * q_len * 8
    return {"attention": attn, "append": append, "total": attn + append}


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def start(self) -> None:
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "", 1).isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def ncu_traffic(workload: str) -> float | None:
    """DRAM bytes per attention launch from the committed ncu summary, if present."""
    f = REPO / "profiles" / f"paged_attention_{workload}.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        line = line.strip()
        if line.startswith("dram_bytes_per_launch_full_size:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ our arm
class DeviceWorkload:
    """One rank's share of the workload, resident on its GPU.  The data depend only on
    (workload, rank, world, growth_tokens); with the default growth they are the bytes the
    benchmark times, so tests can rebuild them and check the kernels' outputs."""

    def __init__(self, workload: str, rank: int, world: int, device: torch.device,
                 growth_tokens: int = POOL_GROWTH) -> None:
        w = WORKLOADS[workload]
        self.workload = workload
        self.device = device
        self.q_len = w["q_len"]
        all_lens, owners = rank_shards(workload, world)
        self.counts = [len(o) for o in owners]  # sequences per rank (w["seqs"] here)
        self.base = all_lens[owners[rank]].astype(np.int64)
        self.b = self.base.size
        # context after the append = base + q_len (the appended tokens sit at base .. )
        self.ctx = self.base + self.q_len
        pages = (self.ctx + BS - 1) // BS
        # 10 % spare blocks, plus room for every sequence to grow by growth_tokens (the e2e
        # steps keep one token per step)
        grow = (growth_tokens + self.q_len + BS - 1) // BS + 1
        self.num_blocks = int(math.ceil(1.1 * pages.sum())) + self.b * grow
        g = torch.Generator(device=device).manual_seed(1234 + rank)
        shape = (self.num_blocks, HKV, BS, D)
        self.kc = torch.randn(shape, generator=g, device=device, dtype=torch.bfloat16)
        self.vc = torch.randn(shape, generator=g, device=device, dtype=torch.bfloat16)
        gc = torch.Generator().manual_seed(99 + rank)
        perm = torch.randperm(self.num_blocks, generator=gc).numpy()
        width = int(pages.max())
        bt = np.zeros((self.b, width), dtype=np.int32)
        s = 0
        for i, p in enumerate(pages.tolist()):
            bt[i, :p] = perm[s:s + p]
            s += p
        self.bt_host = bt
        self.bt = torch.from_numpy(bt).to(device)
        self.cl = torch.from_numpy(self.ctx.astype(np.int32)).to(device)
        slots = []
        for i in range(self.b):
            for j in range(self.q_len):
                pos = int(self.base[i]) + j
                slots.append(int(bt[i, pos // BS]) * BS + pos % BS)
        self.slots = torch.tensor(slots, dtype=torch.int64, device=device)
        self.q = torch.randn(self.b, self.q_len, HQ, D, generator=g, device=device,
                             dtype=torch.bfloat16)
        self.k_new = torch.randn(self.b * self.q_len, HKV, D, generator=g, device=device,
                                 dtype=torch.bfloat16)
        self.v_new = torch.randn_like(self.k_new)
        self.out = torch.empty_like(self.q)
        self.max_ctx = int(self.ctx.max())
        self.bytes = step_bytes(self.ctx, self.q_len)

    def append(self) -> None:
        """The step's KV append: one reshape_and_cache launch through the C ABI."""
        from inferd_b200 import _lib

        lib = _lib.load()
        st = lib.inferd_reshape_and_cache(
            self.k_new.data_ptr(), self.v_new.data_ptr(), self.k_new.stride(0),
            self.k_new.stride(1), self.v_new.stride(0), self.v_new.stride(1),
            self.kc.data_ptr(), self.vc.data_ptr(), self.slots.data_ptr(), self.slots.numel(),
            HKV, D, BS, self.num_blocks, 2, _lib.error_word(self.device).data_ptr(),
            torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(st, "reshape_and_cache")

    def attend(self, gather=None) -> None:
        """The step's paged attention over every sequence, into self.out (and, with a
        PeerGather, into every rank's gather slot from the kernel's epilogue)."""
        from inferd_b200.paged_attn import paged_attention_batched

        paged_attention_batched(self.q, self.kc, self.vc, self.bt, self.cl,
                                max_context_len=self.max_ctx, out=self.out, gather=gather)

    def sequence_pages(self, i: int) -> tuple[np.ndarray, np.ndarray]:
        """Sequence i's K and V pages, read back from the pool in table order as float32
        [pages, kv_heads, block_size, head_dim] (a compact pool whose table is arange)."""
        p = int((self.ctx[i] + BS - 1) // BS)
        ids = self.bt[i, :p].long()
        return (self.kc[ids].float().cpu().numpy(), self.vc[ids].float().cpu().numpy())

    def appended_bit_exact(self) -> bool:
        """The pool holds the step's new K/V bit for bit at every appended slot."""
        s = self.slots.long()
        blk, off = s // BS, s % BS
        return bool(torch.equal(self.kc[blk, :, off, :], self.k_new)
                    and torch.equal(self.vc[blk, :, off, :], self.v_new))


def run_ours(args, rank: int, world: int, device: torch.device) -> dict | None:
    import torch.distributed as dist

    from inferd_b200 import _lib
    from inferd_b200.sharded import OutputGather, PeerGather

    wl = DeviceWorkload(args.workload, rank, world, device,
                        growth_tokens=args.e2e_steps + POOL_GROWTH - E2E_STEPS)
    gather = peer = None
    if world > 1 and args.gather == "nccl":
        # NCCL all-gather of step N's outputs on NCCL's stream, overlapping step N + 1 (the
        # faster of the two on measurement)
        gather = OutputGather(tuple(wl.out.shape[1:]), wl.out.dtype, device, wl.counts,
                              max_ctas=args.gather_ctas)
    elif world > 1:
        # p2p: every rank pushes its outputs into every rank's memory over NVLink and waits
        # for the others' pushes.  fused: the attention kernel's epilogue stores them there
        # itself and a one-CTA kernel publishes the step; the wait for step N - 1 comes at
        # the start of step N, where every rank has long published it.
        if len(set(wl.counts)) != 1:
            raise ValueError(f"--gather {args.gather} needs equal rows per rank, not {wl.counts}")
        peer = PeerGather(tuple(wl.out.shape[1:]), wl.out.dtype, device, wl.b)
    fused = peer is not None and args.gather == "fused"
    stream = torch.cuda.current_stream(device)

    def step(ev=None):
        wl.append()
        if ev is not None:
            ev[0].record(stream)
        if gather is not None:
            wl.out = gather.local()  # double-buffered: the gather of step N - 1 may still read
        if fused and peer._pending:
            peer.wait()
        wl.attend(gather=peer if fused else None)
        if ev is not None:
            ev[1].record(stream)
        if gather is not None:
            gather.start()
        if peer is not None and not fused:
            peer.push(wl.out)
            peer.wait()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    _lib.raise_device_errors(device)

    k = args.steps
    attn_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(k)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(device.index if device.index is not None else 0)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    sampler.start()
    time.sleep(0.25)  # let the sampler attach before the timed region
    torch.cuda._sleep(20_000_000)  # device busy while the host queues the first steps
    t0.record(stream)
    for i in range(k):
        step(attn_ev[i])
    if gather is not None:
        gather.wait_all()  # the last steps' all-gathers belong to the timed region
    if fused:
        peer.wait()  # so does the last step's gather
    t1.record(stream)
    torch.cuda.synchronize(device)
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    attn_ms = sum(a.elapsed_time(b) for a, b in attn_ev) / k
    _lib.raise_device_errors(device)

    # max over ranks of the timed region; bytes summed over ranks
    stats = torch.tensor([elapsed_ms, attn_ms, float(wl.bytes["total"]),
                          float(wl.bytes["attention"]), float(wl.b)], dtype=torch.float64,
                         device=device)
    if world > 1:
        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        elapsed_ms, attn_ms = float(mx[0]), float(mx[1])
        total_bytes, attn_bytes, seqs = float(sm[2]), float(sm[3]), float(sm[4])
    else:
        total_bytes, attn_bytes, seqs = float(stats[2]), float(stats[3]), float(stats[4])
    ms_per_step = elapsed_ms / k
    value_gbs = total_bytes / (ms_per_step * 1e-3) / 1e9

    # checks of the last timed step, before the e2e steps reuse the pool: the append wrote
    # its K/V bit for bit; at N > 1 every rank's rows of the gathered output equal its own
    # output; at N = 1 the CPU leg compares every sequence's output with the oracle
    checks = {"append_bit_exact": wl.appended_bit_exact()}
    gather_us = None
    if world > 1:
        if gather is not None:
            gathered = gather.result()
        else:
            if fused and peer._pending:
                peer.wait()
            gathered = peer._slots[peer._epoch & 1]
        # every rank's rows of the gathered output equal that rank's own output, on every rank
        from inferd_b200.sharded import gather_outputs

        ref = gather_outputs(wl.out, wl.counts)
        mine = torch.equal(gathered, ref)
        flag = torch.tensor([int(mine and checks["append_bit_exact"])], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        checks["gathered_rows_equal_rank_outputs"] = bool(flag.item())
        # the gather alone, back to back, for the record (max over ranks)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize(device)
        g0.record(stream)
        for _ in range(k):
            if gather is not None:
                gather.local()
                gather.start()
            else:  # (fused: the push kernel stands in for the epilogue's extra stores)
                peer.push(wl.out)
                peer.wait()
        if gather is not None:
            gather.wait_all()
        g1.record(stream)
        torch.cuda.synchronize(device)
        _lib.raise_device_errors(device)
        t = torch.tensor([g0.elapsed_time(g1) * 1000.0 / k], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gather_us = round(float(t.item()), 2)
    parity = cpu = None
    if world == 1:
        parity, cpu = cpu_leg(wl, budget_s=0.0 if args.no_cpu_baseline else args.cpu_budget)
    if not all(checks.values()) or (parity is not None and not parity["ok"]):
        raise RuntimeError(f"output check failed: {checks} {parity}")

    if gather is not None:
        gather.close()  # the end-to-end leg gathers on the compute stream, with full grids
    e2e = run_e2e(args, wl, rank, world, device, peer=peer)
    if peer is not None:
        peer.close()

    if rank != 0:
        return None
    peaks = measured_peaks()
    achieved = wl.bytes["attention"] / (attn_ms * 1e-3) / 1e9  # this rank's kernel
    traffic = ncu_traffic(args.workload)
    line = {
        "metric": "paged-decode attn HBM GB/s (% of peak) & decode tok/s at 1/2/4/8 B200",
        "value": round(value_gbs, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": k,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V in bf16, seeded uniform context lengths, "
                "randomly permuted block tables)",
        "config": config_block(args.workload, world),
        "decode_tok_s": round(seqs * wl.q_len / (ms_per_step * 1e-3), 1),
        "attention_ms": round(attn_ms, 5),
        "attention_gbs_per_gpu": round(achieved, 1),
        "pct_of_hbm_peak": round(100.0 * achieved / peaks["hbm_gbs"], 2),
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
            "traffic": traffic, "peak_source": peaks["source"],
            "kernel": "paged_attn_tc_kernel",
        },
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": 2 * k,
    }
    line["checks"] = checks
    if gather_us is not None:
        line["gather"] = {"kind": args.gather, "us_per_step_alone": gather_us,
                          "nccl_max_ctas": args.gather_ctas if args.gather == "nccl" else None,
                          "bytes_per_rank": int(wl.out.numel() * wl.out.element_size()),
                          "how": {"nccl": "NCCL all_gather_into_tensor on NCCL's stream, "
                                          "overlapping the next step",
                                  "p2p": "push kernel (this rank's rows into every rank's buffer "
                                         "over NVLink, epoch flag) + bounded wait kernel, inside "
                                         "the step",
                                  "fused": "the attention epilogue stores the rows into every "
                                           "rank's buffer over NVLink; a one-CTA kernel publishes "
                                           "the epoch; the bounded wait for step N - 1 opens step N"
                                  }[args.gather]}
    if parity is not None:
        line["parity"] = parity
    if cpu is not None and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu
    return line


def config_block(workload: str, world: int) -> dict:
    """The `config` object of both arms' lines: the workload and its sizes per GPU."""
    w = WORKLOADS[workload]
    lens, owners = rank_shards(workload, world)
    ctx = lens[owners[0]] + w["q_len"]
    pages = (ctx + BS - 1) // BS
    grow = (POOL_GROWTH + w["q_len"] + BS - 1) // BS + 1
    attn_gb = step_bytes(ctx, w["q_len"])["attention"] / 1e9
    return {
        "workload": w["label"], "seqs_per_gpu": w["seqs"], "context_lo": w["lo"],
        "context_hi": w["hi"], "q_len": w["q_len"], "q_heads": HQ, "kv_heads": HKV,
        "head_dim": D, "block_size": BS,
        "pool_blocks_per_gpu": int(math.ceil(1.1 * pages.sum())) + w["seqs"] * grow,
        "parallelism": f"sequence shards x{world}, outputs all-gathered over NCCL"
        if world > 1 else "single GPU",
        "l2": "no flush: each step reads >= %.2f GB of KV per GPU (L2 is 126 MB)" % attn_gb,
    }


def run_e2e(args, dwl: DeviceWorkload, rank: int, world: int, device: torch.device,
            peer=None) -> dict:
    """Same step through the public API with pinned host inputs and a host read of the
    result every step: a DecodeGraph replay -- the host-to-device copy of the step's inputs
    (queries and new K/V from pinned memory), the page-table update, the KV append, paged
    attention and the device-to-host copy of the output -- then (N > 1) the all-gather and
    its copy to the host, and a stream sync.  The host side of a step (pages, slots, table
    changes) is DecodeGraph.prepare; decode prepares step N + 1 while step N runs, as an
    engine that schedules ahead does, and verify after its rollback, which needs the step's
    result."""
    import torch.distributed as dist

    from inferd_b200.decode_graph import DecodeGraph
    from inferd_b200.paged_cache import PagedKVCache
    from inferd_b200.sharded import gather_outputs

    ql = dwl.q_len
    cache = PagedKVCache(num_layers=1, num_blocks=dwl.num_blocks, block_size=BS,
                         num_kv_heads=HKV, head_dim=D, dtype=torch.bfloat16, device=device)
    cache.key_cache[0] = dwl.kc
    cache.value_cache[0] = dwl.vc
    used = set()
    ids = list(range(dwl.b))
    for i in ids:
        t = cache.create_sequence(i)
        p = (int(dwl.base[i]) + BS - 1) // BS
        t.blocks = dwl.bt_host[i, :p].tolist()
        t.length = int(dwl.base[i])
        used.update(t.blocks)
    cache.allocator._allocated = set(used)
    cache.allocator._free = [x for x in cache.allocator._free if x not in used]
    graph = DecodeGraph(cache, ids, num_q_heads=HQ, q_len=ql, copy_out=world == 1)
    # the step's inputs: the same data every step, staged once in both pinned sets; every
    # replay copies them to the device
    for q_h, k_h, v_h in graph.input_buffers():
        q_h.copy_(dwl.q.cpu())
        k_h.copy_(dwl.k_new.cpu())
        v_h.copy_(dwl.v_new.cpu())
    out_rows = sum(dwl.counts)
    out_h = torch.empty((out_rows, ql, HQ, D), dtype=torch.bfloat16).pin_memory()
    gathered = torch.empty((out_rows, ql, HQ, D), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    steps = max(1, min(args.steps, args.e2e_steps))
    d2h = out_rows * ql * HQ * D * ELEM
    keep_one = [1] * len(ids)

    def one_step():
        graph.launch()
        if peer is not None:
            peer.push(graph.output)
            out_h.copy_(peer.wait(), non_blocking=True)
        elif world > 1:
            gather_outputs(graph.output, dwl.counts, out=gathered)
            out_h.copy_(gathered, non_blocking=True)
        if ql == 1:
            graph.prepare()  # step N + 1's pages and slots while step N runs
        stream.synchronize()
        if ql > 1:
            # speculative verify: keep one accepted token, roll the rest of the window back
            graph.rollback(keep_one)
            graph.prepare()

    graph.prepare()
    one_step()  # warm the path
    # every step grows each context by one token net, so the bytes of the timed steps are
    # known up front: step s attends over base + s + q_len keys per sequence
    base = np.asarray([cache.sequence_length(i) for i in ids], dtype=np.int64)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        one_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1)
    graph.abort()  # the step prepared for after the last timed one
    if [cache.sequence_length(i) for i in ids] != (base + steps).tolist():
        raise RuntimeError("context lengths after the timed steps differ from the byte count's")
    total_bytes = float(sum(step_bytes(base + s + ql, ql)["total"] for s in range(steps)))
    h2d = graph.staged_bytes()  # inputs, slots, lengths and table changes of one replay
    t = torch.tensor([ms, total_bytes], dtype=torch.float64, device=device)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms, total_bytes = float(mx[0]), float(sm[1])
    return {"value": round(total_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "steps": steps, "ms_per_step": round(ms / steps, 5),
            "d2h": ("the attention's epilogue stores the output rows to pinned host memory "
                    "as the grid runs" if graph._host_rows is not None else
                    "one device-to-host copy after the attention") if world == 1 else
                   "all-gather, then one device-to-host copy",
            "note": "one DecodeGraph replay per step (inputs H2D from pinned memory, page-table "
                    "update, KV append, attention, output D2H); contexts grow by one token per "
                    "step (verify: the window is appended, verified, and all but one token "
                    "rolled back); decode prepares the next step while the current one runs"}


# ------------------------------------------------------------------ FP8 linear (config 4)
FP8_N, FP8_K = 17408, 5120
FP8_PEAK_NOMINAL_TFLOPS = 4500.0  # dense e4m3 per B200 (no measured FP8 figure on this pool)


def run_fp8(args, device: torch.device) -> list[dict]:
    """Config 4: W [17408, 5120] e4m3 from N(0, 0.02) bf16 quantised per channel ("fp8",
    weight-only) or per tensor ("fp8-dynamic", activations quantised per tensor on every
    call), x ~ N(0,1) bf16 [M, 5120].  Three weight copies (267 MB > L2) rotate between
    calls so every call streams its weight from HBM.  One line per M."""
    from functools import partial

    from inferd_b200.fp8_linear import (fp8_dynamic_linear, fp8_linear, pack_fp8_weight,
                                        quantize_fp8_dynamic, quantize_fp8_per_channel)

    dynamic = args.workload == "fp8-dynamic"
    quantize = quantize_fp8_dynamic if dynamic else quantize_fp8_per_channel
    linear = partial(fp8_dynamic_linear, granularity="tensor") if dynamic else fp8_linear

    peaks = measured_peaks()
    p = REPO / "MEASURED_PEAKS.json"
    bf16_peak = json.loads(p.read_text()).get("bf16_tflops") if p.exists() else 1590.0
    g = torch.Generator(device=device).manual_seed(4)
    copies = []
    for _ in range(3):
        w = torch.randn(FP8_N, FP8_K, generator=g, device=device, dtype=torch.float32).mul_(0.02)
        q, s = quantize(w.to(torch.bfloat16))
        copies.append((pack_fp8_weight(q), s) if args.fp8_layout == "packed" else (q, s))
        del w, q
    stream = torch.cuda.current_stream(device)
    shape = (FP8_N, FP8_K) if args.fp8_layout == "packed" else None
    lines = []
    for m in [int(v) for v in args.fp8_m.split(",")]:
        x = torch.randn(m, FP8_K, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
        out = torch.empty(m, FP8_N, dtype=torch.bfloat16, device=device)
        for i in range(args.warmup):
            q, s = copies[i % 3]
            linear(x, q, s, out=out, packed_shape=shape)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # keep the GPU busy while the host queues the timed calls, so the events time the
        # device and not the Python/ctypes call overhead
        torch.cuda._sleep(20_000_000)
        e0.record(stream)
        for i in range(args.steps):
            q, s = copies[i % 3]
            linear(x, q, s, out=out, packed_shape=shape)
        e1.record(stream)
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / args.steps
        nbytes = FP8_N * FP8_K + FP8_N * 4 + m * FP8_K * 2 + m * FP8_N * 2
        flops = 2.0 * m * FP8_N * FP8_K
        gbs = nbytes / (ms * 1e-3) / 1e9
        tfs = flops / (ms * 1e-3) / 1e12
        planes = 1 if dynamic else 2  # e4m3 activation planes the tensor pipe multiplies
        lines.append({
            "metric": ("fp8-dynamic linear, per-tensor scales (config 4)" if dynamic
                       else "fp8 weight-only linear (config 4)"), "m": m, "n": FP8_N, "k": FP8_K,
            "ms": round(ms, 5), "value": round(tfs, 1), "unit": "TFLOP/s",
            "hbm_gbs": round(gbs, 1), "pct_of_hbm_peak": round(100 * gbs / peaks["hbm_gbs"], 2),
            "pct_of_fp8_nominal_peak": round(100 * tfs / FP8_PEAK_NOMINAL_TFLOPS, 2),
            "pct_of_measured_bf16_peak": round(100 * tfs / bf16_peak, 2),
            "tensor_flops_issued": ("1x algorithmic (one e4m3 activation plane)" if dynamic
                                    else "2x algorithmic (two e4m3 activation planes)"),
            "roofline": {
                "bound": "tensor" if m >= 128 else "hbm",
                "achieved": round(tfs, 1) if m >= 128 else round(gbs, 1),
                "peak": round(2 * bf16_peak, 1) if m >= 128 else peaks["hbm_gbs"],
                "unit": "TFLOP/s" if m >= 128 else "GB/s",
                "frac": round(tfs / (2 * bf16_peak), 4) if m >= 128 else round(gbs / peaks["hbm_gbs"], 4),
                "tensor_pipe_frac": round(planes * tfs / (2 * bf16_peak), 4),
                "peak_source": "of measured: e4m3 dense peak = 2 x the measured cuBLAS bf16 burst"
                               if m >= 128 else "of measured: HBM copy bandwidth",
            },
            "calls_timed": args.steps,
            "timing": ("one CUDA event pair around the timed calls (absmax + quantise + GEMM per call)"
                       if dynamic else "one CUDA event pair around the timed calls (split + GEMM per call)"),
            "l2": "three weight copies rotated (267 MB > 126 MB L2)",
            "weight_layout": args.fp8_layout,
        })
    return lines


# ------------------------------------------------------------------ decode-step sampling
SAMP_ROWS, SAMP_VOCAB, SAMP_T, SAMP_TOP_P = 64, 151936, 0.7, 0.9


def run_sampling(args, device: torch.device) -> list[dict]:
    """Decode-step sampling for a batch of 64 sequences over a 151,936-entry vocabulary
    (the Qwen tokenizer's embedding width), bf16 logits ~ N(0, 3^2), temperature 0.7,
    top_p 0.9.  Two lines: nucleus_probs (fp32 probabilities written) and the fused sampler
    (one token per row, no probabilities).  Eight logits copies (156 MB) and eight output
    buffers rotate so no call finds its data in L2.  The timed calls go straight to the C
    ABI (the Python wrapper's per-call checks would otherwise be the bottleneck)."""
    import oracle
    from inferd_b200 import _lib

    lib = _lib.load()
    g = torch.Generator(device=device).manual_seed(7)
    rows, vocab = SAMP_ROWS, SAMP_VOCAB
    copies = [(torch.randn(rows, vocab, generator=g, device=device) * 3.0).to(torch.bfloat16)
              for _ in range(8)]
    outs = [torch.empty(rows, vocab, dtype=torch.float32, device=device) for _ in range(8)]
    toks = torch.empty(rows, dtype=torch.int64, device=device)
    err = _lib.error_word(device)
    stream = torch.cuda.current_stream(device)
    peaks = measured_peaks()

    def call(i, with_probs):
        x = copies[i % 8]
        st = lib.inferd_nucleus_sample(
            outs[i % 8].data_ptr() if with_probs else None, vocab,
            None if with_probs else toks.data_ptr(), x.data_ptr(), 2, vocab, rows, vocab,
            None, SAMP_T, None, SAMP_TOP_P, 1234, i * rows, err.data_ptr(), stream.cuda_stream)
        _lib.check(st, "nucleus_sample")

    lines = []
    for with_probs in (True, False):
        for i in range(args.warmup):
            call(i, with_probs)
        torch.cuda.synchronize(device)
        _lib.raise_device_errors(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)
        e0.record(stream)
        for i in range(args.steps):
            call(i, with_probs)
        e1.record(stream)
        torch.cuda.synchronize(device)
        _lib.raise_device_errors(device)
        ms = e0.elapsed_time(e1) / args.steps
        nbytes = rows * vocab * 2 + (rows * vocab * 4 if with_probs else rows * 8)
        gbs = nbytes / (ms * 1e-3) / 1e9
        lines.append({
            "metric": "decode-step sampling (temperature + top-p)",
            "variant": "nucleus_probs" if with_probs else "sample_nucleus",
            "rows": rows, "vocab": vocab, "temperature": SAMP_T, "top_p": SAMP_TOP_P,
            "logits_dtype": "bf16", "us_per_call": round(ms * 1000, 2),
            "rows_per_s": round(rows / (ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "bytes_per_call": nbytes, "peak_source": peaks["source"],
                         "kernel": "nucleus16_kernel"},  # the bf16 logits' kernel
            "l2": "eight rotating logits copies (156 MB) and outputs",
            "calls_timed": args.steps,
        })
    if not args.no_cpu_baseline:
        # the oracle restates the reference's per-row softmax + sort + cumsum in numpy
        x = copies[0][:4].float().cpu().numpy()
        t0 = time.perf_counter()
        done = 0
        while time.perf_counter() - t0 < min(args.cpu_budget, 10.0) or done == 0:
            oracle.nucleus_probs(x[done % 4], SAMP_T, SAMP_TOP_P)
            done += 1
        dt = time.perf_counter() - t0
        cpu = {"value": round(done / dt, 2), "unit": "rows/s", "cores": _cpu_threads(), "kind": "port",
               "sample": f"{done} rows of nucleus_probs in numpy (softmax, stable sort, cumsum), {dt:.1f} s"}
        for line in lines:
            line["cpu_baseline"] = cpu
    return lines


# ------------------------------------------------------------------ CPU baseline (oracle)
class CpuWork:
    """The oracle (numpy restatement of the reference's per-sequence gather + attention)
    on a sample of the workload's sequences, bf16 data widened to fp32 like the reference's
    fp32 path."""

    def __init__(self, workload: str, max_seqs: int = 8) -> None:
        w = WORKLOADS[workload]
        lens = context_lengths(workload, 1)[:max_seqs].astype(np.int64) + w["q_len"]
        self.q_len = w["q_len"]
        self.lens = lens
        pages = (lens + BS - 1) // BS
        nb = int(pages.sum())
        rng = np.random.default_rng(7)
        self.kc = rng.standard_normal((nb, HKV, BS, D), dtype=np.float32)
        self.vc = rng.standard_normal((nb, HKV, BS, D), dtype=np.float32)
        perm = rng.permutation(nb)
        self.tables, s = [], 0
        for p in pages.tolist():
            self.tables.append(perm[s:s + p])
            s += p
        self.q = rng.standard_normal((lens.size, self.q_len, HQ, D), dtype=np.float32)

    def run_seq(self, i: int) -> int:
        import oracle

        L = int(self.lens[i])
        if self.q_len == 1:
            oracle.paged_attention(self.q[i, 0], self.kc, self.vc, self.tables[i], L)
        else:
            k, v = oracle.gather_paged_kv(self.kc, self.vc, self.tables[i], L)
            oracle.verify_attention(self.q[i], k, v)
        return step_bytes([L], self.q_len)["total"]


ATOL_BF16, RTOL_BF16 = 2e-2, 1e-2  # attention tolerance against the fp32 oracle


def _oracle_sequence(q: np.ndarray, kp: np.ndarray, vp: np.ndarray, ctx: int) -> np.ndarray:
    """The oracle's output for one sequence: q [q_len, Hq, D] over its compact pages
    kp / vp [pages, Hkv, BS, D] (table = arange)."""
    import oracle

    table = np.arange(kp.shape[0])
    if q.shape[0] == 1:
        return oracle.paged_attention(q[0], kp, vp, table, ctx)[None]
    k, v = oracle.gather_paged_kv(kp, vp, table, ctx)
    return oracle.verify_attention(q, k, v)


def cpu_leg(wl: DeviceWorkload, budget_s: float = 15.0) -> tuple[dict, dict | None]:
    """The CPU leg at N = 1, run on the benchmarked sequences themselves (their pages read
    back from HBM after the timed steps, bf16 widened to fp32).

    parity: the oracle (numpy restatement of the reference's per-sequence gather + GQA
    attention, causal inside a verify window) against the last timed step's output, every
    sequence, at 2e-2 max-abs and 1e-2 relative (max-abs error over max |oracle|).
    cpu_baseline: the same oracle timed on the host cores for about budget_s seconds,
    cycling over the first sequences (up to 8, at most 512 MB of fp32 pages held)."""
    out = wl.out.float().cpu().numpy()
    q = wl.q.float().cpu().numpy()
    worst_abs = worst_rel = 0.0
    kept, kept_bytes = [], 0
    for i in range(wl.b):
        kp, vp = wl.sequence_pages(i)
        ctx = int(wl.ctx[i])
        ref = _oracle_sequence(q[i], kp, vp, ctx)
        err = float(np.abs(out[i] - ref).max())
        worst_abs = max(worst_abs, err)
        worst_rel = max(worst_rel, err / max(float(np.abs(ref).max()), 1e-6))
        if len(kept) < 8 and kept_bytes + kp.nbytes + vp.nbytes <= 512 << 20:
            kept.append((q[i], kp, vp, ctx))
            kept_bytes += kp.nbytes + vp.nbytes
        del kp, vp
    parity = {"ok": worst_abs <= ATOL_BF16 and worst_rel <= RTOL_BF16,
              "max_abs_err": round(worst_abs, 6), "max_rel_err": round(worst_rel, 6),
              "seqs_checked": wl.b, "append_checked": "bit-exact at every appended slot",
              "tolerance": "max-abs <= 2e-2 and max-abs / max|oracle| <= 1e-2 per sequence",
              "oracle": "numpy fp32 restatement of the reference's gather + attention"}
    if budget_s <= 0:
        return parity, None
    t0 = time.perf_counter()
    done = nbytes = 0
    while time.perf_counter() - t0 < budget_s or done == 0:
        qi, kp, vp, ctx = kept[done % len(kept)]
        _oracle_sequence(qi, kp, vp, ctx)
        nbytes += step_bytes([ctx], wl.q_len)["total"]
        done += 1
    dt = time.perf_counter() - t0
    cpu = {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": _cpu_threads(),
           "kind": "port",
           "sample": f"{done} single-sequence steps of the oracle (numpy fp32 per-sequence gather "
                     f"+ GQA attention{', causal window' if wl.q_len > 1 else ''}) over the first "
                     f"{len(kept)} benchmarked sequences, read back from HBM, {dt:.1f} s"}
    return parity, cpu


def _cpu_threads() -> int:
    try:
        import threadpoolctl

        info = threadpoolctl.threadpool_info()
        n = max((d.get("num_threads", 1) for d in info), default=1)
        return int(n)
    except Exception:  # pragma: no cover - informational only
        return os.cpu_count() or 1


def run_reference(args, rank: int, world: int) -> dict | None:
    """Reference arm: the oracle port of the reference's CPU path, timed on host cores.
    Each step is one sequence of the workload (cycling), all host threads available."""
    if rank != 0:
        return None
    work = CpuWork(args.workload)
    for i in range(args.warmup):
        work.run_seq(i % work.lens.size)
    t0 = time.perf_counter()
    nbytes = 0
    for i in range(args.steps):
        nbytes += work.run_seq(i % work.lens.size)
    dt = time.perf_counter() - t0
    v = round(nbytes / dt / 1e9, 3)
    return {
        "metric": "paged-decode attn HBM GB/s (% of peak) & decode tok/s at 1/2/4/8 B200",
        "impl": "reference", "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_block(args.workload, world),
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": _cpu_threads(), "kind": "port",
                         "sample": "one sequence of the workload per step, cycling over the "
                                   f"first {work.lens.size} sequences"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------ main
def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["fp8", "fp8-dynamic", "sampling"],
                    default="decode")
    ap.add_argument("--fp8-m", default="1,8,32,128,256", help="token counts for --workload fp8")
    ap.add_argument("--fp8-layout", choices=["packed", "rowmajor"], default="packed")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--gather", choices=["p2p", "nccl", "fused"], default="nccl",
                    help="N > 1: how each step's outputs reach every GPU")
    ap.add_argument("--gather-ctas", type=int, default=0,
                    help="--gather nccl: NCCL CTAs for the overlapped all-gather, and as many "
                         "SMs left out of the attention grid (0: NCCL's default, full grid)")
    ap.add_argument("--e2e-steps", type=int, default=E2E_STEPS)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.workload == "sampling":
        if rank == 0:
            for line in run_sampling(args, device):
                print(json.dumps(line), flush=True)
        return 0
    if args.workload in ("fp8", "fp8-dynamic"):
        if rank == 0:
            for line in run_fp8(args, device):
                print(json.dumps(line), flush=True)
        return 0
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device,
                                timeout=datetime.timedelta(seconds=120))
    line = None
    try:
        line = run_ours(args, rank, world, device)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
