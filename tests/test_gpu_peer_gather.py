"""The output gather over NVLink peer memory (csrc/peer.cu, inferd_b200.sharded.PeerGather).

One GPU: the gather of a one-rank group through the C ABI and the Python class (every
step's slot equals the pushed rows, slots alternate), and a bounded wait that runs out (a
flag that nothing sets) reporting INFERD_ERR_DEVICE_TIMEOUT with the context still usable.
Two GPUs (skipped with fewer): two NCCL ranks gather several steps of different rows and
must agree with NCCL's own all-gather of the same tensors bit for bit.
"""

from __future__ import annotations

import ctypes
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferd_b200 import _lib
from inferd_b200.sharded import PeerGather, _DeviceBytes

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_push_and_wait_one_rank_through_c_abi(cuda_device):
    lib = _lib.load()
    rows, width = 8, 256  # 8 rows x 256 bf16 = 4 KiB per rank
    nbytes = rows * width * 2
    total = 512 + 2 * nbytes
    ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    _lib.check(lib.inferd_peer_alloc(total, ctypes.byref(ptr), handle), "peer_alloc")
    try:
        base = ptr.value
        own = torch.as_tensor(_DeviceBytes(base, total), device=cuda_device)
        flags = torch.tensor([base], dtype=torch.int64, device=cuda_device)
        err = _lib.error_word(cuda_device)
        stream = _lib.stream_of(cuda_device)
        for epoch in range(1, 6):
            src = torch.randn(rows, width, device=cuda_device).to(torch.bfloat16)
            slot = epoch & 1
            dst = torch.tensor([base + 512 + slot * nbytes], dtype=torch.int64, device=cuda_device)
            _lib.check(lib.inferd_gather_push(src.data_ptr(), nbytes, dst.data_ptr(), flags.data_ptr(),
                                              base + 256, 0, 1, epoch, stream), "gather_push")
            _lib.check(lib.inferd_gather_wait(base, 1, epoch, 0, err.data_ptr(), stream), "gather_wait")
            torch.cuda.synchronize()
            _lib.raise_device_errors(cuda_device)
            got = own[512 + slot * nbytes:512 + (slot + 1) * nbytes].view(torch.bfloat16).view(rows, width)
            assert torch.equal(got, src)
            assert int(own[:4].view(torch.int32)[0]) == epoch
        # bad arguments are refused before anything is launched
        assert lib.inferd_gather_push(src.data_ptr(), nbytes + 2, dst.data_ptr(), flags.data_ptr(),
                                      base + 256, 0, 1, 9, stream) == _lib.ERR_INVALID_ARGUMENT
        assert lib.inferd_gather_push(src.data_ptr(), nbytes, dst.data_ptr(), flags.data_ptr(),
                                      base + 256, 1, 1, 9, stream) == _lib.ERR_INVALID_ARGUMENT
    finally:
        torch.cuda.synchronize()
        lib.inferd_peer_free(ptr.value)


def test_wait_for_a_flag_nothing_sets_times_out(cuda_device):
    # the failure the bounded wait exists for: a rank that never publishes.  The wait gives
    # up after 1 ms, records the timeout, and the GPU keeps working.
    lib = _lib.load()
    ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    _lib.check(lib.inferd_peer_alloc(512 + 32, ctypes.byref(ptr), handle), "peer_alloc")
    try:
        err = _lib.error_word(cuda_device)
        st = lib.inferd_gather_wait(ptr.value, 2, 5, 1_000_000, err.data_ptr(), _lib.stream_of(cuda_device))
        assert st == _lib.OK
        torch.cuda.synchronize()
        assert int(err.item()) == _lib.ERR_DEVICE_TIMEOUT
        err.zero_()
        x = torch.arange(10, device=cuda_device)
        assert int(x.sum()) == 45
    finally:
        torch.cuda.synchronize()
        lib.inferd_peer_free(ptr.value)


def test_peer_gather_one_rank_group(cuda_device):
    port = _free_port()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        g = PeerGather((4, 128), torch.bfloat16, cuda_device, 3)
        for step in range(4):
            local = torch.randn(3, 4, 128, device=cuda_device).to(torch.bfloat16)
            g.push(local)
            with pytest.raises(RuntimeError):
                g.push(local)  # the wait comes first
            out = g.wait()
            assert out.shape == (3, 4, 128) and torch.equal(out, local)
        with pytest.raises(ValueError):
            g.push(torch.zeros(2, 4, 128, device=cuda_device, dtype=torch.bfloat16))
        g.close()
        _lib.raise_device_errors(cuda_device)
    finally:
        dist.destroy_process_group()


def _two_rank_worker(rank: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    ok = True
    try:
        g = PeerGather((32, 128), torch.bfloat16, dev, 16, timeout_s=1.0)
        ref = torch.empty(32, 32, 128, dtype=torch.bfloat16, device=dev)
        for step in range(6):
            gen = torch.Generator(device=dev).manual_seed(100 * step + rank)
            local = torch.randn(16, 32, 128, generator=gen, device=dev).to(torch.bfloat16)
            g.push(local)
            out = g.wait()
            dist.all_gather_into_tensor(ref, local)
            torch.cuda.synchronize(dev)
            ok &= bool(torch.equal(out, ref))
        _lib.raise_device_errors(dev)
        g.close()
    except Exception as e:  # reported to the parent, which fails the test
        ok = repr(e)
    finally:
        dist.destroy_process_group()
    q.put((rank, ok))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_peer_gather_two_ranks_match_nccl_all_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == {0: True, 1: True}, got


def _attn_inputs(device, seed, b=6, hq=32, hkv=8, d=128, q_len=1):
    g = torch.Generator(device=device).manual_seed(seed)
    lens = torch.randint(20, 700, (b,), generator=g, device=device).to(torch.int32)
    pages = (lens + 15) // 16
    nb = int(pages.sum()) + 4
    kc = torch.randn(nb, hkv, 16, d, generator=g, device=device).to(torch.bfloat16)
    vc = torch.randn(nb, hkv, 16, d, generator=g, device=device).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g, device=device).to(torch.int32)
    bt = torch.zeros(b, int(pages.max()), dtype=torch.int32, device=device)
    s = 0
    for i, p in enumerate(pages.tolist()):
        bt[i, :p] = perm[s:s + p]
        s += p
    q = torch.randn(b, q_len, hq, d, generator=g, device=device).to(torch.bfloat16)
    return q, kc, vc, bt, lens


@pytest.mark.parametrize("q_len", [1, 5])
def test_attention_epilogue_gather_one_rank(cuda_device, q_len):
    # the gathered slot holds exactly what the attention wrote to `out`, step after step
    from inferd_b200 import paged_attention_batched

    port = _free_port()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        g = PeerGather((q_len, 32, 128), torch.bfloat16, cuda_device, 6)
        for step in range(4):
            q, kc, vc, bt, cl = _attn_inputs(cuda_device, 10 * step + q_len, q_len=q_len)
            if g._pending:
                g.wait()
            out = paged_attention_batched(q, kc, vc, bt, cl, gather=g)
            ref = paged_attention_batched(q, kc, vc, bt, cl)
            slot = g.wait()
            torch.cuda.synchronize()
            assert torch.equal(out, ref) and torch.equal(slot, out)
        g.close()
        _lib.raise_device_errors(cuda_device)
    finally:
        dist.destroy_process_group()


def _fused_worker(rank: int, port: int, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    ok = True
    try:
        from inferd_b200 import paged_attention_batched

        g = PeerGather((1, 32, 128), torch.bfloat16, dev, 6, timeout_s=1.0)
        ref = torch.empty(12, 1, 32, 128, dtype=torch.bfloat16, device=dev)
        for step in range(5):
            q, kc, vc, bt, cl = _attn_inputs(dev, 100 * step + rank)
            if g._pending:
                g.wait()
            out = paged_attention_batched(q, kc, vc, bt, cl, gather=g)
            full = g.wait()
            dist.all_gather_into_tensor(ref, out)
            torch.cuda.synchronize(dev)
            ok &= bool(torch.equal(full, ref))
        _lib.raise_device_errors(dev)
        g.close()
    except Exception as e:  # reported to the parent, which fails the test
        ok = repr(e)
    finally:
        dist.destroy_process_group()
    results.put((rank, ok))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_attention_epilogue_gather_two_ranks_match_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == {0: True, 1: True}, got
