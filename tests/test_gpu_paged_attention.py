"""GPU parity of the paged attention kernels against the CPU oracle and reference goldens.

Tolerances: fp32 pools (generic kernel) use the reference's own test tolerance
(rtol 1e-4, atol 1e-5, tests/test_paged_equiv.py:104 of the reference); bf16 / fp16
pools (tensor-core kernel) must be within 2e-2 max-abs and 1e-2 relative (max-abs error
over max |reference|) of the fp32 oracle on the same bf16-rounded inputs.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from inferd_b200 import (
    _lib,
    paged_attention,
    paged_attention_batched,
    paged_attention_reference,
    dense_attention,
)

pytestmark = pytest.mark.gpu

ATOL_BF16 = 2e-2
RTOL_BF16 = 1e-2


def assert_bf16_close(out: np.ndarray, ref: np.ndarray, what: str = "") -> None:
    err = float(np.abs(out - ref).max()) if out.size else 0.0
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    assert err <= ATOL_BF16, f"{what}: max abs error {err}"
    assert err <= RTOL_BF16 * max(scale, 1e-6) or err <= 1e-4, f"{what}: rel error {err / scale}"


def make_pool(num_blocks, hkv, bs, d, dtype, gen, device):
    kc = torch.randn(num_blocks, hkv, bs, d, generator=gen).to(dtype)
    vc = torch.randn(num_blocks, hkv, bs, d, generator=gen).to(dtype)
    return kc, vc, kc.to(device), vc.to(device)


def random_tables(lens, bs, num_blocks, gen):
    pages = [(L + bs - 1) // bs for L in lens]
    perm = torch.randperm(num_blocks, generator=gen)
    width = max(pages + [1])
    bt = torch.zeros(len(lens), width, dtype=torch.int32)
    s = 0
    for i, p in enumerate(pages):
        bt[i, :p] = perm[s:s + p].to(torch.int32)
        s += p
    assert s <= num_blocks
    return bt


def run_batched(cuda_device, lens, q_len, hq, hkv, dtype, seed, d=128, bs=16, extra_blocks=8,
                poison=False):
    g = torch.Generator().manual_seed(seed)
    nb = sum((L + bs - 1) // bs for L in lens) + extra_blocks
    kc, vc, kcd, vcd = make_pool(nb, hkv, bs, d, dtype, g, cuda_device)
    if poison:
        # stale pool bytes past every sequence end must not leak into the result
        kcd.fill_(float("nan"))
        vcd.fill_(float("nan"))
    bt = random_tables(lens, bs, nb, g)
    if poison:
        for i, L in enumerate(lens):
            for p in range((L + bs - 1) // bs):
                blk = int(bt[i, p])
                n = min(bs, L - p * bs)
                kcd[blk, :, :n] = kc[blk, :, :n].to(cuda_device)
                vcd[blk, :, :n] = vc[blk, :, :n].to(cuda_device)
    cl = torch.tensor(lens, dtype=torch.int32)
    q = torch.randn(len(lens), q_len, hq, d, generator=g).to(dtype)
    out = paged_attention_batched(q.to(cuda_device), kcd, vcd, bt.to(cuda_device),
                                  cl.to(cuda_device), max_context_len=max(lens + [0]))
    torch.cuda.synchronize()
    _lib.raise_device_errors(cuda_device)
    ref = oracle.batched_paged_attention(q.float().numpy(), kc.float().numpy(),
                                         vc.float().numpy(), bt.numpy(), cl.numpy())
    return out.float().cpu().numpy(), ref


# ------------------------------------------------------------- reference unit sweep
@pytest.mark.parametrize("kv_heads,q_heads", [(2, 4), (4, 4), (2, 8)])
@pytest.mark.parametrize("seq_len", [1, 15, 16, 17, 31, 32, 33])
def test_reference_unit_sweep(cuda_device, golden, kv_heads, q_heads, seq_len):
    # reference tests/test_paged_equiv.py:71-104 (head_dim 8, fp32), inputs and outputs
    # recorded from the reference itself
    tag = f"unit_{kv_heads}_{q_heads}_{seq_len}"
    from inferd_b200.paged_cache import PagedKVCache

    cache = PagedKVCache(num_layers=1, num_blocks=16, block_size=16, num_kv_heads=kv_heads,
                         head_dim=8, dtype=torch.float32, device=cuda_device)
    cache.create_sequence(0)
    key = torch.from_numpy(golden[tag + "_key"]).to(cuda_device)
    value = torch.from_numpy(golden[tag + "_value"]).to(cuda_device)
    query = torch.from_numpy(golden[tag + "_query"]).to(cuda_device)
    cache.append_tokens(0, [key], [value])
    table = cache.block_table(0)
    assert table.cpu().numpy().tolist() == golden[tag + "_table"].tolist()
    out = paged_attention(query, cache.key_cache[0], cache.value_cache[0], table, seq_len)
    np.testing.assert_allclose(out.cpu().numpy(), golden[tag + "_sdpa"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(out.cpu().numpy(), golden[tag + "_paged"], rtol=1e-4, atol=1e-5)
    ref_path = paged_attention(query, cache.key_cache[0], cache.value_cache[0], table, seq_len,
                               backend="reference")
    np.testing.assert_allclose(ref_path.cpu().numpy(), golden[tag + "_paged"], rtol=1e-4,
                               atol=1e-5)


# ------------------------------------------------------------- config 1
def _cfg1_device(cuda_device, dtype):
    from tests.golden.make_golden import CFG1, cfg1_inputs

    inp = cfg1_inputs()
    kc = torch.from_numpy(inp["key_cache"]).to(dtype).to(cuda_device)
    vc = torch.from_numpy(inp["value_cache"]).to(dtype).to(cuda_device)
    return CFG1, inp, kc, vc


def test_cfg1_fp32_matches_reference(cuda_device, golden):
    c, inp, kc, vc = _cfg1_device(cuda_device, torch.float32)
    for b, L in enumerate(c["lens"]):
        q = torch.from_numpy(inp["query"][b]).to(cuda_device)
        out = paged_attention(q, kc, vc, torch.from_numpy(inp["tables"][b]), L)
        np.testing.assert_allclose(out.cpu().numpy(), golden[f"cfg1_out_fp32_{b}"],
                                   rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cfg1_half_within_tolerance_of_fp32_reference(cuda_device, golden, dtype):
    c, inp, kc, vc = _cfg1_device(cuda_device, dtype)
    kc32 = kc.float().cpu().numpy()
    vc32 = vc.float().cpu().numpy()
    for b, L in enumerate(c["lens"]):
        q = torch.from_numpy(inp["query"][b]).to(dtype)
        out = paged_attention(q.to(cuda_device), kc, vc, torch.from_numpy(inp["tables"][b]), L)
        ref = oracle.paged_attention(q.float().numpy(), kc32, vc32, inp["tables"][b], L)
        assert_bf16_close(out.float().cpu().numpy(), ref, f"cfg1 seq {b}")
        # tighter than the reference's own bf16 recipe is to fp32 (informational bound)
        if dtype == torch.bfloat16:
            ref_bf16_err = np.abs(golden[f"cfg1_out_bf16_{b}"] - golden[f"cfg1_out_fp32_{b}"]).max()
            ours = np.abs(out.float().cpu().numpy() - golden[f"cfg1_out_fp32_{b}"]).max()
            assert ours <= max(ref_bf16_err, 4e-3)


# ------------------------------------------------------------- batched decode
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_batched_decode_edge_lengths(cuda_device, dtype):
    lens = [0, 1, 2, 15, 16, 17, 31, 32, 33, 100, 255, 256, 257, 1000]
    out, ref = run_batched(cuda_device, lens, 1, 32, 8, dtype, seed=1)
    assert_bf16_close(out, ref, "edge lengths")
    assert np.all(out[0] == 0)  # no keys -> zeros, like the reference's empty einsum


def test_batched_decode_stale_pool_bytes_do_not_leak(cuda_device):
    lens = [1, 7, 16, 23, 300]
    out, ref = run_batched(cuda_device, lens, 1, 32, 8, torch.bfloat16, seed=2, poison=True)
    assert np.isfinite(out).all()
    assert_bf16_close(out, ref, "poisoned pool")


def test_batched_decode_uniform_lengths_config2_shape(cuda_device):
    # config-2 shape (32 q heads over 8 kv heads, head_dim 128, block 16), lengths drawn
    # uniformly from [512, 8192], 16 sequences so the oracle finishes in seconds
    rng = np.random.default_rng(5)
    lens = rng.integers(512, 8193, size=16).tolist()
    out, ref = run_batched(cuda_device, lens, 1, 32, 8, torch.bfloat16, seed=5)
    assert_bf16_close(out, ref, "config-2 shape")


def test_single_long_sequence_split_across_ctas(cuda_device):
    # one sequence of 16k keys is cut into many CTA ranges: exercises the partial merge
    out, ref = run_batched(cuda_device, [16384], 1, 32, 8, torch.bfloat16, seed=6)
    assert_bf16_close(out, ref, "long sequence")


@pytest.mark.parametrize("reserve,q_len", [(8, 1), (100, 1), (12, 4)])
def test_grid_with_reserved_sms(cuda_device, reserve, q_len):
    # a grid that leaves SMs to a collective splits the pages differently (other cut
    # segments and merges); the results stay within the same bound of the oracle
    from inferd_b200 import reserve_sms

    rng = np.random.default_rng(40 + reserve)
    lens = rng.integers(300, 6000, size=12).tolist()
    prev = reserve_sms(reserve)
    try:
        assert _lib.load().inferd_paged_attention_reserved_sms() == reserve
        out, ref = run_batched(cuda_device, lens, q_len, 32, 8, torch.bfloat16, seed=40 + reserve)
    finally:
        reserve_sms(prev)
    assert_bf16_close(out, ref, f"{reserve} SMs reserved")
    with pytest.raises(ValueError):
        reserve_sms(torch.cuda.get_device_properties(cuda_device).multi_processor_count)


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 2), (64, 8), (32, 4)])
def test_gqa_ratios(cuda_device, hq, hkv):
    lens = [5, 64, 333, 1024]
    out, ref = run_batched(cuda_device, lens, 1, hq, hkv, torch.bfloat16, seed=7)
    assert_bf16_close(out, ref, f"gqa {hq}/{hkv}")


def test_int64_block_tables_and_repeat_calls(cuda_device):
    g = torch.Generator().manual_seed(8)
    lens = [40, 700, 5]
    nb = 64
    kc, vc, kcd, vcd = make_pool(nb, 8, 16, 128, torch.bfloat16, g, cuda_device)
    bt = random_tables(lens, 16, nb, g).to(torch.int64)
    cl = torch.tensor(lens, dtype=torch.int32)
    q = torch.randn(3, 1, 32, 128, generator=g).to(torch.bfloat16)
    outs = [paged_attention_batched(q.to(cuda_device), kcd, vcd, bt.to(cuda_device),
                                    cl.to(cuda_device)) for _ in range(3)]
    torch.cuda.synchronize()
    # the ticket counters are reset by every call: repeated calls are bitwise identical
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    ref = oracle.batched_paged_attention(q.float().numpy(), kc.float().numpy(),
                                         vc.float().numpy(), bt.numpy(), cl.numpy())
    assert_bf16_close(outs[0].float().cpu().numpy(), ref, "int64 tables")


def test_workspace_shared_across_call_shapes(cuda_device):
    # one workspace serves calls of different (num_seqs, q_len) in sequence; a call's
    # partials must never land on the next call's ticket counters
    rng = np.random.default_rng(40)
    shapes = [([12000], 1), (rng.integers(600, 3000, 16).tolist(), 5),
              (rng.integers(100, 5000, 40).tolist(), 1), ([9000, 7000, 8000], 2),
              ([20000], 1)]
    for i, (lens, q_len) in enumerate(shapes):
        out, ref = run_batched(cuda_device, lens, q_len, 32, 8, torch.bfloat16, seed=40 + i)
        assert_bf16_close(out, ref, f"shape {i}")


def test_bad_block_id_raises_index_error(cuda_device):
    kb = torch.zeros(4, 8, 16, 128, dtype=torch.bfloat16, device=cuda_device)
    q = torch.zeros(32, 128, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(IndexError):
        paged_attention(q, kb, kb, torch.tensor([0, 17]), 20)


def test_argument_errors_match_reference(cuda_device):
    kb = torch.zeros(4, 8, 16, 128, dtype=torch.bfloat16, device=cuda_device)
    q = torch.zeros(32, 128, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        paged_attention(q, kb, kb, torch.tensor([0]), 20)           # table too short
    with pytest.raises(ValueError):
        paged_attention(q, kb, kb, torch.tensor([0]), -1)
    with pytest.raises(ValueError):
        paged_attention(q, kb, kb, torch.tensor([0]), 1, backend="triton")
    with pytest.raises(ValueError):
        paged_attention(q[:30], kb, kb, torch.tensor([0]), 1)       # 30 % 8 != 0


def test_out_off_device_is_rejected(cuda_device):
    # the kernel writes `out` through its raw pointer: a host tensor, even pinned, is refused
    # before anything is launched
    kb = torch.zeros(4, 2, 16, 128, dtype=torch.bfloat16, device=cuda_device)
    q = torch.zeros(1, 1, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    bt = torch.zeros(1, 1, dtype=torch.int32, device=cuda_device)
    cl = torch.ones(1, dtype=torch.int32, device=cuda_device)
    for out in (torch.empty(1, 1, 8, 128, dtype=torch.bfloat16),
                torch.empty(1, 1, 8, 128, dtype=torch.bfloat16, pin_memory=True)):
        with pytest.raises(ValueError):
            paged_attention_batched(q, kb, kb, bt, cl, out=out)


# ------------------------------------------------------------- verify (q_len > 1)
@pytest.mark.parametrize("case", range(4))
def test_verify_matches_hf_eager_golden(cuda_device, golden, case):
    hq, hkv, d, L, ql = golden["verify_cases"][case].tolist()
    q = torch.from_numpy(golden[f"verify_{case}_query"])
    k = torch.from_numpy(golden[f"verify_{case}_key"])
    v = torch.from_numpy(golden[f"verify_{case}_value"])
    ref = golden[f"verify_{case}_out"]
    # the oracle restatement agrees with HF's eager attention
    np.testing.assert_allclose(oracle.verify_attention(q.numpy(), k.numpy(), v.numpy()), ref,
                               rtol=1e-4, atol=1e-5)
    from inferd_b200.paged_cache import PagedKVCache

    for dtype in (torch.float32, torch.bfloat16):
        cache = PagedKVCache(num_layers=1, num_blocks=(L + 15) // 16 + 2, block_size=16,
                             num_kv_heads=hkv, head_dim=d, dtype=dtype, device=cuda_device)
        cache.create_sequence(0)
        cache.append_tokens(0, [k.to(dtype).to(cuda_device)], [v.to(dtype).to(cuda_device)])
        bt, cl, mx = cache.decode_metadata([0])
        out = paged_attention_batched(q.to(dtype).unsqueeze(0).to(cuda_device),
                                      cache.key_cache[0], cache.value_cache[0], bt, cl,
                                      max_context_len=mx)[0].float().cpu().numpy()
        if dtype == torch.float32:
            np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-5)
        else:
            r16 = oracle.verify_attention(q.to(dtype).float().numpy(), k.to(dtype).float().numpy(),
                                          v.to(dtype).float().numpy())
            assert_bf16_close(out, r16, f"verify case {case}")


def test_verify_config3_shape(cuda_device):
    # config-3 shape: k=4 drafts + 1 = 5 queries, 32/8 heads, lengths in [1024, 4096]
    rng = np.random.default_rng(9)
    lens = rng.integers(1024, 4097, size=8).tolist()
    out, ref = run_batched(cuda_device, lens, 5, 32, 8, torch.bfloat16, seed=9)
    assert_bf16_close(out, ref, "verify config-3 shape")


@pytest.mark.parametrize("q_len", [5, 8])
def test_verify_single_long_sequence_many_pieces(cuda_device, q_len):
    # one 20k-key sequence over all warps: each kv head's segment is cut into ~150 pieces,
    # more than one 32-piece chunk of the merge kernel; repeated calls are bitwise identical
    # (the cut markers are cleared by every call)
    out, ref = run_batched(cuda_device, [20000], q_len, 32, 8, torch.bfloat16, seed=50 + q_len)
    assert_bf16_close(out, ref, f"long verify q_len {q_len}")
    out2, _ = run_batched(cuda_device, [20000], q_len, 32, 8, torch.bfloat16, seed=50 + q_len)
    assert np.array_equal(out, out2)


@pytest.mark.parametrize("q_len", [2, 3, 4, 8])
def test_verify_window_sizes(cuda_device, q_len):
    lens = [q_len, q_len + 1, 17, 40, 513]
    out, ref = run_batched(cuda_device, lens, q_len, 32, 8, torch.bfloat16, seed=10 + q_len)
    assert_bf16_close(out, ref, f"verify q_len {q_len}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_verify_stale_pool_bytes_and_empty_sequences(cuda_device, dtype):
    # NaN in every pool byte past each sequence end (and in unused blocks) must not reach
    # the output; a sequence without keys gives zero rows
    lens = [0, 5, 16, 23, 64, 65, 300, 1000]
    out, ref = run_batched(cuda_device, lens, 5, 32, 8, dtype, seed=21, poison=True)
    assert np.isfinite(out).all()
    assert_bf16_close(out, ref, "poisoned pool, verify")
    assert np.all(out[0] == 0)


@pytest.mark.parametrize("q_len,hq,hkv", [(2, 64, 8), (4, 64, 8), (3, 24, 8), (8, 32, 8)])
def test_verify_row_counts(cuda_device, q_len, hq, hkv):
    # 16, 32, 9 and 32 query rows per kv head
    lens = [1, 9, 63, 64, 129, 2000]
    out, ref = run_batched(cuda_device, lens, q_len, hq, hkv, torch.bfloat16, seed=30 + q_len)
    assert_bf16_close(out, ref, f"q_len {q_len}, {hq}/{hkv} heads")


def test_verify_short_context_rows_are_zero(cuda_device):
    # queries whose position is negative (context shorter than the window) see no keys
    out, ref = run_batched(cuda_device, [2, 30], 5, 16, 4, torch.bfloat16, seed=20)
    assert_bf16_close(out, ref, "short context")
    assert np.all(out[0, :3] == 0)


# ------------------------------------------------------------- dense + reference backend
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_dense_attention_matches_oracle(cuda_device, dtype):
    g = torch.Generator().manual_seed(30)
    q = torch.randn(16, 64, generator=g).to(dtype)
    k = torch.randn(77, 4, 64, generator=g).to(dtype)
    v = torch.randn(77, 4, 64, generator=g).to(dtype)
    out = dense_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    ref = oracle.dense_attention(q.float().numpy(), k.float().numpy(), v.float().numpy())
    if dtype == torch.float32:
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-5)
    else:
        assert_bf16_close(out.float().cpu().numpy(), ref, "dense bf16")


def test_reference_backend_equals_fused(cuda_device):
    g = torch.Generator().manual_seed(31)
    kc, vc, kcd, vcd = make_pool(32, 8, 16, 128, torch.bfloat16, g, cuda_device)
    table = torch.randperm(32, generator=g)[:20]
    q = torch.randn(32, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    a = paged_attention(q, kcd, vcd, table, 300)
    b = paged_attention_reference(q, kcd, vcd, table, 300)
    np.testing.assert_allclose(a.float().cpu().numpy(), b.float().cpu().numpy(), atol=2e-2)
    ref = oracle.paged_attention(q.float().cpu().numpy(), kc.float().numpy(), vc.float().numpy(),
                                 table.numpy(), 300)
    assert_bf16_close(a.float().cpu().numpy(), ref, "fused")
    assert_bf16_close(b.float().cpu().numpy(), ref, "gather + dense")


def test_default_scale_is_inverse_sqrt_head_dim(cuda_device):
    g = torch.Generator().manual_seed(32)
    kc, vc, kcd, vcd = make_pool(8, 8, 16, 128, torch.bfloat16, g, cuda_device)
    q = torch.randn(32, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    table = torch.arange(8)
    a = paged_attention(q, kcd, vcd, table, 100)
    b = paged_attention(q, kcd, vcd, table, 100, scale=1.0 / math.sqrt(128))
    assert torch.equal(a, b)
