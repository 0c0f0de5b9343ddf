"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference source tree is checked out (read-only is fine), naming its root
with --reference or the INFERD_REFERENCE environment variable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <reference checkout>

It imports the reference's own core.paged_attn / core.paged_cache, the transformers
eager attention the reference's speculative verify forward runs, and torch's
float8_e4m3fn cast, runs them on seeded inputs and saves inputs (or the seeds that
regenerate them) and outputs.  The GPU box never runs this script; tests read only the
committed .npz / .json files.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# Config 1 of the benchmark definition: 4 sequences, lengths {17, 64, 129, 300}, 16 query
# heads over 4 KV heads, head_dim 128, block_size 16, pool of 128 blocks, tables drawn as
# slices of a seeded permutation of the pool.  Inputs come from numpy's PCG64 with this
# seed, so the tests regenerate them instead of storing 8 MB of pool.
CFG1_SEED = 0
CFG1 = dict(lens=[17, 64, 129, 300], q_heads=16, kv_heads=4, head_dim=128, block_size=16,
            num_blocks=128)


def cfg1_inputs(seed: int = CFG1_SEED):
    """Deterministic config-1 inputs (shared with tests/test_oracle_golden.py)."""
    rng = np.random.default_rng(seed)
    c = CFG1
    shape = (c["num_blocks"], c["kv_heads"], c["block_size"], c["head_dim"])
    key_cache = rng.standard_normal(shape, dtype=np.float32)
    value_cache = rng.standard_normal(shape, dtype=np.float32)
    perm = rng.permutation(c["num_blocks"])
    tables, start = [], 0
    for L in c["lens"]:
        n = (L + c["block_size"] - 1) // c["block_size"]
        tables.append(perm[start:start + n].astype(np.int64))
        start += n
    query = rng.standard_normal((len(c["lens"]), c["q_heads"], c["head_dim"]), dtype=np.float32)
    new_k = rng.standard_normal((len(c["lens"]), c["kv_heads"], c["head_dim"]), dtype=np.float32)
    new_v = rng.standard_normal((len(c["lens"]), c["kv_heads"], c["head_dim"]), dtype=np.float32)
    return dict(key_cache=key_cache, value_cache=value_cache, perm=perm, tables=tables,
                query=query, new_k=new_k, new_v=new_v)


def _bf16_round(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def gen_unit_sweep(pa, pc, out: dict) -> None:
    """tests/test_paged_equiv.py:71-104 of the reference, recorded case by case."""
    torch.manual_seed(0)
    lengths = [1, 15, 16, 17, 31, 32, 33]
    for kv_heads, q_heads in [(2, 4), (4, 4), (2, 8)]:
        for seq_len in lengths:
            cache = pc.PagedKVCache(num_layers=1, num_blocks=16, block_size=16,
                                    num_kv_heads=kv_heads, head_dim=8, dtype=torch.float32)
            cache.create_sequence(0)
            key = torch.randn(seq_len, kv_heads, 8)
            value = torch.randn(seq_len, kv_heads, 8)
            query = torch.randn(q_heads, 8)
            cache.append_tokens(0, [key], [value])
            table = cache.block_table(0)
            out_paged = pa.paged_attention(query, cache.key_cache[0], cache.value_cache[0],
                                           table, seq_len)
            out_sdpa = pa.sdpa_reference(query, key, value)
            tag = f"unit_{kv_heads}_{q_heads}_{seq_len}"
            out[tag + "_key"] = key.numpy()
            out[tag + "_value"] = value.numpy()
            out[tag + "_query"] = query.numpy()
            out[tag + "_table"] = table.numpy()
            out[tag + "_paged"] = out_paged.numpy()
            out[tag + "_sdpa"] = out_sdpa.numpy()


def gen_cfg1(pa, pc, out: dict) -> None:
    c = CFG1
    inp = cfg1_inputs()
    kc = torch.from_numpy(inp["key_cache"])
    vc = torch.from_numpy(inp["value_cache"])
    for b, L in enumerate(c["lens"]):
        table = torch.from_numpy(inp["tables"][b])
        q = torch.from_numpy(inp["query"][b])
        out[f"cfg1_out_fp32_{b}"] = pa.paged_attention(q, kc, vc, table, L).numpy()
        k, v = pa.gather_paged_kv(kc, vc, table, L)
        out[f"cfg1_sdpa_fp32_{b}"] = pa.sdpa_reference(q, k, v).numpy()
        # the reference's own bf16 recipe on bf16-rounded inputs (informational)
        out[f"cfg1_out_bf16_{b}"] = pa.paged_attention(
            q.to(torch.bfloat16), kc.to(torch.bfloat16), vc.to(torch.bfloat16), table, L
        ).float().numpy()

    # KV append of one token per sequence at slot L_i through the reference cache, with
    # the pool pre-filled and the page tables set to the permuted tables.
    cache = pc.PagedKVCache(num_layers=1, num_blocks=c["num_blocks"], block_size=c["block_size"],
                            num_kv_heads=c["kv_heads"], head_dim=c["head_dim"], dtype=torch.float32)
    cache.key_cache[0] = kc.clone()
    cache.value_cache[0] = vc.clone()
    used = set()
    for b, L in enumerate(c["lens"]):
        t = cache.create_sequence(b)
        t.blocks = [int(x) for x in inp["tables"][b]]
        t.length = L
        used.update(t.blocks)
    cache.allocator._allocated = set(used)
    cache.allocator._free = [x for x in cache.allocator._free if x not in used]
    for b in range(len(c["lens"])):
        cache.append_tokens(b, [torch.from_numpy(inp["new_k"][b:b + 1])],
                            [torch.from_numpy(inp["new_v"][b:b + 1])])
    cache.assert_consistent()
    slots = []
    tables_after = np.full((len(c["lens"]), 32), -1, dtype=np.int64)
    for b, L in enumerate(c["lens"]):
        blk, off = cache.sequences[b].block_for_pos(L)
        slots.append(blk * c["block_size"] + off)
        bl = cache.sequences[b].blocks
        tables_after[b, :len(bl)] = bl
        assert torch.equal(cache.key_cache[0][blk, :, off, :], torch.from_numpy(inp["new_k"][b]))
    out["cfg1_append_slots"] = np.array(slots, dtype=np.int64)
    out["cfg1_tables_after"] = tables_after
    # checksum of the reference pool after the append (bit pattern of float32)
    out["cfg1_pool_k_after_sum"] = np.array(
        [cache.key_cache[0].numpy().view(np.uint32).astype(np.uint64).sum()], dtype=np.uint64)
    out["cfg1_pool_v_after_sum"] = np.array(
        [cache.value_cache[0].numpy().view(np.uint32).astype(np.uint64).sum()], dtype=np.uint64)


def gen_verify(out: dict) -> None:
    """HF eager attention with the causal verify mask (the path core/spec_decode.py:135
    reaches through the target model)."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import eager_attention_forward

    cases = [(8, 2, 16, 37, 5), (4, 4, 8, 5, 5), (32, 8, 128, 100, 5), (16, 4, 128, 21, 3)]
    g = torch.Generator().manual_seed(1)
    for i, (hq, hkv, d, L, ql) in enumerate(cases):
        q = torch.randn(1, hq, ql, d, generator=g)
        k = torch.randn(1, hkv, L, d, generator=g)
        v = torch.randn(1, hkv, L, d, generator=g)
        mask = torch.zeros(1, 1, ql, L)
        for qi in range(ql):
            mask[0, 0, qi, L - ql + qi + 1:] = torch.finfo(torch.float32).min
        module = types.SimpleNamespace(num_key_value_groups=hq // hkv, training=False)
        o, _ = eager_attention_forward(module, q, k, v, mask, 1.0 / math.sqrt(d))
        tag = f"verify_{i}"
        out[tag + "_query"] = q[0].transpose(0, 1).contiguous().numpy()   # [ql, hq, d]
        out[tag + "_key"] = k[0].transpose(0, 1).contiguous().numpy()     # [L, hkv, d]
        out[tag + "_value"] = v[0].transpose(0, 1).contiguous().numpy()
        out[tag + "_out"] = o[0].numpy()                                  # [ql, hq, d]
    out["verify_cases"] = np.array(cases, dtype=np.int64)


def gen_fp8(out: dict) -> None:
    g = torch.Generator().manual_seed(2)
    w = (torch.randn(48, 160, generator=g) * 0.02).to(torch.bfloat16)
    w[5] = 0.0  # an all-zero output channel
    amax = w.float().abs().amax(dim=1)
    s = amax / 448.0
    s = torch.where(s > 0, s, torch.ones_like(s))
    q = (w.float() / s[:, None]).to(torch.float8_e4m3fn)
    x = torch.randn(3, 160, generator=g).to(torch.bfloat16)
    y = x.double() @ (q.double() * s.double()[:, None]).T
    out["fp8_w"] = w.float().numpy()
    out["fp8_scale"] = s.numpy()
    out["fp8_q"] = q.view(torch.uint8).numpy()
    out["fp8_x"] = x.float().numpy()
    out["fp8_y"] = y.numpy()
    out["fp8_y_bf16"] = y.to(torch.bfloat16).float().numpy()
    # e4m3 encoder edge cases: ties, subnormals, powers of two, saturation boundary
    vals = [0.0, -0.0, 2 ** -10, 1.5 * 2 ** -9, 2.5 * 2 ** -9, 2 ** -9, 2 ** -6, 7 * 2 ** -9,
            7.5 * 2 ** -9, 1.0, 1.0625, 1.1875, 1.5, 15.5, 240.0, 248.0, 256.0, 272.0, 288.0,
            416.0, 432.0, 440.0, 448.0, 455.0, -448.0, -3.3, 0.0123, 100.7, -2 ** -8]
    vals += list(torch.randn(200, generator=g).mul(50).tolist())
    t = torch.tensor(vals, dtype=torch.float32)
    t = t.clamp(-448.0, 448.0)
    out["e4m3_in"] = t.numpy()
    out["e4m3_code"] = t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    out["e4m3_all_codes_value"] = torch.arange(256, dtype=torch.uint8).view(
        torch.float8_e4m3fn).float().numpy()


# decode-step sampling: (vocab, temperature, top_p, rows) cases for the reference's
# nucleus_probs (core/spec_decode.py:14-31) on seeded N(0, 3^2) float32 logits
SAMPLING_SEED = 11
SAMPLING_CASES = [
    (4096, 1.0, 1.0, 1), (4096, 0.7, 0.9, 1), (4096, 1.3, 0.5, 1), (4096, 0.7, 0.05, 1),
    (4096, 0.0, 0.9, 1), (1000, 1.0, 0.95, 4), (32000, 0.7, 0.9, 1), (32000, 1.0, 0.99, 1),
    (7, 0.5, 0.3, 3),
]


def gen_sampling(out: dict) -> None:
    """Outputs of the reference's own nucleus_probs.  core/spec_decode.py imports its
    package's CUDA-library bootstrap (inferd.env) first; that module is stubbed here, so
    only the sampling code runs."""
    for name in ("inferd", "inferd.env"):
        sys.modules.setdefault(name, types.ModuleType(name))
    from core.spec_decode import nucleus_probs  # noqa: E402  (reference module)

    rng = np.random.default_rng(SAMPLING_SEED)
    for i, (v, t, p, rows) in enumerate(SAMPLING_CASES):
        logits = (rng.standard_normal((rows, v), dtype=np.float32) * np.float32(3.0)).astype(np.float32)
        probs = nucleus_probs(torch.from_numpy(logits.copy()), t, p)
        out[f"samp_{i}_logits"] = logits
        out[f"samp_{i}_probs"] = probs.numpy().astype(np.float32)
    # the reference's own selfcheck logits (core/spec_decode.py:182-187)
    sc = torch.tensor([[10.0, 9.0, 1.0, -5.0]])
    out["samp_selfcheck_logits"] = sc.numpy()
    out["samp_selfcheck_p_1"] = nucleus_probs(sc, 1.0, 1.0).numpy()
    out["samp_selfcheck_p_05"] = nucleus_probs(sc, 1.0, 0.5).numpy()


def gen_cache_trace(pc) -> dict:
    """Allocator / page-table behaviour of the reference cache under a scripted trace."""
    trace: dict = {}
    # reference tests/test_paged_equiv.py:106-125
    cache = pc.PagedKVCache(num_layers=1, num_blocks=4, block_size=2, num_kv_heads=1,
                            head_dim=1, dtype=torch.float32)
    cache.create_sequence(1)
    cache.create_sequence(2)
    one = [torch.ones(3, 1, 1)]
    cache.append_tokens(1, one, one)
    first = list(cache.sequences[1].blocks)
    cache.free_sequence(1)
    cache.append_tokens(2, one, one)
    trace["reuse"] = {"first": first, "second": list(cache.sequences[2].blocks)}

    # random trace
    rng = random.Random(3)
    cache = pc.PagedKVCache(num_layers=2, num_blocks=24, block_size=4, num_kv_heads=1,
                            head_dim=2, dtype=torch.float32)
    ops = []
    live: list[int] = []
    next_id = 0
    for _ in range(120):
        r = rng.random()
        if r < 0.25 or not live:
            cache.create_sequence(next_id)
            live.append(next_id)
            ops.append({"op": "create", "seq": next_id})
            next_id += 1
        elif r < 0.8:
            sid = rng.choice(live)
            n = rng.randint(0, 9)
            kv = [torch.zeros(n, 1, 2) for _ in range(2)]
            try:
                cache.append_tokens(sid, kv, kv)
                res = "ok"
            except MemoryError:
                res = "MemoryError"
            ops.append({"op": "append", "seq": sid, "n": n, "result": res,
                        "blocks": list(cache.sequences[sid].blocks),
                        "length": cache.sequences[sid].length,
                        "free": cache.allocator.free_count})
        else:
            sid = rng.choice(live)
            live.remove(sid)
            cache.free_sequence(sid)
            ops.append({"op": "free", "seq": sid, "free": cache.allocator.free_count})
        cache.assert_consistent()
    trace["ops"] = ops
    trace["block_size"] = 4
    trace["num_blocks"] = 24
    return trace


def _torchao_dynamic_quant(t: torch.Tensor, per_row: bool):
    """torchao 0.17.0's dynamic float8 scaling restated with the torch ops it calls
    (_choose_scale_float8 then _quantize_affine_float8): amax of |t| (per tensor or per
    row), s = amax / 448 in fp32, q = clamp(t.float() / s, -448, 448) cast to e4m3."""
    amax = t.abs().amax(dim=1, keepdim=True) if per_row else t.abs().amax()
    s = amax.float() / torch.finfo(torch.float8_e4m3fn).max
    q = (t.float() / s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q, s


def gen_fp8_dynamic(out: dict) -> None:
    """The fp8-dynamic recipe (bench/model_loader.py:53-55): weights and activations
    quantised with torchao's dynamic scaling; per tensor (torchao's default) the product
    comes from torch._scaled_mm itself, per row from the same formula in float64 (CPU
    _scaled_mm takes per-tensor scales only)."""
    g = torch.Generator().manual_seed(4)
    cases = [("tensor", 5, 96, 320), ("row", 4, 64, 256), ("tensor", 17, 48, 128)]
    for i, (gran, m, n, k) in enumerate(cases):
        per_row = gran == "row"
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        x[0, 3] = 30.0  # an outlier sets the tensor's scale
        if per_row:
            w[7] = 0.0
            x[1, 5:9] = torch.tensor([1e-3, -2e-3, 5e-4, 0.0]).to(torch.bfloat16)
        qw, sw = _torchao_dynamic_quant(w, per_row)
        qx, sx = _torchao_dynamic_quant(x, per_row)
        if per_row:
            y = ((qx.double() @ qw.double().T) * sx.double() * sw.double().T).to(torch.bfloat16)
        else:
            y = torch._scaled_mm(qx, qw.t(), scale_a=sx, scale_b=sw, out_dtype=torch.bfloat16)
        tag = f"dyn_{i}"
        out[tag + "_w"] = w.float().numpy()
        out[tag + "_x"] = x.float().numpy()
        out[tag + "_qw"] = qw.view(torch.uint8).numpy()
        out[tag + "_sw"] = sw.reshape(-1).numpy()
        out[tag + "_qx"] = qx.view(torch.uint8).numpy()
        out[tag + "_sx"] = sx.reshape(-1).numpy()
        out[tag + "_y"] = y.float().numpy()
    out["dyn_cases"] = np.array([[0 if c[0] == "tensor" else 1, c[1], c[2], c[3]] for c in cases], dtype=np.int64)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("INFERD_REFERENCE"),
                    help="root of the reference checkout (default: $INFERD_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or INFERD_REFERENCE")
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    import core.paged_attn as pa  # noqa: E402  (reference module)
    import core.paged_cache as pc  # noqa: E402  (reference module)

    out: dict = {}
    gen_unit_sweep(pa, pc, out)
    gen_cfg1(pa, pc, out)
    gen_verify(out)
    gen_fp8(out)
    np.savez_compressed(HERE / "reference_golden.npz", **out)
    dyn: dict = {}
    gen_fp8_dynamic(dyn)
    np.savez_compressed(HERE / "fp8_dynamic_golden.npz", **dyn)
    samp: dict = {}
    gen_sampling(samp)
    np.savez_compressed(HERE / "sampling_golden.npz", **samp)
    trace = gen_cache_trace(pc)
    (HERE / "cache_trace.json").write_text(json.dumps(trace, indent=0))
    print(f"wrote {len(out)} arrays and {len(trace['ops'])} trace ops")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
