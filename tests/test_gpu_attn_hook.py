"""The HF attention hook's own routes (core/paged_attn_interface.py:25-75), called directly
and inside a tiny random-init Qwen3.5.

* b == 1, q_len == 1 (the reference's route): paged_ref_attention_forward against
  transformers' eager_attention_forward on the same tensors;
* "batched_decode" (b > 1, q_len == 1) with left-padded rows, the mask given as HF's 4-D
  additive float mask or as a boolean mask;
* "verify" (b == 1, q_len = k + 1, causal over the cached prefix).

Attention tolerances are the paged-attention ones: fp32 at rtol 1e-4 / atol 1e-5 (the
reference's own test tolerance, tests/test_paged_equiv.py:104 of the reference); bf16
within 2e-2 max-abs and 1e-2 relative of the fp32 computation on the same bf16 inputs.

At model level two runs of the same bf16 model differ only in their attention function,
and rounding differences grow through the layers, so a fixed logits tolerance says little.
There the bound is relative to HF's own bf16 error: the hooked bf16 model must be no further
from the fp32 model (same bf16-rounded weights) than stock bf16 eager is, within 25 %.
"""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

m = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")

ATOL_BF16, RTOL_BF16 = 2e-2, 1e-2


class _Module(torch.nn.Module):
    """The attributes eager_attention_forward reads from its attention module."""

    def __init__(self, groups: int) -> None:
        super().__init__()
        self.num_key_value_groups = groups
        self.eval()


def _eager(module, q, k, v, mask, scaling):
    """transformers' own eager attention in fp32 on the CPU (the function install() wraps)."""
    from inferd_b200 import paged_attn_interface as pai

    real = pai._real_eager or m.eager_attention_forward
    out, _ = real(module, q.float().cpu(), k.float().cpu(), v.float().cpu(),
                  None if mask is None else mask.float().cpu(), scaling)
    return out


def _close(out: torch.Tensor, ref: torch.Tensor, dtype, what: str) -> None:
    out, ref = out.float().cpu(), ref.float().cpu()
    if dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5, msg=what)
        return
    err = float((out - ref).abs().max())
    scale = float(ref.abs().max())
    assert err <= ATOL_BF16, f"{what}: max abs error {err}"
    assert err <= RTOL_BF16 * max(scale, 1e-6), f"{what}: relative error {err / scale}"


@pytest.fixture
def hook():
    from inferd_b200 import paged_attn_interface as pai

    pai.uninstall()
    yield pai
    pai.uninstall()
    pai._routes = frozenset({"decode"})


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("kv_len", [1, 16, 17, 300, 2049])
def test_reference_route_b1_q1_matches_eager(cuda_device, hook, dtype, kv_len):
    g = torch.Generator().manual_seed(kv_len)
    hq, hkv, d = 32, 8, 128
    q = torch.randn(1, hq, 1, d, generator=g).to(dtype)
    k = torch.randn(1, hkv, kv_len, d, generator=g).to(dtype)
    v = torch.randn(1, hkv, kv_len, d, generator=g).to(dtype)
    mod = _Module(hq // hkv)
    scaling = 1.0 / math.sqrt(d)
    out, weights = hook.paged_ref_attention_forward(
        mod, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, scaling)
    assert weights is None and out.shape == (1, 1, hq, d) and out.dtype == dtype
    _close(out, _eager(mod, q, k, v, None, scaling), dtype, f"b=1 q=1 L={kv_len}")


def _left_padded(lengths, kv_len, hq, hkv, d, dtype, seed):
    """Keys of unequal length, left-padded to kv_len, and HF's masks for the last query."""
    g = torch.Generator().manual_seed(seed)
    b = len(lengths)
    q = torch.randn(b, hq, 1, d, generator=g).to(dtype)
    k = torch.randn(b, hkv, kv_len, d, generator=g).to(dtype)
    v = torch.randn(b, hkv, kv_len, d, generator=g).to(dtype)
    visible = torch.zeros(b, 1, 1, kv_len, dtype=torch.bool)
    for i, n in enumerate(lengths):
        visible[i, 0, 0, kv_len - n:] = True
    additive = torch.zeros(b, 1, 1, kv_len, dtype=torch.float32)
    additive.masked_fill_(~visible, torch.finfo(torch.float32).min)
    return q, k, v, visible, additive


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("mask_kind", ["additive", "bool"])
def test_batched_decode_route_left_padded_rows(cuda_device, hook, dtype, mask_kind):
    lengths = [5, 17, 33, 100, 1, 64]
    kv_len, hq, hkv, d = 100, 32, 8, 128
    q, k, v, visible, additive = _left_padded(lengths, kv_len, hq, hkv, d, dtype, seed=11)
    mod = _Module(hq // hkv)
    scaling = 1.0 / math.sqrt(d)
    hook.install(routes=("batched_decode",))
    mask = additive if mask_kind == "additive" else visible
    dev_mask = mask.to(cuda_device) if mask_kind == "bool" else mask.to(dtype).to(cuda_device)
    assert hook._row_lengths(dev_mask, len(lengths), kv_len) == lengths
    out, _ = hook.paged_ref_attention_forward(
        mod, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), dev_mask, scaling)
    assert out.shape == (len(lengths), 1, hq, d)
    _close(out, _eager(mod, q, k, v, additive, scaling), dtype, f"batched decode {mask_kind}")
    # through the installed wrapper too (what the HF layers call)
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mm

    out2, _ = mm.eager_attention_forward(
        mod, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), dev_mask, scaling)
    assert torch.equal(out2, out)


def test_batched_decode_needs_its_route(cuda_device, hook):
    # without the route, b > 1 goes to the real eager function (the reference's behaviour)
    lengths = [3, 9]
    q, k, v, _, additive = _left_padded(lengths, 9, 8, 2, 128, torch.float32, seed=3)
    mod = _Module(4)
    hook.install()
    out, weights = hook.paged_ref_attention_forward(
        mod, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), additive.to(cuda_device), 0.1)
    assert weights is not None  # eager returns its attention weights; the paged routes None
    torch.testing.assert_close(out.cpu(), _eager(mod, q, k, v, additive, 0.1), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("q_len,prefix", [(2, 40), (5, 1000), (8, 16)])
def test_verify_route_causal_window(cuda_device, hook, dtype, q_len, prefix):
    g = torch.Generator().manual_seed(q_len * 1000 + prefix)
    hq, hkv, d = 16, 4, 128
    kv_len = prefix + q_len
    q = torch.randn(1, hq, q_len, d, generator=g).to(dtype)
    k = torch.randn(1, hkv, kv_len, d, generator=g).to(dtype)
    v = torch.randn(1, hkv, kv_len, d, generator=g).to(dtype)
    # HF's causal mask for a window at positions prefix .. prefix + q_len - 1
    pos_q = torch.arange(prefix, kv_len)[:, None]
    pos_k = torch.arange(kv_len)[None, :]
    causal = torch.zeros(1, 1, q_len, kv_len)
    causal.masked_fill_(pos_k > pos_q, torch.finfo(torch.float32).min)
    mod = _Module(hq // hkv)
    scaling = 1.0 / math.sqrt(d)
    hook.install(routes=("verify",))
    out, weights = hook.paged_ref_attention_forward(
        mod, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
        causal.to(dtype).to(cuda_device), scaling)
    assert weights is None and out.shape == (1, q_len, hq, d)
    _close(out, _eager(mod, q, k, v, causal, scaling), dtype, f"verify q_len={q_len}")


# ------------------------------------------------------------------ model level
def _model(dtype, device):
    torch.manual_seed(0)
    cfg = m.Qwen3_5TextConfig(
        vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
        num_attention_heads=8, num_key_value_heads=2, head_dim=128, linear_num_key_heads=2,
        linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
        layer_types=["linear_attention", "full_attention", "linear_attention", "full_attention"])
    cfg._attn_implementation = "eager"
    model = m.Qwen3_5ForCausalLM(cfg).to(torch.bfloat16)  # bf16-rounded weights for every run
    return model.to(device=device, dtype=dtype).eval()


def _decode_logits(model, prompts, steps, device):
    """Left-padded batched greedy decode through HF's own cache: logits of every step."""
    from transformers import DynamicCache

    b = len(prompts)
    width = max(len(p) for p in prompts)
    ids = torch.zeros(b, width, dtype=torch.long)
    mask = torch.zeros(b, width, dtype=torch.long)
    for i, p in enumerate(prompts):
        ids[i, width - len(p):] = torch.tensor(p)
        mask[i, width - len(p):] = 1
    ids, mask = ids.to(device), mask.to(device)
    pos = (mask.cumsum(-1) - 1).clamp(min=0)
    kv = DynamicCache(config=model.config)
    out = []
    with torch.no_grad():
        lg = model(ids, attention_mask=mask, position_ids=pos, past_key_values=kv,
                   use_cache=True).logits[:, -1]
        out.append(lg.float().cpu())
        tok = torch.tensor([[7], [11], [13]][:b], device=device)
        for _ in range(steps):
            mask = torch.cat([mask, torch.ones(b, 1, dtype=mask.dtype, device=device)], dim=1)
            pos = pos[:, -1:] + 1
            lg = model(tok, attention_mask=mask, position_ids=pos, past_key_values=kv,
                       use_cache=True).logits[:, -1]
            out.append(lg.float().cpu())
            tok = (tok * 5 + 3) % 500
    return torch.stack(out)


def test_model_batched_decode_route_left_padded(cuda_device, hook):
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 23, 40)]
    steps = 6
    f32 = _model(torch.float32, cuda_device)
    bf16 = _model(torch.bfloat16, cuda_device)
    truth = _decode_logits(f32, prompts, steps, cuda_device)
    stock = _decode_logits(bf16, prompts, steps, cuda_device)
    hook.install(routes=("batched_decode",))
    ours32 = _decode_logits(f32, prompts, steps, cuda_device)
    ours = _decode_logits(bf16, prompts, steps, cuda_device)
    # fp32: the paged kernels reproduce eager up to summation order
    assert float((ours32 - truth).abs().max()) < 2e-3
    # bf16: no further from the fp32 model than HF's own bf16 eager path
    err_ours = float((ours - truth).abs().max())
    err_stock = float((stock - truth).abs().max())
    assert err_ours <= 1.25 * err_stock + 1e-3, (err_ours, err_stock)


def test_model_verify_route_window(cuda_device, hook):
    from transformers import DynamicCache

    g = torch.Generator().manual_seed(22)
    prompt = torch.randint(0, 512, (37,), generator=g).tolist()
    window = torch.randint(0, 512, (5,), generator=g).tolist()

    def run(model):
        kv = DynamicCache(config=model.config)
        with torch.no_grad():
            model(torch.tensor([prompt], device=cuda_device), past_key_values=kv, use_cache=True)
            return model(torch.tensor([window], device=cuda_device), past_key_values=kv,
                         use_cache=True).logits[0].float().cpu()

    f32 = _model(torch.float32, cuda_device)
    truth = run(f32)
    bf16 = _model(torch.bfloat16, cuda_device)
    stock = run(bf16)
    hook.install(routes=("verify",))
    ours32 = run(f32)
    ours = run(bf16)
    assert float((ours32 - truth).abs().max()) < 2e-3
    err_ours = float((ours - truth).abs().max())
    err_stock = float((stock - truth).abs().max())
    assert err_ours <= 1.25 * err_stock + 1e-3, (err_ours, err_stock)
