"""FP8 (e4m3) linears on tcgen05 tensor cores (drop-in for the reference's load-time
torchao quantisation, bench/model_loader.py:46-58 and :82-88), both of its recipes:

"fp8" -- Float8WeightOnlyConfig: e4m3 weights, bf16 activations.

    q, s = quantize_fp8_per_channel(weight)        # load time, per output channel
    y = fp8_linear(x, q, s)                        # every forward: y = x @ (q * s)^T

  Inside the kernel the activations are split exactly into two e4m3 planes so the FP8
  tensor pipe can be used without the ~3 % error of a single e4m3 copy.

"fp8-dynamic" -- Float8DynamicActivationFloat8WeightConfig (PerTensor by default, PerRow
optional): weights and, on every forward, activations quantised to e4m3 with
s = amax / 448; y = s_x * s_w * (q_x @ q_w^T) -- one e4m3 plane, half the tensor work.

    q, s = quantize_fp8_dynamic(weight)            # load time, per tensor
    y = fp8_dynamic_linear(x, q, s)

    quantize_model_fp8(model, recipe="fp8" | "fp8-dynamic", modules_to_not_convert=("lm_head",))

The reference keeps lm_head in bf16 (`modules_to_not_convert=["lm_head"]`); the model
helper does the same by default.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib

E4M3_MAX = 448.0
RECIPES = ("fp8", "fp8-dynamic")
GRANULARITY = {"tensor": 0, "row": 1}  # torchao PerTensor() / PerRow()


def quantize_fp8_per_channel(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """W [N, K] (bf16 / fp16 / fp32, CUDA) -> (q float8_e4m3fn [N, K], s float32 [N]).

    s[n] = max_k |W[n, k]| / 448 (1 for an all-zero row), q = e4m3(W / s) rounded to
    nearest even -- the same bits torch's float8_e4m3fn cast produces for W.float() / s.
    """
    if weight.ndim != 2:
        raise ValueError("weight must be [out_features, in_features]")
    dev = _lib.require_cuda(weight)
    w = weight if weight.is_contiguous() else weight.contiguous()
    n, k = w.shape
    q = torch.empty((n, k), dtype=torch.uint8, device=dev)
    s = torch.empty((n,), dtype=torch.float32, device=dev)
    lib = _lib.load()
    st = lib.inferd_fp8_quantize_per_channel(w.data_ptr(), _lib.dtype_code(w.dtype), q.data_ptr(),
                                             s.data_ptr(), n, k, _lib.stream_of(dev))
    _lib.check(st, "fp8_quantize_per_channel")
    return q.view(torch.float8_e4m3fn), s


def pack_fp8_weight(w_e4m3: torch.Tensor) -> torch.Tensor:
    """Row-major e4m3 [N, K] -> the packed tile layout fp8_linear streams fastest (uint8).

    Every 128-row x 128-byte tile becomes one contiguous 16 KiB block in the MMA's
    128-byte-swizzled shared-memory form; done once at load time.
    """
    if w_e4m3.ndim != 2:
        raise ValueError("weight must be [N, K]")
    dev = _lib.require_cuda(w_e4m3)
    q = w_e4m3.contiguous().view(torch.uint8)
    n, k = q.shape
    lib = _lib.load()
    packed = torch.empty(lib.inferd_fp8_packed_weight_bytes(n, k), dtype=torch.uint8, device=dev)
    _lib.check(lib.inferd_fp8_pack_weights(q.data_ptr(), packed.data_ptr(), n, k, _lib.stream_of(dev)),
               "fp8_pack_weights")
    return packed


_WS: dict[int, torch.Tensor] = {}


def _workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None or ws.numel() < nbytes:
        # zeroed: the tile tickets at its head must start at zero (calls leave them zero)
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WS[idx] = ws
    return ws


def _granularity(granularity: str) -> int:
    try:
        return GRANULARITY[granularity]
    except KeyError:
        raise ValueError(f"granularity must be one of {sorted(GRANULARITY)}, got {granularity!r}") from None


def quantize_fp8_dynamic(x: torch.Tensor, granularity: str = "tensor") -> tuple[torch.Tensor, torch.Tensor]:
    """x [rows, K] (bf16 / fp16 / fp32, CUDA) -> (q float8_e4m3fn [rows, K], s float32 [rows]).

    torchao's dynamic float8 scaling: s = amax / 448 over the whole tensor ("tensor", every
    entry of s the same) or per row ("row"), 1 when amax is 0; q = e4m3(x / s), saturating.
    Load time for the weights of the fp8-dynamic recipe; fp8_dynamic_linear applies the
    same rule to the activations of every forward."""
    if x.ndim != 2:
        raise ValueError("expected a [rows, K] tensor")
    g = _granularity(granularity)
    dev = _lib.require_cuda(x)
    xc = x if x.is_contiguous() else x.contiguous()
    rows, k = xc.shape
    q = torch.empty((rows, k), dtype=torch.uint8, device=dev)
    s = torch.empty((rows,), dtype=torch.float32, device=dev)
    scratch = torch.empty((max(rows, 1),), dtype=torch.float32, device=dev) if g == 0 else None
    lib = _lib.load()
    st = lib.inferd_fp8_quantize_dynamic(xc.data_ptr(), _lib.dtype_code(xc.dtype), q.data_ptr(), s.data_ptr(),
                                         rows, k, g, _lib.ptr(scratch), _lib.stream_of(dev))
    _lib.check(st, "fp8_quantize_dynamic")
    return q.view(torch.float8_e4m3fn), s


def _linear_args(x, w_e4m3, w_scale, packed_shape, name):
    if x.dtype != torch.bfloat16:
        raise ValueError(f"{name} takes bf16 activations")
    if packed_shape is not None:
        n, k = packed_shape
        layout = 1
    else:
        if w_e4m3.ndim != 2:
            raise ValueError("w_e4m3 must be [N, K]")
        n, k = w_e4m3.shape
        layout = 0
    if w_scale.ndim != 1 or w_scale.shape[0] != n:
        raise ValueError("w_scale must be [N]")
    if x.shape[-1] != k:
        raise ValueError(f"x has {x.shape[-1]} features, weight expects {k}")
    if w_scale.dtype != torch.float32:
        raise ValueError("w_scale must be float32")
    dev = _lib.require_cuda(x, w_e4m3, w_scale)
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous() if x2.data_ptr() % 16 == 0 else x2.clone()
    return dev, x2, n, k, layout


def _out_view(out: torch.Tensor, dev: torch.device, m: int, n: int, what: str) -> torch.Tensor:
    """out as the kernel's [m, n] bf16 output: contiguous, bf16, m * n elements, on dev."""
    _lib.check_out(out, dev, what)
    if out.dtype != torch.bfloat16 or out.numel() != m * n or not out.is_contiguous():
        raise ValueError(f"{what}: out must be a contiguous bf16 tensor of {m} x {n} elements")
    return out.view(m, n)


def fp8_dynamic_linear(x: torch.Tensor, w_e4m3: torch.Tensor, w_scale: torch.Tensor,
                       bias: torch.Tensor | None = None, *, granularity: str = "tensor",
                       out: torch.Tensor | None = None,
                       packed_shape: tuple[int, int] | None = None) -> torch.Tensor:
    """y = s_x * (q_x @ (w_e4m3 * w_scale[:, None])^T) (+ bias), bf16 in and out, with
    (q_x, s_x) = quantize_fp8_dynamic(x, granularity) computed on the fly (torchao's
    Float8DynamicActivationFloat8WeightConfig forward: scaled e4m3 x e4m3 matmul, fp32
    accumulation, output in the activations' dtype).  Weights as for fp8_linear."""
    g = _granularity(granularity)
    dev, x2, n, k, layout = _linear_args(x, w_e4m3, w_scale, packed_shape, "fp8_dynamic_linear")
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=torch.bfloat16, device=dev) if out is None else _out_view(out, dev, m, n, "fp8_dynamic_linear")
    if m:
        lib = _lib.load()
        ws = _workspace(dev, lib.inferd_fp8_linear_workspace_bytes(m, n, k, dev.index or 0))
        w = w_e4m3 if w_e4m3.is_contiguous() else w_e4m3.contiguous()
        st = lib.inferd_fp8_dynamic_linear(y.data_ptr(), x2.data_ptr(), w.data_ptr(), w_scale.data_ptr(),
                                           m, n, k, layout, g, ws.data_ptr(), ws.numel(), _lib.stream_of(dev))
        _lib.check(st, "fp8_dynamic_linear")
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y.view(*x.shape[:-1], n)


def fp8_linear(x: torch.Tensor, w_e4m3: torch.Tensor, w_scale: torch.Tensor,
               bias: torch.Tensor | None = None, *, out: torch.Tensor | None = None,
               packed_shape: tuple[int, int] | None = None) -> torch.Tensor:
    """y = x @ (w_e4m3 * w_scale[:, None])^T (+ bias), bf16 in and out.

    x [..., K] bf16, w_scale [N] fp32.  w_e4m3 is either the row-major codes [N, K]
    (float8_e4m3fn or uint8) or, with packed_shape=(N, K), the buffer from pack_fp8_weight.
    """
    dev, x2, n, k, layout = _linear_args(x, w_e4m3, w_scale, packed_shape, "fp8_linear")
    m = x2.shape[0]
    if out is None:
        y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    else:
        y = _out_view(out, dev, m, n, "fp8_linear")
    if m:
        lib = _lib.load()
        ws_bytes = lib.inferd_fp8_linear_workspace_bytes(m, n, k, dev.index or 0)
        ws = _workspace(dev, ws_bytes)
        w = w_e4m3 if w_e4m3.is_contiguous() else w_e4m3.contiguous()
        st = lib.inferd_fp8_linear(y.data_ptr(), x2.data_ptr(), w.data_ptr(), w_scale.data_ptr(),
                                   m, n, k, layout, ws.data_ptr(), ws.numel(), _lib.stream_of(dev))
        _lib.check(st, "fp8_linear")
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y.view(*x.shape[:-1], n)


class Fp8Linear(nn.Module):
    """nn.Linear replacement holding e4m3 weights (packed tile layout) and per-channel
    fp32 scales."""

    def __init__(self, w_e4m3: torch.Tensor, w_scale: torch.Tensor,
                 bias: torch.Tensor | None = None) -> None:
        super().__init__()
        self.out_features, self.in_features = w_e4m3.shape
        self.register_buffer("weight_packed", pack_fp8_weight(w_e4m3))
        self.register_buffer("weight_scale", w_scale)
        if bias is not None:
            self.register_buffer("bias", bias.to(torch.bfloat16))
        else:
            self.bias = None

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "Fp8Linear":
        q, s = quantize_fp8_per_channel(linear.weight.detach())
        return cls(q, s, None if linear.bias is None else linear.bias.detach())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fp8_linear(x.to(torch.bfloat16), self.weight_packed, self.weight_scale, self.bias,
                          packed_shape=(self.out_features, self.in_features))

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, e4m3 weight-only"


class Fp8DynamicLinear(nn.Module):
    """nn.Linear replacement for the fp8-dynamic recipe: e4m3 weights (packed tile layout)
    with a per-tensor (or per-row) scale, activations quantised on every forward."""

    def __init__(self, w_e4m3: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None = None,
                 granularity: str = "tensor") -> None:
        super().__init__()
        _granularity(granularity)
        self.granularity = granularity
        self.out_features, self.in_features = w_e4m3.shape
        self.register_buffer("weight_packed", pack_fp8_weight(w_e4m3))
        self.register_buffer("weight_scale", w_scale)
        if bias is not None:
            self.register_buffer("bias", bias.to(torch.bfloat16))
        else:
            self.bias = None

    @classmethod
    def from_linear(cls, linear: nn.Linear, granularity: str = "tensor") -> "Fp8DynamicLinear":
        q, s = quantize_fp8_dynamic(linear.weight.detach(), granularity)
        return cls(q, s, None if linear.bias is None else linear.bias.detach(), granularity)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fp8_dynamic_linear(x.to(torch.bfloat16), self.weight_packed, self.weight_scale, self.bias,
                                  granularity=self.granularity,
                                  packed_shape=(self.out_features, self.in_features))

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"e4m3 weights and dynamic e4m3 activations (per {self.granularity})")


def quantize_model_fp8(model: nn.Module, modules_to_not_convert=("lm_head",), *, recipe: str = "fp8",
                       granularity: str = "tensor") -> nn.Module:
    """Swap every nn.Linear of `model` (except names ending in modules_to_not_convert) for
    an Fp8Linear (recipe "fp8") or an Fp8DynamicLinear (recipe "fp8-dynamic"), as
    TorchAoConfig(Float8WeightOnlyConfig() / Float8DynamicActivationFloat8WeightConfig(),
    modules_to_not_convert=["lm_head"]) does at load time in the reference
    (bench/model_loader.py:46-58, :82-88).  An unknown recipe is a ValueError, as there."""
    if recipe not in RECIPES:
        raise ValueError(f"unknown fp8 recipe {recipe!r}")
    if recipe == "fp8-dynamic":
        _granularity(granularity)
    skip = tuple(modules_to_not_convert or ())
    for name, module in list(model.named_modules()):
        for child_name, child in list(module.named_children()):
            full = f"{name}.{child_name}" if name else child_name
            if isinstance(child, nn.Linear) and not any(full == s or full.endswith("." + s) for s in skip):
                new = (Fp8Linear.from_linear(child) if recipe == "fp8"
                       else Fp8DynamicLinear.from_linear(child, granularity))
                setattr(module, child_name, new)
    return model
