"""FP8 (e4m3) weight-only linear on tcgen05 tensor cores (drop-in for the reference's
load-time torchao quantisation, bench/model_loader.py:46-58 and :82-88).

    q, s = quantize_fp8_per_channel(weight)        # load time, per output channel
    y = fp8_linear(x, q, s)                        # every forward: y = x @ (q * s)^T
    quantize_model_fp8(model, modules_to_not_convert=("lm_head",))

The reference keeps lm_head in bf16 (`modules_to_not_convert=["lm_head"]`); the model
helper does the same by default.  Activations stay bf16 at the interface; inside the
kernel they are split exactly into two e4m3 planes so the FP8 tensor pipe can be used
without the ~3 % error of a single e4m3 copy (see include/inferd_b200.h).
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib

E4M3_MAX = 448.0


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


def fp8_linear(x: torch.Tensor, w_e4m3: torch.Tensor, w_scale: torch.Tensor,
               bias: torch.Tensor | None = None, *, out: torch.Tensor | None = None,
               packed_shape: tuple[int, int] | None = None) -> torch.Tensor:
    """y = x @ (w_e4m3 * w_scale[:, None])^T (+ bias), bf16 in and out.

    x [..., K] bf16, w_scale [N] fp32.  w_e4m3 is either the row-major codes [N, K]
    (float8_e4m3fn or uint8) or, with packed_shape=(N, K), the buffer from pack_fp8_weight.
    """
    if x.dtype != torch.bfloat16:
        raise ValueError("fp8_linear takes bf16 activations")
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
    m = x2.shape[0]
    if out is None:
        y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    else:
        y = out.view(m, n)
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


def quantize_model_fp8(model: nn.Module, modules_to_not_convert=("lm_head",)) -> nn.Module:
    """Swap every nn.Linear of `model` (except names ending in modules_to_not_convert) for
    an Fp8Linear, as TorchAoConfig(Float8WeightOnlyConfig(), modules_to_not_convert=
    ["lm_head"]) does at load time in the reference (bench/model_loader.py:58, :82-88)."""
    skip = tuple(modules_to_not_convert or ())
    for name, module in list(model.named_modules()):
        for child_name, child in list(module.named_children()):
            full = f"{name}.{child_name}" if name else child_name
            if isinstance(child, nn.Linear) and not any(full == s or full.endswith("." + s) for s in skip):
                setattr(module, child_name, Fp8Linear.from_linear(child))
    return model
