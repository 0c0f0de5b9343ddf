"""Decode-step sampling on the GPU: drop-in for core/spec_decode.py:14-35.

    probs = nucleus_probs(logits_row, temperature, top_p)     # [..., V] fp32, as the reference
    token = sample_from(probs)                                # [rows, 1] int64 (multinomial)
    token = sample_nucleus(logits, temperature, top_p)        # both in one kernel, no probs

The reference computes nucleus_probs with a full descending sort per row and draws with
torch.multinomial, one row and one host sync at a time (core/scheduler.py:341-342,
core/spec_decode.py:127-160).  Here one kernel handles any number of rows: the top-p cut
comes from a radix select in shared memory (no sort), per-row temperature and top_p may
be tensors (the scheduler's per-request settings), and the draw never leaves the GPU.

Differences a caller can observe: equal probabilities at the top-p boundary are kept in
index order (the reference's torch.sort leaves their order unspecified), and the draws
come from Philox4x32-10 seeded from torch's default CPU generator (or the `generator`
argument), so they are reproducible under torch.manual_seed but are not the same draws
torch.multinomial would make.
"""

from __future__ import annotations

import torch

from . import _lib

_SYNC_CHECKS = True
_MAX_VOCAB = 262144


def set_sync_checks(enabled: bool) -> bool:
    """Turn the per-call device error check (one host sync) on or off; returns the old value."""
    global _SYNC_CHECKS
    prev = _SYNC_CHECKS
    _SYNC_CHECKS = bool(enabled)
    return prev


def _rows(t: torch.Tensor) -> torch.Tensor:
    if t.ndim == 0:
        raise ValueError("expected a [..., vocab] tensor")
    x = t.reshape(-1, t.shape[-1])
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def _seed(generator: torch.Generator | None) -> int:
    return int(torch.randint(0, 2**63 - 1, (1,), generator=generator, dtype=torch.int64).item())


def _per_row(v, n: int, dev: torch.device, name: str):
    """(device pointer or None, scalar) for a float or a [rows] tensor argument."""
    if isinstance(v, torch.Tensor):
        t = v.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
        if t.numel() == 1:
            return t, None, float(t.item())
        if t.numel() != n:
            raise ValueError(f"{name} has {t.numel()} values for {n} rows")
        return t, t.data_ptr(), 0.0
    return None, None, float(v)


def _launch(logits: torch.Tensor, temperature, top_p, *, want_probs: bool, want_tokens: bool,
            generator: torch.Generator | None):
    dev = _lib.require_cuda(logits)
    x = _rows(logits)
    rows, vocab = x.shape
    if vocab > _MAX_VOCAB:
        raise ValueError(f"vocab {vocab} exceeds {_MAX_VOCAB}")
    keep_t, t_ptr, t_val = _per_row(temperature, rows, dev, "temperature")
    keep_p, p_ptr, p_val = _per_row(top_p, rows, dev, "top_p")
    if p_ptr is None and not p_val > 0:
        raise ValueError("top_p must be positive")
    probs = torch.empty((rows, vocab), dtype=torch.float32, device=dev) if want_probs else None
    tokens = torch.empty((rows,), dtype=torch.int64, device=dev) if want_tokens else None
    seed = _seed(generator) if want_tokens else 0
    lib = _lib.load()
    st = lib.inferd_nucleus_sample(
        _lib.ptr(probs), vocab, _lib.ptr(tokens), x.data_ptr(), _lib.dtype_code(x.dtype), x.stride(0),
        rows, vocab, t_ptr, t_val, p_ptr, p_val, seed, 0, _lib.error_word(dev).data_ptr(),
        _lib.stream_of(dev))
    _lib.check(st, "nucleus_sample")
    del keep_t, keep_p
    if _SYNC_CHECKS:
        _lib.raise_device_errors(dev)
    return probs, tokens


def nucleus_probs(logits_row: torch.Tensor, temperature: float, top_p: float) -> torch.Tensor:
    """Full-vocab probabilities after temperature and top-p (core/spec_decode.py:14-31).

    logits_row [..., V] (fp32 / fp16 / bf16, CUDA); returns fp32 of the same shape.
    temperature <= 0 gives a one-hot row at the argmax.  temperature and top_p may also be
    [rows] tensors (one value per row)."""
    probs, _ = _launch(logits_row, temperature, top_p, want_probs=True, want_tokens=False,
                       generator=None)
    return probs.view(logits_row.shape)


def sample_from(probs: torch.Tensor, *, generator: torch.Generator | None = None) -> torch.Tensor:
    """One multinomial draw per row (core/spec_decode.py:34-35): probs [rows, V] or [V]
    non-negative fp32 weights -> [rows, 1] int64 (torch.multinomial's shape)."""
    dev = _lib.require_cuda(probs)
    x = _rows(probs.float() if probs.dtype != torch.float32 else probs)
    rows, vocab = x.shape
    if vocab > _MAX_VOCAB:
        raise ValueError(f"vocab {vocab} exceeds {_MAX_VOCAB}")
    tokens = torch.empty((rows,), dtype=torch.int64, device=dev)
    lib = _lib.load()
    st = lib.inferd_sample_probs(tokens.data_ptr(), x.data_ptr(), x.stride(0), rows, vocab,
                                 _seed(generator), 0, _lib.error_word(dev).data_ptr(),
                                 _lib.stream_of(dev))
    _lib.check(st, "sample_probs")
    if _SYNC_CHECKS:
        _lib.raise_device_errors(dev)
    return tokens.view(rows, 1)


def sample_nucleus(logits: torch.Tensor, temperature, top_p, *,
                   generator: torch.Generator | None = None, return_probs: bool = False):
    """sample_from(nucleus_probs(logits, temperature, top_p)) in one kernel: [rows, 1] int64
    (and the probabilities when return_probs)."""
    probs, tokens = _launch(logits, temperature, top_p, want_probs=return_probs,
                            want_tokens=True, generator=generator)
    tokens = tokens.view(-1, 1)
    return (tokens, probs.view(logits.shape)) if return_probs else tokens


def accept_resample(p: torch.Tensor, q: torch.Tensor, proposals: torch.Tensor, *,
                    generator: torch.Generator | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The accept / resample step of a speculative round (core/spec_decode.py:145-161) for a
    batch, in one launch and without host synchronisation.

    p [B, gamma + 1, V] fp32: the target's probabilities (p[:, k] verifies draft token k,
    p[:, gamma] is the bonus distribution); q [B, gamma, V] fp32: the draft's; proposals
    [B, gamma] int64.  Returns (accepted [B] int32, tokens [B, gamma + 1] int64): sequence b
    emits tokens[b, :accepted[b] + 1] (the accepted drafts, then the token drawn from the
    residual clamp(p - q, 0) at the first rejection, or from p[:, gamma] when all were
    accepted); the remaining entries are -1.  Random draws follow the kernels' Philox
    streams under a seed taken from `generator` (torch's default generator when None), so
    they are reproducible under torch.manual_seed but are not torch.rand / torch.multinomial's.
    """
    dev = _lib.require_cuda(p, q, proposals)
    if p.ndim != 3 or q.ndim != 3 or proposals.ndim != 2:
        raise ValueError("expected p [B, gamma + 1, V], q [B, gamma, V], proposals [B, gamma]")
    b, g1, vocab = p.shape
    gamma = g1 - 1
    if tuple(q.shape) != (b, gamma, vocab) or tuple(proposals.shape) != (b, gamma):
        raise ValueError(f"q must be [{b}, {gamma}, {vocab}] and proposals [{b}, {gamma}]")
    if vocab > _MAX_VOCAB:
        raise ValueError(f"vocab {vocab} exceeds {_MAX_VOCAB}")
    p = p.float().contiguous()
    q = q.float().contiguous()
    props = proposals.to(torch.int64).contiguous()
    accepted = torch.empty((b,), dtype=torch.int32, device=dev)
    tokens = torch.empty((b, gamma + 1), dtype=torch.int64, device=dev)
    if b == 0:
        return accepted, tokens
    lib = _lib.load()
    st = lib.inferd_spec_accept(
        accepted.data_ptr(), tokens.data_ptr(), gamma + 1, p.data_ptr(), (gamma + 1) * vocab, vocab,
        q.data_ptr() if gamma else None, gamma * vocab, vocab, props.data_ptr() if gamma else None,
        max(gamma, 1), b, gamma, vocab, _seed(generator), 0, _lib.error_word(dev).data_ptr(),
        _lib.stream_of(dev))
    _lib.check(st, "spec_accept")
    if _SYNC_CHECKS:
        _lib.raise_device_errors(dev)
    return accepted, tokens
