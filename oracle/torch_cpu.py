"""PyTorch-CPU restatement of the reference's eager ConvRot path -- TEST AND
BASELINE INFRASTRUCTURE ONLY (imported by tests/ and by bench.py's CPU legs).

This is the timed CPU baseline: the same contract as ``oracle/convrot_oracle.py``
written with torch CPU tensor ops so that it runs multi-threaded at the speed
of an eager framework, like the reference's MLX eager path on its CPU device:

* ``prepare`` -- ``prepare_convrot_activation`` (core.py:161-167):
  ``regular_hadamard`` (core.py:64-94) in bf16 with per-op rounding (torch's
  CPU bf16 ops compute in float32 and round each result to nearest even), then
  ``quantize_signed_int4_rowwise`` (core.py:149-158);
* ``linear`` -- the layer with ``backend="reference"`` (core.py:1292-1313):
  prep, then ``reference_w4a4_matmul`` (core.py:1155-1171): unpack both
  operands, an fp32 matmul (exact: every partial sum is an integer below
  2^24), ``* xs * ws + bias`` in float32, cast to bf16.

``tests/test_oracle.py`` checks it bit for bit against the NumPy oracle.
"""

from __future__ import annotations

import math

import torch


def regular_hadamard(x: torch.Tensor, group_size: int = 256) -> torch.Tensor:
    """core.py:64-94 on a CPU tensor of any float dtype (per-op rounding)."""

    features = x.shape[-1]
    groups = features // group_size
    prefix = (*x.shape[:-1], groups)
    y = x.reshape(*prefix, group_size)
    stride = 1
    while stride < group_size:
        y = y.reshape(*prefix, group_size // (4 * stride), 4, stride)
        a, b, c, d = y[..., 0, :], y[..., 1, :], y[..., 2, :], y[..., 3, :]
        y = torch.stack([a + b + c - d, a + b - c + d, a - b + c + d, -a + b + c + d], dim=-2)
        y = y.reshape(*prefix, group_size)
        stride *= 4
    return (y / math.sqrt(group_size)).reshape(x.shape)


def quantize_codes(x: torch.Tensor):
    """core.py:149-158 without packing: (int8 codes, float32 scales)."""

    absmax = x.abs().amax(dim=-1, keepdim=True)
    absmax = torch.maximum(absmax, torch.tensor(1e-10, dtype=x.dtype))
    scales = absmax / 7
    q = torch.round(x / scales).nan_to_num(0.0).clamp(-7, 7).to(torch.int8)
    return q, scales.reshape(-1).to(torch.float32)


def prepare(x: torch.Tensor, group_size: int = 256):
    return quantize_codes(regular_hadamard(x, group_size))


def pack(values: torch.Tensor) -> torch.Tensor:
    v = values.to(torch.int32)
    return ((v[..., 0::2] & 0xF) | ((v[..., 1::2] & 0xF) << 4)).to(torch.uint8)


def unpack(packed: torch.Tensor) -> torch.Tensor:
    d = packed.to(torch.int32)
    lo = d & 0xF
    hi = (d >> 4) & 0xF
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack([lo, hi], dim=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2).to(torch.int8)


def epilogue(dots: torch.Tensor, xs, ws, bias, out_dtype=torch.bfloat16) -> torch.Tensor:
    out = dots * xs[:, None]
    out = out * ws[None, :]
    out = out + bias[None, :]
    return out.to(out_dtype)


def linear(x: torch.Tensor, qweight_nk: torch.Tensor, ws, bias, group_size: int = 256,
           weight_unpacked: torch.Tensor | None = None) -> torch.Tensor:
    """The reference layer's eager CPU path; ``weight_unpacked`` (float32 (N, K))
    may be passed to time the unpack separately."""

    codes, xs = prepare(x, group_size)
    w = weight_unpacked if weight_unpacked is not None else unpack(qweight_nk).to(torch.float32)
    dots = codes.to(torch.float32) @ w.T
    return epilogue(dots, xs, ws, bias, x.dtype)
