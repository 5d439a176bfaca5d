"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch


def dev():
    return torch.device("cuda:0")


def bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    """uint16 bf16 bit patterns -> a bf16 CUDA tensor."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev())


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def cuda(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev())


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def f32_from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << np.uint32(16)).view(np.float32)


def assert_no_device_error():
    from convrot_mlx_b200 import _lib

    assert _lib.take_device_error() == 0
