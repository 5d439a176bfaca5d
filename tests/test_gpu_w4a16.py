"""W4A16 tcgen05 GEMM (kind::f16) vs the reference fixtures and a float32 model.

The reference (core.py:1123-1152) accumulates ``rot @ w`` in float32 in its
own order; the kernel accumulates the same exact products in float32 in
tensor-core order.  Parity is therefore to float32 rounding of the dots,
whose error grows with K: float32 outputs within 1e-5 * max(1, K / 4096) of
the output scale, 16-bit outputs within one unit in the last place of the
expected value plus that amount (near-zero outputs, where dots * ws cancels
the bias, carry the absolute float32 error), and rel-L2 under 1e-3.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import convrot_mlx_b200 as cr
from convrot_mlx_b200 import _lib
from tests.conftest import load_golden
from tests.gpu_util import assert_no_device_error, bf16_tensor, cuda, dev, host

pytestmark = pytest.mark.gpu

F32_RTOL = 1e-5        # |got - want| <= F32_RTOL * max(1, K / 4096) * max|want| (summation order only)
REL_L2_16BIT = 1e-3    # 16-bit outputs: rel-L2 bound of the north-star contract; per element
                       # |got - want| <= ulp(want) + F32_RTOL * max(1, K / 4096) * max|want|


def _model(act: torch.Tensor, qweight_kn: torch.Tensor, ws: torch.Tensor, bias, out_dtype) -> torch.Tensor:
    """core.py:1123-1152 in float32 on the device (float64 dots, then the
    reference's float32 epilogue): fl(dots * ws) + bias, cast."""
    w = cr.unpack_signed_int4(qweight_kn).to(torch.float64)          # (K, N)
    dots = (act.to(torch.float64) @ w).to(torch.float32)
    out = dots * ws[None, :]
    if bias is not None:
        out = out + bias[None, :]
    return out.to(out_dtype)


def _ulp(want: torch.Tensor) -> torch.Tensor:
    """One unit in the last place of each 16-bit value (as float32)."""
    mant = 7 if want.dtype == torch.bfloat16 else 10
    a = want.float().abs()
    e = torch.floor(torch.log2(a.clamp_min(2.0 ** -126)))
    return torch.where(a > 0, torch.exp2(e - mant), torch.zeros_like(a))


def _check(got: torch.Tensor, want: torch.Tensor, k: int):
    assert got.shape == want.shape and got.dtype == want.dtype
    g, w = got.float(), want.float()
    abs_tol = F32_RTOL * max(1.0, k / 4096) * max(float(w.abs().max()), 1e-30)
    if got.dtype == torch.float32:
        assert float((g - w).abs().max()) <= abs_tol
    else:
        rel = float((g - w).norm() / w.norm().clamp_min(1e-30))
        assert rel <= REL_L2_16BIT, rel
        bound = _ulp(want) + abs_tol
        assert bool(((g - w).abs() <= bound).all()), float(((g - w).abs() - bound).max())


@pytest.mark.parametrize("act_name,act_dtype", [("bf16", torch.bfloat16), ("f16", torch.float16)])
def test_w4a16_fixture(act_name, act_dtype):
    # reference tests/test_core.py (w4a16 fixture, seed 2026082303): N = 46, K = 64
    g = load_golden("w4a16_s2026082303")
    act = cuda(g[f"act_{act_name}_as_f32"]).to(act_dtype)
    out = cr.mpp_w4a16_matmul(act, cuda(g["qweight_kn"]), cuda(g["wscales"]), cuda(g["bias"]),
                              output_dtype=torch.float32)
    want = cuda(g[f"out_{act_name}_f32"])
    tol = F32_RTOL * float(want.abs().max())
    assert float((out - want).abs().max()) <= tol
    assert_no_device_error()


@pytest.mark.parametrize("name,group", [("layer_kn_g256_s2026082304", 256), ("layer_kn_g64_s2026082306", 64)])
def test_layer_w4a16_contract(name, group):
    # reference tests/test_core.py:404-448 (mpp-w4a16 backend)
    g = load_golden(name)
    qnk, ws = cr.quantize_convrot_weight(bf16_tensor(g["w_bf16"]), group)
    k = g["x_bf16"].shape[-1]
    layer = cr.ConvRotLinear(k, 34, group_size=group, backend="mpp-w4a16").cuda()
    layer.qweight = cr.repack_nk_weight_for_mpp(qnk)
    layer.scales = ws
    layer.bias = cuda(g["bias"])
    out = layer(bf16_tensor(g["x_bf16"]))
    assert tuple(out.shape) == (2, 7, 34)
    _check(out, bf16_tensor(g["w4a16_bf16"]), k)
    assert_no_device_error()


SHAPES = [(1, 64, 32), (37, 128, 64), (129, 256, 96), (256, 3072, 3072), (300, 1024, 512), (513, 1728, 3072),
          (1536, 3072, 9216), (700, 15360, 256), (64, 2688, 34)]


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("act_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_w4a16_kn_vs_model(m, k, n, act_dtype, out_dtype):
    gen = torch.Generator(device=dev()).manual_seed(m * 7 + k * 3 + n)
    act = torch.randn((m, k), generator=gen, device=dev()).to(act_dtype)
    w = torch.randint(-8, 8, (k, n), generator=gen, device=dev(), dtype=torch.int8)
    q = cr.pack_signed_int4(w)
    ws = torch.rand((n,), generator=gen, device=dev()) * 0.01
    bias = torch.randn((n,), generator=gen, device=dev()) * 0.01
    out = cr.mpp_w4a16_matmul(act, q, ws, bias, output_dtype=out_dtype)
    _check(out, _model(act, q, ws, bias, out_dtype), k)
    assert_no_device_error()


@pytest.mark.parametrize("m,k,n", [(37, 128, 46), (256, 3072, 3072), (300, 1024, 520)])
def test_w4a16_nk_through_c_abi(m, k, n):
    # N x packed-K weights through the C ABI directly (no host padding)
    gen = torch.Generator(device=dev()).manual_seed(m + k + n)
    act = torch.randn((m, k), generator=gen, device=dev()).to(torch.bfloat16)
    w = torch.randint(-8, 8, (n, k), generator=gen, device=dev(), dtype=torch.int8)
    qnk = cr.pack_signed_int4(w)
    ws = torch.rand((n,), generator=gen, device=dev())
    out = torch.empty((m, n), dtype=torch.float32, device=dev())
    lib = _lib.load()
    _lib.check(lib.convrot_w4a16_gemm(_lib.ptr(act), _lib.BF16, _lib.ptr(qnk), _lib.LAYOUT_NK, _lib.ptr(ws), None,
                                      _lib.ptr(out), _lib.F32, m, n, k, _lib.stream_of(act)), "w4a16 nk")
    want = _model(act, cr.pack_signed_int4(w.t().contiguous()), ws, None, torch.float32)
    _check(out, want, k)
    assert_no_device_error()


def test_w4a16_rejects_unaligned_k_in_c_abi():
    act = torch.zeros((4, 96), dtype=torch.bfloat16, device=dev())
    q = torch.zeros((96, 16), dtype=torch.uint8, device=dev())
    ws = torch.ones(32, device=dev())
    out = torch.empty((4, 32), dtype=torch.bfloat16, device=dev())
    rc = _lib.load().convrot_w4a16_gemm(_lib.ptr(act), _lib.BF16, _lib.ptr(q), _lib.LAYOUT_KN, _lib.ptr(ws), None,
                                        _lib.ptr(out), _lib.BF16, 4, 32, 96, _lib.stream_of(act))
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"divisible by 64" in _lib.load().convrot_last_error()
