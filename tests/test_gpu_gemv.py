"""The register-fragment W4A4 GEMV for at most 8 activation rows (the default
kernel for m <= 8, pinned here by route 4 of convrot_set_gemm_route): bitwise against the oracle's exact integer dot and
the reference epilogue order (core.py:932-936) on both weight layouts, every
output dtype, m from 1 to 8, ragged n, K that is not a multiple of the
kernel's K unit, K split over clusters of 1 to 8 CTAs and warps with empty K
ranges, no bias, the widest int32 sums, and the FLUX modulation shapes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from convrot_mlx_b200 import _lib
from oracle import convrot_oracle as O
from tests.gpu_util import assert_no_device_error, dev, host

pytestmark = pytest.mark.gpu

_DT = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}


@pytest.fixture(autouse=True)
def gemv_route():
    _lib.check(_lib.load().convrot_set_gemm_route(4), "route")
    yield
    _lib.check(_lib.load().convrot_set_gemm_route(0), "route")


def _case(m, k, n, seed, extreme=False):
    rng = np.random.default_rng(seed)
    if extreme:  # every product at its largest magnitude: the int32 sums at their widest
        codes = np.full((m, k), -7, dtype=np.int8)
        w = np.full((n, k), -8, dtype=np.int8)
    else:
        codes = rng.integers(-7, 8, size=(m, k), dtype=np.int8)
        w = rng.integers(-8, 8, size=(n, k), dtype=np.int8)
    xs = (rng.random(m, dtype=np.float32) * 0.1 + 1e-3).astype(np.float32)
    ws = (rng.random(n, dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    bias = (rng.normal(size=n) * 0.01).astype(np.float32)
    return codes, w, xs, ws, bias


def _run(codes, w, xs, ws, bias, layout, out_dtype):
    m, k = codes.shape
    n = w.shape[0]
    q = O.pack_signed_int4(w.T.copy()) if layout == _lib.LAYOUT_KN else O.pack_signed_int4(w)
    a, qd = torch.from_numpy(codes).to(dev()), torch.from_numpy(q).to(dev())
    xsd, wsd = torch.from_numpy(xs).to(dev()), torch.from_numpy(ws).to(dev())
    bd = None if bias is None else torch.from_numpy(bias).to(dev())
    out = torch.full((m, n), float("nan"), dtype=out_dtype, device=dev())
    _lib.check(_lib.load().convrot_w4a4_gemm(_lib.ptr(a), _lib.ptr(qd), layout, _lib.ptr(xsd), _lib.ptr(wsd),
                                             None if bd is None else _lib.ptr(bd), _lib.ptr(out),
                                             _lib.DTYPE_CODES[out_dtype], m, n, k, _lib.stream_of(a)), "gemm")
    torch.cuda.synchronize()
    return out


def _want_bits(want, out_dtype):
    if out_dtype == torch.bfloat16:
        return O.bf16_bits(want).view(np.int16)
    if out_dtype == torch.float16:
        return want.astype(np.float16).view(np.int16)
    return want.astype(np.float32).view(np.int32)


def _check(m, k, n, layout, out_dtype, seed, bias=True, extreme=False):
    codes, w, xs, ws, b = _case(m, k, n, seed, extreme)
    if not bias:
        b = None
    got = _run(codes, w, xs, ws, b, layout, out_dtype)
    want = O.w4a4_epilogue(O.integer_dot(codes, w), xs, ws, b if b is not None else np.zeros(n, np.float32),
                           _DT[out_dtype])
    got_bits = host(got.view(torch.int16) if out_dtype != torch.float32 else got.view(torch.int32))
    np.testing.assert_array_equal(got_bits, _want_bits(want, out_dtype))
    assert_no_device_error()


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_gemv_bitwise(layout, m, out_dtype):
    _check(m, 1024, 768, layout, out_dtype, 10 * m + layout)


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
@pytest.mark.parametrize("k,n", [
    (32, 16),        # one K unit: seven of eight warps have nothing to do
    (96, 48),        # K not a multiple of 128, n below one column block
    (160, 144),      # partial last 128-k unit (N x packed-K), ragged last column block
    (3104, 272),     # K = 97 units of 32, clusters of 8
    (4096, 4112),    # ragged n past the 128-column blocks
])
def test_gemv_ragged_shapes(layout, k, n):
    _check(7, k, n, layout, torch.bfloat16, k + n)


@pytest.mark.parametrize("n", [40, 1000])
def test_gemv_any_n_with_nk_weights(n):
    _check(4, 512, n, _lib.LAYOUT_NK, torch.bfloat16, n)


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
def test_gemv_no_bias_and_widest_sums(layout):
    _check(8, 2048, 256, layout, torch.float32, 3, bias=False)
    _check(8, 8192, 128, layout, torch.float32, 4, extreme=True)


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
@pytest.mark.parametrize("m,k,n", [(8, 3072, 18432), (1, 3072, 9216), (2, 3072, 3072)])
def test_gemv_flux_modulation_shapes(layout, m, k, n):
    _check(m, k, n, layout, torch.bfloat16, m + n)


def test_unsupported_shapes_fall_back():
    # n % 16 != 0 with K x packed-N weights: the GEMV does not apply and the
    # call takes the tile kernels, still exact
    _check(3, 256, 40, _lib.LAYOUT_KN, torch.bfloat16, 9)
    assert _lib.load().convrot_set_gemm_route(5) == _lib.ERR_INVALID


def test_default_route_takes_the_gemv():
    _lib.check(_lib.load().convrot_set_gemm_route(0), "route")
    _check(8, 3072, 1024, _lib.LAYOUT_KN, torch.bfloat16, 11)
    _check(1, 1024, 200, _lib.LAYOUT_NK, torch.float16, 12)
