"""The swap-AB W4A4 GEMM for few activation rows (m <= 64): bitwise against
the oracle's exact integer dot and the reference epilogue order
(core.py:932-936), on both weight layouts, every output dtype, ragged m and
n, a partial last K stage, K split over clusters of 1 to 8 CTAs, and the
shapes of the FLUX modulation linears (m = batch)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import convrot_mlx_b200 as cr
from convrot_mlx_b200 import _lib
from oracle import convrot_oracle as O
from tests.gpu_util import assert_no_device_error, dev, host

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def swap_ab_route():
    """Every m <= 64 shape on the swap-AB kernel (the default routing takes it
    only for m <= 8)."""
    _lib.check(_lib.load().convrot_set_gemm_route(3), "route")
    yield
    _lib.check(_lib.load().convrot_set_gemm_route(0), "route")


_DT = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}


def _case(m, k, n, seed):
    rng = np.random.default_rng(seed)
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
    xsd, wsd, bd = (torch.from_numpy(v).to(dev()) for v in (xs, ws, bias))
    out = torch.empty((m, n), dtype=out_dtype, device=dev())
    _lib.check(_lib.load().convrot_w4a4_gemm(_lib.ptr(a), _lib.ptr(qd), layout, _lib.ptr(xsd), _lib.ptr(wsd),
                                             _lib.ptr(bd), _lib.ptr(out), _lib.DTYPE_CODES[out_dtype], m, n, k,
                                             _lib.stream_of(a)), "gemm")
    torch.cuda.synchronize()
    return out


def _expected(codes, w, xs, ws, bias, out_dtype):
    return O.w4a4_epilogue(O.integer_dot(codes, w), xs, ws, bias, _DT[out_dtype])


def _bits(out, out_dtype):
    h = host(out.view(torch.int16) if out_dtype != torch.float32 else out.view(torch.int32))
    return h


def _want_bits(want, out_dtype):
    if out_dtype == torch.bfloat16:
        return O.bf16_bits(want).view(np.int16)
    if out_dtype == torch.float16:
        return want.astype(np.float16).view(np.int16)
    return want.astype(np.float32).view(np.int32)


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
@pytest.mark.parametrize("m,k,n", [(1, 1024, 1024), (2, 3072, 256), (8, 3072, 2304), (16, 128, 64),
                                   (17, 384, 200), (33, 2048, 320), (64, 1024, 1024), (64, 15360, 3072),
                                   (5, 12288, 96)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_small_m_bit_exact(layout, m, k, n, out_dtype):
    if layout == _lib.LAYOUT_KN and n % 2:
        pytest.skip("K x packed-N needs even n")
    codes, w, xs, ws, bias = _case(m, k, n, m * 1000 + k + n)
    got = _run(codes, w, xs, ws, bias, layout, out_dtype)
    want = _expected(codes, w, xs, ws, bias, out_dtype)
    np.testing.assert_array_equal(_bits(got, out_dtype), _want_bits(want, out_dtype))
    assert_no_device_error()


@pytest.mark.parametrize("m", [1, 8])
def test_flux_modulation_shapes(m):
    # double-block modulation (3072 -> 6 x 3072) and single-block (3072 -> 3 x 3072)
    for n in (18432, 9216):
        codes, w, xs, ws, bias = _case(m, 3072, n, n + m)
        got = _run(codes, w, xs, ws, bias, _lib.LAYOUT_KN, torch.bfloat16)
        want = _expected(codes, w, xs, ws, bias, torch.bfloat16)
        np.testing.assert_array_equal(_bits(got, torch.bfloat16), _want_bits(want, torch.bfloat16))
    assert_no_device_error()


def test_integer_extremes_small_m():
    # every product +-49 or -8 * -7: the int32 partial sums of a 8-way K split stay exact
    m, k, n = 3, 15360, 128
    codes = np.full((m, k), 7, np.int8)
    codes[1] = -7
    w = np.full((n, k), -7, np.int8)
    w[::2] = -8
    xs, ws, bias = np.ones(m, np.float32), np.ones(n, np.float32), np.zeros(n, np.float32)
    got = _run(codes, w, xs, ws, bias, _lib.LAYOUT_KN, torch.float32)
    np.testing.assert_array_equal(host(got), O.integer_dot(codes, w).astype(np.float32))
    assert_no_device_error()


def test_layer_with_batch_rows_matches_oracle():
    # ConvRotLinear at m = 8 (a DiT modulation linear at batch 8) through prep + the small-m GEMM
    k, n, m = 3072, 6144, 8
    g = torch.Generator(device=dev()).manual_seed(3)
    wd = (torch.randn((n, k), generator=g, device=dev()) * 0.02).to(torch.bfloat16)
    layer = cr.ConvRotLinear(k, n, device=dev())
    qnk, ws = cr.quantize_convrot_weight(wd)
    layer.qweight, layer.scales = cr.repack_nk_weight_for_mpp(qnk), ws
    layer.bias = torch.randn((n,), generator=g, device=dev()) * 0.01
    x = torch.randn((m, k), generator=g, device=dev()).to(torch.bfloat16)
    got = layer(x)
    xb = (host(x.view(torch.int16)).view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    want = O.convrot_linear_w4a4(xb, host(qnk), "nk", host(ws), host(layer.bias), 256)
    np.testing.assert_array_equal(host(got.view(torch.int16)).view(np.uint16), O.bf16_bits(want))
    assert_no_device_error()
