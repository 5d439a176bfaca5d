"""Modulated LayerNorm fused into the activation preparation
(convrot_modnorm_prepare_i8, ConvRotLinear.forward_modulated_norm).

* Constant rows make the norm exactly zero (mean exact, variance 0), so xm
  is the shift vector itself and the codes must equal the oracle's
  prepare_i8(shift) bit for bit: this pins the modulation arithmetic, the
  row-to-sample mapping with strided modulation vectors, and the rotate +
  quantize path.
* On random rows the kernel's float32 row statistics may differ from any
  other summation order in the last bit, which can move a y or xm across a
  bf16 rounding boundary and a code by one (the tolerance stated for fp32
  summation order): codes are compared with the oracle of a float64
  LayerNorm, at most 0.1% differing and none by more than one; the layer's
  bf16 output stays within rel-L2 1e-3 of the unfused torch path.
* The same kernel fed by a FLUX single block's cat(attention, gelu(mlp))
  (convrot_gelu_concat_prepare_i8, ConvRotLinear.forward_gelu_concat) is
  bit for bit prepare_i8 of the concatenation.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import convrot_mlx_b200 as cr
from convrot_mlx_b200 import _lib
from convrot_mlx_b200.core import modulated_norm_prepare_i8
from oracle import convrot_oracle as O
from tests.gpu_util import assert_no_device_error, bf16_bits, dev, f32_from_bf16_bits, host

pytestmark = pytest.mark.gpu


def _mods(batch, k, seed, strided):
    g = torch.Generator(device=dev()).manual_seed(seed)
    if strided:  # chunks of one (batch, 1, 6k) modulation output, as in a DiT block
        m = (torch.randn((batch, 1, 6 * k), generator=g, device=dev()) * 0.5).to(torch.bfloat16)
        chunks = m.chunk(6, dim=-1)
        return chunks[0], chunks[1]
    shift = (torch.randn((batch, 1, k), generator=g, device=dev()) * 0.5).to(torch.bfloat16)
    scale = (torch.randn((batch, 1, k), generator=g, device=dev()) * 0.5).to(torch.bfloat16)
    return shift, scale


@pytest.mark.parametrize("group", [64, 256])
@pytest.mark.parametrize("strided", [False, True])
@pytest.mark.parametrize("k", [3072, 1024, 2560])
def test_constant_rows_give_prep_of_shift(group, strided, k):
    batch, tokens = 3, 5
    shift, scale = _mods(batch, k, 7 + k, strided)
    consts = torch.tensor([1.0, -2.0, 0.5], device=dev())
    x = (torch.ones((batch, tokens, k), device=dev()) * consts[:, None, None]).to(torch.bfloat16)
    codes, scales = modulated_norm_prepare_i8(x, shift, scale, 1e-6, group)
    sh = f32_from_bf16_bits(bf16_bits(shift.reshape(batch, k)))
    want_c, want_s = O.prepare_convrot_activation_i8(np.repeat(sh, tokens, axis=0), group)
    np.testing.assert_array_equal(host(codes), want_c)
    np.testing.assert_array_equal(host(scales), want_s)
    assert_no_device_error()


def _xm_reference(x, shift, scale, eps):
    """float64 LayerNorm statistics, then the kernel's rounding points."""

    xf = x.astype(np.float64)
    mean = xf.mean(axis=-1, keepdims=True)
    var = ((xf - mean) ** 2).mean(axis=-1, keepdims=True)
    y = O.round_bf16(((xf - mean) / np.sqrt(var + eps)).astype(np.float32))
    t = O.round_bf16((1.0 + scale.astype(np.float64)).astype(np.float32))
    xm = (y.astype(np.float64) * t + shift).astype(np.float32)
    return O.round_bf16(xm)


@pytest.mark.parametrize("group", [64, 256])
def test_random_rows_within_summation_order_tolerance(group):
    batch, tokens, k = 2, 300, 3072
    g = torch.Generator(device=dev()).manual_seed(group)
    x = torch.randn((batch, tokens, k), generator=g, device=dev()) * 2.0 + 0.3
    x[..., ::97] *= 20.0  # outlier channels
    x = x.to(torch.bfloat16)
    shift, scale = _mods(batch, k, 11, True)
    codes, scales = modulated_norm_prepare_i8(x, shift, scale, 1e-6, group)
    xb = f32_from_bf16_bits(bf16_bits(x)).reshape(batch, tokens, k)
    sh = f32_from_bf16_bits(bf16_bits(shift.reshape(batch, 1, k)))
    sc = f32_from_bf16_bits(bf16_bits(scale.reshape(batch, 1, k)))
    xm = _xm_reference(xb, sh, sc, 1e-6).reshape(-1, k)
    want_c, want_s = O.prepare_convrot_activation_i8(xm, group)
    got_c = host(codes).astype(np.int32)
    diff = np.abs(got_c - want_c.astype(np.int32))
    assert diff.max() <= 1
    assert (diff != 0).mean() <= 1e-3, (diff != 0).mean()
    rel = np.abs(host(scales) - want_s) / want_s
    assert rel.max() <= 2.0 ** -7  # at most one bf16 ulp of the row absmax
    assert (rel != 0).mean() <= 0.01
    assert_no_device_error()


@pytest.mark.parametrize("backend", ["mpp-w4a4", "reference"])
def test_layer_forward_modulated_norm_tracks_unfused(backend):
    batch, tokens, k, n = 2, 257, 3072, 1536
    g = torch.Generator(device=dev()).manual_seed(5)
    w = (torch.randn((n, k), generator=g, device=dev()) * 0.02).to(torch.bfloat16)
    layer = cr.ConvRotLinear(k, n, backend=backend, device=dev())
    qnk, ws = cr.quantize_convrot_weight(w)
    layer.qweight = cr.repack_nk_weight_for_mpp(qnk) if backend == "mpp-w4a4" else qnk
    layer.scales = ws
    layer.bias = torch.randn((n,), generator=g, device=dev()) * 0.01
    x = torch.randn((batch, tokens, k), generator=g, device=dev()).to(torch.bfloat16)
    shift, scale = _mods(batch, k, 3, True)
    got = layer.forward_modulated_norm(x, shift, scale, 1e-6).float()
    normed = torch.nn.functional.layer_norm(x, (k,), eps=1e-6)
    want = layer(torch.addcmul(shift, normed, 1 + scale)).float()
    assert got.shape == (batch, tokens, n)
    rel = float((got - want).norm() / want.norm())
    assert rel <= 1e-3, rel
    assert_no_device_error()


def test_fused_prep_argument_errors():
    lib = _lib.load()
    x = torch.zeros((4, 256), dtype=torch.bfloat16, device=dev())
    s = torch.zeros((1, 256), dtype=torch.bfloat16, device=dev())
    codes = torch.empty((4, 256), dtype=torch.int8, device=dev())
    sc = torch.empty((4,), dtype=torch.float32, device=dev())
    args = lambda dtype, group, rpm, stride: (_lib.ptr(x), dtype, 4, 256, group, _lib.ptr(s), _lib.ptr(s), rpm,  # noqa: E731
                                              stride, 1e-6, _lib.ptr(codes), _lib.ptr(sc), None)
    assert lib.convrot_modnorm_prepare_i8(*args(_lib.F16, 256, 4, 256)) == _lib.ERR_UNSUPPORTED
    assert lib.convrot_modnorm_prepare_i8(*args(_lib.BF16, 16, 4, 256)) == _lib.ERR_UNSUPPORTED
    assert lib.convrot_modnorm_prepare_i8(*args(_lib.BF16, 256, 0, 256)) == _lib.ERR_INVALID
    assert lib.convrot_modnorm_prepare_i8(*args(_lib.BF16, 256, 4, 100)) == _lib.ERR_INVALID
    assert lib.convrot_modnorm_prepare_i8(*args(_lib.BF16, 256, 4, 256)) == _lib.OK
    with pytest.raises(ValueError):
        modulated_norm_prepare_i8(x.float(), s, s)
    torch.cuda.synchronize()
    assert_no_device_error()


@pytest.mark.parametrize("group", [64, 256])
@pytest.mark.parametrize("da,dm", [(3072, 12288), (512, 2048)])
def test_gelu_concat_prep_equals_prep_of_the_concatenation(group, da, dm):
    # the single-block output projection's input, cat(attention, gelu(mlp half
    # of a wider tensor)): fused, it must give exactly prepare_i8 of the
    # concatenation built by the DiT's glue kernel (the same GELU form)
    import flux_dit
    from convrot_mlx_b200.core import gelu_concat_prepare_i8

    flux_dit.build_glue()
    g = torch.Generator(device=dev()).manual_seed(da + group)
    a = torch.randn((2, 37, da), generator=g, device=dev()).to(torch.bfloat16)
    h = (torch.randn((2, 37, 3 * da + dm), generator=g, device=dev()) * 2.5).to(torch.bfloat16)
    m = h[..., 3 * da:]
    codes, scales = gelu_concat_prepare_i8(a, m, group)
    cat = flux_dit.gelu_concat(a, m)
    want_c, want_s = cr.metal_fused_prepare_convrot_activation_i8(cat.reshape(-1, da + dm), group)
    assert torch.equal(codes, want_c)
    assert torch.equal(scales, want_s)
    assert_no_device_error()


def test_layer_forward_gelu_concat_equals_unfused():
    import flux_dit

    flux_dit.build_glue()
    da, dm, n = 512, 2048, 512
    g = torch.Generator(device=dev()).manual_seed(21)
    w = (torch.randn((n, da + dm), generator=g, device=dev()) * 0.02).to(torch.bfloat16)
    layer = cr.ConvRotLinear(da + dm, n, device=dev())
    qnk, ws = cr.quantize_convrot_weight(w)
    layer.qweight, layer.scales = cr.repack_nk_weight_for_mpp(qnk), ws
    layer.bias = torch.randn((n,), generator=g, device=dev()) * 0.01
    a = torch.randn((3, 50, da), generator=g, device=dev()).to(torch.bfloat16)
    h = torch.randn((3, 50, 3 * da + dm), generator=g, device=dev()).to(torch.bfloat16)
    got = layer.forward_gelu_concat(a, h[..., 3 * da:])
    want = layer(flux_dit.gelu_concat(a, h[..., 3 * da:]))
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # and within bf16 rounding of torch's own tanh GELU
    ref = layer(torch.cat((a, torch.nn.functional.gelu(h[..., 3 * da:], approximate="tanh")), -1)).float()
    assert float((got.float() - ref).norm() / ref.norm()) < 1e-2
    assert_no_device_error()
