"""ConvRotLinear (the drop-in layer) vs the reference fixtures, bitwise."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import convrot_mlx_b200 as cr
from oracle import convrot_oracle as O
from tests.conftest import golden_manifest, load_golden, seeded_bf16_normal
from tests.gpu_util import assert_no_device_error, bf16_bits, bf16_tensor, cuda, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("backend", ["metal", "metal-k32", "metal-k64", "metal-m32n32-k64", "mlx-expanded-fp32",
                                     "reference"])
def test_layer_nk_contract(backend):
    # reference tests/test_core.py:375-402
    g = load_golden("layer_nk_s29")
    w = bf16_tensor(g["w_bf16"])
    qweight, wscales = cr.quantize_convrot_weight(w)
    np.testing.assert_array_equal(host(qweight), g["qweight_nk"])
    np.testing.assert_array_equal(host(wscales), g["wscales"])
    layer = cr.ConvRotLinear(256, 33, backend=backend).cuda()
    layer.qweight = qweight
    layer.scales = wscales
    layer.bias = cuda(g["bias"])
    out = layer(bf16_tensor(g["x_bf16"]))
    assert tuple(out.shape) == (2, 7, 33)
    np.testing.assert_array_equal(bf16_bits(out), g["out_bf16"])


@pytest.mark.parametrize("name,group", [("layer_kn_g256_s2026082304", 256), ("layer_kn_g64_s2026082306", 64)])
def test_layer_kn_w4a4_contract(name, group):
    # reference tests/test_core.py:404-448 (there shape/finiteness; here bitwise)
    g = load_golden(name)
    qnk, ws = cr.quantize_convrot_weight(bf16_tensor(g["w_bf16"]), group)
    np.testing.assert_array_equal(host(qnk), g["qweight_nk"])
    qkn = cr.repack_nk_weight_for_mpp(qnk)
    np.testing.assert_array_equal(host(qkn), g["qweight_kn"])
    k = g["x_bf16"].shape[-1]
    layer = cr.ConvRotLinear(k, 34, group_size=group, backend="mpp-w4a4").cuda()
    layer.qweight = qkn
    layer.scales = ws
    layer.bias = cuda(g["bias"])
    out = layer(bf16_tensor(g["x_bf16"]))
    assert tuple(out.shape) == (2, 7, 34)
    np.testing.assert_array_equal(bf16_bits(out), g["w4a4_bf16"])


def test_config1_layer():
    # K = N = 1024, M = 64, no bias, group 256, NK weights
    g = load_golden("config1_s20260823")
    m = golden_manifest()["cases"]["config1_s20260823"]
    x, w = seeded_bf16_normal(m["seed"], (64, 1024), (1024, 1024))
    qweight, ws = cr.quantize_convrot_weight(bf16_tensor(O.bf16_bits(w)))
    np.testing.assert_array_equal(host(qweight), g["qweight_nk"])
    np.testing.assert_array_equal(host(ws), g["wscales"])
    layer = cr.ConvRotLinear(1024, 1024, bias=False, backend="reference").cuda()
    layer.qweight = qweight
    layer.scales = ws
    out = layer(bf16_tensor(g["x_bf16"]))
    np.testing.assert_array_equal(bf16_bits(out), g["out_bf16"])
    # and the default backend with the repacked weight
    layer_kn = cr.ConvRotLinear(1024, 1024, bias=False).cuda()
    layer_kn.qweight = cr.repack_nk_weight_for_mpp(qweight)
    layer_kn.scales = ws
    np.testing.assert_array_equal(bf16_bits(layer_kn(bf16_tensor(g["x_bf16"]))), g["out_bf16"])
    assert_no_device_error()


def test_layer_flux_shape_vs_oracle():
    # a FLUX-sized linear (M = 1536, K = 3072, N = 3072) against the oracle, bitwise
    rng = np.random.default_rng(7)
    x = O.round_bf16(rng.normal(size=(1536, 3072)).astype(np.float32))
    x[:, rng.choice(3072, 31, replace=False)] *= 20.0
    x = O.round_bf16(x)
    w = O.round_bf16((rng.normal(size=(3072, 3072)) * 0.02).astype(np.float32))
    b = (rng.normal(size=3072) * 0.01).astype(np.float32)
    qnk, ws = O.quantize_convrot_weight(w, 256)
    qkn = O.repack_nk_weight_for_mpp(qnk)
    expected = O.convrot_linear_w4a4(x, qkn, "kn", ws, b, 256)
    layer = cr.ConvRotLinear(3072, 3072).cuda()
    layer.qweight = cuda(qkn)
    layer.scales = cuda(ws)
    layer.bias = cuda(b)
    out = layer(bf16_tensor(O.bf16_bits(x)))
    np.testing.assert_array_equal(bf16_bits(out), O.bf16_bits(expected))
