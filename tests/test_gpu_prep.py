"""Fused rotate + quantize kernels vs the reference fixtures and the oracle (bitwise)."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import convrot_mlx_b200 as cr
from oracle import convrot_oracle as O
from tests.conftest import bf16_from_bits, golden_manifest, load_golden, seeded_bf16_normal
from tests.gpu_util import assert_no_device_error, bf16_bits, bf16_tensor, cuda, host

pytestmark = pytest.mark.gpu


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["prep_g256_s17", "prep_g256_s18", "prep_g256_s1801"])
def test_fused_prep_matches_reference_fixture(name):
    # reference tests/test_core.py:54-86 (19 x 512, bf16, group 256)
    g = load_golden(name)
    x = bf16_tensor(g["x_bf16"])
    qact, scales = cr.metal_fused_prepare_convrot_activation(x)
    np.testing.assert_array_equal(host(qact), g["qact"])
    np.testing.assert_array_equal(host(scales), g["scales"])
    codes, scales_i8 = cr.metal_fused_prepare_convrot_activation_i8(x)
    np.testing.assert_array_equal(host(codes), g["codes"])
    np.testing.assert_array_equal(host(scales_i8), g["scales"])
    q2, s2 = cr.prepare_convrot_activation(x)
    np.testing.assert_array_equal(host(q2), g["qact"])
    np.testing.assert_array_equal(host(s2), g["scales"])


def test_fused_rotation_matches_reference_fixture():
    # reference tests/test_core.py:88-96
    g = load_golden("rotate_g256_s1802")
    rot = cr.metal_fused_rotate_convrot_activation(bf16_tensor(g["x_bf16"]))
    np.testing.assert_array_equal(bf16_bits(rot), g["rot_bf16"])


def test_group64_matches_reference_fixture():
    # reference tests/test_core.py:98-126 (17 x 2688, group 64)
    g = load_golden("prep_g64_s2026082305")
    x = bf16_tensor(g["x_bf16"])
    qact, scales = cr.metal_fused_prepare_convrot_activation(x, 64)
    np.testing.assert_array_equal(host(qact), g["qact"])
    np.testing.assert_array_equal(host(scales), g["scales"])
    codes, s8 = cr.metal_fused_prepare_convrot_activation_i8(x, 64)
    np.testing.assert_array_equal(host(codes), g["codes"])
    np.testing.assert_array_equal(host(s8), g["scales"])
    rot = cr.metal_fused_rotate_convrot_activation(x, 64)
    np.testing.assert_array_equal(bf16_bits(rot), g["rot_bf16"])


def test_route_shape_matches_reference_digest():
    # reference tests/test_core.py:128-137 (1536 x 3072)
    m = golden_manifest()["cases"]["prep_route_s20260823"]
    (x,) = seeded_bf16_normal(m["seed"], tuple(m["shape"]))
    xt = bf16_tensor(O.bf16_bits(x))
    qact, scales = cr.metal_fused_prepare_convrot_activation(xt)
    assert _sha(host(qact)) == m["qact_sha256"]
    assert _sha(host(scales)) == m["scales_sha256"]
    codes, _ = cr.metal_fused_prepare_convrot_activation_i8(xt)
    assert _sha(host(codes)) == m["codes_sha256"]


def test_kronecker_rotation_fp32():
    # reference tests/test_core.py:177-184
    g = load_golden("kron_f32_s17")
    rot = host(cr.regular_hadamard(cuda(g["x"])))
    np.testing.assert_array_equal(rot, g["rot"])
    h = O.regular_hadamard_matrix(256)
    expected = np.concatenate([g["x"][:, :256] @ h, g["x"][:, 256:] @ h], axis=1)
    np.testing.assert_allclose(rot, expected, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("name", ["quant_f16_s23", "quant_f16_s28"])
def test_float16_rowwise_quantization(name):
    # reference tests/test_core.py:311-327, :357-373 (no rotation, float16)
    g = load_golden(name)
    qact, xs = cr.quantize_signed_int4_rowwise(cuda(g["act_f16"]))
    qw, ws = cr.quantize_signed_int4_rowwise(cuda(g["w_f16"]))
    np.testing.assert_array_equal(host(qact), g["qact"])
    np.testing.assert_array_equal(host(xs), g["xscales"])
    np.testing.assert_array_equal(host(qw), g["qweight"])
    np.testing.assert_array_equal(host(ws), g["wscales"])


@pytest.mark.parametrize("group", [16, 64, 256, 1024])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("shape", [(5, 1024), (3, 3072), (2, 15360), (7, 2048 + 1024)])
def test_prep_matches_oracle_all_groups_and_dtypes(group, dtype, shape):
    rows, k = shape
    if k % group:
        pytest.skip("features not divisible by the group")
    rng = np.random.default_rng(1000 + group + k)
    x = rng.normal(size=shape).astype(np.float32)
    x[:, rng.choice(k, max(1, k // 100), replace=False)] *= 20.0  # outlier channels
    x = O.round_to(dtype, x)
    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[dtype]
    xt = torch.from_numpy(x).to("cuda").to(tdt)
    q, s = cr.prepare_convrot_activation(xt, group)
    eq, es = O.prepare_convrot_activation(x, group, dtype)
    np.testing.assert_array_equal(host(q), eq)
    np.testing.assert_array_equal(host(s), es)
    codes, s8 = cr.metal_fused_prepare_convrot_activation_i8(xt, group) if group in (64, 256) else (None, None)
    if codes is not None:
        np.testing.assert_array_equal(host(codes), O.unpack_signed_int4(eq))
    rot = cr.regular_hadamard(xt, group)
    er = O.regular_hadamard(x, group, dtype)
    np.testing.assert_array_equal(host(rot.float()), er)


def test_prep_edge_rows():
    # all-zero row (absmax floor), a single huge value, negative zeros, inf-free extremes
    x = np.zeros((4, 512), np.float32)
    x[1, 7] = 3.0e38
    x[2, :] = -0.0
    x[3, ::3] = 1e-30
    xb = O.round_bf16(x)
    xt = bf16_tensor(O.bf16_bits(xb))
    q, s = cr.metal_fused_prepare_convrot_activation(xt)
    eq, es = O.prepare_convrot_activation(xb, 256)
    np.testing.assert_array_equal(host(q), eq)
    np.testing.assert_array_equal(host(s), es)


def test_prep_odd_group_count_and_single_group():
    # K / G odd: the pair partner of the middle group is absent
    for k, g in ((256, 256), (768, 256), (64 * 5, 64), (2688, 64)):
        rng = np.random.default_rng(k + g)
        x = O.round_bf16(rng.normal(size=(9, k)).astype(np.float32))
        q, s = cr.prepare_convrot_activation(bf16_tensor(O.bf16_bits(x)), g)
        eq, es = O.prepare_convrot_activation(x, g)
        np.testing.assert_array_equal(host(q), eq)
        np.testing.assert_array_equal(host(s), es)


def test_prep_empty_rows():
    x = torch.empty((0, 512), dtype=torch.bfloat16, device="cuda")
    q, s = cr.metal_fused_prepare_convrot_activation(x)
    assert q.shape == (0, 256) and s.shape == (0,)


def test_prep_full_size_config2():
    # 4096 x 3072, 1% outlier channels x20, groups 64 and 256
    rng = np.random.default_rng(20260823)
    x = rng.normal(size=(4096, 3072)).astype(np.float32)
    x[:, rng.choice(3072, 31, replace=False)] *= 20.0
    xb = O.round_bf16(x)
    xt = bf16_tensor(O.bf16_bits(xb))
    for g in (64, 256):
        codes, s = cr.metal_fused_prepare_convrot_activation_i8(xt, g)
        ec, es = O.prepare_convrot_activation_i8(xb, g)
        np.testing.assert_array_equal(host(codes), ec)
        np.testing.assert_array_equal(host(s), es)
    assert_no_device_error()
