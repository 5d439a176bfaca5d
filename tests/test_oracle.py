"""The NumPy oracle against the golden fixtures generated from the reference.

These run on CPU only.  They pin ``oracle/convrot_oracle.py`` (the checker of
every GPU parity test) to the reference's own eager functions and to the
known-answer tests of the reference's ``tests/test_core.py``.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import convrot_oracle as O
from tests.conftest import bf16_from_bits, golden_manifest, load_golden, seeded_bf16_normal


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["prep_g256_s17", "prep_g256_s18", "prep_g256_s1801"])
def test_prep_g256_matches_reference(name):
    # reference tests/test_core.py:54-86
    g = load_golden(name)
    x = bf16_from_bits(g["x_bf16"])
    qact, scales = O.prepare_convrot_activation(x, 256)
    np.testing.assert_array_equal(qact, g["qact"])
    np.testing.assert_array_equal(scales, g["scales"])
    codes, scales_i8 = O.prepare_convrot_activation_i8(x, 256)
    np.testing.assert_array_equal(codes, g["codes"])
    np.testing.assert_array_equal(scales_i8, g["scales"])


def test_rotation_g256_matches_reference():
    # reference tests/test_core.py:88-96
    g = load_golden("rotate_g256_s1802")
    rot = O.regular_hadamard(bf16_from_bits(g["x_bf16"]), 256)
    np.testing.assert_array_equal(O.bf16_bits(rot), g["rot_bf16"])


def test_group64_prep_and_rotation_match_reference():
    # reference tests/test_core.py:98-126
    g = load_golden("prep_g64_s2026082305")
    x = bf16_from_bits(g["x_bf16"])
    qact, scales = O.prepare_convrot_activation(x, 64)
    np.testing.assert_array_equal(qact, g["qact"])
    np.testing.assert_array_equal(scales, g["scales"])
    np.testing.assert_array_equal(O.bf16_bits(O.regular_hadamard(x, 64)), g["rot_bf16"])


def test_route_shape_prep_matches_reference_digest():
    # reference tests/test_core.py:128-137 (1536 x 3072)
    m = golden_manifest()["cases"]["prep_route_s20260823"]
    (x,) = seeded_bf16_normal(m["seed"], tuple(m["shape"]))
    assert _sha(O.bf16_bits(x)) == m["x_sha256"]
    qact, scales = O.prepare_convrot_activation(x, 256)
    assert _sha(qact) == m["qact_sha256"]
    assert _sha(scales) == m["scales_sha256"]


def test_kronecker_rotation_fp32():
    # reference tests/test_core.py:42-50, :177-184 (the rotation's own KAT)
    g = load_golden("kron_f32_s17")
    values = g["x"]
    rot = O.regular_hadamard(values, 256, "float32")
    np.testing.assert_array_equal(rot, g["rot"])
    h = O.regular_hadamard_matrix(256)
    expected = np.concatenate([values[:, :256] @ h, values[:, 256:] @ h], axis=1)
    np.testing.assert_allclose(rot, expected, rtol=2e-6, atol=2e-6)


def test_pack_known_answer():
    # reference tests/test_core.py:186-192
    values = np.array([[-8, -7, -1, 0, 1, 7, 3, -4]], dtype=np.int8)
    packed = O.pack_signed_int4(values)
    assert packed.tolist() == [[0x98, 0x0F, 0x71, 0xC3]]
    assert O.unpack_signed_int4(packed).tolist() == values.tolist()
    g = load_golden("pack_kat")
    np.testing.assert_array_equal(packed, g["packed"])


def test_unpack_matches_reference():
    # reference tests/test_core.py:194-201
    g = load_golden("unpack_s2026082300")
    np.testing.assert_array_equal(O.pack_signed_int4(g["values"]), g["packed"])
    np.testing.assert_array_equal(O.unpack_signed_int4(g["packed"]), g["unpacked"])


def test_repack_round_trip_matches_reference():
    # reference tests/test_core.py:203-211
    g = load_golden("repack_s2026082301")
    kn = O.repack_nk_weight_for_mpp(g["packed_nk"])
    assert kn.shape == (64, 23)
    np.testing.assert_array_equal(kn, g["packed_kn"])
    np.testing.assert_array_equal(O.repack_mpp_weight_to_nk(kn), g["packed_nk"])
    with pytest.raises(ValueError, match="even out_features"):
        O.repack_nk_weight_for_mpp(O.pack_signed_int4(np.zeros((3, 4), np.int8)))


def test_w4a4_edges_match_reference():
    # reference tests/test_core.py:213-283
    g = load_golden("edges_s2026082302")
    out = O.reference_w4a4_matmul(g["qact"], g["qweight_nk"], g["xscales"], g["wscales"], g["bias"], "float32")
    np.testing.assert_array_equal(out, g["out_f32"])
    out_bf = O.reference_w4a4_matmul(g["qact"], g["qweight_nk"], g["xscales"], g["wscales"], g["bias"], "bfloat16")
    np.testing.assert_array_equal(O.bf16_bits(out_bf), g["out_bf16"])
    codes = O.unpack_signed_int4(g["qact"])
    kn = O.w4a4_int8_matmul_kn(codes, g["qweight_kn"], g["xscales"], g["wscales"], g["bias"], "float32")
    np.testing.assert_array_equal(kn, g["out_f32"])
    dots = O.integer_dot(codes, O.unpack_signed_int4(g["qweight_nk"]))
    np.testing.assert_array_equal(dots.astype(np.float32), g["out_int"])


def test_w4a16_matches_reference():
    # reference tests/test_core.py:285-309
    g = load_golden("w4a16_s2026082303")
    for name in ("f16", "bf16"):
        out = O.w4a16_matmul(g[f"act_{name}_as_f32"], g["qweight_kn"], g["wscales"], g["bias"], "float32")
        np.testing.assert_allclose(out, g[f"out_{name}_f32"], rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("name", ["quant_f16_s23", "quant_f16_s28"])
def test_float16_rowwise_quantization_matches_reference(name):
    # reference tests/test_core.py:311-327, :357-373
    g = load_golden(name)
    qact, xs = O.quantize_signed_int4_rowwise(g["act_f16"].astype(np.float32), "float16")
    qw, ws = O.quantize_signed_int4_rowwise(g["w_f16"].astype(np.float32), "float16")
    np.testing.assert_array_equal(qact, g["qact"])
    np.testing.assert_array_equal(xs, g["xscales"])
    np.testing.assert_array_equal(qw, g["qweight"])
    np.testing.assert_array_equal(ws, g["wscales"])
    out = O.reference_w4a4_matmul(qact, qw, xs, ws, g["bias"], "float32")
    np.testing.assert_array_equal(out, g["out_f32"])


@pytest.mark.parametrize("name", ["tiles_s29", "expanded_s27"])
def test_bf16_output_matches_reference(name):
    # reference tests/test_core.py:139-175, :329-355
    g = load_golden(name)
    out = O.reference_w4a4_matmul(g["qact"], g["qweight_nk"], g["xscales"], g["wscales"], g["bias"], "bfloat16")
    np.testing.assert_array_equal(O.bf16_bits(out), g["out_bf16"])


def test_layer_contract_nk_matches_reference():
    # reference tests/test_core.py:375-402
    g = load_golden("layer_nk_s29")
    w = bf16_from_bits(g["w_bf16"])
    qw, ws = O.quantize_convrot_weight(w, 256)
    np.testing.assert_array_equal(qw, g["qweight_nk"])
    np.testing.assert_array_equal(ws, g["wscales"])
    out = O.convrot_linear_w4a4(bf16_from_bits(g["x_bf16"]), qw, "nk", ws, g["bias"], 256)
    np.testing.assert_array_equal(O.bf16_bits(out), g["out_bf16"])


@pytest.mark.parametrize("name,group", [("layer_kn_g256_s2026082304", 256), ("layer_kn_g64_s2026082306", 64)])
def test_layer_contract_kn_matches_reference(name, group):
    # reference tests/test_core.py:404-448 (the reference checks only shape and
    # finiteness there; the fixture holds the eager-oracle values)
    g = load_golden(name)
    w = bf16_from_bits(g["w_bf16"])
    qw, ws = O.quantize_convrot_weight(w, group)
    np.testing.assert_array_equal(qw, g["qweight_nk"])
    np.testing.assert_array_equal(O.repack_nk_weight_for_mpp(qw), g["qweight_kn"])
    x = bf16_from_bits(g["x_bf16"])
    out = O.convrot_linear_w4a4(x, g["qweight_kn"], "kn", ws, g["bias"], group)
    np.testing.assert_array_equal(O.bf16_bits(out), g["w4a4_bf16"])
    np.testing.assert_array_equal(O.bf16_bits(O.regular_hadamard(x.reshape(-1, x.shape[-1]), group)), g["rot_bf16"])
    out16 = O.convrot_linear_w4a16(x, g["qweight_kn"], ws, g["bias"], group)
    ref16 = bf16_from_bits(g["w4a16_bf16"])
    # fp32 accumulation order differs (float64-exact here, a BLAS sgemm there):
    # allow one bf16 ulp.
    np.testing.assert_allclose(out16, ref16, rtol=2 ** -7, atol=1e-6)


def test_config1_matches_reference():
    # K=N=1024, M=64, no bias, group 256
    g = load_golden("config1_s20260823")
    m = golden_manifest()["cases"]["config1_s20260823"]
    x, w = seeded_bf16_normal(m["seed"], (64, 1024), (1024, 1024))
    np.testing.assert_array_equal(O.bf16_bits(x), g["x_bf16"])
    assert _sha(O.bf16_bits(w)) == m["w_sha256"]
    qw, ws = O.quantize_convrot_weight(w, 256)
    np.testing.assert_array_equal(qw, g["qweight_nk"])
    np.testing.assert_array_equal(ws, g["wscales"])
    out = O.convrot_linear_w4a4(x, qw, "nk", ws, np.zeros(1024, np.float32), 256)
    np.testing.assert_array_equal(O.bf16_bits(out), g["out_bf16"])


def test_group_size_validation():
    # reference core.py:50-61
    for bad in (1, 2, 8, 32, 48, 128):
        with pytest.raises(ValueError, match="power of 4"):
            O.validate_group_size(bad)
    for good in (4, 16, 64, 256, 1024):
        O.validate_group_size(good)


def test_torch_cpu_port_matches_oracle():
    # the timed CPU baseline (oracle/torch_cpu.py) must be the same contract, bit for bit
    import torch

    from oracle import torch_cpu as TC

    rng = np.random.default_rng(99)
    for k, g in ((512, 256), (2688, 64), (3072, 256)):
        x = O.round_bf16(rng.normal(size=(33, k)).astype(np.float32))
        x[:, rng.choice(k, 5, replace=False)] *= 20.0
        x = O.round_bf16(x)
        xt = torch.from_numpy(x).to(torch.bfloat16)
        codes, scales = TC.prepare(xt, g)
        ec, es = O.prepare_convrot_activation_i8(x, g)
        np.testing.assert_array_equal(codes.numpy(), ec)
        np.testing.assert_array_equal(scales.numpy(), es)
        w = O.round_bf16((rng.normal(size=(40, k)) * 0.02).astype(np.float32))
        qw, ws = O.quantize_convrot_weight(w, g)
        b = rng.normal(size=40).astype(np.float32)
        out = TC.linear(xt, torch.from_numpy(qw), torch.from_numpy(ws), torch.from_numpy(b), g)
        expected = O.convrot_linear_w4a4(x, qw, "nk", ws, b, g)
        np.testing.assert_array_equal(out.view(torch.int16).numpy().view(np.uint16), O.bf16_bits(expected))
        np.testing.assert_array_equal(TC.pack(torch.from_numpy(ec)).numpy(), O.pack_signed_int4(ec))
        np.testing.assert_array_equal(TC.unpack(torch.from_numpy(qw)).numpy(), O.unpack_signed_int4(qw))
