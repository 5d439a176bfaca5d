"""Pack / unpack / repack kernels vs the reference fixtures (bitwise)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import convrot_mlx_b200 as cr
from oracle import convrot_oracle as O
from tests.conftest import load_golden
from tests.gpu_util import cuda, host

pytestmark = pytest.mark.gpu


def test_pack_known_answer():
    # reference tests/test_core.py:186-192
    values = cuda(np.array([[-8, -7, -1, 0, 1, 7, 3, -4]], dtype=np.int8))
    packed = cr.pack_signed_int4(values)
    assert host(packed).tolist() == [[0x98, 0x0F, 0x71, 0xC3]]
    assert host(cr.unpack_signed_int4(packed)).tolist() == [[-8, -7, -1, 0, 1, 7, 3, -4]]


def test_unpack_matches_reference():
    # reference tests/test_core.py:194-201
    g = load_golden("unpack_s2026082300")
    packed = cr.pack_signed_int4(cuda(g["values"]))
    np.testing.assert_array_equal(host(packed), g["packed"])
    np.testing.assert_array_equal(host(cr.metal_unpack_signed_int4(packed)), g["unpacked"])


def test_repack_round_trip():
    # reference tests/test_core.py:203-211
    g = load_golden("repack_s2026082301")
    kn = cr.repack_nk_weight_for_mpp(cuda(g["packed_nk"]))
    assert tuple(kn.shape) == (64, 23)
    np.testing.assert_array_equal(host(kn), g["packed_kn"])
    np.testing.assert_array_equal(host(cr.repack_mpp_weight_to_nk(kn)), g["packed_nk"])


@pytest.mark.parametrize("shape", [(1, 2), (3, 34), (46, 64), (130, 258), (1000, 3000)])
def test_pack_unpack_repack_random(shape):
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    values = rng.integers(-8, 8, size=shape, dtype=np.int8)
    packed = cr.pack_signed_int4(cuda(values))
    np.testing.assert_array_equal(host(packed), O.pack_signed_int4(values))
    np.testing.assert_array_equal(host(cr.unpack_signed_int4(packed)), values)
    if shape[0] % 2 == 0:
        kn = cr.repack_nk_weight_for_mpp(packed)
        np.testing.assert_array_equal(host(kn), O.repack_nk_weight_for_mpp(O.pack_signed_int4(values)))
        if shape[1] % 2 == 0 and (shape[1] // 2) % 2 == 0:
            pass
        back = cr.repack_mpp_weight_to_nk(kn)
        np.testing.assert_array_equal(host(back), host(packed))


def test_pack_wraps_modulo_16():
    # the reference masks with & 0x0F after an int32 cast (core.py:101-104)
    values = torch.tensor([[9, -9, 15, -16]], dtype=torch.int32, device="cuda")
    np.testing.assert_array_equal(host(cr.pack_signed_int4(values)),
                                  O.pack_signed_int4(np.array([[9, -9, 15, -16]], np.int32)))
