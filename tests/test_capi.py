"""Host-side checks of the C ABI and the Python boundary (no GPU needed).

The library loads, exports exactly the entry points ``include/convrot_b200.h``
declares, and rejects invalid arguments before touching the device.  The
Python API raises the reference's ``ValueError`` messages and refuses CPU
tensors (there is no CPU fallback).
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "convrot_b200.h"


def _declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(convrot_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from convrot_mlx_b200 import _lib

    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from convrot_mlx_b200 import _lib

    declared = _declared()
    assert declared, "no declarations parsed"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r"\bT (convrot_[a-z0-9_]+)$", out, flags=re.M)))
    assert exported == declared
    for name in declared:
        assert hasattr(lib, name)
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version(lib):
    assert lib.convrot_abi_version() == 100


def _err(lib):
    return lib.convrot_last_error().decode()


def test_invalid_arguments_fail_before_any_device_work(lib):
    P = ctypes.c_void_p
    fake = P(4096)  # never dereferenced: every call below fails validation first
    assert lib.convrot_prepare_i8(fake, 7, 4, 256, 256, fake, fake, None) == -1
    assert "dtype" in _err(lib)
    assert lib.convrot_prepare_i8(fake, 2, 4, 256, 8, fake, fake, None) == -1
    assert "power of 4" in _err(lib)
    assert lib.convrot_prepare_packed(fake, 2, 4, 320, 256, fake, fake, None) == -1
    assert "not divisible" in _err(lib)
    assert lib.convrot_rotate(fake, 2, 4, 256, 1, fake, None) == -1
    assert lib.convrot_w4a4_gemm(fake, fake, 0, fake, fake, fake, fake, 2, 4, 4, 48, None) == -1
    assert "divisible by 32" in _err(lib)
    assert lib.convrot_w4a4_gemm(fake, fake, 1, fake, fake, fake, fake, 2, 4, 5, 64, None) == -1
    assert "even N" in _err(lib)
    assert lib.convrot_w4a4_gemm(fake, fake, 3, fake, fake, fake, fake, 2, 4, 4, 64, None) == -1
    assert lib.convrot_pack_int4(fake, 3, fake, None) == -1
    assert lib.convrot_repack_int4_transpose(fake, 3, 4, fake, None) == -1
    # empty problems are valid no-ops
    assert lib.convrot_w4a4_gemm(fake, fake, 0, fake, fake, fake, fake, 2, 0, 4, 64, None) == 0
    assert lib.convrot_unpack_int4(fake, 0, fake, None) == 0


def test_gemm_route_range(lib):
    # routes 0-4 (automatic, one-CTA, CTA-pair, swap-AB, GEMV) are accepted
    # and touch no device; anything else is refused with a message
    for route in (1, 2, 3, 4, 0):
        assert lib.convrot_set_gemm_route(route) == 0
    for route in (-1, 5):
        assert lib.convrot_set_gemm_route(route) == -1
        assert "0-4" in _err(lib)
    assert lib.convrot_set_gemm_route(0) == 0


def test_python_validation_matches_reference_messages():
    import convrot_mlx_b200 as cr

    with pytest.raises(ValueError, match="power of 4"):
        cr.regular_hadamard(torch.zeros(2, 48), 48)
    with pytest.raises(ValueError, match="not divisible by ConvRot group size"):
        cr.regular_hadamard(torch.zeros(2, 320), 256)
    with pytest.raises(ValueError, match="last dimension must be even"):
        cr.pack_signed_int4(torch.zeros(2, 3, dtype=torch.int8))
    with pytest.raises(ValueError, match="supports groups"):
        cr.metal_fused_prepare_convrot_activation(torch.zeros(2, 1024), 16)
    with pytest.raises(ValueError, match="expects 2D input"):
        cr.metal_fused_prepare_convrot_activation_i8(torch.zeros(2, 2, 256))
    with pytest.raises(ValueError, match="even out_features"):
        cr.repack_nk_weight_for_mpp(torch.zeros(3, 4, dtype=torch.uint8))
    with pytest.raises(ValueError, match="even in_features"):
        cr.repack_mpp_weight_to_nk(torch.zeros(3, 4, dtype=torch.uint8))
    with pytest.raises(ValueError, match="Unknown ConvRot backend"):
        cr.ConvRotLinear(256, 4, backend="cuda-magic")
    with pytest.raises(ValueError, match="Unknown ConvRot preprocessor"):
        cr.ConvRotLinear(256, 4, preprocessor="numpy")
    with pytest.raises(ValueError, match="even out_features"):
        cr.ConvRotLinear(256, 33, backend="mpp-w4a4")
    with pytest.raises(ValueError, match="not divisible by ConvRot group size"):
        cr.ConvRotLinear(100, 4)
    with pytest.raises(ValueError, match="Unsupported staged tile"):
        cr.core.packed_w4a4_matmul_staged(torch.zeros(1, 1), torch.zeros(1, 1), None, None, None,
                                     output_dtype=torch.bfloat16, tile_k=48)
    with pytest.raises(ValueError, match="consecutive-integer"):
        cr.expanded_fp32_w4a4_matmul(torch.zeros(1, 200000, dtype=torch.uint8), torch.zeros(1, 200000, dtype=torch.uint8),
                                     None, None, None, output_dtype=torch.bfloat16)


def test_cpu_tensors_are_rejected():
    import convrot_mlx_b200 as cr

    with pytest.raises(ValueError, match="no CPU fallback"):
        cr.metal_fused_prepare_convrot_activation(torch.zeros(2, 256, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="no CPU fallback"):
        cr.unpack_signed_int4(torch.zeros(2, 4, dtype=torch.uint8))


def test_layer_layout_and_buffers():
    import convrot_mlx_b200 as cr

    kn = cr.ConvRotLinear(256, 34)
    assert kn.backend == "mpp-w4a4"
    assert kn.weight_layout == "packed-kn-low-nibble-even-output"
    assert tuple(kn.qweight.shape) == (256, 17)
    nk = cr.ConvRotLinear(256, 33, backend="metal", bias=False)
    assert nk.weight_layout == "packed-nk-low-nibble-even-feature"
    assert tuple(nk.qweight.shape) == (33, 128)
    assert nk.source_has_bias is False
    assert torch.equal(nk.bias, torch.zeros(33))
    assert torch.equal(nk.scales, torch.ones(33))
    assert set(dict(nk.named_buffers())) == {"qweight", "scales", "bias"}


def test_eligible_linear():
    import convrot_mlx_b200 as cr

    assert cr.eligible_linear(torch.nn.Linear(512, 8))
    assert not cr.eligible_linear(torch.nn.Linear(64, 8))
    assert cr.eligible_linear(torch.nn.Linear(64, 8), group_size=64)
    assert not cr.eligible_linear(torch.nn.Conv1d(512, 8, 1))


def test_public_api_matches_reference_names():
    import convrot_mlx_b200 as cr

    # src/convrot_mlx/__init__.py:41-75 of the reference
    expected = {
        "CONVROT_GROUP_SIZE", "INT4_MAX", "SUPPORTED_BACKENDS", "SUPPORTED_FUSED_GROUP_SIZES",
        "SUPPORTED_PREPROCESSORS", "ConvRotLinear", "compiled_prepare_convrot_activation",
        "compiled_regular_hadamard", "eligible_linear", "expanded_fp32_w4a4_matmul",
        "metal_fused_prepare_convrot_activation", "metal_fused_prepare_convrot_activation_i8",
        "metal_fused_rotate_convrot_activation", "metal_unpack_signed_int4", "mpp_w4a4_int8_matmul",
        "mpp_w4a4_matmul", "mpp_w4a16_matmul", "pack_signed_int4", "packed_w4a4_matmul",
        "packed_w4a4_matmul_k32", "packed_w4a4_matmul_k64", "packed_w4a4_matmul_k128",
        "packed_w4a4_matmul_k256", "packed_w4a4_matmul_m16n64_k64", "packed_w4a4_matmul_m32n32_k64",
        "prepare_convrot_activation", "quantize_convrot_weight", "quantize_signed_int4_rowwise",
        "reference_w4a4_matmul", "regular_hadamard", "repack_mpp_weight_to_nk", "repack_nk_weight_for_mpp",
        "unpack_signed_int4",
    }
    assert set(cr.__all__) == expected
    assert cr.__version__ == "0.1.0"
    assert cr.SUPPORTED_BACKENDS == frozenset({"metal", "metal-k32", "metal-k64", "metal-m32n32-k64", "mpp-w4a4",
                                               "mpp-w4a16", "mlx-expanded-fp32", "reference"})
