"""The reference's on-disk checkpoint format, without a GPU: the fixtures that
the reference's own convert.py / repack_mpp.py wrote (over the NumPy mlx
stand-in) are pinned to the oracle, and this package reads, validates and
writes them."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from convrot_mlx_b200 import checkpoint as ck
from oracle import convrot_oracle as O
from tests.ckpt_util import CONVERTED, EXTRA, LINEARS, MPP, NK, SOURCE


def _bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


def test_fixture_keys_and_metadata():
    tensors, meta = ck.read_checkpoint(NK)
    want = {f"{n}.{s}" for n in CONVERTED for s in ("qweight", "scales", "bias")}
    want |= {"img_in.weight", "img_in.bias"} | {n for n, _ in EXTRA}
    assert set(tensors) == want
    assert meta["schema"] == ck.CONVROT_SCHEMA
    assert meta["converted_linear_count"] == str(len(CONVERTED))
    assert meta["linear_count"] == str(len(LINEARS))
    for key, value in ck.ALGORITHM_METADATA.items():  # convert.py:41-50 (inspect's required keys)
        assert meta[key] == value
    for name, k, n, bias in LINEARS:
        if name in CONVERTED:
            assert tensors[f"{name}.qweight"].dtype == torch.uint8 and tuple(tensors[f"{name}.qweight"].shape) == (n, k // 2)
            assert tensors[f"{name}.scales"].dtype == torch.float32
            assert tensors[f"{name}.bias"].dtype == torch.float32
    mpp_t, mpp_meta = ck.read_checkpoint(MPP)
    assert mpp_meta["schema"] == ck.CONVROT_MPP_SCHEMA
    assert mpp_meta["weight_layout"] == ck.CONVROT_MPP_WEIGHT_LAYOUT
    for name, k, n, bias in LINEARS:
        if name in CONVERTED:
            assert tuple(mpp_t[f"{name}.qweight"].shape) == (k, n // 2)


def test_fixture_matches_oracle_conversion_and_repack():
    # the reference's converter output equals the oracle's quantize_convrot_weight
    # (core.py:514-527) and its repack equals the oracle's (core.py:123-133)
    source, _ = ck.read_checkpoint(SOURCE)
    nk, _ = ck.read_checkpoint(NK)
    mpp, _ = ck.read_checkpoint(MPP)
    for name, k, n, bias in LINEARS:
        if name not in CONVERTED:
            assert torch.equal(nk[f"{name}.weight"], source[f"{name}.weight"])
            continue
        q, s = O.quantize_convrot_weight(_bf16_np(source[f"{name}.weight"]), 256)
        np.testing.assert_array_equal(nk[f"{name}.qweight"].numpy(), q)
        np.testing.assert_array_equal(nk[f"{name}.scales"].numpy(), s)
        want_bias = _bf16_np(source[f"{name}.bias"]) if bias else np.zeros(n, np.float32)
        np.testing.assert_array_equal(nk[f"{name}.bias"].numpy(), want_bias)
        np.testing.assert_array_equal(mpp[f"{name}.qweight"].numpy(), O.repack_nk_weight_for_mpp(q))


@pytest.mark.parametrize("backend", ["reference", "metal", "mlx-expanded-fp32"])
def test_nk_checkpoint_validates_for_nk_backends(backend):
    _, meta = ck.read_checkpoint(NK)
    ck.validate_checkpoint_metadata(meta, backend)
    with pytest.raises(ValueError, match="requires checkpoint schema"):
        ck.validate_checkpoint_metadata(meta, "mpp-w4a4")


def test_mpp_checkpoint_validation_errors():
    _, meta = ck.read_checkpoint(MPP)
    ck.validate_checkpoint_metadata(meta, "mpp-w4a4")
    ck.validate_checkpoint_metadata(meta, "mpp-w4a16")
    with pytest.raises(ValueError, match="requires checkpoint schema"):
        ck.validate_checkpoint_metadata(meta, "reference")
    with pytest.raises(ValueError, match="unsupported weight layout"):
        ck.validate_checkpoint_metadata(dict(meta, weight_layout="k_by_n"), "mpp-w4a4")
    with pytest.raises(ValueError, match="FLUX.1 Dev source digest"):
        ck.validate_checkpoint_metadata(dict(meta, source_sha256="0" * 64), "mpp-w4a4")
    ck.validate_checkpoint_metadata(dict(meta, source_sha256="0" * 64), "mpp-w4a4", require_source=None)
    with pytest.raises(ValueError, match="group size"):
        ck.validate_checkpoint_metadata(dict(meta, convrot_group_size="64"), "mpp-w4a4")


def test_write_read_round_trip_and_no_overwrite(tmp_path):
    tensors, meta = ck.read_checkpoint(MPP)
    path = tmp_path / "copy.safetensors"
    ck.write_checkpoint(path, tensors, meta)
    back, back_meta = ck.read_checkpoint(path)
    assert back_meta == meta
    assert set(back) == set(tensors)
    for k in tensors:
        assert back[k].dtype == tensors[k].dtype and torch.equal(back[k], tensors[k])
    with pytest.raises(FileExistsError):
        ck.write_checkpoint(path, tensors, meta)
    with pytest.raises(ValueError, match="strings"):
        ck.write_checkpoint(tmp_path / "bad.safetensors", tensors, {"schema": 1})


def test_metadata_builder_matches_the_reference_converter():
    _, meta = ck.read_checkpoint(NK)
    ours = ck.convrot_metadata(converted_linear_count=len(CONVERTED), linear_count=len(LINEARS))
    for key, value in ours.items():
        assert meta[key] == value, key
