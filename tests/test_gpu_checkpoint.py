"""The reference's on-disk checkpoint format through the CUDA kernels: this
package's converter and repack reproduce the files that the reference's own
convert.py / repack_mpp.py wrote (bit for bit, metadata included), and
load_convrot_model loads either schema into a torch model whose swapped
layers then compute the oracle's W4A4 linear exactly."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from convrot_mlx_b200 import checkpoint as ck
from oracle import convrot_oracle as O
from tests.ckpt_util import CONVERTED, LINEARS, MPP, NK, SOURCE, tiny_model
from tests.gpu_util import assert_no_device_error, bf16_bits, dev

pytestmark = pytest.mark.gpu


def _assert_same_tensors(got: dict, want: dict):
    assert set(got) == set(want)
    for k in want:
        assert got[k].dtype == want[k].dtype, k
        assert torch.equal(got[k].cpu(), want[k]), k


def test_convert_reproduces_the_reference_converter():
    source, _ = ck.read_checkpoint(SOURCE)
    want, want_meta = ck.read_checkpoint(NK)
    got = ck.convert_state_dict(source, CONVERTED, device=dev())
    _assert_same_tensors(got, want)
    assert_no_device_error()


def test_repack_reproduces_the_reference_repack():
    nk, nk_meta = ck.read_checkpoint(NK)
    want, want_meta = ck.read_checkpoint(MPP)
    got, got_meta = ck.repack_checkpoint_for_mpp(nk, nk_meta, device=dev())
    _assert_same_tensors(got, want)
    assert got_meta == want_meta
    assert_no_device_error()


@pytest.mark.parametrize("path,backend", [(MPP, "mpp-w4a4"), (NK, "reference")])
def test_load_reference_checkpoint_and_run(path, backend):
    model = tiny_model(dev())
    model, meta, names = ck.load_convrot_model(model, path, backend=backend)
    assert names == CONVERTED
    nk, _ = ck.read_checkpoint(NK)
    g = torch.Generator(device=dev()).manual_seed(31)
    mods = dict(model.named_modules())
    for name, k, n, bias in LINEARS:
        if name not in CONVERTED:
            assert isinstance(mods[name], torch.nn.Linear)
            continue
        layer = mods[name]
        assert layer.backend == backend
        x = torch.randn((19, k), generator=g, device=dev()).to(torch.bfloat16)
        got = bf16_bits(layer(x))
        xb = (bf16_bits(x).astype(np.uint32) << 16).view(np.float32)
        want = O.convrot_linear_w4a4(xb, nk[f"{name}.qweight"].numpy(), "nk", nk[f"{name}.scales"].numpy(),
                                     nk[f"{name}.bias"].numpy(), 256)
        np.testing.assert_array_equal(got, O.bf16_bits(want))
    assert_no_device_error()


def test_convert_model_write_and_load_round_trip(tmp_path):
    # a dense model with the fixture's weights -> our checkpoint -> MPP -> load
    source, _ = ck.read_checkpoint(SOURCE)
    dense = tiny_model(dev())
    dense.load_state_dict({k: v.to(dev()) for k, v in source.items()}, strict=True)
    tensors, meta = ck.convert_model(dense, device=dev(), runtime_revision="test")
    assert meta["converted_linear_count"] == str(len(CONVERTED))
    mpp_t, mpp_meta = ck.repack_checkpoint_for_mpp(tensors, meta, device=dev())
    path = tmp_path / "model.safetensors"
    ck.write_checkpoint(path, mpp_t, mpp_meta)
    loaded, _, names = ck.load_convrot_model(tiny_model(dev()), path, backend="mpp-w4a4")
    want, _ = ck.read_checkpoint(MPP)
    state = loaded.state_dict()
    for k, v in want.items():
        assert torch.equal(state[k].cpu(), v), k
    # a schema that does not match the backend is refused before any swap
    with pytest.raises(ValueError, match="requires checkpoint schema"):
        ck.load_convrot_model(tiny_model(dev()), path, backend="reference")
    assert_no_device_error()
