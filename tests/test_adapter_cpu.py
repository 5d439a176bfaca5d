"""replace_convrot_linears on CPU (no quantization): which layers are swapped,
their shapes, layouts and names -- the eligibility rule of the reference's
adapter (core.py:1316-1321, examples/flux1_dev/adapter.py:45-70)."""

from __future__ import annotations

import pytest
from torch import nn

from convrot_mlx_b200 import ConvRotLinear
from convrot_mlx_b200.adapter import replace_convrot_linears


def _model():
    return nn.Sequential(nn.Linear(64, 256), nn.GELU(), nn.Sequential(nn.Linear(256, 512), nn.Linear(512, 46, bias=False)),
                         nn.Linear(300, 512))


@pytest.mark.parametrize("backend,layout", [("mpp-w4a4", "packed-kn-low-nibble-even-output"),
                                            ("reference", "packed-nk-low-nibble-even-feature")])
def test_replaces_eligible_linears_only(backend, layout):
    m = _model()
    names = replace_convrot_linears(m, backend=backend, quantize=False)
    assert names == ["2.0", "2.1"]
    assert isinstance(m[0], nn.Linear) and isinstance(m[3], nn.Linear)  # in 64 and 300: not multiples of 256
    a, b = m[2][0], m[2][1]
    assert isinstance(a, ConvRotLinear) and isinstance(b, ConvRotLinear)
    assert (a.in_features, a.out_features, b.in_features, b.out_features) == (256, 512, 512, 46)
    assert a.source_has_bias and not b.source_has_bias
    assert a.weight_layout == layout and a.backend == backend
