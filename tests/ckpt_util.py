"""The checkpoint fixtures' topology (written by tests/golden/make_checkpoint_golden.py)."""

from __future__ import annotations

import json

from torch import nn

from tests.conftest import GOLDEN

MANIFEST = json.loads((GOLDEN / "ckpt_manifest.json").read_text())
LINEARS = [tuple(x) for x in MANIFEST["linears"]]
EXTRA = [(n, tuple(s)) for n, s in MANIFEST["extra"]]
CONVERTED = [name for name, k, n, bias in LINEARS if k % 256 == 0]
SOURCE = GOLDEN / "ckpt_source.safetensors"
NK = GOLDEN / "ckpt_nk.safetensors"
MPP = GOLDEN / "ckpt_mpp.safetensors"


def _child(root: nn.Module, dotted: str) -> tuple[nn.Module, str]:
    parts = dotted.split(".")
    mod = root
    for p in parts[:-1]:
        if not hasattr(mod, p):
            mod.add_module(p, nn.Module())
        mod = getattr(mod, p)
    return mod, parts[-1]


def tiny_model(device=None) -> nn.Module:
    """A dense torch model whose module names are the fixture's."""

    import torch

    root = nn.Module()
    for name, k, n, bias in LINEARS:
        parent, leaf = _child(root, name)
        parent.add_module(leaf, nn.Linear(k, n, bias=bias, device=device, dtype=torch.bfloat16))
    for name, shape in EXTRA:
        parent, leaf = _child(root, name)
        parent.register_parameter(leaf, nn.Parameter(torch.ones(shape, device=device, dtype=torch.bfloat16)))
    return root
