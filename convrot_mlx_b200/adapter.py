"""Swap the eligible ``nn.Linear`` layers of a torch model for ConvRotLinear.

The torch counterpart of the reference's FLUX adapter
(``examples/flux1_dev/adapter.py:45-70``, ``replace_convrot_linears``): every
module that ``eligible_linear`` accepts (a 2-D ``nn.Linear`` whose
in_features is a multiple of the group size, core.py:1316-1321) becomes a
``ConvRotLinear`` with the same shape, bias flag and the chosen backend.
The reference builds empty layers and loads converted weights afterwards;
with ``quantize=True`` (the default here) each layer is instead filled from
the dense weight it replaces (``quantize_convrot_weight`` and, for the
``mpp-*`` backends, ``repack_nk_weight_for_mpp``), which is how a model with
no converted checkpoint -- a random-init benchmark model -- gets its W4
weights.
"""

from __future__ import annotations

import torch
from torch import nn

from .core import CONVROT_GROUP_SIZE, ConvRotLinear, eligible_linear, quantize_convrot_weight, repack_nk_weight_for_mpp


def _set_module(root: nn.Module, name: str, module: nn.Module) -> None:
    parent = root
    parts = name.split(".")
    for p in parts[:-1]:
        parent = getattr(parent, p)
    setattr(parent, parts[-1], module)


def replace_convrot_linears(model: nn.Module, *, backend: str = "mpp-w4a4", preprocessor: str = "metal-fused",
                            group_size: int = CONVROT_GROUP_SIZE, quantize: bool = True) -> list[str]:
    """Replace every eligible linear in ``model``; returns the replaced names in
    module order (as the reference's adapter does)."""

    targets = [(name, m) for name, m in model.named_modules() if name and eligible_linear(m, group_size)]
    names = []
    for name, linear in targets:
        w = linear.weight
        layer = ConvRotLinear(linear.in_features, linear.out_features, bias=linear.bias is not None,
                              group_size=group_size, backend=backend, preprocessor=preprocessor, device=w.device)
        if quantize:
            with torch.no_grad():
                qnk, scales = quantize_convrot_weight(w.detach().to(torch.bfloat16), group_size)
                layer.qweight = repack_nk_weight_for_mpp(qnk) if backend.startswith("mpp-") else qnk
                layer.scales = scales
                if linear.bias is not None:
                    layer.bias = linear.bias.detach().to(torch.float32).clone()
        _set_module(model, name, layer)
        names.append(name)
    return names
