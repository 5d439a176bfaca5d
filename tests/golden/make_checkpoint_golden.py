#!/usr/bin/env python3
"""Generate the on-disk checkpoint fixtures under ``tests/golden/`` from the
reference's own conversion scripts.

Runs ``examples/flux1_dev/convert.py`` (``convert``) and
``examples/flux1_dev/repack_mpp.py`` (``repack``) of Lumenbeing/convrot-mlx,
unchanged, with ``mlx`` replaced by the NumPy stand-in of
``_mlx_numpy_shim.py`` and the absent MLX FLUX example package (``flux.*``)
replaced by stubs around a six-linear FLUX-like topology.  The shim's
``load`` / ``save_safetensors`` read and write safetensors through the
``safetensors`` package.  The converter checks the source file's byte count
against the real FLUX.1 Dev file; the tiny source is handed over as a path
whose ``stat()`` reports that count (its hash check is skipped with the
converter's own ``skip_source_hash`` flag).

Writes:
  ckpt_source.safetensors   the tiny bf16 source (seeded ~ N(0, 0.02) weights)
  ckpt_nk.safetensors       convert():  N x packed-K qweights, f32 scales/bias
  ckpt_mpp.safetensors      repack():   K x packed-N qweights
  ckpt_manifest.json        topology, seeds and file digests

Usage (needs the reference checkout; the GPU box does not):

    python tests/golden/make_checkpoint_golden.py --reference /path/to/convrot-mlx
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# name, in_features, out_features, has_bias -- one ineligible input width
# (64, like FLUX's img_in), one biasless linear, one 512-wide input
LINEARS = [
    ("img_in", 64, 32, True),
    ("double_blocks.0.img_attn.qkv", 256, 96, True),
    ("double_blocks.0.img_mlp.0", 256, 128, True),
    ("double_blocks.0.img_mlp.2", 512, 64, True),
    ("single_blocks.0.linear1", 256, 160, False),
    ("final_layer.linear", 256, 64, True),
]
EXTRA = [("double_blocks.0.img_attn.norm.query_norm.scale", (32,))]
SEED = 2026120201
FLUX_SOURCE_BYTES = 23_802_932_552


def _install_stubs(shim):
    """``mlx.core`` load/save, ``mlx.utils`` and the ``flux`` example modules."""

    import torch
    from safetensors import safe_open
    from safetensors.torch import save_file

    def to_torch(a):
        if a.dtype is shim.bfloat16:
            return torch.from_numpy(np.ascontiguousarray(a._v, dtype=np.float32)).to(torch.bfloat16)
        if a.dtype is shim.float16:
            return torch.from_numpy(np.ascontiguousarray(a._v, dtype=np.float32)).to(torch.float16)
        return torch.from_numpy(np.ascontiguousarray(np.asarray(a)))

    def from_torch(t):
        if t.dtype == torch.bfloat16:
            return shim.array(t.float().numpy()).astype(shim.bfloat16)
        if t.dtype == torch.float16:
            return shim.array(t.float().numpy()).astype(shim.float16)
        return shim.array(t.numpy())

    def load(path, return_metadata=False):
        with safe_open(str(path), framework="pt") as f:
            meta = f.metadata() or {}
            weights = {k: from_torch(f.get_tensor(k)) for k in f.keys()}
        return (weights, meta) if return_metadata else weights

    def save_safetensors(path, weights, metadata=None):
        save_file({k: to_torch(v) for k, v in weights.items()}, str(path), metadata=metadata)

    shim.load = load
    shim.save_safetensors = save_safetensors
    shim.clear_cache = lambda: None
    shim.synchronize = lambda: None

    utils = types.ModuleType("mlx.utils")
    utils.tree_flatten = lambda tree: list(tree.items())
    utils.tree_unflatten = lambda items: dict(items)
    sys.modules["mlx.utils"] = utils
    sys.modules["mlx"].utils = utils

    class TinyFlux(shim._Module):
        """The fixture topology, exposing what convert.py uses of Flux."""

        def __init__(self, params=None):
            super().__init__()
            self._linears = {name: shim._Linear(k, n, bias) for name, k, n, bias in LINEARS}

        def sanitize(self, weights):
            return weights

        def parameters(self):
            names = {}
            for name, k, n, bias in LINEARS:
                names[f"{name}.weight"] = None
                if bias:
                    names[f"{name}.bias"] = None
            for name, _ in EXTRA:
                names[name] = None
            return names

        def named_modules(self):
            yield "", self
            yield from self._linears.items()

    flux = types.ModuleType("flux")
    stubs = {
        "flux.model": {"Flux": TinyFlux},
        "flux.utils": {"configs": {"flux-dev": types.SimpleNamespace(params=None, ae_params=None)}},
        "flux.autoencoder": {"AutoEncoder": object},
        "flux.clip": {"CLIPTextModel": object, "CLIPTextModelConfig": object},
        "flux.flux": {"FluxPipeline": object},
        "flux.sampler": {"FluxSampler": object},
        "flux.t5": {"T5Config": object, "T5Encoder": object},
        "flux.tokenizers": {"CLIPTokenizer": object, "T5Tokenizer": object},
    }
    sys.modules["flux"] = flux
    for mod_name, attrs in stubs.items():
        mod = types.ModuleType(mod_name)
        for k, v in attrs.items():
            setattr(mod, k, v)
        sys.modules[mod_name] = mod
        setattr(flux, mod_name.split(".")[1], mod)


class _FluxSizedPath(type(Path())):
    """A real path whose stat() reports the FLUX.1 Dev source byte count."""

    def stat(self, *, follow_symlinks=True):
        st = os.stat(self, follow_symlinks=follow_symlinks)
        fields = list(st)
        fields[6] = FLUX_SOURCE_BYTES  # st_size
        return os.stat_result(fields)


def _sha(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="checkout of Lumenbeing/convrot-mlx")
    parser.add_argument("--out", default=str(HERE))
    args = parser.parse_args()

    import torch
    from safetensors.torch import save_file

    sys.path.insert(0, str(HERE))
    import _mlx_numpy_shim as shim

    shim.install()
    _install_stubs(shim)
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "src"))
    sys.path.insert(0, str(ref))
    from examples.flux1_dev import convert as ref_convert  # the reference, unchanged
    from examples.flux1_dev import repack_mpp as ref_repack

    out = Path(args.out)
    rng = np.random.default_rng(SEED)
    source = {}
    for name, k, n, bias in LINEARS:
        source[f"{name}.weight"] = torch.from_numpy((rng.normal(size=(n, k)) * 0.02).astype(np.float32)).to(
            torch.bfloat16)
        if bias:
            source[f"{name}.bias"] = torch.from_numpy((rng.normal(size=(n,)) * 0.01).astype(np.float32)).to(
                torch.bfloat16)
    for name, shape in EXTRA:
        source[name] = torch.from_numpy((1.0 + rng.normal(size=shape) * 0.1).astype(np.float32)).to(torch.bfloat16)
    src_path = out / "ckpt_source.safetensors"
    save_file(source, str(src_path))

    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        nk_tmp, mpp_tmp = tmp / "nk.safetensors", tmp / "mpp.safetensors"
        ref_convert.convert(_FluxSizedPath(src_path), nk_tmp, tmp / "conversion.json", "fixture-runtime",
                            skip_source_hash=True, logical_output=None)
        ref_repack.repack(nk_tmp, mpp_tmp, tmp / "repack.json", skip_source_hash=True)
        (out / "ckpt_nk.safetensors").write_bytes(nk_tmp.read_bytes())
        (out / "ckpt_mpp.safetensors").write_bytes(mpp_tmp.read_bytes())

    manifest = {
        "generator": "tests/golden/make_checkpoint_golden.py",
        "reference_scripts": ["examples/flux1_dev/convert.py:convert", "examples/flux1_dev/repack_mpp.py:repack"],
        "seed": SEED,
        "linears": [list(x) for x in LINEARS],
        "extra": [[n, list(s)] for n, s in EXTRA],
        "sha256": {p: _sha(out / p) for p in ("ckpt_source.safetensors", "ckpt_nk.safetensors",
                                               "ckpt_mpp.safetensors")},
    }
    (out / "ckpt_manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
