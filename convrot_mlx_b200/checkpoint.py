"""The reference's on-disk ConvRot checkpoint format: safetensors files with
packed W4 linears and string metadata, read and written interchangeably with
Lumenbeing/convrot-mlx.

Two schemas (``examples/flux1_dev/adapter.py:25-29``):

* ``convrot-mlx.flux1-convrot-w4a4.v1`` -- written by the reference's
  converter (``examples/flux1_dev/convert.py:124-177``).  Every converted
  linear ``{name}`` stores ``{name}.qweight`` (N x packed-K uint8, element
  2j in the low nibble), ``{name}.scales`` (N float32) and ``{name}.bias``
  (N float32; zeros when the source linear had none).  Tensors of
  unconverted modules pass through in their source dtype.
* ``convrot-mlx.flux1-convrot-w4-mpp.v1`` -- the lossless K x packed-N
  repack of the same checkpoint (``examples/flux1_dev/repack_mpp.py:
  105-151``): only the qweights change, and the metadata gains the layout
  keys.

``load_convrot_model`` is the torch counterpart of ``load_flow_convrot``
(``adapter.py:73-107``): it checks the metadata the same way (schema for the
backend, MPP weight layout, source digest, group size, converted-layer
count), swaps the model's eligible linears for ``ConvRotLinear`` and loads
every tensor strictly.  Conversion and repacking run on the GPU kernels of
this package (``quantize_convrot_weight``, ``repack_nk_weight_for_mpp``);
reading, writing and validation need no GPU.
"""

from __future__ import annotations

from pathlib import Path

import torch
from torch import nn

from .core import (
    CONVROT_GROUP_SIZE,
    eligible_linear,
    quantize_convrot_weight,
    repack_mpp_weight_to_nk,
    repack_nk_weight_for_mpp,
)

# Format constants of the reference (adapter.py:25-30, convert.py:154-175,
# repack_mpp.py:138-151): they are what makes the files interchangeable.
CONVROT_SCHEMA = "convrot-mlx.flux1-convrot-w4a4.v1"
CONVROT_MPP_SCHEMA = "convrot-mlx.flux1-convrot-w4-mpp.v1"
CONVROT_MPP_WEIGHT_LAYOUT = "signed_twos_complement_low_nibble_even_output_k_by_packed_n"
PACKING_NK = "signed_twos_complement_low_nibble_even_column"
PACKING_KN = "signed_twos_complement_low_nibble_even_output"
# Digest of the FLUX.1 Dev transformer file the reference converts (adapter.py:30).
FLUX1_DEV_SOURCE_SHA256 = "4610115bb0c89560703c892c59ac2742fa821e60ef5871b33493ba544683abd7"

# Metadata of the quantization algorithm itself (convert.py:41-50, :165-173).
ALGORITHM_METADATA = {
    "weight_bits": "4",
    "activation_bits": "4",
    "weight_scale": "rowwise_absmax_div_7",
    "activation_scale": "rowwise_absmax_div_7",
    "packing": PACKING_NK,
}


# ---------------------------------------------------------------------------
# files


def read_checkpoint(path: str | Path) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """All tensors (on the CPU) and the string metadata of a safetensors file."""

    from safetensors import safe_open

    with safe_open(str(path), framework="pt") as f:
        metadata = dict(f.metadata() or {})
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    return tensors, metadata


def write_checkpoint(path: str | Path, tensors: dict[str, torch.Tensor], metadata: dict[str, str]) -> None:
    """Write a safetensors checkpoint; like the reference's scripts, never
    overwrite an existing file (convert.py:65-68, repack_mpp.py:94-95)."""

    from safetensors.torch import save_file

    path = Path(path)
    if path.exists() or path.is_symlink():
        raise FileExistsError(f"Refusing to overwrite existing ConvRot checkpoint: {path}")
    bad = [k for k, v in metadata.items() if not isinstance(k, str) or not isinstance(v, str)]
    if bad:
        raise ValueError(f"checkpoint metadata must map strings to strings; offending keys: {bad[:4]}")
    path.parent.mkdir(parents=True, exist_ok=True)
    save_file({k: v.detach().contiguous().cpu() for k, v in tensors.items()}, str(path), metadata=metadata)


# ---------------------------------------------------------------------------
# conversion (dense -> N x packed-K) and repack (-> K x packed-N)


def convrot_metadata(*, converted_linear_count: int, linear_count: int, group_size: int = CONVROT_GROUP_SIZE,
                     source_sha256: str = FLUX1_DEV_SOURCE_SHA256, **provenance: str) -> dict[str, str]:
    """Metadata of an N x packed-K checkpoint, with the keys the reference's
    converter writes (convert.py:154-175).  ``provenance`` adds or overrides
    string keys such as ``source_bytes`` or ``runtime_revision``."""

    meta = {
        "schema": CONVROT_SCHEMA,
        "source_sha256": source_sha256,
        "convrot_group_size": str(group_size),
        "quant_group_size": "64",
        "reference_algorithm": "plain ConvRot W4A4 eager contract",
        **ALGORITHM_METADATA,
        "converted_linear_count": str(converted_linear_count),
        "linear_count": str(linear_count),
        # descriptive strings of the reference's Metal execution, kept so the
        # files carry the same metadata
        "metal_execution": "packed operands; per-tile int4-to-half expansion; simdgroup half MMA; float accumulation",
        "native_int4_mma": "false",
    }
    meta.update({k: str(v) for k, v in provenance.items()})
    return meta


def convert_state_dict(state: dict[str, torch.Tensor], linear_names: list[str], *,
                       group_size: int = CONVROT_GROUP_SIZE, device=None) -> dict[str, torch.Tensor]:
    """Quantize the named dense linears of a state dict (convert.py:124-150).

    For each name, ``{name}.weight`` (N, K) becomes ``{name}.qweight`` and
    ``{name}.scales`` (quantize_convrot_weight on the GPU) and ``{name}.bias``
    becomes float32 (zeros when absent).  Every other tensor passes through
    unchanged; every source tensor is consumed exactly once.  Linears whose
    in_features is not a multiple of ``group_size`` are rejected."""

    device = torch.device("cuda") if device is None else torch.device(device)
    remaining = dict(state)
    out: dict[str, torch.Tensor] = {}
    for name in linear_names:
        weight = remaining.pop(f"{name}.weight")
        if weight.ndim != 2 or weight.shape[1] % group_size:
            raise ValueError(f"{name}: weight {tuple(weight.shape)} is not a ConvRot-eligible linear")
        qweight, scales = quantize_convrot_weight(weight.to(device), group_size)
        out[f"{name}.qweight"] = qweight.cpu()
        out[f"{name}.scales"] = scales.cpu()
        bias = remaining.pop(f"{name}.bias", None)
        out[f"{name}.bias"] = (torch.zeros(weight.shape[0], dtype=torch.float32) if bias is None
                               else bias.detach().to(torch.float32).cpu())
    out.update(remaining)
    return out


def convert_model(model: nn.Module, *, group_size: int = CONVROT_GROUP_SIZE, device=None,
                  **provenance: str) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """Convert every eligible ``nn.Linear`` of a dense torch model (the
    selection of convert.py:114-123) into checkpoint tensors and metadata."""

    linears = [name for name, m in model.named_modules() if isinstance(m, nn.Linear)]
    selected = [name for name, m in model.named_modules() if name and eligible_linear(m, group_size)]
    state = {k: v.detach() for k, v in model.state_dict().items()}
    tensors = convert_state_dict(state, selected, group_size=group_size, device=device)
    meta = convrot_metadata(converted_linear_count=len(selected), linear_count=len(linears), group_size=group_size,
                            **provenance)
    return tensors, meta


def repack_checkpoint_for_mpp(tensors: dict[str, torch.Tensor], metadata: dict[str, str], *,
                              device=None) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """The lossless N x packed-K -> K x packed-N repack of a whole checkpoint
    (repack_mpp.py:105-151): every ``.qweight`` is transposed on the GPU and
    must round-trip bit for bit; scales, biases and unconverted tensors are
    untouched; the metadata gains the MPP schema and layout keys."""

    validate_checkpoint_metadata(metadata, "reference", require_source=None)
    device = torch.device("cuda") if device is None else torch.device(device)
    names = sorted(k for k in tensors if k.endswith(".qweight"))
    expected = int(metadata.get("converted_linear_count", "-1"))
    if len(names) != expected:
        raise ValueError(f"Found {len(names)} qweights; metadata expects {expected}")
    out = dict(tensors)
    for name in names:
        packed_nk = tensors[name].to(device)
        packed_kn = repack_nk_weight_for_mpp(packed_nk)
        if not torch.equal(repack_mpp_weight_to_nk(packed_kn), packed_nk):
            raise RuntimeError(f"Bit-exact MPP repack gate failed for {name}")
        out[name] = packed_kn.cpu()
    meta = dict(metadata)
    meta.update({
        "schema": CONVROT_MPP_SCHEMA,
        "source_convrot_sha256": metadata.get("source_convrot_sha256", "skipped"),
        "weight_layout": CONVROT_MPP_WEIGHT_LAYOUT,
        "packing": PACKING_KN,
        "activation_bits": "4-or-16-runtime-selected",
        "supported_activation_modes": "a4-values-in-int8,bfloat16,float16",
        "metal_execution": "Metal 4 MPP TensorOps int8-or-float x packed signed-int4",
        "native_int4_mma": "true",
        "lossless_layout_repack": "true",
    })
    return out, meta


# ---------------------------------------------------------------------------
# loading


def validate_checkpoint_metadata(metadata: dict[str, str], backend: str, *,
                                 require_source: str | None = FLUX1_DEV_SOURCE_SHA256,
                                 group_size: int = CONVROT_GROUP_SIZE) -> None:
    """The checks of ``load_flow_convrot`` (adapter.py:77-95), with the same
    messages: the schema must match the backend's weight layout, an MPP
    checkpoint must declare the K x packed-N layout, the source digest must
    match ``require_source`` (None skips that check: a model other than FLUX.1
    Dev) and the group size must match."""

    uses_mpp = backend.startswith("mpp-")
    expected_schema = CONVROT_MPP_SCHEMA if uses_mpp else CONVROT_SCHEMA
    if metadata.get("schema") != expected_schema:
        raise ValueError(
            f"ConvRot backend {backend!r} requires checkpoint schema {expected_schema!r}; "
            f"found {metadata.get('schema')!r}"
        )
    if uses_mpp and metadata.get("weight_layout") != CONVROT_MPP_WEIGHT_LAYOUT:
        raise ValueError(f"MPP ConvRot checkpoint has unsupported weight layout: {metadata.get('weight_layout')!r}")
    if require_source is not None and metadata.get("source_sha256") != require_source:
        raise ValueError("ConvRot checkpoint does not derive from the supported FLUX.1 Dev source digest.")
    if int(metadata.get("convrot_group_size", "0")) != group_size:
        raise ValueError("ConvRot checkpoint group size does not match this runtime.")


def load_convrot_model(model: nn.Module, path: str | Path, *, backend: str = "mpp-w4a4",
                       preprocessor: str = "metal-fused", require_source: str | None = FLUX1_DEV_SOURCE_SHA256,
                       device=None) -> tuple[nn.Module, dict[str, str], list[str]]:
    """Load a converted checkpoint into a dense torch model (adapter.py:73-107).

    Validates the metadata for ``backend``, replaces the model's eligible
    linears by empty ``ConvRotLinear`` layers (``replace_convrot_linears``
    with ``quantize=False``), checks the converted-layer count, then loads
    every tensor with ``strict=True``.  Returns (model, metadata, replaced
    names)."""

    from .adapter import replace_convrot_linears

    tensors, metadata = read_checkpoint(path)
    validate_checkpoint_metadata(metadata, backend, require_source=require_source)
    names = replace_convrot_linears(model, backend=backend, preprocessor=preprocessor,
                                    group_size=int(metadata["convrot_group_size"]), quantize=False)
    if int(metadata.get("converted_linear_count", "-1")) != len(names):
        raise ValueError("ConvRot checkpoint layer count does not match the model topology.")
    if device is None:
        device = next((t.device for t in model.parameters()), None) or next(
            (b.device for b in model.buffers()), torch.device("cpu"))
    model.load_state_dict({k: v.to(device) for k, v in tensors.items()}, strict=True)
    return model, metadata, names


__all__ = [
    "ALGORITHM_METADATA",
    "CONVROT_MPP_SCHEMA",
    "CONVROT_MPP_WEIGHT_LAYOUT",
    "CONVROT_SCHEMA",
    "FLUX1_DEV_SOURCE_SHA256",
    "PACKING_KN",
    "PACKING_NK",
    "convert_model",
    "convert_state_dict",
    "convrot_metadata",
    "load_convrot_model",
    "read_checkpoint",
    "repack_checkpoint_for_mpp",
    "validate_checkpoint_metadata",
    "write_checkpoint",
]
