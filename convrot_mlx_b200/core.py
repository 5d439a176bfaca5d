"""ConvRot W4A4 primitives for B200 (sm_100a), with the reference's Python API.

This module mirrors the public surface of Lumenbeing/convrot-mlx
(``src/convrot_mlx/core.py``): the same function names, arguments, constants,
backend strings and ``ValueError`` messages, over ``torch.Tensor`` on CUDA
instead of ``mx.array``.  Every function runs the hand-written sm_100a kernels
of ``libconvrot_b200.so`` through its C ABI (``include/convrot_b200.h``);
there is no CPU path: CPU tensors are rejected.

Backends (``ConvRotLinear(backend=...)``, core.py:36-47):
  * ``mpp-w4a4`` (default) -- K x packed-N weights; fused prep writes int8
    codes, then one tcgen05 ``kind::i8`` GEMM with the epilogue fused.
  * ``mpp-w4a16`` -- K x packed-N weights; rotated bf16/fp16 activations,
    tcgen05 ``kind::f16`` GEMM.
  * ``metal``, ``metal-k32``, ``metal-k64``, ``metal-m32n32-k64``,
    ``mlx-expanded-fp32``, ``reference`` -- N x packed-K weights; the same
    fused prep and the same W4A4 GEMM reading the NK layout (the reference's
    variants differ only in Apple-specific tiling; their math is identical,
    reference tests core :139-175, :266-283, :329-355).
The ``preprocessor`` argument is accepted and validated; both reference
preprocessors are bitwise equal (reference tests :54-74), and one fused CUDA
kernel serves both.
"""

from __future__ import annotations

import os

import torch
from torch import nn

from . import _lib

CONVROT_GROUP_SIZE = 256
SUPPORTED_FUSED_GROUP_SIZES = frozenset({64, 256})
INT4_MAX = 7
SUPPORTED_BACKENDS = frozenset(
    {
        "metal",
        "metal-k32",
        "metal-k64",
        "metal-m32n32-k64",
        "mpp-w4a4",
        "mpp-w4a16",
        "mlx-expanded-fp32",
        "reference",
    }
)
SUPPORTED_PREPROCESSORS = frozenset({"mlx-compiled", "metal-fused"})

_KN_BACKENDS = frozenset({"mpp-w4a4", "mpp-w4a16"})


# ---------------------------------------------------------------------------
# helpers


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(
                "convrot_mlx_b200 runs on CUDA (sm_100a) only; got a tensor on "
                f"{t.device} (there is no CPU fallback)"
            )


def _dtype_code(dtype: torch.dtype) -> int:
    try:
        return _lib.DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def _validate_group_size(group_size: int) -> None:
    """core.py:50-61."""

    if group_size < 4:
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {group_size}")
    value = group_size
    while value > 1 and value % 4 == 0:
        value //= 4
    if value != 1:
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {group_size}")


def _f32_vec(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float32).contiguous()


# ---------------------------------------------------------------------------
# rotation and quantization (activations and weights)


def regular_hadamard(x: torch.Tensor, group_size: int = CONVROT_GROUP_SIZE) -> torch.Tensor:
    """Right-multiply each feature group by the normalized regular Hadamard.

    core.py:64-94: radix-4 butterfly with per-op rounding in ``x.dtype``.  H is
    symmetric, so the same routine rotates activations (``x @ H``) and weights
    (``W @ H.T``).
    """

    _validate_group_size(group_size)
    features = x.shape[-1]
    if features % group_size:
        raise ValueError(f"features {features} not divisible by ConvRot group size {group_size}")
    _require_cuda(x)
    x2 = x.reshape(-1, features).contiguous()
    out = torch.empty_like(x2)
    lib = _lib.load()
    _lib.check(
        lib.convrot_rotate(_lib.ptr(x2), _dtype_code(x2.dtype), x2.shape[0], features, group_size,
                           _lib.ptr(out), _lib.stream_of(x2)),
        "regular_hadamard",
    )
    return out.reshape(x.shape)


def pack_signed_int4(values: torch.Tensor) -> torch.Tensor:
    """core.py:97-105: two's-complement nibbles, low column first."""

    if values.shape[-1] % 2:
        raise ValueError(f"last dimension must be even, got {values.shape[-1]}")
    _require_cuda(values)
    v = values.to(torch.int8).contiguous()
    out = torch.empty((*values.shape[:-1], values.shape[-1] // 2), dtype=torch.uint8, device=values.device)
    _lib.check(_lib.load().convrot_pack_int4(_lib.ptr(v), v.numel(), _lib.ptr(out), _lib.stream_of(v)),
               "pack_signed_int4")
    return out


def unpack_signed_int4(packed: torch.Tensor) -> torch.Tensor:
    """core.py:108-120: nibbles to int8 in [-8, 7]."""

    _require_cuda(packed)
    p = packed.to(torch.uint8).contiguous()
    out = torch.empty((*packed.shape[:-1], packed.shape[-1] * 2), dtype=torch.int8, device=packed.device)
    _lib.check(_lib.load().convrot_unpack_int4(_lib.ptr(p), p.numel(), _lib.ptr(out), _lib.stream_of(p)),
               "unpack_signed_int4")
    return out


def metal_unpack_signed_int4(packed: torch.Tensor) -> torch.Tensor:
    """core.py:1014-1027 (same kernel as ``unpack_signed_int4``; 2-D only)."""

    if packed.ndim != 2:
        raise ValueError(f"Metal int4 unpack expects a 2D tensor, got {tuple(packed.shape)}")
    return unpack_signed_int4(packed)


def _repack_transpose(qweight: torch.Tensor, odd_message: str) -> torch.Tensor:
    if qweight.ndim != 2:
        raise ValueError(f"MPP weight repack expects a 2D tensor, got {tuple(qweight.shape)}")
    rows, packed_cols = qweight.shape
    if rows % 2:
        raise ValueError(odd_message.format(rows))
    _require_cuda(qweight)
    q = qweight.contiguous()
    out = torch.empty((2 * packed_cols, rows // 2), dtype=torch.uint8, device=q.device)
    _lib.check(
        _lib.load().convrot_repack_int4_transpose(_lib.ptr(q), rows, packed_cols, _lib.ptr(out), _lib.stream_of(q)),
        "repack",
    )
    return out


def repack_nk_weight_for_mpp(qweight: torch.Tensor) -> torch.Tensor:
    """core.py:123-133: bit-exact N x packed-K -> K x packed-N."""

    return _repack_transpose(qweight, "MPP int4 packing requires even out_features, got {}")


def repack_mpp_weight_to_nk(qweight: torch.Tensor) -> torch.Tensor:
    """core.py:136-146: K x packed-N -> N x packed-K."""

    return _repack_transpose(qweight, "row-major int4 packing requires even in_features, got {}")


def _prepare(x: torch.Tensor, group_size: int, packed: bool) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda(x)
    x = x.contiguous()
    rows, features = x.shape
    if packed:
        q = torch.empty((rows, features // 2), dtype=torch.uint8, device=x.device)
        fn = _lib.load().convrot_prepare_packed
    else:
        q = torch.empty((rows, features), dtype=torch.int8, device=x.device)
        fn = _lib.load().convrot_prepare_i8
    scales = torch.empty((rows,), dtype=torch.float32, device=x.device)
    _lib.check(
        fn(_lib.ptr(x), _dtype_code(x.dtype), rows, features, group_size, _lib.ptr(q), _lib.ptr(scales),
           _lib.stream_of(x)),
        "ConvRot activation preparation",
    )
    return q, scales


def quantize_signed_int4_rowwise(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """core.py:149-158: symmetric absmax/7 row quantization (no rotation)."""

    if x.ndim != 2:
        raise ValueError(f"rowwise int4 quantization expects 2D input, got {tuple(x.shape)}")
    return _prepare(x, 1, packed=True)


def prepare_convrot_activation(
    x: torch.Tensor, group_size: int = CONVROT_GROUP_SIZE
) -> tuple[torch.Tensor, torch.Tensor]:
    """core.py:161-167: rotate and row-quantize (one fused kernel)."""

    _validate_group_size(group_size)
    if x.shape[-1] % group_size:
        raise ValueError(f"features {x.shape[-1]} not divisible by ConvRot group size {group_size}")
    if x.ndim != 2:
        raise ValueError(f"rowwise int4 quantization expects 2D input, got {tuple(x.shape)}")
    return _prepare(x, group_size, packed=True)


# The reference compiles the eager graph (core.py:174-175); here the eager
# contract already is one fused kernel.
compiled_prepare_convrot_activation = prepare_convrot_activation
compiled_regular_hadamard = regular_hadamard


def _validate_fused(x: torch.Tensor, group_size: int, what: str) -> None:
    if x.ndim != 2:
        raise ValueError(f"fused ConvRot {what} expects 2D input, got {tuple(x.shape)}")
    if group_size not in SUPPORTED_FUSED_GROUP_SIZES:
        raise ValueError(
            f"fused ConvRot {what} supports groups {sorted(SUPPORTED_FUSED_GROUP_SIZES)}, got {group_size}"
        )
    if x.shape[1] % group_size:
        raise ValueError(f"features {x.shape[1]} not divisible by ConvRot group size {group_size}")


def metal_fused_prepare_convrot_activation(
    x: torch.Tensor, group_size: int = CONVROT_GROUP_SIZE
) -> tuple[torch.Tensor, torch.Tensor]:
    """core.py:425-453: fused Hadamard, row absmax, A4 quantize, and pack."""

    _validate_fused(x, group_size, "activation preparation")
    return _prepare(x, group_size, packed=True)


def metal_fused_prepare_convrot_activation_i8(
    x: torch.Tensor, group_size: int = CONVROT_GROUP_SIZE
) -> tuple[torch.Tensor, torch.Tensor]:
    """core.py:456-484: rotate and A4-quantize straight into int8 codes."""

    _validate_fused(x, group_size, "activation preparation")
    return _prepare(x, group_size, packed=False)


def metal_fused_rotate_convrot_activation(x: torch.Tensor, group_size: int = CONVROT_GROUP_SIZE) -> torch.Tensor:
    """core.py:487-511: rotation only, in one pass (W4A16 path)."""

    _validate_fused(x, group_size, "rotation")
    return regular_hadamard(x, group_size)


def quantize_convrot_weight(
    weight: torch.Tensor, group_size: int = CONVROT_GROUP_SIZE
) -> tuple[torch.Tensor, torch.Tensor]:
    """core.py:514-527: rotate a dense (out, in) weight, store it as packed W4 (NK)."""

    if weight.ndim != 2:
        raise ValueError(f"ConvRot weight must be 2D, got {tuple(weight.shape)}")
    if weight.shape[-1] % group_size:
        raise ValueError(
            f"in_features {weight.shape[-1]} not divisible by ConvRot group size {group_size}"
        )
    _validate_group_size(group_size)
    return _prepare(weight, group_size, packed=True)


def _mod_vectors(v: torch.Tensor, batch: int, features: int) -> tuple[torch.Tensor, int]:
    """A (batch, [1,] features) modulation vector as (tensor, sample stride)
    that the fused kernel can read: unit stride along features, 16-byte
    aligned, sample stride a multiple of 8 elements (else a packed copy)."""

    v2 = v.reshape(v.shape[0], v.shape[-1]) if v.ndim == 3 else v
    if v2.ndim != 2 or v2.shape[-1] != features or v2.shape[0] not in (1, batch):
        raise ValueError(f"modulation vector of shape {tuple(v.shape)} does not match ({batch}, 1, {features})")
    if v2.shape[0] == 1 and batch > 1:
        v2 = v2.expand(batch, features)
    stride = v2.stride(0)
    if v2.stride(1) != 1 or stride % 8 or v2.data_ptr() % 16 or v2.dtype != torch.bfloat16:
        v2 = v2.to(torch.bfloat16).contiguous()
        stride = features
    return v2, stride


def modulated_norm_prepare_i8(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6,
                              group_size: int = CONVROT_GROUP_SIZE) -> tuple[torch.Tensor, torch.Tensor]:
    """int8 codes and row scales of ``prepare(addcmul(shift, layer_norm(x), 1 + scale))``
    in one kernel (``convrot_modnorm_prepare_i8``).  x: (batch, tokens,
    features) or (rows, features) bf16 (then one modulation row); returns
    codes (rows, features) int8 and scales (rows,) float32."""

    _require_cuda(x, shift, scale)
    if x.dtype != torch.bfloat16:
        raise ValueError(f"the fused modulated-norm prep takes bfloat16 activations, got {x.dtype}")
    features = x.shape[-1]
    x3 = x.reshape(1, -1, features) if x.ndim == 2 else x.reshape(x.shape[0], -1, features)
    batch, tokens = x3.shape[0], x3.shape[1]
    x2 = x3.reshape(-1, features).contiguous()
    sh, sh_stride = _mod_vectors(shift, batch, features)
    sc, sc_stride = _mod_vectors(scale, batch, features)
    if sh_stride != sc_stride:
        sh, sc = sh.contiguous(), sc.contiguous()
        sh_stride = sc_stride = features
    rows = x2.shape[0]
    codes = torch.empty((rows, features), dtype=torch.int8, device=x.device)
    scales = torch.empty((rows,), dtype=torch.float32, device=x.device)
    _lib.check(
        _lib.load().convrot_modnorm_prepare_i8(
            _lib.ptr(x2), _lib.BF16, rows, features, group_size, _lib.ptr(sh), _lib.ptr(sc), max(tokens, 1),
            sh_stride, float(eps), _lib.ptr(codes), _lib.ptr(scales), _lib.stream_of(x2)),
        "modulated-norm activation preparation",
    )
    return codes, scales


def gelu_concat_prepare_i8(a: torch.Tensor, m: torch.Tensor,
                           group_size: int = CONVROT_GROUP_SIZE) -> tuple[torch.Tensor, torch.Tensor]:
    """int8 codes and row scales of ``prepare(cat(a, gelu_tanh(m), -1))`` in one
    kernel (``convrot_gelu_concat_prepare_i8``), reading a and m in place: a
    (batch, tokens, da) and m (batch, tokens, dm) bf16, each with unit stride
    along its last dimension (m may be a column slice of a wider tensor)."""

    _require_cuda(a, m)
    if a.dtype != torch.bfloat16 or m.dtype != torch.bfloat16:
        raise ValueError("the fused GELU-concatenation prep takes bfloat16 tensors")
    if a.shape[:-1] != m.shape[:-1]:
        raise ValueError(f"leading shapes differ: {tuple(a.shape)} and {tuple(m.shape)}")
    da, dm = a.shape[-1], m.shape[-1]
    a2 = a.reshape(-1, da)
    m2 = m.reshape(-1, dm)
    if a2.stride(-1) != 1 or a2.stride(0) % 8 or a2.data_ptr() % 16:
        a2 = a2.contiguous()
    if m2.stride(-1) != 1 or m2.stride(0) % 8 or m2.data_ptr() % 16:
        m2 = m2.contiguous()
    rows = a2.shape[0]
    codes = torch.empty((rows, da + dm), dtype=torch.int8, device=a.device)
    scales = torch.empty((rows,), dtype=torch.float32, device=a.device)
    _lib.check(
        _lib.load().convrot_gelu_concat_prepare_i8(
            _lib.ptr(a2), a2.stride(0), da, _lib.ptr(m2), m2.stride(0), dm, rows, group_size, _lib.ptr(codes),
            _lib.ptr(scales), _lib.stream_of(a2)),
        "GELU-concatenation activation preparation",
    )
    return codes, scales


# ---------------------------------------------------------------------------
# GEMMs


def _gemm_w4a4(act_i8, qweight, layout, xscales, wscales, bias, output_dtype, m, n, k) -> torch.Tensor:
    _require_cuda(act_i8, qweight, xscales, wscales, bias)
    out_code = _dtype_code(output_dtype)
    a = act_i8.contiguous()
    w = qweight.contiguous()
    xs = _f32_vec(xscales)
    ws = _f32_vec(wscales)
    b = None if bias is None else _f32_vec(bias)
    out = torch.empty((m, n), dtype=output_dtype, device=a.device)
    _lib.check(
        _lib.load().convrot_w4a4_gemm(
            _lib.ptr(a), _lib.ptr(w), layout, _lib.ptr(xs), _lib.ptr(ws), _lib.ptr(b), _lib.ptr(out),
            out_code, m, n, k, _lib.stream_of(a),
        ),
        "W4A4 GEMM",
    )
    return out


def _validate_mpp_weight_layout(qweight: torch.Tensor, k: int) -> int:
    """core.py:1030-1039."""

    if qweight.ndim != 2:
        raise ValueError(f"MPP W4 weight must be 2D, got {tuple(qweight.shape)}")
    if qweight.shape[0] != k:
        raise ValueError(
            f"MPP W4 weight must use K x packed-N layout; activation K={k}, weight={tuple(qweight.shape)}"
        )
    if k % 32:
        raise ValueError(f"MPP W4 TensorOp requires K divisible by 32, got {k}")
    return qweight.shape[1] * 2


def _validate_mpp_epilogue(m, n, xscales, wscales, bias) -> None:
    """core.py:1042-1058."""

    if xscales is not None and tuple(xscales.shape) != (m,):
        raise ValueError(f"MPP activation scales must have shape {(m,)}, got {tuple(xscales.shape)}")
    if tuple(wscales.shape) != (n,):
        raise ValueError(f"MPP weight scales must have shape {(n,)}, got {tuple(wscales.shape)}")
    if tuple(bias.shape) != (n,):
        raise ValueError(f"MPP bias must have shape {(n,)}, got {tuple(bias.shape)}")


def mpp_w4a4_int8_matmul(activations, qweight, xscales, wscales, bias, *, output_dtype) -> torch.Tensor:
    """core.py:1088-1120: int8 codes x K x packed-N weights, fused epilogue."""

    if activations.ndim != 2 or activations.dtype != torch.int8:
        raise ValueError(
            f"MPP W4A4 requires a 2D int8 activation, got {tuple(activations.shape)} {activations.dtype}"
        )
    m, k = activations.shape
    n = _validate_mpp_weight_layout(qweight, k)
    _validate_mpp_epilogue(m, n, xscales, wscales, bias)
    return _gemm_w4a4(activations, qweight, _lib.LAYOUT_KN, xscales, wscales, bias, output_dtype, m, n, k)


def mpp_w4a4_matmul(qact, qweight, xscales, wscales, bias, *, output_dtype) -> torch.Tensor:
    """core.py:1061-1085: packed A4 activations, unpacked to int8, then the GEMM."""

    if qact.ndim != 2:
        raise ValueError(f"MPP W4A4 activation must be 2D, got {tuple(qact.shape)}")
    m, k = qact.shape[0], qact.shape[1] * 2
    n = _validate_mpp_weight_layout(qweight, k)
    _validate_mpp_epilogue(m, n, xscales, wscales, bias)
    return mpp_w4a4_int8_matmul(
        metal_unpack_signed_int4(qact), qweight, xscales, wscales, bias, output_dtype=output_dtype
    )


def mpp_w4a16_matmul(activations, qweight, wscales, bias, *, output_dtype) -> torch.Tensor:
    """core.py:1123-1152: rotated bf16/fp16 activations x K x packed-N weights."""

    if activations.ndim != 2:
        raise ValueError(f"MPP W4A16 activation must be 2D, got {tuple(activations.shape)}")
    if activations.dtype not in {torch.float16, torch.bfloat16}:
        raise ValueError(
            f"MPP W4A16 requires float16 or bfloat16 activation, got {activations.dtype}"
        )
    m, k = activations.shape
    n = _validate_mpp_weight_layout(qweight, k)
    _validate_mpp_epilogue(m, n, None, wscales, bias)
    return _gemm_w4a16(activations, qweight, _lib.LAYOUT_KN, wscales, bias, output_dtype, m, n, k)


def _gemm_w4a16(act, qweight, layout, wscales, bias, output_dtype, m, n, k) -> torch.Tensor:
    lib = _lib.load()
    _require_cuda(act, qweight, wscales, bias)
    a = act.contiguous()
    w = qweight.contiguous()
    ws = _f32_vec(wscales)
    b = None if bias is None else _f32_vec(bias)
    # The tcgen05 kernel reads 64-value K chunks and, for K x packed-N
    # weights, 16-byte weight rows (N % 32 == 0).  Ragged shapes are padded
    # with zeros on the device (zero codes add nothing to a dot) and the
    # output is cut back to N.
    kp = -(-k // 64) * 64
    np_ = -(-n // 32) * 32 if layout == _lib.LAYOUT_KN else n
    if kp != k:
        a = torch.nn.functional.pad(a, (0, kp - k))
        w = torch.nn.functional.pad(w, (0, (kp - k) // 2)) if layout == _lib.LAYOUT_NK else \
            torch.nn.functional.pad(w, (0, 0, 0, kp - k))
    if np_ != n:
        w = torch.nn.functional.pad(w, (0, (np_ - n) // 2))
        ws = torch.nn.functional.pad(ws, (0, np_ - n))
        b = None if b is None else torch.nn.functional.pad(b, (0, np_ - n))
    out = torch.empty((m, np_), dtype=output_dtype, device=a.device)
    _lib.check(
        lib.convrot_w4a16_gemm(
            _lib.ptr(a), _dtype_code(a.dtype), _lib.ptr(w), layout, _lib.ptr(ws), _lib.ptr(b), _lib.ptr(out),
            _dtype_code(output_dtype), m, np_, kp, _lib.stream_of(a),
        ),
        "W4A16 GEMM",
    )
    return out if np_ == n else out[:, :n].contiguous()


def _validate_packed_nk(qact, qweight, what="packed W4A4"):
    if qact.ndim != 2 or qweight.ndim != 2:
        raise ValueError(f"{what} expects 2D activation and weight tensors")
    if qact.shape[1] != qweight.shape[1]:
        raise ValueError(
            f"packed K mismatch: activation {tuple(qact.shape)}, weight {tuple(qweight.shape)}"
        )


def _nk_matmul(qact, qweight, xscales, wscales, bias, output_dtype) -> torch.Tensor:
    m, n, k = qact.shape[0], qweight.shape[0], qact.shape[1] * 2
    return _gemm_w4a4(unpack_signed_int4(qact), qweight, _lib.LAYOUT_NK, xscales, wscales, bias, output_dtype,
                      m, n, k)


def packed_w4a4_matmul(qact, qweight, xscales, wscales, bias, *, output_dtype) -> torch.Tensor:
    """core.py:745-771: packed A4 x N x packed-K W4 with the fused epilogue."""

    _validate_packed_nk(qact, qweight)
    return _nk_matmul(qact, qweight, xscales, wscales, bias, output_dtype)


def packed_w4a4_matmul_staged(
    qact, qweight, xscales, wscales, bias, *, output_dtype, tile_m: int = 16, tile_n: int = 32, tile_k: int
) -> torch.Tensor:
    """core.py:774-804.  The tile arguments are validated as the reference does
    (core.py:704-719); the sm_100a kernel picks its own tcgen05 tiling."""

    if tile_m not in {16, 32} or tile_n not in {32, 64} or tile_k not in {32, 64, 128, 256}:
        raise ValueError(f"Unsupported staged tile {tile_m}x{tile_n}x{tile_k}")
    _validate_packed_nk(qact, qweight)
    return _nk_matmul(qact, qweight, xscales, wscales, bias, output_dtype)


def packed_w4a4_matmul_k32(*args, **kwargs):
    return packed_w4a4_matmul_staged(*args, **kwargs, tile_k=32)


def packed_w4a4_matmul_k64(*args, **kwargs):
    return packed_w4a4_matmul_staged(*args, **kwargs, tile_k=64)


def packed_w4a4_matmul_k128(*args, **kwargs):
    return packed_w4a4_matmul_staged(*args, **kwargs, tile_k=128)


def packed_w4a4_matmul_k256(*args, **kwargs):
    return packed_w4a4_matmul_staged(*args, **kwargs, tile_k=256)


def packed_w4a4_matmul_m32n32_k64(*args, **kwargs):
    return packed_w4a4_matmul_staged(*args, **kwargs, tile_m=32, tile_n=32, tile_k=64)


def packed_w4a4_matmul_m16n64_k64(*args, **kwargs):
    return packed_w4a4_matmul_staged(*args, **kwargs, tile_m=16, tile_n=64, tile_k=64)


def reference_w4a4_matmul(qact, qweight, xscales, wscales, bias, *, output_dtype) -> torch.Tensor:
    """core.py:1155-1171.  Same result as the eager oracle (exact integer dot,
    then ``dots * xs * ws + bias`` in float32), computed by the W4A4 GEMM."""

    _validate_packed_nk(qact, qweight, "reference W4A4")
    return _nk_matmul(qact, qweight, xscales, wscales, bias, output_dtype)


def expanded_fp32_w4a4_matmul(qact, qweight, xscales, wscales, bias, *, output_dtype) -> torch.Tensor:
    """core.py:1174-1207, including its K guard (``K * 49 < 2**24``)."""

    _validate_packed_nk(qact, qweight, "expanded W4A4")
    feature_count = qact.shape[1] * 2
    if feature_count * INT4_MAX * INT4_MAX >= 2**24:
        raise ValueError(f"K={feature_count} can exceed FP32's consecutive-integer dot range")
    return _nk_matmul(qact, qweight, xscales, wscales, bias, output_dtype)


# ---------------------------------------------------------------------------
# layer


class ConvRotLinear(nn.Module):
    """A linear layer stored and executed under the ConvRot W4A4 contract.

    core.py:1210-1313.  ``qweight``, ``scales`` and ``bias`` are buffers that
    callers assign directly (``layer.qweight = q``), as with the reference.
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        *,
        bias: bool = True,
        group_size: int = CONVROT_GROUP_SIZE,
        backend: str | None = None,
        preprocessor: str | None = None,
        device=None,
    ):
        super().__init__()
        if in_features % group_size:
            raise ValueError(
                f"in_features {in_features} not divisible by ConvRot group size {group_size}"
            )
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.backend = backend or os.getenv("CONVROT_MLX_BACKEND", "mpp-w4a4")
        if self.backend not in SUPPORTED_BACKENDS:
            raise ValueError(
                f"Unknown ConvRot backend {self.backend!r}; expected one of {sorted(SUPPORTED_BACKENDS)}"
            )
        self.preprocessor = preprocessor or os.getenv("CONVROT_MLX_PREPROCESSOR", "metal-fused")
        if self.preprocessor not in SUPPORTED_PREPROCESSORS:
            raise ValueError(
                f"Unknown ConvRot preprocessor {self.preprocessor!r}; "
                f"expected one of {sorted(SUPPORTED_PREPROCESSORS)}"
            )
        if self.backend.startswith("mpp-"):
            if out_features % 2:
                raise ValueError(f"MPP packed weights require even out_features, got {out_features}")
            qweight = torch.zeros((in_features, out_features // 2), dtype=torch.uint8, device=device)
            self.weight_layout = "packed-kn-low-nibble-even-output"
        else:
            qweight = torch.zeros((out_features, in_features // 2), dtype=torch.uint8, device=device)
            self.weight_layout = "packed-nk-low-nibble-even-feature"
        self.register_buffer("qweight", qweight)
        self.register_buffer("scales", torch.ones((out_features,), dtype=torch.float32, device=device))
        # A zero vector gives the kernel one signature for biased and biasless
        # layers (core.py:1255-1258).
        self.register_buffer("bias", torch.zeros((out_features,), dtype=torch.float32, device=device))
        self.source_has_bias = bias

    @property
    def layout_code(self) -> int:
        return _lib.LAYOUT_KN if self.backend in _KN_BACKENDS else _lib.LAYOUT_NK

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"ConvRotLinear expected K={self.in_features}, got {x.shape[-1]}")
        lead = x.shape[:-1]
        x2d = x.reshape(-1, self.in_features)
        m = x2d.shape[0]
        if self.backend == "mpp-w4a16":
            rotated = regular_hadamard(x2d, self.group_size)
            out = _gemm_w4a16(rotated, self.qweight, _lib.LAYOUT_KN, self.scales, self.bias, x.dtype,
                              m, self.out_features, self.in_features)
            return out.reshape(*lead, self.out_features)
        codes, xscales = _prepare(x2d, self.group_size, packed=False)
        out = _gemm_w4a4(codes, self.qweight, self.layout_code, xscales, self.scales, self.bias, x.dtype,
                         m, self.out_features, self.in_features)
        return out.reshape(*lead, self.out_features)

    def forward_modulated_norm(self, x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                               eps: float = 1e-6) -> torch.Tensor:
        """``self(torch.addcmul(shift, layer_norm(x), 1 + scale))`` with the norm,
        the modulation, the rotation and the A4 quantization in one kernel
        (``modulated_norm_prepare_i8``), then the W4A4 GEMM.

        An extension for DiT blocks (no counterpart in the reference, whose
        design notes name the activation-preparation passes as the remaining
        cost, docs/design.md:54-64).  x: (batch, tokens, in_features) bf16;
        shift / scale: (batch, 1, in_features) or (batch, in_features).  The
        W4A16 backend takes the unfused path (it quantizes no activation)."""

        if x.shape[-1] != self.in_features:
            raise ValueError(f"ConvRotLinear expected K={self.in_features}, got {x.shape[-1]}")
        if self.backend == "mpp-w4a16" or x.dtype != torch.bfloat16 or self.group_size not in (64, 256):
            normed = torch.nn.functional.layer_norm(x, (x.shape[-1],), eps=eps)
            return self(torch.addcmul(shift, normed, 1 + scale))
        lead = x.shape[:-1]
        codes, xscales = modulated_norm_prepare_i8(x, shift, scale, eps, self.group_size)
        m = codes.shape[0]
        out = _gemm_w4a4(codes, self.qweight, self.layout_code, xscales, self.scales, self.bias, x.dtype,
                         m, self.out_features, self.in_features)
        return out.reshape(*lead, self.out_features)

    def forward_gelu_concat(self, a: torch.Tensor, m: torch.Tensor) -> torch.Tensor:
        """``self(torch.cat((a, gelu_tanh(m)), -1))`` with the GELU, the
        concatenation, the rotation and the A4 quantization in one kernel
        (``gelu_concat_prepare_i8``), then the W4A4 GEMM: the output
        projection of a FLUX single block.  An extension with no counterpart
        in the reference; the W4A16 backend and other dtypes take the
        unfused path."""

        lead = a.shape[:-1]
        if a.shape[-1] + m.shape[-1] != self.in_features:
            raise ValueError(f"ConvRotLinear expected K={self.in_features}, got {a.shape[-1]} + {m.shape[-1]}")
        if (self.backend == "mpp-w4a16" or a.dtype != torch.bfloat16 or self.group_size not in (64, 256)
                or a.shape[-1] % 16):
            gelu = torch.nn.functional.gelu(m, approximate="tanh")
            return self(torch.cat((a, gelu), dim=-1))
        codes, xscales = gelu_concat_prepare_i8(a, m, self.group_size)
        out = _gemm_w4a4(codes, self.qweight, self.layout_code, xscales, self.scales, self.bias, a.dtype,
                         codes.shape[0], self.out_features, self.in_features)
        return out.reshape(*lead, self.out_features)

    def extra_repr(self) -> str:
        return (
            f"in_features={self.in_features}, out_features={self.out_features}, group_size={self.group_size}, "
            f"backend={self.backend}, layout={self.weight_layout}"
        )


def eligible_linear(module: object, group_size: int = CONVROT_GROUP_SIZE) -> bool:
    """core.py:1316-1321."""

    return (
        isinstance(module, nn.Linear)
        and module.weight.ndim == 2
        and module.weight.shape[1] % group_size == 0
    )
