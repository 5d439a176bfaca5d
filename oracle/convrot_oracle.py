"""CPU restatement of the ConvRot W4A4 contract -- TEST INFRASTRUCTURE ONLY.

This module is the parity oracle for the CUDA path in ``convrot_mlx_b200``.  It
is imported only by ``tests/``, by ``__graft_entry__.smoke()`` (as the checker)
and by the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``.  The
product never routes through it: every public entry point of
``convrot_mlx_b200`` runs the CUDA library and fails loudly without it.

It restates, in NumPy, the eager MLX contract of
``src/convrot_mlx/core.py`` (Lumenbeing/convrot-mlx, MLX 0.32.0):

* ``regular_hadamard``             core.py:64-94   (radix-4 butterfly, per-op
  rounding in the input dtype, lane order ``a+b+c-d, a+b-c+d, a-b+c+d,
  -a+b+c+d``, then ``/ sqrt(g)``)
* ``quantize_signed_int4_rowwise`` core.py:149-158 (absmax floor 1e-10 in the
  input dtype, ``absmax / 7`` in the input dtype, ``round(x / scale)`` half to
  even in the input dtype, clip to [-7, 7])
* ``pack_signed_int4`` / ``unpack_signed_int4`` core.py:97-120
* ``repack_nk_weight_for_mpp`` / ``repack_mpp_weight_to_nk`` core.py:123-146
* ``quantize_convrot_weight``      core.py:514-527
* ``reference_w4a4_matmul``        core.py:1155-1171 and the MPP epilogue
  order ``float(dots) * xs[m] * ws[n] + bias[n]`` of core.py:925-937
* ``mpp_w4a16_matmul``             core.py:1123-1152

Floating-point values of a 16-bit dtype are carried in float32 arrays that hold
exactly representable values; every arithmetic step is computed in float32 and
rounded to the dtype with round-to-nearest-even.  For + - * / this double
rounding equals a correctly rounded 16-bit operation (float32 has 24 >= 2p+2
significand bits for bf16 p=8 and fp16 p=11), which is what MLX's eager bf16 /
fp16 ops and the reference's Metal kernels (explicit ``static_cast<T>`` after
every op, core.py:180-201, :244, :259-261, :291-298) compute.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own eager
functions from core.py over a NumPy stand-in for ``mlx.core`` and stores the
outputs under ``tests/golden/``; ``tests/test_oracle.py`` checks this module
against those fixtures and against every known-answer test the reference's
``tests/test_core.py`` holds (packing KAT :186-192, Kronecker-matrix rotation
:42-50/:177-184, repack shape :203-211).  The bf16 rounding of MLX itself (a
dependency absent from the reference tree) is not pinned by any recorded MLX
output; it follows the Metal kernels' explicit per-op casts.
"""

from __future__ import annotations

import math

import numpy as np

INT4_MAX = 7  # core.py:35
CONVROT_GROUP_SIZE = 256  # core.py:32

_DTYPES = ("float32", "float16", "bfloat16")


# ---------------------------------------------------------------------------
# rounding helpers


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""

    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) << np.uint64(16)
    out = r.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.float32(np.nan)
    return out


def round_to(dtype: str, x) -> np.ndarray:
    """Round float32 values to ``dtype`` and return them as float32."""

    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return round_bf16(x)
    raise ValueError(f"unsupported dtype {dtype!r}")


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The 16-bit patterns of bf16-representable float32 values."""

    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << np.uint32(16)).view(np.float32)


# ---------------------------------------------------------------------------
# contract primitives


def validate_group_size(group_size: int) -> None:
    """core.py:50-61: the group size must be a power of four (>= 4)."""

    if group_size < 4:
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {group_size}")
    value = group_size
    while value > 1 and value % 4 == 0:
        value //= 4
    if value != 1:
        raise ValueError(f"Regular Hadamard size must be a power of 4, got {group_size}")


def regular_hadamard(x, group_size: int = CONVROT_GROUP_SIZE, dtype: str = "bfloat16"):
    """core.py:64-94 with per-op rounding to ``dtype``.

    Each radix-4 stage (stride 1, 4, 16, ...) maps ``(a, b, c, d)`` to
    ``(((a+b)+c)-d, ((a+b)-c)+d, ((a-b)+c)+d, (((-a)+b)+c)+d)``, every add
    rounded (core.py:89-91 evaluates left to right; the Metal lane helper
    core.py:180-201 casts after each op).  The result is divided by
    ``sqrt(group_size)``, a power of two for every power-of-four group.
    """

    validate_group_size(group_size)
    x = round_to(dtype, np.asarray(x, dtype=np.float32))
    features = x.shape[-1]
    if features % group_size:
        raise ValueError(
            f"features {features} not divisible by ConvRot group size {group_size}"
        )
    r = lambda v: round_to(dtype, v)  # noqa: E731
    groups = features // group_size
    prefix = (*x.shape[:-1], groups)
    y = x.reshape(*prefix, group_size)
    stride = 1
    while stride < group_size:
        y = y.reshape(*prefix, group_size // (4 * stride), 4, stride)
        a = y[..., 0, :]
        b = y[..., 1, :]
        c = y[..., 2, :]
        d = y[..., 3, :]
        ab = r(a + b)
        o0 = r(r(ab + c) - d)
        o1 = r(r(ab - c) + d)
        o2 = r(r(r(a - b) + c) + d)
        o3 = r(r(r(-a + b) + c) + d)
        y = np.stack([o0, o1, o2, o3], axis=-2).reshape(*prefix, group_size)
        stride *= 4
    y = r(y / np.float32(math.sqrt(group_size)))
    return y.reshape(x.shape)


def pack_signed_int4(values) -> np.ndarray:
    """core.py:97-105: two's-complement nibbles, element 2j low, 2j+1 high."""

    values = np.asarray(values)
    if values.shape[-1] % 2:
        raise ValueError(f"last dimension must be even, got {values.shape[-1]}")
    v = values.astype(np.int32)
    lo = v[..., 0::2] & 0x0F
    hi = v[..., 1::2] & 0x0F
    return (lo | (hi << 4)).astype(np.uint8)


def unpack_signed_int4(packed) -> np.ndarray:
    """core.py:108-120: nibbles back to int8 in [-8, 7]."""

    data = np.asarray(packed).astype(np.int32)
    lo = data & 0x0F
    hi = (data >> 4) & 0x0F
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    return (
        np.stack([lo, hi], axis=-1)
        .reshape(*data.shape[:-1], data.shape[-1] * 2)
        .astype(np.int8)
    )


def repack_nk_weight_for_mpp(qweight) -> np.ndarray:
    """core.py:123-133: N x packed-K -> K x packed-N (needs even N)."""

    qweight = np.asarray(qweight)
    if qweight.ndim != 2:
        raise ValueError(f"MPP weight repack expects a 2D tensor, got {qweight.shape}")
    unpacked = unpack_signed_int4(qweight)
    if unpacked.shape[0] % 2:
        raise ValueError(
            f"MPP int4 packing requires even out_features, got {unpacked.shape[0]}"
        )
    return pack_signed_int4(unpacked.T)


def repack_mpp_weight_to_nk(qweight) -> np.ndarray:
    """core.py:136-146: K x packed-N -> N x packed-K (needs even K)."""

    qweight = np.asarray(qweight)
    if qweight.ndim != 2:
        raise ValueError(f"MPP weight repack expects a 2D tensor, got {qweight.shape}")
    unpacked = unpack_signed_int4(qweight)
    if unpacked.shape[0] % 2:
        raise ValueError(
            f"row-major int4 packing requires even in_features, got {unpacked.shape[0]}"
        )
    return pack_signed_int4(unpacked.T)


def quantize_codes_rowwise(x, dtype: str = "bfloat16"):
    """core.py:149-158 without the final packing: (int8 codes, float32 scales).

    ``absmax = max(|x|)`` (exact), ``absmax = max(absmax, T(1e-10))``,
    ``scale = T(absmax / 7)``, ``code = clip(rint(T(x / scale)), -7, 7)``.
    A NaN ratio (only possible for an all-zero float16 row, whose 1e-10 floor
    underflows to zero) yields code 0.
    """

    x = round_to(dtype, np.asarray(x, dtype=np.float32))
    if x.ndim != 2:
        raise ValueError(f"rowwise int4 quantization expects 2D input, got {x.shape}")
    absmax = np.max(np.abs(x), axis=-1, keepdims=True) if x.shape[1] else np.zeros(
        (x.shape[0], 1), np.float32
    )
    floor = round_to(dtype, np.float32(1e-10))
    absmax = np.maximum(absmax, floor)
    scales = round_to(dtype, absmax / np.float32(INT4_MAX))
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = round_to(dtype, x / scales)
    q = np.rint(ratio)
    q = np.where(np.isnan(q), 0.0, q)
    q = np.clip(q, -INT4_MAX, INT4_MAX).astype(np.int8)
    return q, scales.reshape(-1).astype(np.float32)


def quantize_signed_int4_rowwise(x, dtype: str = "bfloat16"):
    """core.py:149-158: (packed uint8 (R, K/2), float32 scales (R,))."""

    q, scales = quantize_codes_rowwise(x, dtype)
    return pack_signed_int4(q), scales


def prepare_convrot_activation(x, group_size: int = CONVROT_GROUP_SIZE, dtype: str = "bfloat16"):
    """core.py:161-167 (= the fused Metal kernels K1/K2, tests :65-86)."""

    return quantize_signed_int4_rowwise(regular_hadamard(x, group_size, dtype), dtype)


def prepare_convrot_activation_i8(x, group_size: int = CONVROT_GROUP_SIZE, dtype: str = "bfloat16"):
    """core.py:456-484 semantics: int8 codes and the same scales."""

    return quantize_codes_rowwise(regular_hadamard(x, group_size, dtype), dtype)


def quantize_convrot_weight(weight, group_size: int = CONVROT_GROUP_SIZE, dtype: str = "bfloat16"):
    """core.py:514-527: rotate a dense (out, in) weight, then pack it N x packed-K."""

    weight = np.asarray(weight, dtype=np.float32)
    if weight.ndim != 2:
        raise ValueError(f"ConvRot weight must be 2D, got {weight.shape}")
    if weight.shape[-1] % group_size:
        raise ValueError(
            f"in_features {weight.shape[-1]} not divisible by ConvRot group size {group_size}"
        )
    return quantize_signed_int4_rowwise(regular_hadamard(weight, group_size, dtype), dtype)


# ---------------------------------------------------------------------------
# GEMM oracles


def integer_dot(act_codes, weight_codes_nk) -> np.ndarray:
    """Exact ``sum_k a[m,k] * w[n,k]`` in int64 (the int32 MPP accumulator)."""

    a = np.asarray(act_codes).astype(np.float64)
    w = np.asarray(weight_codes_nk).astype(np.float64)
    # |partial sums| <= 64 K << 2^53: float64 BLAS is exact here and fast.
    return (a @ w.T).astype(np.int64)


def w4a4_epilogue(dots, xscales, wscales, bias, output_dtype: str = "bfloat16"):
    """core.py:932-936 / :1166-1171: ``T(f32(dots) * xs[m] * ws[n] + bias[n])``.

    Evaluated left to right in float32, each product and the sum rounded (no
    fused multiply-add), then rounded once to ``output_dtype``.
    """

    d = np.asarray(dots).astype(np.float32)
    xs = np.asarray(xscales, dtype=np.float32)
    ws = np.asarray(wscales, dtype=np.float32)
    b = np.asarray(bias, dtype=np.float32)
    out = (d * xs[:, None]) * ws[None, :]
    out = out + b[None, :]
    return round_to(output_dtype, out.astype(np.float32))


def reference_w4a4_matmul(qact, qweight_nk, xscales, wscales, bias, output_dtype="bfloat16"):
    """core.py:1155-1171: packed A (M, K/2) x packed NK W (N, K/2)."""

    a = unpack_signed_int4(qact)
    w = unpack_signed_int4(qweight_nk)
    return w4a4_epilogue(integer_dot(a, w), xscales, wscales, bias, output_dtype)


def w4a4_int8_matmul_kn(act_i8, qweight_kn, xscales, wscales, bias, output_dtype="bfloat16"):
    """core.py:1088-1120 math: int8 codes (M, K) x packed KN W (K, N/2)."""

    w_kn = unpack_signed_int4(qweight_kn)  # (K, N)
    return w4a4_epilogue(integer_dot(act_i8, w_kn.T), xscales, wscales, bias, output_dtype)


def w4a16_dots(act, qweight_kn) -> np.ndarray:
    """fp32-accumulated ``act @ w`` computed exactly in float64, rounded to float32."""

    w = unpack_signed_int4(qweight_kn).astype(np.float64)  # (K, N)
    return (np.asarray(act, dtype=np.float64) @ w).astype(np.float32)


def w4a16_matmul(act, qweight_kn, wscales, bias, output_dtype="bfloat16"):
    """core.py:1123-1152: ``T(dots * ws[n] + bias[n])`` with float32 dots."""

    dots = w4a16_dots(act, qweight_kn)
    out = dots * np.asarray(wscales, np.float32)[None, :]
    out = out + np.asarray(bias, np.float32)[None, :]
    return round_to(output_dtype, out.astype(np.float32))


def convrot_linear_w4a4(x, qweight, layout: str, wscales, bias, group_size=256, dtype="bfloat16"):
    """core.py:1261-1313: the layer forward for every W4A4 backend."""

    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    codes, xs = prepare_convrot_activation_i8(x2, group_size, dtype)
    if layout == "kn":
        out = w4a4_int8_matmul_kn(codes, qweight, xs, wscales, bias, dtype)
    else:
        out = w4a4_epilogue(
            integer_dot(codes, unpack_signed_int4(qweight)), xs, wscales, bias, dtype
        )
    return out.reshape(*lead, -1)


def convrot_linear_w4a16(x, qweight_kn, wscales, bias, group_size=256, dtype="bfloat16"):
    """core.py:1268-1277: rotate, then W4A16 with float32 dots."""

    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    rot = regular_hadamard(x.reshape(-1, x.shape[-1]), group_size, dtype)
    return w4a16_matmul(rot, qweight_kn, wscales, bias, dtype).reshape(*lead, -1)


def regular_hadamard_matrix(size: int) -> np.ndarray:
    """Explicit ``H4 kron H4 kron ... / sqrt(size)`` (reference tests :42-50)."""

    h4 = np.array(
        [[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float32
    )
    matrix = h4
    while matrix.shape[0] < size:
        matrix = np.kron(matrix, h4)
    return matrix / np.sqrt(size)
