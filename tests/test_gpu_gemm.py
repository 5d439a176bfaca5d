"""tcgen05 W4A4 GEMM vs the reference fixtures and the oracle.

The integer accumulator is exact, and the epilogue evaluates
``f32(dot) * xs * ws + bias`` in the eager oracle's order without fused
multiply-adds, so every comparison here is bitwise.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import convrot_mlx_b200 as cr
from oracle import convrot_oracle as O
from tests.conftest import load_golden
from tests.gpu_util import assert_no_device_error, bf16_bits, cuda, host

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["auto", "single", "pair", "swap_ab"], autouse=True)
def gemm_kernel(request):
    """Run every GEMM test on each tcgen05 kernel: the default routing (the
    swap-AB kernel for m <= 8, else the CTA-pair kernel where it applies),
    the one-CTA kernel for every shape, the CTA-pair kernel for every shape
    it takes, and the swap-AB kernel for every m <= 64 shape
    (convrot_set_gemm_route)."""
    from convrot_mlx_b200 import _lib

    route = {"auto": 0, "single": 1, "pair": 2, "swap_ab": 3}[request.param]
    _lib.check(_lib.load().convrot_set_gemm_route(route), "route")
    yield request.param
    _lib.check(_lib.load().convrot_set_gemm_route(0), "route")


def test_edges_nk_and_kn_match_reference():
    # reference tests/test_core.py:213-283 (37 x 64 x 46: M, N not multiples of anything)
    g = load_golden("edges_s2026082302")
    qact, qnk, qkn = cuda(g["qact"]), cuda(g["qweight_nk"]), cuda(g["qweight_kn"])
    xs, ws, b = cuda(g["xscales"]), cuda(g["wscales"]), cuda(g["bias"])
    out = cr.mpp_w4a4_matmul(qact, qkn, xs, ws, b, output_dtype=torch.float32)
    np.testing.assert_array_equal(host(out), g["out_f32"])
    ref = cr.reference_w4a4_matmul(qact, qnk, xs, ws, b, output_dtype=torch.float32)
    np.testing.assert_array_equal(host(ref), g["out_f32"])
    ones_x = torch.ones(37, device="cuda")
    ones_w = torch.ones(46, device="cuda")
    zero_b = torch.zeros(46, device="cuda")
    integer = cr.mpp_w4a4_matmul(qact, qkn, ones_x, ones_w, zero_b, output_dtype=torch.float32)
    np.testing.assert_array_equal(host(integer), g["out_int"])
    legacy = cr.packed_w4a4_matmul_m32n32_k64(qact, qnk, xs, ws, b, output_dtype=torch.bfloat16)
    native = cr.mpp_w4a4_matmul(qact, qkn, xs, ws, b, output_dtype=torch.bfloat16)
    np.testing.assert_array_equal(bf16_bits(legacy), g["out_bf16"])
    np.testing.assert_array_equal(bf16_bits(native), g["out_bf16"])


@pytest.mark.parametrize("name", ["tiles_s29", "expanded_s27"])
def test_bf16_output_matches_reference(name):
    # reference tests/test_core.py:139-175, :329-355
    g = load_golden(name)
    args = [cuda(g[k]) for k in ("qact", "qweight_nk", "xscales", "wscales", "bias")]
    fns = [cr.packed_w4a4_matmul, cr.packed_w4a4_matmul_k32, cr.packed_w4a4_matmul_k64, cr.packed_w4a4_matmul_k128,
           cr.packed_w4a4_matmul_k256, cr.packed_w4a4_matmul_m32n32_k64, cr.packed_w4a4_matmul_m16n64_k64,
           cr.expanded_fp32_w4a4_matmul, cr.reference_w4a4_matmul]
    for fn in fns:
        out = fn(*args, output_dtype=torch.bfloat16)
        np.testing.assert_array_equal(bf16_bits(out), g["out_bf16"], err_msg=fn.__name__)


@pytest.mark.parametrize("name", ["quant_f16_s23", "quant_f16_s28"])
def test_float32_output_matches_reference(name):
    # reference tests/test_core.py:311-327, :357-373
    g = load_golden(name)
    out = cr.packed_w4a4_matmul(cuda(g["qact"]), cuda(g["qweight"]), cuda(g["xscales"]), cuda(g["wscales"]),
                                cuda(g["bias"]), output_dtype=torch.float32)
    np.testing.assert_array_equal(host(out), g["out_f32"])


def _random_case(m, n, k, seed):
    rng = np.random.default_rng(seed)
    a = rng.integers(-7, 8, size=(m, k), dtype=np.int8)
    w = rng.integers(-8, 8, size=(n, k), dtype=np.int8)  # -8 exercises the full nibble range
    xs = rng.uniform(0.01, 0.2, size=m).astype(np.float32)
    ws = rng.uniform(0.01, 0.2, size=n).astype(np.float32)
    b = rng.normal(size=n).astype(np.float32)
    return a, w, xs, ws, b


@pytest.mark.parametrize(
    "m,n,k",
    [(1, 2, 32), (37, 46, 64), (128, 256, 128), (129, 258, 160), (300, 520, 1024), (64, 1024, 1024),
     (200, 34, 2688), (513, 1728, 3072), (17, 990, 96), (256, 256, 256), (255, 320, 384), (700, 1024, 2560),
     (33, 64, 128)],
)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_random_shapes_both_layouts(m, n, k, out_dtype):
    a, w, xs, ws, b = _random_case(m, n, k, seed=m * 1000 + n + k)
    names = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}
    expected = O.w4a4_epilogue(O.integer_dot(a, w), xs, ws, b, names[out_dtype])
    at = cuda(a)
    wnk = cuda(O.pack_signed_int4(w))
    out_nk = cr.core._gemm_w4a4(at, wnk, 0, cuda(xs), cuda(ws), cuda(b), out_dtype, m, n, k)
    np.testing.assert_array_equal(host(out_nk.float()), expected)
    if n % 2 == 0:
        wkn = cuda(O.pack_signed_int4(w.T.copy()))
        out_kn = cr.mpp_w4a4_int8_matmul(at, wkn, cuda(xs), cuda(ws), cuda(b), output_dtype=out_dtype)
        np.testing.assert_array_equal(host(out_kn.float()), expected)
    assert_no_device_error()


def test_integer_accumulator_extremes():
    # every product at its extreme (7 * -8), K large: the int32 dot must be exact
    m, n, k = 130, 300, 15360
    a = np.full((m, k), 7, np.int8)
    a[1::2] = -7
    w = np.full((n, k), -8, np.int8)
    w[::3] = 7
    ones_m, ones_n, zeros_n = np.ones(m, np.float32), np.ones(n, np.float32), np.zeros(n, np.float32)
    out = cr.mpp_w4a4_int8_matmul(cuda(a), cuda(O.pack_signed_int4(w.T.copy())), cuda(ones_m), cuda(ones_n),
                                  cuda(zeros_n), output_dtype=torch.float32)
    np.testing.assert_array_equal(host(out), O.integer_dot(a, w).astype(np.float32))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_tiny_and_special_row_scales_exact(out_dtype):
    # The epilogue multiplies the accumulator (16 * dot) by xs / 16 when every
    # row scale of a warp keeps xs / 16 exact, and shifts first otherwise.
    # Rows 0-31 (one epilogue warp) hold scales where xs / 16 is not exact
    # (subnormal results, subnormal xs) or special (0, inf); rows 32-63 are
    # ordinary.  Both forms must match the oracle bit for bit.
    m, n, k = 64, 256, 256
    a, w, xs, ws, b = _random_case(m, n, k, seed=4242)
    special = [0.0, 1e-45, 1e-40, 2.0 ** -126, 2.0 ** -123, 2.0 ** -122 * 1.5, 2.0 ** -121, 1e-30, np.inf, 3.0e38]
    xs[: len(special)] = np.array(special, np.float32)
    xs[len(special):32] = np.float32(2.0 ** -124)
    names = {torch.bfloat16: "bfloat16", torch.float32: "float32"}
    with np.errstate(over="ignore", invalid="ignore"):
        expected = O.w4a4_epilogue(O.integer_dot(a, w), xs, ws, b, names[out_dtype])
    out = cr.mpp_w4a4_int8_matmul(cuda(a), cuda(O.pack_signed_int4(w.T.copy())), cuda(xs), cuda(ws), cuda(b),
                                  output_dtype=out_dtype)
    np.testing.assert_array_equal(host(out.float()), expected)
    assert_no_device_error()


@pytest.mark.parametrize("m,k,n", [(1536, 3072, 3072), (4096, 3072, 12288), (4096, 15360, 3072)])
def test_flux_shapes_integer_exact(m, k, n):
    # BASELINE config 3 shapes: the int32 dots must equal an exact reference.
    # fp32 GEMM of integer operands is exact here (every partial sum < 2^24);
    # TF32 is off so cuBLAS accumulates true fp32 products.
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    a = torch.randint(-7, 8, (m, k), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-8, 8, (n, k), dtype=torch.int8, device="cuda", generator=g)
    wkn = cr.pack_signed_int4(w.t().contiguous())
    ones_m = torch.ones(m, device="cuda")
    ones_n = torch.ones(n, device="cuda")
    zeros_n = torch.zeros(n, device="cuda")
    out = cr.mpp_w4a4_int8_matmul(a, wkn, ones_m, ones_n, zeros_n, output_dtype=torch.float32)
    ref = a.float() @ w.float().t()
    assert torch.equal(out, ref)
    wnk = cr.pack_signed_int4(w)
    out_nk = cr.core._gemm_w4a4(a, wnk, 0, ones_m, ones_n, zeros_n, torch.float32, m, n, k)
    assert torch.equal(out_nk, ref)
    assert_no_device_error()


def test_validation_errors_match_reference_messages():
    a = torch.zeros((4, 64), dtype=torch.int8, device="cuda")
    w = torch.zeros((64, 8), dtype=torch.uint8, device="cuda")
    ones4, ones16, z16 = torch.ones(4, device="cuda"), torch.ones(16, device="cuda"), torch.zeros(16, device="cuda")
    with pytest.raises(ValueError, match="K x packed-N layout"):
        cr.mpp_w4a4_int8_matmul(a, w[:32], ones4, ones16, z16, output_dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="activation scales must have shape"):
        cr.mpp_w4a4_int8_matmul(a, w, ones16, ones16, z16, output_dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="requires a 2D int8 activation"):
        cr.mpp_w4a4_int8_matmul(a.float(), w, ones4, ones16, z16, output_dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="divisible by 32"):
        cr.mpp_w4a4_int8_matmul(a[:, :48].contiguous(), w[:48], ones4, ones16, z16, output_dtype=torch.bfloat16)
