"""convrot_w4a4_linear_static: the W4A4 linear with its intermediate in the
library's fixed device array, for callers that cannot allocate device memory
(a plugin handed only its input and output buffers, or a host framework that
owns the device's memory).

Called through the C ABI, twice in a row on different shapes and layouts, it
must give the same bytes as the allocating path (convrot_prepare_i8 into
caller buffers, then convrot_w4a4_gemm): the W4A4 path is bit-exact, so the
tolerance here is equality.  The second call also shows that the first
call's leftovers in the shared array do not leak into it.  The file's name
makes pytest collect it last.
"""

from __future__ import annotations

import pytest
import torch

from convrot_mlx_b200 import _lib
from tests.gpu_util import assert_no_device_error, dev

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 64 << 20  # CONVROT_LINEAR_STATIC_SCRATCH_BYTES


def _inputs(m, k, n, layout, seed):
    import convrot_mlx_b200 as cr

    g = torch.Generator(device=dev()).manual_seed(seed)
    x = torch.randn((m, k), generator=g, device=dev()).to(torch.bfloat16)
    w = torch.randint(-7, 8, (n, k), generator=g, device=dev(), dtype=torch.int8)
    q = cr.pack_signed_int4(w.t().contiguous()) if layout == _lib.LAYOUT_KN else cr.pack_signed_int4(w)
    ws = torch.rand((n,), generator=g, device=dev()) * 0.01
    bias = torch.randn((n,), generator=g, device=dev()) * 0.01
    return x, q, ws, bias


def _allocating_path(x, q, layout, ws, bias, m, n, k, group):
    lib = _lib.load()
    s = _lib.stream_of(x)
    codes = torch.empty((m, k), dtype=torch.int8, device=dev())
    xs = torch.empty((m,), dtype=torch.float32, device=dev())
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev())
    _lib.check(lib.convrot_prepare_i8(_lib.ptr(x), _lib.BF16, m, k, group, _lib.ptr(codes), _lib.ptr(xs), s), "prep")
    _lib.check(lib.convrot_w4a4_gemm(_lib.ptr(codes), _lib.ptr(q), layout, _lib.ptr(xs), _lib.ptr(ws), _lib.ptr(bias),
                                     _lib.ptr(out), _lib.BF16, m, n, k, s), "gemm")
    return out


def _static_path(x, q, layout, ws, bias, m, n, k, group):
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev())
    rc = _lib.load().convrot_w4a4_linear_static(_lib.ptr(x), _lib.BF16, group, _lib.ptr(q), layout, _lib.ptr(ws),
                                                _lib.ptr(bias), _lib.ptr(out), _lib.BF16, m, n, k, _lib.stream_of(x))
    _lib.check(rc, "convrot_w4a4_linear_static")
    return out


def test_static_linear_matches_allocating_path_twice():
    # two calls in a row on one device: a large KN layer, then a smaller NK
    # one that reads less of the array than the first call wrote
    cases = [(4096, 3072, 3072, _lib.LAYOUT_KN, 256, 11), (300, 1024, 520, _lib.LAYOUT_NK, 64, 12)]
    for m, k, n, layout, group, seed in cases:
        x, q, ws, bias = _inputs(m, k, n, layout, seed)
        got = _static_path(x, q, layout, ws, bias, m, n, k, group)
        want = _allocating_path(x, q, layout, ws, bias, m, n, k, group)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (m, k, n, layout)
    assert_no_device_error()


def test_static_linear_rejects_shapes_beyond_its_array():
    m, k = 8192, 8192  # 64 MiB of codes plus the scales: over the limit
    assert m * k + 4 * m > SCRATCH_LIMIT
    x = torch.zeros((1, 1), dtype=torch.bfloat16, device=dev())  # never read: the size check comes first
    lib = _lib.load()
    rc = lib.convrot_w4a4_linear_static(_lib.ptr(x), _lib.BF16, 256, _lib.ptr(x), _lib.LAYOUT_KN, _lib.ptr(x),
                                        None, _lib.ptr(x), _lib.BF16, m, 256, k, _lib.stream_of(x))
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"scratch" in lib.convrot_last_error()
