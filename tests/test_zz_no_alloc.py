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


def test_static_linear_rejections_enqueue_nothing():
    # m == 0 is a no-op; a call the GEMM would reject (bad output dtype, K not a
    # multiple of 32, odd N for K x packed-N) is refused before the prep kernel
    # is enqueued, so the output buffer keeps its contents
    lib = _lib.load()
    m, k, n = 64, 1024, 256
    x, q, ws, bias = _inputs(m, k, n, _lib.LAYOUT_KN, 21)
    out = torch.full((m, n), 7.0, dtype=torch.bfloat16, device=dev())
    s = _lib.stream_of(x)

    def call(mm, nn, kk, out_dtype=_lib.BF16, layout=_lib.LAYOUT_KN):
        return lib.convrot_w4a4_linear_static(_lib.ptr(x), _lib.BF16, 256, _lib.ptr(q), layout, _lib.ptr(ws),
                                              _lib.ptr(bias), _lib.ptr(out), out_dtype, mm, nn, kk, s)

    assert call(0, n, k) == _lib.OK
    assert call(m, n, k, out_dtype=7) == _lib.ERR_INVALID
    assert call(m, n, 1000) == _lib.ERR_INVALID
    assert call(m, n - 1, k) == _lib.ERR_INVALID
    assert call(m, n, k, layout=5) == _lib.ERR_INVALID
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    assert_no_device_error()


_CAPTURE_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from convrot_mlx_b200 import _lib
lib = _lib.load()
dev = torch.device("cuda", 0)
m, k, n = 128, 512, 256
x = torch.randn((m, k), device=dev).to(torch.bfloat16)
q = torch.randint(0, 256, (k, n // 2), device=dev, dtype=torch.uint8)
ws = torch.rand((n,), device=dev) * 0.01
out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
ref = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
s = torch.cuda.Stream(device=dev)
torch.cuda.synchronize()

def call(o):
    return lib.convrot_w4a4_linear_static(_lib.ptr(x), _lib.BF16, 256, _lib.ptr(q), _lib.LAYOUT_KN, _lib.ptr(ws),
                                          None, _lib.ptr(o), _lib.BF16, m, n, k, _lib.stream_of(x))

g = torch.cuda.CUDAGraph()
with torch.cuda.graph(g, stream=s):
    first = call(out)                                  # first call on the device, inside capture
msg = lib.convrot_last_error().decode()
with torch.cuda.stream(s):
    second = call(ref)                                 # outside capture: looks the address up
g2 = torch.cuda.CUDAGraph()
with torch.cuda.graph(g2, stream=s):
    third = call(out)                                  # address known: captured like any launch
g2.replay()
torch.cuda.synchronize()
same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
print(first, second, third, same, "capture" in msg)
"""


def test_static_linear_first_call_inside_capture_is_refused():
    import subprocess
    import sys

    from tests.conftest import ROOT

    res = subprocess.run([sys.executable, "-c", _CAPTURE_SCRIPT, str(ROOT)], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    first, second, third, same, msg_ok = res.stdout.split()[-5:]
    assert int(first) == _lib.ERR_UNSUPPORTED and msg_ok == "True"
    assert int(second) == _lib.OK and int(third) == _lib.OK and same == "True"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_static_linear_on_a_second_device():
    # the array's address is looked up per device: a call with device 1 current
    with torch.cuda.device(1):
        d1 = torch.device("cuda", 1)
        m, k, n = 512, 1024, 384
        g = torch.Generator(device=d1).manual_seed(4)
        x = torch.randn((m, k), generator=g, device=d1).to(torch.bfloat16)
        w = torch.randint(-7, 8, (k, n), generator=g, device=d1, dtype=torch.int8)
        import convrot_mlx_b200 as cr
        q = cr.pack_signed_int4(w)
        ws = torch.rand((n,), generator=g, device=d1) * 0.01
        lib = _lib.load()
        s = _lib.stream_of(x)
        codes = torch.empty((m, k), dtype=torch.int8, device=d1)
        xs = torch.empty((m,), dtype=torch.float32, device=d1)
        want = torch.empty((m, n), dtype=torch.bfloat16, device=d1)
        got = torch.empty((m, n), dtype=torch.bfloat16, device=d1)
        _lib.check(lib.convrot_prepare_i8(_lib.ptr(x), _lib.BF16, m, k, 256, _lib.ptr(codes), _lib.ptr(xs), s), "p")
        _lib.check(lib.convrot_w4a4_gemm(_lib.ptr(codes), _lib.ptr(q), _lib.LAYOUT_KN, _lib.ptr(xs), _lib.ptr(ws), None,
                                         _lib.ptr(want), _lib.BF16, m, n, k, s), "g")
        _lib.check(lib.convrot_w4a4_linear_static(_lib.ptr(x), _lib.BF16, 256, _lib.ptr(q), _lib.LAYOUT_KN,
                                                  _lib.ptr(ws), None, _lib.ptr(got), _lib.BF16, m, n, k, s), "static")
        torch.cuda.synchronize(d1)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
