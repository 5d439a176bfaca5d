"""Tensor-parallel W4A4 (column split of N): the gathering GEMM, the peer
copies and the flag barrier.

On one GPU: the multi-destination epilogue (every destination receives the
shard's columns at its offset, bit for bit equal to the plain GEMM), the
strided block copy, and the barrier with a world of one and with a peer that
never arrives.  With two or more GPUs: spawned ranks run
``ColumnParallelConvRotLinear`` with every gather (copy engines in 4 and in
1 blocks of rows, epilogue peer stores, the split of peers between the two,
the chunked GEMM storing into every peer) and compare every rank's full
output with the single-GPU ``ConvRotLinear``, bit for bit.
"""

from __future__ import annotations

import ctypes
import os

import pytest
import torch

import convrot_mlx_b200 as cr
from convrot_mlx_b200 import _lib
from tests.gpu_util import assert_no_device_error, dev

pytestmark = pytest.mark.gpu


def _layer(k, n, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn((n, k), generator=g, device=device) * 0.02).to(torch.bfloat16)
    layer = cr.ConvRotLinear(k, n, backend="mpp-w4a4", device=device)
    qnk, ws = cr.quantize_convrot_weight(w)
    layer.qweight = cr.repack_nk_weight_for_mpp(qnk)
    layer.scales = ws
    layer.bias = torch.randn((n,), generator=g, device=device) * 0.01
    return layer


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
@pytest.mark.parametrize("m,k,n,ldc,col", [(300, 1024, 256, 1024, 512), (129, 2048, 64, 160, 96)])
def test_gather_epilogue_two_destinations(layout, m, k, n, ldc, col):
    g = torch.Generator(device=dev()).manual_seed(m + n)
    codes = torch.randint(-7, 8, (m, k), generator=g, device=dev(), dtype=torch.int8)
    w = torch.randint(-8, 8, (n, k), generator=g, device=dev(), dtype=torch.int8)
    q = cr.pack_signed_int4(w.t().contiguous()) if layout == _lib.LAYOUT_KN else cr.pack_signed_int4(w)
    xs = torch.rand(m, generator=g, device=dev())
    ws = torch.rand(n, generator=g, device=dev())
    bias = torch.randn(n, generator=g, device=dev())
    lib = _lib.load()
    want = torch.empty((m, n), dtype=torch.bfloat16, device=dev())
    _lib.check(lib.convrot_w4a4_gemm(_lib.ptr(codes), _lib.ptr(q), layout, _lib.ptr(xs), _lib.ptr(ws), _lib.ptr(bias),
                                     _lib.ptr(want), _lib.BF16, m, n, k, _lib.stream_of(codes)), "gemm")
    sentinel = torch.tensor(-1234.0, dtype=torch.bfloat16)
    outs = [torch.full((m, ldc), sentinel.item(), dtype=torch.bfloat16, device=dev()) for _ in range(2)]
    ptrs = (ctypes.c_void_p * 2)(*[o.data_ptr() for o in outs])
    _lib.check(lib.convrot_w4a4_gemm_gather(_lib.ptr(codes), _lib.ptr(q), layout, _lib.ptr(xs), _lib.ptr(ws),
                                            _lib.ptr(bias), ptrs, 2, ldc, col, _lib.BF16, m, n, k,
                                            _lib.stream_of(codes)), "gather gemm")
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o[:, col:col + n].view(torch.int16), want.view(torch.int16))
        rest = torch.cat([o[:, :col], o[:, col + n:]], dim=1)
        assert bool((rest == sentinel.to(dev())).all())
    assert_no_device_error()


def test_gather_rejects_bad_arguments():
    lib = _lib.load()
    one = (ctypes.c_void_p * 1)(0)
    rc = lib.convrot_w4a4_gemm_gather(None, None, _lib.LAYOUT_KN, None, None, None, one, 0, 64, 0, _lib.BF16,
                                      4, 32, 128, None)
    assert rc == _lib.ERR_INVALID
    rc = lib.convrot_w4a4_gemm_gather(None, None, _lib.LAYOUT_KN, None, None, None, one, 1, 16, 0, _lib.BF16,
                                      4, 32, 128, None)
    assert rc == _lib.ERR_INVALID  # ldc < col_offset + n


def test_copy_2d_moves_a_column_block():
    lib = _lib.load()
    src = torch.arange(64 * 96, dtype=torch.int16, device=dev()).reshape(64, 96)
    dst = torch.full((64, 96), -1, dtype=torch.int16, device=dev())
    # rows 8..40, columns 16..48 (bytes 32..96 of each 192-byte row)
    _lib.check(lib.convrot_copy_2d(ctypes.c_void_p(dst.data_ptr() + (8 * 96 + 16) * 2), 96 * 2,
                                   ctypes.c_void_p(src.data_ptr() + (8 * 96 + 16) * 2), 96 * 2, 32 * 2, 32,
                                   _lib.stream_of(src)), "copy")
    torch.cuda.synchronize()
    want = torch.full_like(dst, -1)
    want[8:40, 16:48] = src[8:40, 16:48]
    assert torch.equal(dst, want)
    assert lib.convrot_copy_2d(_lib.ptr(dst), 10, _lib.ptr(src), 10, 20, 1, None) == _lib.ERR_INVALID


def test_peer_barrier_world_one():
    flags = torch.zeros(1, dtype=torch.int32, device=dev())
    ptrs = (ctypes.c_void_p * 1)(flags.data_ptr())
    lib = _lib.load()
    for epoch in (1, 2, 3):
        _lib.check(lib.convrot_peer_barrier(ctypes.cast(ptrs, ctypes.POINTER(ctypes.c_void_p)), 1, 0, epoch,
                                            _lib.stream_of(flags)), "barrier")
    torch.cuda.synchronize()
    assert int(flags.item()) == 3
    assert lib.convrot_peer_barrier(ctypes.cast(ptrs, ctypes.POINTER(ctypes.c_void_p)), 1, 0, 0, None) == \
        _lib.ERR_INVALID
    assert_no_device_error()


def _tp_rank(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    from convrot_mlx_b200.tp import ColumnParallelConvRotLinear

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=device)
    ok = True
    try:
        m, k, n = 1100, 3072, 64 * 32 * world
        layer = _layer(k, n, 7, device)
        arms = (("auto", 4, None), ("copy-engine", 4, None), ("copy-engine", 1, None), ("epilogue", 1, None),
                ("split", 4, None), ("split", 3, world - 1))  # the last: chunked, every peer by epilogue stores
        for gather, chunks, epi in arms:
            tp = ColumnParallelConvRotLinear.from_full(layer, gather=gather, chunks=chunks, epilogue_peers=epi)
            for step in range(3):
                g = torch.Generator(device=device).manual_seed(100 + step)
                x = torch.randn((m, k), generator=g, device=device).to(torch.bfloat16)
                want = layer(x)
                got = tp(x)
                torch.cuda.synchronize()
                ok &= bool(torch.equal(got.view(torch.int16), want.view(torch.int16)))
            tp._out.clear()
            tp._flags = None
            torch.cuda.synchronize()
            dist.barrier()
        ok &= _lib.take_device_error() == 0
    finally:
        dist.barrier()
        dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write("ok" if ok else "mismatch")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_column_parallel_layer_bit_exact(tmp_path):
    import socket

    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "tp")
    ctx = mp.start_processes(_tp_rank, args=(world, port, path), nprocs=world, join=False, start_method="spawn")
    assert ctx.join(timeout=240) or ctx.join(timeout=60)
    for r in range(world):
        assert open(f"{path}.{r}").read() == "ok", f"rank {r}"


def test_peer_barrier_times_out_cleanly():
    # A world of two in which the other rank never arrives: rank 0's barrier
    # kernel writes its own epoch and then polls a slot that nothing sets.
    # Its wait is bounded (2 s): the kernel must give up, record device error
    # 31, and leave the context usable for the next call.
    import time

    flags = [torch.zeros(2, dtype=torch.int32, device=dev()) for _ in range(2)]
    ptrs = (ctypes.c_void_p * 2)(*[f.data_ptr() for f in flags])
    lib = _lib.load()
    t0 = time.perf_counter()
    _lib.check(lib.convrot_peer_barrier(ctypes.cast(ptrs, ctypes.POINTER(ctypes.c_void_p)), 2, 0, 1,
                                        _lib.stream_of(flags[0])), "barrier")
    code = _lib.take_device_error()  # synchronizes
    elapsed = time.perf_counter() - t0
    assert code == 31
    assert 1.5 < elapsed < 30.0, elapsed
    # rank 0 wrote its epoch into slot 0 of both arrays; slot 1 stayed empty
    assert flags[0].tolist() == [1, 0] and flags[1].tolist() == [1, 0]
    # the GPU still answers: a world-of-one barrier and a small GEMM run normally
    one = (ctypes.c_void_p * 1)(flags[1].data_ptr())
    _lib.check(lib.convrot_peer_barrier(ctypes.cast(one, ctypes.POINTER(ctypes.c_void_p)), 1, 0, 5,
                                        _lib.stream_of(flags[1])), "barrier")
    layer = _layer(256, 64, 3, dev())
    y = layer(torch.ones((4, 256), dtype=torch.bfloat16, device=dev()))
    torch.cuda.synchronize()
    assert bool(torch.isfinite(y.float()).all()) and int(flags[1][0].item()) == 5
    assert_no_device_error()
