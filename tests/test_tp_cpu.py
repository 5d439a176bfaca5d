"""Tensor-parallel host logic on CPU: shard ranges, weight slices, and a
world-size-2 gloo run in which the gathered shards rebuild the full layer."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from convrot_mlx_b200 import _lib
from convrot_mlx_b200.tp import shard_range, shard_weight
from oracle import convrot_oracle as O


def test_shard_range():
    assert shard_range(15360, 8, 0, _lib.LAYOUT_KN) == (0, 1920)
    assert shard_range(15360, 8, 7, _lib.LAYOUT_KN) == (13440, 15360)
    assert shard_range(5120, 4, 2, _lib.LAYOUT_NK) == (2560, 3840)
    with pytest.raises(ValueError):
        shard_range(100, 3, 0, _lib.LAYOUT_NK)       # does not split
    with pytest.raises(ValueError):
        shard_range(13824 + 32 * 3, 8, 0, _lib.LAYOUT_KN)  # shard not a multiple of 32
    with pytest.raises(ValueError):
        shard_range(1024, 2, 2, _lib.LAYOUT_KN)


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
def test_shard_weight_matches_oracle_columns(layout):
    rng = np.random.default_rng(5)
    k, n, world = 128, 256, 4
    w = rng.integers(-8, 8, size=(n, k)).astype(np.int8)
    q = O.pack_signed_int4(w.T.copy()) if layout == _lib.LAYOUT_KN else O.pack_signed_int4(w)
    for r in range(world):
        a, b = shard_range(n, world, r, layout)
        part = shard_weight(torch.from_numpy(q), layout, a, b).numpy()
        want = w[a:b]
        got = O.unpack_signed_int4(part).T if layout == _lib.LAYOUT_KN else O.unpack_signed_int4(part)
        np.testing.assert_array_equal(got, want)


def _gloo_rank(rank, world, port, layout, out_path):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        k, n = 64, 128
        w = rng.integers(-8, 8, size=(n, k)).astype(np.int8)
        q = torch.from_numpy(O.pack_signed_int4(w.T.copy()) if layout == _lib.LAYOUT_KN else O.pack_signed_int4(w))
        a, b = shard_range(n, world, rank, layout)
        part = shard_weight(q, layout, a, b)
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        full = torch.cat(parts, dim=1 if layout == _lib.LAYOUT_KN else 0)
        ok = torch.equal(full, q)
    finally:
        dist.destroy_process_group()
    with open(f"{out_path}.{rank}", "w") as f:
        f.write("ok" if ok else "bad")


@pytest.mark.parametrize("layout", [_lib.LAYOUT_KN, _lib.LAYOUT_NK])
def test_gloo_world_two_gathers_full_weight(tmp_path, layout):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "gloo")
    ctx = mp.start_processes(_gloo_rank, args=(2, port, layout, path), nprocs=2, join=False, start_method="spawn")
    assert ctx.join(timeout=120) or ctx.join(timeout=30)
    for r in range(2):
        assert open(f"{path}.{r}").read() == "ok"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_gather_plan_by_world(world):
    from convrot_mlx_b200.tp import ColumnParallelConvRotLinear

    def layer(gather, epilogue_peers=None, chunks=None):
        tp = object.__new__(ColumnParallelConvRotLinear)  # the plan reads only these four fields
        tp.world, tp.gather, tp.epilogue_peers, tp.chunks = world, gather, epilogue_peers, chunks
        return tp

    def plan(gather, epilogue_peers=None):
        return layer(gather, epilogue_peers).epilogue_peer_count()

    peers = world - 1
    assert plan("epilogue") == peers
    assert plan("copy-engine") == 0
    assert plan("split") == peers // 2
    assert plan("split", 99) == peers
    assert plan("split", 1) == min(1, peers)
    assert plan("auto") == (0 if world <= 4 else peers // 2)
    assert layer("auto").row_blocks() == (4 if world <= 4 else 2)
    assert layer("split", chunks=3).row_blocks() == 3
