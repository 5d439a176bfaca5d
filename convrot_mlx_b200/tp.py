"""Tensor-parallel ConvRot W4A4 linear: column split of N over the GPUs of one node.

The multi-GPU form of ``ConvRotLinear`` (core.py:1213-1313 of the reference,
which runs on a single Apple GPU).  Rank r of a process group of ``world``
GPUs owns output columns ``[r * N / world, (r + 1) * N / world)``: that slice
of the packed weight (K x packed-N: a column slice of the bytes; N x
packed-K: a row slice), of the weight scales and of the bias.  The
activation is replicated and every rank runs the fused rotate + quantize on
it (cheaper than broadcasting the codes).  Every rank's full (M, N) output
buffer is symmetric memory, mapped on every GPU, and the all-gather crosses
NVLink in one of these ways:

* ``gather="copy-engine"``: the GEMM runs in ``row_blocks()`` blocks of rows
  into this rank's own buffer; after each block one strided copy per peer
  (``convrot_copy_2d``) pushes it into the peers' buffers on side streams,
  so the copy engines carry block i while the SMs compute block i + 1.
* ``gather="epilogue"``: the GEMM's epilogue (``convrot_w4a4_gemm_gather``)
  stores each output tile into every rank's buffer itself, as peer stores.
* ``gather="split"``: both at once, for different peers.  The chunked
  GEMM's epilogue stores into this rank's buffer and those of the next
  ``epilogue_peers`` ranks; the copy engines push each block to the rest.
  The two use separate hardware: on B200, with all 8 ranks pushing at once,
  the copy engines carry ~400 GB/s per GPU and the epilogue's peer stores
  ~370 GB/s, below the ~770 GB/s a GPU's links take.
* ``gather="auto"`` (the default): copy engines alone in 4 row blocks up
  to 4 ranks (where they carry 650-740 GB/s), above that the split with
  ``(world - 1) // 2`` epilogue peers in 2 row blocks (at 8 GPUs 4.9 ms per
  step of the video-DiT linears against 5.7 ms for either gather alone).

Either way a flag barrier (``convrot_peer_barrier``) then makes every rank's
full output visible.

Buffers are symmetric-memory tensors (``torch.distributed._symmetric_memory``,
CUDA backend, multicast off) allocated once per (rows, dtype).  Outputs
alternate between two buffers: a rank that has passed call i + 1's barrier
knows every rank has finished call i (whose output it may still be reading
until its own call i + 1), so call i + 2 may overwrite buffer i % 2.  The
tensor returned by ``forward`` is therefore valid until the call after next.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist
from torch import nn

from . import _lib
from .core import (
    CONVROT_GROUP_SIZE,
    ConvRotLinear,
    _dtype_code,
    _f32_vec,
    _prepare,
)

_MAX_WORLD = 8
_GATHERS = ("auto", "copy-engine", "epilogue", "split")


def shard_range(out_features: int, world: int, rank: int, layout: int) -> tuple[int, int]:
    """Columns ``[start, stop)`` owned by ``rank``.

    N must split evenly; for K x packed-N weights each shard must also be a
    whole number of 16-byte rows (N / world % 32 == 0), as the two-CTA GEMM
    reads weight rows with TMA.
    """

    if not 1 <= world <= _MAX_WORLD:
        raise ValueError(f"world size must be in [1, {_MAX_WORLD}], got {world}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    if out_features % world:
        raise ValueError(f"out_features {out_features} does not split over {world} ranks")
    shard = out_features // world
    if layout == _lib.LAYOUT_KN and shard % 32:
        raise ValueError(f"K x packed-N shards need out_features / world % 32 == 0, got {shard}")
    return rank * shard, (rank + 1) * shard


def shard_weight(qweight: torch.Tensor, layout: int, start: int, stop: int) -> torch.Tensor:
    """The packed weight of columns [start, stop) (both even)."""

    if start % 2 or stop % 2:
        raise ValueError("shard bounds must be even (two columns per packed byte)")
    if layout == _lib.LAYOUT_KN:
        return qweight[:, start // 2 : stop // 2].contiguous()
    return qweight[start:stop].contiguous()


class ColumnParallelConvRotLinear(nn.Module):
    """One rank's shard of a ConvRotLinear split over N (see the module doc)."""

    def __init__(self, in_features: int, out_features: int, *, group: dist.ProcessGroup | None = None,
                 bias: bool = True, group_size: int = CONVROT_GROUP_SIZE, backend: str = "mpp-w4a4",
                 device=None, gather: str = "auto", chunks: int | None = None,
                 epilogue_peers: int | None = None) -> None:
        super().__init__()
        if gather not in _GATHERS:
            raise ValueError(f"gather must be one of {_GATHERS}, got {gather!r}")
        if chunks is not None and chunks < 1:
            raise ValueError(f"chunks must be positive, got {chunks}")
        if epilogue_peers is not None and epilogue_peers < 0:
            raise ValueError(f"epilogue_peers must be non-negative, got {epilogue_peers}")
        self.gather = gather
        self.chunks = chunks
        self.epilogue_peers = epilogue_peers
        self._side = None  # copy-engine gather: one stream per peer
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        if backend == "mpp-w4a16":
            raise ValueError("the tensor-parallel layer implements the W4A4 backends")
        local = ConvRotLinear(in_features, out_features, bias=bias, group_size=group_size, backend=backend,
                              device=device)
        self.layout = local.layout_code
        self.start, self.stop = shard_range(out_features, self.world, self.rank, self.layout)
        self.shard_features = self.stop - self.start
        self.register_buffer("qweight", shard_weight(local.qweight, self.layout, self.start, self.stop))
        self.register_buffer("scales", local.scales[self.start : self.stop].clone())
        self.register_buffer("bias", local.bias[self.start : self.stop].clone())
        self.source_has_bias = bias
        self._out = {}      # (rows, dtype) -> two (tensor, peer pointer array, handle)
        self._flags = None  # (tensor, peer pointer array)
        self._epoch = 0     # barrier epoch (never 0)
        self._calls = 0     # output buffer = calls % 2

    @classmethod
    def from_full(cls, layer: ConvRotLinear, group: dist.ProcessGroup | None = None, *, gather: str = "auto",
                  chunks: int | None = None, epilogue_peers: int | None = None) -> "ColumnParallelConvRotLinear":
        """Shard a full (already quantized) ConvRotLinear on every rank."""

        tp = cls(layer.in_features, layer.out_features, group=group, bias=layer.source_has_bias,
                 group_size=layer.group_size, backend=layer.backend, device=layer.qweight.device, gather=gather,
                 chunks=chunks, epilogue_peers=epilogue_peers)
        tp.qweight = shard_weight(layer.qweight, tp.layout, tp.start, tp.stop)
        tp.scales = _f32_vec(layer.scales)[tp.start : tp.stop].clone()
        tp.bias = _f32_vec(layer.bias)[tp.start : tp.stop].clone()
        return tp

    # -- symmetric buffers ---------------------------------------------------

    def _symmetric(self, shape, dtype):
        import torch.distributed._symmetric_memory as symm

        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")  # plain peer stores only
        try:
            symm.set_backend("CUDA")
        except Exception:  # already set
            pass
        t = symm.empty(*shape, dtype=dtype, device=self.qweight.device)
        handle = symm.rendezvous(t, self.group)
        ptrs = (ctypes.c_void_p * self.world)(*[int(p) for p in handle.buffer_ptrs])
        return t, ptrs, handle

    def _output(self, rows: int, dtype: torch.dtype, which: int):
        key = (rows, dtype)
        if key not in self._out:
            self._out[key] = [self._symmetric((rows, self.out_features), dtype) for _ in range(2)]
        return self._out[key][which]

    def _flag_arrays(self):
        if self._flags is None:
            t, ptrs, handle = self._symmetric((self.world,), torch.int32)
            t.zero_()
            torch.cuda.synchronize(t.device)
            dist.barrier(self.group)  # every rank's flags are zero before any barrier kernel runs
            self._flags = (t, ptrs, handle)
        return self._flags

    # -- forward ---------------------------------------------------------------

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"ConvRotLinear expected K={self.in_features}, got {x.shape[-1]}")
        lead = x.shape[:-1]
        x2d = x.reshape(-1, self.in_features)
        m = x2d.shape[0]
        _, flag_ptrs, _ = self._flag_arrays()
        self._epoch = (self._epoch % 0x7FFFFFFF) + 1
        self._calls += 1
        out, out_ptrs, _ = self._output(m, x.dtype, self._calls & 1)
        lib = _lib.load()
        stream = _lib.stream_of(x2d)
        codes, xscales = _prepare(x2d, self.group_size, packed=False)
        epi = self.epilogue_peer_count()
        if self.world == 1 or (epi == self.world - 1 and self.gather != "split"):
            _lib.check(
                lib.convrot_w4a4_gemm_gather(
                    _lib.ptr(codes), _lib.ptr(self.qweight), self.layout, _lib.ptr(xscales), _lib.ptr(self.scales),
                    _lib.ptr(self.bias), out_ptrs, self.world, self.out_features, self.start, _dtype_code(x.dtype),
                    m, self.shard_features, self.in_features, stream,
                ),
                "tensor-parallel W4A4 GEMM",
            )
        else:
            self._gemm_and_copy(lib, codes, xscales, out, out_ptrs, m, x.dtype, stream, epi)
        _lib.check(lib.convrot_peer_barrier(ctypes.cast(flag_ptrs, ctypes.POINTER(ctypes.c_void_p)), self.world,
                                            self.rank, self._epoch, stream), "peer barrier")
        return out.reshape(*lead, self.out_features)

    def epilogue_peer_count(self) -> int:
        """How many peers the GEMM's epilogue stores into; the copy engines
        serve the other ``world - 1 - epilogue_peer_count()``."""

        peers = self.world - 1
        if self.gather == "epilogue" or peers == 0:
            return peers
        if self.gather == "copy-engine":
            return 0
        if self.gather == "split":
            return min(peers, peers // 2 if self.epilogue_peers is None else self.epilogue_peers)
        return 0 if self.world <= 4 else peers // 2

    def row_blocks(self) -> int:
        """Blocks of rows of the chunked gathers: ``chunks`` if given, else 4
        up to 4 ranks and 2 above (at 8 ranks each block's GEMM is small, and
        per-block costs outweigh the finer overlap)."""

        if self.chunks is not None:
            return self.chunks
        return 4 if self.world <= 4 else 2

    def _gemm_and_copy(self, lib, codes, xscales, out, out_ptrs, m, dtype, stream, epi: int) -> None:
        """The chunked gathers: the shard GEMM in blocks of rows into this
        rank's buffer and those of the next ``epi`` ranks (epilogue peer
        stores), each block pushed to the remaining peers by a strided copy
        on a side stream while the next block computes; the current stream
        then waits for every copy."""

        dev = out.device
        cur = torch.cuda.current_stream(dev)
        if self._side is None:
            self._side = [torch.cuda.Stream(device=dev) for _ in range(self.world)]
        elt = out.element_size()
        ldc = self.out_features
        k = self.in_features
        rows = -(-m // self.row_blocks())
        rows = -(-rows // 256) * 256  # whole 256-row pair tiles
        own = out.data_ptr()
        order = [(self.rank + i) % self.world for i in range(1, self.world)]
        by_epilogue, by_copy = order[:epi], order[epi:]
        bases = [own] + [int(out_ptrs[p]) for p in by_epilogue]
        for r0 in range(0, m, rows):
            mr = min(rows, m - r0)
            dst = (ctypes.c_void_p * len(bases))(*[b + r0 * ldc * elt for b in bases])
            _lib.check(
                lib.convrot_w4a4_gemm_gather(
                    ctypes.c_void_p(codes.data_ptr() + r0 * k), _lib.ptr(self.qweight), self.layout,
                    ctypes.c_void_p(xscales.data_ptr() + 4 * r0), _lib.ptr(self.scales), _lib.ptr(self.bias), dst,
                    len(bases), ldc, self.start, _dtype_code(dtype), mr, self.shard_features, k, stream,
                ),
                "tensor-parallel W4A4 GEMM",
            )
            if not by_copy:
                continue
            done = torch.cuda.Event()
            done.record(cur)
            offset = (r0 * ldc + self.start) * elt
            for p in by_copy:
                side = self._side[p]
                side.wait_event(done)
                _lib.check(lib.convrot_copy_2d(ctypes.c_void_p(int(out_ptrs[p]) + offset), ldc * elt,
                                               ctypes.c_void_p(own + offset), ldc * elt, self.shard_features * elt,
                                               mr, ctypes.c_void_p(side.cuda_stream)), "peer copy")
        for p in by_copy:
            copied = torch.cuda.Event()
            copied.record(self._side[p])
            cur.wait_event(copied)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, world={self.world}, "
                f"rank={self.rank}, columns=[{self.start}, {self.stop}), gather={self.gather}, "
                f"epilogue_peers={self.epilogue_peer_count()}")
