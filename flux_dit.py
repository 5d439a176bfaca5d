"""A random-init FLUX.1-dev-architecture diffusion transformer: the DiT
workload of ``bench.py`` and of ``tests/test_gpu_dit.py``.

Provenance.  Written for this repository from the published description of
the FLUX.1 [dev] transformer (Black Forest Labs, reference implementation
github.com/black-forest-labs/flux, Apache-2.0): 19 double-stream and 38
single-stream blocks, hidden width 3072, 24 heads of 128, MLP ratio 4,
three-axis rotary position embedding with axis widths (16, 56, 56) and base
10000, 64 latent channels in and out, a 4096-wide text context, a 768-wide
pooled vector, timestep and guidance embeddings, and adaptive-LayerNorm
("modulation") conditioning.  No code of that project is reproduced here;
a random-init benchmark model needs the architecture's shapes and the order
of its operations, not its weights or exact numerics.  The reference
(Lumenbeing/convrot-mlx) runs FLUX through Apple's MLX example model
(``examples/flux1_dev/adapter.py``), which is not vendored.

Every linear whose input width is a multiple of 256 is eligible for the
ConvRot swap (313 of 314).  Where a block feeds a modulated LayerNorm
straight into a linear -- ``linear((1 + scale) * LN(x) + shift)``, the qkv and
first MLP projections of both streams and the single blocks' fused
projection -- and the linear is a ``ConvRotLinear`` with
``fuse_modulated_norm`` set on the model, the norm, the modulation, the
rotation and the A4 quantization run as one kernel
(``ConvRotLinear.forward_modulated_norm``); with the attention glue on as
well, the single blocks' output projection likewise quantizes
cat(attention, gelu(mlp)) straight from its two parts
(``ConvRotLinear.forward_gelu_concat``).

``fuse_attention_glue`` (both arms of the benchmark) runs the q/k RMSNorm,
the rotary embedding and the attention layout of q, k, v as one kernel, and
the single blocks' GELU with the concatenation after attention as another
(``flux_dit_glue.cu``, built by ``build_glue``).
"""

from __future__ import annotations

import ctypes
import math
import shutil
import subprocess
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import nn

_HERE = Path(__file__).resolve().parent
_GLUE_SRC = _HERE / "flux_dit_glue.cu"
_GLUE_LIB = _HERE / "libflux_dit_glue.so"
_glue = None


def build_glue(force: bool = False) -> Path:
    """Compile ``flux_dit_glue.cu`` (the attention glue of this model: q/k
    RMSNorm + rotary embedding + attention layout) for sm_100a, in-tree."""

    if force or not _GLUE_LIB.exists() or _GLUE_LIB.stat().st_mtime < _GLUE_SRC.stat().st_mtime:
        nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
        subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
                        "-Xcompiler", "-fPIC", "-shared", str(_GLUE_SRC), "-o", str(_GLUE_LIB)],
                       check=True, capture_output=True)
    return _GLUE_LIB


def glue():
    """The attention-glue library, or None when it was not built."""

    global _glue
    if _glue is None and _GLUE_LIB.exists():
        lib = ctypes.CDLL(str(_GLUE_LIB))
        P, I64 = ctypes.c_void_p, ctypes.c_int64
        lib.flux_qk_norm_rope.argtypes = [P, I64, I64, I64, I64, P, P, ctypes.c_float, P, I64, I64, P, P, P, P]
        lib.flux_qk_norm_rope.restype = ctypes.c_int
        lib.flux_gelu_concat.argtypes = [P, I64, P, I64, I64, I64, I64, P, P]
        lib.flux_gelu_concat.restype = ctypes.c_int
        _glue = lib
    return _glue

FLUX_DEV = dict(hidden=3072, heads=24, mlp_ratio=4.0, depth=19, depth_single=38, in_channels=64, context=4096,
                vec=768, axes=(16, 56, 56), theta=10000)

LN_EPS = 1e-6


def timestep_features(t: torch.Tensor, width: int = 256, base: float = 10000.0, multiplier: float = 1000.0):
    """Sinusoidal features of a (batch,) time value: cosines then sines of
    ``multiplier * t`` at ``width / 2`` geometrically spaced frequencies."""

    half = width // 2
    exponents = torch.arange(half, dtype=torch.float32, device=t.device) * (-math.log(base) / half)
    angles = (multiplier * t.float())[:, None] * torch.exp(exponents)[None, :]
    return torch.cat((angles.cos(), angles.sin()), dim=1)


def rotary_tables(ids: torch.Tensor, axes, theta: float) -> torch.Tensor:
    """Unit complex rotations, (batch, 1, tokens, sum(axes) / 2) complex64,
    for the three-axis rotary embedding: the pairs of head dimensions of axis
    a turn by ``position_a * theta ** (-2 j / width_a)``."""

    angles = []
    for a, width in enumerate(axes):
        j = torch.arange(width // 2, dtype=torch.float64, device=ids.device)
        inv_freq = theta ** (-2.0 * j / width)
        angles.append(ids[..., a].double()[..., None] * inv_freq)
    ang = torch.cat(angles, dim=-1)
    return torch.polar(torch.ones_like(ang), ang).to(torch.complex64)[:, None]


def rotate_pairs(x: torch.Tensor, rot: torch.Tensor) -> torch.Tensor:
    """Rotate consecutive pairs (x[2j], x[2j + 1]) of the head dimension of x
    (batch, heads, tokens, dim) by the angles of ``rotary_tables``: one
    complex multiply per pair in float32, (x0 + i x1) (cos + i sin)."""

    xc = torch.view_as_complex(x.float().unflatten(-1, (-1, 2)))
    return torch.view_as_real(xc * rot).flatten(-2).to(x.dtype)


class RMSNorm(nn.Module):
    def __init__(self, width: int):
        super().__init__()
        self.scale = nn.Parameter(torch.ones(width))

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.scale.to(x.dtype), 1e-6)


class Modulation(nn.Module):
    """SiLU(vec) -> one linear -> ``count`` (batch, 1, width) chunks."""

    def __init__(self, width: int, count: int):
        super().__init__()
        self.count = count
        self.lin = nn.Linear(width, count * width)

    def forward(self, vec):
        return self.lin(F.silu(vec)).unsqueeze(1).chunk(self.count, dim=-1)


class Embedder(nn.Module):
    """Two-layer MLP embedder (linear, SiLU, linear)."""

    def __init__(self, width_in: int, width: int):
        super().__init__()
        self.in_layer = nn.Linear(width_in, width)
        self.out_layer = nn.Linear(width, width)

    def forward(self, x):
        return self.out_layer(F.silu(self.in_layer(x)))


def modulated_linear(model_flags, linear: nn.Module, x, shift, scale):
    """``linear((1 + scale) * LayerNorm(x) + shift)``, fused into one kernel
    before the GEMM when the model asks for it and the linear supports it."""

    fused = getattr(linear, "forward_modulated_norm", None)
    if fused is not None and model_flags.get("fuse_modulated_norm", False):
        return fused(x, shift, scale, LN_EPS)
    normed = F.layer_norm(x, (x.shape[-1],), eps=LN_EPS)
    return linear(torch.addcmul(shift, normed, 1 + scale))


def split_heads(qkv: torch.Tensor, heads: int):
    """(batch, tokens, 3 * heads * dim) -> three (batch, heads, tokens, dim)."""

    b, n, _ = qkv.shape
    q, k, v = qkv.view(b, n, 3, heads, -1).permute(2, 0, 3, 1, 4)
    return q, k, v


class Attention(nn.Module):
    def __init__(self, width: int, heads: int):
        super().__init__()
        self.heads = heads
        self.qkv = nn.Linear(width, 3 * width)
        self.q_norm = RMSNorm(width // heads)
        self.k_norm = RMSNorm(width // heads)
        self.proj = nn.Linear(width, width)

    def qkv_heads(self, qkv):
        q, k, v = split_heads(qkv, self.heads)
        return self.q_norm(q), self.k_norm(k), v


def attend(q, k, v, rot):
    q, k = rotate_pairs(q, rot), rotate_pairs(k, rot)
    o = F.scaled_dot_product_attention(q, k, v)
    return o.transpose(1, 2).flatten(2)


def fused_attention_inputs(parts, rot, heads):
    """q, k, v (batch, heads, tokens, 128) for attention from one or more
    projection outputs, each (qkv rows (batch, tokens, >= 3 heads 128), its
    Attention / block with q_norm and k_norm), placed side by side along the
    tokens: the q/k RMSNorm, the rotary embedding and the layout change in
    one kernel per part (``flux_dit_glue.cu``)."""

    b = parts[0][0].shape[0]
    total = sum(x.shape[1] for x, _ in parts)
    dev = parts[0][0].device
    q, k, v = (torch.empty((b, heads, total, 128), dtype=torch.bfloat16, device=dev) for _ in range(3))
    rot_f = torch.view_as_real(rot[:, 0].contiguous())  # (batch, total, 64, 2)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    off = 0
    lib = glue()
    for x, owner in parts:
        qs = owner.q_norm.scale.to(torch.bfloat16)
        ks = owner.k_norm.scale.to(torch.bfloat16)
        rc = lib.flux_qk_norm_rope(x.data_ptr(), x.stride(1), b, x.shape[1], heads, qs.data_ptr(), ks.data_ptr(),
                                   1e-6, rot_f.data_ptr(), off, total, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                   stream)
        if rc != 0:
            raise RuntimeError(f"flux_qk_norm_rope failed ({rc})")
        off += x.shape[1]
    o = F.scaled_dot_product_attention(q, k, v)
    return o.transpose(1, 2).flatten(2)


def gelu_concat(a: torch.Tensor, m: torch.Tensor) -> torch.Tensor:
    """``torch.cat((a, gelu_tanh(m)), -1)`` in one kernel; m may be a column
    slice of a wider tensor (rows of a fixed stride)."""

    b, n = a.shape[0], a.shape[1]
    out = torch.empty((b, n, a.shape[2] + m.shape[2]), dtype=torch.bfloat16, device=a.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(a.device).cuda_stream)
    rc = glue().flux_gelu_concat(a.data_ptr(), a.stride(1), m.data_ptr(), m.stride(1), b * n, a.shape[2], m.shape[2],
                                 out.data_ptr(), stream)
    if rc != 0:
        raise RuntimeError(f"flux_gelu_concat failed ({rc})")
    return out


def _use_glue(flags, x) -> bool:
    return flags.get("fuse_attention_glue", False) and x.is_cuda and x.dtype == torch.bfloat16 and glue() is not None


class DoubleStreamBlock(nn.Module):
    """Image and text tokens keep separate weights and join for attention."""

    def __init__(self, width: int, heads: int, mlp: int, flags: dict):
        super().__init__()
        self.flags = flags
        self.img_mod, self.txt_mod = Modulation(width, 6), Modulation(width, 6)
        self.img_attn, self.txt_attn = Attention(width, heads), Attention(width, heads)
        self.img_mlp = nn.Sequential(nn.Linear(width, mlp), nn.GELU(approximate="tanh"), nn.Linear(mlp, width))
        self.txt_mlp = nn.Sequential(nn.Linear(width, mlp), nn.GELU(approximate="tanh"), nn.Linear(mlp, width))

    def _stream_mlp(self, x, mod, mlp):
        h = modulated_linear(self.flags, mlp[0], x, mod[3], mod[4])
        return torch.addcmul(x, mod[5], mlp[2](mlp[1](h)))

    def forward(self, img, txt, vec, rot):
        im, tm = self.img_mod(vec), self.txt_mod(vec)
        t_qkv = modulated_linear(self.flags, self.txt_attn.qkv, txt, tm[0], tm[1])
        i_qkv = modulated_linear(self.flags, self.img_attn.qkv, img, im[0], im[1])
        if _use_glue(self.flags, t_qkv):
            a = fused_attention_inputs([(t_qkv, self.txt_attn), (i_qkv, self.img_attn)], rot, self.txt_attn.heads)
        else:
            tq, tk, tv = self.txt_attn.qkv_heads(t_qkv)
            iq, ik, iv = self.img_attn.qkv_heads(i_qkv)
            a = attend(torch.cat((tq, iq), 2), torch.cat((tk, ik), 2), torch.cat((tv, iv), 2), rot)
        n_txt = txt.shape[1]
        txt = torch.addcmul(txt, tm[2], self.txt_attn.proj(a[:, :n_txt]))
        img = torch.addcmul(img, im[2], self.img_attn.proj(a[:, n_txt:]))
        return self._stream_mlp(img, im, self.img_mlp), self._stream_mlp(txt, tm, self.txt_mlp)


class SingleStreamBlock(nn.Module):
    """One weight set over the joined sequence; attention and MLP in parallel
    from one fused input projection, joined again by one output projection."""

    def __init__(self, width: int, heads: int, mlp: int, flags: dict):
        super().__init__()
        self.flags = flags
        self.width, self.heads, self.mlp = width, heads, mlp
        self.linear1 = nn.Linear(width, 3 * width + mlp)
        self.linear2 = nn.Linear(width + mlp, width)
        self.q_norm, self.k_norm = RMSNorm(width // heads), RMSNorm(width // heads)
        self.act = nn.GELU(approximate="tanh")
        self.modulation = Modulation(width, 3)

    def forward(self, x, vec, rot):
        shift, scale, gate = self.modulation(vec)
        h = modulated_linear(self.flags, self.linear1, x, shift, scale)
        qkv, m = h.split((3 * self.width, self.mlp), dim=-1)
        if _use_glue(self.flags, h):
            a = fused_attention_inputs([(h, self)], rot, self.heads)
            fused = getattr(self.linear2, "forward_gelu_concat", None)
            if fused is not None and self.flags.get("fuse_modulated_norm", False):
                return torch.addcmul(x, gate, fused(a, m))
            return torch.addcmul(x, gate, self.linear2(gelu_concat(a, m)))
        q, k, v = split_heads(qkv, self.heads)
        a = attend(self.q_norm(q), self.k_norm(k), v, rot)
        return torch.addcmul(x, gate, self.linear2(torch.cat((a, self.act(m)), dim=-1)))


class FluxDiT(nn.Module):
    """The FLUX.1-dev transformer: (latents, text, rotary tables, t, pooled
    vector, guidance) -> predicted velocity of the latents."""

    def __init__(self, cfg=FLUX_DEV):
        super().__init__()
        width, heads = cfg["hidden"], cfg["heads"]
        mlp = int(width * cfg["mlp_ratio"])
        self.cfg = cfg
        self.flags = {"fuse_modulated_norm": False, "fuse_attention_glue": False}
        self.img_in = nn.Linear(cfg["in_channels"], width)
        self.time_in = Embedder(256, width)
        self.guidance_in = Embedder(256, width)
        self.vector_in = Embedder(cfg["vec"], width)
        self.txt_in = nn.Linear(cfg["context"], width)
        self.double_blocks = nn.ModuleList(
            [DoubleStreamBlock(width, heads, mlp, self.flags) for _ in range(cfg["depth"])])
        self.single_blocks = nn.ModuleList(
            [SingleStreamBlock(width, heads, mlp, self.flags) for _ in range(cfg["depth_single"])])
        self.final_mod = Modulation(width, 2)
        self.final_linear = nn.Linear(width, cfg["in_channels"])

    @property
    def fuse_attention_glue(self) -> bool:
        return self.flags["fuse_attention_glue"]

    @fuse_attention_glue.setter
    def fuse_attention_glue(self, on: bool) -> None:
        self.flags["fuse_attention_glue"] = bool(on)

    @property
    def fuse_modulated_norm(self) -> bool:
        return self.flags["fuse_modulated_norm"]

    @fuse_modulated_norm.setter
    def fuse_modulated_norm(self, on: bool) -> None:
        self.flags["fuse_modulated_norm"] = bool(on)

    def rotary(self, ids):
        return rotary_tables(ids, self.cfg["axes"], self.cfg["theta"])

    def forward(self, img, txt, rot, t, y, guidance):
        dt = img.dtype
        vec = self.time_in(timestep_features(t).to(dt)) + self.guidance_in(timestep_features(guidance).to(dt))
        vec = vec + self.vector_in(y)
        img, txt = self.img_in(img), self.txt_in(txt)
        for blk in self.double_blocks:
            img, txt = blk(img, txt, vec, rot)
        x = torch.cat((txt, img), dim=1)
        for blk in self.single_blocks:
            x = blk(x, vec, rot)
        x = x[:, txt.shape[1]:]
        shift, scale = self.final_mod(vec)
        x = torch.addcmul(shift, F.layer_norm(x, (x.shape[-1],), eps=LN_EPS), 1 + scale)
        return self.final_linear(x)


def build_flux_dit(device, seed: int, cfg=FLUX_DEV) -> FluxDiT:
    """Random-init bf16 model: linear weights ~ N(0, 0.02), biases ~ N(0,
    0.01), norm scales 1.  Built on the meta device and materialized in bf16,
    so no float32 copy of the ~12 B parameters is ever held."""

    with torch.device("meta"):
        model = FluxDiT(cfg)
    model = model.to_empty(device=device).to(torch.bfloat16)
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, nn.Linear):
                m.weight.normal_(0.0, 0.02, generator=g)
                if m.bias is not None:
                    m.bias.normal_(0.0, 0.01, generator=g)
            elif isinstance(m, RMSNorm):
                m.scale.fill_(1.0)
    return model.eval()


def dit_inputs(batch: int, device, seed: int, cfg=FLUX_DEV, img_tokens: int = 1024, txt_tokens: int = 512):
    """Seeded synthetic latents, text context and pooled vector, and the
    position ids (text at 0; image on a square grid along axes 1 and 2)."""

    g = torch.Generator(device=device).manual_seed(seed)
    side = int(round(img_tokens ** 0.5))
    img = torch.randn((batch, img_tokens, cfg["in_channels"]), generator=g, device=device).to(torch.bfloat16)
    txt = torch.randn((batch, txt_tokens, cfg["context"]), generator=g, device=device).to(torch.bfloat16)
    y = torch.randn((batch, cfg["vec"]), generator=g, device=device).to(torch.bfloat16)
    ids = torch.zeros((batch, txt_tokens + img_tokens, 3), device=device)
    rows = torch.arange(img_tokens, device=device)
    ids[:, txt_tokens:, 1] = (rows // side).float()
    ids[:, txt_tokens:, 2] = (rows % side).float()
    return img, txt, y, ids


def linear_ops_per_sample(cfg=FLUX_DEV, tokens: int = 1536) -> int:
    """Multiply-add ops (2 per MAC) of the block linears for one sample and
    one forward (the embedders and final layer are negligible)."""

    d = cfg["hidden"]
    mlp = int(d * cfg["mlp_ratio"])
    double = cfg["depth"] * 2 * tokens * d * (3 * d + d + 2 * mlp)
    single = cfg["depth_single"] * 2 * tokens * (d * (3 * d + mlp) + (d + mlp) * d)
    return double + single
