"""The FLUX-architecture DiT of flux_dit.py with its eligible
linears swapped by replace_convrot_linears: every swapped layer equals a
ConvRotLinear built by hand from the same dense weight (bit for bit), and
the W4A4 model stays close to the dense bf16 one (a loose sanity bound: W4A4
quantizes every linear's input and weight to 15 levels)."""

from __future__ import annotations

import pytest
import torch

import flux_dit
import convrot_mlx_b200 as cr
from convrot_mlx_b200.adapter import replace_convrot_linears
from tests.gpu_util import assert_no_device_error, dev

pytestmark = pytest.mark.gpu

TINY = dict(flux_dit.FLUX_DEV, hidden=512, heads=4, depth=2, depth_single=2, context=512, vec=256)


def test_swapped_layers_match_hand_built_layers():
    model = flux_dit.build_flux_dit(dev(), 5, TINY)
    dense = {n: m.weight.detach().clone() for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)}
    biases = {n: m.bias.detach().clone() for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)}
    names = replace_convrot_linears(model, backend="mpp-w4a4")
    assert len(names) == sum(1 for n in dense if n != "img_in")
    g = torch.Generator(device=dev()).manual_seed(9)
    for name in names[:6] + names[-3:]:
        layer = dict(model.named_modules())[name]
        w = dense[name]
        ref = cr.ConvRotLinear(w.shape[1], w.shape[0], backend="mpp-w4a4", device=dev())
        qnk, ws = cr.quantize_convrot_weight(w)
        ref.qweight, ref.scales, ref.bias = cr.repack_nk_weight_for_mpp(qnk), ws, biases[name].float()
        x = torch.randn((37, w.shape[1]), generator=g, device=dev()).to(torch.bfloat16)
        assert torch.equal(layer(x).view(torch.int16), ref(x).view(torch.int16)), name
    assert_no_device_error()


def test_w4a4_dit_tracks_dense_dit():
    model = flux_dit.build_flux_dit(dev(), 6, TINY)
    img, txt, y, ids = flux_dit.dit_inputs(2, dev(), 7, TINY, img_tokens=64, txt_tokens=32)
    t = torch.tensor([0.7, 0.3], device=dev())
    guide = torch.full((2,), 3.5, device=dev())
    with torch.no_grad():
        pe = model.rotary(ids)
        want = model(img, txt, pe, t, y, guide).float()
        replace_convrot_linears(model, backend="mpp-w4a4")
        got = model(img, txt, pe, t, y, guide).float()
    assert bool(torch.isfinite(got).all())
    rel = float((got - want).norm() / want.norm())
    assert 0.0 < rel < 0.5, rel
    assert_no_device_error()


def test_fused_modulated_norm_codes_inside_the_dit(monkeypatch):
    # every modulated-norm projection of a W4A4 DiT forward, fused: on the same
    # inputs its codes equal those of layer_norm + addcmul + prep up to the
    # float32 order of the LayerNorm statistics (a code off by one, rarely).
    # Whole-model outputs are not compared: a random-init W4A4 model amplifies
    # a single flipped code by orders of magnitude.
    from convrot_mlx_b200.core import _prepare, modulated_norm_prepare_i8

    model = flux_dit.build_flux_dit(dev(), 8, TINY)
    img, txt, y, ids = flux_dit.dit_inputs(2, dev(), 9, TINY, img_tokens=64, txt_tokens=32)
    t = torch.tensor([0.6, 0.2], device=dev())
    guide = torch.full((2,), 3.5, device=dev())
    stats = []
    orig = cr.ConvRotLinear.forward_modulated_norm

    def checked(self, x, shift, scale, eps=1e-6):
        k = x.shape[-1]
        fc, fs = modulated_norm_prepare_i8(x, shift, scale, eps, self.group_size)
        xm = torch.addcmul(shift, torch.nn.functional.layer_norm(x, (k,), eps=eps), 1 + scale)
        uc, us = _prepare(xm.reshape(-1, k), self.group_size, packed=False)
        d = (fc.int() - uc.int()).abs()
        stats.append((int(d.max()), float((d != 0).float().mean()), float(((fs - us).abs() / us).max())))
        return orig(self, x, shift, scale, eps)

    monkeypatch.setattr(cr.ConvRotLinear, "forward_modulated_norm", checked)
    with torch.no_grad():
        pe = model.rotary(ids)
        replace_convrot_linears(model, backend="mpp-w4a4")
        model.fuse_modulated_norm = True
        out = model(img, txt, pe, t, y, guide)
    assert bool(torch.isfinite(out.float()).all())
    assert len(stats) == 4 * TINY["depth"] + TINY["depth_single"]
    assert all(s[0] <= 1 for s in stats), stats
    assert max(s[1] for s in stats) <= 1e-3, stats
    assert max(s[2] for s in stats) <= 2.0 ** -7, stats
    assert_no_device_error()


def test_attention_glue_tracks_torch_ops():
    # q/k RMSNorm + rotary + attention layout in one kernel, against the torch
    # ops it replaces: the two streams side by side, and a single-block row
    # with extra MLP columns (row stride > 3 heads x 128)
    flux_dit.build_glue()
    g = torch.Generator(device=dev()).manual_seed(11)
    b, heads, lt, li = 2, 4, 24, 40
    ids = torch.zeros((b, lt + li, 3), device=dev())
    ids[:, lt:, 1] = torch.arange(li, device=dev()).float() // 8
    ids[:, lt:, 2] = torch.arange(li, device=dev()).float() % 8
    rot = flux_dit.rotary_tables(ids, (16, 56, 56), 10000)
    owners = [flux_dit.Attention(heads * 128, heads).to(dev()), flux_dit.Attention(heads * 128, heads).to(dev())]
    for o in owners:
        o.q_norm.scale.data = (1 + 0.1 * torch.randn(128, generator=g, device=dev())).to(torch.bfloat16)
        o.k_norm.scale.data = (1 + 0.1 * torch.randn(128, generator=g, device=dev())).to(torch.bfloat16)
    t_qkv = torch.randn((b, lt, 3 * heads * 128), generator=g, device=dev()).to(torch.bfloat16)
    wide = torch.randn((b, li, 3 * heads * 128 + 256), generator=g, device=dev()).to(torch.bfloat16)
    i_qkv = wide[..., : 3 * heads * 128]
    with torch.no_grad():
        got = flux_dit.fused_attention_inputs([(t_qkv, owners[0]), (wide, owners[1])], rot, heads).float()
        tq, tk, tv = owners[0].qkv_heads(t_qkv)
        iq, ik, iv = owners[1].qkv_heads(i_qkv)
        want = flux_dit.attend(torch.cat((tq, iq), 2), torch.cat((tk, ik), 2), torch.cat((tv, iv), 2), rot).float()
    rel = float((got - want).norm() / want.norm())
    assert rel < 5e-3, rel


def test_dense_dit_with_attention_glue_tracks_torch_ops():
    model = flux_dit.build_flux_dit(dev(), 12, TINY)
    img, txt, y, ids = flux_dit.dit_inputs(2, dev(), 13, TINY, img_tokens=64, txt_tokens=32)
    t = torch.tensor([0.4, 0.9], device=dev())
    guide = torch.full((2,), 3.5, device=dev())
    flux_dit.build_glue()
    with torch.no_grad():
        rot = model.rotary(ids)
        want = model(img, txt, rot, t, y, guide).float()
        model.fuse_attention_glue = True
        got = model(img, txt, rot, t, y, guide).float()
    rel = float((got - want).norm() / want.norm())
    assert rel < 2e-2, rel


def test_gelu_concat_tracks_torch_ops():
    flux_dit.build_glue()
    g = torch.Generator(device=dev()).manual_seed(14)
    a = torch.randn((2, 33, 512), generator=g, device=dev()).to(torch.bfloat16)
    h = (torch.randn((2, 33, 3 * 512 + 2048), generator=g, device=dev()) * 3).to(torch.bfloat16)
    m = h[..., 3 * 512:]
    got = flux_dit.gelu_concat(a, m).float()
    want = torch.cat((a, torch.nn.functional.gelu(m, approximate="tanh")), dim=-1).float()
    assert torch.equal(got[..., :512], want[..., :512])
    diff = (got - want).abs()
    assert float(diff.max()) <= float(want.abs().max()) * 2.0 ** -7  # within one bf16 ulp of the largest value
    assert float((diff != 0).float().mean()) < 0.05
