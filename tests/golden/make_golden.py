#!/usr/bin/env python3
"""Generate the golden fixtures under ``tests/golden/`` from the reference.

Runs the reference's own eager functions (``src/convrot_mlx/core.py`` of
Lumenbeing/convrot-mlx) with ``mlx`` replaced by the NumPy stand-in in
``_mlx_numpy_shim.py``.  Every case mirrors a test of the reference's
``tests/test_core.py`` (same seeds, same draw order, same shapes) or a
BASELINE configuration, and stores inputs and expected outputs.

Usage (needs the reference checkout; the GPU box does not):

    python tests/golden/make_golden.py --reference /path/to/convrot-mlx

The fixtures are committed; tests never import the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _bits(a) -> np.ndarray:
    """bf16 bit patterns of a shim bf16 array (stored as float32)."""
    v = np.ascontiguousarray(a._v, dtype=np.float32)
    return (v.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a._v, dtype=np.float32)


def _np(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a))


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="checkout of Lumenbeing/convrot-mlx")
    parser.add_argument("--out", default=str(HERE))
    args = parser.parse_args()

    sys.path.insert(0, str(HERE))
    import _mlx_numpy_shim as shim

    shim.install()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import mlx.core as mx  # the shim

    import convrot_mlx as cr  # the reference, unchanged

    out = Path(args.out)
    cases: dict[str, dict[str, np.ndarray]] = {}
    manifest: dict[str, object] = {"generator": "tests/golden/make_golden.py", "cases": {}}

    def bf16_values(rng, shape):
        return mx.array(rng.normal(size=shape).astype(np.float32)).astype(mx.bfloat16)

    # test_core.py:54-96 -- prep exactness at 19x512 bf16, group 256
    for seed in (17, 18, 1801):
        rng = np.random.default_rng(seed)
        values = bf16_values(rng, (19, 512))
        qact, scales = cr.prepare_convrot_activation(values)
        cases[f"prep_g256_s{seed}"] = {
            "x_bf16": _bits(values),
            "qact": _np(qact),
            "codes": _np(cr.unpack_signed_int4(qact)),
            "scales": _f32(scales),
        }
    rng = np.random.default_rng(1802)
    values = bf16_values(rng, (19, 512))
    cases["rotate_g256_s1802"] = {"x_bf16": _bits(values), "rot_bf16": _bits(cr.regular_hadamard(values))}

    # test_core.py:98-126 -- group 64 at 17x2688
    rng = np.random.default_rng(2026082305)
    values = bf16_values(rng, (17, 2688))
    qact, scales = cr.prepare_convrot_activation(values, 64)
    cases["prep_g64_s2026082305"] = {
        "x_bf16": _bits(values),
        "qact": _np(qact),
        "codes": _np(cr.unpack_signed_int4(qact)),
        "scales": _f32(scales),
        "rot_bf16": _bits(cr.regular_hadamard(values, 64)),
    }

    # test_core.py:128-137 -- route shape 1536x3072 (input regenerated from the seed)
    rng = np.random.default_rng(20260823)
    values = bf16_values(rng, (1536, 3072))
    qact, scales = cr.prepare_convrot_activation(values)
    qact_np, scales_np = _np(qact), _f32(scales)
    cases["prep_route_s20260823"] = {"qact_head": qact_np[:8], "scales": scales_np}
    manifest["cases"]["prep_route_s20260823"] = {
        "seed": 20260823,
        "shape": [1536, 3072],
        "group_size": 256,
        "x_sha256": _sha(_bits(values)),
        "qact_sha256": _sha(qact_np),
        "codes_sha256": _sha(_np(cr.unpack_signed_int4(qact))),
        "scales_sha256": _sha(scales_np),
    }

    # test_core.py:139-175 -- integer oracle, bf16 output, 17x512 x 39x512
    rng = np.random.default_rng(29)
    qact = cr.pack_signed_int4(mx.array(rng.integers(-7, 8, size=(17, 512), dtype=np.int8)))
    qweight = cr.pack_signed_int4(mx.array(rng.integers(-7, 8, size=(39, 512), dtype=np.int8)))
    xs = mx.array(rng.uniform(0.01, 0.2, size=(17,)).astype(np.float32))
    ws = mx.array(rng.uniform(0.01, 0.2, size=(39,)).astype(np.float32))
    bias = mx.array(rng.normal(size=(39,)).astype(np.float32))
    expected = cr.reference_w4a4_matmul(qact, qweight, xs, ws, bias, output_dtype=mx.bfloat16)
    cases["tiles_s29"] = {
        "qact": _np(qact), "qweight_nk": _np(qweight), "xscales": _f32(xs),
        "wscales": _f32(ws), "bias": _f32(bias), "out_bf16": _bits(expected),
    }

    # test_core.py:177-184 -- rotation vs the explicit Kronecker matrix (fp32)
    rng = np.random.default_rng(17)
    values = rng.normal(size=(3, 512)).astype(np.float32)
    result = cr.regular_hadamard(mx.array(values))
    cases["kron_f32_s17"] = {"x": values, "rot": _f32(result)}

    # test_core.py:186-192 -- packing known-answer test
    kat = mx.array(np.array([[-8, -7, -1, 0, 1, 7, 3, -4]], dtype=np.int8))
    packed = cr.pack_signed_int4(kat)
    cases["pack_kat"] = {"values": _np(kat), "packed": _np(packed), "unpacked": _np(cr.unpack_signed_int4(packed))}

    # test_core.py:194-201 -- unpack 37x64 with -8
    rng = np.random.default_rng(2026082300)
    values = mx.array(rng.integers(-8, 8, size=(37, 64), dtype=np.int8))
    packed = cr.pack_signed_int4(values)
    cases["unpack_s2026082300"] = {"values": _np(values), "packed": _np(packed), "unpacked": _np(cr.unpack_signed_int4(packed))}

    # test_core.py:203-211 -- NK(46x64) -> KN(64x23) -> NK
    rng = np.random.default_rng(2026082301)
    values = mx.array(rng.integers(-7, 8, size=(46, 64), dtype=np.int8))
    packed_nk = cr.pack_signed_int4(values)
    packed_kn = cr.repack_nk_weight_for_mpp(packed_nk)
    cases["repack_s2026082301"] = {
        "values": _np(values), "packed_nk": _np(packed_nk), "packed_kn": _np(packed_kn),
        "round_trip": _np(cr.repack_mpp_weight_to_nk(packed_kn)),
    }

    # test_core.py:213-283 -- W4A4 at edges 37x64 x 46x64
    rng = np.random.default_rng(2026082302)
    acts = mx.array(rng.integers(-7, 8, size=(37, 64), dtype=np.int8))
    wts = mx.array(rng.integers(-7, 8, size=(46, 64), dtype=np.int8))
    qact = cr.pack_signed_int4(acts)
    qweight_nk = cr.pack_signed_int4(wts)
    qweight_kn = cr.repack_nk_weight_for_mpp(qweight_nk)
    xs = mx.array(rng.uniform(0.01, 0.2, size=(37,)).astype(np.float32))
    ws = mx.array(rng.uniform(0.01, 0.2, size=(46,)).astype(np.float32))
    bias = mx.array(rng.normal(size=(46,)).astype(np.float32))
    ones_x = mx.ones((37,), dtype=mx.float32)
    ones_w = mx.ones((46,), dtype=mx.float32)
    zero_b = mx.zeros((46,), dtype=mx.float32)
    cases["edges_s2026082302"] = {
        "qact": _np(qact), "qweight_nk": _np(qweight_nk), "qweight_kn": _np(qweight_kn),
        "xscales": _f32(xs), "wscales": _f32(ws), "bias": _f32(bias),
        "out_f32": _f32(cr.reference_w4a4_matmul(qact, qweight_nk, xs, ws, bias, output_dtype=mx.float32)),
        "out_int": _f32(cr.reference_w4a4_matmul(qact, qweight_nk, ones_x, ones_w, zero_b, output_dtype=mx.float32)),
        "out_bf16": _bits(cr.reference_w4a4_matmul(qact, qweight_nk, xs, ws, bias, output_dtype=mx.bfloat16)),
    }

    # test_core.py:285-309 -- W4A16 float16 / bfloat16 at 37x64 x 46x64
    rng = np.random.default_rng(2026082303)
    wts = mx.array(rng.integers(-7, 8, size=(46, 64), dtype=np.int8))
    qweight_kn = cr.repack_nk_weight_for_mpp(cr.pack_signed_int4(wts))
    ws = mx.array(rng.uniform(0.01, 0.2, size=(46,)).astype(np.float32))
    bias = mx.array(rng.normal(size=(46,)).astype(np.float32))
    case = {"qweight_kn": _np(qweight_kn), "wscales": _f32(ws), "bias": _f32(bias)}
    for name, dt in (("f16", mx.float16), ("bf16", mx.bfloat16)):
        acts = mx.array(rng.normal(size=(37, 64)).astype(np.float32)).astype(dt)
        expected = (acts.astype(mx.float32) @ wts.astype(mx.float32).T) * ws[None, :] + bias[None, :]
        case[f"act_{name}_as_f32"] = _f32(acts)
        case[f"out_{name}_f32"] = _f32(expected)
    cases["w4a16_s2026082303"] = case

    # test_core.py:311-327 and :357-373 -- float16 rowwise quantization + oracle
    for seed, k in ((23, 256), (28, 1024)):
        rng = np.random.default_rng(seed)
        acts = mx.array(rng.normal(size=(19, k)).astype(np.float16))
        wts = mx.array(rng.normal(size=(37, k)).astype(np.float16))
        qact, xs = cr.quantize_signed_int4_rowwise(acts)
        qweight, ws = cr.quantize_signed_int4_rowwise(wts)
        bias = mx.array(rng.normal(size=(37,)).astype(np.float32))
        cases[f"quant_f16_s{seed}"] = {
            "act_f16": np.asarray(acts).astype(np.float16), "w_f16": np.asarray(wts).astype(np.float16),
            "qact": _np(qact), "xscales": _f32(xs), "qweight": _np(qweight), "wscales": _f32(ws),
            "bias": _f32(bias),
            "out_f32": _f32(cr.reference_w4a4_matmul(qact, qweight, xs, ws, bias, output_dtype=mx.float32)),
        }

    # test_core.py:329-355 -- 31x1024 x 61x1024, bf16 output
    rng = np.random.default_rng(27)
    acts = mx.array(rng.integers(-7, 8, size=(31, 1024), dtype=np.int8))
    wts = mx.array(rng.integers(-7, 8, size=(61, 1024), dtype=np.int8))
    qact, qweight = cr.pack_signed_int4(acts), cr.pack_signed_int4(wts)
    xs = mx.array(rng.uniform(0.01, 0.2, size=(31,)).astype(np.float32))
    ws = mx.array(rng.uniform(0.01, 0.2, size=(61,)).astype(np.float32))
    bias = mx.array(rng.normal(size=(61,)).astype(np.float32))
    cases["expanded_s27"] = {
        "qact": _np(qact), "qweight_nk": _np(qweight), "xscales": _f32(xs), "wscales": _f32(ws),
        "bias": _f32(bias),
        "out_bf16": _bits(cr.reference_w4a4_matmul(qact, qweight, xs, ws, bias, output_dtype=mx.bfloat16)),
    }

    # test_core.py:375-402 -- the layer contract, NK layout, bf16, (2,7,256) -> 33
    rng = np.random.default_rng(29)
    dense_w = mx.array(rng.normal(size=(33, 256)).astype(np.float32)).astype(mx.bfloat16)
    dense_b = mx.array(rng.normal(size=(33,)).astype(np.float32))
    qweight, ws = cr.quantize_convrot_weight(dense_w)
    values = mx.array(rng.normal(size=(2, 7, 256)).astype(np.float32)).astype(mx.bfloat16)
    rotated = cr.regular_hadamard(values.reshape(-1, 256))
    qact, xs = cr.quantize_signed_int4_rowwise(rotated)
    expected = cr.reference_w4a4_matmul(qact, qweight, xs, ws, dense_b, output_dtype=mx.bfloat16).reshape(2, 7, 33)
    cases["layer_nk_s29"] = {
        "w_bf16": _bits(dense_w), "bias": _f32(dense_b), "qweight_nk": _np(qweight), "wscales": _f32(ws),
        "x_bf16": _bits(values), "out_bf16": _bits(expected),
    }

    # test_core.py:404-448 -- MPP (KN) layers, both activation modes, g256 and g64
    for seed, k, g in ((2026082304, 256, 256), (2026082306, 2688, 64)):
        rng = np.random.default_rng(seed)
        dense_w = mx.array(rng.normal(size=(34, k)).astype(np.float32)).astype(mx.bfloat16)
        dense_b = mx.array(rng.normal(size=(34,)).astype(np.float32))
        qweight_nk, ws = cr.quantize_convrot_weight(dense_w, g)
        qweight_kn = cr.repack_nk_weight_for_mpp(qweight_nk)
        values = mx.array(rng.normal(size=(2, 7, k)).astype(np.float32)).astype(mx.bfloat16)
        x2 = values.reshape(-1, k)
        qact, xs = cr.prepare_convrot_activation(x2, g)
        w4a4 = cr.reference_w4a4_matmul(qact, qweight_nk, xs, ws, dense_b, output_dtype=mx.bfloat16)
        rot = cr.regular_hadamard(x2, g)
        w_f32 = cr.unpack_signed_int4(qweight_nk).astype(mx.float32)
        w4a16 = ((rot.astype(mx.float32) @ w_f32.T) * ws[None, :] + dense_b[None, :]).astype(mx.bfloat16)
        cases[f"layer_kn_g{g}_s{seed}"] = {
            "w_bf16": _bits(dense_w), "bias": _f32(dense_b), "qweight_nk": _np(qweight_nk),
            "qweight_kn": _np(qweight_kn), "wscales": _f32(ws), "x_bf16": _bits(values),
            "w4a4_bf16": _bits(w4a4).reshape(2, 7, 34), "w4a16_bf16": _bits(w4a16).reshape(2, 7, 34),
            "rot_bf16": _bits(rot),
        }

    # ConvRotLinear K=N=1024, M=64, no bias, group 256
    rng = np.random.default_rng(20260823)
    x = mx.array(rng.normal(size=(64, 1024)).astype(np.float32)).astype(mx.bfloat16)
    w = mx.array(rng.normal(size=(1024, 1024)).astype(np.float32)).astype(mx.bfloat16)
    qweight_nk, ws = cr.quantize_convrot_weight(w)
    zero_b = mx.zeros((1024,), dtype=mx.float32)
    qact, xs = cr.prepare_convrot_activation(x)
    y = cr.reference_w4a4_matmul(qact, qweight_nk, xs, ws, zero_b, output_dtype=mx.bfloat16)
    manifest["cases"]["config1_s20260823"] = {"w_sha256": _sha(_bits(w)), "seed": 20260823}
    cases["config1_s20260823"] = {
        "x_bf16": _bits(x), "qweight_nk": _np(qweight_nk),
        "wscales": _f32(ws), "qact": _np(qact), "xscales": _f32(xs), "out_bf16": _bits(y),
    }

    for name, arrays in cases.items():
        np.savez_compressed(out / f"{name}.npz", **arrays)
        entry = manifest["cases"].setdefault(name, {})
        entry["arrays"] = {k: {"shape": list(v.shape), "dtype": str(v.dtype), "sha256": _sha(v)} for k, v in arrays.items()}
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(cases)} fixtures to {out}")


if __name__ == "__main__":
    main()
