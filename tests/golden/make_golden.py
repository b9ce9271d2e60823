"""Generate the golden vectors that pin the CPU oracle to the reference.

Run once, in a checkout that has the reference sources (``--reference``
points at the root of xuOAO/practice_cuda).  Every expected value below is
produced by a function of the reference itself, evaluated eagerly on the CPU:

* per-channel quant: ``fp8_per_channel_quant_torch_compile``'s eager body
  (``fp8_training/fp8_bench/kernels/quant/per_channel.py:9-29``);
* per-block quant: the reference has no torch per-block quantizer, but its
  per-block kernel (``kernels/quant/per_block.py:40-48``) applies, to every
  tile, exactly the per-tensor formula of the legacy test reference
  ``fp8_quant_ref`` (``kernels/fp8_bmm/test/fp8_quant_test.py:28-42``:
  ``q = max / amax``, ``deq = q.reciprocal()``) -- so each tile's bytes and
  scale are produced by calling ``fp8_quant_ref`` on that tile (fp32);
* per-tensor quant: ``fp8_quant_ref`` (E4M3 and E5M2);
* dynamic float8 casts of the FP8 training linear: ``hp_tensor_to_float8_dynamic``
  (``fp8_training/fp8_bench/modules/float8/float8_scaling_utils.py:29-72``),
  tensorwise and axiswise (``axiswise_dim=-1``), E4M3 and E5M2;
* scaled BMM: the registry's ``QuantResult.dequantize`` followed by an fp32
  ``torch.bmm`` (``bench_bmm.py:414-419``), and the legacy ``fp8_quant_bmm_ref``
  (``kernels/fp8_bmm/test/fp8_quant_bmm_test.py:100-114``).

The product never reads these files; ``tests/test_oracle_golden.py`` checks the
oracle against them and the GPU tests check the CUDA path against the oracle.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_module(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def synthetic(shape, *, std=1.0, outliers=False, seed=0, dtype=torch.bfloat16):
    """Seeded synthetic input: N(0, std), optionally numel//1000 entries x100."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g, dtype=torch.float32) * std
    if outliers:
        flat = x.view(-1)
        idx = torch.randperm(flat.numel(), generator=g)[: max(1, flat.numel() // 1000)]
        flat[idx] *= 100.0
    return x.to(dtype)


def u8(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8).clone()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.pt"))
    args = ap.parse_args()

    ref = os.path.abspath(args.reference)
    sys.path.insert(0, os.path.join(ref, "fp8_training"))
    sys.path.insert(0, os.path.join(ref, "kernels", "fp8_bmm"))
    from fp8_bench.kernels.quant.per_channel import fp8_per_channel_quant_torch_compile
    from fp8_bench.registry import QuantResult

    per_channel_eager = fp8_per_channel_quant_torch_compile._torchdynamo_orig_callable
    qtest = _load_module(os.path.join(ref, "kernels", "fp8_bmm", "test", "fp8_quant_test.py"), "ref_fp8_quant_test")
    btest = _load_module(os.path.join(ref, "kernels", "fp8_bmm", "test", "fp8_quant_bmm_test.py"), "ref_fp8_quant_bmm_test")
    fp8_quant_ref = qtest.fp8_quant_ref
    fp8_quant_bmm_ref = btest.fp8_quant_bmm_ref

    e4m3 = torch.float8_e4m3fn
    cases: dict[str, dict] = {}

    # ---- per-channel -------------------------------------------------------
    pc_inputs = {
        "pc_bf16_2d": synthetic((96, 384), outliers=True, seed=1),
        "pc_f32_3d": synthetic((2, 40, 264), seed=2, dtype=torch.float32),
        "pc_bf16_ragged": synthetic((3, 17, 33), std=0.02, seed=3),
    }
    zero_rows = synthetic((8, 128), seed=4)
    zero_rows[2].zero_()
    zero_rows[:, 5] = 0
    pc_inputs["pc_bf16_zero_rows"] = zero_rows
    for name, x in pc_inputs.items():
        for axis in (-2, -1):
            y, s = per_channel_eager(x, axis, e4m3, 1e-12)
            cases[f"{name}_axis{axis}"] = {
                "kind": "per_channel", "x": x, "channel_axis": axis,
                "y_u8": u8(y), "scale": s.clone(),
            }

    # ---- per-block ---------------------------------------------------------
    def per_block_by_tiles(x, bm, bn):
        xb = x.unsqueeze(0) if x.ndim == 2 else x
        b, m, n = xb.shape
        mb, nb = -(-m // bm), -(-n // bn)
        y = torch.empty((b, m, n), dtype=e4m3)
        s = torch.empty((b, mb, nb), dtype=torch.float32)
        for bi in range(b):
            for i in range(mb):
                for j in range(nb):
                    tile = xb[bi, i * bm:(i + 1) * bm, j * bn:(j + 1) * bn].float()
                    q, d = fp8_quant_ref(tile)
                    y[bi, i * bm:(i + 1) * bm, j * bn:(j + 1) * bn] = q
                    s[bi, i, j] = d
        if x.ndim == 2:
            return y[0], s[0]
        return y, s

    pb_inputs = [
        ("pb_act_1x128", synthetic((48, 512), outliers=True, seed=5), 1, 128),
        ("pb_act_1x128_3d", synthetic((2, 24, 384), seed=6), 1, 128),
        ("pb_act_1x128_ragged", synthetic((3, 7, 200), seed=7), 1, 128),
        ("pb_w_128x128", synthetic((256, 384), std=0.02, seed=8), 128, 128),
        ("pb_w_128x128_ragged", synthetic((200, 136), std=0.02, seed=9), 128, 128),
        ("pb_b_128x1", synthetic((1, 256, 48), std=0.02, seed=10), 128, 1),
        ("pb_f32_64x32", synthetic((96, 80), seed=11, dtype=torch.float32), 64, 32),
    ]
    for name, x, bm, bn in pb_inputs:
        y, s = per_block_by_tiles(x, bm, bn)
        cases[name] = {"kind": "per_block", "x": x, "block_m": bm, "block_n": bn,
                       "y_u8": u8(y), "scale": s.clone()}

    # ---- per-tensor (legacy test reference, fp32 inputs as in its tests) ----
    for name, x, dt, rng in [
        ("pt_e4m3", synthetic((64, 96), seed=12, dtype=torch.float32), e4m3, 448.0),
        ("pt_e4m3_3d", synthetic((3, 17, 33), seed=13, dtype=torch.float32), e4m3, 448.0),
        ("pt_e5m2", synthetic((64, 128), seed=14, dtype=torch.float32), torch.float8_e5m2, 57344.0),
    ]:
        y, r = fp8_quant_ref(x, quant_dtype=dt, fp8_range=rng)
        cases[name] = {"kind": "per_tensor", "x": x, "fp8_dtype": str(dt), "fp8_range": rng,
                       "y_u8": u8(y), "scale": r.clone()}

    # ---- dynamic float8 casts (FP8 training linear) ---------------------------
    from fp8_bench.modules.float8.config import ScalingGranularity
    from fp8_bench.modules.float8.float8_scaling_utils import hp_tensor_to_float8_dynamic
    from fp8_bench.modules.float8.float8_training_tensor import LinearMMConfig

    zero_row = synthetic((2, 6, 96), seed=27)
    zero_row[1, 3].zero_()
    for name, x in [
        ("f8dyn_bf16", synthetic((2, 40, 264), outliers=True, seed=28)),
        ("f8dyn_f32", synthetic((3, 17, 48), std=0.02, seed=29, dtype=torch.float32)),
        ("f8dyn_bf16_zero_row", zero_row),
    ]:
        for dt in (e4m3, torch.float8_e5m2):
            for axis in (False, True):
                kw = ({"scaling_granularity": ScalingGranularity.AXISWISE, "axiswise_dim": -1} if axis else {})
                t = hp_tensor_to_float8_dynamic(x, dt, LinearMMConfig(), **kw)
                cases[f"{name}_{str(dt).split('_')[-1]}_{'axis' if axis else 'tensor'}"] = {
                    "kind": "float8_dynamic", "x": x, "fp8_dtype": str(dt), "axiswise": axis,
                    "y_u8": u8(t._data), "scale": t._scale.clone()}

    # ---- scaled BMM: registry dequantize + fp32 bmm --------------------------
    def bmm_case(name, a_x, b_x, a_kind, b_kind, bias=None):
        qa = _quantize_with_ref(a_kind, a_x, per_channel_eager, per_block_by_tiles, fp8_quant_ref, QuantResult)
        qb = _quantize_with_ref(b_kind, b_x, per_channel_eager, per_block_by_tiles, fp8_quant_ref, QuantResult)
        out = torch.bmm(qa.dequantize(), qb.dequantize())
        if bias is not None:
            out += bias.float()
        cases[name] = {
            "kind": "bmm", "a_kind": a_kind, "b_kind": b_kind,
            "a_u8": u8(qa.tensor), "a_scale": qa.dequant_scale.clone(),
            "b_u8": u8(qb.tensor), "b_scale": qb.dequant_scale.clone(),
            "bias": bias, "out_f32": out.clone(),
        }

    bmm_case("bmm_block_1x128_128x128", synthetic((2, 64, 256), outliers=True, seed=15),
             synthetic((2, 256, 192), std=0.02, seed=16), ("block", 1, 128), ("block", 128, 128))
    bmm_case("bmm_block_1d", synthetic((1, 48, 384), seed=17),
             synthetic((1, 384, 40), std=0.02, seed=18), ("block", 1, 128), ("block", 128, 1))
    bmm_case("bmm_block_2d", synthetic((1, 200, 256), seed=19),
             synthetic((1, 256, 136), std=0.02, seed=20), ("block", 128, 128), ("block", 128, 128),
             bias=synthetic((1, 200, 136), seed=21))
    bmm_case("bmm_channel", synthetic((1, 80, 192), seed=22),
             synthetic((1, 192, 96), std=0.02, seed=23), ("channel", -2), ("channel", -1))
    bmm_case("bmm_tensor", synthetic((2, 33, 65), seed=24, dtype=torch.float32),
             synthetic((2, 65, 47), std=0.02, seed=25, dtype=torch.float32), ("tensor",), ("tensor",))

    # ---- legacy scalar-scale BMM -------------------------------------------
    g = torch.Generator().manual_seed(26)
    a = (torch.randn((3, 33, 47), generator=g) * 0.5).to(e4m3)
    b = (torch.randn((3, 47, 65), generator=g) * 0.5).to(e4m3)
    bias = torch.randn((3, 33, 65), generator=g)
    cases["legacy_bmm"] = {
        "kind": "legacy_bmm", "a_u8": u8(a), "b_u8": u8(b), "bias": bias, "scale": 1.5,
        "out_f32": fp8_quant_bmm_ref(a, b, 1.5, bias=bias, out_dtype=torch.float32),
    }

    torch.save(cases, args.out)
    print(f"wrote {len(cases)} cases to {args.out}")


def _quantize_with_ref(kind, x, per_channel_eager, per_block_by_tiles, fp8_quant_ref, QuantResult):
    e4m3 = torch.float8_e4m3fn
    if kind[0] == "block":
        _, bm, bn = kind
        y, s = per_block_by_tiles(x, bm, bn)
        return QuantResult(y, s, "ref", "block", {"block_m": bm, "block_n": bn})
    if kind[0] == "channel":
        y, s = per_channel_eager(x, kind[1], e4m3, 1e-12)
        return QuantResult(y, s, "ref", "channel", {"channel_axis": kind[1]})
    y, r = fp8_quant_ref(x.float())
    return QuantResult(y, r, "ref", "tensor", {})


if __name__ == "__main__":
    main()
