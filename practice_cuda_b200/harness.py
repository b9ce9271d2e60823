"""Run the reference's own benchmark harnesses with this library installed.

    python -m practice_cuda_b200.harness [--reference PATH] [--bmm-case NAME:B,M,N,K]
                                          [--quant-case NAME:D0,D1[,D2]] HARNESS [harness args...]

``HARNESS`` is one of the reference's entry modules -- ``bench_quant``,
``bench_bmm``, ``profile_one`` (``fp8_training/fp8_bench/{bench_quant.py:36-134,
bench_bmm.py:59-434, profile_one.py:52-129}``).  Before its ``main()`` runs,
:func:`practice_cuda_b200.registry.install_into` registers every ``b200_*``
quant / BMM impl in the reference's registry, so ``--impl b200_...`` selects
these kernels next to the reference's ``triton_*`` impls, in the same table
and the same JSONL schema (``utils.py:153-158``).  ``--bmm-case`` /
``--quant-case`` add shapes to a suite named ``b200_extra`` (e.g. the
32 x 4096 x 2048 x 7168 per-block BMM), selected with ``--suite b200_extra``.

``--reference`` is the directory that holds the reference's ``fp8_bench``
package (default: ``$PCB200_REFERENCE``, then ``baseline/_ref`` next to this
repository).
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys

HARNESSES = ("bench_quant", "bench_bmm", "profile_one")


def _default_reference() -> str:
    env = os.environ.get("PCB200_REFERENCE")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--reference", default=_default_reference())
    ap.add_argument("--bmm-case", action="append", default=[], help="NAME:B,M,N,K added to suite b200_extra")
    ap.add_argument("--quant-case", action="append", default=[], help="NAME:D0,D1[,D2] added to suite b200_extra")
    ap.add_argument("harness", choices=HARNESSES)
    ap.add_argument("rest", nargs=argparse.REMAINDER)
    args = ap.parse_args(argv)
    if not os.path.isdir(os.path.join(args.reference, "fp8_bench")):
        raise SystemExit(f"no fp8_bench package under {args.reference}")
    sys.path.insert(0, args.reference)

    ref_registry = importlib.import_module("fp8_bench.registry")
    from .registry import install_into

    install_into(ref_registry)
    cases = importlib.import_module("fp8_bench.cases")
    if args.bmm_case:
        extra = cases.BMM_SUITES.setdefault("b200_extra", [])
        for spec in args.bmm_case:
            name, dims = spec.split(":")
            b, m, n, k = (int(v) for v in dims.split(","))
            extra.append(cases.BMMCase(name, b, m, n, k))
    if args.quant_case:
        extra = cases.QUANT_SUITES.setdefault("b200_extra", [])
        for spec in args.quant_case:
            name, dims = spec.split(":")
            extra.append(cases.QuantCase(name, tuple(int(v) for v in dims.split(","))))
    module = importlib.import_module(f"fp8_bench.{args.harness}")
    sys.argv = [f"fp8_bench.{args.harness}"] + [a for a in args.rest if a != "--"]
    module.main()


if __name__ == "__main__":
    main()
