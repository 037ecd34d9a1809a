"""Regenerate the xt-text golden fixtures from the reference tracer.

Runs the reference's pure-Python tracer (``xtile/dsl.py`` of sjjeong94/xtile)
in place -- it needs no native module when ``parse_module`` is the identity
(reference ``xtile/dsl.py:1001-1029``) -- over the programs of ``cases.py`` and
writes one ``dsl_text/<name>.mlir`` per program.  Only needed where a checkout
of the reference exists; the fixtures it writes are committed.

    python tests/golden/make_golden.py --reference <path to xtile checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def load_reference_dsl(root: Path):
    path = root / "xtile" / "dsl.py"
    spec = importlib.util.spec_from_file_location("xtile_reference_dsl", path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = module
    spec.loader.exec_module(module)
    return module


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, type=Path)
    args = parser.parse_args()
    ref = load_reference_dsl(args.reference)
    sys.path.insert(0, str(HERE))
    from cases import build_cases

    out_dir = HERE / "dsl_text"
    out_dir.mkdir(exist_ok=True)
    for name, fn, kargs, grid, db in build_cases(ref):
        text = ref.convert(fn, args=kargs, grid=grid, double_buffering=db,
                           parse_module=lambda s: s)
        (out_dir / f"{name}.mlir").write_text(text + "\n")
        print("wrote", name)


if __name__ == "__main__":
    main()
