"""Command-line driver over xt-dialect text, in the manner of the reference's
``xt-opt`` (``xt-opt/xt-opt.cpp``, exercised by the ``RUN:`` lines of
``test/xt/*.mlir``).

    python -m xtile_b200.xt_opt [STAGE FLAGS] [--split-input-file] [--plan] FILE|-

It reads the text, parses and verifies it (the reference's diagnostics), runs
the requested stages in the order given and prints the module.  Stage flags:
``--xt-serialize`` (grid unrolling, as the reference), ``--xt-to-nova``,
``--nova-optimize``, ``--nova-threading``, ``--nova-barrier``,
``--nova-allocate`` and ``--nova-to-x1`` (on this backend they annotate the
B200 kernel plan).  ``--split-input-file`` treats each ``// -----`` separated
part as its own module, as mlir-opt does; ``--plan`` appends each function's
kernel plan as a comment.  Diagnostics go to stderr as ``FILE:LINE: error:``;
the exit status is 1 if any part failed.  ``--canonicalize`` is refused: this
backend has no rewrite patterns.
"""
from __future__ import annotations

import argparse
import json
import re
import sys

from . import api

_STAGE_FLAGS = (
    ("--xt-serialize", "xt_serialize"),
    ("--xt-to-nova", "xt_to_nova"),
    ("--nova-optimize", "nova_optimize"),
    ("--nova-threading", "nova_threading"),
    ("--nova-barrier", "nova_barrier"),
    ("--nova-allocate", "nova_allocate"),
    ("--nova-to-x1", "nova_to_x1"),
)
_SPLIT = re.compile(r"^// -----[ \t]*$", re.MULTILINE)
_LINE = re.compile(r"^line (\d+): (.*)$")


def _split(text: str) -> list[tuple[int, str]]:
    """Parts of ``text`` with the 0-based line each starts on."""
    parts, start = [], 0
    for m in _SPLIT.finditer(text):
        parts.append((text.count("\n", 0, start), text[start:m.start()]))
        start = m.end() + 1  # past the separator line's newline
    parts.append((text.count("\n", 0, start), text[start:]))
    return parts


def _report(name: str, first_line: int, err: Exception) -> None:
    lines = str(err).splitlines()
    body = lines[1:] if len(lines) > 1 else lines
    for ln in body:
        m = _LINE.match(ln)
        if m:
            print(f"{name}:{first_line + int(m.group(1))}: error: {m.group(2)}", file=sys.stderr)
        else:
            print(f"{name}:{first_line + 1}: error: {ln}", file=sys.stderr)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="xt-opt", description="xt optimizer driver (B200 backend)")
    for flag, stage in _STAGE_FLAGS:
        ap.add_argument(flag, dest="stages", action="append_const", const=stage)
    ap.add_argument("--split-input-file", action="store_true")
    ap.add_argument("--plan", action="store_true", help="append each function's B200 kernel plan")
    ap.add_argument("--canonicalize", action="store_true")
    ap.add_argument("input", help="xt text file, or - for stdin")
    args = ap.parse_args(argv)
    if args.canonicalize:
        print("xt-opt: --canonicalize is not available: this backend has no rewrite patterns", file=sys.stderr)
        return 2
    name = "<stdin>" if args.input == "-" else args.input
    text = sys.stdin.read() if args.input == "-" else open(args.input, encoding="utf-8").read()
    parts = _split(text) if args.split_input_file else [(0, text)]
    outs, status = [], 0
    for first_line, part in parts:
        try:
            module = api.parse(part)
            for stage in args.stages or ():
                module = getattr(api, stage)(module)
            out = api._module_asm(module)
            if args.plan:
                for f in module.func_names():
                    try:
                        out += f"\n// plan @{f}: {json.dumps(module.plan(f))}"
                    except RuntimeError as e:
                        out += f"\n// plan @{f}: unsupported: {e}"
            outs.append(out)
        except (ValueError, RuntimeError) as e:
            _report(name, first_line, e)
            status = 1
    if outs:
        print("\n// -----\n".join(outs))
    return status


if __name__ == "__main__":
    sys.exit(main())
