"""Command-line driver over xt-dialect text, in the manner of the reference's
``xt-opt`` (``xt-opt/xt-opt.cpp``, exercised by the ``RUN:`` lines of
``test/xt/*.mlir``).

    python -m xtile_b200.xt_opt [STAGE FLAGS] [--split-input-file] [--plan] FILE|-

It reads the text, parses and verifies it (the reference's diagnostics), runs
the requested stages in the order given and prints the module.  Stage flags:
``--xt-serialize`` (grid unrolling, as the reference), ``--xt-to-nova``,
``--nova-optimize``, ``--nova-threading``, ``--nova-barrier``,
``--nova-allocate`` and ``--nova-to-x1`` (on this backend they annotate the
B200 kernel plan), and ``--canonicalize`` (the xt dialect's folds of
``x + 0`` and ``x - 0``, ``lib/xt/XTOps.cpp:395-449``, then dead-op erasure).
``--split-input-file`` treats each ``// -----`` separated part as its own
module, as mlir-opt does; ``--plan`` appends each function's kernel plan as a
comment.  Diagnostics go to stderr as ``FILE:LINE: error:``; the exit status
is 1 if any part failed.

Values are printed with MLIR's own numbering, as the reference's xt-opt
prints them: function arguments ``%arg0, %arg1, ...``, op results ``%0,
%1, ...`` in order, and the three results of ``xt.get_tile_block_id`` as
three separate values.  ``--keep-names`` prints the source's names instead.
"""
from __future__ import annotations

import argparse
import json
import re
import sys

from . import api

_STAGE_FLAGS = (
    ("--canonicalize", "canonicalize"),
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


_VALUE = re.compile(r"%([\w.$-]+)(?:#(\d+))?")
_DEF = re.compile(r"^(\s*)%([\w.$-]+)(?::(\d+))?\s*=\s*")


def mlir_ssa_names(text: str) -> str:
    """Renames every function's values the way MLIR's printer numbers them."""
    out, names, counter = [], {}, 0
    for line in text.splitlines():
        if line.lstrip().startswith("func.func"):
            names, counter = {}, 0
            header, sep, rest = line.partition("(")
            for k, arg in enumerate(re.findall(r"%([\w.$-]+)\s*:", rest)):
                names[arg] = f"arg{k}"
            out.append(header + sep + _VALUE.sub(lambda m: "%" + names.get(m.group(1), m.group(1)), rest))
            continue
        lhs = ""
        m = _DEF.match(line)
        if m:
            indent, name, count = m.group(1), m.group(2), m.group(3)
            if count:  # a result group: one separate value per result
                ids = []
                for i in range(int(count)):
                    names[(name, str(i))] = str(counter)
                    ids.append(f"%{counter}")
                    counter += 1
                lhs = indent + ", ".join(ids) + " = "
            else:
                names[name] = str(counter)
                lhs = f"{indent}%{counter} = "
                counter += 1
            line = line[m.end():]

        def use(v):
            key = (v.group(1), v.group(2)) if v.group(2) is not None else v.group(1)
            return "%" + names[key] if key in names else v.group(0)

        out.append(lhs + _VALUE.sub(use, line))
    return "\n".join(out)


def _parse_part(part: str) -> api.Module:
    """Parses one input the way mlir-opt reads a file: text whose first op
    (after comments) is a ``module`` is that module, kept with its line
    numbers; bare functions are wrapped in one, as ``xtile.parse`` does."""
    body = [ln.strip() for ln in part.splitlines() if ln.strip() and not ln.strip().startswith("//")]
    if body and body[0].startswith("module"):
        return api.Module(api._native.parse(part), source_asm=part)
    return api.parse(part)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="xt-opt", description="xt optimizer driver (B200 backend)")
    for flag, stage in _STAGE_FLAGS:
        ap.add_argument(flag, dest="stages", action="append_const", const=stage)
    ap.add_argument("--split-input-file", action="store_true")
    ap.add_argument("--plan", action="store_true", help="append each function's B200 kernel plan")
    ap.add_argument("--keep-names", action="store_true", help="print the source's value names, not MLIR's")
    ap.add_argument("input", help="xt text file, or - for stdin")
    args = ap.parse_args(argv)
    name = "<stdin>" if args.input == "-" else args.input
    text = sys.stdin.read() if args.input == "-" else open(args.input, encoding="utf-8").read()
    parts = _split(text) if args.split_input_file else [(0, text)]
    outs, status = [], 0
    for first_line, part in parts:
        try:
            module = _parse_part(part)
            for stage in args.stages or ():
                module = getattr(api, stage)(module)
            out = api._module_asm(module)
            if not args.keep_names:
                out = mlir_ssa_names(out)
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
