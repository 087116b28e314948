"""Load kvlang ``.kv`` source into a kvspace, in the slot layout kvfunc reads.

The reference relies on the external Go command ``kvlang load`` for this step
(deepx_op_gpukernelcompiler/workflow.py:5).  This loader covers the subset of
kvlang that the fusion fixtures use — one or more straight-line functions

    def name(arg, ...) -> (out, ...) {
        tensor.op(read, ...) -> write, ...
    }

with ``//`` comments — and writes the slots that ``kvfunc.read_func`` expects
(kvfunc.py:1-8):

    /func/<pkg>/<name>          = signature string
    /func/<pkg>/<name>/[i,0]    = opcode
    /func/<pkg>/<name>/[i,-j]   = j-th read operand (1-based)
    /func/<pkg>/<name>/[i,j]    = j-th write operand (1-based)
"""
from __future__ import annotations

import re
from pathlib import Path

_FUNC_RE = re.compile(r"def\s+(\w+)\s*\(([^)]*)\)\s*->\s*\(([^)]*)\)\s*\{(.*?)\}", re.S)
_OP_RE = re.compile(r"^([\w.]+)\s*\(([^)]*)\)\s*->\s*(.+)$")


class KvSyntaxError(ValueError):
    pass


def _split(names: str) -> list[str]:
    return [n.strip() for n in names.split(",") if n.strip()]


def parse_kv(source: str) -> list[dict]:
    """Parse kvlang source into ``[{"name", "signature", "ops": [...]}]``."""
    text = "\n".join(line.split("//", 1)[0] for line in source.splitlines())
    funcs = []
    for m in _FUNC_RE.finditer(text):
        name, args, outs, body = m.groups()
        ops = []
        for raw in body.splitlines():
            line = raw.strip().rstrip(";")
            if not line:
                continue
            om = _OP_RE.match(line)
            if om is None:
                raise KvSyntaxError(f"{name}: cannot parse instruction {line!r}")
            op, reads, writes = om.groups()
            ops.append({"op": op, "reads": _split(reads), "writes": _split(writes)})
        sig = f"def {name}({', '.join(_split(args))}) -> ({', '.join(_split(outs))})"
        funcs.append({"name": name, "signature": sig, "ops": ops})
    if not funcs and source.strip():
        raise KvSyntaxError("no function definition found")
    return funcs


def store_func(kv, pkg: str, func: dict) -> str:
    """Write one parsed function into `kv`; returns its path."""
    path = f"/func/{pkg}/{func['name']}"
    kv.set(path, func["signature"])
    for i, op in enumerate(func["ops"]):
        kv.set(f"{path}/[{i},0]", op["op"])
        for j, r in enumerate(op["reads"], start=1):
            kv.set(f"{path}/[{i},-{j}]", r)
        for j, w in enumerate(op["writes"], start=1):
            kv.set(f"{path}/[{i},{j}]", w)
    return path


def load_file(kv, path: str | Path, pkg: str | None = None) -> list[str]:
    """Load every function of one ``.kv`` file under ``/func/<pkg>/``."""
    p = Path(path)
    pkg = pkg or p.parent.name
    return [store_func(kv, pkg, f) for f in parse_kv(p.read_text(encoding="utf-8"))]


def load_dir(kv, directory: str | Path, pkg: str | None = None) -> list[str]:
    """Load every ``*.kv`` file in `directory` (package name = directory name)."""
    d = Path(directory)
    paths = []
    for f in sorted(d.glob("*.kv")):
        paths += load_file(kv, f, pkg or d.name)
    return paths
