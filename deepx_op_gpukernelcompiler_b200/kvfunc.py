"""kvfunc: read kvlang functions out of kvspace.

Same API and slot walk as the reference (deepx_op_gpukernelcompiler/
kvfunc.py:13-60): a function lives at

    /func/<pkg>/<name>          = signature string
    /func/<pkg>/<name>/[i,0]    = opcode of instruction i
    /func/<pkg>/<name>/[i,-j]   = j-th read operand
    /func/<pkg>/<name>/[i,j]    = j-th write operand

and reading stops at the first instruction index without an opcode.  `kv` is
any object with the kvspace client surface (``get``/``list``); the local
stand-in is ``kvspace_local.KVSpace``.
"""
from __future__ import annotations

from .kvspace_local import not_found_errors

_NOT_FOUND = not_found_errors()


def _get_str(kv, key: str) -> str | None:
    """String value at `key`, or None if absent or not a string (kvfunc.py:55-60)."""
    try:
        v = kv.get(key)
    except _NOT_FOUND:
        return None
    return v.as_str() if v.kind == "string" else None


def _operands(kv, path: str, i: int, sign: str) -> list[str]:
    out = []
    j = 1
    while (val := _get_str(kv, f"{path}/[{i},{sign}{j}]")) is not None:
        out.append(val)
        j += 1
    return out


def read_func(kv, path: str) -> dict:
    """Read one function: ``{"signature": str, "ops": [{"op", "reads", "writes"}]}``.

    Mirrors kvfunc.py:13-34; a missing signature raises the store's
    not-found error, as the reference's ``kv.get(path)`` does.
    """
    signature = kv.get(path).as_str()
    ops = []
    i = 0
    while (opcode := _get_str(kv, f"{path}/[{i},0]")) is not None:
        ops.append({"op": opcode,
                    "reads": _operands(kv, path, i, "-"),
                    "writes": _operands(kv, path, i, "")})
        i += 1
    return {"signature": signature, "ops": ops}


def list_funcs(kv, prefix: str = "/func/fusion_cases") -> list:
    """Sorted names of the functions stored under `prefix` (kvfunc.py:37-52).

    Instruction slots (children starting with ``[``) and non-string children
    are skipped; a prefix with nothing under it yields ``[]``.
    """
    try:
        children = kv.list(prefix)
    except _NOT_FOUND:
        return []
    names = []
    for child in children:
        if child.startswith("["):
            continue
        try:
            if kv.get(f"{prefix}/{child}").kind == "string":
                names.append(child)
        except _NOT_FOUND:
            continue
    return sorted(names)
