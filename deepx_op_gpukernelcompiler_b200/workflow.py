"""op-gpu workflow CLI: kvlang code -> kvspace -> read /func/ -> classify -> run.

Mirrors the reference CLI (deepx_op_gpukernelcompiler/workflow.py:1-111):

  python -m deepx_op_gpukernelcompiler_b200.workflow [--fusion b200] <path> | --all

plus ``--load DIR`` to load ``.kv`` files into the in-process kvspace first
(the reference leaves that step to the external ``kvlang load``), and
``--prefix`` for ``--all`` (default ``/func/fusion_cases``).  Exit status 1
on a non-compilable pattern or an engine error, as in the reference.
"""
from __future__ import annotations

import sys

from . import kvload
from .fusion import classify
from .kernel import ENGINES, compile_and_test
from .kvfunc import list_funcs, read_func
from .kvspace_local import connect, local_space

STATUS_ICON = {
    "compilable": "✅",
    "needs_template": "🟡",
    "multi_kernel": "🔷",
    "not_fusable": "⚪",
    "not_matched": "⚪",
}

USAGE = ("usage: python -m deepx_op_gpukernelcompiler_b200.workflow "
         "[--fusion b200] [--load DIR] [--prefix P] <path> | --all")


def _pop_opt(args: list, name: str, default=None):
    if name in args:
        i = args.index(name)
        if i + 1 >= len(args):
            print(f"{name} needs a value")
            sys.exit(1)
        val = args[i + 1]
        del args[i:i + 2]
        return val
    return default


def main(argv: list | None = None) -> None:
    args = list(sys.argv[1:] if argv is None else argv)
    fusion = _pop_opt(args, "--fusion", "b200")
    load_dir = _pop_opt(args, "--load")
    prefix = _pop_opt(args, "--prefix", "/func/fusion_cases")
    if fusion not in ENGINES:
        print(f"unknown fusion engine: {fusion}")
        sys.exit(1)
    if load_dir is not None:
        kv = local_space()
        kvload.load_dir(kv, load_dir, pkg=prefix.rstrip("/").rsplit("/", 1)[-1])
    else:
        kv = connect()
    if args and args[0] == "--all":
        _run_all(kv, fusion, prefix)
    elif args:
        _run_one(kv, args[0], fusion)
    else:
        print(USAGE)
        sys.exit(1)


def _run_one(kv, path: str, fusion: str) -> None:
    func = read_func(kv, path)
    print(f"read {path}")
    for o in func["ops"]:
        print(f"  {o['op']}({','.join(o.get('reads', []))}) → {','.join(o.get('writes', []))}")
    pattern, _template, activation, status = classify(func["ops"])
    print(f"\nfuse: {pattern or '—'}  status: {status}  engine: {fusion}"
          f"  activation: {activation or 'none'}")
    if status != "compilable":
        print(f"  {STATUS_ICON.get(status, '⚪')} {status}")
        sys.exit(1)
    result = compile_and_test(kv, path, fusion=fusion)
    if result.error:
        print(f"❌ {result.error}")
        sys.exit(1)
    print(f"  max diff: {result.diff:.6f}  {'✅' if result.success else '❌'}")
    print(f"  {fusion}: {result.tl_ms:.4f} ms")
    print(f"  PyTorch: {result.pt_ms:.4f} ms")
    print(f"  speedup: {result.pt_ms / result.tl_ms:.2f}×")


def _run_all(kv, fusion: str, prefix: str = "/func/fusion_cases") -> None:
    funcs = list_funcs(kv, prefix)
    if not funcs:
        print(f"no functions found in {prefix}/")
        sys.exit(1)
    print(f"engine: {fusion}")
    print(f"{'func':<28} {'pattern':<20} {'status':<16} {'diff':>9} "
          f"{fusion:>9} {'PyTorch':>9} {'sp':>6}")
    print("-" * 102)
    counts: dict[str, int] = {}
    for name in funcs:
        path = f"{prefix}/{name}"
        func = read_func(kv, path)
        pattern, _, _, status = classify(func["ops"])
        counts[status] = counts.get(status, 0) + 1
        if status == "compilable":
            r = compile_and_test(kv, path, fusion=fusion)
            sp = r.pt_ms / r.tl_ms if r.tl_ms > 0 else 0
            print(f"{name:<28} {pattern:<20} {status:<16} {r.diff:>9.6f} "
                  f"{r.tl_ms:>8.4f}ms {r.pt_ms:>8.4f}ms {sp:>5.2f}×")
        else:
            ops = "→".join(o["op"].replace("tensor.", "") for o in func["ops"] if o["op"] != "return")
            print(f"{name:<28} {pattern or '—':<20} {STATUS_ICON.get(status, '⚪')} "
                  f"{status:<14} {'—':>9}  ({ops})")
    print("\n─ summary ─")
    for s in ["compilable", "needs_template", "multi_kernel", "not_fusable", "not_matched"]:
        if counts.get(s):
            print(f"  {STATUS_ICON.get(s, '⚪')} {s}: {counts[s]}")


if __name__ == "__main__":
    main()
