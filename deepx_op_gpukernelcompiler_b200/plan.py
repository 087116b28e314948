"""Compiled plans: the compile-request -> plan -> call flow of the reference docs.

The reference design (doc/kvlang-to-tilelang-interface.md:100-129,194-218)
compiles a fused function once per (pattern, shapes, dtype) from a JSON
request and calls the result with raw pointers,
``kernel_fn(x_ptr, W_ptr, b_ptr, out_ptr, cuda_stream)``.  The reference
never built it.  Here a request such as

    {"func": "__fusion_0", "pattern": "linear_relu", "ops": ["matmul", "add", "relu"],
     "inputs":  [{"shape": [512, 256], "dtype": "float16"},
                 {"shape": [256, 512], "dtype": "float16"},
                 {"shape": [512],      "dtype": "float16"}],
     "outputs": [{"shape": [512, 512], "dtype": "float16"}],
     "accum_dtype": "float32"}

is checked against the pattern table (``fusion.FUSION_DB``) and compiled into
a native plan (``dx_plan_create``), cached by its key.  A ``PlanCache`` given
a kvspace store also records each compiled version there, keyed by a hash of
its shape, as the docs' lazy-compile lifecycle describes
(doc/kvlang-to-tilelang-interface.md:194-218): the record at
``/func/<func>_b200/<shape hash>`` names the library, its ABI version, the
entry point and the kernel variant, so another process (or a non-Python
dispatcher) sees which versions exist and how to call them.  Supported patterns:
every ``linear*`` pattern, ``linear_residual``, and the single-GEMM
``needs_template`` neighbours the engine runs on the same kernels:
``attention_output`` (a plain GEMM) and ``attention_score`` (GEMM times a
scale; the request's optional ``"scale"`` gives its value).  The two-GEMM
``mlp_residual`` chain (Y = GELU(X W1 + b1) W2 + b2 + X; inputs X[M,K],
W1[K,H], b1[H], W2[H,K], b2[K]) compiles into two native plans, the second
taking X as its residual; its record lists both calls.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import threading
from dataclasses import dataclass

import torch

from . import _native as nat
from .fusion import FUSION_DB
from .linear import DTYPE_CODES, _workspace, activation_code

DTYPE_NAMES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
DTYPE_OF = {v: k for k, v in DTYPE_NAMES.items()}

# pattern -> (activation, has bias input, has residual input)
PLAN_PATTERNS = {
    "linear": (None, True, False),
    "linear_relu": ("relu", True, False),
    "linear_gelu": ("gelu", True, False),
    "linear_silu": ("silu", True, False),
    "linear_swish": ("swish", True, False),
    "linear_residual": (None, True, True),
    "attention_output": (None, False, False),
    "attention_score": (None, False, False),
}
# Chains of two plans: pattern -> activation of the first GEMM.  For these a
# request's N is the hidden width H and the output is [M, K].
CHAIN_PATTERNS = {"mlp_residual": "gelu"}


class CompileError(ValueError):
    """The request does not describe a fused linear this engine can plan."""


@dataclass(frozen=True)
class CompileRequest:
    func: str
    pattern: str
    ops: tuple
    M: int
    N: int
    K: int
    dtype: torch.dtype
    scale: float = 1.0

    @property
    def key(self) -> tuple:
        return (self.pattern, self.M, self.N, self.K, self.dtype, self.scale)

    @property
    def shape_hash(self) -> str:
        """16 hex digits identifying (pattern, M, N, K, dtype, scale)."""
        canon = json.dumps({"pattern": self.pattern, "M": self.M, "N": self.N, "K": self.K,
                            "dtype": DTYPE_OF[self.dtype], "scale": self.scale}, sort_keys=True)
        return hashlib.sha1(canon.encode()).hexdigest()[:16]

    def to_json(self) -> dict:
        """A compile request that parses back to this one."""
        dt = DTYPE_OF[self.dtype]
        if self.pattern in CHAIN_PATTERNS:
            M, H, K = self.M, self.N, self.K
            inputs = [{"shape": s_, "dtype": dt} for s_ in ([M, K], [K, H], [H], [H, K], [K])]
            return {"func": self.func, "pattern": self.pattern, "ops": list(self.ops),
                    "inputs": inputs, "outputs": [{"shape": [M, K], "dtype": dt}],
                    "accum_dtype": "float32", "scale": self.scale}
        _, has_bias, has_res = PLAN_PATTERNS[self.pattern]
        inputs = [{"shape": [self.M, self.K], "dtype": dt}, {"shape": [self.K, self.N], "dtype": dt}]
        if has_bias:
            inputs.append({"shape": [self.N], "dtype": dt})
        if has_res:
            inputs.append({"shape": [self.M, self.N], "dtype": dt})
        if self.pattern == "attention_score":
            inputs.append({"shape": [1], "dtype": dt})
        return {"func": self.func, "pattern": self.pattern, "ops": list(self.ops),
                "inputs": inputs, "outputs": [{"shape": [self.M, self.N], "dtype": dt}],
                "accum_dtype": "float32", "scale": self.scale}

    @classmethod
    def from_json(cls, request) -> "CompileRequest":
        req = json.loads(request) if isinstance(request, (str, bytes)) else dict(request)
        try:
            pattern = req["pattern"]
            ops = tuple(req["ops"])
            inputs = req["inputs"]
            outputs = req["outputs"]
        except KeyError as e:
            raise CompileError(f"compile request lacks {e.args[0]!r}") from None
        chain = tuple(op if op.startswith("tensor.") else f"tensor.{op}" for op in ops)
        row = FUSION_DB.get(chain)
        if row is None or row[0] != pattern:
            raise CompileError(f"ops {list(ops)} do not form pattern {pattern!r}")
        if pattern not in PLAN_PATTERNS and pattern not in CHAIN_PATTERNS:
            raise CompileError(f"pattern {pattern!r} is not a fused GEMM or chain the engine "
                               f"plans (status {row[2]})")
        if req.get("accum_dtype", "float32") != "float32":
            raise CompileError("only float32 accumulation is supported")
        if pattern in CHAIN_PATTERNS:
            return cls._chain_from_json(req, pattern, ops, inputs, outputs)
        _, has_bias, has_res = PLAN_PATTERNS[pattern]
        n_in = 2 + int(has_bias) + int(has_res) + (1 if pattern == "attention_score" else 0)
        if len(inputs) != n_in or len(outputs) != 1:
            raise CompileError(f"{pattern} takes {n_in} inputs and 1 output, got "
                               f"{len(inputs)} and {len(outputs)}")
        dtypes = {t["dtype"] for t in list(inputs[:2]) + list(outputs)}
        if len(dtypes) != 1 or next(iter(dtypes)) not in DTYPE_NAMES:
            raise CompileError(f"inputs/outputs must share one of {list(DTYPE_NAMES)}")
        (M, K), (K2, N) = inputs[0]["shape"], inputs[1]["shape"]
        if K != K2:
            raise CompileError(f"inner dimensions differ: {K} vs {K2}")
        if list(outputs[0]["shape"]) != [M, N]:
            raise CompileError(f"output shape {outputs[0]['shape']} is not [{M}, {N}]")
        if has_bias and list(inputs[2]["shape"]) != [N]:
            raise CompileError(f"bias shape {inputs[2]['shape']} is not [{N}]")
        if has_res and list(inputs[3]["shape"]) != [M, N]:
            raise CompileError(f"residual shape {inputs[3]['shape']} is not [{M}, {N}]")
        return cls(req.get("func", ""), pattern, ops, int(M), int(N), int(K),
                   DTYPE_NAMES[next(iter(dtypes))], float(req.get("scale", 1.0)))

    @classmethod
    def _chain_from_json(cls, req, pattern, ops, inputs, outputs) -> "CompileRequest":
        if len(inputs) != 5 or len(outputs) != 1:
            raise CompileError(f"{pattern} takes 5 inputs (X, W1, b1, W2, b2) and 1 output, got "
                               f"{len(inputs)} and {len(outputs)}")
        dtypes = {t["dtype"] for t in list(inputs) + list(outputs)}
        if len(dtypes) != 1 or next(iter(dtypes)) not in DTYPE_NAMES:
            raise CompileError(f"inputs/outputs must share one of {list(DTYPE_NAMES)}")
        (M, K), (K1, H) = inputs[0]["shape"], inputs[1]["shape"]
        want = [[M, K], [K, H], [H], [H, K], [K]]
        got = [list(t["shape"]) for t in inputs]
        if K1 != K or got != want:
            raise CompileError(f"{pattern} input shapes {got} are not {want}")
        if list(outputs[0]["shape"]) != [M, K]:
            raise CompileError(f"output shape {outputs[0]['shape']} is not [{M}, {K}]")
        return cls(req.get("func", ""), pattern, ops, int(M), int(H), int(K),
                   DTYPE_NAMES[next(iter(dtypes))], float(req.get("scale", 1.0)))


class Plan:
    """A native plan: call(x, W, b=None, out=None, residual=None) -> out."""

    def __init__(self, request: CompileRequest, kernel: str = "auto"):
        act, self.has_bias, self.has_residual = PLAN_PATTERNS[request.pattern]
        self.request = request
        self._lib = nat.load()
        handle = ctypes.c_void_p()
        nat.check("dx_plan_create", self._lib.dx_plan_create(
            ctypes.byref(handle), request.M, request.N, request.K, DTYPE_CODES[request.dtype],
            activation_code(act), request.scale, nat.KERNEL_NAMES[kernel]))
        self._handle = handle
        # The native plan holds one workspace pointer: setting it and calling
        # must not interleave between threads (each stream has its own workspace).
        self._call_lock = threading.Lock()

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            self._lib.dx_plan_destroy(handle)
            self._handle = None

    def __call__(self, x: torch.Tensor, W: torch.Tensor, b: torch.Tensor | None = None,
                 out: torch.Tensor | None = None,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
        r = self.request
        for name, t, shape in (("x", x, (r.M, r.K)), ("W", W, (r.K, r.N))):
            if tuple(t.shape) != shape or t.dtype != r.dtype or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous {r.dtype} tensor of shape {shape}")
        if (b is not None) != self.has_bias:
            raise ValueError(f"{r.pattern} {'needs' if self.has_bias else 'takes no'} bias")
        if (residual is not None) != self.has_residual:
            raise ValueError(f"{r.pattern} {'needs' if self.has_residual else 'takes no'} residual")
        if out is None:
            out = torch.empty((r.M, r.N), dtype=r.dtype, device=x.device)
        with torch.cuda.device(x.device), self._call_lock:
            stream = torch.cuda.current_stream(x.device).cuda_stream
            need = self._lib.dx_plan_workspace_size(self._handle)
            ws = _workspace(x.device, stream, need)
            nat.check("dx_plan_set_workspace", self._lib.dx_plan_set_workspace(
                self._handle, ws.data_ptr() if ws is not None else None,
                ws.numel() if ws is not None else 0))
            rc = self._lib.dx_plan_call_residual(
                self._handle, x.data_ptr(), W.data_ptr(), b.data_ptr() if b is not None else None,
                residual.data_ptr() if residual is not None else None, out.data_ptr(), stream)
        nat.check("dx_plan_call", rc)
        return out


class ChainPlan:
    """Two native plans for a two-GEMM chain (``mlp_residual``):
    call(x, W1, b1, W2, b2, out=None, hidden=None) -> out, where
    hidden = act(x W1 + b1) and out = hidden W2 + b2 + x."""

    def __init__(self, request: CompileRequest, kernel: str = "auto"):
        self.request = request
        M, H, K, dt = request.M, request.N, request.K, request.dtype
        act = CHAIN_PATTERNS[request.pattern]
        up = CompileRequest(request.func, "linear_gelu", ("matmul", "add", "gelu"), M, H, K, dt)
        down = CompileRequest(request.func, "linear_residual", ("matmul", "add", "add"), M, K, H,
                              dt)
        self.up = Plan(up, kernel)
        self.down = Plan(down, kernel)
        del act  # the up plan's activation (linear_gelu) is the chain's GELU

    def __call__(self, x: torch.Tensor, W1: torch.Tensor, b1: torch.Tensor, W2: torch.Tensor,
                 b2: torch.Tensor, out: torch.Tensor | None = None,
                 hidden: torch.Tensor | None = None) -> torch.Tensor:
        H = self.up(x, W1, b1, out=hidden)
        return self.down(H, W2, b2, out=out, residual=x)


def record_key(req: CompileRequest, prefix: str = "/func") -> str:
    """kvspace key of a compiled version: ``<prefix>/<func>_b200/<shape hash>``."""
    return f"{prefix.rstrip('/')}/{req.func or req.pattern}_b200/{req.shape_hash}"


def plan_record(req: CompileRequest) -> dict:
    """What a dispatcher needs to call a compiled version without Python."""
    lib = nat.load()
    if req.pattern in CHAIN_PATTERNS:
        names = {v: k for k, v in nat.KERNEL_NAMES.items()}
        M, H, K = req.M, req.N, req.K
        dt = DTYPE_CODES[req.dtype]
        return {"request": req.to_json(), "shape_hash": req.shape_hash,
                "library": nat.LIB_PATH.name, "abi_version": int(lib.dx_version()),
                "create": "dx_plan_create",
                "calls": [
                    {"entry": "dx_plan_call", "M": M, "N": H, "K": K,
                     "act": CHAIN_PATTERNS[req.pattern], "args": ["X", "W1", "b1", "hidden"],
                     "kernel": names.get(lib.dx_select_kernel(M, H, K, dt), "?")},
                    {"entry": "dx_plan_call_residual", "M": M, "N": K, "K": H, "act": None,
                     "args": ["hidden", "W2", "b2", "X", "out"],
                     "kernel": names.get(lib.dx_select_kernel(M, K, H, dt), "?")}]}
    kernel = lib.dx_select_kernel(req.M, req.N, req.K, DTYPE_CODES[req.dtype])
    names = {v: k for k, v in nat.KERNEL_NAMES.items()}
    return {"request": req.to_json(), "shape_hash": req.shape_hash,
            "library": nat.LIB_PATH.name, "abi_version": int(lib.dx_version()),
            "create": "dx_plan_create",
            "entry": "dx_plan_call_residual" if PLAN_PATTERNS[req.pattern][2] else "dx_plan_call",
            "kernel": names.get(kernel, str(kernel))}


class PlanCache:
    """Plans keyed by (pattern, M, N, K, dtype, scale): the docs' shape-keyed
    compiled-kernel cache (doc/kvlang-to-tilelang-interface.md:194-218).

    With ``kv`` (a kvspace store: ``get``/``set``/``list``), every compiled
    version is also recorded under ``record_key``; a request whose record is
    already in the store counts as a kvspace hit (``kv_hits``) and its plan is
    rebuilt from the stored request, which must match the one asked for."""

    def __init__(self, kv=None, prefix: str = "/func"):
        self._plans: dict[tuple, Plan | ChainPlan] = {}
        self._lock = threading.Lock()
        self.kv = kv
        self.prefix = prefix
        self.hits = 0
        self.kv_hits = 0
        self.misses = 0

    def _stored(self, req: CompileRequest) -> dict | None:
        if self.kv is None:
            return None
        try:
            value = self.kv.get(record_key(req, self.prefix))
        except KeyError:  # the store's ErrNotFound derives from KeyError
            return None
        record = json.loads(value.as_str())
        if CompileRequest.from_json(record["request"]).key != req.key:
            raise CompileError(f"kvspace record {record_key(req, self.prefix)} holds another "
                               f"request (shape-hash collision)")
        return record

    def get(self, request) -> "Plan | ChainPlan":
        req = request if isinstance(request, CompileRequest) else CompileRequest.from_json(request)
        with self._lock:
            plan = self._plans.get(req.key)
            if plan is not None:
                self.hits += 1
                return plan
            stored = self._stored(req)
            plan = ChainPlan(req) if req.pattern in CHAIN_PATTERNS else Plan(req)
            if stored is not None:
                self.kv_hits += 1
            else:
                self.misses += 1
                if self.kv is not None:
                    self.kv.set(record_key(req, self.prefix), json.dumps(plan_record(req)))
            self._plans[req.key] = plan
            return plan

    def records(self, func: str) -> dict[str, dict]:
        """Compiled versions of ``func`` recorded in the store, by shape hash."""
        if self.kv is None:
            return {}
        base = f"{self.prefix.rstrip('/')}/{func}_b200"
        try:
            names = self.kv.list(base)
        except KeyError:
            return {}
        return {h: json.loads(self.kv.get(f"{base}/{h}").as_str()) for h in names}

    def __len__(self) -> int:
        return len(self._plans)


_default_cache = PlanCache()
_kv_caches: dict[int, PlanCache] = {}
_kv_caches_lock = threading.Lock()


def compile_request(request, kv=None) -> Plan:
    """Compile (or fetch from a cache) the plan for a request.  Without ``kv``
    the process-wide cache is used; with a kvspace store, a cache bound to that
    store (one per store) records the compiled version there."""
    if kv is None:
        return _default_cache.get(request)
    with _kv_caches_lock:
        cache = _kv_caches.get(id(kv))
        if cache is None or cache.kv is not kv:
            cache = _kv_caches[id(kv)] = PlanCache(kv)
    return cache.get(request)
