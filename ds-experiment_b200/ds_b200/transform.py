"""The DS pass on torch programs: f64 / f32 arithmetic rewritten to DS.

The reference rewrites a StableHLO function (DsTransformPass.cpp:199-467):
float arguments and constants enter as (hi, lo) pairs (emitFromFloat,
:211-218, :232-244), add / subtract / multiply become DS operations
(:282-321), dot_general the DS product (:337-370), a single-input reduce
whose body is one add, subtract or multiply the DS reduce (:376-448),
broadcast_in_dim is applied to hi and lo alike (:259-279), and every DS
value that reaches func.return is recombined (emitToFloat, :451-461).  An
operation the pass does not know, or one with an operand that is not DS,
stays as it was.  A PJRT proxy runs the pass whenever JAX compiles a module
(ds_pjrt_plugin.cpp:134-159).

Here the program is a torch function.  It is captured with torch.fx the
first time it is called with a given signature (that is the compile-time
interception), and it is lowered onto this library's targets by the same rules:

- a connected elementwise DAG of add / sub / mul / neg becomes ONE
  generated kernel (ds_fused_run), where the pass emits a chain of f32 ops;
- `sum` / `prod` over DS values become ds_reduce_packed (ds_reduce_from_f64
  for an f64 argument, which splits as it loads); a reduction of an
  elementwise DAG over all or over its trailing dimensions runs in the DAG's
  own kernel (ds_fused_reduce, ds_fused_reduce_rows);
- `matmul` / `mm` / `bmm` / `@` become ds_dot_general_f64 (tensor cores);
- layout operations (reshape, view, unsqueeze, squeeze, expand, transpose,
  permute, t, T, mT, flatten, contiguous) act on hi and lo alike, as the
  pass's broadcast_in_dim does; implicit broadcasting happens inside the
  fused kernels;
- DS values are recombined where the program returns them, to the dtype
  the program gives them (f64, or f32 as hi + lo in f32).

    from ds_b200 import ds_transform

    @ds_transform
    def f(a, b, c):
        return ((a + b) * c).sum(dim=1), a @ b

    s, p = f(a, b, c)          # CUDA tensors in and out, DS arithmetic inside
    print(f.explain(a, b, c))  # the lowered program, one line per launch

By design, this differs from the reference in three places:
- An operation left alone that reads a computed DS value gets that value
  recombined.  The reference keeps the original float operation alive and
  reads its plain result.  Arguments are read as they are, in both.
- The product is the exact-split tensor-core dot_general, not four f32
  dots (the pass's :359-365).
- A reduce of an f64 argument accumulates each thread's elements in f64
  before the DS tree.
"""
from __future__ import annotations

import inspect
import math
import operator
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.fx as fx
from torch.fx.node import map_aggregate

from . import _lib, fuse, ops

_KIND_OF = {torch.float64: "f64", torch.float32: "f32"}
_MAX_OPS = 256     # ds_fused_run's limits per program
_MAX_INPUTS = 16

ADD, SUB, MUL, NEG = _lib.DS_FUSED_ADD, _lib.DS_FUSED_SUB, _lib.DS_FUSED_MUL, _lib.DS_FUSED_NEG
POS = -1  # unary plus: the operand itself

# Elementwise operations the pass rewrites (stablehlo add / subtract /
# multiply / negate), by fx target: a function, or ("method", name).
_EW = {
    operator.add: ADD, operator.sub: SUB, operator.mul: MUL, operator.neg: NEG, operator.pos: POS,
    torch.add: ADD, torch.sub: SUB, torch.subtract: SUB, torch.mul: MUL, torch.multiply: MUL,
    torch.neg: NEG, torch.negative: NEG,
    ("method", "add"): ADD, ("method", "sub"): SUB, ("method", "subtract"): SUB,
    ("method", "mul"): MUL, ("method", "multiply"): MUL, ("method", "neg"): NEG,
    ("method", "negative"): NEG,
}
# Reductions: the body the pass would see (sum -> add, prod -> multiply) and its init.
_REDUCE = {torch.sum: ("add", 0.0), ("method", "sum"): ("add", 0.0),
           torch.prod: ("mul", 1.0), ("method", "prod"): ("mul", 1.0)}
_DOT = {torch.matmul, operator.matmul, torch.mm, torch.bmm, ("method", "matmul"),
        ("method", "mm"), ("method", "bmm")}
_LAYOUT_METHODS = {"reshape", "view", "unsqueeze", "squeeze", "expand", "transpose", "permute",
                   "t", "flatten", "contiguous"}
_LAYOUT_FUNCS = {torch.reshape: "reshape", torch.unsqueeze: "unsqueeze", torch.squeeze: "squeeze",
                 torch.transpose: "transpose", torch.permute: "permute", torch.t: "t",
                 torch.flatten: "flatten"}
_LAYOUT_ATTRS = {"T", "mT"}


def _key(node: fx.Node):
    return ("method", node.target) if node.op == "call_method" else node.target


def _is_number(x) -> bool:
    return isinstance(x, (int, float)) and not isinstance(x, bool)


class _Const:
    """A constant operand: emitFromFloat of `value` in the program.  A 0-d
    float tensor constant of the graph keeps its tensor in `slot` for the
    operations that read it as it is."""
    __slots__ = ("value", "slot")

    def __init__(self, value: float, slot: Optional[str] = None):
        self.value, self.slot = float(value), slot


class _Pending:
    """An elementwise DS operation that has not been emitted yet."""
    __slots__ = ("code", "operands")

    def __init__(self, code: int, operands: list):
        self.code, self.operands = code, operands


class _Leaf:
    """A DS value held in a tensor at run time: kind "f64" / "f32" (split as
    it is read) or "packed" ([..., 2] hi, lo).  `raw` marks a program input
    (an argument or constant, or a view of one), which operations left alone
    read as it is."""
    __slots__ = ("slot", "kind", "raw")

    def __init__(self, slot: str, kind: str, raw: bool):
        self.slot, self.kind, self.raw = slot, kind, raw


class _Plain:
    """A value the pass leaves alone (not DS)."""
    __slots__ = ("slot",)

    def __init__(self, slot: str):
        self.slot = slot


class _SlotRef:
    """Stands for an environment slot inside an argument template."""
    __slots__ = ("slot",)

    def __init__(self, slot: str):
        self.slot = slot

    def __repr__(self):
        return f"%{self.slot}"


def _subst(template, env):
    return map_aggregate(template, lambda a: env[a.slot] if isinstance(a, _SlotRef) else a)


# ---- run-time steps --------------------------------------------------------------
# Each step reads its inputs from the environment (slot -> value) and writes
# one slot; `text` is its line in explain().


class _FusedStep:
    def __init__(self, out, prog, inputs, kinds, out_kind, shape):
        self.out, self.inputs, self.shape = out, list(inputs), tuple(shape)
        self.prepared = fuse.Prepared(prog, kinds, out_kind)
        names = ", ".join(f"%{s}:{k}" for s, k in zip(inputs, kinds))
        self.text = (f"%{out} = ds_fused_run[{len(prog)} ops]({names}) -> {out_kind} "
                     f"{list(self.shape)}")

    def run(self, env):
        env[self.out] = self.prepared([env[s] for s in self.inputs], self.shape)


class _ReduceStep:
    def __init__(self, out, src, kind, dims, body, init, shape):
        self.out, self.src, self.kind = out, src, kind
        self.dims, self.body, self.init, self.shape = tuple(dims), body, init, tuple(shape)
        target = "ds_reduce_packed" if kind == "packed" else "ds_reduce_from_f64"
        self.text = (f"%{out} = {target}(%{src}, dimensions={list(self.dims)}, body={body}, "
                     f"init={init}) -> packed {list(self.shape)}")

    def run(self, env):
        x = env[self.src]
        if self.kind == "packed":
            if x.dim() == 1:  # a 0-d DS value: reduce it as one element
                x = x.reshape(1, 2)
            hi, lo = ops.ds_reduce_packed(x.contiguous(), init=(self.init, 0.0),
                                          dimensions=self.dims, body=self.body)
        else:
            if x.dim() == 0:
                x = x.reshape(1)
            hi, lo = ops.ds_reduce_from_f64(x.contiguous(), init=self.init, dimensions=self.dims,
                                            body=self.body)
        env[self.out] = torch.stack([hi, lo], dim=-1).reshape(self.shape + (2,))


class _FusedReduceStep:
    """A pending elementwise value reduced over all its dimensions in the
    same kernel (ds_fused_reduce): its values are never written."""

    def __init__(self, out, prog, inputs, kinds, map_shape, body, init, shape):
        self.out, self.inputs = out, list(inputs)
        self.map_shape, self.body, self.init, self.shape = tuple(map_shape), body, init, tuple(shape)
        self.prepared = fuse.Prepared(prog, kinds, "packed")
        names = ", ".join(f"%{s}:{k}" for s, k in zip(inputs, kinds))
        self.text = (f"%{out} = ds_fused_reduce[{len(prog)} ops]({names}) over "
                     f"{list(self.map_shape)}, body={body}, init={init} -> packed {list(self.shape)}")

    def run(self, env):
        hi, lo = self.prepared.reduce([env[s] for s in self.inputs], self.map_shape, self.body,
                                      (self.init, 0.0))
        env[self.out] = torch.stack([hi, lo], dim=-1).reshape(self.shape + (2,))


class _FusedReduceRowsStep:
    """A pending elementwise value reduced over its trailing dimensions in
    the same kernel (ds_fused_reduce_rows): one block folds a whole row."""

    def __init__(self, out, prog, inputs, kinds, map_shape, n_reduced, body, init, shape):
        self.out, self.inputs = out, list(inputs)
        self.map_shape, self.n_reduced = tuple(map_shape), int(n_reduced)
        self.body, self.init, self.shape = body, init, tuple(shape)
        self.prepared = fuse.Prepared(prog, kinds, "packed")
        names = ", ".join(f"%{s}:{k}" for s, k in zip(inputs, kinds))
        self.text = (f"%{out} = ds_fused_reduce_rows[{len(prog)} ops]({names}) over "
                     f"{list(self.map_shape)}, last {self.n_reduced} dims, body={body}, "
                     f"init={init} -> packed {list(self.shape)}")

    def run(self, env):
        hi, lo = self.prepared.reduce_rows([env[s] for s in self.inputs], self.map_shape,
                                           self.n_reduced, self.body, (self.init, 0.0))
        env[self.out] = torch.stack([hi, lo], dim=-1).reshape(self.shape + (2,))


def ds_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """torch.matmul's shape rules over ds_dot_general_f64 (f64 operands):
    1-D operands gain and lose a unit dimension, batch dimensions broadcast,
    and a 2-D right operand shares one product over all the left rows."""
    ad, bd = a.dim(), b.dim()
    if ad == 0 or bd == 0:
        raise ValueError("matmul operands need at least one dimension")
    a2 = a.unsqueeze(0) if ad == 1 else a
    b2 = b.unsqueeze(-1) if bd == 1 else b
    if b2.dim() == 2:
        lead = tuple(a2.shape[:-1])
        r = ops.ds_dot_general_f64(a2.reshape(-1, a2.shape[-1]).contiguous(), b2.contiguous())
        r = r.reshape(lead + (b2.shape[-1],))
    else:
        batch = tuple(torch.broadcast_shapes(a2.shape[:-2], b2.shape[:-2]))
        A = a2.expand(batch + tuple(a2.shape[-2:])).reshape((-1,) + tuple(a2.shape[-2:]))
        B = b2.expand(batch + tuple(b2.shape[-2:])).reshape((-1,) + tuple(b2.shape[-2:]))
        r = ops.ds_dot_general_f64(A.contiguous(), B.contiguous(), lhs_batch=(0,), rhs_batch=(0,))
        r = r.reshape(batch + (A.shape[-2], B.shape[-1]))
    if ad == 1:
        r = r.squeeze(-2)
    if bd == 1:
        r = r.squeeze(-1)
    return r


class _DotStep:
    def __init__(self, out, a, b, shape):
        self.out, self.a, self.b, self.shape = out, a, b, tuple(shape)
        self.text = f"%{out} = ds_dot_general_f64(%{a}, %{b}) -> f64 {list(self.shape)}"

    def run(self, env):
        env[self.out] = ds_matmul(env[self.a], env[self.b])


def packed_layout(p: torch.Tensor, name: str, args: Sequence, kwargs: Dict) -> torch.Tensor:
    """Layout operation `name` of a DS tensor's logical shape applied to its
    packed storage p[..., 2] (hi and lo move together)."""
    r = p.dim() - 1

    def nd(d, extra=0):
        d = int(d)
        return d + r + extra if d < 0 else d

    def seq(a):
        return tuple(a[0]) if len(a) == 1 and isinstance(a[0], (tuple, list, torch.Size)) \
            else tuple(a)
    if name in ("reshape", "view"):
        shape = seq(args) if args else tuple(kwargs["shape"])
        return p.reshape(shape + (2,))
    if name == "unsqueeze":
        return p.unsqueeze(nd(args[0] if args else kwargs["dim"], 1))
    if name == "squeeze":
        dim = args[0] if args else kwargs.get("dim")
        if dim is None:
            dims = [i for i in range(r) if p.shape[i] == 1]
        else:
            dims = [nd(d) for d in (dim if isinstance(dim, (tuple, list)) else (dim,))]
            dims = [d for d in dims if p.shape[d] == 1]
        return p.reshape(tuple(s for i, s in enumerate(p.shape[:r]) if i not in dims) + (2,))
    if name == "expand":
        return p.expand(seq(args) + (2,))
    if name == "transpose":
        a0, a1 = (args[0], args[1]) if len(args) == 2 else (kwargs["dim0"], kwargs["dim1"])
        return p.transpose(nd(a0), nd(a1))
    if name == "permute":
        dims = seq(args) if args else tuple(kwargs["dims"])
        return p.permute(tuple(nd(d) for d in dims) + (r,))
    if name == "t":
        return p.transpose(0, 1) if r == 2 else p
    if name == "T":
        return p.permute(tuple(reversed(range(r))) + (r,))
    if name == "mT":
        return p.transpose(r - 2, r - 1)
    if name == "flatten":
        s = nd(args[0] if len(args) > 0 else kwargs.get("start_dim", 0)) if r else 0
        e = nd(args[1] if len(args) > 1 else kwargs.get("end_dim", -1)) if r else 0
        if r == 0:
            return p.reshape(1, 2)
        shape = tuple(p.shape[:s]) + (math.prod(p.shape[s:e + 1]),) + tuple(p.shape[e + 1:r])
        return p.reshape(shape + (2,))
    if name == "contiguous":
        return p.contiguous()
    raise ValueError(f"no packed layout rule for {name}")


class _LayoutStep:
    def __init__(self, out, src, kind, name, args, kwargs):
        self.out, self.src, self.kind = out, src, kind
        self.name, self.args, self.kwargs = name, args, kwargs
        self.text = f"%{out} = {name}(%{src}:{kind}, {args}, {kwargs}) -> {kind}"

    def run(self, env):
        x = env[self.src]
        args, kwargs = _subst(self.args, env), _subst(self.kwargs, env)
        if self.kind == "packed":
            env[self.out] = packed_layout(x, self.name, args, kwargs)
        elif self.name in _LAYOUT_ATTRS:
            env[self.out] = getattr(x, self.name)
        else:
            env[self.out] = getattr(x, self.name)(*args, **kwargs)


class _PlainStep:
    """An operation the pass leaves alone, run by torch."""

    def __init__(self, out, node: fx.Node, args, kwargs, gm):
        self.out, self.op, self.target = out, node.op, node.target
        self.args, self.kwargs = args, kwargs
        self.fn = None
        if node.op == "call_function":
            self.fn = node.target
        elif node.op == "call_module":
            self.fn = gm.get_submodule(node.target)
        name = getattr(node.target, "__name__", str(node.target))
        self.text = f"%{out} = torch {name}{tuple(args)}"

    def run(self, env):
        args, kwargs = _subst(self.args, env), _subst(self.kwargs, env)
        if self.op == "call_method":
            env[self.out] = getattr(args[0], self.target)(*args[1:], **kwargs)
        else:
            env[self.out] = self.fn(*args, **kwargs)


# ---- lowering ----------------------------------------------------------------------


def _meta(node: fx.Node):
    """(dtype, shape) of a tensor-valued node after shape propagation, else None."""
    tm = node.meta.get("tensor_meta")
    if tm is None or not hasattr(tm, "dtype"):
        return None
    return tm.dtype, tuple(tm.shape)


def _float_kind(node: fx.Node) -> Optional[str]:
    m = _meta(node)
    return _KIND_OF.get(m[0]) if m else None


def _reduce_dims(node: fx.Node, src: fx.Node):
    """(dims, keepdim) of a sum / prod node, or None if it is not a plain
    reduction of src (a dtype change, an out= argument, a symbolic dim)."""
    args, kw = list(node.args[1:]), dict(node.kwargs)
    dim = args.pop(0) if args else kw.pop("dim", None)
    keepdim = args.pop(0) if args else kw.pop("keepdim", False)
    dtype = kw.pop("dtype", None)
    if args or kw or isinstance(dim, fx.Node) or isinstance(keepdim, fx.Node):
        return None
    in_dtype, shape = _meta(src)
    if dtype is not None and dtype != in_dtype:
        return None
    rank = len(shape)
    if dim is None or (isinstance(dim, (tuple, list)) and len(dim) == 0):
        dims = tuple(range(rank))
    else:
        ds = dim if isinstance(dim, (tuple, list)) else (dim,)
        if not all(isinstance(d, int) for d in ds) or rank == 0:
            return None
        dims = tuple(sorted({d % rank for d in ds}))
    out = [1 if i in dims else s for i, s in enumerate(shape)] if keepdim else \
        [s for i, s in enumerate(shape) if i not in dims]
    if tuple(out) != _meta(node)[1]:
        return None
    return dims, bool(keepdim)


class _Lowering:
    """Walks the captured graph once and emits the step list.

    Node states: _Leaf (a DS value in a tensor), _Pending (an elementwise DS
    operation, emitted later inside a fused program), _Plain (left alone).
    A pending value is emitted where something other than an elementwise
    DS operation reads it: as packed for a reduce or a layout operation, f64
    for a product, its own dtype for an operation left alone or the return.
    A pending value read in two of these forms, or by one such consumer and
    by other elementwise operations, is emitted once, packed, where it is
    defined; one form for several consumers is one cached program."""

    def __init__(self, gm: fx.GraphModule, args: Sequence):
        self.gm = gm
        self.args = args
        self.state: Dict[fx.Node, Any] = {}
        self.steps: List[Any] = []
        self.consts: Dict[str, torch.Tensor] = {}
        self.cache: Dict[tuple, str] = {}
        self.device = next((a.device for a in args if isinstance(a, torch.Tensor)), None)
        self._n = 0
        self._demands: Dict[fx.Node, set] = {}
        self._ew_users: Dict[fx.Node, int] = {}

    def slot(self, base: str) -> str:
        self._n += 1
        return f"{base}.{self._n}"

    # -- classification ------------------------------------------------------------

    def is_ds(self, x) -> bool:
        return isinstance(x, fx.Node) and isinstance(self.state.get(x), (_Leaf, _Pending))

    def ew_operands(self, node: fx.Node):
        """(code, operands) of an elementwise DS operation, else None.  A
        number becomes a constant of the result's precision (an f32 program
        has f32 constants, as stablehlo would)."""
        code = _EW.get(_key(node))
        kind = _float_kind(node)
        if code is None or kind is None:
            return None
        args, kw = list(node.args), dict(node.kwargs)
        alpha = kw.pop("alpha", None) if code in (ADD, SUB) else None
        if "other" in kw and len(args) == 1:
            args.append(kw.pop("other"))
        if kw or len(args) != (1 if code in (NEG, POS) else 2):
            return None
        if isinstance(alpha, fx.Node) or not (alpha is None or _is_number(alpha)):
            return None
        def const(v):
            return _Const(float(np.float32(v)) if kind == "f32" else float(v))
        operands = []
        for a in args:
            if isinstance(a, fx.Node):
                st = self.state.get(a)
                if isinstance(st, _Const):
                    operands.append(const(st.value))
                elif self.is_ds(a):
                    operands.append(a)
                else:
                    return None
            elif _is_number(a):
                operands.append(const(a))
            else:
                return None
        if not any(isinstance(o, fx.Node) for o in operands):
            return None
        if alpha is not None and float(alpha) != 1.0:
            operands[1] = _Pending(MUL, [operands[1], const(alpha)])
        return code, operands

    def classify(self, node: fx.Node):
        """('ew', code, operands) | ('reduce', src, dims, keepdim, body, init) |
        ('dot', a, b) | ('layout', src, name, args, kwargs) | ('plain',)."""
        if node.op not in ("call_function", "call_method"):
            return ("plain",)
        ew = self.ew_operands(node)
        if ew is not None:
            return ("ew",) + ew
        key = _key(node)
        first = node.args[0] if node.args else None
        if key in _REDUCE and self.is_ds(first) and _float_kind(node):
            spec = _reduce_dims(node, first)
            if spec is not None:
                body, init = _REDUCE[key]
                return ("reduce", first, spec[0], spec[1], body, init)
        if key in _DOT and len(node.args) == 2 and not node.kwargs and _float_kind(node):
            a, b = node.args
            if self.is_ds(a) and self.is_ds(b):
                return ("dot", a, b)
        name = None
        if node.op == "call_method" and node.target in _LAYOUT_METHODS:
            name = node.target
        elif node.op == "call_function" and node.target in _LAYOUT_FUNCS:
            name = _LAYOUT_FUNCS[node.target]
        elif node.op == "call_function" and node.target is getattr and \
                len(node.args) == 2 and node.args[1] in _LAYOUT_ATTRS:
            name = node.args[1]
        if name is not None and self.is_ds(first) and _float_kind(node):
            rest = tuple(node.args[2:] if name in _LAYOUT_ATTRS else node.args[1:])
            flat = []
            map_aggregate((rest, dict(node.kwargs)), lambda a: flat.append(a) or a)
            if not any(self.is_ds(a) for a in flat):
                return ("layout", first, name, rest, dict(node.kwargs))
        return ("plain",)

    # -- the walk ------------------------------------------------------------------

    def _input_state(self, node: fx.Node, value):
        if isinstance(value, torch.Tensor) and value.dtype in _KIND_OF:
            if node.op == "get_attr" and value.dim() == 0:
                return _Const(value.item(), node.name)
            return _Leaf(node.name, _KIND_OF[value.dtype], True)
        return _Plain(node.name)

    def _pending_nodes(self, operands):
        """The Node operands (through unnamed operations) that are pending."""
        out = []
        for o in operands:
            if isinstance(o, _Pending):
                out += self._pending_nodes(o.operands)
            elif isinstance(o, fx.Node) and isinstance(self.state.get(o), _Pending):
                out.append(o)
        return out

    def _count_uses(self, cls):
        """Pass 1 bookkeeping: how many elementwise DS users and how many
        other readers each pending node has."""
        kind = cls[0]
        if kind == "ew":
            for o in self._pending_nodes(cls[2]):
                self._ew_users[o] = self._ew_users.get(o, 0) + 1
            return
        if kind in ("reduce", "dot", "layout"):
            reads = [cls[1]] + ([cls[2]] if kind == "dot" else [])
        else:
            reads = []
        for r in reads:
            if isinstance(self.state.get(r), _Pending):
                self._demands.setdefault(r, set()).add("f64" if kind == "dot" else "packed")

    def _count_plain(self, node: fx.Node):
        for a in node.all_input_nodes:
            if isinstance(self.state.get(a), _Pending):
                self._demands.setdefault(a, set()).add(_float_kind(a) or "f64")

    def lower(self):
        nodes = list(self.gm.graph.nodes)
        placeholders = [n for n in nodes if n.op == "placeholder"]
        if len(placeholders) != len(self.args):
            raise TypeError(f"the program takes {len(placeholders)} positional arguments, "
                            f"got {len(self.args)}")
        values = dict(zip(placeholders, self.args))
        # pass 1: classify every node (states stand in for what they will be)
        classes = {}
        for node in nodes:
            if node.op in ("placeholder", "get_attr"):
                v = values[node] if node.op == "placeholder" else self._attr(node)
                self.state[node] = self._input_state(node, v)
                continue
            if node.op == "output":
                self._count_plain(node)
                continue
            cls = self.classify(node) if node.op != "call_module" else ("plain",)
            classes[node] = cls
            if cls[0] == "plain":
                self._count_plain(node)
                self.state[node] = _Plain(node.name)
            else:
                self._count_uses(cls)
                self.state[node] = _Pending(0, []) if cls[0] == "ew" else _Leaf(node.name, "", False)
        # pass 2: emit
        self.state = {}
        self._cone: Dict[fx.Node, Tuple[set, set, int]] = {}
        inputs, output = [], None
        for node in nodes:
            if node.op == "placeholder":
                self.state[node] = self._input_state(node, values[node])
                inputs.append(node.name)
            elif node.op == "get_attr":
                self._emit_attr(node)
            elif node.op == "output":
                output = map_aggregate(node.args[0], lambda a: _SlotRef(self.output_slot(a))
                                       if isinstance(a, fx.Node) else a)
            else:
                getattr(self, "_emit_" + classes[node][0])(node, classes[node])
        return inputs, self.steps, output, self.consts

    def _attr(self, node: fx.Node):
        obj = self.gm
        for part in node.target.split("."):
            obj = getattr(obj, part)
        return obj

    def _emit_attr(self, node: fx.Node):
        v = self._attr(node)
        if isinstance(v, torch.Tensor) and self.device is not None and v.device != self.device:
            v = v.to(self.device)
        self.consts[node.name] = v
        self.state[node] = self._input_state(node, v)

    def _shape(self, node: fx.Node):
        return _meta(node)[1]

    # -- pending values and programs ------------------------------------------------

    def _cone_of(self, operands):
        """(pending nodes, leaf slots, constants) a program for these operands reads."""
        nodes, leaves, consts = set(), set(), 0
        for o in operands:
            if isinstance(o, _Const):
                consts += 1
            elif isinstance(o, _Pending):
                n, l, c = self._cone_of(o.operands)
                nodes |= n
                leaves |= l
                consts += c + 1
            else:
                st = self.state[o]
                if isinstance(st, _Const):
                    consts += 1
                elif isinstance(st, _Leaf):
                    leaves.add(st.slot)
                else:
                    n, l, c = self._cone[o]
                    nodes |= n
                    leaves |= l
                    consts += c
        return nodes, leaves, consts

    def _emit_ew(self, node: fx.Node, cls):
        _, code, operands = cls
        st = _Pending(code, operands)
        self.state[node] = st
        for attempt in range(2):
            nodes, leaves, consts = self._cone_of(operands)
            size = len(nodes) + 1 + len(leaves) + consts
            if size <= _MAX_OPS - 8 and len(leaves) <= _MAX_INPUTS:
                break
            # too large for one program: the pending operands become packed leaves
            for o in self._pending_nodes(operands):
                self._materialize(o)
        else:
            raise RuntimeError("an elementwise DS operation does not fit one program")
        self._cone[node] = (nodes | {node}, leaves, consts)
        # read in two forms, or by a consumer and by later programs: emit it
        # once, packed (one form for several consumers is one cached program)
        d, u = len(self._demands.get(node, ())), self._ew_users.get(node, 0)
        if d >= 2 or (d >= 1 and u >= 1):
            self._materialize(node)

    def _materialize(self, node: fx.Node):
        """Emit a pending node once, packed, and read it from there on."""
        if isinstance(self.state[node], _Pending):
            slot = self.need(node, "packed")
            self.state[node] = _Leaf(slot, "packed", False)

    def _program(self, root: fx.Node):
        prog, slots, kinds, index, memo = [], [], [], {}, {}

        def emit(x):
            if isinstance(x, _Const):
                prog.append((_lib.DS_FUSED_CONST, 0, 0, x.value))
                return len(prog) - 1
            k = x if isinstance(x, fx.Node) else id(x)
            if k in memo:
                return memo[k]
            st = self.state[x] if isinstance(x, fx.Node) else x
            if isinstance(st, _Const):
                prog.append((_lib.DS_FUSED_CONST, 0, 0, st.value))
                r = len(prog) - 1
            elif isinstance(st, _Leaf):
                if st.slot not in index:
                    index[st.slot] = len(slots)
                    slots.append(st.slot)
                    kinds.append(st.kind)
                prog.append((_lib.DS_FUSED_INPUT, index[st.slot], 0, 0.0))
                r = len(prog) - 1
            elif st.code == POS:
                r = emit(st.operands[0])
            else:
                ids = [emit(o) for o in st.operands]
                prog.append((st.code, ids[0], ids[1] if len(ids) > 1 else 0, 0.0))
                r = len(prog) - 1
            memo[k] = r
            return r
        emit(root)
        return prog, slots, kinds

    def need(self, node: fx.Node, kind: str, output: bool = False) -> str:
        """A slot holding node's DS value as `kind` ("f64", "f32", "packed").
        With `output`, an argument is recombined from its DS split (what
        the pass returns) rather than passed through."""
        st = self.state[node]
        if isinstance(st, _Leaf):
            if st.kind == kind and not (output and st.raw):
                return st.slot
            key = ("convert", st.slot, kind)
        elif isinstance(st, _Pending):
            key = ("pending", node, kind)
        else:
            raise TypeError(f"{node.name} is not a DS value")
        slot = self.cache.get(key)
        if slot is None:
            prog, slots, kinds = self._program(node)
            slot = self.slot(node.name)
            self.steps.append(_FusedStep(slot, prog, slots, kinds, kind, self._shape(node)))
            self.cache[key] = slot
        return slot

    # -- the other operations ----------------------------------------------------------

    def _emit_reduce(self, node: fx.Node, cls):
        _, src, dims, keepdim, body, init = cls
        st = self.state[src]
        rank = len(self._shape(src))
        if isinstance(st, _Pending) and rank > 0 and tuple(dims) == tuple(range(rank)):
            # a full reduction of an elementwise DAG: one kernel, no stores
            prog, slots, kinds = self._program(src)
            out = self.slot(node.name)
            self.steps.append(_FusedReduceStep(out, prog, slots, kinds, self._shape(src), body,
                                               init, self._shape(node)))
            self.state[node] = _Leaf(out, "packed", False)
            return
        k = len(dims)
        if isinstance(st, _Pending) and 0 < k < rank and tuple(dims) == tuple(range(rank - k, rank)):
            # its trailing dimensions: one kernel, a block per row, no stores
            prog, slots, kinds = self._program(src)
            out = self.slot(node.name)
            self.steps.append(_FusedReduceRowsStep(out, prog, slots, kinds, self._shape(src), k,
                                                   body, init, self._shape(node)))
            self.state[node] = _Leaf(out, "packed", False)
            return
        if isinstance(st, _Leaf) and st.kind == "f64":
            slot, kind = st.slot, "f64"
        else:
            slot, kind = self.need(src, "packed"), "packed"
        if len(self._shape(src)) == 0:
            dims = (0,)  # run as a one-element vector
        out = self.slot(node.name)
        self.steps.append(_ReduceStep(out, slot, kind, dims, body, init, self._shape(node)))
        self.state[node] = _Leaf(out, "packed", False)

    def _emit_dot(self, node: fx.Node, cls):
        _, a, b = cls
        sa, sb = self.need(a, "f64"), self.need(b, "f64")
        out = self.slot(node.name)
        self.steps.append(_DotStep(out, sa, sb, self._shape(node)))
        self.state[node] = _Leaf(out, "f64", False)

    def _emit_layout(self, node: fx.Node, cls):
        _, src, name, args, kwargs = cls
        st = self.state[src]
        if isinstance(st, _Leaf):
            slot, kind, raw = st.slot, st.kind, st.raw
        else:
            slot, kind, raw = self.need(src, "packed"), "packed", False
        args, kwargs = self._template(args), self._template(kwargs)
        out = self.slot(node.name)
        self.steps.append(_LayoutStep(out, slot, kind, name, args, kwargs))
        self.state[node] = _Leaf(out, kind, raw)

    def plain_slot(self, node: fx.Node) -> str:
        """The slot an operation left alone reads: arguments and constants
        as they are, computed DS values recombined to their own dtype."""
        st = self.state[node]
        if isinstance(st, (_Plain, _Const)):
            return st.slot
        if isinstance(st, _Leaf) and st.raw:
            return st.slot
        return self.need(node, _float_kind(node) or "f64")

    def output_slot(self, node: fx.Node) -> str:
        st = self.state[node]
        if isinstance(st, (_Plain, _Const)):
            return st.slot
        return self.need(node, _float_kind(node) or "f64", output=True)

    def _template(self, x):
        return map_aggregate(x, lambda a: _SlotRef(self.plain_slot(a))
                             if isinstance(a, fx.Node) else a)

    def _emit_plain(self, node: fx.Node, cls):
        out = node.name
        self.steps.append(_PlainStep(out, node, self._template(node.args),
                                     self._template(dict(node.kwargs)), self.gm))
        self.state[node] = _Plain(out)


# ---- the user-facing transform ----------------------------------------------------------


class _Plan:
    """The lowered program for one argument signature: its steps, the slots
    of the captured inputs, the constants, the output template and the
    values of the trailing parameters the call left at their defaults."""

    def __init__(self, gm, inputs, steps, output, consts, defaults=()):
        self.gm, self.inputs, self.steps = gm, inputs, steps
        self.output, self.consts = output, consts
        self.defaults = list(defaults)

    def run(self, args):
        env = dict(self.consts)
        env.update(zip(self.inputs, list(args) + self.defaults))
        for st in self.steps:
            st.run(env)
        return _subst(self.output, env)

    def run_graph(self, args):
        """Run as a CUDA graph: the first call runs the plan once (compiling
        its programs), then captures it over static copies of the tensor
        arguments; every call copies its tensors in and replays.  The
        returned tensors are the graph's own and are overwritten by the
        next call.  A plan that cannot be captured (a host sync in an
        operation left to torch) runs eagerly from then on."""
        g = getattr(self, "_graph", None)
        if g is None:
            out = self.run(args)  # compiles the programs and warms the allocator
            try:
                static = [a.clone() if isinstance(a, torch.Tensor) else a for a in args]
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    self.run(static)
                torch.cuda.current_stream().wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    static_out = self.run(static)
                self._graph = (graph, static, static_out)
            except Exception:
                self._graph = False
            return out
        if g is False:
            return self.run(args)
        graph, static, static_out = g
        for dst, src in zip(static, args):
            if isinstance(dst, torch.Tensor):
                dst.copy_(src)
        graph.replay()
        return static_out

    def launches(self) -> Dict[str, int]:
        """How many steps of each kind the plan runs (fused programs,
        reductions, products, layout and untouched torch operations)."""
        counts: Dict[str, int] = {}
        for st in self.steps:
            k = type(st).__name__.strip("_").replace("Step", "").lower()
            counts[k] = counts.get(k, 0) + 1
        return counts

    def explain(self) -> str:
        lines = [f"inputs: {', '.join('%' + s for s in self.inputs)}"]
        lines += [st.text for st in self.steps]
        lines.append(f"return {self.output}")
        return "\n".join(lines)


def _signature_key(args):
    key = []
    for a in args:
        if isinstance(a, torch.Tensor):
            key.append(("tensor", a.dtype, tuple(a.shape), str(a.device)))
        else:
            try:
                hash(a)
                key.append(("value", type(a).__name__, a))
            except TypeError:
                key.append(("object", id(a)))
    return tuple(key)


class DsFunction:
    """A torch function run with DS arithmetic (see the module docstring).
    Tensor arguments are captured symbolically; any other argument is baked
    into the capture, so each value gets its own plan."""

    def __init__(self, fn: Callable, graphs: bool = False):
        self.fn = fn
        self.graphs = graphs
        self._plans: Dict[tuple, _Plan] = {}
        self.__doc__ = getattr(fn, "__doc__", None)
        self.__name__ = getattr(fn, "__name__", type(fn).__name__)

    def plan(self, *args) -> _Plan:
        key = _signature_key(args)
        p = self._plans.get(key)
        if p is None:
            if len(self._plans) >= _MAX_PLANS:
                self._plans.clear()  # many baked-in values: start over
            p = self._plans[key] = self._build(args)
        return p

    def _build(self, args) -> _Plan:
        target = self.fn.forward if isinstance(self.fn, torch.nn.Module) else self.fn
        params = [q for q in inspect.signature(target).parameters.values()
                  if q.kind in (q.POSITIONAL_ONLY, q.POSITIONAL_OR_KEYWORD)]
        if len(params) < len(args):
            raise TypeError(f"{self.__name__} takes {len(params)} positional arguments")
        concrete = {q.name: a for q, a in zip(params, args) if not isinstance(a, torch.Tensor)}
        for q in params[len(args):]:
            if q.default is q.empty:
                raise TypeError(f"{self.__name__} needs argument {q.name!r}")
            concrete[q.name] = q.default
        gm = fx.symbolic_trace(self.fn, concrete_args=concrete or None)
        _expand_linear(gm)
        full = list(args) + [concrete[q.name] for q in params[len(args):]]
        _propagate_shapes(gm, full)
        inputs, steps, output, consts = _Lowering(gm, full).lower()
        return _Plan(gm, inputs, steps, output, consts, full[len(args):])

    def __call__(self, *args):
        p = self.plan(*args)
        return p.run_graph(args) if self.graphs else p.run(args)

    def explain(self, *args) -> str:
        """The lowered program for these arguments, one line per step."""
        return self.plan(*args).explain()


_MAX_PLANS = 64


def _expand_linear(gm: fx.GraphModule) -> None:
    """nn.Linear modules and F.linear calls as the operations they are,
    x @ W.T (+ b), which is how a dense layer reaches the pass: a
    dot_general and an add (DsTransformPass.cpp:282-370)."""
    g = gm.graph
    for node in list(g.nodes):
        if node.op == "call_module" and isinstance(gm.get_submodule(node.target), torch.nn.Linear):
            mod = gm.get_submodule(node.target)
            x = node.args[0] if node.args else node.kwargs.get("input")
            with g.inserting_before(node):
                w = g.get_attr(f"{node.target}.weight")
                b = g.get_attr(f"{node.target}.bias") if mod.bias is not None else None
        elif node.op == "call_function" and node.target is torch.nn.functional.linear:
            args = list(node.args) + [None] * (3 - len(node.args))
            x = args[0] if args[0] is not None else node.kwargs.get("input")
            w = args[1] if args[1] is not None else node.kwargs.get("weight")
            b = args[2] if args[2] is not None else node.kwargs.get("bias")
        else:
            continue
        with g.inserting_before(node):
            wt = g.call_function(getattr, (w, "T"))
            y = g.call_function(operator.matmul, (x, wt))
            if b is not None:
                y = g.call_function(operator.add, (y, b))
        node.replace_all_uses_with(y)
        g.erase_node(node)
    g.lint()
    gm.recompile()


def _propagate_shapes(gm: fx.GraphModule, args):
    """dtype and shape of every node, without running the program: with fake
    tensors (module parameters and constants included), else on meta
    tensors; a program that supports neither runs once as it is."""
    from torch.fx.passes.shape_prop import ShapeProp
    try:
        from torch._subclasses.fake_tensor import FakeTensorMode
        ShapeProp(gm, fake_mode=FakeTensorMode(allow_non_fake_inputs=True)).propagate(*args)
        return
    except Exception:
        pass
    meta = [torch.empty_strided(a.shape, a.stride(), dtype=a.dtype, device="meta")
            if isinstance(a, torch.Tensor) else a for a in args]
    try:
        ShapeProp(gm).propagate(*meta)
    except Exception:
        ShapeProp(gm).propagate(*args)


def ds_transform(fn: Optional[Callable] = None, *, graphs: bool = False):
    """Decorator: run `fn` (a function or module of torch tensors) with its
    f64 / f32 arithmetic rewritten to DS, as the reference's DS pass does.
    With graphs=True each plan is captured once as a CUDA graph and
    replayed (one host call per invocation however many launches the plan
    has; results are overwritten by the next call):

        @ds_transform(graphs=True)
        def f(x, y): ...
    """
    if fn is None:
        return lambda f: DsFunction(f, graphs)
    return DsFunction(fn, graphs)
