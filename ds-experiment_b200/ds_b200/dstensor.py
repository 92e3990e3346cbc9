"""Double-single tensors that keep their (hi, lo) pairs between calls.

The reference recombines to f64 (or f32) at every module boundary
(DsTransformPass.cpp:451-461, `emitToFloat` before `func.return`), so a value
that crosses a jit boundary loses its lo word unless it is f64 there
(README.md:493-498).  A `DSTensor` keeps the packed wire format `[..., 2]`
f32 (hi, lo) of the `ds_*` targets as its storage, so a DS value can be
stored, passed around and computed with again without a round trip through
f64.

Elementwise arithmetic is lazy: `+`, `-`, `*` and unary `-` on DSTensors,
torch f64/f32 tensors and Python numbers build an expression, and the
expression runs as ONE generated kernel (`ds_b200.fuse`) when the value is
needed -- `packed`, `to_f64()`, `to_f32()`, `sum()`, `matmul()` -- with the
same DS operations, in the same order, as one target call per operation.

    a = DSTensor.from_f64(x)
    b = (a + y) * a - 0.1          # nothing runs yet
    s = b.sum()                    # one fused kernel, then one packed reduce
    c = b.to_f64()
"""
from __future__ import annotations

from typing import Dict, List, Tuple, Union

import torch

from . import _lib, fuse, ops

Number = Union[int, float]

# An expression node: ("leaf", key) | ("const", value) | (code, a, b) | ("neg", a)
_MAX_OPS = 200  # an expression this large is materialised before it grows
_MAX_INPUTS = 16  # distinct tensors one generated program reads


class DSTensor:
    """A DS tensor: packed `[..., 2]` f32 storage, or a pending expression."""

    __slots__ = ("_packed", "_expr", "_leaves", "_shape", "_device", "_n_ops")

    def __init__(self, packed: torch.Tensor):
        if packed.dtype != torch.float32 or packed.dim() == 0 or packed.shape[-1] != 2:
            raise ValueError("DSTensor storage is float32 with last dim == 2")
        if not packed.is_cuda:
            raise ValueError("DSTensor storage must be a CUDA tensor")
        self._packed = packed.contiguous()
        self._expr = None
        self._leaves: Dict[int, Tuple[str, torch.Tensor]] = {}
        self._shape = tuple(packed.shape[:-1])
        self._device = packed.device
        self._n_ops = 0

    # ---- construction -----------------------------------------------------

    @staticmethod
    def from_f64(t: torch.Tensor) -> "DSTensor":
        """emitFromFloat of an f64 tensor: hi = (float)x, lo = (float)(x - hi)."""
        return DSTensor(ops.ds_from_f64(t.contiguous()))

    @staticmethod
    def from_f32(t: torch.Tensor) -> "DSTensor":
        """An f32 tensor as (v, 0)."""
        return DSTensor(ops.ds_from_f32(t.contiguous()))

    @classmethod
    def _lazy(cls, expr, leaves, shape, device, n_ops) -> "DSTensor":
        obj = cls.__new__(cls)
        obj._packed = None
        obj._expr = expr
        obj._leaves = leaves
        obj._shape = shape
        obj._device = device
        obj._n_ops = n_ops
        return obj

    @property
    def shape(self) -> Tuple[int, ...]:
        return self._shape

    @property
    def device(self) -> torch.device:
        return self._device

    def __repr__(self):
        state = "materialised" if self._packed is not None else f"pending ({self._n_ops} ops)"
        return f"DSTensor(shape={self._shape}, device={self._device}, {state})"

    # ---- lazy elementwise arithmetic --------------------------------------

    def _operand(self):
        if self._packed is not None:
            key = id(self._packed)
            return ("leaf", key), {key: ("packed", self._packed)}, self._shape, 0
        return self._expr, self._leaves, self._shape, self._n_ops

    def _bin(self, code, other, swap=False):
        o = _as_operand(other, self._device)
        if o is NotImplemented:
            return NotImplemented
        a = self._operand()
        if swap:
            a, o = o, a
        if a[3] + o[3] + 1 > _MAX_OPS or len(set(a[1]) | set(o[1])) > _MAX_INPUTS:
            # keep generated programs within the target's limits
            a = _force(a, self._device)
            o = _force(o, self._device)
        leaves = dict(a[1])
        leaves.update(o[1])
        try:
            shape = tuple(torch.broadcast_shapes(a[2], o[2]))
        except RuntimeError as e:
            raise ValueError(f"DSTensor shapes do not broadcast: {e}") from None
        return DSTensor._lazy((code, a[0], o[0]), leaves, shape, self._device, a[3] + o[3] + 1)

    def __add__(self, o):
        return self._bin(_lib.DS_FUSED_ADD, o)

    def __radd__(self, o):
        return self._bin(_lib.DS_FUSED_ADD, o, swap=True)

    def __sub__(self, o):
        return self._bin(_lib.DS_FUSED_SUB, o)

    def __rsub__(self, o):
        return self._bin(_lib.DS_FUSED_SUB, o, swap=True)

    def __mul__(self, o):
        return self._bin(_lib.DS_FUSED_MUL, o)

    def __rmul__(self, o):
        return self._bin(_lib.DS_FUSED_MUL, o, swap=True)

    def __neg__(self):
        e, leaves, shape, n = self._operand()
        return DSTensor._lazy(("neg", e), dict(leaves), shape, self._device, n + 1)

    # ---- materialisation ---------------------------------------------------

    @property
    def packed(self) -> torch.Tensor:
        """The packed (hi, lo) storage, running the pending expression."""
        if self._packed is None:
            self._packed = _run(self._expr, self._leaves, self._shape, self._device, "packed")
            self._expr, self._leaves, self._n_ops = None, {}, 0
        return self._packed

    def materialize(self) -> "DSTensor":
        self.packed
        return self

    def to_f64(self) -> torch.Tensor:
        """(double)hi + (double)lo; a pending expression recombines in its kernel."""
        if self._packed is not None:
            return ops.ds_to_f64(self._packed)
        return _run(self._expr, self._leaves, self._shape, self._device, "f64")

    def to_f32(self) -> torch.Tensor:
        """hi + lo in f32, as ds_to_f32."""
        if self._packed is not None:
            return ops.ds_to_f32(self._packed)
        return _run(self._expr, self._leaves, self._shape, self._device, "f32")

    # ---- reduce and contraction ---------------------------------------------

    def sum(self, dimensions=None) -> "DSTensor":
        """DS sum over `dimensions` (default: all), the result kept as DS.
        A pending expression summed over all its dimensions, or over its
        trailing ones, runs as one kernel that never stores its values
        (ds_fused_reduce, ds_fused_reduce_rows)."""
        rank = len(self._shape)
        if self._packed is None and dimensions is None and rank > 0:
            prepared, tensors = _prepare(self._expr, self._leaves, "packed")
            hi, lo = prepared.reduce(tensors, self._shape, "add")
            return DSTensor(torch.stack([hi, lo], dim=-1))
        dims = None if dimensions is None else tuple(sorted({int(d) % max(rank, 1)
                                                              for d in dimensions}))
        if self._packed is None and dims and 0 < len(dims) < rank and \
                dims == tuple(range(rank - len(dims), rank)):
            # the trailing dimensions of a pending expression: one kernel per row
            prepared, tensors = _prepare(self._expr, self._leaves, "packed")
            hi, lo = prepared.reduce_rows(tensors, self._shape, len(dims), "add")
            return DSTensor(torch.stack([hi, lo], dim=-1))
        p = self.packed
        hi, lo = ops.ds_reduce_packed(p, dimensions=dims)
        return DSTensor(torch.stack([hi, lo], dim=-1))

    def matmul(self, other: "DSTensor") -> "DSTensor":
        """A @ B in DS arithmetic (the tensor-core dot_general).  The operands
        enter as hi + lo in f64, which is exact for a DS pair."""
        if not isinstance(other, DSTensor):
            raise TypeError("matmul takes a DSTensor")
        return DSTensor.from_f64(ops.ds_matmul_f64(self.to_f64(), other.to_f64()))

    __matmul__ = matmul


def _as_operand(x, device):
    if isinstance(x, DSTensor):
        return x._operand()
    if isinstance(x, torch.Tensor):
        if x.dtype not in (torch.float64, torch.float32):
            raise TypeError(f"DSTensor arithmetic takes float64/float32 tensors, got {x.dtype}")
        if x.device != device:
            raise ValueError("operands must be on one device")
        x = x.contiguous()
        kind = "f64" if x.dtype == torch.float64 else "f32"
        return ("leaf", id(x)), {id(x): (kind, x)}, tuple(x.shape), 0
    if isinstance(x, (int, float)) and not isinstance(x, bool):
        return ("const", float(x)), {}, (), 1
    return NotImplemented


def _force(operand, device):
    """The operand with a pending expression run into packed storage."""
    if operand[0][0] in ("leaf", "const"):
        return operand  # already a leaf or a constant
    expr, leaves, shape, _ = operand
    return DSTensor(_run(expr, leaves, shape, device, "packed"))._operand()


def _run(expr, leaves, shape, device, out_kind) -> torch.Tensor:
    """Emit the expression as a fused program over its leaves and run it."""
    prog, inputs = _emit(expr, leaves)
    return fuse.run_program(prog, inputs, out_kind, shape)


def _prepare(expr, leaves, out_kind):
    prog, inputs = _emit(expr, leaves)
    return fuse.Prepared(prog, [k for k, _ in inputs], out_kind), [t for _, t in inputs]


def _emit(expr, leaves):
    """The expression as an operation list over its distinct leaves:
    (ops, [(kind, tensor)])."""
    prog: List[Tuple[int, int, int, float]] = []
    inputs: List[Tuple[str, torch.Tensor]] = []
    input_of: Dict[int, int] = {}
    memo: Dict[int, int] = {}

    def emit(node) -> int:
        # leaves are emitted once per tensor, other nodes once per node
        nid = ("leaf", node[1]) if node[0] == "leaf" else id(node)
        if nid in memo:
            return memo[nid]
        tag = node[0]
        if tag == "leaf":
            key = node[1]
            if key not in input_of:
                input_of[key] = len(inputs)
                inputs.append(leaves[key])
            prog.append((_lib.DS_FUSED_INPUT, input_of[key], 0, 0.0))
        elif tag == "const":
            prog.append((_lib.DS_FUSED_CONST, 0, 0, node[1]))
        elif tag == "neg":
            a = emit(node[1])
            prog.append((_lib.DS_FUSED_NEG, a, 0, 0.0))
        else:
            a = emit(node[1])
            b = emit(node[2])
            prog.append((tag, a, b, 0.0))
        memo[nid] = len(prog) - 1
        return memo[nid]

    emit(expr)
    if not inputs:
        raise ValueError("a DSTensor expression needs at least one tensor")
    return prog, inputs
