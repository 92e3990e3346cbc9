"""DSTensor expression building on the host: the lazy arithmetic turns into
one fused operation list, shared subexpressions and repeated tensors are
emitted once, and Python numbers become constants."""
import torch

from ds_b200 import _lib, fuse
from ds_b200 import dstensor as dst


def leaf(t, kind):
    return dst.DSTensor._lazy(("leaf", id(t)), {id(t): (kind, t)}, tuple(t.shape), t.device, 0)


def test_expression_becomes_one_program(monkeypatch):
    seen = {}

    def fake_run(prog, inputs, out_kind, shape):
        seen.update(prog=prog, inputs=inputs, out_kind=out_kind, shape=shape)
        return torch.zeros(tuple(shape) + ((2,) if out_kind == "packed" else ()))

    monkeypatch.setattr(fuse, "run_program", fake_run)
    x = torch.zeros(3, 4, dtype=torch.float64)
    y = torch.zeros(4, dtype=torch.float32)
    a = leaf(x, "f64")
    b = (a + y) * a - 0.5
    assert b.shape == (3, 4)
    b.to_f64()
    codes = [op[0] for op in seen["prog"]]
    assert codes == [_lib.DS_FUSED_INPUT, _lib.DS_FUSED_INPUT, _lib.DS_FUSED_ADD,
                     _lib.DS_FUSED_MUL, _lib.DS_FUSED_CONST, _lib.DS_FUSED_SUB]
    # x appears twice in the expression but is loaded once
    assert [k for k, _ in seen["inputs"]] == ["f64", "f32"]
    assert seen["prog"][3][1:3] == (2, 0) and seen["prog"][4][3] == 0.5
    assert seen["out_kind"] == "f64" and seen["shape"] == (3, 4)


def test_shared_subexpression_emitted_once(monkeypatch):
    seen = {}
    monkeypatch.setattr(fuse, "run_program",
                        lambda prog, inputs, out_kind, shape: seen.setdefault("prog", prog) and
                        torch.zeros(tuple(shape) + (2,)))
    x = torch.zeros(5, dtype=torch.float64)
    a = leaf(x, "f64")
    s = a * a
    (s + s).packed
    muls = [op for op in seen["prog"] if op[0] == _lib.DS_FUSED_MUL]
    assert len(muls) == 1


def test_bad_broadcast_raises():
    a = leaf(torch.zeros(3, 4, dtype=torch.float64), "f64")
    try:
        a + torch.zeros(3, dtype=torch.float64)
    except ValueError:
        return
    raise AssertionError("expected a broadcast error")
