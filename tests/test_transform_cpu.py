"""The DS transform of torch programs, on the host.

The lowering (which operations become fused programs, reductions, products,
layout steps or stay torch operations, and where values are recombined)
runs here on CPU tensors with the library's launches replaced by the C
oracle: fused programs are evaluated operation by operation with the
oracle's ds_add / ds_sub / ds_mul (cpp/ds_add.cpp, ds_sub.cpp, ds_mul.cpp
restated), reductions (fused or not) with its sequential DS fold.  The results must equal,
bit for bit, the same DS operations composed by hand, which is what the
reference's pass emits for the program (DsTransformPass.cpp:211-461).
"""
import numpy as np
import pytest
import torch

from conftest import assert_bits_equal
from ds_b200 import _lib, fuse, ops
from ds_b200 import transform as tr


@pytest.fixture
def oracle_backend(monkeypatch, dso):
    """Run every launch of a plan with the oracle on the host."""

    def run_prepared(self, tensors, shape):
        shape = tuple(shape)

        def full(p):
            return np.ascontiguousarray(np.broadcast_to(p, shape + (2,)))
        vals = []
        for code, a, b, v in self.ops:
            if code == _lib.DS_FUSED_INPUT:
                t, k = tensors[a].detach().numpy(), self.kinds[a]
                p = dso.ds_from_f64(t) if k == "f64" else (dso.ds_from_f32(t) if k == "f32" else t)
                vals.append(full(p))
            elif code == _lib.DS_FUSED_CONST:
                vals.append(full(dso.ds_from_f64(np.array(v))))
            elif code == _lib.DS_FUSED_ADD:
                vals.append(dso.ds_add(vals[a], vals[b]))
            elif code == _lib.DS_FUSED_SUB:
                vals.append(dso.ds_sub(vals[a], vals[b]))
            elif code == _lib.DS_FUSED_MUL:
                vals.append(dso.ds_mul(vals[a], vals[b]))
            else:
                vals.append(-vals[a])
        conv = {"f64": dso.ds_to_f64, "f32": dso.ds_to_f32, "packed": lambda x: x}
        return torch.from_numpy(np.array(conv[self.out_kind](vals[-1])))  # keeps 0-d

    def rows(x, dims, rank):
        keep = [d for d in range(rank) if d not in dims]
        moved = np.transpose(x, keep + list(dims) + list(range(rank, x.ndim)))
        out_shape = tuple(x.shape[d] for d in keep)
        return moved.reshape((int(np.prod(out_shape)), -1) + x.shape[rank:]), out_shape

    def reduce_packed(x, init=(0.0, 0.0), dimensions=None, body="add"):
        p = x.detach().numpy()
        rank = p.ndim - 1
        dims = tuple(range(rank)) if dimensions is None else tuple(dimensions)
        r, shape = rows(p, dims, rank)
        res = [dso.ds_reduce_ds_seq(q[:, 0], q[:, 1], body, init) for q in r]
        hi = np.array([h for h, _ in res], np.float32).reshape(shape)
        lo = np.array([l for _, l in res], np.float32).reshape(shape)
        return torch.from_numpy(hi), torch.from_numpy(lo)

    def reduce_from_f64(x, init=0.0, dimensions=None, body="add"):
        p = x.detach().numpy()
        dims = tuple(range(p.ndim)) if dimensions is None else tuple(dimensions)
        r, shape = rows(p, dims, p.ndim)
        res = [dso.ds_reduce_f64_seq(q, body, (init, 0.0)) for q in r]
        hi = np.array([h for h, _ in res], np.float32).reshape(shape)
        lo = np.array([l for _, l in res], np.float32).reshape(shape)
        return torch.from_numpy(hi), torch.from_numpy(lo)

    def dot_f64(a, b, lhs_batch=(), rhs_batch=(), **kw):
        with torch.no_grad():
            return torch.matmul(a, b)

    def reduce_prepared(self, tensors, shape, body="add", init=(0.0, 0.0)):
        flat = run_prepared(self, tensors, shape).numpy().reshape(-1, 2)
        h, l = dso.ds_reduce_ds_seq(flat[:, 0], flat[:, 1], body, init)
        return torch.tensor(h), torch.tensor(l)

    def reduce_rows_prepared(self, tensors, shape, n_reduced, body="add", init=(0.0, 0.0)):
        vals = run_prepared(self, tensors, shape).numpy()
        out_shape = tuple(shape)[:len(shape) - n_reduced]
        rows = vals.reshape((int(np.prod(out_shape)), -1, 2))
        res = [dso.ds_reduce_ds_seq(r[:, 0], r[:, 1], body, init) for r in rows]
        hi = np.array([h for h, _ in res], np.float32).reshape(out_shape)
        lo = np.array([l for _, l in res], np.float32).reshape(out_shape)
        return torch.from_numpy(hi), torch.from_numpy(lo)

    monkeypatch.setattr(fuse.Prepared, "__call__", run_prepared)
    monkeypatch.setattr(fuse.Prepared, "reduce", reduce_prepared)
    monkeypatch.setattr(fuse.Prepared, "reduce_rows", reduce_rows_prepared)
    monkeypatch.setattr(ops, "ds_reduce_packed", reduce_packed)
    monkeypatch.setattr(ops, "ds_reduce_from_f64", reduce_from_f64)
    monkeypatch.setattr(ops, "ds_dot_general_f64", dot_f64)
    return dso


def rand(shape, seed, dtype=torch.float64):
    return torch.from_numpy(np.random.default_rng(seed).uniform(-1, 1, shape)).to(dtype)


def P(dso, t):
    """The DS split of a tensor (emitFromFloat)."""
    a = t.numpy()
    return dso.ds_from_f64(a) if a.dtype == np.float64 else dso.ds_from_f32(a)


def C(dso, v, shape):
    return np.ascontiguousarray(np.broadcast_to(dso.ds_from_f64(np.array(v)), tuple(shape) + (2,)))


# ---- lowering shape ---------------------------------------------------------------------


def test_elementwise_dag_is_one_program():
    @tr.ds_transform
    def f(a, b, c):
        return (a + b) * c - 0.1 * a

    x = torch.zeros(4, 8, dtype=torch.float64)
    plan = f.plan(x, x, x)
    assert plan.launches() == {"fused": 1}
    step = plan.steps[0]
    codes = [o[0] for o in step.prepared.ops]
    assert codes.count(_lib.DS_FUSED_INPUT) == 3      # a is loaded once
    assert codes.count(_lib.DS_FUSED_CONST) == 1
    assert step.prepared.out_kind == "f64"
    assert "ds_fused_run" in f.explain(x, x, x)


def test_reduce_reads_packed_and_dot_reads_f64():
    @tr.ds_transform
    def f(a, b, w):
        y = a * b
        return y.sum(dim=1), y @ w

    x = torch.zeros(4, 8, dtype=torch.float64)
    plan = f.plan(x, x, torch.zeros(8, 3, dtype=torch.float64))
    kinds = [(type(s).__name__, getattr(getattr(s, "prepared", None), "out_kind", None))
             for s in plan.steps]
    # y is read by two non-elementwise consumers: emitted once, packed
    assert kinds[0] == ("_FusedStep", "packed")
    assert ("_ReduceStep", None) in kinds and ("_DotStep", None) in kinds
    assert plan.launches()["fused"] == 3  # y packed, y as f64 for the product, the sum's recombine


def test_long_chains_split_into_programs_within_limits():
    @tr.ds_transform
    def f(x, y):
        for _ in range(400):
            x = x * y + y
        return x

    t = torch.zeros(5, dtype=torch.float32)
    plan = f.plan(t, t)
    assert plan.launches()["fused"] >= 4
    for s in plan.steps:
        assert len(s.prepared.ops) <= 256 and len(s.inputs) <= 16


def test_signature_and_values_make_plans():
    calls = []

    @tr.ds_transform
    def f(x, alpha):
        calls.append(alpha)
        return x * alpha

    x = torch.zeros(3, dtype=torch.float64)
    f.plan(x, 0.5)
    f.plan(x, 0.5)
    f.plan(x, 0.25)
    f.plan(torch.zeros(4, dtype=torch.float64), 0.5)
    assert len(f._plans) == 3


def test_wrong_argument_count():
    f = tr.ds_transform(lambda a, b: a + b)
    with pytest.raises(TypeError):
        f.plan(torch.zeros(2, dtype=torch.float64))


# ---- results equal the hand-composed DS operations ---------------------------------------


def test_elementwise_bits(oracle_backend):
    dso = oracle_backend

    @tr.ds_transform
    def f(a, b, c):
        return (a + b) * c - 0.1 * a, -(a * b) + 3

    a, b, c = rand((6, 7), 1), rand((6, 7), 2), rand((7,), 3)
    got1, got2 = f(a, b, c)
    A, B, Cc = P(dso, a), P(dso, b), P(dso, c.expand(6, 7).contiguous())
    want1 = dso.ds_sub(dso.ds_mul(dso.ds_add(A, B), Cc), dso.ds_mul(C(dso, 0.1, (6, 7)), A))
    want2 = dso.ds_add(-dso.ds_mul(A, B), C(dso, 3.0, (6, 7)))
    assert_bits_equal(got1.numpy(), dso.ds_to_f64(want1), "chain")
    assert_bits_equal(got2.numpy(), dso.ds_to_f64(want2), "neg")


def test_f32_program_has_f32_constants(oracle_backend):
    """In an f32 program the pass sees f32 constants: 0.1 enters as (0.1f, 0)."""
    dso = oracle_backend

    @tr.ds_transform
    def f(x):
        return x * 0.1 + torch.tensor(0.3, dtype=torch.float64) * x

    x = rand((9,), 4, torch.float32)
    got = f(x)
    X = P(dso, x)
    c1 = C(dso, float(np.float32(0.1)), (9,))
    c2 = C(dso, float(np.float32(0.3)), (9,))
    want = dso.ds_add(dso.ds_mul(X, c1), dso.ds_mul(c2, X))
    assert got.dtype == torch.float32
    assert_bits_equal(got.numpy(), dso.ds_to_f32(want), "f32")


def test_add_alpha(oracle_backend):
    dso = oracle_backend

    @tr.ds_transform
    def f(x, y):
        return torch.add(x, y, alpha=2.0), x.sub(y)

    x, y = rand((5,), 5), rand((5,), 6)
    g1, g2 = f(x, y)
    X, Y = P(dso, x), P(dso, y)
    assert_bits_equal(g1.numpy(), dso.ds_to_f64(dso.ds_add(X, dso.ds_mul(Y, C(dso, 2.0, (5,))))))
    assert_bits_equal(g2.numpy(), dso.ds_to_f64(dso.ds_sub(X, Y)))


def test_reduce_bits(oracle_backend):
    dso = oracle_backend

    @tr.ds_transform
    def f(x, y):
        z = x * y - 1.0
        return z.sum(dim=1), torch.sum(z, dim=0, keepdim=True), z.prod(1), z.sum()

    x, y = rand((4, 6), 7), rand((4, 6), 8)
    s1, s0, p1, s = f(x, y)
    Z = dso.ds_sub(dso.ds_mul(P(dso, x), P(dso, y)), C(dso, 1.0, (4, 6)))
    w1 = [dso.ds_reduce_ds_seq(Z[i, :, 0], Z[i, :, 1]) for i in range(4)]
    w0 = [dso.ds_reduce_ds_seq(Z[:, j, 0], Z[:, j, 1]) for j in range(6)]
    wp = [dso.ds_reduce_ds_seq(Z[i, :, 0], Z[i, :, 1], "mul", (1.0, 0.0)) for i in range(4)]
    wa = dso.ds_reduce_ds_seq(Z[..., 0].ravel(), Z[..., 1].ravel())

    def rec(pairs):
        return dso.ds_to_f64(np.array([[h, l] for h, l in pairs], np.float32))
    assert_bits_equal(s1.numpy(), rec(w1), "sum dim 1")
    assert s0.shape == (1, 6)
    assert_bits_equal(s0.numpy().ravel(), rec(w0), "sum dim 0 keepdim")
    assert_bits_equal(p1.numpy(), rec(wp), "prod")
    assert_bits_equal(s.numpy(), rec([wa])[0], "sum all")


def test_reduce_of_argument_splits_on_load(oracle_backend):
    dso = oracle_backend
    f = tr.ds_transform(lambda x: x.sum(dim=-1))
    x = rand((3, 50), 9)
    assert "ds_reduce_from_f64" in f.explain(x)
    got = f(x)
    want = [dso.ds_reduce_f64_seq(x.numpy()[i]) for i in range(3)]
    assert_bits_equal(got.numpy(), dso.ds_to_f64(np.array(want, np.float32)))


def test_layout_moves_hi_and_lo(oracle_backend):
    dso = oracle_backend

    @tr.ds_transform
    def f(a, b):
        y = a * b
        return y.T + a.T, y.reshape(2, -1).sum(dim=1), y.unsqueeze(0).expand(2, 3, 4), y.flatten()

    a, b = rand((3, 4), 10), rand((3, 4), 11)
    g1, g2, g3, g4 = f(a, b)
    Y = dso.ds_mul(P(dso, a), P(dso, b))
    YT = np.ascontiguousarray(Y.transpose(1, 0, 2))
    AT = np.ascontiguousarray(P(dso, a).transpose(1, 0, 2))
    assert_bits_equal(g1.numpy(), dso.ds_to_f64(dso.ds_add(YT, AT)), "transpose")
    Yr = Y.reshape(2, 6, 2)
    w = [dso.ds_reduce_ds_seq(Yr[i, :, 0], Yr[i, :, 1]) for i in range(2)]
    assert_bits_equal(g2.numpy(), dso.ds_to_f64(np.array(w, np.float32)), "reshape")
    assert g3.shape == (2, 3, 4)
    assert_bits_equal(g3.numpy()[1], dso.ds_to_f64(Y), "expand")
    assert_bits_equal(g4.numpy(), dso.ds_to_f64(Y).ravel(), "flatten")


def test_untouched_operations_read_recombined_values(oracle_backend):
    """exp is not a DS operation: it reads the recombined DS value, and its
    result stays f64 (the multiply after it is then not DS either)."""
    dso = oracle_backend

    @tr.ds_transform
    def f(a, b):
        y = a + b
        return torch.exp(y) * b, y

    a, b = rand((8,), 12), rand((8,), 13)
    e, y = f(a, b)
    Y = dso.ds_to_f64(dso.ds_add(P(dso, a), P(dso, b)))
    assert_bits_equal(y.numpy(), Y, "y")
    assert_bits_equal(e.numpy(), (torch.exp(torch.from_numpy(Y)) * b).numpy(), "exp")
    assert f.plan(a, b).launches() == {"fused": 1, "plain": 2}


def test_arguments_return_ds_rounded_and_plain_reads_them_raw(oracle_backend):
    dso = oracle_backend

    @tr.ds_transform
    def f(a):
        return a, torch.sqrt(a * a), a.sqrt()

    a = torch.tensor([1.0 + 2.0 ** -25 + 2.0 ** -52, 2.0, 0.1], dtype=torch.float64)
    r, s, q = f(a)
    assert_bits_equal(r.numpy(), dso.ds_to_f64(P(dso, a)), "return")
    assert r[0].item() == 1.0 + 2.0 ** -25  # lo keeps 24 bits: the 2^-52 bit is dropped
    assert_bits_equal(q.numpy(), torch.sqrt(a).numpy(), "raw read")
    sq = dso.ds_to_f64(dso.ds_mul(P(dso, a), P(dso, a)))
    assert_bits_equal(s.numpy(), np.sqrt(sq), "recombined read")


def test_matmul_shapes(oracle_backend):
    f = tr.ds_transform(lambda a, b: a @ b)
    cases = [((5,), (5,)), ((3, 5), (5,)), ((5,), (5, 4)), ((2, 3, 5), (5, 4)),
             ((2, 3, 5), (2, 5, 4)), ((1, 3, 5), (2, 5, 4))]
    for sa, sb in cases:
        a, b = rand(sa, 14), rand(sb, 15)
        got = f(a, b)
        want = torch.matmul(a, b)
        assert got.shape == want.shape, (sa, sb)
        assert torch.allclose(got, want, rtol=1e-12, atol=1e-12), (sa, sb)


def test_module_parameters_are_ds_constants(oracle_backend):
    dso = oracle_backend

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(rand((6,), 16), requires_grad=False)

        def forward(self, x):
            return (x * self.w + 1.0).sum()

    m = M()
    f = tr.ds_transform(m)
    x = rand((6,), 17)
    got = f(x)
    Z = dso.ds_add(dso.ds_mul(P(dso, x), P(dso, m.w.detach())), C(dso, 1.0, (6,)))
    h, l = dso.ds_reduce_ds_seq(Z[:, 0], Z[:, 1])
    assert_bits_equal(got.numpy(), dso.ds_to_f64(np.array([h, l], np.float32)), "module")


def test_shared_value_emitted_once(oracle_backend):
    dso = oracle_backend

    @tr.ds_transform
    def f(a, b):
        y = a * b
        return y * y, y.sum(), y

    a, b = rand((10,), 18), rand((10,), 19)
    plan = f.plan(a, b)
    muls = [sum(1 for o in s.prepared.ops if o[0] == _lib.DS_FUSED_MUL)
            for s in plan.steps if isinstance(s, tr._FusedStep)]
    assert sum(muls) == 2  # a*b once (packed), then y*y
    g1, g2, g3 = f(a, b)
    Y = dso.ds_mul(P(dso, a), P(dso, b))
    assert_bits_equal(g1.numpy(), dso.ds_to_f64(dso.ds_mul(Y, Y)), "y*y")
    assert_bits_equal(g3.numpy(), dso.ds_to_f64(Y), "y")


def test_integer_and_comparison_operations_stay_torch(oracle_backend):
    @tr.ds_transform
    def f(x, n):
        m = x > 0
        return torch.where(m, x + 1.0, x - 1.0), n * 2

    x = rand((7,), 20)
    n = torch.arange(7)
    got, k = f(x, n)
    assert torch.equal(k, n * 2)
    assert got.dtype == torch.float64 and got.shape == (7,)


def test_full_reduction_of_a_dag_is_one_kernel(oracle_backend):
    dso = oracle_backend

    @tr.ds_transform
    def f(a, b, c):
        return ((a + b) * c).sum(), (a * b).sum(dim=0)

    a, b, c = rand((40, 3), 21), rand((40, 3), 22), rand((3,), 23)
    plan = f.plan(a, b, c)
    kinds = [type(st).__name__ for st in plan.steps]
    assert kinds.count("_FusedReduceStep") == 1      # the full sum, no packed store
    assert kinds.count("_ReduceStep") == 1           # the partial one reads a packed value
    assert "ds_fused_reduce" in f.explain(a, b, c)
    s, p = f(a, b, c)
    Z = dso.ds_mul(dso.ds_add(P(dso, a), P(dso, b)), P(dso, c.expand(40, 3).contiguous()))
    h, l = dso.ds_reduce_ds_seq(Z[..., 0].ravel(), Z[..., 1].ravel())
    assert_bits_equal(s.numpy(), dso.ds_to_f64(np.array([h, l], np.float32)), "fused sum")


def test_reduce_kernels_compile():
    """The generated reduction kernels compile with NVRTC for sm_100a."""
    I, Cn, A, M = (_lib.DS_FUSED_INPUT, _lib.DS_FUSED_CONST, _lib.DS_FUSED_ADD,
                   _lib.DS_FUSED_MUL)
    p = fuse.Prepared([(I, 0, 0, 0.0), (I, 1, 0, 0.0), (A, 0, 1, 0.0), (I, 2, 0, 0.0),
                       (M, 2, 3, 0.0)], ["f64", "f64", "f32"], "packed")
    p.reduce_compile_check([(1000,), (1000,), (1000,)], (1000,), "add")
    p.reduce_compile_check([(10, 1), (1, 7), (7,)], (10, 7), "mul")
    q = fuse.Prepared([(I, 0, 0, 0.0), (Cn, 0, 0, 0.5), (M, 0, 1, 0.0)], ["packed"], "packed")
    q.reduce_compile_check([(33, 2)], (33,), "add")
    with pytest.raises(ValueError):
        q.reduce_compile_check([(33, 2)], (33,), "sub")


def test_linear_layers_lower_to_product_and_add(oracle_backend):
    """nn.Linear and F.linear become x @ W.T + b: a product, then a DS add."""
    dso = oracle_backend

    class Net(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.fc = torch.nn.Linear(6, 4).double()
            self.w2 = torch.nn.Parameter(rand((3, 4), 24), requires_grad=False)

        def forward(self, x):
            h = self.fc(x) * 2.0
            return torch.nn.functional.linear(h, self.w2)

    torch.manual_seed(0)
    net = Net()
    f = tr.ds_transform(net)
    x = rand((5, 6), 25)
    counts = f.plan(x).launches()
    assert counts.get("dot") == 2 and "plain" not in counts
    got = f(x)
    with torch.no_grad():
        h = (x @ net.fc.weight.T)
        H = dso.ds_mul(dso.ds_add(P(dso, h), P(dso, net.fc.bias.expand(5, 4).contiguous())),
                       C(dso, 2.0, (5, 4)))
        want = torch.from_numpy(dso.ds_to_f64(H)) @ net.w2.T
    assert torch.allclose(got, want, rtol=1e-12, atol=1e-12)


def test_default_parameters_are_baked_in(oracle_backend):
    dso = oracle_backend

    def f(x, alpha=2.0):
        return x * alpha

    g = tr.ds_transform(f)
    x = rand((6,), 26)
    assert_bits_equal(g(x).numpy(), dso.ds_to_f64(dso.ds_mul(P(dso, x), C(dso, 2.0, (6,)))), "default")
    assert_bits_equal(g(x, 0.5).numpy(), dso.ds_to_f64(dso.ds_mul(P(dso, x), C(dso, 0.5, (6,)))),
                      "given")


def test_trailing_reduction_of_a_dag_is_one_kernel(oracle_backend):
    """sum over the last dimensions of an elementwise DAG: ds_fused_reduce_rows;
    over leading dimensions it still goes through a packed value."""
    dso = oracle_backend

    @tr.ds_transform
    def f(a, b):
        return (a * b - 1.0).sum(dim=-1), (a + b).sum(dim=(1, 2), keepdim=True), (a * a).sum(dim=0)

    a, b = rand((3, 4, 5), 27), rand((3, 4, 5), 28)
    plan = f.plan(a, b)
    kinds = [type(st).__name__ for st in plan.steps]
    assert kinds.count("_FusedReduceRowsStep") == 2 and kinds.count("_ReduceStep") == 1
    assert "ds_fused_reduce_rows" in f.explain(a, b)
    r1, r2, r0 = f(a, b)
    A, B = P(dso, a), P(dso, b)
    Z = dso.ds_sub(dso.ds_mul(A, B), C(dso, 1.0, (3, 4, 5))).reshape(12, 5, 2)
    want = [dso.ds_reduce_ds_seq(z[:, 0], z[:, 1]) for z in Z]
    assert_bits_equal(r1.numpy(), dso.ds_to_f64(np.array(want, np.float32)).reshape(3, 4), "rows")
    assert r2.shape == (3, 1, 1) and r0.shape == (4, 5)
    Y = dso.ds_add(A, B).reshape(3, 20, 2)
    want2 = [dso.ds_reduce_ds_seq(y[:, 0], y[:, 1]) for y in Y]
    assert_bits_equal(r2.numpy().ravel(), dso.ds_to_f64(np.array(want2, np.float32)), "keepdim")


def test_row_reduce_kernels_compile():
    I, A, M = _lib.DS_FUSED_INPUT, _lib.DS_FUSED_ADD, _lib.DS_FUSED_MUL
    p = fuse.Prepared([(I, 0, 0, 0.0), (I, 1, 0, 0.0), (A, 0, 1, 0.0), (I, 2, 0, 0.0),
                       (M, 2, 3, 0.0)], ["f64", "f64", "f32"], "packed")
    p.reduce_rows_compile_check([(10, 100), (10, 100), (100,)], (10, 100), 1, "add")
    p.reduce_rows_compile_check([(4, 5, 6), (4, 5, 6), (6,)], (4, 5, 6), 2, "mul")
    with pytest.raises(_lib.DsInvalidArgument):
        p.reduce_rows_compile_check([(10, 100), (10, 100), (100,)], (10, 100), 3, "add")
