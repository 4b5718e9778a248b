"""Scalar AD lenses (src/ad.rs) and GF(2) linear maps (src/vect.rs) through
libdop's host entry points.  These are the crate's own tests, restated:
residual contents (src/ad.rs:273-320), cotangents against forward-mode dual
numbers over a catalogue of expressions at every point of {-2..2}^arity
(:322-372), and the linear-category / Kronecker laws (src/vect.rs:137-155).
Both are exact (rationals, bits), so the checks are equalities.  Host code
only: no GPU is touched.
"""
from fractions import Fraction

import pytest

from dop import DopError
from dop import ad, vect
from dop.ad import IfEq, Let, Mul, Neg, Var, Const
from dop.ad import Add as AddE


# -------------------------------------------------- forward-mode reference
def dual_eval(e, env):
    """Value and derivative of e at env, env a list of (value, tangent)."""
    k = e.kind
    if k == ad.VAR:
        return env[e.var]
    if k == ad.CONST:
        return (e.q, Fraction(0))
    if k == ad.NEG:
        v, t = dual_eval(e.args[0], env)
        return (-v, -t)
    if k == ad.ADD:
        (a, da), (b, db) = dual_eval(e.args[0], env), dual_eval(e.args[1], env)
        return (a + b, da + db)
    if k == ad.MUL:
        (a, da), (b, db) = dual_eval(e.args[0], env), dual_eval(e.args[1], env)
        return (a * b, a * db + da * b)
    if k == ad.LET:
        bound = dual_eval(e.args[0], env)
        return dual_eval(e.args[1], [bound] + list(env))
    if k == ad.IFEQ:
        v1, v2 = dual_eval(e.args[0], env)[0], dual_eval(e.args[1], env)[0]
        return dual_eval(e.args[2] if v1 == v2 else e.args[3], env)
    raise AssertionError(k)


def catalogue():
    x, y = Var(0), Var(1)
    return [
        (AddE(Mul(x, x), y), 2),
        (Let(Mul(Var(0), Var(1)), AddE(Var(0), Var(0))), 2),
        (Var(0), 2),
        (IfEq(x, Const(0), y, Mul(x, y)), 2),
        (AddE(x, y), 2),
        (Mul(x, y), 2),
        (Neg(x), 1),
    ]


def test_residuals_store_only_what_the_backward_pass_reads():
    env = [3, 4]
    x, y = Var(0), Var(1)
    assert ad.stored_scalars(ad.forward(AddE(x, y), env)[1]) == []
    assert ad.stored_scalars(ad.forward(Neg(x), env)[1]) == []
    assert ad.stored_scalars(ad.forward(Mul(x, y), env)[1]) == [3, 4]
    assert ad.stored_scalars(ad.forward(x, env)[1]) == []
    # the taken branch is a projection: nothing stored
    then = IfEq(x, Const(3), y, Mul(x, y))
    assert ad.stored_scalars(ad.forward(then, env)[1]) == []
    other = IfEq(x, Const(0), y, Mul(x, y))
    assert ad.stored_scalars(ad.forward(other, env)[1]) == [3, 4]


def test_cotangents_match_dual_numbers():
    coords = [-2, -1, 0, 1, 2]
    for expr, arity in catalogue():
        points = [[a] for a in coords] if arity == 1 else [[a, b] for a in coords for b in coords]
        for point in points:
            for d in range(arity):
                dual = [(Fraction(v), Fraction(1 if i == d else 0)) for i, v in enumerate(point)]
                value, tangent = dual_eval(expr, dual)
                got, tape = ad.forward(expr, point)
                assert got == value
                cot = ad.backward(expr, tape, 1, arity)
                assert cot[d] == tangent, (expr, point, d)
                # the put is a function of the residual and the cotangent alone
                assert ad.backward(expr, tape, 1, arity) == cot


def test_rational_values_and_errors():
    half = Fraction(1, 2)
    v, tape = ad.forward(Mul(Var(0), AddE(Var(0), Const(Fraction(1, 3)))), [half])
    assert v == half * (half + Fraction(1, 3))
    assert ad.backward(Mul(Var(0), AddE(Var(0), Const(Fraction(1, 3)))), tape, 2, 1) == \
        [2 * (2 * half + Fraction(1, 3))]
    with pytest.raises(DopError):
        ad.forward(Var(3), [1])  # variable outside the environment
    with pytest.raises(DopError):
        ad.forward(Mul(Var(0), Var(0)), [Fraction(2 ** 40)])  # i64 overflow


def test_linear_category_and_tensor():
    for n in range(3):
        idn = vect.identity(n)
        for f in vect.all_maps(n, n):
            assert vect.compose(idn, f) == f
            assert vect.compose(f, idn) == f
            assert vect.add(f, f) == vect.zero(n, n)
            assert vect.compose(vect.transpose(vect.transpose(f)), vect.identity(n)) == f
    for a in range(2):
        for b in range(2):
            for f in vect.all_maps(a, a):
                for g in vect.all_maps(b, b):
                    t = vect.kronecker(f, g)
                    assert (t.dom, t.cod) == (a * b, a * b)
            assert vect.kronecker(vect.identity(a), vect.identity(b)) == vect.identity(a * b)


def test_transpose_is_the_adjoint():
    """<f x, y> = <x, f^T y> over GF(2), every map 2 -> 3 and every x, y."""
    def dot(u, v):
        return bin(u & v).count("1") & 1
    for f in vect.all_maps(2, 3):
        ft = vect.transpose(f)
        for xv in range(4):
            for yv in range(8):
                assert dot(f.apply_vec(xv), yv) == dot(xv, ft.apply_vec(yv))


def test_lin_shape_errors():
    with pytest.raises(DopError):
        vect.compose(vect.identity(2), vect.identity(3))
    with pytest.raises(DopError):
        vect.kronecker(vect.identity(6), vect.identity(6))  # 36 > 32 dimensions
    assert len(vect.all_maps(2, 2)) == 16 and len(vect.all_maps(0, 3)) == 1
