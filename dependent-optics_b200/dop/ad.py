"""Exact rational reverse-mode AD with an explicit residual (the crate's
src/ad.rs), through libdop's host entry points `dop_ad_*`.

`forward(expr, env) -> (value, tape)` is `ad::forward` (src/ad.rs:76-129);
the tape stores only what the backward map reads (both factors of a
product, the branch a conditional took).  `backward(expr, tape, cot,
env_len)` is `ad::backward` (:131-176) and `stored_scalars(tape)` is
`ad::stored_scalars` (:179-196).  Rationals are `fractions.Fraction`.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from fractions import Fraction

from ._lib import ExprNode, Qc, check, lib

VAR, CONST, NEG, ADD, MUL, LET, IFEQ = range(7)


@dataclass(frozen=True)
class Expr:
    """A node of `ad::Expr` (src/ad.rs:49-59); build with the helpers below."""
    kind: int
    args: tuple = ()
    var: int = 0
    q: Fraction = Fraction(0)


def Var(i: int) -> Expr:
    return Expr(VAR, var=i)


def Const(q) -> Expr:
    return Expr(CONST, q=Fraction(q))


def Neg(e: Expr) -> Expr:
    return Expr(NEG, (e,))


def Add(a: Expr, b: Expr) -> Expr:
    return Expr(ADD, (a, b))


def Mul(a: Expr, b: Expr) -> Expr:
    return Expr(MUL, (a, b))


def Let(bound: Expr, body: Expr) -> Expr:
    """`let x = bound in body`, x at de Bruijn index 0 inside body."""
    return Expr(LET, (bound, body))


def IfEq(c1: Expr, c2: Expr, then: Expr, other: Expr) -> Expr:
    return Expr(IFEQ, (c1, c2, then, other))


def _q(x) -> Qc:
    f = Fraction(x)
    return Qc(f.numerator, f.denominator)


def _flatten(expr: Expr):
    nodes = []

    def go(e: Expr) -> int:
        kids = [go(a) for a in e.args]
        n = ExprNode()
        n.kind = e.kind
        for name, k in zip("abcd", kids):
            setattr(n, name, k)
        n.var = e.var
        n.q = _q(e.q)
        nodes.append(n)
        return len(nodes) - 1

    root = go(expr)
    arr = (ExprNode * len(nodes))(*nodes)
    return arr, len(nodes), root


class Tape:
    """The residual of one forward (owned by libdop)."""

    def __init__(self, handle, flat):
        self._h, self._flat = handle, flat

    def __del__(self):
        try:
            if self._h:
                lib().dop_ad_tape_destroy(self._h)
                self._h = None
        except Exception:
            pass


def forward(expr: Expr, env) -> tuple:
    flat = _flatten(expr)
    arr, n, root = flat
    e = (Qc * max(1, len(env)))(*[_q(v) for v in env])
    val = Qc()
    h = C.c_void_p()
    check(lib().dop_ad_forward(arr, n, root, e, len(env), C.byref(val), C.byref(h)))
    return Fraction(val.n, val.d), Tape(h, flat)


def backward(expr: Expr, tape: Tape, cot, env_len: int) -> list:
    arr, n, root = tape._flat
    out = (Qc * max(1, env_len))()
    check(lib().dop_ad_backward(arr, n, root, tape._h, _q(cot), env_len, out))
    return [Fraction(out[i].n, out[i].d) for i in range(env_len)]


def stored_scalars(tape: Tape) -> list:
    cnt = C.c_int64()
    check(lib().dop_ad_stored_scalars(tape._h, None, 0, C.byref(cnt)))
    out = (Qc * max(1, cnt.value))()
    check(lib().dop_ad_stored_scalars(tape._h, out, cnt.value, C.byref(cnt)))
    return [Fraction(out[i].n, out[i].d) for i in range(cnt.value)]
