"""GF(2) linear maps (the crate's src/vect.rs) through libdop's host entry
points `dop_lin_*`.  A map stores the image of each basis vector as a bitset
(`columns[j]`); `transpose` is the adjoint of a linear map."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from ._lib import LinC, check, lib


@dataclass(frozen=True)
class Lin:
    dom: int
    cod: int
    columns: tuple

    def _c(self) -> LinC:
        c = LinC()
        c.dom, c.cod = self.dom, self.cod
        for j, col in enumerate(self.columns):
            c.columns[j] = col
        return c

    @staticmethod
    def _of(c: LinC) -> "Lin":
        return Lin(c.dom, c.cod, tuple(c.columns[j] for j in range(c.dom)))

    def apply_vec(self, v: int) -> int:
        return lib().dop_lin_apply(C.byref(self._c()), v)


def _call(fn, *args) -> Lin:
    out = LinC()
    check(fn(*args, C.byref(out)))
    return Lin._of(out)


def zero(dom: int, cod: int) -> Lin:
    return _call(lib().dop_lin_zero, dom, cod)


def identity(n: int) -> Lin:
    return _call(lib().dop_lin_identity, n)


def compose(g: Lin, f: Lin) -> Lin:
    """g after f."""
    return _call(lib().dop_lin_compose, C.byref(g._c()), C.byref(f._c()))


def add(f: Lin, g: Lin) -> Lin:
    return _call(lib().dop_lin_add, C.byref(f._c()), C.byref(g._c()))


def transpose(f: Lin) -> Lin:
    return _call(lib().dop_lin_transpose, C.byref(f._c()))


def kronecker(f: Lin, g: Lin) -> Lin:
    return _call(lib().dop_lin_kronecker, C.byref(f._c()), C.byref(g._c()))


def all_maps(dom: int, cod: int) -> list:
    """Every map dom -> cod, in the crate's enumeration order (`vect::all`)."""
    n = C.c_int64()
    check(lib().dop_lin_all(dom, cod, None, 0, C.byref(n)))
    out = (LinC * max(1, n.value))()
    check(lib().dop_lin_all(dom, cod, out, n.value, C.byref(n)))
    return [Lin._of(out[i]) for i in range(n.value)]
