"""Sheaf-program lowering stand-in: the producer of the backend's input format.

Sheaf (Rust) lowers a value-and-grad call in four steps: ANF conversion of the
inlined body, reverse-mode AD over the ANF bindings, simplification, and
emission of StableHLO text.  None of that runs in this environment (no Rust
toolchain), yet the backend consumes exactly that text.  This module restates
those steps in Python so that tests and the benchmark can produce modules of
the same form:

* ANF bindings of Sheaf builtin calls          (sheaf/src/autodiff/reverse.rs:52-161)
* reverse-mode rules, one per builtin          (sheaf/src/autodiff/reverse.rs:513-1075)
* `simplify` of each backward binding          (sheaf/src/autodiff/mod.rs:139-178)
* builtin codegen (sum/mean/var/where/...)     (sheaf/src/lowering/codegen/*.rs)
* StableHLO text emission, line for line       (sheaf/src/lowering/stablehlo/*.rs)
* value-and-grad assembly + `reduce_broadcast_grad`
                                               (sheaf/src/runtime/jit/vag.rs:611-647,
                                                sheaf/src/lowering/codegen/autodiff.rs:147)

The backend never imports this module; it is the caller's side of the
boundary.  Known deviation: scalar config captures (`n_embd`, ...) are baked as
literals, which is what Sheaf does for scalars that reach shape positions
(sheaf/src/runtime/jit/vag.rs:132-180, 357-359).
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np


# ---------------------------------------------------------------------------
# Sheaf expression atoms
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class Sym:
    name: str


@dataclass(frozen=True)
class Kw:
    name: str


@dataclass(frozen=True)
class Vec:
    items: tuple

    def __init__(self, items):
        object.__setattr__(self, "items", tuple(items))


@dataclass
class Call:
    fn: str
    args: list


def _is_float(a):
    return isinstance(a, float)


def _is_int(a):
    return isinstance(a, int) and not isinstance(a, bool)


# ---------------------------------------------------------------------------
# Types and number formatting (sheaf/src/lowering/stablehlo/mod.rs:136-160,
# constants.rs:10-27,121-145)
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class Ty:
    shape: tuple
    dtype: str = "f32"

    def mlir(self) -> str:
        if not self.shape:
            return f"tensor<{self.dtype}>"
        return "tensor<" + "x".join(str(d) for d in self.shape) + f"x{self.dtype}>"


SCALAR = Ty((), "f32")


def fmt_f64(v: float) -> str:
    """Rust `{:.1}` for integral finite values, else Rust `{}` (never exponent)."""
    v = float(v)
    if math.isfinite(v) and v == math.floor(v):
        return "%.1f" % v
    return np.format_float_positional(v, unique=True, trim="-")


def _dense_attr(data, shape, dim=0):
    if dim == len(shape) - 1:
        return "[" + ", ".join(fmt_f64(x) for x in data[: shape[dim]]) + "]"
    stride = int(np.prod(shape[dim + 1:]))
    return "[" + ", ".join(_dense_attr(data[i * stride:], shape, dim + 1)
                           for i in range(shape[dim])) + "]"


# ---------------------------------------------------------------------------
# StableHLO emitter (mirrors StableHLOEmitter's text forms)
# ---------------------------------------------------------------------------

class Emitter:
    def __init__(self):
        self.counter = 0
        self.body: List[str] = []
        self.known: Dict[str, float] = {}
        self.mean_cache: Dict[tuple, tuple] = {}

    def fresh(self) -> str:
        r = f"%{self.counter}"
        self.counter += 1
        return r

    def line(self, s: str):
        self.body.append(s)

    # constants ------------------------------------------------------------
    def constant_f32(self, v: float) -> str:
        r = self.fresh()
        self.line(f"    {r} = stablehlo.constant dense<{fmt_f64(v)}> : tensor<f32>")
        self.known[r] = float(v)
        return r

    def nd_constant(self, data, shape) -> Tuple[str, Ty]:
        r = self.fresh()
        ty = Ty(tuple(shape))
        vals = fmt_f64(data[0]) if not shape else _dense_attr(list(data), list(shape))
        self.line(f"    {r} = stablehlo.constant dense<{vals}> : {ty.mlir()}")
        return r, ty

    def splat(self, value: float, shape) -> Tuple[str, Ty]:
        r = self.fresh()
        ty = Ty(tuple(shape))
        self.line(f"    {r} = stablehlo.constant dense<{fmt_f64(value)}> : {ty.mlir()}")
        return r, ty

    def raw_constant(self, text: str) -> str:
        r = self.fresh()
        self.line(f"    {r} = stablehlo.constant dense<{text}> : tensor<f32>")
        return r

    # broadcasting (broadcast.rs) -----------------------------------------
    @staticmethod
    def broadcast_types(lt: Ty, rt: Ty) -> Ty:
        if not lt.shape and not rt.shape:
            return lt
        if not lt.shape:
            return rt
        if not rt.shape:
            return lt
        dt = "bf16" if (lt.dtype == "bf16" and rt.dtype == "bf16") else "f32"
        n = max(len(lt.shape), len(rt.shape))
        ls = (1,) * (n - len(lt.shape)) + lt.shape
        rs = (1,) * (n - len(rt.shape)) + rt.shape
        return Ty(tuple(max(a, b) for a, b in zip(ls, rs)), dt)

    def broadcast(self, x: str, ft: Ty, tt: Ty) -> str:
        fs, ts = ft.shape, tt.shape
        if not fs:
            dims = []
        else:
            off = len(ts) - len(fs)
            ra = list(range(off, len(ts)))
            if all(s == ts[ra[i]] or s == 1 for i, s in enumerate(fs)):
                dims = ra
            else:
                mapping, start = [], 0
                for s in fs:
                    for j in range(start, len(ts)):
                        if ts[j] == s or s == 1:
                            mapping.append(j)
                            start = j + 1
                            break
                dims = mapping if len(mapping) == len(fs) else ra
        r = self.fresh()
        self.line(f"    {r} = stablehlo.broadcast_in_dim {x}, dims = [{', '.join(map(str, dims))}]"
                  f" : ({ft.mlir()}) -> {tt.mlir()}")
        return r

    def maybe_broadcast(self, a, b, at, bt, rt):
        if at.shape != rt.shape and rt.shape:
            a = self.broadcast(a, at, rt)
        if bt.shape != rt.shape and rt.shape:
            b = self.broadcast(b, bt, rt)
        return a, b

    # elementwise (operations.rs) -----------------------------------------
    BINOPS = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide", "**": "power",
              "min": "minimum", "max": "maximum"}
    UNOPS = {"tanh": "tanh", "sqrt": "sqrt", "exp": "exponential", "log": "log", "not": "not",
             "abs": "abs", "neg": "negate", "sin": "sine", "cos": "cosine"}

    def binop(self, op, a, b, at, bt):
        rt = self.broadcast_types(at, bt)
        a2, b2 = self.maybe_broadcast(a, b, at, bt, rt)
        r = self.fresh()
        self.line(f"    {r} = stablehlo.{self.BINOPS[op]} {a2}, {b2} : {rt.mlir()}")
        if a2 in self.known and b2 in self.known:
            lv, rv = self.known[a2], self.known[b2]
            res = {"+": lv + rv, "-": lv - rv, "*": lv * rv,
                   "min": min(lv, rv), "max": max(lv, rv)}.get(op)
            if op == "/" and rv != 0:
                res = lv / rv
            if res is not None:
                self.known[r] = res
        return r, rt

    def unary(self, op, a, at) -> str:
        r = self.fresh()
        self.line(f"    {r} = stablehlo.{self.UNOPS[op]} {a} : {at.mlir()}")
        return r

    def raw_unary(self, opname, a, at) -> str:
        r = self.fresh()
        self.line(f"    {r} = stablehlo.{opname} {a} : {at.mlir()}")
        return r

    def raw_binary(self, opname, a, b, t) -> str:
        r = self.fresh()
        self.line(f"    {r} = stablehlo.{opname} {a}, {b} : {t.mlir()}")
        return r

    def convert(self, a, ft: Ty, tt: Ty) -> str:
        r = self.fresh()
        self.line(f"    {r} = stablehlo.convert {a} : ({ft.mlir()}) -> {tt.mlir()}")
        return r

    # reductions (reduce_ops.rs) ------------------------------------------
    @staticmethod
    def _axis(shape, axis):
        nd = len(shape)
        ax = nd + axis if axis < 0 else axis
        return min(ax, max(nd - 1, 0))

    def _reduce(self, kind, x, t: Ty, axis, keepdims, init):
        if not t.shape:
            return x, t
        ax = self._axis(t.shape, axis)
        red = tuple(d for i, d in enumerate(t.shape) if i != ax)
        rt = Ty(red) if red else SCALAR
        r = self.fresh()
        self.line(f"    {r} = stablehlo.reduce({x} init: {init}) applies stablehlo.{kind} across "
                  f"dimensions = [{ax}] : ({t.mlir()}, tensor<f32>) -> {rt.mlir()}")
        if keepdims:
            ks = list(t.shape)
            ks[ax] = 1
            kt = Ty(tuple(ks))
            k = self.fresh()
            self.line(f"    {k} = stablehlo.reshape {r} : ({rt.mlir()}) -> {kt.mlir()}")
            return k, kt
        return r, rt

    def reduce_sum(self, x, t, axis, keepdims):
        if not t.shape:
            return x, t
        z = self.constant_f32(0.0)
        return self._reduce("add", x, t, axis, keepdims, z)

    def reduce_max(self, x, t, axis, keepdims):
        if not t.shape:
            return x, t
        init = self.raw_constant("0xFF800000")
        return self._reduce("maximum", x, t, axis, keepdims, init)

    def reduce_min(self, x, t, axis, keepdims):
        if not t.shape:
            return x, t
        init = self.raw_constant("0x7F800000")
        return self._reduce("minimum", x, t, axis, keepdims, init)

    def reduce_mean(self, x, t, axis, keepdims):
        if not t.shape:
            return x, t
        nd = len(t.shape)
        ax = nd + axis if axis < 0 else axis
        key = (x, ax, keepdims)
        if key in self.mean_cache:
            return self.mean_cache[key]
        n = float(t.shape[ax])
        s, st = self.reduce_sum(x, t, axis, keepdims)
        nr = self.constant_f32(n)
        r = self.fresh()
        if st == SCALAR:
            self.line(f"    {r} = stablehlo.divide {s}, {nr} : {st.mlir()}")
        else:
            b = self.fresh()
            self.line(f"    {b} = stablehlo.broadcast_in_dim {nr}, dims = [] : (tensor<f32>) -> {st.mlir()}")
            self.line(f"    {r} = stablehlo.divide {s}, {b} : {st.mlir()}")
        self.mean_cache[key] = (r, st)
        return r, st

    # shapes (shape_ops.rs) -----------------------------------------------
    def reshape(self, x, t: Ty, shape) -> Tuple[str, Ty]:
        r = self.fresh()
        rt = Ty(tuple(shape), t.dtype)
        self.line(f"    {r} = stablehlo.reshape {x} : ({t.mlir()}) -> {rt.mlir()}")
        return r, rt

    def transpose(self, x, t: Ty, perm) -> Tuple[str, Ty]:
        if len(t.shape) <= 1:
            return x, t
        rt = Ty(tuple(t.shape[p] for p in perm))
        r = self.fresh()
        self.line(f"    {r} = stablehlo.transpose {x}, dims = [{', '.join(map(str, perm))}]"
                  f" : ({t.mlir()}) -> {rt.mlir()}")
        return r, rt

    def iota(self, shape, dim) -> Tuple[str, Ty]:
        r = self.fresh()
        t = Ty(tuple(shape))
        self.line(f"    {r} = stablehlo.iota dim = {dim} : {t.mlir()}")
        return r, t

    def slice_axis(self, x, t: Ty, start, end, axis) -> Tuple[str, Ty]:
        nd = len(t.shape)
        st = [0] * nd
        lim = list(t.shape)
        st[axis], lim[axis] = start, end
        dims = ", ".join(f"{s}:{l}:1" for s, l in zip(st, lim))
        shp = list(t.shape)
        shp[axis] = end - start
        rt = Ty(tuple(shp), t.dtype)
        r = self.fresh()
        self.line(f"    {r} = stablehlo.slice {x} [{dims}] : ({t.mlir()}) -> {rt.mlir()}")
        return r, rt

    # compare / select (compare_ops.rs) -----------------------------------
    def compare(self, op, a, b, at, bt):
        ot = self.broadcast_types(at, bt)
        a, b = self.maybe_broadcast(a, b, at, bt, ot)
        T = ot.mlir()
        zero = self.constant_f32(0.0)
        zero_bc = self.broadcast(zero, SCALAR, ot)
        one = self.constant_f32(1.0)
        one_bc = self.broadcast(one, SCALAR, ot)
        if op in (">=", ">", "<=", "<"):
            first, second = (a, b) if op in (">=", ">") else (b, a)
            d = self.fresh()
            self.line(f"    {d} = stablehlo.subtract {first}, {second} : {T}")
            sg = self.fresh()
            self.line(f"    {sg} = stablehlo.sign {d} : {T}")
            if op in (">=", "<="):
                sh = self.fresh()
                self.line(f"    {sh} = stablehlo.add {sg}, {one_bc} : {T}")
                c = self.fresh()
                self.line(f"    {c} = stablehlo.clamp {zero_bc}, {sh}, {one_bc} : {T}")
            else:
                c = self.fresh()
                self.line(f"    {c} = stablehlo.clamp {zero_bc}, {sg}, {one_bc} : {T}")
            return c, ot
        d = self.fresh()
        self.line(f"    {d} = stablehlo.subtract {a}, {b} : {T}")
        ad = self.fresh()
        self.line(f"    {ad} = stablehlo.abs {d} : {T}")
        cp = self.fresh()
        self.line(f"    {cp} = stablehlo.minimum {ad}, {one_bc} : {T}")
        if op in ("=", "=="):
            res = self.fresh()
            self.line(f"    {res} = stablehlo.subtract {one_bc}, {cp} : {T}")
            return res, ot
        if op == "!=":
            return cp, ot
        raise ValueError(op)

    def select(self, p, a, b, pt: Ty, at: Ty):
        rt = at
        zero = self.constant_f32(0.0)
        zb = self.broadcast(zero, SCALAR, pt)
        it = Ty(pt.shape, "i1")
        pi = self.fresh()
        self.line(f"    {pi} = stablehlo.compare NE, {p}, {zb}, FLOAT : ({pt.mlir()}, {pt.mlir()}) -> {it.mlir()}")
        r = self.fresh()
        self.line(f"    {r} = stablehlo.select {pi}, {a}, {b} : {it.mlir()}, {rt.mlir()}")
        return r, rt

    @staticmethod
    def _bshape2(a, b):
        n = max(len(a), len(b))
        a = (1,) * (n - len(a)) + tuple(a)
        b = (1,) * (n - len(b)) + tuple(b)
        return tuple(max(x, y) for x, y in zip(a, b))

    def where(self, c, x, y, ct, xt, yt):
        rs = self._bshape2(self._bshape2(xt.shape, yt.shape), ct.shape)
        if ct.shape != rs:
            tgt = Ty(rs)
            c, ct = self.broadcast(c, ct, tgt), tgt
        if xt.shape != rs:
            tgt = Ty(rs)
            x, xt = self.broadcast(x, xt, tgt), tgt
        if yt.shape != rs:
            tgt = Ty(rs)
            y, yt = self.broadcast(y, yt, tgt), tgt
        return self.select(c, x, y, ct, xt)

    def tril(self, x, t: Ty):
        r = self.fresh()
        m, n = t.shape
        ri, rit = self.fresh(), Ty((m, n))
        self.line(f"    {ri} = stablehlo.iota dim = 0 : {rit.mlir()}")
        ci = self.fresh()
        self.line(f"    {ci} = stablehlo.iota dim = 1 : {rit.mlir()}")
        mask, _ = self.compare(">=", ri, ci, rit, rit)
        self.line(f"    {r} = stablehlo.multiply {x}, {mask} : {t.mlir()}")
        return r, t

    def one_hot(self, idx, it: Ty, nc: int):
        if not it.shape:
            out = Ty((nc,))
            cls, clt = self.iota((nc,), 0)
            ib = self.broadcast(idx, it, clt)
            mask, mt = self.compare("==", ib, cls, clt, clt)
        else:
            out = Ty(tuple(it.shape) + (nc,))
            cls, clt = self.iota(out.shape, len(out.shape) - 1)
            et = Ty(tuple(it.shape) + (1,))
            r2 = self.fresh()
            self.line(f"    {r2} = stablehlo.reshape {idx} : ({it.mlir()}) -> {et.mlir()}")
            ib = self.broadcast(r2, et, clt)
            mask, mt = self.compare("==", ib, cls, clt, clt)
        one = self.constant_f32(1.0)
        zero = self.constant_f32(0.0)
        ones = self.broadcast(one, SCALAR, out)
        zeros = self.broadcast(zero, SCALAR, out)
        return self.select(mask, ones, zeros, mt, out)

    # dot (dot_ops.rs:16-241) ---------------------------------------------
    def _dot_line(self, r, a, b, at, bt, rt, lc, rc, batch=0, indent="  "):
        if batch:
            bd = ", ".join(str(i) for i in range(batch))
            self.line(f"{indent}{r} = stablehlo.dot_general {a}, {b}, batching_dims = [{bd}] x [{bd}], "
                      f"contracting_dims = [{lc}] x [{rc}] : ({at.mlir()}, {bt.mlir()}) -> {rt.mlir()}")
        else:
            self.line(f"{indent}{r} = stablehlo.dot_general {a}, {b}, contracting_dims = [{lc}] x [{rc}]"
                      f" : ({at.mlir()}, {bt.mlir()}) -> {rt.mlir()}")

    def matmul(self, a, b, at: Ty, bt: Ty):
        ls, rs = at.shape, bt.shape
        lr, rr = len(ls), len(rs)
        if lr == 0 or rr == 0:
            return self.binop("*", a, b, at, bt)
        if lr == 1 and rr == 1:
            rt = Ty(())
            r = self.fresh()
            self._dot_line(r, a, b, at, bt, rt, 0, 0, indent="    ")
            return r, rt
        if lr == 1:
            rt = Ty(tuple(rs[:rr - 2]) + tuple(rs[rr - 1:]))
            r = self.fresh()
            self._dot_line(r, a, b, at, bt, rt, 0, rr - 2, indent="    ")
            return r, rt
        if rr == 1:
            rt = Ty(tuple(ls[:lr - 1]))
            r = self.fresh()
            self._dot_line(r, a, b, at, bt, rt, lr - 1, 0, indent="    ")
            return r, rt
        nb = 0 if rr <= 2 else max(min(lr, rr) - 2, 0)
        lc, rc = lr - 1, nb
        res = tuple(ls[:nb]) + tuple(ls[nb:lr - 1]) + tuple(rs[nb + 1:])
        l1 = 0
        if lr > 2 and rr <= 2:
            for d in ls[:lr - 2]:
                if d == 1:
                    l1 += 1
                else:
                    break
        r1 = 0
        if rr > 2 and lr <= 2:
            for d in rs[:rr - 2]:
                if d == 1:
                    r1 += 1
                else:
                    break
        if l1 > 0:
            af, aft = self.reshape(a, at, ls[l1:])
            frt = Ty(res[l1:])
            r = self.fresh()
            self._dot_line(r, af, b, aft, bt, frt, lc - l1, rc, indent=" ")
            return self.reshape(r, frt, res)
        if r1 > 0:
            bf, bft = self.reshape(b, bt, rs[r1:])
            frt = Ty(res[r1:])
            r = self.fresh()
            self._dot_line(r, a, bf, at, bft, frt, lc, rc - r1, indent=" ")
            return self.reshape(r, frt, res)
        if nb > 0 and all(d == 1 for d in ls[:nb]) and all(d == 1 for d in rs[:nb]):
            a2s = (int(np.prod(ls[nb:lr - 1])), ls[lr - 1])
            b2s = (rs[nb], int(np.prod(rs[nb + 1:])))
            af, aft = self.reshape(a, at, a2s)
            bf, bft = self.reshape(b, bt, b2s)
            rt2 = Ty((a2s[0], b2s[1]))
            r = self.fresh()
            self._dot_line(r, af, bf, aft, bft, rt2, 1, 0, indent=" ")
            return self.reshape(r, rt2, res)
        npeel = 0
        for i in range(nb):
            if ls[i] == 1 and rs[i] == 1:
                npeel += 1
            else:
                break
        if npeel > 0:
            af, aft = self.reshape(a, at, ls[npeel:])
            bf, bft = self.reshape(b, bt, rs[npeel:])
            frt = Ty(res[npeel:])
            r = self.fresh()
            self._dot_line(r, af, bf, aft, bft, frt, lc - npeel, rc - npeel, batch=nb - npeel, indent=" ")
            return self.reshape(r, frt, res)
        rt = Ty(res)
        r = self.fresh()
        self._dot_line(r, a, b, at, bt, rt, lc, rc, batch=nb, indent="  ")
        return r, rt

    def einsum(self, a, b, at: Ty, bt: Ty, spec: str):
        """Two-input einsum as one dot_general (+ transpose), dot_ops.rs:244-461."""
        spec = "".join(spec.split())
        ins, out = spec.split("->")
        ls, rs = ins.split(",")
        if "..." in ls or "..." in rs or "..." in out:
            raise NotImplementedError("einsum with ellipsis")
        size = {}
        for c, d in zip(ls, at.shape):
            size[c] = d
        for c, d in zip(rs, bt.shape):
            size[c] = d
        lb, rb, lc, rc = [], [], [], []
        for i, c in enumerate(ls):
            if c in rs:
                if c in out:
                    lb.append(i)
                    rb.append(rs.index(c))
                else:
                    lc.append(i)
                    rc.append(rs.index(c))
        batch_labels = [ls[i] for i in lb]
        contract = {ls[i] for i in lc}
        lrem = [c for c in ls if c not in batch_labels and c not in contract]
        rrem = [c for c in rs if c not in batch_labels and c not in contract]
        dot_labels = batch_labels + lrem + rrem
        dt = Ty(tuple(size[c] for c in dot_labels))
        r = self.fresh()
        fm = lambda xs: ", ".join(map(str, xs))
        if not lb:
            self.line(f"    {r} = stablehlo.dot_general {a}, {b}, contracting_dims = [{fm(lc)}] x [{fm(rc)}]"
                      f" : ({at.mlir()}, {bt.mlir()}) -> {dt.mlir()}")
        else:
            self.line(f"    {r} = stablehlo.dot_general {a}, {b}, batching_dims = [{fm(lb)}] x [{fm(rb)}], "
                      f"contracting_dims = [{fm(lc)}] x [{fm(rc)}] : ({at.mlir()}, {bt.mlir()}) -> {dt.mlir()}")
        if dot_labels == list(out):
            return r, dt
        perm = [dot_labels.index(c) for c in out]
        return self.transpose(r, dt, perm)

    # gather (indexing_ops.rs:399-475) ------------------------------------
    def gather_axis0(self, op, ot: Ty, idx, it: Ty):
        iit = Ty(it.shape, "i32")
        ii = self.convert(idx, it, iit)
        rsh = tuple(it.shape) + (1,)
        i3 = self.fresh()
        i3t = Ty(rsh, "i32")
        self.line(f"    {i3} = stablehlo.reshape {ii} : ({iit.mlir()}) -> {i3t.mlir()}")
        row = tuple(ot.shape[1:])
        rt = Ty(tuple(it.shape) + row)
        ir = len(it.shape)
        offs = ", ".join(str(d) for d in range(ir, ir + len(row)))
        sizes = ", ".join(str(d) for d in (1,) + row)
        r = self.fresh()
        self.line(f"    {r} = \"stablehlo.gather\"({op}, {i3}) {{\n"
                  f"      dimension_numbers = #stablehlo.gather<\n"
                  f"        offset_dims = [{offs}],\n"
                  f"        collapsed_slice_dims = [0],\n"
                  f"        operand_batching_dims = [],\n"
                  f"        start_indices_batching_dims = [],\n"
                  f"        start_index_map = [0],\n"
                  f"        index_vector_dim = {len(rsh) - 1}>,\n"
                  f"      slice_sizes = array<i64: {sizes}>,\n"
                  f"      indices_are_sorted = false\n"
                  f"    }} : ({ot.mlir()}, {i3t.mlir()}) -> {rt.mlir()}")
        return r, rt

    def pad(self, x, t: Ty, target, axis, lo, hi):
        z = self.constant_f32(0.0)
        rt = Ty(tuple(target))
        nd = len(t.shape)
        low = ", ".join(str(lo) if i == axis else "0" for i in range(nd))
        high = ", ".join(str(hi) if i == axis else "0" for i in range(nd))
        inter = ", ".join("0" for _ in range(nd))
        r = self.fresh()
        self.line(f"    {r} = stablehlo.pad {x}, {z}, low = [{low}], high = [{high}], interior = [{inter}]"
                  f" : ({t.mlir()}, tensor<f32>) -> {rt.mlir()}")
        return r, rt


# ---------------------------------------------------------------------------
# Builtin codegen (sheaf/src/lowering/codegen/*.rs)
# ---------------------------------------------------------------------------

def _kwargs(args):
    """Split Sheaf keyword arguments: returns (positionals, {kw: value})."""
    pos, kws, i = [], {}, 0
    while i < len(args):
        a = args[i]
        if isinstance(a, Kw):
            nxt = args[i + 1] if i + 1 < len(args) else None
            if a.name == "keepdims":
                if isinstance(nxt, bool):
                    kws["keepdims"] = nxt
                    i += 2
                else:
                    kws["keepdims"] = True
                    i += 1
                continue
            kws[a.name] = nxt
            i += 2
            continue
        pos.append(a)
        i += 1
    return pos, kws


class Codegen:
    """Lowers Sheaf builtin calls to StableHLO through an Emitter."""

    def __init__(self, em: Emitter):
        self.em = em
        self.env: Dict[str, Tuple[str, Ty]] = {}

    def bind(self, name, reg, ty):
        self.env[name] = (reg, ty)

    def gen(self, e) -> Tuple[str, Any]:
        em = self.em
        if isinstance(e, Sym):
            return self.env[e.name]
        if isinstance(e, bool):
            return em.constant_f32(1.0 if e else 0.0), SCALAR
        if isinstance(e, (int, float)):
            return em.constant_f32(float(e)), SCALAR
        if isinstance(e, Vec):
            arr = np.array([_lit(x) for x in e.items], dtype=np.float64) if not any(
                isinstance(x, Vec) for x in e.items) else np.array(_nested(e), dtype=np.float64)
            return em.nd_constant(arr.reshape(-1).tolist(), arr.shape)
        if isinstance(e, Call):
            return self.call(e.fn, e.args)
        raise TypeError(e)

    def shape_of(self, e):
        return self.gen(e)[1].shape

    def call(self, fn, args):
        em = self.em
        g = self.gen
        if fn == "stop-gradient":
            return g(args[0])
        if fn in ("+", "-", "*", "/") and len(args) >= 2:
            r, t = g(args[0])
            for a in args[1:]:
                br, bt = g(a)
                r, t = em.binop(fn, r, br, t, bt)
            return r, t
        if fn == "-" and len(args) == 1:
            r, t = g(args[0])
            return em.unary("neg", r, t), t
        if fn in ("**", "min", "max") and len(args) == 2 and not isinstance(args[1], Kw):
            a, at = g(args[0])
            b, bt = g(args[1])
            return em.binop(fn, a, b, at, bt)
        if fn in ("maximum", "minimum"):
            a, at = g(args[0])
            b, bt = g(args[1])
            return em.binop("max" if fn == "maximum" else "min", a, b, at, bt)
        if fn in ("=", "==", "!=", "<", "<=", ">", ">="):
            a, at = g(args[0])
            b, bt = g(args[1])
            return em.compare(fn, a, b, at, bt)
        if fn == "@":
            a, at = g(args[0])
            b, bt = g(args[1])
            return em.matmul(a, b, at, bt)
        if fn == "einsum":
            a, at = g(args[1])
            b, bt = g(args[2])
            return em.einsum(a, b, at, bt, args[0])
        if fn in ("sqrt", "exp", "log", "abs", "neg", "sin", "cos", "tanh"):
            a, at = g(args[0])
            return em.unary(fn, a, at), at
        if fn in ("sum", "mean", "max", "min", "var"):
            x, xt = g(args[0])
            _, kw = _kwargs(args[1:])
            axis = kw.get("axis")
            keep = kw.get("keepdims", False)
            if fn == "var":
                if axis is not None:
                    m, mt = em.reduce_mean(x, xt, axis, True)
                    d, dt = em.binop("-", x, m, xt, mt)
                    s, st = em.binop("*", d, d, dt, dt)
                    return em.reduce_mean(s, st, axis, keep)
                raise NotImplementedError("var without axis")
            red = {"sum": em.reduce_sum, "mean": em.reduce_mean,
                   "max": em.reduce_max, "min": em.reduce_min}[fn]
            if axis is not None:
                return red(x, xt, int(axis), keep)
            r, t = x, xt
            for _ in range(len(xt.shape)):
                r, t = red(r, t, -1, False)
            return r, t
        if fn in ("transpose", "tr"):
            x, xt = g(args[0])
            if len(args) == 2:
                perm = [int(v) for v in args[1].items]
            else:
                nd = max(len(xt.shape), 2)
                perm = list(range(nd))
                perm[nd - 2], perm[nd - 1] = perm[nd - 1], perm[nd - 2]
            return em.transpose(x, xt, perm)
        if fn == "reshape":
            x, xt = g(args[0])
            shp = [int(v) for v in args[1].items]
            if any(d < 0 for d in shp):
                known = int(np.prod([d for d in shp if d > 0]))
                total = int(np.prod(xt.shape)) if xt.shape else 1
                shp[[i for i, d in enumerate(shp) if d < 0][0]] = total // known
            return em.reshape(x, xt, shp)
        if fn == "swapaxes":
            x, xt = g(args[0])
            nd = len(xt.shape)
            a1, a2 = int(args[1]), int(args[2])
            a1 = nd + a1 if a1 < 0 else a1
            a2 = nd + a2 if a2 < 0 else a2
            perm = list(range(nd))
            perm[a1], perm[a2] = a2, a1
            return em.transpose(x, xt, perm)
        if fn == "broadcast":
            x, xt = g(args[0])
            tt = Ty(tuple(int(v) for v in args[1].items))
            return em.broadcast(x, xt, tt), tt
        if fn in ("ones", "zeros"):
            shp = tuple(int(v) for v in args[0].items)
            return em.splat(1.0 if fn == "ones" else 0.0, shp)
        if fn == "tril":
            x, xt = g(args[0])
            return em.tril(x, xt)
        if fn == "where":
            c, ct = g(args[0])
            x, xt = g(args[1])
            y, yt = g(args[2])
            return em.where(c, x, y, ct, xt, yt)
        if fn == "one-hot":
            idx, it = g(args[0])
            nc = args[1]
            if isinstance(nc, Sym):
                reg, _ = g(nc)
                nc = em.known[reg]
            return em.one_hot(idx, it, int(nc))
        if fn == "slice":
            x, xt = g(args[0])
            pos, kw = _kwargs(args[1:])
            axis = int(kw.get("axis", 0))
            nd = len(xt.shape)
            axis = nd + axis if axis < 0 else axis
            start = int(pos[0])
            end = int(pos[1]) if len(pos) > 1 else xt.shape[axis]
            return em.slice_axis(x, xt, start, end, axis)
        if fn == "get":
            op, ot = g(args[0])
            idx, it = g(args[1])
            return em.gather_axis0(op, ot, idx, it)
        if fn == "shape":
            _, xt = g(args[0])
            ax = int(args[1])
            ax = len(xt.shape) + ax if ax < 0 else ax
            v = float(xt.shape[ax])
            return em.constant_f32(v), SCALAR
        if fn == "sum_to_shape":
            r, t = g(args[0])
            tgt = tuple(int(v) for v in args[1].items)
            if t.shape == tgt:
                return r, t
            for _ in range(max(len(t.shape) - len(tgt), 0)):
                r, t = em.reduce_sum(r, t, 0, False)
            cur = t.shape
            for i in reversed(range(min(len(cur), len(tgt)))):
                if tgt[i] == 1 and cur[i] > 1:
                    r, t = em.reduce_sum(r, t, i, True)
            return r, t
        if fn == "slice_grad":
            r, t = g(args[0])
            tgt = tuple(int(v) for v in args[1].items)
            start = int(args[2])
            axis = next((i for i, (a, b) in enumerate(zip(t.shape, tgt)) if a != b), 0)
            end = start + t.shape[axis]
            return em.pad(r, t, tgt, axis, start, tgt[axis] - end)
        raise NotImplementedError(f"builtin {fn}")


def _lit(x):
    if isinstance(x, bool):
        return 1.0 if x else 0.0
    return float(x)


def _nested(v):
    if isinstance(v, Vec):
        return [_nested(x) for x in v.items]
    return _lit(v)


# ---------------------------------------------------------------------------
# Tracer: builds the ANF forward bindings of an inlined Sheaf body
# ---------------------------------------------------------------------------

class Tracer:
    """Records Sheaf builtin calls as ANF bindings and lowers them eagerly.

    Lowering each binding as it is recorded matches Sheaf's VAG pipeline,
    which emits the forward bindings before running reverse-mode AD on them
    (sheaf/src/runtime/jit/vag.rs:486-494)."""

    def __init__(self):
        self.em = Emitter()
        self.cg = Codegen(self.em)
        self.bindings: List[Tuple[str, Call]] = []
        self.shapes: Dict[str, tuple] = {}
        self.args: List[Tuple[str, Ty]] = []
        self._n = 0

    def arg(self, name: str, shape, dtype="f32") -> Sym:
        t = Ty(tuple(shape), dtype)
        reg = f"%arg{len(self.args)}"
        self.args.append((name, t))
        self.cg.bind(name, reg, t)
        self.shapes[name] = t.shape
        return Sym(name)

    def __call__(self, fn: str, *args) -> Sym:
        name = f"__anf_{self._n}"
        self._n += 1
        call = Call(fn, list(args))
        reg, ty = self.cg.call(fn, call.args)
        self.cg.bind(name, reg, ty)
        self.shapes[name] = ty.shape
        self.bindings.append((name, call))
        return Sym(name)

    def shape(self, s) -> tuple:
        if isinstance(s, Sym):
            return self.shapes[s.name]
        return ()


# ---------------------------------------------------------------------------
# Reverse-mode AD over ANF bindings (sheaf/src/autodiff/reverse.rs:209-1075)
# ---------------------------------------------------------------------------

class MissingRule(Exception):
    pass


def _zeroish(e):
    return (isinstance(e, float) and e == 0.0) or (_is_int(e) and e == 0)


def simplify(e):
    """sheaf/src/autodiff/mod.rs:139-178."""
    if not isinstance(e, Call):
        return e
    args = [simplify(a) for a in e.args]
    fn = e.fn
    if fn == "+" and len(args) == 2:
        if isinstance(args[0], float) and args[0] == 0.0:
            return args[1]
        if isinstance(args[1], float) and args[1] == 0.0:
            return args[0]
    if fn == "*" and len(args) == 2:
        if (isinstance(args[0], float) and args[0] == 0.0) or (isinstance(args[1], float) and args[1] == 0.0):
            return 0.0
        if isinstance(args[0], float) and args[0] == 1.0:
            return args[1]
        if isinstance(args[1], float) and args[1] == 1.0:
            return args[0]
    if fn == "-" and len(args) == 2 and isinstance(args[1], float) and args[1] == 0.0:
        return args[0]
    if fn in ("transpose", "tr") and len(args) == 1 and isinstance(args[0], Call) \
            and args[0].fn in ("transpose", "tr") and len(args[0].args) == 1:
        return args[0].args[0]
    return Call(fn, args)


def _kwint(args, key):
    for i, a in enumerate(args):
        if isinstance(a, Kw) and a.name == key and i + 1 < len(args) and _is_int(args[i + 1]):
            return args[i + 1]
    return None


def reverse_grad(bindings, body: Sym, wrt: Sequence[str], shapes: Dict[str, tuple], depends):
    back: List[Tuple[str, Any]] = []
    adj: Dict[str, str] = {}

    def emit(value) -> str:
        name = f"__grad_{len(back)}"
        back.append((name, value))
        return name

    def accumulate(var, contrib):
        if _zeroish(contrib):
            return
        if var not in adj:
            adj[var] = emit(contrib)
        else:
            c = emit(contrib)
            adj[var] = emit(Call("+", [Sym(adj[var]), Sym(c)]))

    def acc(arg, contrib):
        if isinstance(arg, Sym):
            accumulate(arg.name, contrib)

    def shp(arg):
        return shapes.get(arg.name) if isinstance(arg, Sym) else None

    def unb(a, target):
        ts = shp(target)
        if ts is not None:
            return Sym(emit(Call("sum_to_shape", [a, Vec(ts)])))
        return a

    def C(fn, *a):
        return Call(fn, list(a))

    adj[body.name] = emit(1.0)
    for name, call in reversed(bindings):
        if name not in adj:
            continue
        g = Sym(adj[name])
        fn, args = call.fn, call.args
        if fn == "stop-gradient":
            continue
        if fn == "+":
            acc(args[0], unb(g, args[0]))
            acc(args[1], unb(g, args[1]))
        elif fn == "-" and len(args) == 2:
            acc(args[0], unb(g, args[0]))
            neg = emit(C("*", -1.0, g))
            acc(args[1], unb(Sym(neg), args[1]))
        elif fn == "-" and len(args) == 1:
            acc(args[0], Sym(emit(C("*", -1.0, g))))
        elif fn == "*":
            da = emit(C("*", g, args[1]))
            acc(args[0], unb(Sym(da), args[0]))
            db = emit(C("*", g, args[0]))
            acc(args[1], unb(Sym(db), args[1]))
        elif fn == "/" and len(args) == 2:
            da = emit(C("/", g, args[1]))
            acc(args[0], unb(Sym(da), args[0]))
            bsq = emit(C("*", args[1], args[1]))
            ab2 = emit(C("/", args[0], Sym(bsq)))
            neg = emit(C("*", -1.0, Sym(ab2)))
            db = emit(C("*", g, Sym(neg)))
            acc(args[1], unb(Sym(db), args[1]))
        elif fn == "@":
            sa, sb = shp(args[0]), shp(args[1])
            an = len(sa) if sa is not None else 2
            bn = len(sb) if sb is not None else 2
            if bn == 1:
                da = emit(C("*", g, args[1]))
                acc(args[0], unb(Sym(da), args[0]))
            elif an == 1:
                if sb is not None:
                    n = sb[-1]
                    row = emit(C("reshape", g, Vec([1, n])))
                    bt = emit(C("transpose", args[1]))
                    d2 = emit(C("@", Sym(row), Sym(bt)))
                    da = emit(C("reshape", Sym(d2), Vec([sb[0]])))
                    acc(args[0], Sym(da))
                else:
                    bt = emit(C("transpose", args[1]))
                    da = emit(C("@", g, Sym(bt)))
                    acc(args[0], unb(Sym(da), args[0]))
            else:
                bt = emit(C("transpose", args[1]))
                da = emit(C("@", g, Sym(bt)))
                acc(args[0], unb(Sym(da), args[0]))
            if an == 1:
                if sa is not None and sb is not None:
                    col = emit(C("reshape", args[0], Vec([sa[0], 1])))
                    row = emit(C("reshape", g, Vec([1, sb[-1]])))
                    db = emit(C("@", Sym(col), Sym(row)))
                    acc(args[1], unb(Sym(db), args[1]))
                else:
                    at = emit(C("transpose", args[0]))
                    db = emit(C("@", Sym(at), g))
                    acc(args[1], unb(Sym(db), args[1]))
            else:
                at = emit(C("transpose", args[0]))
                db = emit(C("@", Sym(at), g))
                acc(args[1], unb(Sym(db), args[1]))
        elif fn == "einsum" and len(args) == 3 and isinstance(args[0], str):
            ins, out = args[0].split("->")
            ls, rs = [p.strip() for p in ins.split(",")]
            out = out.strip()
            da = emit(C("einsum", f"{out},{rs}->{ls}", g, args[2]))
            acc(args[1], Sym(da))
            db = emit(C("einsum", f"{ls},{out}->{rs}", args[1], g))
            acc(args[2], Sym(db))
        elif fn in ("transpose", "tr"):
            acc(args[0], Sym(emit(C("transpose", g))))
        elif fn == "reshape":
            s = shp(args[0])
            if s is not None:
                acc(args[0], Sym(emit(C("reshape", g, Vec(s)))))
            else:
                acc(args[0], g)
        elif fn == "swapaxes" and len(args) == 3:
            acc(args[0], Sym(emit(C("swapaxes", g, args[1], args[2]))))
        elif fn == "sum":
            s = shp(args[0])
            if s is not None:
                acc(args[0], Sym(emit(C("broadcast", g, Vec(s)))))
            else:
                acc(args[0], g)
        elif fn == "mean":
            s = shp(args[0])
            if s is not None:
                ax = _kwint(args, "axis")
                if ax is not None:
                    n = s[len(s) + ax if ax < 0 else ax]
                else:
                    n = int(np.prod(s))
                sc = emit(C("/", g, float(n)))
                acc(args[0], Sym(emit(C("broadcast", Sym(sc), Vec(s)))))
            else:
                acc(args[0], g)
        elif fn == "var":
            s = shp(args[0])
            if s is not None:
                ax = _kwint(args, "axis")
                margs = [args[0]]
                if ax is not None:
                    margs += [Kw("axis"), ax]
                margs += [Kw("keepdims"), True]
                m = emit(Call("mean", margs))
                d = emit(C("-", args[0], Sym(m)))
                n = s[len(s) + ax if ax < 0 else ax] if ax is not None else int(np.prod(s))
                sc = emit(C("*", 2.0 / n, Sym(d)))
                ct = emit(C("*", g, Sym(sc)))
                acc(args[0], unb(Sym(ct), args[0]))
            else:
                acc(args[0], g)
        elif fn in ("max", "min") and (len(args) == 1 or isinstance(args[1], Kw)):
            ax = _kwint(args, "axis")
            fa = [args[0]]
            if ax is not None:
                fa += [Kw("axis"), ax, Kw("keepdims"), True]
            fv = emit(Call(fn, fa))
            mask = emit(C("==", args[0], Sym(fv)))
            s = shp(args[0])
            if s is not None:
                bc = emit(C("broadcast", g, Vec(s)))
                acc(args[0], Sym(emit(C("*", Sym(bc), Sym(mask)))))
            else:
                acc(args[0], Sym(emit(C("*", g, Sym(mask)))))
        elif fn == "exp":
            acc(args[0], Sym(emit(C("*", g, Sym(name)))))
        elif fn == "log":
            inv = emit(C("/", 1.0, args[0]))
            acc(args[0], Sym(emit(C("*", g, Sym(inv)))))
        elif fn == "sqrt":
            sq = emit(C("sqrt", args[0]))
            two = emit(C("*", 2.0, Sym(sq)))
            inv = emit(C("/", 1.0, Sym(two)))
            acc(args[0], Sym(emit(C("*", g, Sym(inv)))))
        elif fn == "tanh":
            t2 = emit(C("*", Sym(name), Sym(name)))
            loc = emit(C("-", 1.0, Sym(t2)))
            acc(args[0], Sym(emit(C("*", g, Sym(loc)))))
        elif fn == "sin":
            c = emit(C("cos", args[0]))
            acc(args[0], Sym(emit(C("*", g, Sym(c)))))
        elif fn == "cos":
            s = emit(C("sin", args[0]))
            ng = emit(C("*", -1.0, Sym(s)))
            acc(args[0], Sym(emit(C("*", g, Sym(ng)))))
        elif fn in ("maximum", "minimum") and len(args) == 2:
            cond = emit(C(">=" if fn == "maximum" else "<=", args[0], args[1]))
            da = emit(C("where", Sym(cond), g, 0.0))
            db = emit(C("where", Sym(cond), 0.0, g))
            acc(args[0], Sym(da))
            acc(args[1], Sym(db))
        elif fn == "where" and len(args) == 3:
            da = emit(C("where", args[0], g, 0.0))
            db = emit(C("where", args[0], 0.0, g))
            acc(args[1], Sym(da))
            acc(args[2], Sym(db))
        elif fn == "slice" and len(args) >= 3:
            s = shp(args[0])
            if s is not None:
                acc(args[0], Sym(emit(C("slice_grad", g, Vec(s), args[1]))))
            else:
                acc(args[0], g)
        elif fn == "neg":
            acc(args[0], Sym(emit(C("*", -1.0, g))))
        elif fn == "abs":
            cond = emit(C(">=", args[0], 0.0))
            sg = emit(C("where", Sym(cond), 1.0, -1.0))
            acc(args[0], Sym(emit(C("*", g, Sym(sg)))))
        elif fn == "**" and len(args) == 2:
            n = args[1]
            if not isinstance(n, (int, float)) or isinstance(n, bool):
                if depends.get(name, True):
                    raise MissingRule("**")
                continue
            n = float(n)
            pw = emit(C("**", args[0], n - 1.0))
            loc = emit(C("*", n, Sym(pw)))
            acc(args[0], Sym(emit(C("*", g, Sym(loc)))))
        elif fn == "get" and len(args) == 2:
            v = emit(C("shape", args[0], 0))
            oh = emit(C("one-hot", args[1], Sym(v)))
            oht = emit(C("tr", Sym(oh)))
            acc(args[0], Sym(emit(C("@", Sym(oht), g))))
        else:
            if depends.get(name, True):
                raise MissingRule(fn)
    return [(n, simplify(v)) for n, v in back], adj


def _depends(bindings, wrt):
    dep = {w: True for w in wrt}

    def d(e):
        if isinstance(e, Sym):
            return dep.get(e.name, False)
        if isinstance(e, Vec):
            return any(d(x) for x in e.items)
        if isinstance(e, Call):
            return any(d(x) for x in e.args)
        return False
    for n, c in bindings:
        dep[n] = d(c)
    return dep


# ---------------------------------------------------------------------------
# Module assembly
# ---------------------------------------------------------------------------

def _module(name: str, fn_name: str, args: List[Tuple[str, Ty]], body: List[str],
            results: List[Tuple[str, Ty]]) -> str:
    params = ", ".join(f"%arg{i}: {t.mlir()}" for i, (_, t) in enumerate(args))
    if len(results) == 1:
        ret_ty = results[0][1].mlir()
    else:
        ret_ty = "(" + ", ".join(t.mlir() for _, t in results) + ")"
    lines = ["// Generated by Sheaf", "//", "", f"module @{name} {{",
             f" func.func @{fn_name}({params}) -> {ret_ty} {{"]
    lines += body
    lines.append(f"    return {', '.join(r for r, _ in results)} : {', '.join(t.mlir() for _, t in results)}")
    lines.append(" }")
    lines.append("}")
    return "\n".join(lines) + "\n"


def _module_name(prefix: str, key: str) -> str:
    return f"{prefix}_{hashlib.sha1(key.encode()).hexdigest()[:16]}"


@dataclass
class Lowered:
    """A lowered module plus the metadata a caller keeps beside it."""
    text: str
    module: str
    function: str
    arg_names: List[str]
    arg_types: List[Ty]
    result_types: List[Ty]

    @property
    def qualified(self) -> str:
        return f"{self.module}.{self.function}"


def lower_value_and_grad(build, wrt: List[Tuple[str, tuple]], captures: List[Tuple[str, tuple]],
                         key: str = "") -> Lowered:
    """Lower `((value-and-grad loss-fn) params)`.

    `wrt` lists the parameter leaves in flattened (sorted-key) order, `captures`
    the tensor captures that become trailing function arguments.  `build(tr,
    syms)` records the inlined loss body on the tracer and returns the loss
    symbol.  Output: `(loss, grad leaves...)` as `func.func @value_and_grad`
    (sheaf/src/runtime/jit/vag.rs:611-619)."""
    tr = Tracer()
    syms = {}
    for n, s in wrt:
        syms[n] = tr.arg(n, s)
    for n, s in captures:
        syms[n] = tr.arg(n, s)
    loss = build(tr, syms)
    loss_reg, loss_ty = tr.cg.env[loss.name]
    wrt_names = [n for n, _ in wrt]
    dep = _depends(tr.bindings, wrt_names)
    back, adj = reverse_grad(tr.bindings, loss, wrt_names, tr.shapes, dep)
    for n, v in back:
        reg, ty = tr.cg.gen(v)
        tr.cg.bind(n, reg, ty)
    results = [(loss_reg, loss_ty)]
    for n, s in wrt:
        pty = Ty(tuple(s))
        if n in adj:
            reg, ty = tr.cg.env[adj[n]]
        else:
            reg, ty = tr.cg.gen(Call("zeros", [Vec(s)]) if s else 0.0)
        reg, ty = _reduce_broadcast_grad(tr.em, reg, ty, pty)
        results.append((reg, ty))
    mod = _module_name("__vag", key or "\n".join(tr.em.body))
    text = _module(mod, "value_and_grad", tr.args, tr.em.body, results)
    return Lowered(text, mod, "value_and_grad", [n for n, _ in tr.args], [t for _, t in tr.args],
                   [t for _, t in results])


def lower_forward(build, args: List[Tuple[str, tuple]], fn_name: str, key: str = "") -> Lowered:
    """Lower a JIT-compiled forward function (sheaf/src/runtime/jit/compile.rs:340-479)."""
    tr = Tracer()
    syms = {n: tr.arg(n, s) for n, s in args}
    out = build(tr, syms)
    outs = out if isinstance(out, (list, tuple)) else [out]
    results = [tr.cg.env[o.name] for o in outs]
    mod = _module_name("__jit", key or "\n".join(tr.em.body))
    text = _module(mod, fn_name, tr.args, tr.em.body, results)
    return Lowered(text, mod, fn_name, [n for n, _ in tr.args], [t for _, t in tr.args],
                   [t for _, t in results])


def _reduce_broadcast_grad(em: Emitter, reg, gty: Ty, pty: Ty):
    """sheaf/src/lowering/codegen/autodiff.rs:147-191."""
    gs, ps = gty.shape, pty.shape
    if gs == ps:
        return reg, gty
    if not gs and ps:
        return em.broadcast(reg, gty, pty), pty
    ge, pe = int(np.prod(gs)), int(np.prod(ps))
    if ge == pe and ge > 0:
        return em.reshape(reg, gty, ps)
    extra = max(len(gs) - len(ps), 0)
    if extra == 0 or tuple(gs[extra:]) != tuple(ps):
        return reg, gty
    for _ in range(extra):
        reg, gty = em.reduce_sum(reg, gty, 0, False)
    return reg, gty
