"""CPU oracle: a numpy interpreter of the StableHLO text subset Sheaf emits.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by `__graft_entry__.smoke()` and
by bench.py's CPU-baseline leg as the checker; never by the product path.

Scope: every op form produced by Sheaf's emitter
  constant / add subtract multiply divide power maximum minimum remainder
                                        sheaf/src/lowering/stablehlo/operations.rs:10-68
  tanh sqrt exponential log abs negate sine cosine not sign
                                        operations.rs:71-151, compare_ops.rs:15-121
  convert                               operations.rs:154-165
  broadcast_in_dim (dims = [...])       broadcast.rs:38-108
  reduce add/maximum/minimum/multiply   reduce_ops.rs:13-291
  reshape / transpose / iota / concatenate / reverse
                                        shape_ops.rs:10-165, indexing_ops.rs:181-204
  dot_general (batching + contracting)  dot_ops.rs:16-241, 418-443
  compare NE FLOAT / select / clamp     compare_ops.rs:131-176, 15-121
  slice / pad                           indexing_ops.rs:75-371, codegen/builtins.rs:228-296
  "stablehlo.gather" (axis-0 form)      indexing_ops.rs:399-475

Arithmetic follows StableHLO semantics.  Values are computed in float64 by
default (`dtype=np.float32` emulates the f32 graph), which makes this the
fp64-accumulate reference for large-shape parity.  The parser here is written
independently of the backend's C++ parser, so the two cross-check each other.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

_TENSOR_RE = re.compile(r"tensor<([^<>]*)>")


def parse_type(s: str):
    s = s.strip()
    m = _TENSOR_RE.fullmatch(s)
    if not m:
        raise ValueError(f"bad type {s!r}")
    parts = m.group(1).split("x")
    return tuple(int(p) for p in parts[:-1]), parts[-1]


def _ints(s: str) -> List[int]:
    s = s.strip()
    if not s:
        return []
    return [int(x) for x in s.split(",") if x.strip()]


def _split_types(s: str) -> List[str]:
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur.strip())
    return out


def _dense_values(payload: str, shape, dtype):
    payload = payload.strip()
    np_dt = np.float64 if dtype in ("f32", "f64", "bf16") else (np.bool_ if dtype == "i1" else np.int64)
    if payload.startswith("0x"):
        bits = int(payload, 16)
        v = np.array([bits], dtype=np.uint32).view(np.float32)[0]
        return np.full(shape, v, dtype=np_dt)
    if payload.startswith("["):
        flat = [float(x) for x in re.findall(r"[-+]?[0-9.]+(?:[eE][-+]?[0-9]+)?|nan|inf", payload)]
        return np.array(flat, dtype=np_dt).reshape(shape)
    if payload in ("true", "false"):
        return np.full(shape, payload == "true", dtype=np_dt)
    return np.full(shape, float(payload), dtype=np_dt)


@dataclass
class Op:
    results: List[str]
    kind: str
    operands: List[str]
    attrs: dict
    out_types: List[tuple]


@dataclass
class Func:
    name: str
    params: List[tuple]
    ops: List[Op] = field(default_factory=list)
    ret: List[str] = field(default_factory=list)


def _statements(body: str) -> List[str]:
    """Join multi-line statements (the gather op spans several lines)."""
    out, cur, depth = [], "", 0
    for raw in body.splitlines():
        line = raw.split("//", 1)[0] if not raw.strip().startswith('"') else raw
        if not line.strip():
            continue
        cur = (cur + " " + line.strip()) if cur else line.strip()
        depth += line.count("{") - line.count("}")
        if depth <= 0:
            out.append(cur)
            cur, depth = "", 0
    if cur:
        out.append(cur)
    return out


_BIN = {"add", "subtract", "multiply", "divide", "power", "maximum", "minimum", "remainder", "and", "or"}
_UN = {"tanh", "sqrt", "exponential", "log", "abs", "negate", "sine", "cosine", "not", "sign",
       "floor", "ceil", "rsqrt", "logistic"}


def parse_module(text: str) -> Dict[str, Func]:
    funcs: Dict[str, Func] = {}
    mod_name = None
    m = re.search(r"module\s+@([\w.$-]+)", text)
    if m:
        mod_name = m.group(1)
    # split into functions
    for fm in re.finditer(r"func\.func\s+@([\w.$-]+)\(([^)]*)\)\s*->\s*(.*?)\{", text):
        name = fm.group(1)
        params = []
        for p in _split_types(fm.group(2)):
            if not p:
                continue
            params.append(parse_type(p.split(":", 1)[1]))
        start = fm.end()
        depth, i = 1, start
        while depth and i < len(text):
            if text[i] == "{":
                depth += 1
            elif text[i] == "}":
                depth -= 1
            i += 1
        body = text[start:i - 1]
        f = Func(name, params)
        for st in _statements(body):
            if st.startswith("return"):
                vals = st[len("return"):].split(":", 1)[0]
                f.ret = [v.strip() for v in vals.split(",") if v.strip()]
                continue
            f.ops.append(_parse_op(st))
        funcs[name] = f
        if mod_name:
            funcs[f"{mod_name}.{name}"] = f
    return funcs


def _parse_op(st: str) -> Op:
    lhs, rhs = st.split("=", 1)
    results = [r.strip() for r in lhs.split(",")]
    rhs = rhs.strip()
    if rhs.startswith('"stablehlo.gather"'):
        m = re.match(r'"stablehlo\.gather"\((%\w+),\s*(%\w+)\)\s*\{(.*)\}\s*:\s*\((.*)\)\s*->\s*(tensor<[^>]*>)\s*$', rhs)
        attrs_s = m.group(3)
        attrs = {
            "offset_dims": _ints(re.search(r"offset_dims = \[([^\]]*)\]", attrs_s).group(1)),
            "collapsed": _ints(re.search(r"collapsed_slice_dims = \[([^\]]*)\]", attrs_s).group(1)),
            "start_index_map": _ints(re.search(r"start_index_map = \[([^\]]*)\]", attrs_s).group(1)),
            "index_vector_dim": int(re.search(r"index_vector_dim = (\d+)", attrs_s).group(1)),
            "slice_sizes": _ints(re.search(r"slice_sizes = array<i64: ([^>]*)>", attrs_s).group(1)),
        }
        return Op(results, "gather", [m.group(1), m.group(2)], attrs, [parse_type(m.group(5))])
    if rhs.startswith('"stablehlo.sort"'):
        # keys, payload sorted along `dimension` by a GT / LT comparator on the keys
        # (the top_k form, lowering/stablehlo/indexing_ops.rs:476-540)
        m = re.match(r'"stablehlo\.sort"\((%\w+),\s*(%\w+)\)', rhs)
        d = re.search(r"comparison_direction (\w+)>", rhs).group(1)
        dim = int(re.search(r"dimension = (\d+)", rhs).group(1))
        tys = _split_types(rhs.rsplit("->", 1)[1].strip().strip("()"))
        return Op(results, "sort", [m.group(1), m.group(2)], {"dir": d, "dim": dim},
                  [parse_type(t) for t in tys])
    m = re.match(r"stablehlo\.(\w+)\s*(.*)$", rhs)
    kind, rest = m.group(1), m.group(2)
    if kind == "constant":
        mm = re.match(r"dense<(.*)>\s*:\s*(tensor<[^>]*>)$", rest)
        shape, dt = parse_type(mm.group(2))
        return Op(results, "constant", [], {"value": _dense_values(mm.group(1), shape, dt)}, [(shape, dt)])
    if kind == "reduce":
        mm = re.match(r"\((%\w+) init: (%\w+)\) applies stablehlo\.(\w+) across dimensions = \[([^\]]*)\]"
                      r"\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        return Op(results, "reduce", [mm.group(1), mm.group(2)],
                  {"body": mm.group(3), "dims": _ints(mm.group(4))}, [parse_type(mm.group(6))])
    if kind == "iota":
        mm = re.match(r"dim = (\d+)\s*:\s*(.*)$", rest)
        return Op(results, "iota", [], {"dim": int(mm.group(1))}, [parse_type(mm.group(2))])
    if kind == "dot_general":
        mm = re.match(r"(%\w+),\s*(%\w+),\s*(?:batching_dims = \[([^\]]*)\] x \[([^\]]*)\],\s*)?"
                      r"contracting_dims = \[([^\]]*)\] x \[([^\]]*)\]\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        return Op(results, "dot_general", [mm.group(1), mm.group(2)],
                  {"lb": _ints(mm.group(3) or ""), "rb": _ints(mm.group(4) or ""),
                   "lc": _ints(mm.group(5)), "rc": _ints(mm.group(6))}, [parse_type(mm.group(8))])
    if kind == "compare":
        mm = re.match(r"(\w+),\s*(%\w+),\s*(%\w+)(?:,\s*(\w+))?\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        return Op(results, "compare", [mm.group(2), mm.group(3)], {"dir": mm.group(1)},
                  [parse_type(mm.group(6))])
    if kind == "slice":
        mm = re.match(r"(%\w+)\s*\[([^\]]*)\]\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        trip = [tuple(int(v) for v in d.split(":")) for d in mm.group(2).split(",")]
        return Op(results, "slice", [mm.group(1)], {"trip": trip}, [parse_type(mm.group(4))])
    if kind == "pad":
        mm = re.match(r"(%\w+),\s*(%\w+),\s*low = \[([^\]]*)\],\s*high = \[([^\]]*)\],\s*interior = \[([^\]]*)\]"
                      r"\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        return Op(results, "pad", [mm.group(1), mm.group(2)],
                  {"lo": _ints(mm.group(3)), "hi": _ints(mm.group(4)), "in": _ints(mm.group(5))},
                  [parse_type(mm.group(7))])
    if kind in ("broadcast_in_dim", "transpose", "reverse"):
        mm = re.match(r"(%\w+),\s*dims = \[([^\]]*)\]\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        return Op(results, kind, [mm.group(1)], {"dims": _ints(mm.group(2))}, [parse_type(mm.group(4))])
    if kind == "concatenate":
        mm = re.match(r"(.*),\s*dim = (\d+)\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        ops = [o.strip() for o in mm.group(1).split(",")]
        return Op(results, kind, ops, {"dim": int(mm.group(2))}, [parse_type(mm.group(4))])
    if kind in ("reshape", "convert", "bitcast_convert"):
        mm = re.match(r"(%\w+)\s*:\s*\((.*)\)\s*->\s*(.*)$", rest)
        return Op(results, kind, [mm.group(1)], {}, [parse_type(mm.group(3))])
    if kind == "select":
        mm = re.match(r"(%\w+),\s*(%\w+),\s*(%\w+)\s*:\s*(.*)$", rest)
        tys = _split_types(mm.group(4))
        return Op(results, kind, [mm.group(1), mm.group(2), mm.group(3)], {}, [parse_type(tys[-1])])
    if kind == "clamp":
        mm = re.match(r"(%\w+),\s*(%\w+),\s*(%\w+)\s*:\s*(.*)$", rest)
        return Op(results, kind, [mm.group(1), mm.group(2), mm.group(3)], {}, [parse_type(mm.group(4))])
    if kind in _BIN:
        mm = re.match(r"(%\w+),\s*(%\w+)\s*:\s*(.*)$", rest)
        return Op(results, kind, [mm.group(1), mm.group(2)], {}, [parse_type(mm.group(3))])
    if kind in _UN:
        mm = re.match(r"(%\w+)\s*:\s*(.*)$", rest)
        return Op(results, kind, [mm.group(1)], {}, [parse_type(mm.group(2))])
    raise NotImplementedError(f"oracle: unsupported op {kind}")


# Optional operand transform of dot_general (tests use it to model reduced-
# precision tensor-core operands); None in normal use.
_DOT_HOOK = None


def _wrap32(x):
    """Two's-complement wraparound of integers to 32 bits (StableHLO i32)."""
    x = np.asarray(x, dtype=np.int64)
    return ((x + (1 << 31)) & 0xFFFFFFFF) - (1 << 31)


def _bf16_rne(x):
    """Values rounded to bf16, round to nearest even (of the f32 value), as an
    op on bf16 tensors produces; NaN and infinities pass through."""
    f = np.asarray(x, np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    return np.where(np.isfinite(f), r, f)


def _as(x, dt, dtype):
    if dt == "bf16":
        # a bf16 argument holds the upper 16 bits of the host f32 value (the
        # runtime truncates on upload, sheaf/src/runtime/buffer_convert.rs:28-40)
        f = np.ascontiguousarray(x, np.float32)
        return (f.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32).astype(dtype)
    if dt in ("f32", "f64"):
        return np.asarray(x, dtype=dtype)
    if dt == "i1":
        return np.asarray(x, dtype=np.bool_)
    return np.asarray(x, dtype=np.int64)


def evaluate(f: Func, inputs: Sequence[np.ndarray], dtype=np.float64) -> List[np.ndarray]:
    if len(inputs) != len(f.params):
        raise ValueError(f"expected {len(f.params)} inputs, got {len(inputs)}")
    env: Dict[str, np.ndarray] = {}
    for i, (x, (shape, dt)) in enumerate(zip(inputs, f.params)):
        a = np.asarray(x)
        if tuple(a.shape) != tuple(shape):
            raise ValueError(f"input {i}: shape {a.shape} != {shape}")
        env[f"%arg{i}"] = _as(a, dt, dtype)
    # last use of every value, so that dead intermediates are dropped (the VAG
    # graphs hold thousands of values; keeping them all exhausts host memory)
    last: Dict[str, int] = {}
    for i, op in enumerate(f.ops):
        for o in op.operands:
            last[o] = i
    keep = set(f.ret)
    for oi, op in enumerate(f.ops):
        v = [env[o] for o in op.operands]
        for o in set(op.operands):
            if last.get(o) == oi and o not in keep:
                del env[o]
        (oshape, odt), = op.out_types[:1]
        k = op.kind
        if k == "sort":
            keys = np.asarray(v[0], np.float32 if dtype == np.float32 else np.float64)
            order = np.argsort(-keys if op.attrs["dir"] == "GT" else keys, axis=op.attrs["dim"], kind="stable")
            env[op.results[0]] = np.take_along_axis(np.asarray(v[0]), order, axis=op.attrs["dim"])
            env[op.results[1]] = np.take_along_axis(np.asarray(v[1]), order, axis=op.attrs["dim"])
            continue
        if k == "constant":
            r = op.attrs["value"]
        elif k == "add":
            r = v[0] + v[1]
        elif k == "subtract":
            r = v[0] - v[1]
        elif k == "multiply":
            r = v[0] * v[1]
        elif k == "divide":
            with np.errstate(divide="ignore", invalid="ignore"):
                r = v[0] / v[1]
        elif k == "power":
            with np.errstate(divide="ignore", invalid="ignore"):
                r = np.power(v[0], v[1])
        elif k == "maximum":
            r = np.maximum(v[0], v[1])
        elif k == "minimum":
            r = np.minimum(v[0], v[1])
        elif k == "remainder":
            r = np.fmod(v[0], v[1])
        elif k == "tanh":
            r = np.tanh(v[0])
        elif k == "sqrt":
            with np.errstate(invalid="ignore"):
                r = np.sqrt(v[0])
        elif k == "exponential":
            with np.errstate(over="ignore"):
                r = np.exp(v[0])
        elif k == "log":
            with np.errstate(divide="ignore", invalid="ignore"):
                r = np.log(v[0])
        elif k == "abs":
            r = np.abs(v[0])
        elif k == "negate":
            r = -v[0]
        elif k == "sine":
            r = np.sin(v[0])
        elif k == "cosine":
            r = np.cos(v[0])
        elif k == "sign":
            r = np.sign(v[0])
        elif k == "floor":
            r = np.floor(v[0])
        elif k == "ceil":
            r = np.ceil(v[0])
        elif k == "not":
            r = np.logical_not(v[0]) if v[0].dtype == np.bool_ else ~v[0]
        elif k == "clamp":
            r = np.minimum(np.maximum(v[1], v[0]), v[2])
        elif k == "bitcast_convert":
            # 32-bit reinterpretation (f32 <-> i32); f32 values are rounded to
            # f32 first (the f64 evaluation mode carries them wider)
            if odt == "i32" and v[0].dtype.kind == "f":
                r = np.asarray(v[0], np.float32).view(np.int32).astype(np.int64)
            elif odt in ("f32",) and v[0].dtype.kind != "f":
                r = _wrap32(v[0]).astype(np.int32).view(np.float32).astype(dtype)
            else:
                r = v[0]
        elif k == "convert":
            if odt in ("f32", "bf16", "f64"):
                r = v[0].astype(dtype)
            elif odt == "i1":
                r = v[0] != 0
            else:
                r = np.trunc(v[0]).astype(np.int64) if v[0].dtype.kind == "f" else v[0].astype(np.int64)
        elif k == "broadcast_in_dim":
            dims = op.attrs["dims"]
            src = v[0]
            shp = [1] * len(oshape)
            for i, d in enumerate(dims):
                shp[d] = src.shape[i]
            r = np.broadcast_to(src.reshape(shp), oshape)
        elif k == "reshape":
            r = v[0].reshape(oshape)
        elif k == "transpose":
            r = np.transpose(v[0], op.attrs["dims"])
        elif k == "reverse":
            r = np.flip(v[0], axis=tuple(op.attrs["dims"]))
        elif k == "iota":
            d = op.attrs["dim"]
            ar = np.arange(oshape[d], dtype=dtype if odt in ("f32", "f64", "bf16") else np.int64)
            shp = [1] * len(oshape)
            shp[d] = oshape[d]
            r = np.broadcast_to(ar.reshape(shp), oshape)
        elif k == "reduce":
            axes = tuple(op.attrs["dims"])
            body = op.attrs["body"]
            init = v[1]
            if body == "add":
                r = v[0].sum(axis=axes) + init
            elif body == "maximum":
                r = np.maximum(v[0].max(axis=axes, initial=-np.inf), init)
            elif body == "minimum":
                r = np.minimum(v[0].min(axis=axes, initial=np.inf), init)
            elif body == "multiply":
                r = v[0].prod(axis=axes) * init
            else:
                raise NotImplementedError(body)
        elif k == "dot_general":
            a, b = v
            lb, rb, lc, rc = (op.attrs[x] for x in ("lb", "rb", "lc", "rc"))
            lf = [d for d in range(a.ndim) if d not in lb and d not in lc]
            rf = [d for d in range(b.ndim) if d not in rb and d not in rc]
            at = np.transpose(a, lb + lf + lc)
            bt = np.transpose(b, rb + rc + rf)
            nb = len(lb)
            bshape = at.shape[:nb]
            M = int(np.prod([a.shape[d] for d in lf]))
            N = int(np.prod([b.shape[d] for d in rf]))
            K = int(np.prod([a.shape[d] for d in lc]))
            am, bm = at.reshape(bshape + (M, K)), bt.reshape(bshape + (K, N))
            if _DOT_HOOK is not None:
                am, bm = _DOT_HOOK(op, am, bm)
            r = np.matmul(am, bm)
            r = r.reshape(oshape)
        elif k == "compare":
            a, b = v
            dr = op.attrs["dir"]
            r = {"EQ": a == b, "NE": a != b, "LT": a < b, "LE": a <= b, "GT": a > b, "GE": a >= b}[dr]
        elif k == "select":
            r = np.where(v[0], v[1], v[2])
        elif k == "slice":
            sl = tuple(slice(s, l, st) for s, l, st in op.attrs["trip"])
            r = v[0][sl]
        elif k == "pad":
            lo, hi, it = op.attrs["lo"], op.attrs["hi"], op.attrs["in"]
            if any(l < 0 for l in lo) or any(h < 0 for h in hi):
                raise NotImplementedError("negative padding")
            r = np.full(oshape, v[1], dtype=v[0].dtype)
            sl = tuple(slice(l, l + (s - 1) * (i + 1) + 1, i + 1) if s else slice(l, l)
                       for l, s, i in zip(lo, v[0].shape, it))
            r[sl] = v[0]
        elif k == "concatenate":
            r = np.concatenate(v, axis=op.attrs["dim"])
        elif k == "gather":
            operand, idx = v
            at = op.attrs
            if at["collapsed"] != [0] or at["start_index_map"] != [0]:
                raise NotImplementedError("gather form")
            ii = np.take(idx, 0, axis=at["index_vector_dim"])
            ii = np.clip(ii, 0, operand.shape[0] - at["slice_sizes"][0])
            r = operand[ii]
        else:
            raise NotImplementedError(k)
        r = np.asarray(r)
        if odt in ("f32", "bf16", "f64"):
            # no copy when the type already matches (broadcast views stay views)
            r = r.astype(dtype, copy=False)
            if odt == "bf16":
                r = _bf16_rne(r).astype(dtype)
        elif odt == "i32":
            r = _wrap32(r)
        if tuple(r.shape) != tuple(oshape):
            raise ValueError(f"{op.results[0]} ({k}): shape {r.shape} != {oshape}")
        for name in op.results:
            env[name] = r
    return [np.array(env[r]) for r in f.ret]


def run(text: str, fn: str, inputs: Sequence[np.ndarray], dtype=np.float64) -> List[np.ndarray]:
    funcs = parse_module(text)
    if fn not in funcs:
        raise KeyError(f"function {fn!r} not in module ({sorted(funcs)})")
    return evaluate(funcs[fn], inputs, dtype)
