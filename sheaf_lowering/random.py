"""StableHLO text of Sheaf's JIT random ops, as its emitter writes them
(sheaf/src/lowering/stablehlo/random_ops.rs): random-key (:11-45),
random-normal (:50-273), random-uniform (:275-417), random-randint
(:419-607), random-split (:634-756), plus the device program of
`init-gpt-params` (examples/nanoGPT/model.shf:17-43) built from them.

Keys are tensor<2xf32> holding two i32 halves through bitcast_convert.  The
hash is i32 arithmetic with wraparound:
    x = ((iota + lo) * 1540483477 + hi) * 668265263 + 1013904223
    u = f32(abs(x)) / 2^31
normal = sqrt(-2 log(u1 + 1e-7)) * cos(2 pi u2) over the two halves of a 2N
sample; randint = clamp(floor(u * (high - low)) + low, low, high - 1); split
i of (lo, hi): (((lo + i) * 2069105475 + 1013904223), hi + lo + i).
These forms are the interface (what the JIT hands to the runtime), so they are
reproduced op for op; the Python that writes them is this project's.
"""
from __future__ import annotations

import math
from typing import List, Sequence, Tuple

from .lower import Lowered


def _ty(shape: Sequence[int], dt: str) -> str:
    return "tensor<" + "".join(f"{d}x" for d in shape) + dt + ">"


def _f32_lit(v: float) -> str:
    r = repr(float(v))
    return r if ("e" in r or "." in r) else r + ".0"


class RandomEmitter:
    def __init__(self):
        self.lines: List[str] = []
        self.n = 0

    def reg(self) -> str:
        self.n += 1
        return f"%rng{self.n}"

    def emit(self, text: str) -> str:
        r = self.reg()
        self.lines.append(f"    {r} = {text}")
        return r

    def const_i32(self, v: int) -> str:
        return self.emit(f"stablehlo.constant dense<{int(v)}> : tensor<i32>")

    def const_f32(self, v: float) -> str:
        return self.emit(f"stablehlo.constant dense<{_f32_lit(v)}> : tensor<f32>")

    def bcast(self, scalar: str, shape, dt: str) -> str:
        return self.emit(f"stablehlo.broadcast_in_dim {scalar}, dims = [] : ({_ty((), dt)}) -> {_ty(shape, dt)}")

    def bitcast(self, x: str, shape, src: str, dst: str) -> str:
        return self.emit(f"stablehlo.bitcast_convert {x} : ({_ty(shape, src)}) -> {_ty(shape, dst)}")

    # --- keys ----------------------------------------------------------------
    def key_from_seed(self, seed: int) -> str:
        lo = self.const_i32(seed & 0xFFFFFFFF)
        hi = self.const_i32((seed >> 32) & 0xFFFFFFFF)
        lo1 = self.emit(f"stablehlo.reshape {lo} : (tensor<i32>) -> tensor<1xi32>")
        hi1 = self.emit(f"stablehlo.reshape {hi} : (tensor<i32>) -> tensor<1xi32>")
        k = self.emit(f"stablehlo.concatenate {lo1}, {hi1}, dim = 0 : (tensor<1xi32>, tensor<1xi32>) -> tensor<2xi32>")
        return self.bitcast(k, (2,), "i32", "f32")

    def _halves(self, key: str) -> Tuple[str, str]:
        k = self.bitcast(key, (2,), "f32", "i32")
        lo1 = self.emit(f"stablehlo.slice {k} [0:1:1] : (tensor<2xi32>) -> tensor<1xi32>")
        lo = self.emit(f"stablehlo.reshape {lo1} : (tensor<1xi32>) -> tensor<i32>")
        hi1 = self.emit(f"stablehlo.slice {k} [1:2:1] : (tensor<2xi32>) -> tensor<1xi32>")
        hi = self.emit(f"stablehlo.reshape {hi1} : (tensor<1xi32>) -> tensor<i32>")
        return lo, hi

    def split(self, key: str, n: int) -> List[str]:
        lo, hi = self._halves(key)
        c_mult, c_add = self.const_i32(2069105475), self.const_i32(1013904223)
        keys = []
        for i in range(n):
            off = lo if i == 0 else self.emit(f"stablehlo.add {lo}, {self.const_i32(i)} : tensor<i32>")
            mul = self.emit(f"stablehlo.multiply {off}, {c_mult} : tensor<i32>")
            nlo = self.emit(f"stablehlo.add {mul}, {c_add} : tensor<i32>")
            nhi = self.emit(f"stablehlo.add {hi}, {off} : tensor<i32>")
            lo1 = self.emit(f"stablehlo.reshape {nlo} : (tensor<i32>) -> tensor<1xi32>")
            hi1 = self.emit(f"stablehlo.reshape {nhi} : (tensor<i32>) -> tensor<1xi32>")
            k = self.emit(f"stablehlo.concatenate {lo1}, {hi1}, dim = 0 : (tensor<1xi32>, tensor<1xi32>) -> tensor<2xi32>")
            keys.append(self.bitcast(k, (2,), "i32", "f32"))
        return keys

    # --- samples -------------------------------------------------------------
    def _uniform_flat(self, key: str, n: int) -> str:
        """u in [0, 1) for the hash of iota(n) under key (f32 tensor<n>)."""
        lo, hi = self._halves(key)
        it = self.emit(f"stablehlo.iota dim = 0 : {_ty((n,), 'i32')}")
        lob, hib = self.bcast(lo, (n,), "i32"), self.bcast(hi, (n,), "i32")
        c1 = self.bcast(self.const_i32(1540483477), (n,), "i32")
        x0 = self.emit(f"stablehlo.add {it}, {lob} : {_ty((n,), 'i32')}")
        x1 = self.emit(f"stablehlo.multiply {x0}, {c1} : {_ty((n,), 'i32')}")
        x2 = self.emit(f"stablehlo.add {x1}, {hib} : {_ty((n,), 'i32')}")
        c2 = self.bcast(self.const_i32(668265263), (n,), "i32")
        c3 = self.bcast(self.const_i32(1013904223), (n,), "i32")
        x3 = self.emit(f"stablehlo.multiply {x2}, {c2} : {_ty((n,), 'i32')}")
        x4 = self.emit(f"stablehlo.add {x3}, {c3} : {_ty((n,), 'i32')}")
        ax = self.emit(f"stablehlo.abs {x4} : {_ty((n,), 'i32')}")
        fx = self.emit(f"stablehlo.convert {ax} : ({_ty((n,), 'i32')}) -> {_ty((n,), 'f32')}")
        mx = self.bcast(self.const_f32(2147483648.0), (n,), "f32")
        return self.emit(f"stablehlo.divide {fx}, {mx} : {_ty((n,), 'f32')}")

    def _shaped(self, flat: str, n: int, shape) -> str:
        if len(shape) == 1 and shape[0] == n:
            return flat
        return self.emit(f"stablehlo.reshape {flat} : ({_ty((n,), 'f32')}) -> {_ty(shape, 'f32')}")

    def uniform(self, key: str, shape) -> str:
        n = int(math.prod(shape))
        return self._shaped(self._uniform_flat(key, n), n, shape)

    def normal(self, key: str, shape) -> str:
        n = int(math.prod(shape))
        u = self._uniform_flat(key, 2 * n)
        t1, t2 = _ty((2 * n,), "f32"), _ty((n,), "f32")
        u1 = self.emit(f"stablehlo.slice {u} [0:{n}:1] : ({t1}) -> {t2}")
        u2 = self.emit(f"stablehlo.slice {u} [{n}:{2 * n}:1] : ({t1}) -> {t2}")
        eps = self.bcast(self.const_f32(1e-7), (n,), "f32")
        us = self.emit(f"stablehlo.add {u1}, {eps} : {t2}")
        lg = self.emit(f"stablehlo.log {us} : {t2}")
        m2 = self.bcast(self.const_f32(-2.0), (n,), "f32")
        ml = self.emit(f"stablehlo.multiply {m2}, {lg} : {t2}")
        rad = self.emit(f"stablehlo.sqrt {ml} : {t2}")
        tau = self.bcast(self.const_f32(2.0 * math.pi), (n,), "f32")
        th = self.emit(f"stablehlo.multiply {tau}, {u2} : {t2}")
        ct = self.emit(f"stablehlo.cosine {th} : {t2}")
        flat = self.emit(f"stablehlo.multiply {rad}, {ct} : {t2}")
        return self._shaped(flat, n, shape)

    def randint(self, key: str, shape, low: int, high: int) -> str:
        n = int(math.prod(shape))
        t = _ty((n,), "f32")
        u = self._uniform_flat(key, n)
        rng = self.bcast(self.const_f32(float(high - low)), (n,), "f32")
        sc = self.emit(f"stablehlo.multiply {u}, {rng} : {t}")
        fl = self.emit(f"stablehlo.floor {sc} : {t}")
        lo = self.bcast(self.const_f32(float(low)), (n,), "f32")
        sh = self.emit(f"stablehlo.add {fl}, {lo} : {t}")
        hm = self.bcast(self.const_f32(float(high - 1)), (n,), "f32")
        cl = self.emit(f"stablehlo.clamp {lo}, {sh}, {hm} : {t}")
        return self._shaped(cl, n, shape)

    def scale(self, x: str, shape, c: float) -> str:
        cb = self.bcast(self.const_f32(c), shape, "f32")
        return self.emit(f"stablehlo.multiply {x}, {cb} : {_ty(shape, 'f32')}")

    def ones(self, shape) -> str:
        return self.bcast(self.const_f32(1.0), shape, "f32")


def _module(name: str, args: List[Tuple[str, str]], body: List[str], rets: List[Tuple[str, str]]) -> Lowered:
    ps = ", ".join(f"%arg{i}: {t}" for i, (_, t) in enumerate(args))
    rt = rets[0][1] if len(rets) == 1 else "(" + ", ".join(t for _, t in rets) + ")"
    lines = [f"module @{name} {{", f" func.func @main({ps}) -> {rt} {{"] + body
    lines.append(f"    return {', '.join(r for r, _ in rets)} : {', '.join(t for _, t in rets)}")
    lines += [" }", "}"]
    return Lowered("\n".join(lines) + "\n", name, "main", [a for a, _ in args], [], [])


def sample_program(kind: str, shape, low: int = 0, high: int = 10, seed: int = None) -> Lowered:
    """One random op on a key argument (or, with `seed`, on random-key(seed))."""
    e = RandomEmitter()
    key = e.key_from_seed(seed) if seed is not None else "%arg0"
    if kind == "normal":
        out = e.normal(key, shape)
    elif kind == "uniform":
        out = e.uniform(key, shape)
    elif kind == "randint":
        out = e.randint(key, shape, low, high)
    elif kind == "split":
        keys = e.split(key, 4)
        return _module(f"rng_split_{len(e.lines)}", [] if seed is not None else [("key", "tensor<2xf32>")],
                       e.lines, [(k, "tensor<2xf32>") for k in keys])
    else:
        raise ValueError(kind)
    return _module(f"rng_{kind}_{'x'.join(map(str, shape))}", [] if seed is not None else [("key", "tensor<2xf32>")],
                   e.lines, [(out, _ty(shape, "f32"))])


def gpt_init_program(c) -> Lowered:
    """`(init-gpt-params key config)` (examples/nanoGPT/model.shf:17-43) as one
    device function of the key, returning the parameter leaves in Sheaf's
    sorted-key order (the order the value-and-grad functions take them)."""
    e = RandomEmitter()
    V, D, B, L = c.vocab_size, c.n_embd, c.block_size, c.n_layer
    k_wte, k_wpe, k_blocks, k_head = e.split("%arg0", 4)
    block_keys = e.split(k_blocks, L)
    leaves = {}
    for i, bk in enumerate(block_keys):
        k_attn, k_proj, k_fc, k_fc2 = e.split(bk, 4)
        p = f"transformer.h.{i}."
        leaves[p + "attn.c_attn.weight"] = (e.scale(e.normal(k_attn, (3 * D, D)), (3 * D, D), 0.02), (3 * D, D))
        leaves[p + "attn.c_proj.weight"] = (e.scale(e.normal(k_proj, (D, D)), (D, D), 0.02), (D, D))
        leaves[p + "mlp.c_fc.weight"] = (e.scale(e.normal(k_fc, (4 * D, D)), (4 * D, D), 0.02), (4 * D, D))
        leaves[p + "mlp.c_proj.weight"] = (e.scale(e.normal(k_fc2, (D, 4 * D)), (D, 4 * D), 0.02), (D, 4 * D))
        leaves[p + "ln_1.weight"] = (e.ones((D,)), (D,))
        leaves[p + "ln_2.weight"] = (e.ones((D,)), (D,))
    leaves["transformer.wte.weight"] = (e.scale(e.normal(k_wte, (V, D)), (V, D), 0.02), (V, D))
    leaves["transformer.wpe.weight"] = (e.scale(e.normal(k_wpe, (B, D)), (B, D), 0.02), (B, D))
    leaves["transformer.ln_f.weight"] = (e.ones((D,)), (D,))
    leaves["lm_head.weight"] = (e.scale(e.normal(k_head, (V, D)), (V, D), 0.02), (V, D))
    rets = [(leaves[k][0], _ty(leaves[k][1], "f32")) for k in sorted(leaves)]
    low = _module(f"init_gpt_L{L}_D{D}", [("key", "tensor<2xf32>")], e.lines, rets)
    low.result_names = sorted(leaves)
    return low


def key_of_seed(seed: int):
    """Host value of random-key(seed): the two i32 halves' bits as f32."""
    import numpy as np
    return np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], dtype=np.uint32).view(np.float32)
