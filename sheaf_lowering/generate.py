"""`generate-token` (examples/nanoGPT/model.shf:116-125) as one device
function: gpt-forward on the [1, T] window, the last position's logits / temp,
top_k (stablehlo.sort of the logits with an iota payload, descending, stable,
then the first K: lowering/stablehlo/indexing_ops.rs:476-540), softmax,
random-split of the key, `choice` (random_ops.rs:758-833: u from the subkey's
low half, cumulative sum as tril(ones) @ probs, index = K - count(cumsum >= u),
clamped) and the chosen token id (gather of the top-k indices).  Returns
(next_id, new_key), the {:next_id :key} map of the reference.
"""
from __future__ import annotations

import re

from . import models as M
from .lower import SCALAR, Emitter, Lowered, Ty
from .random import RandomEmitter


def _tail(e: Emitter, rng: RandomEmitter, logits: str, T: int, V: int, top_k: int, temp: float, key: str):
    K = min(top_k, V)
    row = e.fresh()
    e.line(f"    {row} = stablehlo.slice {logits} [0:1:1, {T - 1}:{T}:1, 0:{V}:1] : "
           f"(tensor<1x{T}x{V}xf32>) -> tensor<1x1x{V}xf32>")
    last = e.fresh()
    e.line(f"    {last} = stablehlo.reshape {row} : (tensor<1x1x{V}xf32>) -> tensor<{V}xf32>")
    vt = Ty((V,))
    scaled, _ = e.binop("/", last, e.constant_f32(temp), vt, SCALAR)
    # top_k: sort descending with an iota payload, keep the first K
    io = e.fresh()
    e.line(f"    {io} = stablehlo.iota dim = 0 : tensor<{V}xi32>")
    sv, si = e.fresh(), e.fresh()
    a, b, c_, d, p = (e.fresh() for _ in range(5))
    e.line(f'    {sv}, {si} = "stablehlo.sort"({scaled}, {io}) ({{\n'
           f"    ^bb0({a}: tensor<f32>, {b}: tensor<f32>, {c_}: tensor<i32>, {d}: tensor<i32>):\n"
           f'      {p} = "stablehlo.compare"({a}, {b}) {{comparison_direction = #stablehlo<comparison_direction GT>}} '
           f": (tensor<f32>, tensor<f32>) -> tensor<i1>\n"
           f'      "stablehlo.return"({p}) : (tensor<i1>) -> ()\n'
           f"    }}) {{dimension = 0 : i64, is_stable = true}} : (tensor<{V}xf32>, tensor<{V}xi32>) -> "
           f"(tensor<{V}xf32>, tensor<{V}xi32>)")
    tv, tvt = e.slice_axis(sv, vt, 0, K, 0)
    ti = e.fresh()
    e.line(f"    {ti} = stablehlo.slice {si} [0:{K}:1] : (tensor<{V}xi32>) -> tensor<{K}xi32>")
    kt = Ty((K,))
    tif = e.convert(ti, Ty((K,), "i32"), kt)
    # softmax over the K values (lib/nn.shf:28-30)
    mx, mt = e.reduce_max(tv, tvt, -1, True)
    dlt, dt = e.binop("-", tv, mx, tvt, mt)
    ex = e.unary("exp", dlt, dt)
    sm, st = e.reduce_sum(ex, dt, -1, True)
    probs, _ = e.binop("/", ex, sm, dt, st)
    # [new-key subkey] (random-split key)
    new_key, subkey = rng.split(key, 2)
    # choice: u from the subkey's low half
    kb = rng.bitcast(subkey, (2,), "f32", "i32")
    lo1 = rng.emit(f"stablehlo.slice {kb} [0:1:1] : (tensor<2xi32>) -> tensor<1xi32>")
    lo = rng.emit(f"stablehlo.reshape {lo1} : (tensor<1xi32>) -> tensor<i32>")
    ab = rng.emit(f"stablehlo.abs {lo} : tensor<i32>")
    uf = rng.emit(f"stablehlo.convert {ab} : (tensor<i32>) -> tensor<f32>")
    u = rng.emit(f"stablehlo.divide {uf}, {rng.const_f32(2147483648.0)} : tensor<f32>")
    ones, ot = e.splat(1.0, (K, K))
    tri, tt = e.tril(ones, ot)
    cs, cst = e.matmul(tri, probs, tt, kt)
    mask, mkt = e.compare(">=", cs, u, cst, SCALAR)
    cnt, _ = e.reduce_sum(mask, mkt, 0, False)
    idx, _ = e.binop("-", e.constant_f32(float(K)), cnt, SCALAR, SCALAR)
    cl = e.fresh()
    e.line(f"    {cl} = stablehlo.clamp {e.constant_f32(0.0)}, {idx}, {e.constant_f32(float(K - 1))} : tensor<f32>")
    nid, _ = e.gather_axis0(tif, kt, cl, SCALAR)
    return nid, new_key


def gpt_generate_program(c, top_k: int = 200, temp: float = 0.8) -> Lowered:
    """One generation step on a [1, T] token window (T = block size)."""
    fwd = M.gpt_fwd(c, batch=1)
    lines = fwd.text.splitlines()
    fi = next(i for i, l in enumerate(lines) if "func.func" in l)
    ri = next(i for i in range(len(lines) - 1, -1, -1) if lines[i].strip().startswith("return"))
    logits = lines[ri].split()[1]
    body = lines[fi + 1:ri]
    top = max(int(n) for n in re.findall(r"%(\d+)\b", "\n".join(body)))
    e = Emitter()
    e.counter = top + 1
    rng = RandomEmitter()
    n_args = len(fwd.arg_names)
    key = f"%arg{n_args}"
    nid, new_key = _tail(e, rng, logits, c.T, c.vocab_size, top_k, temp, key)
    sig = lines[fi]
    m = re.match(r"(\s*func\.func @)\w+\((.*)\)\s*->\s*.*\{\s*$", sig)
    params = m.group(2) + f", {key}: tensor<2xf32>"
    # the emitters interleave: keep the random ops before their first use by
    # emitting them first (they depend only on the key argument)
    head = [l.replace(f"module @{fwd.module} ", f"module @{fwd.module}_gen ") for l in lines[:fi]]
    out = head + [f"{m.group(1)}generate_token({params}) -> (tensor<f32>, tensor<2xf32>) {{"]
    out += body + rng.lines + e.body
    out += [f"    return {nid}, {new_key} : tensor<f32>, tensor<2xf32>", " }", "}"]
    return Lowered("\n".join(out) + "\n", fwd.module + "_gen", "generate_token", fwd.arg_names + ["key"], [], [])


# ---------------------------------------------------------------------------
# Decoding with a key/value cache (the roadmap's KV-cache item,
# docs/roadmap.md:40-41; the reference's sample.shf reruns the whole window):
# one new token at position `pos` per call.  Each layer's cache holds the keys
# and values of positions 0..T-1 ([H, T, 64]); the call writes this
# position's key and value into it (a 0/1 blend with one_hot(pos), exact in
# float) and attends over positions <= pos (one_hot(pos) @ tril(ones) marks
# them).  Fed a prompt one token at a time, the logits at position p equal the
# full forward's logits at p on the prefix 0..p.
# ---------------------------------------------------------------------------

def cache_leaves(c):
    Hd = c.n_embd // c.n_head
    out = []
    for i in range(c.n_layer):
        out += [(f"cache.{i}.k", (c.n_head, c.T, Hd)), (f"cache.{i}.v", (c.n_head, c.T, Hd))]
    return out


def _decode_forward(t, s, c):
    from .lower import Vec
    D, H, T = c.n_embd, c.n_head, c.T
    Hd = D // H
    tok, pos = s["token"], s["pos"]
    x = t("+", t("get", s["transformer.wte.weight"], tok),
          t("reshape", t("get", s["transformer.wpe.weight"], pos), Vec([1, 1, D])))
    oh = t("one-hot", pos, T)                                   # [1, T]
    valid = t("@", oh, t("tril", t("ones", Vec([T, T]))))       # positions <= pos
    m3 = t("reshape", oh, Vec([1, T, 1]))
    keep = t("-", 1.0, m3)
    caches = []
    for i in range(c.n_layer):
        p = f"transformer.h.{i}."
        h = M.layer_norm_nb(t, x, s[p + "ln_1.weight"])
        W = s[p + "attn.c_attn.weight"]

        def heads(w):
            return t("swapaxes", t("reshape", t("@", h, t("tr", w)), Vec([1, H, Hd])), 0, 1)  # [H, 1, Hd]
        q = heads(t("slice", W, 0, D))
        k = heads(t("slice", W, D, 2 * D))
        v = heads(t("slice", W, 2 * D, 3 * D))
        K = t("+", t("*", s[f"cache.{i}.k"], keep), t("*", k, m3))
        Vc = t("+", t("*", s[f"cache.{i}.v"], keep), t("*", v, m3))
        att = t("/", t("@", q, t("swapaxes", K, -1, -2)), t("sqrt", float(Hd)))    # [H, 1, T]
        att = M.softmax(t, t("where", t("==", valid, 1.0), att, -1e10))
        y = t("reshape", t("swapaxes", t("@", att, Vc), 0, 1), Vec([1, 1, D]))
        x = t("+", x, t("@", y, t("tr", s[p + "attn.c_proj.weight"])))
        x = t("+", x, M.mlp_block(t, M.layer_norm_nb(t, x, s[p + "ln_2.weight"]), s, p))
        caches += [K, Vc]
    x = M.layer_norm_nb(t, x, s["transformer.ln_f.weight"])
    return [t("@", x, t("tr", s["lm_head.weight"]))] + caches   # logits [1, 1, V]


def gpt_decode_forward_program(c) -> Lowered:
    """The decoding step's forward: (params..., caches..., token [1, 1], pos [1])
    -> (logits [1, 1, V], caches...)."""
    from .lower import lower_forward
    args = M.gpt_param_leaves(c) + cache_leaves(c) + [("token", (1, 1)), ("pos", (1,))]
    return lower_forward(lambda t, s: _decode_forward(t, s, c), args, "decode_fwd", key=f"gpt-decode-{c}")


def gpt_decode_program(c, top_k: int = 200, temp: float = 0.8) -> Lowered:
    """One decoding step: (params..., caches..., token [1, 1], pos [1], key) ->
    (next_id, new_key, caches...), sampling as generate-token does."""
    fwd = gpt_decode_forward_program(c)
    lines = fwd.text.splitlines()
    fi = next(i for i, l in enumerate(lines) if "func.func" in l)
    ri = next(i for i in range(len(lines) - 1, -1, -1) if lines[i].strip().startswith("return"))
    ret = lines[ri].strip()[len("return"):].split(":")[0]
    vals = [x.strip() for x in ret.split(",")]
    logits, cache_vals = vals[0], vals[1:]
    body = lines[fi + 1:ri]
    top = max(int(n) for n in re.findall(r"%(\d+)\b", "\n".join(body)))
    e = Emitter()
    e.counter = top + 1
    rng = RandomEmitter()
    key = f"%arg{len(fwd.arg_names)}"
    nid, new_key = _tail(e, rng, logits, 1, c.vocab_size, top_k, temp, key)
    sig = lines[fi]
    m = re.match(r"(\s*func\.func @)\w+\((.*)\)\s*->\s*.*\{\s*$", sig)
    params = m.group(2) + f", {key}: tensor<2xf32>"
    Hd = c.n_embd // c.n_head
    ct = f"tensor<{c.n_head}x{c.T}x{Hd}xf32>"
    head = [l.replace(f"module @{fwd.module} ", f"module @{fwd.module}_dec ") for l in lines[:fi]]
    res_types = ", ".join(["tensor<f32>", "tensor<2xf32>"] + [ct] * len(cache_vals))
    out = head + [f"{m.group(1)}decode_token({params}) -> ({res_types}) {{"]
    out += body + rng.lines + e.body
    out += [f"    return {', '.join([nid, new_key] + cache_vals)} : {res_types}", " }", "}"]
    return Lowered("\n".join(out) + "\n", fwd.module + "_dec", "decode_token", fwd.arg_names + ["key"], [], [])
