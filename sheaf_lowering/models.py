"""Sheaf programs of the benchmark configurations, lowered as Sheaf lowers them.

Each builder records the *inlined* Sheaf body on a Tracer: stdlib functions
(`gelu`, `softmax`, `log-softmax`, `cross-entropy-loss`, `mse-loss`,
`linear`) are expanded into their primitive calls exactly as written in
sheaf/lib/nn.shf:14-134, and the GPT model follows
examples/nanoGPT/model.shf:11-113 (`layer-norm-nb`, `causal-self-attention`,
`mlp-block`, `transformer-block`, `gpt-forward`).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Tuple

import numpy as np

from .lower import Kw, Lowered, Sym, Ty, Vec, lower_forward, lower_value_and_grad

KEEP = Kw("keepdims")
AXIS = Kw("axis")


# ---------------------------------------------------------------------------
# stdlib composites (sheaf/lib/nn.shf)
# ---------------------------------------------------------------------------

def gelu(t, x):
    # (* 0.5 (* x (+ 1.0 (tanh (* 0.7978846 (+ x (* 0.044715 (* x (* x x)))))))))
    return t("*", 0.5, t("*", x, t("+", 1.0, t("tanh", t("*", 0.7978846,
             t("+", x, t("*", 0.044715, t("*", x, t("*", x, x)))))))))


def relu(t, x):
    return t("maximum", x, 0.0)


def sigmoid(t, x):
    return t("/", 1.0, t("+", 1.0, t("exp", t("-", 0, x))))


def softmax(t, x):
    e = t("exp", t("-", x, t("max", x, AXIS, -1, KEEP)))
    return t("/", e, t("sum", e, AXIS, -1, KEEP))


def log_softmax(t, x):
    s = t("-", x, t("max", x, AXIS, -1, KEEP))
    return t("-", s, t("log", t("sum", t("exp", s), AXIS, -1, KEEP)))


def cross_entropy_loss(t, logits, targets):
    V = t.shape(logits)[-1]
    log_p = log_softmax(t, t("reshape", logits, Vec([-1, V])))
    flat = t("reshape", targets, Vec([-1]))
    mask = t("one-hot", flat, V)
    tlp = t("sum", t("*", log_p, mask), AXIS, -1)
    return t("*", t("mean", tlp), -1.0)


def layer_norm(t, x, gamma, beta, axis=-1):
    m = t("mean", x, AXIS, axis, KEEP)
    v = t("var", x, AXIS, axis, KEEP)
    return t("+", t("*", t("/", t("-", x, m), t("sqrt", t("+", v, 1e-5))), gamma), beta)


def mse_loss(t, pred, true):
    d = t("-", pred, true)
    return t("mean", t("*", d, d))


def linear(t, x, w, b):
    return t("+", t("@", x, w), b)


# ---------------------------------------------------------------------------
# GPT (examples/nanoGPT/model.shf, benchmarks/bench_vag_sheaf.shf)
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class GPTConfig:
    n_layer: int
    n_head: int
    n_embd: int
    block_size: int
    vocab_size: int
    batch: int
    seq: int = 0

    @property
    def T(self):
        return self.seq or self.block_size

    @property
    def tokens(self):
        return self.batch * self.T


NANOGPT = GPTConfig(n_layer=6, n_head=6, n_embd=384, block_size=256, vocab_size=65, batch=64)
GPT2_SMALL = GPTConfig(n_layer=12, n_head=12, n_embd=768, block_size=1024, vocab_size=50304, batch=8)


def gpt_param_leaves(c: GPTConfig) -> List[Tuple[str, tuple]]:
    """Flattened parameter leaves in Sheaf's sorted-key order
    (dict keys sorted, lists in order: sheaf/src/runtime/buffer_convert.rs:191-224)."""
    D, V = c.n_embd, c.vocab_size
    leaves = [("lm_head.weight", (V, D))]
    for i in range(c.n_layer):
        p = f"transformer.h.{i}."
        leaves += [(p + "attn.c_attn.weight", (3 * D, D)),
                   (p + "attn.c_proj.weight", (D, D)),
                   (p + "ln_1.weight", (D,)),
                   (p + "ln_2.weight", (D,)),
                   (p + "mlp.c_fc.weight", (4 * D, D)),
                   (p + "mlp.c_proj.weight", (D, 4 * D))]
    leaves += [("transformer.ln_f.weight", (D,)),
               ("transformer.wpe.weight", (c.block_size, D)),
               ("transformer.wte.weight", (V, D))]
    return leaves


def layer_norm_nb(t, x, gamma):
    m = t("mean", x, AXIS, -1, KEEP)
    v = t("var", x, AXIS, -1, KEEP)
    return t("*", t("/", t("-", x, m), t("sqrt", t("+", v, 1e-5))), gamma)


def causal_self_attention(t, x, p, prefix, c: GPTConfig):
    D, H = c.n_embd, c.n_head
    Hd = D // H
    T = t.shape(x)[-2]
    W = p[prefix + "attn.c_attn.weight"]
    Wq = t("slice", W, 0, D)
    Wk = t("slice", W, D, 2 * D)
    Wv = t("slice", W, 2 * D, 3 * D)
    q = t("swapaxes", t("reshape", t("@", x, t("tr", Wq)), Vec([-1, T, H, Hd])), 1, 2)
    k = t("swapaxes", t("reshape", t("@", x, t("tr", Wk)), Vec([-1, T, H, Hd])), 1, 2)
    v = t("swapaxes", t("reshape", t("@", x, t("tr", Wv)), Vec([-1, T, H, Hd])), 1, 2)
    scores = t("/", t("@", q, t("swapaxes", k, -1, -2)), t("sqrt", float(Hd)))
    mask = t("==", t("tril", t("ones", Vec([T, T]))), 1.0)
    att = softmax(t, t("where", mask, scores, -1e10))
    y = t("reshape", t("swapaxes", t("@", att, v), 1, 2), Vec([-1, T, D]))
    return t("@", y, t("tr", p[prefix + "attn.c_proj.weight"]))


def mlp_block(t, x, p, prefix):
    h = gelu(t, t("@", x, t("tr", p[prefix + "mlp.c_fc.weight"])))
    return t("@", h, t("tr", p[prefix + "mlp.c_proj.weight"]))


def transformer_block(t, x, p, i, c):
    prefix = f"transformer.h.{i}."
    h = t("+", x, causal_self_attention(t, layer_norm_nb(t, x, p[prefix + "ln_1.weight"]), p, prefix, c))
    return t("+", h, mlp_block(t, layer_norm_nb(t, h, p[prefix + "ln_2.weight"]), p, prefix))


def gpt_forward(t, idx, p, c: GPTConfig):
    T = t.shape(idx)[-1]
    D = c.n_embd
    wte = p["transformer.wte.weight"]
    wpe = p["transformer.wpe.weight"]
    x = t("+", t("get", wte, idx), t("reshape", t("slice", wpe, 0, T), Vec([1, T, D])))
    for i in range(c.n_layer):
        x = transformer_block(t, x, p, i, c)
    x = layer_norm_nb(t, x, p["transformer.ln_f.weight"])
    return t("@", x, t("tr", p["lm_head.weight"]))


def gpt_vag(c: GPTConfig, batch: int = None) -> Lowered:
    """`((value-and-grad (fn [p] (cross-entropy-loss (gpt-forward x p config) y))) params)`
    (examples/nanoGPT/train.shf:26-28)."""
    B = batch if batch is not None else c.batch
    leaves = gpt_param_leaves(c)

    def build(t, s):
        logits = gpt_forward(t, s["x"], s, c)
        return cross_entropy_loss(t, logits, s["y"])
    return lower_value_and_grad(build, leaves, [("x", (B, c.T)), ("y", (B, c.T))],
                                key=f"gpt-vag-{c}-{B}")


def gpt_fwd(c: GPTConfig, batch: int = None) -> Lowered:
    """`(gpt-forward idx params config)` as a JIT forward function."""
    B = batch if batch is not None else c.batch
    args = gpt_param_leaves(c) + [("idx", (B, c.T))]

    def build(t, s):
        return gpt_forward(t, s["idx"], s, c)
    return lower_forward(build, args, "gpt_forward", key=f"gpt-fwd-{c}-{B}")


def gpt_inputs(c: GPTConfig, batch: int = None, seed: int = 0) -> Dict[str, np.ndarray]:
    """Seeded synthetic inputs: weights N(0, 0.02), LN gammas 1, tokens U[0, V)
    (examples/nanoGPT/model.shf:18-43); y = x shifted by one token within a
    longer random stream (examples/nanoGPT/train.shf:15-21)."""
    B = batch if batch is not None else c.batch
    rng = np.random.default_rng(seed)
    out = {}
    for n, s in gpt_param_leaves(c):
        if n.endswith(("ln_1.weight", "ln_2.weight", "ln_f.weight")):
            out[n] = np.ones(s, np.float32)
        else:
            out[n] = (rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    stream = rng.integers(0, c.vocab_size, size=(B, c.T + 1))
    out["x"] = stream[:, :-1].astype(np.float32)
    out["y"] = stream[:, 1:].astype(np.float32)
    out["idx"] = out["x"]
    return out


# ---------------------------------------------------------------------------
# The reference's own benchmark programs (benchmarks/bench_vag_sheaf.shf,
# benchmarks/bench_forward.shf): GPT-2 124M (12 layers, d768, 12 heads,
# vocabulary 50257, block 1024) on one sequence of 64 tokens; the value-and-
# grad program's loss is the mean of the logits.  The model code is the same
# as examples/nanoGPT's (`(transpose W)` of a matrix is `(tr W)`).
# ---------------------------------------------------------------------------

GPT2_BENCH = GPTConfig(n_layer=12, n_head=12, n_embd=768, block_size=1024, vocab_size=50257, batch=1, seq=64)


def bench_vag_program(c: GPTConfig = GPT2_BENCH) -> Lowered:
    """`(value-and-grad (fn [p] (mean (forward idx p config))))`
    (benchmarks/bench_vag_sheaf.shf:86-101)."""
    leaves = gpt_param_leaves(c)

    def build(t, s):
        return t("mean", gpt_forward(t, s["idx"], s, c))
    return lower_value_and_grad(build, leaves, [("idx", (c.batch, c.T))], key=f"bench-vag-{c}")


def bench_forward_program(c: GPTConfig = GPT2_BENCH) -> Lowered:
    """`(forward idx params config)` (benchmarks/bench_forward.shf:75-87)."""
    args = gpt_param_leaves(c) + [("idx", (c.batch, c.T))]

    def build(t, s):
        return gpt_forward(t, s["idx"], s, c)
    return lower_forward(build, args, "forward", key=f"bench-fwd-{c}")


def bench_inputs(c: GPTConfig = GPT2_BENCH, seed: int = 42) -> Dict[str, np.ndarray]:
    """Seeded stand-ins for init-params (bench_vag_sheaf.shf:57-76): matrices
    N(0, 1) / sqrt(fan-in) (sqrt(D), or sqrt(4 D) for mlp.c_proj), LN gammas 1,
    lm_head equal to wte (both drawn from key k1 there); idx U[0, V) of
    [1, 64]."""
    rng = np.random.default_rng(seed)
    D = c.n_embd
    out = {}
    for n, shp in gpt_param_leaves(c):
        if n.endswith(("ln_1.weight", "ln_2.weight", "ln_f.weight")):
            out[n] = np.ones(shp, np.float32)
        elif n == "lm_head.weight":
            continue
        else:
            scale = np.sqrt(4 * D) if n.endswith("mlp.c_proj.weight") else np.sqrt(D)
            out[n] = (rng.standard_normal(shp, dtype=np.float32) / np.float32(scale)).astype(np.float32)
    out["lm_head.weight"] = out["transformer.wte.weight"].copy()
    out["idx"] = rng.integers(0, c.vocab_size, size=(c.batch, c.T)).astype(np.float32)
    return out


# ---------------------------------------------------------------------------
# MLP value-and-grad: linear -> gelu -> linear, mse-loss
# ---------------------------------------------------------------------------

MLP_SHAPES = {"x": (256, 784), "W1": (784, 512), "W2": (512, 10), "b1": (512,), "b2": (10,)}


def mlp_vag(batch: int = 256) -> Lowered:
    leaves = [("W1", (784, 512)), ("W2", (512, 10)), ("b1", (512,)), ("b2", (10,))]

    def build(t, s):
        h = gelu(t, linear(t, s["x"], s["W1"], s["b1"]))
        return mse_loss(t, linear(t, h, s["W2"], s["b2"]), s["y"])
    return lower_value_and_grad(build, leaves, [("x", (batch, 784)), ("y", (batch, 10))],
                                key=f"mlp-vag-{batch}")


def mlp_inputs(batch: int = 256, seed: int = 0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    lim1 = np.sqrt(6.0 / (784 + 512))
    lim2 = np.sqrt(6.0 / (512 + 10))
    labels = rng.integers(0, 10, size=batch)
    y = np.zeros((batch, 10), np.float32)
    y[np.arange(batch), labels] = 1.0
    return {
        "x": rng.standard_normal((batch, 784), dtype=np.float32),
        "y": y,
        "W1": rng.uniform(-lim1, lim1, (784, 512)).astype(np.float32),
        "W2": rng.uniform(-lim2, lim2, (512, 10)).astype(np.float32),
        "b1": np.zeros(512, np.float32),
        "b2": np.zeros(10, np.float32),
    }


# ---------------------------------------------------------------------------
# Op-level sweep: softmax and layer-norm on [R, D], gelu on [N], each forward
# and VJP.  The VJP is Sheaf's value-and-grad of sum(op(x) * g) with respect
# to x, for a captured cotangent g: its gradient output is VJP_op(x, g).
# ---------------------------------------------------------------------------

SWEEP_OPS = ("softmax", "layer-norm", "gelu")


def _sweep_body(op, t, s):
    if op == "softmax":
        return softmax(t, s["x"])
    if op == "layer-norm":
        return layer_norm(t, s["x"], s["gamma"], s["beta"])
    if op == "gelu":
        return gelu(t, s["x"])
    raise ValueError(op)


def sweep_program(op: str, shape: Tuple[int, ...], vjp: bool, dtype: str = "f32") -> Lowered:
    """`(op x)` as a JIT forward function, or `((value-and-grad (fn [x] (sum
    (* (op x) g)))) x)`.  dtype "bf16": the same program on bf16 tensors (every
    tensor type of the f32 text, constants included, as bf16: each op then
    rounds its result to bf16, as Sheaf's bf16 tensors compute)."""
    D = shape[-1]
    extra = [("gamma", (D,)), ("beta", (D,))] if op == "layer-norm" else []
    key = f"sweep-{op}-{'x'.join(map(str, shape))}-{'vjp' if vjp else 'fwd'}"
    if vjp:
        def build(t, s):
            return t("sum", t("*", _sweep_body(op, t, s), s["g"]))
        low = lower_value_and_grad(build, [("x", shape)], [("g", shape)] + extra, key=key)
    else:
        def build(t, s):
            return _sweep_body(op, t, s)
        low = lower_forward(build, [("x", shape)] + extra, op.replace("-", "_"), key=key)
    if dtype == "f32":
        return low
    if dtype != "bf16":
        raise ValueError(dtype)
    import re
    text = re.sub(r"(tensor<(?:[0-9]+x)*)f32>", r"\1bf16>", low.text)
    text = text.replace(low.module, low.module + "_bf16")
    bf = [Ty(t.shape, "bf16") for t in low.arg_types]
    rf = [Ty(t.shape, "bf16") for t in low.result_types]
    return Lowered(text, low.module + "_bf16", low.function, low.arg_names, bf, rf)


def sweep_inputs(op: str, shape: Tuple[int, ...], vjp: bool, seed: int = 0) -> Dict[str, np.ndarray]:
    """Seeded N(0, 1) inputs (and cotangent); layer-norm gamma 1, beta 0."""
    rng = np.random.default_rng(seed)
    out = {"x": rng.standard_normal(shape, dtype=np.float32)}
    if vjp:
        out["g"] = rng.standard_normal(shape, dtype=np.float32)
    if op == "layer-norm":
        out["gamma"] = np.ones(shape[-1], np.float32)
        out["beta"] = np.zeros(shape[-1], np.float32)
    return out
