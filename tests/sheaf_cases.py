"""The reference's value-and-grad test programs, lowered to StableHLO text.

Each case restates one Sheaf test expression (sheaf/tests/vag_tests.yaml,
sheaf/tests/interpreter_tests.yaml:753-762, README.md:33-43) as tracer calls,
with stdlib functions inlined the way Sheaf's JIT inlines sheaf/lib/nn.shf.
`CASES[name]()` returns (Lowered module, list of inputs in argument order).
"""
import numpy as np

from sheaf_lowering import models as M
from sheaf_lowering.lower import Kw, Vec, lower_value_and_grad

AX, KEEP = Kw("axis"), Kw("keepdims")


def _vag(name, build, x, captures=()):
    x = np.asarray(x, np.float32)
    caps = [(n, np.asarray(v, np.float32).shape) for n, v in captures]
    low = lower_value_and_grad(lambda t, s: build(t, s), [("x", x.shape)], caps, key=name)
    return low, [x] + [np.asarray(v, np.float32) for _, v in captures]


def _simple(name, body, x):
    return lambda: _vag(name, lambda t, s: body(t, s["x"]), x)


CASES = {
    "vag-add": _simple("vag-add", lambda t, x: t("sum", t("+", x, Vec([10.0, 20.0]))), [1.0, 2.0]),
    "vag-sub": _simple("vag-sub", lambda t, x: t("sum", t("-", x, Vec([10.0, 20.0]))), [1.0, 2.0]),
    "vag-neg": _simple("vag-neg", lambda t, x: t("sum", t("-", x)), [1.0, 2.0]),
    "vag-mul": _simple("vag-mul", lambda t, x: t("sum", t("*", x, Vec([3.0, 4.0]))), [1.0, 2.0]),
    "vag-div": _simple("vag-div", lambda t, x: t("sum", t("/", x, Vec([2.0, 4.0]))), [1.0, 2.0]),
    "vag-pow": _simple("vag-pow", lambda t, x: t("sum", t("**", x, 3.0)), [1.0, 2.0]),
    "vag-exp": _simple("vag-exp", lambda t, x: t("sum", t("exp", x)), [0.0, 1.0]),
    "vag-log": _simple("vag-log", lambda t, x: t("sum", t("log", x)), [1.0, 2.0]),
    "vag-sqrt": _simple("vag-sqrt", lambda t, x: t("sum", t("sqrt", x)), [4.0, 9.0]),
    "vag-abs": _simple("vag-abs", lambda t, x: t("sum", t("abs", x)), [-3.0, 2.0]),
    "vag-tanh": _simple("vag-tanh", lambda t, x: t("sum", t("tanh", x)), [0.0, 1.0]),
    "vag-relu": _simple("vag-relu", lambda t, x: t("sum", M.relu(t, x)), [-1.0, 2.0]),
    "vag-sigmoid": _simple("vag-sigmoid", lambda t, x: t("sum", M.sigmoid(t, x)), [0.0]),
    "vag-gelu": _simple("vag-gelu", lambda t, x: t("sum", M.gelu(t, x)), [0.0, 1.0]),
    "vag-softmax": _simple("vag-softmax",
                           lambda t, x: t("sum", t("*", M.softmax(t, x), Vec([1.0, 0.0, 0.0]))),
                           [1.0, 2.0, 3.0]),
    "vag-log-softmax": _simple("vag-log-softmax", lambda t, x: t("sum", M.log_softmax(t, x)),
                               [1.0, 2.0, 3.0]),
    "vag-sum": _simple("vag-sum", lambda t, x: t("sum", x), [1.0, 2.0, 3.0]),
    "vag-mean": _simple("vag-mean", lambda t, x: t("mean", x), [1.0, 2.0, 3.0]),
    "vag-maximum": _simple("vag-maximum", lambda t, x: t("sum", t("maximum", x, 0.0)), [-1.0, 2.0, -3.0]),
    "vag-matmul": _simple("vag-matmul", lambda t, w: t("sum", t("@", Vec([Vec([1.0, 2.0])]), w)),
                          [[1.0, 0.0], [0.0, 1.0]]),
    "vag-einsum": _simple("vag-einsum",
                          lambda t, w: t("sum", t("einsum", "ij,jk->ik", Vec([Vec([1.0, 2.0])]), w)),
                          [[1.0, 0.0], [0.0, 1.0]]),
    "vag-slice": _simple("vag-slice", lambda t, x: t("sum", t("slice", x, 0, 2)), [1.0, 2.0, 3.0, 4.0]),
    "vag-slice-axis": _simple("vag-slice-axis", lambda t, x: t("sum", t("slice", x, 0, 2, AX, -1)),
                              [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]]),
    "vag-ce-slice": _simple("vag-ce-slice", lambda t, w: M.cross_entropy_loss(
        t, t("slice", t("@", Vec([Vec([1.0, 2.0, 3.0, 4.0])]), w), 0, 3, AX, -1), Vec([2.0])),
        np.eye(4, dtype=np.float32)),
    "vag-get-embedding": _simple("vag-get-embedding", lambda t, e: t("sum", t("get", e, Vec([0.0, 1.0]))),
                                 [[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]]),
    "vag-get-embedding-repeated": _simple("vag-get-embedding-repeated",
                                          lambda t, e: t("sum", t("get", e, Vec([0.0, 0.0, 1.0]))),
                                          [[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]]),
    "vag-where": _simple("vag-where", lambda t, x: t("sum", t("where", t(">", x, 0.0), x, t("*", x, 0.1))),
                         [-2.0, 3.0]),
    "vag-cross-entropy-loss": _simple("vag-cross-entropy-loss", lambda t, w: M.cross_entropy_loss(
        t, t("@", Vec([Vec([1.0, 2.0, 3.0])]), w), Vec([2.0])), np.eye(3, dtype=np.float32)),
    "vag-let-lambda": _simple("vag-let-lambda", lambda t, w: t("sum", t("@", Vec([Vec([1.0, 2.0])]), w)),
                              [[1.0, 0.0], [0.0, 1.0]]),
    "vag-defn-calling-defn": _simple("vag-defn-calling-defn",
                                     lambda t, w: t("sum", t("@", Vec([Vec([1.0, 2.0])]), w)),
                                     [[1.0, 0.0], [0.0, 1.0]]),
    "vag-dict-capture": _simple("vag-dict-capture",
                                lambda t, w: t("*", 0.5, t("sum", t("@", Vec([Vec([1.0, 2.0])]), w))),
                                [[1.0, 0.0], [0.0, 1.0]]),
    "vag-layer-norm": _simple("vag-layer-norm", lambda t, x: (lambda ln1, ln2: t("sum", t("*", ln1, ln2)))(
        M.layer_norm(t, x, Vec([2.0, 1.0]), Vec([0.0, 0.0])),
        M.layer_norm(t, x, Vec([2.0, 1.0]), Vec([0.0, 0.0]))), [3.0, 5.0]),
    "vag-matmul-batched-transpose": _simple(
        "vag-matmul-batched-transpose",
        lambda t, w: (lambda h: t("sum", t("@", t("@", h, w), t("transpose", t("@", h, w), Vec([0, 2, 1])))))(
            Vec([Vec([Vec([1.0, 1.0]), Vec([1.0, 1.0])]), Vec([Vec([1.0, 1.0]), Vec([1.0, 1.0])])])),
        [[1.0, 1.0], [1.0, 1.0]]),
    "vag-stop-gradient": _simple("vag-stop-gradient", lambda t, x: t("sum", t("stop-gradient", x)),
                                 [1.0, 2.0, 3.0]),
    "vag-stop-gradient-partial": _simple("vag-stop-gradient-partial",
                                         lambda t, x: t("sum", t("+", x, t("stop-gradient", x))), [1.0, 2.0]),
    "vag-stop-gradient-matmul": _simple("vag-stop-gradient-matmul",
                                        lambda t, w: t("sum", t("stop-gradient", t("@", Vec([Vec([1.0, 2.0])]), w))),
                                        [[1.0, 0.0], [0.0, 1.0]]),
    "vag-stop-gradient-baseline": _simple("vag-stop-gradient-baseline",
                                          lambda t, x: t("sum", t("*", x, t("stop-gradient", x))), [3.0, 4.0]),
}


def readme_mse():
    """README.md:33-43: x, y captured; W = zeros[2,4]."""
    x = np.array([[1.0, 0.0], [0.0, 1.0]], np.float32)
    y = np.array([[1.0, 1.0, 0.0, 0.0], [0.0, 0.0, 1.0, 1.0]], np.float32)
    W = np.zeros((2, 4), np.float32)
    low = lower_value_and_grad(lambda t, s: M.mse_loss(t, t("@", s["x_in"], s["x"]), s["y_in"]),
                               [("x", (2, 4))], [("x_in", (2, 2)), ("y_in", (2, 4))], key="readme-mse")
    return low, [W, x, y]


def mlp_golden():
    """sheaf/tests/interpreter_tests.yaml:753-762, inputs from the interpreter RNG."""
    from oracle.rng import random_normal
    W = random_normal(0, (4, 2))
    b = np.zeros(2, np.float32)
    x = random_normal(1, (3, 4))
    y = random_normal(2, (3, 2))
    low = lower_value_and_grad(
        lambda t, s: t("mean", t("**", t("-", t("+", t("@", s["x_in"], s["W"]), s["b"]), s["y_in"]), 2)),
        [("W", (4, 2)), ("b", (2,))], [("x_in", (3, 4)), ("y_in", (3, 2))], key="vag-mlp-loss")
    return low, [W, b, x, y]


CASES["readme-mse"] = readme_mse
CASES["vag-mlp-loss"] = mlp_golden
