"""Fused attention (tcgen05, TF32) against the oracle.

In TF32 mode the planner replaces the causal softmax attention region that
Sheaf's `causal_self_attention` lowers to, and its reverse-mode graph, with the
three fused kernels of kernels/attention.cu.  These tests build that region
alone (and inside a one-layer GPT), check that the plan really uses the fused
steps, and compare loss and gradients with the float64 oracle: 2e-3 relative
on the loss, 2e-3 norm-relative on every gradient (the tensor-core bound).
"""
import re

import numpy as np
import pytest

from oracle.stablehlo_ref import run
from sheaf_b200 import session as S
from sheaf_lowering import models as M
from sheaf_lowering.lower import Vec, lower_forward, lower_value_and_grad

pytestmark = pytest.mark.gpu
HD = 64


def _attention(t, q, k, v, causal):
    T = t.shape(q)[-2]
    scores = t("/", t("@", q, t("swapaxes", k, -1, -2)), t("sqrt", float(HD)))
    if causal:
        mask = t("==", t("tril", t("ones", Vec([T, T]))), 1.0)
        scores = t("where", mask, scores, -1e10)
    return t("@", M.softmax(t, scores), v)


def attention_vag(B, H, T, causal):
    """loss = sum((Y * w)^2): no cancellation in the loss, and dY = 2 Y w^2
    varies across rows and columns."""
    shp = (B, H, T, HD)

    def build(t, s):
        y = t("*", _attention(t, s["q"], s["k"], s["v"], causal), s["w"])
        return t("sum", t("*", y, y))
    return lower_value_and_grad(build, [("k", shp), ("q", shp), ("v", shp)], [("w", shp)],
                                key=f"attn-vag-{B}-{H}-{T}-{causal}")


def attention_fwd(B, H, T, causal):
    shp = (B, H, T, HD)

    def build(t, s):
        return _attention(t, s["q"], s["k"], s["v"], causal)
    return lower_forward(build, [("q", shp), ("k", shp), ("v", shp)], "attention",
                         key=f"attn-fwd-{B}-{H}-{T}-{causal}")


def _inputs(low, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(t.shape).astype(np.float32) for t in low.arg_types]


def _fused_steps(low):
    rep = S.inspect_module(low.text, precision="tf32")
    return int(re.search(r"attention=(\d+)", rep).group(1))


def _check(outs, ref, scalar_first=True):
    errs = []
    if scalar_first:
        errs.append(abs(float(outs[0]) - float(ref[0])) / abs(float(ref[0])))
        outs, ref = outs[1:], ref[1:]
    for o, r in zip(outs, ref):
        errs.append(np.linalg.norm(o.astype(np.float64) - r) / max(np.linalg.norm(r), 1e-30))
    assert max(errs) <= 2e-3, errs


# up to GPT-2's context (1024) and one length past it
@pytest.mark.parametrize("T", [128, 256, 1024, 1280])
@pytest.mark.parametrize("causal", [True, False])
def test_attention_value_and_grad(tf32_session, T, causal):
    low = attention_vag(2, 3, T, causal)
    assert _fused_steps(low) == 2
    ins = _inputs(low, seed=T + causal)
    tf32_session.load_stablehlo(low.text)
    outs = tf32_session.call(low.qualified, ins)
    _check(outs, run(low.text, low.qualified, ins))


def test_attention_forward(tf32_session):
    low = attention_fwd(2, 2, 384, True)
    assert _fused_steps(low) == 1
    ins = _inputs(low, seed=7)
    tf32_session.load_stablehlo(low.text)
    outs = tf32_session.call(low.qualified, ins)
    _check(outs, run(low.text, low.qualified, ins), scalar_first=False)


def test_fused_attention_is_deterministic(tf32_session):
    low = attention_vag(4, 2, 256, True)
    ins = _inputs(low, seed=11)
    tf32_session.load_stablehlo(low.text)
    a = tf32_session.call(low.qualified, ins)
    b = tf32_session.call(low.qualified, ins)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_gpt_layer_with_fused_attention(tf32_session):
    c = M.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=128, vocab_size=65, batch=2)
    low = M.gpt_vag(c)
    assert _fused_steps(low) == 2
    inp = M.gpt_inputs(c, seed=4)
    ins = [inp[n] for n in low.arg_names]
    tf32_session.load_stablehlo(low.text)
    outs = tf32_session.call(low.qualified, ins)
    _check(outs, run(low.text, low.qualified, ins))


def _errs(outs, ref):
    e = [abs(float(outs[0]) - float(ref[0])) / abs(float(ref[0]))]
    for o, r in zip(outs[1:], ref[1:]):
        e.append(float(np.linalg.norm(o.astype(np.float64) - r) / np.linalg.norm(r)))
    return e


def test_nanogpt_full_batch_fused_matches_fp32(tf32_session, fp32_session):
    """Full nanoGPT batch (64 x 256): the fused TF32 step and the unfused TF32
    step of the same graph, both against the exact-f32 step, each within the
    2e-3 tensor-core bound (loss relative, every gradient norm-relative):
    fusing attention must not cost accuracy."""
    from sheaf_b200.session import B200Session
    low = M.gpt_vag(M.NANOGPT)
    inp = M.gpt_inputs(M.NANOGPT, seed=1)
    ins = [inp[n] for n in low.arg_names]
    tf32_session.load_stablehlo(low.text)
    fp32_session.load_stablehlo(low.text)
    fused = tf32_session.call(low.qualified, ins)
    exact = [x.astype(np.float64) for x in fp32_session.call(low.qualified, ins)]
    unfused_sess = B200Session(precision="tf32", fuse_attention=False)
    try:
        unfused_sess.load_stablehlo(low.text)
        unfused = unfused_sess.call(low.qualified, ins)
    finally:
        unfused_sess.close()
    ef, eu = _errs(fused, exact), _errs(unfused, exact)
    assert max(ef) <= 2e-3, max(ef)
    assert max(eu) <= 2e-3, max(eu)
