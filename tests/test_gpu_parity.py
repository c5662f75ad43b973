"""GPU parity through the C ABI: the reference goldens, the MLP and GPT
value-and-grad graphs, checked against the CPU oracle.

Tolerances: fp32 mode 1e-5 relative on the loss and 1e-4 max-relative on
gradients (f32 re-association through deep graphs); tf32 tensor-core
mode 2e-3 relative on the loss and 2e-3 norm-relative on gradients (the
stated bound for tensor-core contractions).
"""
import json
import os

import numpy as np
import pytest

from oracle.stablehlo_ref import run
from sheaf_cases import CASES
from sheaf_lowering import models as M

pytestmark = pytest.mark.gpu
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "vag_goldens.json")))["cases"]


def _call(sess, low, ins):
    if not sess.has_function(low.qualified):
        sess.load_stablehlo(low.text)
    return sess.call(low.qualified, ins)


@pytest.mark.parametrize("name", sorted(CASES))
def test_golden_case_on_gpu(fp32_session, name):
    low, ins = CASES[name]()
    outs = _call(fp32_session, low, ins)
    ref = run(low.text, low.qualified, ins)
    g = GOLD[name]
    assert abs(float(outs[0]) - g["loss"]) <= 1e-4 * max(1.0, abs(g["loss"]))
    if "grad" in g:
        exp = np.array(g["grad"], np.float64)
        np.testing.assert_allclose(outs[1].reshape(exp.shape), exp, rtol=1e-4, atol=2e-5)
    for o, r in zip(outs, ref):
        np.testing.assert_allclose(o, r, rtol=1e-5, atol=1e-6)


def _grad_errs(outs, ref):
    errs = []
    for o, r in zip(outs[1:], ref[1:]):
        denom = max(np.linalg.norm(r), 1e-30)
        errs.append(np.linalg.norm(o.astype(np.float64) - r) / denom)
    return errs


def test_mlp_value_and_grad_full_size(fp32_session):
    low = M.mlp_vag()
    inp = M.mlp_inputs()
    ins = [inp[n] for n in low.arg_names]
    outs = _call(fp32_session, low, ins)
    ref = run(low.text, low.qualified, ins)
    assert abs(outs[0] - ref[0]) <= 1e-5 * abs(ref[0])
    for o, r in zip(outs[1:], ref[1:]):
        assert np.max(np.abs(o - r)) <= 1e-4 * np.max(np.abs(r)) + 1e-9


SMALL_GPT = M.GPTConfig(n_layer=2, n_head=2, n_embd=64, block_size=32, vocab_size=65, batch=4)


def test_small_gpt_value_and_grad_fp32(fp32_session):
    low = M.gpt_vag(SMALL_GPT)
    inp = M.gpt_inputs(SMALL_GPT, seed=1)
    ins = [inp[n] for n in low.arg_names]
    outs = _call(fp32_session, low, ins)
    ref = run(low.text, low.qualified, ins)
    assert abs(outs[0] - ref[0]) <= 1e-5 * abs(ref[0])
    for o, r in zip(outs[1:], ref[1:]):
        assert np.max(np.abs(o - r)) <= 1e-4 * np.max(np.abs(r)) + 1e-9


def test_small_gpt_forward_fp32(fp32_session):
    low = M.gpt_fwd(SMALL_GPT)
    inp = M.gpt_inputs(SMALL_GPT, seed=2)
    ins = [inp[n] for n in low.arg_names]
    outs = _call(fp32_session, low, ins)
    ref = run(low.text, low.qualified, ins)
    np.testing.assert_allclose(outs[0], ref[0], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("prec", ["tf32"])
def test_nanogpt_dims_value_and_grad_tensor_cores(request, prec):
    """nanoGPT model dimensions (6 layers, D384, H6, T256, V65) at batch 4."""
    sess = request.getfixturevalue(f"{prec}_session")
    low = M.gpt_vag(M.NANOGPT, batch=4)
    inp = M.gpt_inputs(M.NANOGPT, batch=4, seed=0)
    ins = [inp[n] for n in low.arg_names]
    outs = _call(sess, low, ins)
    ref = run(low.text, low.qualified, ins)
    assert abs(outs[0] - ref[0]) <= 2e-3 * abs(ref[0])
    errs = _grad_errs(outs, ref)
    assert max(errs) <= 2e-3, (prec, max(errs), int(np.argmax(errs)))


def test_repeated_calls_are_bitwise_identical(fp32_session):
    low = M.gpt_vag(SMALL_GPT)
    inp = M.gpt_inputs(SMALL_GPT, seed=5)
    ins = [inp[n] for n in low.arg_names]
    a = _call(fp32_session, low, ins)
    b = _call(fp32_session, low, ins)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_nanogpt_full_batch_properties(tf32_session):
    """Full nanoGPT batch (64x256): size-independent properties, since the
    oracle is too slow at this size: finite outputs, loss near ln(V) for
    N(0, 0.02) weights, and exact data-parallel linearity of the loss
    (mean over two half batches == full-batch loss)."""
    c = M.NANOGPT
    low = M.gpt_vag(c)
    half = M.gpt_vag(c, batch=32)
    inp = M.gpt_inputs(c, seed=7)
    ins = [inp[n] for n in low.arg_names]
    outs = _call(tf32_session, low, ins)
    assert all(np.isfinite(o).all() for o in outs)
    # N(0, 0.02) weights give logits of small spread: the loss sits just above ln(V)
    assert 0 < float(outs[0]) - np.log(c.vocab_size) < 0.15
    parts = []
    for h in range(2):
        hi = [inp[n][h * 32:(h + 1) * 32] if n in ("x", "y") else inp[n] for n in half.arg_names]
        parts.append(_call(tf32_session, half, hi))
    loss_avg = 0.5 * (parts[0][0] + parts[1][0])
    assert abs(loss_avg - outs[0]) <= 1e-4 * abs(outs[0])
    for j in range(1, len(outs)):
        g = 0.5 * (parts[0][j] + parts[1][j])
        assert np.linalg.norm(g - outs[j]) <= 2e-3 * np.linalg.norm(outs[j]) + 1e-12
