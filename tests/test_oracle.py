"""The CPU oracle, pinned against the reference's own known answers."""
import json
import os

import numpy as np
import pytest

from oracle.rng import random_normal
from oracle.stablehlo_ref import run
from sheaf_cases import CASES
from sheaf_lowering import models as M

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "vag_goldens.json")))["cases"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    """Finite-difference goldens of sheaf/tests/vag_tests.yaml (1e-4 on scalars, as
    sheaf/tests/interpreter_tests.rs:91-116 compares them)."""
    low, ins = CASES[name]()
    outs = run(low.text, low.qualified, ins)
    g = GOLD[name]
    assert abs(float(outs[0]) - g["loss"]) <= 1e-4 * max(1.0, abs(g["loss"]))
    if "grad" in g:
        exp = np.array(g["grad"], np.float64)
        np.testing.assert_allclose(outs[1].reshape(exp.shape), exp, rtol=1e-4, atol=2e-5)


def test_oracle_f32_mode_matches_f64():
    low, ins = CASES["vag-layer-norm"]()
    a = run(low.text, low.qualified, ins, dtype=np.float64)
    b = run(low.text, low.qualified, ins, dtype=np.float32)
    np.testing.assert_allclose(a[0], b[0], rtol=1e-5)


def test_splitmix_rng_reproduces_reference_inputs():
    """The MLP golden (4.080512) only holds with the reference's RNG stream."""
    w = random_normal(0, (4, 2))
    assert w.dtype == np.float32 and np.isfinite(w).all()
    low, ins = CASES["vag-mlp-loss"]()
    assert abs(float(run(low.text, low.qualified, ins)[0]) - 4.080512) < 1e-5


def test_lowered_gpt_gradient_matches_finite_differences():
    c = M.GPTConfig(n_layer=1, n_head=2, n_embd=16, block_size=8, vocab_size=13, batch=2)
    low = M.gpt_vag(c)
    inp = M.gpt_inputs(c, seed=3)
    ins = [inp[n].astype(np.float64) for n in low.arg_names]
    outs = run(low.text, low.qualified, ins)
    rng = np.random.default_rng(0)
    for name in ["transformer.h.0.attn.c_attn.weight", "transformer.wte.weight", "transformer.h.0.ln_2.weight",
                 "transformer.wpe.weight", "lm_head.weight"]:
        i = low.arg_names.index(name)
        g = outs[1 + i]
        idx = tuple(int(rng.integers(0, d)) for d in g.shape)
        eps = 1e-5
        p = [x.copy() for x in ins]
        p[i][idx] += eps
        lp = run(low.text, low.qualified, p)[0]
        p[i][idx] -= 2 * eps
        lm = run(low.text, low.qualified, p)[0]
        fd = (lp - lm) / (2 * eps)
        assert abs(fd - g[idx]) <= 1e-6 + 1e-4 * abs(fd), (name, fd, g[idx])


def test_oracle_rejects_wrong_arity():
    low, ins = CASES["vag-add"]()
    with pytest.raises(ValueError):
        run(low.text, low.qualified, ins + ins)
