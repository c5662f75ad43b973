"""Parity at the benchmark configurations' full sizes, against the f32 oracle.

  * nanoGPT value-and-grad, the bench line's configuration: 6 layers, d_model
    384, 6 heads, ctx 256, vocab 65, batch 64 x 256;
  * nanoGPT forward (the same model, batch 64 x 256);
  * GPT-2-small dimensions (12 layers, d_model 768, 12 heads, ctx 1024, vocab
    50304) value-and-grad at batch 1.

Tolerances (the stated contract for tensor-core contractions): TF32 mode,
2e-3 relative on the loss and 2e-3 norm-relative on every gradient leaf and on
the forward logits; fp32 mode (CUDA-core contractions), 1e-5 norm-relative on
the forward logits.  The oracle interprets the same StableHLO text in float32
(oracle/stablehlo_ref.py); it runs in spawned worker processes while the GPU
computes.
"""
import numpy as np
import pytest

import oracle_jobs
from sheaf_lowering import models as M

pytestmark = pytest.mark.gpu

# name -> (kind, config name, batch, seed)
CASES = {
    "nanogpt_vag_64x256": ("vag", "NANOGPT", 64, 11),
    "nanogpt_fwd_64x256": ("fwd", "NANOGPT", 64, 12),
    "gpt2_small_vag_1x1024": ("vag", "GPT2_SMALL", 1, 13),
}


def _lower(kind, cfg_name, batch):
    cfg = getattr(M, cfg_name)
    return M.gpt_vag(cfg, batch=batch) if kind == "vag" else M.gpt_fwd(cfg, batch=batch)


@pytest.fixture(scope="module")
def oracle_results():
    """Lowered graphs and the oracle's pending results, submitted together
    before any of this module's GPU work."""
    lows, pending = {}, {}
    for name, (kind, cfg_name, batch, seed) in CASES.items():
        low = _lower(kind, cfg_name, batch)
        lows[name] = low
        pending[name] = oracle_jobs.pool().apply_async(
            oracle_jobs.evaluate, (low.text, low.qualified, list(low.arg_names), cfg_name, batch, seed))
    return lows, pending


def _gpu(sess, low, name):
    kind, cfg_name, batch, seed = CASES[name]
    inp = oracle_jobs.inputs(cfg_name, batch, seed)
    if not sess.has_function(low.qualified):
        sess.load_stablehlo(low.text)
    return sess.call(low.qualified, [inp[n] for n in low.arg_names])


def _rel(o, r):
    r = np.asarray(r, np.float64)
    return float(np.linalg.norm(np.asarray(o, np.float64) - r) / max(np.linalg.norm(r), 1e-30))


def _check_vag(outs, ref, names, bound):
    assert abs(float(outs[0]) - float(ref[0])) <= bound * abs(float(ref[0])), (float(outs[0]), float(ref[0]))
    errs = [_rel(o, r) for o, r in zip(outs[1:], ref[1:])]
    worst = int(np.argmax(errs))
    leaves = [n for n in names if n not in ("x", "y")]
    assert max(errs) <= bound, (leaves[worst], max(errs))


@pytest.mark.parametrize("name", ["nanogpt_vag_64x256", "gpt2_small_vag_1x1024"])
def test_value_and_grad_full_size_tf32(tf32_session, oracle_results, name):
    lows, pending = oracle_results
    low = lows[name]
    outs = _gpu(tf32_session, low, name)
    ref = pending[name].get(timeout=1800)
    _check_vag(outs, ref, low.arg_names, 2e-3)


def test_nanogpt_forward_full_batch(tf32_session, fp32_session, oracle_results):
    lows, pending = oracle_results
    name = "nanogpt_fwd_64x256"
    low = lows[name]
    tf = _gpu(tf32_session, low, name)
    fp = _gpu(fp32_session, low, name)
    ref = pending[name].get(timeout=1800)
    assert _rel(tf[0], ref[0]) <= 2e-3
    assert _rel(fp[0], ref[0]) <= 1e-5
