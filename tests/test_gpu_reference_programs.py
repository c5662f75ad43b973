"""The reference's own benchmark programs on the GPU against the f32 oracle:
benchmarks/bench_forward.shf (GPT-2 124M forward, 1 x 64 tokens, vocabulary
50257) and benchmarks/bench_vag_sheaf.shf (value-and-grad of the mean of the
logits).  The vocabulary of 50257 puts every lm_head operand off 16-byte rows
(the padded-operand path of the tensor-core GEMMs).

Tolerances: TF32 mode 2e-3 norm-relative on the logits and on every gradient
leaf; fp32 mode 1e-5 norm-relative on the logits.  The loss is the mean of
3.2 M logits of magnitude ~1 that cancel to ~3e-4, so its error is bounded
relative to the mean absolute logit: 2e-3 of it.
"""
import numpy as np
import pytest

from oracle.stablehlo_ref import run
from sheaf_lowering import models as M

pytestmark = pytest.mark.gpu


def _rel(o, r):
    r = np.asarray(r, np.float64)
    return float(np.linalg.norm(np.asarray(o, np.float64) - r) / max(np.linalg.norm(r), 1e-30))


@pytest.fixture(scope="module")
def inputs():
    return M.bench_inputs()


def test_bench_forward(tf32_session, fp32_session, inputs):
    low = M.bench_forward_program()
    ins = [inputs[n] for n in low.arg_names]
    ref = run(low.text, low.qualified, ins, dtype=np.float32)[0]
    for sess, bound in ((tf32_session, 2e-3), (fp32_session, 1e-5)):
        if not sess.has_function(low.qualified):
            sess.load_stablehlo(low.text)
        got = sess.call(low.qualified, ins)[0]
        assert got.shape == (1, 64, 50257)
        assert _rel(got, ref) <= bound, (sess.precision, _rel(got, ref))


def test_bench_value_and_grad(tf32_session, inputs):
    low = M.bench_vag_program()
    ins = [inputs[n] for n in low.arg_names]
    ref = run(low.text, low.qualified, ins, dtype=np.float32)
    if not tf32_session.has_function(low.qualified):
        tf32_session.load_stablehlo(low.text)
    outs = tf32_session.call(low.qualified, ins)
    fwd = M.bench_forward_program()
    scale = float(np.mean(np.abs(run(fwd.text, fwd.qualified, [inputs[n] for n in fwd.arg_names],
                                     dtype=np.float32)[0])))
    assert abs(float(outs[0]) - float(ref[0])) <= 2e-3 * scale, (float(outs[0]), float(ref[0]), scale)
    errs = [_rel(o, r) for o, r in zip(outs[1:], ref[1:])]
    assert max(errs) <= 2e-3, max(errs)
