"""Embedding gradients as row scatter-adds, on the GPU against the oracle.

Sheaf writes the gradient of `(get table idx)` as transpose(one_hot(idx, V)) @
adj (sheaf/src/autodiff/reverse.rs:1015-1041); the backend runs it as a
deterministic scatter-add of adj's rows (kernels/scatter.cu).  Checked in fp32
mode at 1e-5 relative (the scatter-add sums in f32 in row order; the oracle
interprets the one-hot product): repeated indices, indices outside [0, V)
(their one-hot rows are zero), batched and unbatched index tensors, and a GPT
value-and-grad whose tokens repeat heavily.
"""
import numpy as np
import pytest

from oracle.stablehlo_ref import run
from sheaf_lowering import models as M

pytestmark = pytest.mark.gpu


def one_hot_grad_module(n, v, d):
    """The emitter's form of transpose(one_hot(idx, v)) @ adj for a 1-D idx."""
    t = f"tensor<{n}x{v}xf32>"
    return f"""module @emb {{
 func.func @f(%arg0: tensor<{n}xf32>, %arg1: tensor<{n}x{d}xf32>) -> tensor<{v}x{d}xf32> {{
    %0 = stablehlo.reshape %arg0 : (tensor<{n}xf32>) -> tensor<{n}x1xf32>
    %1 = stablehlo.broadcast_in_dim %0, dims = [0, 1] : (tensor<{n}x1xf32>) -> {t}
    %2 = stablehlo.iota dim = 1 : {t}
    %3 = stablehlo.subtract %1, %2 : {t}
    %4 = stablehlo.abs %3 : {t}
    %c1 = stablehlo.constant dense<1.0> : tensor<f32>
    %5 = stablehlo.broadcast_in_dim %c1, dims = [] : (tensor<f32>) -> {t}
    %6 = stablehlo.minimum %4, %5 : {t}
    %7 = stablehlo.subtract %5, %6 : {t}
    %c0 = stablehlo.constant dense<0.0> : tensor<f32>
    %8 = stablehlo.broadcast_in_dim %c0, dims = [] : (tensor<f32>) -> {t}
    %9 = stablehlo.compare NE, %7, %8, FLOAT : ({t}, {t}) -> tensor<{n}x{v}xi1>
    %10 = stablehlo.select %9, %5, %8 : tensor<{n}x{v}xi1>, {t}
    %11 = stablehlo.transpose %10, dims = [1, 0] : ({t}) -> tensor<{v}x{n}xf32>
    %12 = stablehlo.dot_general %11, %arg1, contracting_dims = [1] x [0] : (tensor<{v}x{n}xf32>, tensor<{n}x{d}xf32>) -> tensor<{v}x{d}xf32>
    return %12 : tensor<{v}x{d}xf32>
 }}
}}
"""


@pytest.mark.parametrize("n,v,d", [(3000, 97, 64), (1024, 50304, 96), (200, 13, 30)])
def test_scatter_add_matches_one_hot_product(fp32_session, n, v, d):
    from sheaf_b200 import session as S
    text = one_hot_grad_module(n, v, d)
    assert "scatter=1" in S.inspect_module(text, "fp32")  # the product was rewritten
    rng = np.random.default_rng(n)
    idx = rng.integers(0, min(v, 7), n).astype(np.float32)  # heavy repetition
    idx[::17] = rng.integers(0, v, len(idx[::17]))
    idx[5], idx[11], idx[23] = -1, v, v + 5  # outside [0, v): no row
    adj = rng.standard_normal((n, d), dtype=np.float32)
    fp32_session.load_stablehlo(text)
    got = fp32_session.call("emb.f", [idx, adj])[0]
    ref = run(text, "emb.f", [idx, adj])[0]
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
    # deterministic: bit-identical on a second call
    assert np.array_equal(got, fp32_session.call("emb.f", [idx, adj])[0])


def test_gpt_value_and_grad_with_repeated_tokens(fp32_session):
    c = M.GPTConfig(n_layer=1, n_head=2, n_embd=64, block_size=32, vocab_size=65, batch=4)
    low = M.gpt_vag(c)
    inp = M.gpt_inputs(c, seed=21)
    rng = np.random.default_rng(21)
    inp["x"] = rng.integers(0, 3, inp["x"].shape).astype(np.float32)  # three tokens only
    ins = [inp[n] for n in low.arg_names]
    fp32_session.load_stablehlo(low.text)
    outs = fp32_session.call(low.qualified, ins)
    ref = run(low.text, low.qualified, ins)
    for o, r in zip(outs, ref):
        np.testing.assert_allclose(o, r, rtol=1e-4, atol=1e-6)
