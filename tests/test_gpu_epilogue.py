"""GEMM epilogue fusion on the GPU through the C ABI: a dot_general followed by
Sheaf's gelu (sheaf/lib/nn.shf: 0.5 x (1 + tanh(0.7978846 (x + 0.044715
x^3)))) plans as one GEMM step that writes both h = x @ W and gelu(h).

Checked against an f64 reference of the same graph: h and gelu(h) at the
TF32 tolerance (2e-3 norm-relative; bf16 tensors 1e-5), and gelu(h) against
gelu of the returned h (the epilogue reads the accumulator that h is stored
from: 1e-6).  Shapes cover the fused tensor-core epilogue (TMA stores and,
for a row length that is not a multiple of 4, plain stores), a split-K GEMM
(the unfused gelu kernel runs after the partial sums are added) and a
skinny GEMM (CUDA cores, then the unfused kernel).
"""
import numpy as np
import pytest

from sheaf_b200 import session as S

pytestmark = pytest.mark.gpu


def _module(name, m, n, k, et="f32"):
    t = f"tensor<{m}x{n}xf32>"
    cst = lambda nm, v: (f"    %{nm}c = stablehlo.constant dense<{v}> : tensor<f32>\n"
                         f"    %{nm} = stablehlo.broadcast_in_dim %{nm}c, dims = [] : (tensor<f32>) -> {t}\n")
    return (f"module @{name} {{\n func.func @f(%arg0: tensor<{m}x{k}x{et}>, %arg1: tensor<{k}x{n}x{et}>) -> ({t}, {t}) {{\n"
            f"    %h = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : "
            f"(tensor<{m}x{k}x{et}>, tensor<{k}x{n}x{et}>) -> {t}\n"
            + cst("half", "5.000000e-01") + cst("one", "1.000000e+00") + cst("a", "4.471500e-02")
            + cst("b", "7.978846e-01") +
            f"    %x2 = stablehlo.multiply %h, %h : {t}\n"
            f"    %x3 = stablehlo.multiply %h, %x2 : {t}\n"
            f"    %ax3 = stablehlo.multiply %a, %x3 : {t}\n"
            f"    %in = stablehlo.add %h, %ax3 : {t}\n"
            f"    %bin = stablehlo.multiply %b, %in : {t}\n"
            f"    %th = stablehlo.tanh %bin : {t}\n"
            f"    %opt = stablehlo.add %one, %th : {t}\n"
            f"    %xo = stablehlo.multiply %h, %opt : {t}\n"
            f"    %g = stablehlo.multiply %half, %xo : {t}\n"
            f"    return %h, %g : {t}, {t}\n }}\n}}\n")


def _gelu(x):
    return 0.5 * (x * (1.0 + np.tanh(0.7978846 * (x + 0.044715 * (x * (x * x))))))


def _trunc(x):
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def _run(sess, m, n, k, bf16=False, seed=0):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = (rng.standard_normal((k, n), dtype=np.float32) / np.sqrt(k)).astype(np.float32)
    name = f"epi_{m}_{n}_{k}_{int(bf16)}"
    text = _module(name, m, n, k, "bf16" if bf16 else "f32")
    if not sess.has_function(f"{name}.f"):
        sess.load_stablehlo(text)
    outs = sess.call_device(f"{name}.f", [sess.buffer(a, bf16=bf16), sess.buffer(b, bf16=bf16)])
    h, g = (o.to_host() for o in outs)
    for o in outs:
        o.release()
    x, y = (_trunc(a), _trunc(b)) if bf16 else (a, b)
    ref_h = x.astype(np.float64) @ y.astype(np.float64)
    return text, name, h, g, ref_h


@pytest.mark.parametrize("shape", [(1024, 1536, 384), (512, 130, 256), (128, 256, 8192), (4, 512, 384)],
                         ids=["tensor-cores", "plain-stores", "split-k", "skinny"])
def test_gelu_epilogue_tf32(tf32_session, shape):
    text, name, h, g, ref_h = _run(tf32_session, *shape)
    fused = [r for r in S.plan_steps(text, f"{name}.f", "tf32") if r["kind"] == "gemm"]
    assert len(fused) == 1 and fused[0]["epi"] == 1
    assert _rel(h, ref_h) <= 2e-3
    assert _rel(g, _gelu(ref_h)) <= 2e-3
    assert _rel(g, _gelu(h.astype(np.float64))) <= 1e-6


@pytest.mark.parametrize("shape", [(1024, 1536, 384), (128, 256, 8192)], ids=["tensor-cores", "split-k"])
def test_gelu_epilogue_bf16_tensors(tf32_session, shape):
    # bf16 operands run on the tensor cores in every mode; the fused plan is
    # the tf32 session's
    _, _, h, g, ref_h = _run(tf32_session, *shape, bf16=True, seed=1)
    assert _rel(h, ref_h) <= 1e-5
    assert _rel(g, _gelu(ref_h)) <= 1e-5
    assert _rel(g, _gelu(h.astype(np.float64))) <= 1e-6
