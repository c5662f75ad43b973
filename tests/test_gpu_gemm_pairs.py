"""Two independent GEMMs in one tensor-core launch, as a layer's backward pass
issues them: dX = G @ W^T and dW = G^T @ X, both reading the output gradient
G [T, O] (W [O, I], X [T, I]).

The runtime runs consecutive independent GEMM steps as one launch (the tiles
of the first product, then those of the second).  Checked here: both results
are bit-identical to the same products run as single-GEMM functions (each
product's summation order depends only on its shape: the split-K rule is the
same either way), they are within the TF32 bound of an f64 product (2e-3
norm-relative; bf16 tensors 1e-5), a replayed call of the pair is one GEMM
launch plus the batched split-K reduction, a pair whose second output the
plan placed where the first product's operand was runs correctly (the two
products run at the same time, so such a pair is launched one by one), and
the nanoGPT backward at batch 8 runs in fewer launches than its GEMM steps
would take one by one.
"""
import numpy as np
import pytest

from sheaf_b200 import session as S

pytestmark = pytest.mark.gpu


def _ty(et, *d):
    return "tensor<" + "x".join(str(x) for x in d) + f"x{et}>"


def _modules(tag, T, I, O, et):
    """(pair module, dX module, dW module) texts; arguments G, W, X."""
    g, w, x = _ty(et, T, O), _ty(et, O, I), _ty(et, T, I)
    dx, dw = _ty("f32", T, I), _ty("f32", O, I)
    head = f" func.func @f(%arg0: {g}, %arg1: {w}, %arg2: {x}) -> "
    l_dx = f"    %dx = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : ({g}, {w}) -> {dx}\n"
    l_gt = f"    %gt = stablehlo.transpose %arg0, dims = [1, 0] : ({g}) -> {_ty(et, O, T)}\n"
    l_dw = (f"    %dw = stablehlo.dot_general %gt, %arg2, contracting_dims = [1] x [0] : "
            f"({_ty(et, O, T)}, {x}) -> {dw}\n")
    pair = (f"module @pair{tag} {{\n{head}({dx}, {dw}) {{\n{l_dx}{l_gt}{l_dw}"
            f"    return %dx, %dw : {dx}, {dw}\n }}\n}}\n")
    one_dx = f"module @dx{tag} {{\n{head}{dx} {{\n{l_dx}    return %dx : {dx}\n }}\n}}\n"
    one_dw = f"module @dw{tag} {{\n{head}{dw} {{\n{l_gt}{l_dw}    return %dw : {dw}\n }}\n}}\n"
    return pair, one_dx, one_dw


def _trunc(x):
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def _rel(o, r):
    return float(np.linalg.norm(np.asarray(o, np.float64) - r) / np.linalg.norm(r))


def _call(sess, name, bufs, times=3):
    """Outputs of the last of `times` calls (the first runs eagerly, the second
    is captured, the third replays) and the kernels that call launched."""
    for k in range(times):
        n0 = S.library().sb_kernel_launch_count()
        outs = sess.call_device(name, bufs)
        res = [o.to_host() for o in outs]
        n = S.library().sb_kernel_launch_count() - n0
        for o in outs:
            o.release()
    return res, n


SHAPES = [(2048, 1536, 384), (2048, 384, 1536), (2048, 384, 384), (2048, 1152, 384), (1000, 200, 136)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_pair_matches_single_launches(tf32_session, shape, bf16):
    T, I, O = shape
    rng = np.random.default_rng(T + I + O)
    g = rng.standard_normal((T, O), dtype=np.float32)
    w = (rng.standard_normal((O, I), dtype=np.float32) / np.sqrt(O)).astype(np.float32)
    x = rng.standard_normal((T, I), dtype=np.float32)
    tag = f"_{T}_{I}_{O}_{int(bf16)}"
    texts = _modules(tag, T, I, O, "bf16" if bf16 else "f32")
    for t in texts:
        name = t.split("@", 1)[1].split(" ", 1)[0] + ".f"
        if not tf32_session.has_function(name):
            tf32_session.load_stablehlo(t)
    bufs = [tf32_session.buffer(a, bf16=bf16) for a in (g, w, x)]
    (dx, dw), n_pair = _call(tf32_session, f"pair{tag}.f", bufs)
    (dx1,), n_dx = _call(tf32_session, f"dx{tag}.f", bufs)
    (dw1,), n_dw = _call(tf32_session, f"dw{tag}.f", bufs)
    assert np.array_equal(dx.view(np.uint32), dx1.view(np.uint32))
    assert np.array_equal(dw.view(np.uint32), dw1.view(np.uint32))
    # one launch fewer than the two products on their own (the pair's split-K
    # partials share the one reduction launch)
    assert n_pair < n_dx + n_dw, (n_pair, n_dx, n_dw)
    gg, ww, xx = (_trunc(a) for a in (g, w, x)) if bf16 else (g, w, x)
    gg, ww, xx = (a.astype(np.float64) for a in (gg, ww, xx))
    tol = 1e-5 if bf16 else 2e-3
    assert _rel(dx, gg @ ww) <= tol
    assert _rel(dw, gg.T @ xx) <= tol


def _reuse_module(tag, T, I, O):
    """dW = G^T @ (X*X) then dX = G @ W, with X*X read last by dW and dX (same
    shape) consumed by a loop: the plan may put dX where X*X was, which the
    pair must not do while dW still reads it."""
    g, w, x = _ty("f32", T, O), _ty("f32", O, I), _ty("f32", T, I)
    dw, gt = _ty("f32", O, I), _ty("f32", O, T)
    return (f"module @reuse{tag} {{\n func.func @f(%arg0: {g}, %arg1: {w}, %arg2: {x}) -> ({dw}, {x}) {{\n"
            f"    %t = stablehlo.multiply %arg2, %arg2 : {x}\n"
            f"    %gt = stablehlo.transpose %arg0, dims = [1, 0] : ({g}) -> {gt}\n"
            f"    %dw = stablehlo.dot_general %gt, %t, contracting_dims = [1] x [0] : ({gt}, {x}) -> {dw}\n"
            f"    %dx = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : ({g}, {w}) -> {x}\n"
            f"    %y = stablehlo.add %dx, %dx : {x}\n"
            f"    return %dw, %y : {dw}, {x}\n }}\n}}\n")


@pytest.mark.parametrize("shape", [(2048, 384, 1152), (2048, 1536, 384)], ids=lambda s: "x".join(map(str, s)))
def test_pair_never_writes_what_the_other_reads(tf32_session, shape):
    T, I, O = shape
    rng = np.random.default_rng(7)
    g = rng.standard_normal((T, O), dtype=np.float32)
    w = (rng.standard_normal((O, I), dtype=np.float32) / np.sqrt(O)).astype(np.float32)
    x = rng.standard_normal((T, I), dtype=np.float32)
    tag = f"_{T}_{I}_{O}"
    if not tf32_session.has_function(f"reuse{tag}.f"):
        tf32_session.load_stablehlo(_reuse_module(tag, T, I, O))
    bufs = [tf32_session.buffer(a) for a in (g, w, x)]
    (dw, y), _ = _call(tf32_session, f"reuse{tag}.f", bufs)
    gg, ww, xx = (a.astype(np.float64) for a in (g, w, x))
    assert _rel(dw, gg.T @ (xx * xx)) <= 2e-3
    assert _rel(y, 2 * (gg @ ww)) <= 2e-3


_COUNT = """
import sys
sys.path.insert(0, {root!r})
from sheaf_b200 import session as S
from sheaf_lowering import models as M
c = M.NANOGPT
low = M.gpt_vag(c, batch=8)
sess = S.B200Session(device=0, precision="tf32")
sess.load_stablehlo(low.text)
inp = M.gpt_inputs(c, batch=8)
bufs = [sess.buffer(inp[n]) for n in low.arg_names]
for k in range(3):
    n0 = S.library().sb_kernel_launch_count()
    outs = sess.call_device(low.qualified, bufs)
    loss = outs[0].to_host()
    n = S.library().sb_kernel_launch_count() - n0
    for o in outs:
        o.release()
print(n, float(loss))
"""


def test_nanogpt_backward_pairs_its_gemms():
    """nanoGPT value-and-grad at batch 8, replayed: with pairing the step
    takes at least 12 launches fewer than with every GEMM on its own
    (SHEAF_B200_GEMM_PAIRS=0; three of a layer's four dX/dW pairs write a
    gradient output, which no operand shares memory with), for the same loss."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = {}
    for pairs in ("1", "0"):
        env = dict(os.environ, SHEAF_B200_GEMM_PAIRS=pairs)
        r = subprocess.run(["timeout", "-k", "10", "300", sys.executable, "-c", _COUNT.format(root=root)],
                           capture_output=True, text=True, env=env)
        assert r.returncode == 0, r.stderr[-2000:]
        n, loss = r.stdout.split()
        res[pairs] = (int(n), float(loss))
    assert res["1"][1] == res["0"][1]
    assert res["1"][0] <= res["0"][0] - 12, res
