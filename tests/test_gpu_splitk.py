"""Split-K GEMMs on the GPU through the C ABI.

A GEMM whose 128 x 128 tiles do not cover the SMs is cut into K slices by a
fixed rule on the shape; each slice's partial product goes to the workspace
and a reduction kernel adds them in slice order.  Checked here: the result
against an f64 product (TF32 operands: 2e-3 norm-relative; bf16 tensors:
1e-5), bit-identical results over repeated calls, every tile configuration,
the weight-gradient layout X^T @ G, and a ragged edge (M, N not multiples of
the tile, N not a multiple of 4).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _module(name, m, n, k, layout, et):
    ty = lambda e, *d: "tensor<" + "x".join(str(x) for x in d) + f"x{e}>"
    at, bt = layout[0] == "t", layout[1] == "t"
    sa = ty(et, k, m) if at else ty(et, m, k)
    sb = ty(et, n, k) if bt else ty(et, k, n)
    body, lhs, rhs = [], "%arg0", "%arg1"
    if at:
        body.append(f"    %ta = stablehlo.transpose %arg0, dims = [1, 0] : ({sa}) -> {ty(et, m, k)}")
        lhs = "%ta"
    if bt:
        body.append(f"    %tb = stablehlo.transpose %arg1, dims = [1, 0] : ({sb}) -> {ty(et, k, n)}")
        rhs = "%tb"
    out = ty("f32", m, n)
    body.append(f"    %0 = stablehlo.dot_general {lhs}, {rhs}, contracting_dims = [1] x [0] : "
                f"({ty(et, m, k)}, {ty(et, k, n)}) -> {out}")
    return (f"module @{name} {{\n func.func @f(%arg0: {sa}, %arg1: {sb}) -> {out} {{\n" + "\n".join(body) +
            f"\n    return %0 : {out}\n }}\n}}\n")


def _trunc(x):
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def _calls(sess, m, n, k, layout, bf16=False, repeats=3, seed=0, tag=""):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((k, m) if layout[0] == "t" else (m, k), dtype=np.float32)
    b = rng.standard_normal((n, k) if layout[1] == "t" else (k, n), dtype=np.float32)
    name = f"splitk{tag}_{m}_{n}_{k}_{layout}_{int(bf16)}"
    if not sess.has_function(f"{name}.f"):
        sess.load_stablehlo(_module(name, m, n, k, layout, "bf16" if bf16 else "f32"))
    ba, bb = sess.buffer(a, bf16=bf16), sess.buffer(b, bf16=bf16)
    outs = []
    for _ in range(repeats):
        o = sess.call_device(f"{name}.f", [ba, bb])
        outs.append(o[0].to_host())
        for x in o:
            x.release()
    x, y = (_trunc(a), _trunc(b)) if bf16 else (a, b)
    x, y = x.astype(np.float64), y.astype(np.float64)
    if layout[0] == "t":
        x = x.T
    if layout[1] == "t":
        y = y.T
    return outs, x @ y


def _rel(o, r):
    return float(np.linalg.norm(np.asarray(o, np.float64) - r) / np.linalg.norm(r))


@pytest.mark.parametrize("shape", [(128, 128, 8192, "nn"), (384, 1536, 2048, "tn"), (200, 130, 4100, "nt"),
                                   (768, 768, 8192, "tn")], ids=lambda s: "x".join(map(str, s[:3])) + s[3])
def test_splitk_tf32_matches_and_repeats(tf32_session, shape):
    outs, ref = _calls(tf32_session, *shape)
    assert _rel(outs[0], ref) <= 2e-3
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))


@pytest.mark.parametrize("shape", [(128, 128, 8192, "nn"), (384, 1536, 2048, "tn")],
                         ids=lambda s: "x".join(map(str, s[:3])) + s[3])
def test_splitk_bf16_tensors(fp32_session, shape):
    outs, ref = _calls(fp32_session, *shape, bf16=True, seed=1)
    assert _rel(outs[0], ref) <= 1e-5
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))


@pytest.mark.parametrize("cfg", range(6))
def test_splitk_every_tile_configuration(tf32_session, cfg):
    os.environ["SHEAF_B200_GEMM_CONFIG"] = str(cfg)
    try:
        outs, ref = _calls(tf32_session, 384, 520, 4096, "tn", repeats=2, seed=cfg, tag=f"c{cfg}")
    finally:
        del os.environ["SHEAF_B200_GEMM_CONFIG"]
    assert _rel(outs[0], ref) <= 2e-3
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
