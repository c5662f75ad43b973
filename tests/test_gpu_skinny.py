"""Skinny GEMMs on the GPU through the C ABI: dot_general with at most 8 rows
in A (the one-position decoding step: x[1, D] @ W^T, q @ K^T, att @ V) or at
most 8 columns in B (run as the transposed product).

These run on CUDA cores in f32 FMA in every precision mode, so the check is
1e-5 norm-relative against an f64 product of the same values, in the fp32, tf32
and bf16 sessions alike (a TF32 contraction would miss it by two orders of
magnitude).  Layouts cover K-contiguous B with 4-wide loads, N-contiguous B,
transposed A (element loads), K not a multiple of 4, batched products and
bf16 tensors.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _module(name, m, n, k, layout, batch, et):
    pre = [batch] if batch else []
    ty = lambda e, *d: "tensor<" + "x".join(str(x) for x in pre + list(d)) + f"x{e}>"
    at, bt = layout[0] == "t", layout[1] == "t"
    sa = ty(et, k, m) if at else ty(et, m, k)
    sb = ty(et, n, k) if bt else ty(et, k, n)
    perm = "[0, 2, 1]" if batch else "[1, 0]"
    body, lhs, rhs = [], "%arg0", "%arg1"
    if at:
        body.append(f"    %ta = stablehlo.transpose %arg0, dims = {perm} : ({sa}) -> {ty(et, m, k)}")
        lhs = "%ta"
    if bt:
        body.append(f"    %tb = stablehlo.transpose %arg1, dims = {perm} : ({sb}) -> {ty(et, k, n)}")
        rhs = "%tb"
    dims = "batching_dims = [0] x [0], contracting_dims = [2] x [1]" if batch else "contracting_dims = [1] x [0]"
    out = ty("f32", m, n)
    body.append(f"    %0 = stablehlo.dot_general {lhs}, {rhs}, {dims} : ({ty(et, m, k)}, {ty(et, k, n)}) -> {out}")
    return (f"module @{name} {{\n func.func @f(%arg0: {sa}, %arg1: {sb}) -> {out} {{\n" + "\n".join(body) +
            f"\n    return %0 : {out}\n }}\n}}\n")


def _trunc(x):
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def _check(sess, tag, m, n, k, layout, batch=0, bf16=False, seed=0):
    from sheaf_b200.session import library
    rng = np.random.default_rng(seed)
    pre = (batch,) if batch else ()
    a = rng.standard_normal(pre + ((k, m) if layout[0] == "t" else (m, k)), dtype=np.float32)
    b = rng.standard_normal(pre + ((n, k) if layout[1] == "t" else (k, n)), dtype=np.float32)
    name = f"skinny_{tag}_{m}_{n}_{k}_{layout}_{batch}_{int(bf16)}"
    if not sess.has_function(f"{name}.f"):
        sess.load_stablehlo(_module(name, m, n, k, layout, batch, "bf16" if bf16 else "f32"))
    ba, bb = sess.buffer(a, bf16=bf16), sess.buffer(b, bf16=bf16)
    lib = library()
    n0 = lib.sb_kernel_launch_count()
    outs = sess.call_device(f"{name}.f", [ba, bb])
    launches = lib.sb_kernel_launch_count() - n0
    got = outs[0].to_host().astype(np.float64)
    for o in outs:
        o.release()
    x, y = (_trunc(a), _trunc(b)) if bf16 else (a, b)
    x, y = x.astype(np.float64), y.astype(np.float64)
    if layout[0] == "t":
        x = np.swapaxes(x, -1, -2)
    if layout[1] == "t":
        y = np.swapaxes(y, -1, -2)
    ref = x @ y
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    return rel, launches


SHAPES = [
    (1, 1152, 384, "nt"),   # decode q/k/v projection, x @ W^T (4-wide K-contiguous loads)
    (1, 384, 1536, "nt"),   # decode MLP down-projection
    (3, 65, 384, "nt"),     # vocabulary 65 head, 3 rows
    (8, 512, 784, "nn"),    # N-contiguous weights (x @ W), 8 rows
    (1, 256, 256, "nn"),
    (5, 300, 130, "tn"),    # A stored transposed: element loads
    (2, 100, 99, "nt"),     # K not a multiple of 4
    (1000, 3, 384, "nn"),   # 3 columns: the transposed product
    (4096, 8, 128, "tn"),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:3])) + s[3])
@pytest.mark.parametrize("mode", ["fp32", "tf32"])
def test_skinny_matmul_f32(fp32_session, tf32_session, mode, shape):
    sess = fp32_session if mode == "fp32" else tf32_session
    rel, launches = _check(sess, mode, *shape)
    assert rel <= 1e-5, rel
    assert launches == 1  # one kernel, no padding copies or split-K partials


@pytest.mark.parametrize("shape", SHAPES[:4] + SHAPES[7:], ids=lambda s: "x".join(map(str, s[:3])) + s[3])
def test_skinny_matmul_bf16_tensors(bf16_session, shape):
    rel, _ = _check(bf16_session, "bf", *shape, bf16=True, seed=1)
    assert rel <= 1e-5, rel


def test_skinny_batched_attention_shapes(tf32_session):
    # q @ K^T and att @ V of one decoding position over 6 heads
    rel, _ = _check(tf32_session, "att", 1, 256, 64, "nt", batch=6, seed=2)
    assert rel <= 1e-5, rel
    rel, _ = _check(tf32_session, "att", 1, 64, 256, "nn", batch=6, seed=3)
    assert rel <= 1e-5, rel
