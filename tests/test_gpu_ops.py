"""Op-level GPU parity for every StableHLO form the backend executes, at shapes
that reach each kernel strategy (row / block / split-column reductions,
strided GEMM operands, index maps), against the oracle.  fp32 mode: 1e-5
relative on non-contraction ops."""
import numpy as np
import pytest

from oracle.stablehlo_ref import run
from sheaf_b200.session import plan_steps

pytestmark = pytest.mark.gpu

_N = [0]


def module(params, body, rets):
    """params: list of type strings; body: list of lines; rets: [(name, type)]."""
    _N[0] += 1
    ps = ", ".join(f"%arg{i}: {t}" for i, t in enumerate(params))
    rt = rets[0][1] if len(rets) == 1 else "(" + ", ".join(t for _, t in rets) + ")"
    lines = [f"module @ops_{_N[0]} {{", f" func.func @f({ps}) -> {rt} {{"]
    lines += ["    " + b for b in body]
    lines.append(f"    return {', '.join(n for n, _ in rets)} : {', '.join(t for _, t in rets)}")
    lines += [" }", "}"]
    return f"ops_{_N[0]}.f", "\n".join(lines) + "\n"


def check(sess, name, text, ins, rtol=1e-5, atol=1e-6):
    sess.load_stablehlo(text)
    outs = sess.call(name, ins)
    ref = run(text, name, ins)
    for o, r in zip(outs, ref):
        np.testing.assert_allclose(o, r.astype(o.dtype), rtol=rtol, atol=atol)
    return outs


R = np.random.default_rng(0)


def rnd(*s):
    return R.standard_normal(s).astype(np.float32)


@pytest.mark.parametrize("shape,dim", [((4096, 64), 0), ((64, 4096), 1), ((3, 8192), 1), ((7, 5, 300), 1),
                                       ((16384, 1536), 0), ((6, 70000), 1), ((2, 3, 4), 0),
                                       # full and few-output reductions of long rows (split rows)
                                       ((1024, 2048), (0, 1)), ((3, 40000), 1),
                                       # many rows onto few columns (split columns, 4-wide and scalar)
                                       ((16, 512, 384), (0, 1)), ((40000, 65), 0), ((9000, 12), 0)])
@pytest.mark.parametrize("body", ["add", "maximum", "minimum"])
def test_reduce(fp32_session, shape, dim, body):
    dims = (dim,) if isinstance(dim, int) else tuple(dim)
    t = "tensor<" + "x".join(map(str, shape)) + "xf32>"
    out = [d for i, d in enumerate(shape) if i not in dims]
    ot = "tensor<" + "".join(f"{d}x" for d in out) + "f32>"
    init = {"add": "0.0", "maximum": "0xFF800000", "minimum": "0x7F800000"}[body]
    dl = ", ".join(map(str, dims))
    name, text = module([t], [f"%0 = stablehlo.constant dense<{init}> : tensor<f32>",
                              f"%1 = stablehlo.reduce(%arg0 init: %0) applies stablehlo.{body} across dimensions = [{dl}] : ({t}, tensor<f32>) -> {ot}"],
                        [("%1", ot)])
    # f32 sums of R unit normals: rounding error grows like sqrt(R) (blocked
    # summation), ~2e-4 at R = 16384; max/min are exact.
    R = int(np.prod([shape[d] for d in dims]))
    rtol = 2e-5 if body == "add" else 0
    atol = 2e-4 * max(1.0, (R / 4096) ** 0.5) if body == "add" else 0
    check(fp32_session, name, text, [rnd(*shape)], rtol=rtol, atol=atol)


def chain_module(shape, d1, d2, out1, out2):
    t = "tensor<" + "x".join(map(str, shape)) + "xf32>"
    return module([t], ["%0 = stablehlo.constant dense<0.0> : tensor<f32>",
                        f"%1 = stablehlo.multiply %arg0, %arg0 : {t}",
                        f"%2 = stablehlo.reduce(%1 init: %0) applies stablehlo.add across dimensions = [{d1}] : ({t}, tensor<f32>) -> {out1}",
                        f"%3 = stablehlo.reduce(%2 init: %0) applies stablehlo.add across dimensions = [{d2}] : ({out1}, tensor<f32>) -> {out2}"],
                  [("%3", out2)])


def test_reduce_chain_merged(fp32_session):
    # reduce(reduce(x*x, [0]), [0]): the planner merges the column chain into
    # one reduction over dims [0, 1]
    name, text = chain_module((64, 96, 400), "0", "0", "tensor<96x400xf32>", "tensor<400xf32>")
    check(fp32_session, name, text, [rnd(64, 96, 400)], rtol=2e-5, atol=1e-4)
    assert [st["kind"] for st in plan_steps(text, name, "fp32")] == ["reduce"]


def test_reduce_chain_rows_then_all(fp32_session):
    # reduce(reduce(x*x, [2]), [0, 1]) stays two kernels (row sums, then a small sum)
    name, text = chain_module((64, 96, 400), "2", "0, 1", "tensor<64x96xf32>", "tensor<f32>")
    check(fp32_session, name, text, [rnd(64, 96, 400)], rtol=2e-5, atol=0)
    assert [st["kind"] for st in plan_steps(text, name, "fp32")] == ["reduce", "reduce"]


def test_layernorm_reduce_epilogues(fp32_session):
    from test_abi import LAYERNORM
    check(fp32_session, "ln.f", LAYERNORM, [rnd(64, 32, 64)], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("fixture", ["fp32_session", "tf32_session"])
def test_transposed_gemm_outputs(request, fixture):
    from test_abi import TRANSPOSED_WGRAD
    sess = request.getfixturevalue(fixture)
    ins = [rnd(4, 64, 96), rnd(4, 64, 160), rnd(96, 64), rnd(64, 160)]
    if fixture == "fp32_session":
        check(sess, "tw.f", TRANSPOSED_WGRAD, ins, rtol=1e-4, atol=1e-4)
    else:
        sess.load_stablehlo(TRANSPOSED_WGRAD)
        outs = sess.call("tw.f", ins)
        for o, r in zip(outs, run(TRANSPOSED_WGRAD, "tw.f", ins)):
            assert np.linalg.norm(o - r) / np.linalg.norm(r) <= 2e-3


def test_elementwise_chain_with_broadcasts(fp32_session):
    name, text = module(["tensor<37x129xf32>", "tensor<129xf32>", "tensor<37x1xf32>"], [
        "%0 = stablehlo.broadcast_in_dim %arg1, dims = [1] : (tensor<129xf32>) -> tensor<37x129xf32>",
        "%1 = stablehlo.broadcast_in_dim %arg2, dims = [0, 1] : (tensor<37x1xf32>) -> tensor<37x129xf32>",
        "%2 = stablehlo.multiply %arg0, %0 : tensor<37x129xf32>",
        "%3 = stablehlo.subtract %2, %1 : tensor<37x129xf32>",
        "%4 = stablehlo.tanh %3 : tensor<37x129xf32>",
        "%5 = stablehlo.exponential %4 : tensor<37x129xf32>",
        "%6 = stablehlo.abs %3 : tensor<37x129xf32>",
        "%7 = stablehlo.log %6 : tensor<37x129xf32>",
        "%8 = stablehlo.sqrt %6 : tensor<37x129xf32>",
        "%9 = stablehlo.divide %5, %8 : tensor<37x129xf32>",
        "%10 = stablehlo.power %6, %5 : tensor<37x129xf32>",
        "%11 = stablehlo.sign %3 : tensor<37x129xf32>",
        "%12 = stablehlo.negate %11 : tensor<37x129xf32>",
        "%13 = stablehlo.add %9, %12 : tensor<37x129xf32>",
        "%14 = stablehlo.maximum %13, %7 : tensor<37x129xf32>",
        "%15 = stablehlo.minimum %14, %10 : tensor<37x129xf32>",
    ], [("%15", "tensor<37x129xf32>"), ("%7", "tensor<37x129xf32>")])
    check(fp32_session, name, text, [rnd(37, 129), rnd(129), rnd(37, 1)], rtol=2e-6, atol=1e-6)


def test_compare_select_clamp_convert_iota(fp32_session):
    T = "tensor<5x7xf32>"
    name, text = module([T, T], [
        "%0 = stablehlo.constant dense<0.0> : tensor<f32>",
        "%1 = stablehlo.broadcast_in_dim %0, dims = [] : (tensor<f32>) -> tensor<5x7xf32>",
        "%2 = stablehlo.compare GT, %arg0, %1, FLOAT : (tensor<5x7xf32>, tensor<5x7xf32>) -> tensor<5x7xi1>",
        "%3 = stablehlo.select %2, %arg0, %arg1 : tensor<5x7xi1>, tensor<5x7xf32>",
        "%4 = stablehlo.iota dim = 1 : tensor<5x7xf32>",
        "%5 = stablehlo.constant dense<1.0> : tensor<f32>",
        "%6 = stablehlo.broadcast_in_dim %5, dims = [] : (tensor<f32>) -> tensor<5x7xf32>",
        "%7 = stablehlo.clamp %1, %3, %6 : tensor<5x7xf32>",
        "%8 = stablehlo.add %7, %4 : tensor<5x7xf32>",
        "%9 = stablehlo.convert %8 : (tensor<5x7xf32>) -> tensor<5x7xi32>",
        "%10 = stablehlo.convert %9 : (tensor<5x7xi32>) -> tensor<5x7xf32>",
        "%11 = stablehlo.compare LE, %arg0, %arg1, FLOAT : (tensor<5x7xf32>, tensor<5x7xf32>) -> tensor<5x7xi1>",
        "%12 = stablehlo.convert %11 : (tensor<5x7xi1>) -> tensor<5x7xf32>",
        "%13 = stablehlo.add %10, %12 : tensor<5x7xf32>",
    ], [("%13", T), ("%8", T)])
    check(fp32_session, name, text, [rnd(5, 7) * 3, rnd(5, 7)])


def test_index_maps(fp32_session):
    name, text = module(["tensor<4x6x10xf32>", "tensor<3x10xf32>"], [
        "%0 = stablehlo.transpose %arg0, dims = [2, 0, 1] : (tensor<4x6x10xf32>) -> tensor<10x4x6xf32>",
        "%1 = stablehlo.reshape %0 : (tensor<10x4x6xf32>) -> tensor<10x24xf32>",
        "%2 = stablehlo.slice %1 [1:9:2, 3:24:3] : (tensor<10x24xf32>) -> tensor<4x7xf32>",
        "%3 = stablehlo.reverse %2, dims = [1] : (tensor<4x7xf32>) -> tensor<4x7xf32>",
        "%4 = stablehlo.constant dense<-2.5> : tensor<f32>",
        "%5 = stablehlo.pad %3, %4, low = [1, 0], high = [2, 3], interior = [0, 1] : (tensor<4x7xf32>, tensor<f32>) -> tensor<7x16xf32>",
        "%6 = stablehlo.slice %arg1 [0:3:1, 0:10:1] : (tensor<3x10xf32>) -> tensor<3x10xf32>",
        "%7 = stablehlo.reshape %6 : (tensor<3x10xf32>) -> tensor<30xf32>",
        "%8 = stablehlo.slice %7 [0:16:1] : (tensor<30xf32>) -> tensor<16xf32>",
        "%9 = stablehlo.reshape %8 : (tensor<16xf32>) -> tensor<1x16xf32>",
        "%10 = stablehlo.concatenate %5, %9, dim = 0 : (tensor<7x16xf32>, tensor<1x16xf32>) -> tensor<8x16xf32>",
        "%11 = stablehlo.exponential %10 : tensor<8x16xf32>",
    ], [("%11", "tensor<8x16xf32>")])
    check(fp32_session, name, text, [rnd(4, 6, 10), rnd(3, 10)])


def test_gather_with_out_of_range_indices_clamps(fp32_session):
    name, text = module(["tensor<7x5xf32>", "tensor<2x3xf32>"], [
        "%0 = stablehlo.convert %arg1 : (tensor<2x3xf32>) -> tensor<2x3xi32>",
        "%1 = stablehlo.reshape %0 : (tensor<2x3xi32>) -> tensor<2x3x1xi32>",
        '%2 = "stablehlo.gather"(%arg0, %1) {\n dimension_numbers = #stablehlo.gather<\n offset_dims = [2],\n'
        ' collapsed_slice_dims = [0],\n operand_batching_dims = [],\n start_indices_batching_dims = [],\n'
        ' start_index_map = [0],\n index_vector_dim = 2>,\n slice_sizes = array<i64: 1, 5>,\n'
        ' indices_are_sorted = false\n } : (tensor<7x5xf32>, tensor<2x3x1xi32>) -> tensor<2x3x5xf32>',
    ], [("%2", "tensor<2x3x5xf32>")])
    idx = np.array([[0, 6, 3], [9, -2, 1]], np.float32)
    check(fp32_session, name, text, [rnd(7, 5), idx], rtol=0, atol=0)


@pytest.mark.parametrize("case", ["2d", "2d_bt", "2d_at", "batched", "batched_tt", "3d_x_2d", "vecmat", "matvec", "dot"])
@pytest.mark.parametrize("prec", ["fp32", "tf32", "bf16"])
def test_dot_general_layouts(request, case, prec):
    sess = request.getfixturevalue(f"{prec}_session")
    M_, N_, K_ = 200, 136, 72
    if case == "2d":
        ps, ins = ["tensor<200x72xf32>", "tensor<72x136xf32>"], [rnd(M_, K_), rnd(K_, N_)]
        body = ["%0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : (tensor<200x72xf32>, tensor<72x136xf32>) -> tensor<200x136xf32>"]
        rt = "tensor<200x136xf32>"
    elif case == "2d_bt":
        ps, ins = ["tensor<200x72xf32>", "tensor<136x72xf32>"], [rnd(M_, K_), rnd(N_, K_)]
        body = ["%t = stablehlo.transpose %arg1, dims = [1, 0] : (tensor<136x72xf32>) -> tensor<72x136xf32>",
                "%0 = stablehlo.dot_general %arg0, %t, contracting_dims = [1] x [0] : (tensor<200x72xf32>, tensor<72x136xf32>) -> tensor<200x136xf32>"]
        rt = "tensor<200x136xf32>"
    elif case == "2d_at":
        ps, ins = ["tensor<72x200xf32>", "tensor<72x136xf32>"], [rnd(K_, M_), rnd(K_, N_)]
        body = ["%t = stablehlo.transpose %arg0, dims = [1, 0] : (tensor<72x200xf32>) -> tensor<200x72xf32>",
                "%0 = stablehlo.dot_general %t, %arg1, contracting_dims = [1] x [0] : (tensor<200x72xf32>, tensor<72x136xf32>) -> tensor<200x136xf32>"]
        rt = "tensor<200x136xf32>"
    elif case == "batched":
        ps, ins = ["tensor<3x200x72xf32>", "tensor<3x72x136xf32>"], [rnd(3, M_, K_), rnd(3, K_, N_)]
        body = ["%0 = stablehlo.dot_general %arg0, %arg1, batching_dims = [0] x [0], contracting_dims = [2] x [1] : (tensor<3x200x72xf32>, tensor<3x72x136xf32>) -> tensor<3x200x136xf32>"]
        rt = "tensor<3x200x136xf32>"
    elif case == "batched_tt":
        ps, ins = ["tensor<2x3x72x200xf32>", "tensor<2x3x136x72xf32>"], [rnd(2, 3, K_, M_), rnd(2, 3, N_, K_)]
        body = ["%a = stablehlo.transpose %arg0, dims = [0, 1, 3, 2] : (tensor<2x3x72x200xf32>) -> tensor<2x3x200x72xf32>",
                "%b = stablehlo.transpose %arg1, dims = [0, 1, 3, 2] : (tensor<2x3x136x72xf32>) -> tensor<2x3x72x136xf32>",
                "%0 = stablehlo.dot_general %a, %b, batching_dims = [0, 1] x [0, 1], contracting_dims = [3] x [2] : (tensor<2x3x200x72xf32>, tensor<2x3x72x136xf32>) -> tensor<2x3x200x136xf32>"]
        rt = "tensor<2x3x200x136xf32>"
    elif case == "3d_x_2d":
        ps, ins = ["tensor<4x50x72xf32>", "tensor<72x136xf32>"], [rnd(4, 50, K_), rnd(K_, N_)]
        body = ["%0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [2] x [0] : (tensor<4x50x72xf32>, tensor<72x136xf32>) -> tensor<4x50x136xf32>"]
        rt = "tensor<4x50x136xf32>"
    elif case == "vecmat":
        ps, ins = ["tensor<72xf32>", "tensor<72x136xf32>"], [rnd(K_), rnd(K_, N_)]
        body = ["%0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [0] x [0] : (tensor<72xf32>, tensor<72x136xf32>) -> tensor<136xf32>"]
        rt = "tensor<136xf32>"
    elif case == "matvec":
        ps, ins = ["tensor<200x72xf32>", "tensor<72xf32>"], [rnd(M_, K_), rnd(K_)]
        body = ["%0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : (tensor<200x72xf32>, tensor<72xf32>) -> tensor<200xf32>"]
        rt = "tensor<200xf32>"
    else:
        ps, ins = ["tensor<72xf32>", "tensor<72xf32>"], [rnd(K_), rnd(K_)]
        body = ["%0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [0] x [0] : (tensor<72xf32>, tensor<72xf32>) -> tensor<f32>"]
        rt = "tensor<f32>"
    name, text = module(ps, body, [("%0", rt)])
    sess.load_stablehlo(text)
    out = sess.call(name, ins)[0]
    ref = run(text, name, ins)[0]
    if prec == "fp32":
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4)
    elif case == "dot":
        # a single 72-term dot product can cancel: bound the error by the sum
        # of |a_k b_k|, the scale TF32 operand rounding errors accumulate on
        scale = float(np.sum(np.abs(ins[0].astype(np.float64) * ins[1])))
        assert abs(float(out) - float(ref)) <= (2e-3 if prec == "tf32" else 6e-3) * scale
    else:
        err = np.linalg.norm(out - ref) / np.linalg.norm(ref)
        assert err <= (2e-3 if prec == "tf32" else 6e-3), err


def test_large_gemm_shapes_match_oracle(tf32_session):
    """M, N, K not multiples of the tile, K large."""
    M_, N_, K_ = 1000, 392, 1536
    name, text = module(["tensor<1000x1536xf32>", "tensor<392x1536xf32>"], [
        "%t = stablehlo.transpose %arg1, dims = [1, 0] : (tensor<392x1536xf32>) -> tensor<1536x392xf32>",
        "%0 = stablehlo.dot_general %arg0, %t, contracting_dims = [1] x [0] : (tensor<1000x1536xf32>, tensor<1536x392xf32>) -> tensor<1000x392xf32>"],
        [("%0", "tensor<1000x392xf32>")])
    ins = [rnd(M_, K_), rnd(N_, K_)]
    tf32_session.load_stablehlo(text)
    out = tf32_session.call(name, ins)[0]
    ref = run(text, name, ins)[0]
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) <= 2e-3


@pytest.mark.parametrize("config", [None, 0, 1, 2, 3, 4, 5])
@pytest.mark.parametrize("shape", [(1000, 1100, 520, 1), (300, 512, 200, 1), (260, 512, 96, 3), (700, 64, 300, 1),
                                   (1000, 300, 800, 1), (520, 272, 1000, 2), (384, 384, 4096, 1),
                                   # row strides that are not a multiple of 4 floats (padded operand copies)
                                   (1000, 65, 384, 1), (65, 384, 4000, 1), (700, 384, 65, 1), (130, 70, 333, 2)])
@pytest.mark.parametrize("at,bt", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_tiles_and_layouts(tf32_session, monkeypatch, config, shape, at, bt):
    """Every tcgen05 GEMM configuration (SHEAF_B200_GEMM_CONFIG: single-CTA
    128 x 64 / 128 x 128 tiles with two TMEM accumulators, CTA-pair 256 x 128 /
    256 x 192 / 256 x 256 tiles) and the cost-model choice (None), with ragged
    M/N/K edges, K-major and MN-major operands, batched, split-K, and operands
    whose row stride is not 16-byte aligned (copied to padded buffers)."""
    if config is not None:
        monkeypatch.setenv("SHEAF_B200_GEMM_CONFIG", str(config))
    M_, N_, K_, B_ = shape
    lead = [B_] if B_ > 1 else []
    sa = lead + ([K_, M_] if at else [M_, K_])
    sb = lead + ([N_, K_] if bt else [K_, N_])
    ty = lambda s: "tensor<" + "x".join(map(str, s)) + "xf32>"
    nb = len(lead)
    perm = "[" + ", ".join(map(str, list(range(nb)) + [nb + 1, nb])) + "]"
    body, a, b = [], "%arg0", "%arg1"
    if at:
        body.append(f"%ta = stablehlo.transpose %arg0, dims = {perm} : ({ty(sa)}) -> {ty(lead + [M_, K_])}")
        a = "%ta"
    if bt:
        body.append(f"%tb = stablehlo.transpose %arg1, dims = {perm} : ({ty(sb)}) -> {ty(lead + [K_, N_])}")
        b = "%tb"
    batch = "batching_dims = [0] x [0], " if nb else ""
    rt = ty(lead + [M_, N_])
    body.append(f"%0 = stablehlo.dot_general {a}, {b}, {batch}contracting_dims = [{nb + 1}] x [{nb}] : "
                f"({ty(lead + [M_, K_])}, {ty(lead + [K_, N_])}) -> {rt}")
    name, text = module([ty(sa), ty(sb)], body, [("%0", rt)])
    ins = [rnd(*sa), rnd(*sb)]
    tf32_session.load_stablehlo(text)
    out = tf32_session.call(name, ins)[0]
    A = ins[0].astype(np.float64)
    Bm = ins[1].astype(np.float64)
    if at:
        A = np.swapaxes(A, -1, -2)
    if bt:
        Bm = np.swapaxes(Bm, -1, -2)
    ref = np.matmul(A, Bm)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) <= 2e-3


@pytest.mark.parametrize("shape,layout", [((1000, 300, 800), "nt"), ((384, 384, 16384), "tn"), ((2048, 256, 512), "nn")])
def test_gemm_configs_bit_identical(tf32_session, monkeypatch, shape, layout):
    """Every tensor-core configuration gives the same bits (tiling changes, the
    K summation order does not), so the measured configuration choice cannot
    change results between runs."""
    M_, N_, K_ = shape
    at, bt = layout[0] == "t", layout[1] == "t"
    ty = lambda r, c: f"tensor<{r}x{c}xf32>"
    sa, sb = (ty(K_, M_) if at else ty(M_, K_)), (ty(N_, K_) if bt else ty(K_, N_))
    body, a, b = [], "%arg0", "%arg1"
    if at:
        body.append(f"%ta = stablehlo.transpose %arg0, dims = [1, 0] : ({sa}) -> {ty(M_, K_)}")
        a = "%ta"
    if bt:
        body.append(f"%tb = stablehlo.transpose %arg1, dims = [1, 0] : ({sb}) -> {ty(K_, N_)}")
        b = "%tb"
    body.append(f"%0 = stablehlo.dot_general {a}, {b}, contracting_dims = [1] x [0] : "
                f"({ty(M_, K_)}, {ty(K_, N_)}) -> {ty(M_, N_)}")
    name, text = module([sa, sb], body, [("%0", ty(M_, N_))])
    ins = [rnd(K_, M_) if at else rnd(M_, K_), rnd(N_, K_) if bt else rnd(K_, N_)]
    outs = []
    for cfg in range(6):
        monkeypatch.setenv("SHEAF_B200_GEMM_CONFIG", str(cfg))
        tf32_session.load_stablehlo(text)
        outs.append(tf32_session.call(name, ins)[0])
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_input_validation_errors(fp32_session):
    from sheaf_b200.session import B200Error
    name, text = module(["tensor<4xf32>"], ["%0 = stablehlo.exponential %arg0 : tensor<4xf32>"], [("%0", "tensor<4xf32>")])
    fp32_session.load_stablehlo(text)
    with pytest.raises(B200Error) as e:
        fp32_session.call(name, [np.zeros(5, np.float32)])
    assert e.value.code == 3 and "shape mismatch" in str(e.value)
    with pytest.raises(B200Error) as e:
        fp32_session.call(name, [])
    assert e.value.code == 3
    with pytest.raises(B200Error) as e:
        fp32_session.call("nope.f", [np.zeros(4, np.float32)])
    assert e.value.code == 5


def test_returned_parameter_and_duplicate_outputs(fp32_session):
    name, text = module(["tensor<3xf32>"], [
        "%0 = stablehlo.constant dense<0.0> : tensor<2x2xf32>",
        "%1 = stablehlo.exponential %arg0 : tensor<3xf32>"],
        [("%arg0", "tensor<3xf32>"), ("%1", "tensor<3xf32>"), ("%1", "tensor<3xf32>"), ("%0", "tensor<2x2xf32>")])
    check(fp32_session, name, text, [rnd(3)])


def test_merged_sibling_projections(fp32_session):
    """The q/k/v projections merged into one GEMM give the three products."""
    from test_abi import QKV
    check(fp32_session, "qkv.f", QKV, [rnd(8, 128, 64), rnd(192, 64)], rtol=1e-4, atol=1e-4)


def test_row_group_with_column_reduction(fp32_session):
    """Row group with a column-reduction member (per-block partials, finish
    kernel) against the oracle, twice (the partials buffer is reused)."""
    from test_abi import LN_BWD_COLS
    for _ in range(2):
        ins = [rnd(16, 128, 128), rnd(16, 128, 128)]
        check(fp32_session, "lnc.f", LN_BWD_COLS, ins, rtol=1e-4, atol=1e-4)


def test_profile_report_counts_every_launch(fp32_session):
    """The per-step launch counts of the profile report add up to the kernels
    the library's launch counter sees for the same call (fp32: no rounded
    parameter copies outside the steps)."""
    from sheaf_lowering import models as M
    from sheaf_b200.session import library
    c = M.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=128, vocab_size=65, batch=2)
    low = M.gpt_vag(c)
    inp = M.gpt_inputs(c, seed=1)
    ins = [inp[n] for n in low.arg_names]
    fp32_session.load_stablehlo(low.text)
    fp32_session.call(low.qualified, ins)
    lib = library()
    n0 = lib.sb_kernel_launch_count()
    fp32_session.call(low.qualified, ins)
    per_call = lib.sb_kernel_launch_count() - n0
    fp32_session.profile_report(reset=True)
    fp32_session.set_profiling(True)
    fp32_session.call(low.qualified, ins)
    fp32_session.set_profiling(False)
    rows = [r for r in fp32_session.profile_report() if r["function"] == low.qualified]
    assert rows and sum(r["launches_per_call"] for r in rows) == per_call
