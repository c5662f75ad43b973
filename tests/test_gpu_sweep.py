"""The op sweep (softmax, layer-norm, gelu; forward and VJP; f32 and bf16) on
the GPU against the oracle.

Tolerances: f32, 1e-5 norm-relative (non-contraction ops); bf16, where every
op rounds its result to bf16 (2^-9 relative) and the two implementations sum
rows in different orders, 1e-2 norm-relative.  Sizes: every D of the sweep
(384, 768, 4096) on 4096 rows and gelu on 2^20 elements, plus the full sweep
sizes ([65536, 768], gelu on 2^28 elements) in f32, the oracle running in
spawned workers meanwhile.
"""
import numpy as np
import pytest

import oracle_jobs
from oracle.stablehlo_ref import run
from sheaf_lowering import models as M

pytestmark = pytest.mark.gpu


def _rel(o, r):
    r = np.asarray(r, np.float64)
    return float(np.linalg.norm(np.asarray(o, np.float64) - r) / max(np.linalg.norm(r), 1e-30))


def _gpu(sess, low, inp, bf16):
    if not sess.has_function(low.qualified):
        sess.load_stablehlo(low.text)
    bufs = [sess.buffer(inp[n], bf16=bf16) for n in low.arg_names]
    outs = sess.call_device(low.qualified, bufs)
    host = [o.to_host() for o in outs]
    for o in outs + bufs:
        o.release()
    return host


CASES = [(op, shape, vjp) for op in ("softmax", "layer-norm") for shape in ((4096, 384), (4096, 768), (4096, 4096))
         for vjp in (False, True)] + [("gelu", (1 << 20,), vjp) for vjp in (False, True)]


@pytest.mark.parametrize("op,shape,vjp", CASES)
def test_sweep_f32(fp32_session, op, shape, vjp):
    low = M.sweep_program(op, shape, vjp)
    inp = M.sweep_inputs(op, shape, vjp, seed=3)
    got = _gpu(fp32_session, low, inp, False)
    ref = run(low.text, low.qualified, [inp[n] for n in low.arg_names], dtype=np.float32)
    for g, r in zip(got, ref):
        assert _rel(g, r) <= 1e-5


@pytest.mark.parametrize("op,shape,vjp", [c for c in CASES if c[1] in ((4096, 768), (1 << 20,))])
def test_sweep_bf16(fp32_session, op, shape, vjp):
    low = M.sweep_program(op, shape, vjp, "bf16")
    inp = M.sweep_inputs(op, shape, vjp, seed=4)
    got = _gpu(fp32_session, low, inp, True)
    ref = run(low.text, low.qualified, [inp[n] for n in low.arg_names], dtype=np.float32)
    assert len(got) == len(ref)
    for g, r in zip(got[-1:], ref[-1:]):  # the op's output, or the VJP's dx
        assert _rel(g, r) <= 1e-2


FULL = [("softmax", (65536, 768), True), ("layer-norm", (65536, 768), True), ("gelu", (1 << 28,), True),
        ("gelu", (1 << 28,), False)]


@pytest.fixture(scope="module")
def full_refs():
    return {c: oracle_jobs.pool().apply_async(oracle_jobs.sweep_last_output, c + (5,)) for c in FULL}


@pytest.mark.parametrize("case", FULL)
def test_sweep_full_size_f32(fp32_session, full_refs, case):
    op, shape, vjp = case
    low = M.sweep_program(op, shape, vjp)
    inp = M.sweep_inputs(op, shape, vjp, seed=5)
    got = _gpu(fp32_session, low, inp, False)[-1]
    ref = full_refs[case].get(timeout=1800)
    assert _rel(got, ref) <= 1e-5
