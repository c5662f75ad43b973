"""Sheaf's JIT random ops (random-key/split/uniform/normal/randint) as device
kernels: the emitted StableHLO (sheaf_lowering/random.py) checked against
an independent restatement of the i32 hash on the host, and the device
results against the oracle: the integer hash, uniforms, randints and keys bit
for bit, normals (log/cos/sqrt on two math libraries) to a few ulps."""
import numpy as np
import pytest

from oracle.stablehlo_ref import run
from sheaf_lowering import models as M
from sheaf_lowering import random as RG


def _w(x):
    x = np.asarray(x, np.int64)
    return ((x + (1 << 31)) & 0xFFFFFFFF) - (1 << 31)


def _hash_uniform(lo, hi, n):
    """random_ops.rs:100-180 restated directly: i32 hash of iota(n), abs, / 2^31."""
    i = np.arange(n, dtype=np.int64)
    x = _w(_w(_w(_w((i + lo) * 1540483477) + hi) * 668265263) + 1013904223)
    return _w(np.abs(x)).astype(np.float32) / np.float32(2147483648.0)


SEEDS = [0, 42, (1 << 33) + 7, (1 << 63) - 1]


@pytest.mark.parametrize("seed", SEEDS)
def test_emitted_hash_matches_restatement(seed):
    low = RG.sample_program("uniform", (7, 9))
    key = RG.key_of_seed(seed)
    u = run(low.text, low.qualified, [key], dtype=np.float32)[0]
    lo, hi = (int(v) for v in key.view(np.int32))
    assert np.array_equal(u.ravel(), _hash_uniform(lo, hi, 63))


def test_split_and_randint_forms():
    key = RG.key_of_seed(42)
    low = RG.sample_program("split", None)
    ks = [k.view(np.int32) for k in run(low.text, low.qualified, [key], dtype=np.float32)]
    for i, k in enumerate(ks):
        assert int(k[0]) == int(_w((42 + i) * 2069105475 + 1013904223)) and int(k[1]) == 42 + i
    low = RG.sample_program("randint", (5000,), 3, 9)
    r = run(low.text, low.qualified, [key], dtype=np.float32)[0]
    assert r.min() == 3 and r.max() == 8 and np.all(r == np.floor(r))


def test_init_program_plans_with_sorted_leaves(lib):
    from sheaf_b200.session import inspect_module
    low = RG.gpt_init_program(M.NANOGPT)
    assert low.result_names == sorted(n for n, _ in M.gpt_param_leaves(M.NANOGPT))
    assert "loop=" in inspect_module(low.text, "fp32")


GPU = pytest.mark.gpu


@GPU
@pytest.mark.parametrize("kind,shape", [("uniform", (1000,)), ("uniform", (33, 65)), ("randint", (4096,)),
                                        ("normal", (777,)), ("normal", (64, 384)), ("split", None)])
@pytest.mark.parametrize("seed", [3, (1 << 35) + 11])
def test_device_random_ops(fp32_session, kind, shape, seed):
    low = RG.sample_program(kind, shape, 2, 50)
    key = RG.key_of_seed(seed)
    fp32_session.load_stablehlo(low.text)
    outs = fp32_session.call(low.qualified, [key])
    refs = run(low.text, low.qualified, [key], dtype=np.float32)
    for o, r in zip(outs, refs):
        if kind == "normal":
            np.testing.assert_allclose(o, r, rtol=1e-5, atol=2e-6)
        else:
            assert np.array_equal(o.view(np.int32), r.astype(np.float32).view(np.int32))


@GPU
def test_device_random_key_from_seed_constant(fp32_session):
    low = RG.sample_program("uniform", (256,), seed=(1 << 40) + 12345)
    fp32_session.load_stablehlo(low.text)
    out = fp32_session.call(low.qualified, [])[0]
    assert np.array_equal(out, _hash_uniform(12345, 256, 256))


@GPU
def test_device_gpt_init_params(fp32_session):
    c = M.GPTConfig(2, 2, 64, 32, 65, 1, 32)
    low = RG.gpt_init_program(c)
    key = RG.key_of_seed(1337)
    fp32_session.load_stablehlo(low.text)
    outs = fp32_session.call(low.qualified, [key])
    refs = run(low.text, low.qualified, [key], dtype=np.float32)
    for name, o, r in zip(low.result_names, outs, refs):
        assert o.shape == r.shape, name
        np.testing.assert_allclose(o, r, rtol=1e-5, atol=1e-7, err_msg=name)
    std = np.std(outs[low.result_names.index("transformer.h.0.attn.c_attn.weight")])
    assert 0.015 < std < 0.025
