"""Fused optimizer step (clip-by-global-norm + AdamW): the oracle pinned on the
reference's adamw-step goldens (CPU), and the device kernel against the oracle
(GPU, through the C ABI)."""
import json
import os

import numpy as np
import pytest

from oracle import optim_ref as R

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "optim_goldens.json")))["cases"]


@pytest.mark.parametrize("name", sorted(GOLD))
def test_oracle_matches_reference_goldens(name):
    c = GOLD[name]
    p, m, v, t = R.adamw_step([np.float32([c["p"]])], [np.float32([c["g"]])], [np.float32([c["m"]])],
                              [np.float32([c["v"]])], c["t"], c["lr"], c["b1"], c["b2"], c["eps"], c["wd"])
    assert t == c["t"] + 1
    # the reference prints 5-6 significant digits
    assert abs(float(p[0][0]) - c["expected_p"]) <= 1e-5


def test_oracle_clip_by_global_norm():
    g = [np.float32([3.0]), np.float32([[4.0]])]
    assert R.global_norm(g) == np.float32(5.0)
    c = R.clip_by_global_norm(g, 1.0)
    np.testing.assert_allclose([c[0][0], c[1][0][0]], [0.6, 0.8], rtol=1e-6)
    # below the threshold the factor is 1
    c = R.clip_by_global_norm(g, 10.0)
    assert c[0][0] == np.float32(3.0) and c[1][0][0] == np.float32(4.0)


def _leaves(rng, sizes, scale=1.0):
    return [(rng.standard_normal(s) * scale).astype(np.float32) for s in sizes]


SIZES = [(1,), (3,), (1000,), (65, 384), (100003,), (384,)]


@pytest.mark.gpu
@pytest.mark.parametrize("max_norm", [0.0, 1.0, 1e6])
def test_device_adamw_matches_oracle(tf32_session, max_norm):
    rng = np.random.default_rng(7)
    p, g = _leaves(rng, SIZES), _leaves(rng, SIZES, 0.3)
    m, v = _leaves(rng, SIZES, 0.01), [np.abs(x) for x in _leaves(rng, SIZES, 1e-3)]
    hp = dict(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1)
    t = 4
    bp, bg, bm, bv = ([tf32_session.buffer(x) for x in xs] for xs in (p, g, m, v))
    t1, norm = tf32_session.adamw_step(bp, bg, bm, bv, t, max_grad_norm=max_norm, return_norm=True, **hp)
    rp, rm, rv, rt = R.train_update(p, g, m, v, t, max_norm=max_norm, **hp)
    assert t1 == rt == t + 1
    assert abs(norm - float(R.global_norm(g))) <= 1e-5 * float(R.global_norm(g))
    for dev, ref in ((bp, rp), (bm, rm), (bv, rv)):
        for d, r in zip(dev, ref):
            np.testing.assert_allclose(d.to_host(), r, rtol=2e-6, atol=1e-7)
    # gradients are left untouched
    for d, r in zip(bg, g):
        assert np.array_equal(d.to_host(), r)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(GOLD))
def test_device_adamw_reference_goldens(tf32_session, name):
    c = GOLD[name]
    bufs = [tf32_session.buffer(np.float32([c[k]])) for k in ("p", "g", "m", "v")]
    t1 = tf32_session.adamw_step(*([b] for b in bufs), c["t"], c["lr"], c["b1"], c["b2"], c["eps"], c["wd"])
    assert t1 == c["t"] + 1
    assert abs(float(bufs[0].to_host()[0]) - c["expected_p"]) <= 1e-5


@pytest.mark.gpu
def test_device_adamw_deterministic_and_validates(tf32_session):
    from sheaf_b200.session import B200Error
    rng = np.random.default_rng(3)
    g = _leaves(rng, SIZES)
    norms = []
    for _ in range(2):
        bp, bm, bv = ([tf32_session.buffer(np.zeros(s, np.float32)) for s in SIZES] for _ in range(3))
        bg = [tf32_session.buffer(x) for x in g]
        _, n = tf32_session.adamw_step(bp, bg, bm, bv, 0, 1e-3, 0.9, 0.999, 1e-8, 0.0, max_grad_norm=1.0,
                                       return_norm=True)
        norms.append((n, [b.to_host() for b in bp]))
    assert norms[0][0] == norms[1][0]
    for a, b in zip(norms[0][1], norms[1][1]):
        assert np.array_equal(a, b)
    # mismatched leaf sizes are rejected before any launch
    with pytest.raises(B200Error):
        tf32_session.adamw_step([tf32_session.buffer(np.zeros(3, np.float32))],
                                [tf32_session.buffer(np.zeros(4, np.float32))],
                                [tf32_session.buffer(np.zeros(3, np.float32))],
                                [tf32_session.buffer(np.zeros(3, np.float32))], 0, 1e-3, 0.9, 0.999, 1e-8, 0.0)
