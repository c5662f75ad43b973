"""Ahead-of-time bundles: a module built on the host loads into a session whose
kernel cache is empty without compiling anything, and computes exactly what
the same module loaded from text computes."""
import os

import numpy as np
import pytest

from sheaf_lowering import models as M
from sheaf_b200.session import B200Error, B200Session, build_bundle

pytestmark = pytest.mark.gpu


def test_bundle_loads_without_compiling(lib, tmp_path, tf32_session):
    c = M.GPTConfig(2, 2, 64, 128, 65, 2, 128)
    low = M.gpt_vag(c, batch=2)
    inp = M.gpt_inputs(c, batch=2, seed=1)
    args = [inp[n] for n in low.arg_names]
    bundle = build_bundle(low.text, "tf32")
    empty = tmp_path / "cache"
    empty.mkdir()
    s = B200Session(device=0, precision="tf32", cache_dir=str(empty))
    try:
        s.load_bundle(bundle)
        assert os.listdir(empty) == []  # nothing was compiled or cached
        got = s.call(low.qualified, args)
    finally:
        s.close()
    tf32_session.load_stablehlo(low.text)
    ref = tf32_session.call(low.qualified, args)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


def test_bundle_precision_must_match(lib, fp32_session):
    low, = [M.mlp_vag(batch=8)]
    with pytest.raises(B200Error):
        fp32_session.load_bundle(build_bundle(low.text, "tf32"))
    with pytest.raises(B200Error):
        fp32_session.load_bundle(b"not a bundle")
