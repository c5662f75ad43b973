"""CUDA-graph replay of calls (from the second call of a function on).

Checked through the C ABI: replays give bit-identical results to the eager
first call; inputs at a new address each call (a fresh token batch) are
staged and read correctly; outputs held by the caller make the next call use
another output slot (or run eagerly once all slots are held), without
changing any result; the launch counter counts the replayed kernels.
"""
import numpy as np
import pytest

from sheaf_lowering import models as M

pytestmark = pytest.mark.gpu

C = M.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=128, vocab_size=65, batch=2)


@pytest.fixture(scope="module")
def gpt(lib):
    from sheaf_b200.session import B200Session
    sess = B200Session(precision="tf32")
    low = M.gpt_vag(C)
    sess.load_stablehlo(low.text)
    yield sess, low
    sess.close()


def _inputs(seed):
    return M.gpt_inputs(C, seed=seed)


def _call(sess, low, inp, bufs=None):
    bufs = bufs or {}
    args = [bufs.get(n) or sess.buffer(inp[n]) for n in low.arg_names]
    outs = sess.call_device(low.qualified, args)
    return outs, [o.to_host() for o in outs]


def test_replay_is_bit_identical_to_the_eager_call(gpt):
    sess, low = gpt
    inp = _inputs(1)
    params = {n: sess.buffer(inp[n]) for n in low.arg_names if n not in ("x", "y")}
    results = []
    for _ in range(4):  # call 1 eager, then capture + replays
        outs, host = _call(sess, low, inp, params)
        results.append(host)
        for o in outs:
            o.release()
    for r in results[1:]:
        for a, b in zip(results[0], r):
            assert np.array_equal(a, b)


def test_new_token_batches_each_call(gpt):
    sess, low = gpt
    inp0 = _inputs(2)
    params = {n: sess.buffer(inp0[n]) for n in low.arg_names if n not in ("x", "y")}
    batches = [_inputs(10 + k) for k in range(3)]
    ref = []
    for b in batches:  # reference: each batch at least once
        outs, host = _call(sess, low, {**inp0, "x": b["x"], "y": b["y"]}, params)
        ref.append(host)
        for o in outs:
            o.release()
    for k in (2, 0, 1, 2):  # x and y in new buffers every call
        outs, host = _call(sess, low, {**inp0, "x": batches[k]["x"], "y": batches[k]["y"]}, params)
        for a, b in zip(ref[k], host):
            assert np.array_equal(a, b)
        for o in outs:
            o.release()


def test_held_outputs_are_never_overwritten(gpt):
    from sheaf_b200 import session as S
    sess, low = gpt
    inp = _inputs(3)
    params = {n: sess.buffer(inp[n]) for n in low.arg_names if n not in ("x", "y")}
    held = []
    n0 = S.library().sb_kernel_launch_count()
    for k in range(7):  # more calls than output slots, none released
        b = _inputs(20 + k)
        outs, host = _call(sess, low, {**inp, "x": b["x"], "y": b["y"]}, params)
        held.append((outs, host))
    assert S.library().sb_kernel_launch_count() > n0
    sess.synchronize()
    for outs, host in held:  # every call's outputs still hold that call's values
        for o, h in zip(outs, host):
            assert np.array_equal(o.to_host(), h)
        for o in outs:
            o.release()


def test_read_only_host_tensors_are_uploaded_once(gpt):
    """IreeSession's buffer cache (iree_session.rs:612-660): an immutable host
    tensor passed again is not uploaded again; a writeable one is."""
    sess, low = gpt
    inp = _inputs(5)
    frozen = {}
    for n in low.arg_names:
        a = np.array(inp[n])
        a.setflags(write=False)
        frozen[n] = a
    h0, m0 = sess.upload_hits, sess.upload_misses
    first = sess.call(low.qualified, [frozen[n] for n in low.arg_names])
    assert sess.upload_misses - m0 == len(low.arg_names)
    second = sess.call(low.qualified, [frozen[n] for n in low.arg_names])
    assert sess.upload_hits - h0 == len(low.arg_names)
    for a, b in zip(first, second):
        assert np.array_equal(a, b)
    # a writeable array is uploaded on every call (it may have changed)
    m1 = sess.upload_misses
    sess.call(low.qualified, [inp[n] for n in low.arg_names])
    assert sess.upload_misses == m1
