"""The allocation-free split-K GEMM entry point against the session GEMM.

`sb_gemm_f32_splitk_noalloc` serves callers that cannot allocate device memory
(memory owned by another framework, allocator-free paths): its split-K partial
products live in a static device array instead of a workspace.  Here it is
called through the C ABI on device buffers owned by a session, twice in a row
with different shapes (both split K, so the second call reuses the array the
first one filled), and each result is compared with what the regular entry
point (`sb_session_call` on the equivalent `dot_general`) computes.  This file
is collected last so a failure here cannot hide any other test's result.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dot_module(name, m, n, k):
    ta, tb, tc = f"tensor<{m}x{k}xf32>", f"tensor<{k}x{n}xf32>", f"tensor<{m}x{n}xf32>"
    return (f"module @{name} {{\n func.func @f(%arg0: {ta}, %arg1: {tb}) -> {tc} {{\n"
            f"    %0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : ({ta}, {tb}) -> {tc}\n"
            f"    return %0 : {tc}\n }}\n}}\n")


def _noalloc(lib, sess, a, b, c, m, n, k):
    return lib.sb_gemm_f32_splitk_noalloc(ctypes.c_void_p(a.device_pointer), ctypes.c_void_p(b.device_pointer),
                                          ctypes.c_void_p(c.device_pointer), m, n, k,
                                          ctypes.c_void_p(sess.cuda_stream))


def _device_free_bytes():
    import torch
    torch.cuda.synchronize(0)
    return torch.cuda.mem_get_info(0)[0]


@pytest.mark.parametrize("shapes", [[(256, 256, 16384), (200, 136, 4096)]])
def test_noalloc_gemm_matches_session_gemm_on_two_calls(lib, fp32_session, shapes):
    rng = np.random.default_rng(7)
    # everything the session allocates (reference results, operand buffers) is
    # set up first, so that only the two allocation-free calls run between the
    # two readings of the device's free memory
    cases = []
    for call, (m, n, k) in enumerate(shapes):
        a_h = rng.standard_normal((m, k), dtype=np.float32)
        b_h = rng.standard_normal((k, n), dtype=np.float32)
        name = f"noalloc_ref_{call}_{m}_{n}_{k}"
        fp32_session.load_stablehlo(_dot_module(name, m, n, k))
        ref = fp32_session.call(f"{name}.f", [a_h, b_h])[0]
        a, b = fp32_session.buffer(a_h), fp32_session.buffer(b_h)
        c = fp32_session.buffer(np.full((m, n), np.nan, np.float32))
        cases.append((m, n, k, a, b, c, ref))
    # the first call on the device looks up the static array's address, which
    # makes CUDA load the module holding it (lazy loading): the array's 16 MiB
    # appear then, once per process, like any module's code and data
    w = fp32_session.buffer(np.zeros((128, 2048), np.float32))
    assert _noalloc(lib, fp32_session, w, fp32_session.buffer(np.zeros((2048, 128), np.float32)),
                    fp32_session.buffer(np.zeros((128, 128), np.float32)), 128, 128, 2048) == 0
    fp32_session.synchronize()
    free_before = _device_free_bytes()
    for m, n, k, a, b, c, _ in cases:
        assert _noalloc(lib, fp32_session, a, b, c, m, n, k) == 0
    fp32_session.synchronize()
    # the calls took no device memory (the static array was there already)
    assert _device_free_bytes() == free_before
    for m, n, k, a, b, c, ref in cases:
        out = c.to_host()
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5 * np.sqrt(k))
        # both entry points run the same CUDA-core split-K schedule
        assert np.array_equal(out, ref)


def test_noalloc_gemm_rejects_partials_beyond_the_static_array(lib, fp32_session):
    m = n = 1024
    k = 65536  # 64 tiles -> 5 K slices x 1M partials > 4M floats
    a = fp32_session.buffer(np.zeros((m, 1), np.float32))  # never read: the call is rejected first
    assert _noalloc(lib, fp32_session, a, a, a, m, n, k) == 8  # SB_STATUS_RESOURCE_EXHAUSTED
    assert _noalloc(lib, fp32_session, a, a, a, -1, n, k) == 3  # SB_STATUS_INVALID_ARGUMENT
    # more rows than one CUDA-core launch covers (65535 tiles of 128)
    assert _noalloc(lib, fp32_session, a, a, a, 65535 * 128 + 1, 1, 1) == 3
