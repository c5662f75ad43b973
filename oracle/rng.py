"""CPU restatement of the Sheaf interpreter's RNG (test infrastructure only).

Follows sheaf/src/interpreter/builtins/random.rs:
  random-key  seed -> [lo, hi] as f32                          (:14-28)
  key->seed   lo | hi << 32                                     (:30-44)
  splitmix64  state += 0x9e3779b97f4a7c15; mix; (z >> 11) / 2^53 in f32 (:68-75)
  random-normal  Box-Muller pairs in f32, u1 clamped at 1e-10  (:77-99)
Used to reproduce the reference's seeded test inputs (e.g. the MLP
value-and-grad golden at sheaf/tests/interpreter_tests.yaml:753-762).
"""
import numpy as np

_M64 = (1 << 64) - 1


def key_to_seed(seed: int) -> int:
    lo = float(np.float32(seed & 0xFFFFFFFF))
    hi = float(np.float32((seed >> 32) & 0xFFFFFFFF))
    return (int(lo) | (int(hi) << 32)) & _M64


def _splitmix(state):
    state = (state + 0x9E3779B97F4A7C15) & _M64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    z = z ^ (z >> 31)
    return state, np.float32(np.float32(z >> 11) / np.float32(1 << 53))


def random_normal(seed: int, shape) -> np.ndarray:
    state = key_to_seed(seed)
    n = int(np.prod(shape))
    out = []
    two_pi = np.float32(2.0) * np.float32(np.pi)
    while len(out) < n:
        state, u1 = _splitmix(state)
        u1 = max(u1, np.float32(1e-10))
        state, u2 = _splitmix(state)
        r = np.sqrt(np.float32(-2.0) * np.log(np.float32(u1)))
        th = np.float32(two_pi * u2)
        out.append(np.float32(r * np.cos(th)))
        if len(out) < n:
            out.append(np.float32(r * np.sin(th)))
    return np.array(out[:n], dtype=np.float32).reshape(shape)


def random_uniform(seed: int, shape) -> np.ndarray:
    state = key_to_seed(seed)
    n = int(np.prod(shape))
    out = []
    for _ in range(n):
        state, u = _splitmix(state)
        out.append(u)
    return np.array(out, dtype=np.float32).reshape(shape)
