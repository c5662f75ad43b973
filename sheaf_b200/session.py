"""Python host mirror of Sheaf's `IreeSession` over the libsheafb200 C ABI.

Method names and behaviour follow sheaf/src/runtime/iree_session.rs:
  `B200Session(...)`              IreeSession::new (:174)
  `load_stablehlo(text)`          iree-compile + IreeSession::load_vmfb (:373)
  `call(name, args)`              IreeSession::call (:409): host arrays in, host arrays out
  `call_device(name, args)`       IreeSession::call_device (:574): outputs stay on the GPU
  `DeviceBuffer.to_host()`        DeviceBufferInner::to_host (device_buffer.rs:47)
Host tensors are f32 (Sheaf's `Value::Tensor` is `ArrayD<f32>`,
sheaf/src/interpreter/value.rs:69-93); integer index tensors travel as f32
(buffer_convert.rs:41-47).  Errors raise `B200Error` carrying the status code.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsheafb200.so")

ELEMENT_TYPE_FLOAT_32 = (0x21 << 24) | 32
ELEMENT_TYPE_BFLOAT_16 = (0x31 << 24) | 16
ELEMENT_TYPE_INT_32 = (0x11 << 24) | 32

PRECISIONS = {"fp32": 0, "tf32": 1, "bf16": 2}
REDUCE = {None: 0, "none": 0, "sum": 1, "mean": 2}

_NP_OF_ETYPE = {ELEMENT_TYPE_FLOAT_32: np.float32, ELEMENT_TYPE_INT_32: np.int32}
_ETYPE_OF_NP = {np.dtype(np.float32): ELEMENT_TYPE_FLOAT_32, np.dtype(np.int32): ELEMENT_TYPE_INT_32}


class B200Error(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class _Options(ctypes.Structure):
    _fields_ = [("device_ordinal", ctypes.c_int32), ("precision", ctypes.c_int32),
                ("rank", ctypes.c_int32), ("world_size", ctypes.c_int32),
                ("nccl_unique_id", ctypes.c_uint8 * 128), ("collective_timeout_ms", ctypes.c_int64),
                ("kernel_cache_dir", ctypes.c_char_p), ("flags", ctypes.c_uint32)]


class _AdamwOptions(ctypes.Structure):
    _fields_ = [("learning_rate", ctypes.c_float), ("beta1", ctypes.c_float), ("beta2", ctypes.c_float),
                ("epsilon", ctypes.c_float), ("weight_decay", ctypes.c_float), ("max_grad_norm", ctypes.c_float),
                ("step", ctypes.c_int64)]


class _Stats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("host_bytes_peak", "host_bytes_allocated", "host_bytes_freed",
                                                "device_bytes_peak", "device_bytes_allocated", "device_bytes_freed")]


# Every symbol include/sheaf_b200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
SIGNATURES = {
    "sb_status_code_of": (ctypes.c_int, [_P]),
    "sb_status_message": (ctypes.c_char_p, [_P]),
    "sb_status_free": (None, [_P]),
    "sb_session_options_initialize": (None, [ctypes.POINTER(_Options)]),
    "sb_session_create": (_P, [ctypes.POINTER(_Options), ctypes.POINTER(_P)]),
    "sb_session_release": (None, [_P]),
    "sb_session_synchronize": (_P, [_P]),
    "sb_session_allocator_stats": (_P, [_P, ctypes.POINTER(_Stats)]),
    "sb_session_cuda_stream": (_P, [_P]),
    "sb_session_set_profiling": (_P, [_P, ctypes.c_int]),
    "sb_session_profile_report": (_P, [_P, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t,
                                       ctypes.POINTER(ctypes.c_size_t)]),
    "sb_session_load_stablehlo": (_P, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "sb_session_has_function": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "sb_session_call": (_P, [_P, ctypes.c_char_p, ctypes.POINTER(_P), ctypes.c_size_t,
                             ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(_P), ctypes.c_size_t,
                             ctypes.POINTER(ctypes.c_size_t)]),
    "sb_buffer_allocate_copy": (_P, [_P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint32,
                                     _P, ctypes.c_size_t, ctypes.POINTER(_P)]),
    "sb_buffer_wrap_device": (_P, [_P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint32,
                                   _P, ctypes.c_size_t, ctypes.POINTER(_P)]),
    "sb_buffer_d2h": (_P, [_P, _P, _P, ctypes.c_size_t, ctypes.c_int64]),
    "sb_buffer_retain": (None, [_P]),
    "sb_buffer_release": (None, [_P]),
    "sb_buffer_rank": (ctypes.c_size_t, [_P]),
    "sb_buffer_dim": (ctypes.c_uint64, [_P, ctypes.c_size_t]),
    "sb_buffer_element_type": (ctypes.c_uint32, [_P]),
    "sb_buffer_byte_length": (ctypes.c_size_t, [_P]),
    "sb_buffer_device_pointer": (_P, [_P]),
    "sb_nccl_get_unique_id": (_P, [ctypes.POINTER(ctypes.c_uint8)]),
    "sb_module_build_bundle": (_P, [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_uint32, _P,
                                    ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "sb_session_load_bundle": (_P, [_P, _P, ctypes.c_size_t]),
    "sb_adamw_options_initialize": (None, [ctypes.POINTER(_AdamwOptions)]),
    "sb_optimizer_adamw_step": (_P, [_P, ctypes.c_size_t, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P),
                                     ctypes.POINTER(_P), ctypes.POINTER(_AdamwOptions), ctypes.POINTER(ctypes.c_float)]),
    "sb_gemm_f32_splitk_noalloc": (ctypes.c_int, [_P, _P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _P]),
    "sb_module_inspect": (_P, [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_char_p, ctypes.c_size_t]),
    "sb_module_kernel_source": (_P, [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_char_p,
                                     ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "sb_module_plan_steps": (_P, [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_int32,
                                  ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "sb_version": (ctypes.c_char_p, []),
    "sb_kernel_launch_count": (ctypes.c_uint64, []),
}

_lib = None


def library(path: str = LIB_PATH):
    """Loads libsheafb200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise B200Error(14, f"{path} is missing: build it with `python -m sheaf_b200.build`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _check(st):
    if st:
        lib = library()
        code = lib.sb_status_code_of(st)
        msg = lib.sb_status_message(st).decode(errors="replace")
        lib.sb_status_free(st)
        raise B200Error(code, msg)


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    _check(library().sb_nccl_get_unique_id(buf))
    return bytes(buf)


def inspect_module(text: str, precision: str = "tf32") -> str:
    """Parses, plans and compiles a module on the host (no GPU needed)."""
    out = ctypes.create_string_buffer(1 << 16)
    raw = text.encode()
    _check(library().sb_module_inspect(raw, len(raw), PRECISIONS[precision], out, len(out)))
    return out.value.decode()


def plan_steps(text: str, function: str, precision: str = "tf32") -> List[dict]:
    """The execution plan of one function (host only): one dict per step."""
    raw = text.encode()
    n = ctypes.c_size_t(0)
    _check(library().sb_module_plan_steps(raw, len(raw), function.encode(), PRECISIONS[precision], None, 0,
                                          ctypes.byref(n)))
    out = ctypes.create_string_buffer(n.value + 1)
    _check(library().sb_module_plan_steps(raw, len(raw), function.encode(), PRECISIONS[precision], out, len(out),
                                          ctypes.byref(n)))
    lines = out.value.decode().strip().splitlines()
    keys = lines[0].split(",")
    rows = []
    for ln in lines[1:]:
        r = dict(zip(keys, ln.split(",")))
        for k in keys:
            if k not in ("kind", "kernel"):
                r[k] = float(r[k]) if k == "flops" else int(r[k])
        rows.append(r)
    return rows


def build_bundle(text: str, precision: str = "tf32", fuse_attention: bool = True) -> bytes:
    """Ahead-of-time artifact of a module (host only, like `sheaf build`): the
    text plus every fused kernel compiled for sm_100a; B200Session.load_bundle
    loads it without compiling."""
    raw = text.encode()
    flags = 0 if fuse_attention else FLAG_NO_ATTENTION_FUSION
    n = ctypes.c_size_t(0)
    _check(library().sb_module_build_bundle(raw, len(raw), PRECISIONS[precision], flags, None, 0, ctypes.byref(n)))
    buf = (ctypes.c_uint8 * n.value)()
    _check(library().sb_module_build_bundle(raw, len(raw), PRECISIONS[precision], flags, buf, n.value,
                                            ctypes.byref(n)))
    return bytes(buf)


def kernel_source(text: str, function: str) -> str:
    raw = text.encode()
    n = ctypes.c_size_t(0)
    _check(library().sb_module_kernel_source(raw, len(raw), function.encode(), None, 0, ctypes.byref(n)))
    out = ctypes.create_string_buffer(n.value + 1)
    _check(library().sb_module_kernel_source(raw, len(raw), function.encode(), out, len(out), ctypes.byref(n)))
    return out.value.decode()


class DeviceBuffer:
    """A device tensor owned through one reference on an `sb_buffer`."""

    def __init__(self, session: "B200Session", handle, keepalive=None):
        self._s = session
        self._h = handle
        self._keep = keepalive
        self._shape = None
        self._et = None

    # shape and element type are read from the library on first use (a call
    # returns one buffer per gradient leaf; most are only passed on)
    @property
    def shape(self):
        if self._shape is None:
            lib = library()
            self._shape = tuple(int(lib.sb_buffer_dim(self._h, i)) for i in range(lib.sb_buffer_rank(self._h)))
        return self._shape

    @property
    def element_type(self):
        if self._et is None:
            self._et = int(library().sb_buffer_element_type(self._h))
        return self._et

    @property
    def handle(self):
        return self._h

    @property
    def nbytes(self) -> int:
        return int(library().sb_buffer_byte_length(self._h))

    @property
    def device_pointer(self) -> int:
        return int(library().sb_buffer_device_pointer(self._h) or 0)

    def to_host(self, timeout_ms: int = 0) -> np.ndarray:
        if self.element_type == ELEMENT_TYPE_BFLOAT_16:
            # bf16 -> f32 by widening the 16 bits (device_buffer.rs:53-75)
            raw = np.empty(self.shape, dtype=np.uint16)
            _check(library().sb_buffer_d2h(self._s._h, self._h, raw.ctypes.data_as(ctypes.c_void_p), raw.nbytes,
                                           timeout_ms))
            return (raw.astype(np.uint32) << 16).view(np.float32)
        dt = _NP_OF_ETYPE.get(self.element_type, np.float32)
        out = np.empty(self.shape, dtype=dt)
        _check(library().sb_buffer_d2h(self._s._h, self._h, out.ctypes.data_as(ctypes.c_void_p), out.nbytes,
                                       timeout_ms))
        return out

    def release(self):
        if self._h:
            library().sb_buffer_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


FLAG_NO_ATTENTION_FUSION = 2  # SB_SESSION_FLAG_NO_ATTENTION_FUSION
FLAG_OVERLAP_ALLREDUCE = 4  # SB_SESSION_FLAG_OVERLAP_ALLREDUCE


class B200Session:
    """One GPU, one stream.  `world_size > 1` makes `call_device(..., reduce=...)`
    combine outputs across data-parallel ranks with NCCL."""

    def __init__(self, device: int = 0, precision: str = "tf32", rank: int = 0, world_size: int = 1,
                 nccl_id: Optional[bytes] = None, timeout_ms: int = 600000, cache_dir: Optional[str] = None,
                 fuse_attention: bool = True, overlap_allreduce: bool = False):
        lib = library()
        o = _Options()
        lib.sb_session_options_initialize(ctypes.byref(o))
        if not fuse_attention:
            o.flags |= FLAG_NO_ATTENTION_FUSION
        if overlap_allreduce:
            o.flags |= FLAG_OVERLAP_ALLREDUCE
        o.device_ordinal = device
        o.precision = PRECISIONS[precision]
        o.rank = rank
        o.world_size = world_size
        o.collective_timeout_ms = timeout_ms
        if nccl_id is not None:
            ctypes.memmove(o.nccl_unique_id, nccl_id, 128)
        self._cache = cache_dir.encode() if cache_dir else None
        o.kernel_cache_dir = self._cache
        h = ctypes.c_void_p()
        _check(lib.sb_session_create(ctypes.byref(o), ctypes.byref(h)))
        self._h = h
        self.precision = precision
        self.world_size = world_size
        self.rank = rank
        # uploaded host tensors, per function and argument position
        # (IreeSession's buffer cache, iree_session.rs:612-660)
        self._uploads: dict = {}
        self.upload_hits = 0
        self.upload_misses = 0

    def close(self):
        if getattr(self, "_h", None):
            for per_fn in self._uploads.values():
                for entries in per_fn:
                    for _, b in entries:
                        b.release()
            self._uploads = {}
            library().sb_session_release(self._h)
            self._h = None

    # at most this many uploads are kept per argument position
    UPLOAD_CACHE_ENTRIES = 8

    def _upload(self, name: str, i: int, nargs: int, a) -> "DeviceBuffer":
        """Device buffer for host argument i of function `name`.  As Sheaf's
        session skips re-uploading a tensor it has seen (buffer_cache.rs:9-40:
        identity of an immutable Arc'd tensor), an ndarray that cannot be
        written (`a.flags.writeable` False) is uploaded once and found again by
        identity (the cache holds a reference, so the identity stays unique);
        the 8 most recent uploads per argument position are kept.  Writeable
        arrays may change in place between calls and are uploaded every time."""
        if not isinstance(a, np.ndarray) or a.flags.writeable:
            return None
        per_fn = self._uploads.setdefault(name, [])
        while len(per_fn) < nargs:
            per_fn.append([])
        entries = per_fn[i]
        for k, (arr, buf) in enumerate(entries):
            if arr is a:
                self.upload_hits += 1
                if k:
                    entries.insert(0, entries.pop(k))
                return buf
        self.upload_misses += 1
        buf = self.buffer(a)
        entries.insert(0, (a, buf))
        if len(entries) > self.UPLOAD_CACHE_ENTRIES:
            entries.pop()[1].release()
        return buf

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_stablehlo(self, text: str):
        raw = text.encode()
        _check(library().sb_session_load_stablehlo(self._h, raw, len(raw)))

    def load_bundle(self, bundle: bytes):
        """Loads an ahead-of-time bundle (`build_bundle`): no kernel compilation."""
        buf = (ctypes.c_uint8 * len(bundle)).from_buffer_copy(bundle)
        _check(library().sb_session_load_bundle(self._h, buf, len(bundle)))

    def has_function(self, name: str) -> bool:
        return bool(library().sb_session_has_function(self._h, name.encode()))

    @property
    def cuda_stream(self) -> int:
        return int(library().sb_session_cuda_stream(self._h) or 0)

    def synchronize(self):
        _check(library().sb_session_synchronize(self._h))

    def set_profiling(self, enable: bool):
        _check(library().sb_session_set_profiling(self._h, 1 if enable else 0))

    def profile_report(self, reset: bool = True) -> List[dict]:
        """Per-step accumulated device time (see sb_session_profile_report)."""
        n = ctypes.c_size_t(0)
        _check(library().sb_session_profile_report(self._h, 0, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value + 1)
        _check(library().sb_session_profile_report(self._h, 1 if reset else 0, buf, len(buf), ctypes.byref(n)))
        lines = buf.value.decode().strip().splitlines()
        keys = lines[0].split(",")
        rows = []
        for ln in lines[1:]:
            vals = ln.split(",")
            r = dict(zip(keys, vals))
            for k in ("step", "calls", "elements", "bytes", "launches_per_call"):
                r[k] = int(r[k])
            for k in ("total_ms", "flops"):
                r[k] = float(r[k])
            rows.append(r)
        return rows

    def allocator_stats(self) -> dict:
        st = _Stats()
        _check(library().sb_session_allocator_stats(self._h, ctypes.byref(st)))
        return {n: getattr(st, n) for n, _ in _Stats._fields_}

    # buffers -----------------------------------------------------------------
    def buffer(self, array, bf16: bool = False) -> DeviceBuffer:
        """Device copy of a host tensor.  With bf16=True the f32 values are
        stored as bf16 by keeping their upper 16 bits, as Sheaf uploads a
        bf16 tensor (buffer_convert.rs:28-40)."""
        if bf16:
            a = np.ascontiguousarray(array, dtype=np.float32)
            bits = (a.view(np.uint32) >> 16).astype(np.uint16)
            shape = (ctypes.c_uint64 * max(a.ndim, 1))(*a.shape)
            h = ctypes.c_void_p()
            _check(library().sb_buffer_allocate_copy(self._h, a.ndim, shape, ELEMENT_TYPE_BFLOAT_16,
                                                     bits.ctypes.data_as(ctypes.c_void_p), bits.nbytes,
                                                     ctypes.byref(h)))
            return DeviceBuffer(self, h)
        a = np.ascontiguousarray(array)
        if a.dtype == np.float64 or a.dtype.kind in "iub" and a.dtype != np.int32:
            a = a.astype(np.float32)
        if a.dtype not in _ETYPE_OF_NP:
            raise B200Error(3, f"unsupported host dtype {a.dtype}")
        shape = (ctypes.c_uint64 * max(a.ndim, 1))(*a.shape)
        h = ctypes.c_void_p()
        _check(library().sb_buffer_allocate_copy(self._h, a.ndim, shape, _ETYPE_OF_NP[a.dtype],
                                                 a.ctypes.data_as(ctypes.c_void_p), a.nbytes, ctypes.byref(h)))
        return DeviceBuffer(self, h)

    def wrap_torch(self, t) -> DeviceBuffer:
        """Zero-copy view of a contiguous CUDA torch tensor (kept alive by the buffer)."""
        import torch
        if not t.is_cuda or not t.is_contiguous():
            raise B200Error(3, "wrap_torch needs a contiguous CUDA tensor")
        et = {torch.float32: ELEMENT_TYPE_FLOAT_32, torch.int32: ELEMENT_TYPE_INT_32,
              torch.bfloat16: ELEMENT_TYPE_BFLOAT_16}[t.dtype]
        shape = (ctypes.c_uint64 * max(t.dim(), 1))(*t.shape)
        h = ctypes.c_void_p()
        _check(library().sb_buffer_wrap_device(self._h, t.dim(), shape, et, ctypes.c_void_p(t.data_ptr()),
                                               t.numel() * t.element_size(), ctypes.byref(h)))
        return DeviceBuffer(self, h, keepalive=t)

    # calls -------------------------------------------------------------------
    def call_device(self, name: str, args: Sequence, reduce: Optional[Sequence] = None) -> List[DeviceBuffer]:
        bufs = []
        for i, a in enumerate(args):
            if isinstance(a, DeviceBuffer):
                bufs.append(a)
                continue
            b = self._upload(name, i, len(args), a)
            bufs.append(b if b is not None else self.buffer(a))
        arr = (ctypes.c_void_p * max(len(bufs), 1))(*[b.handle for b in bufs])
        cap = 4096
        outs = (ctypes.c_void_p * cap)()
        n = ctypes.c_size_t(0)
        red = None
        if reduce is not None:
            red = (ctypes.c_int32 * len(reduce))(*[REDUCE[r] for r in reduce])
        _check(library().sb_session_call(self._h, name.encode(), arr, len(bufs), red, outs, cap, ctypes.byref(n)))
        return [DeviceBuffer(self, ctypes.c_void_p(outs[i])) for i in range(n.value)]

    # optimizer ---------------------------------------------------------------
    def adamw_step(self, params: Sequence[DeviceBuffer], grads: Sequence[DeviceBuffer], m: Sequence[DeviceBuffer],
                   v: Sequence[DeviceBuffer], t: int, lr: float, b1: float, b2: float, eps: float, wd: float,
                   max_grad_norm: float = 0.0, return_norm: bool = False):
        """`(clip-by-global-norm g max_grad_norm)` then `(adamw-step params g m v t lr b1 b2 eps wd)`
        (sheaf/lib/optim.shf:77-83, :36-58) over the leaf lists, in place on
        the device buffers.  Returns the new t (t + 1), and with return_norm
        the gradients' global norm before clipping (waits for the step)."""
        n = len(params)
        if not (len(grads) == len(m) == len(v) == n):
            raise B200Error(3, "params, grads, m and v must have the same number of leaves")
        arr = lambda bs: (ctypes.c_void_p * max(n, 1))(*[b.handle for b in bs])
        o = _AdamwOptions()
        library().sb_adamw_options_initialize(ctypes.byref(o))
        o.learning_rate, o.beta1, o.beta2, o.epsilon, o.weight_decay = lr, b1, b2, eps, wd
        o.max_grad_norm, o.step = max_grad_norm, t
        norm = ctypes.c_float(0.0)
        _check(library().sb_optimizer_adamw_step(self._h, n, arr(params), arr(grads), arr(m), arr(v), ctypes.byref(o),
                                                 ctypes.byref(norm) if return_norm else None))
        return (t + 1, norm.value) if return_norm else t + 1

    def call(self, name: str, args: Sequence) -> List[np.ndarray]:
        outs = self.call_device(name, args)
        res = [o.to_host() for o in outs]
        for o in outs:
            o.release()
        return res
