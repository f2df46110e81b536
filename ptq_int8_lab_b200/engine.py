# -*- coding: utf-8 -*-
"""Host-side mirror of the reference engine interface over the C ABI (include/ptq8.h).

Reference interface (06-gpu-int8/cpp) and its counterpart here:

  ``Model::load(path, err)``          (ptq_model.h:72-91)      -> ``Model.load(path)``
  ``load_ptqc(path, n, out, err)``    (ptq_model.h:425-503)    -> ``load_ptqc(path, n_expected)``
  ``Int8Engine::build(m, wb, ab)``    (int8_engine.cuh:132)    -> ``Int8Engine.build(model, w_bits, a_bits, ...)``
  ``Int8Engine::set_act_mode``        (int8_engine.cuh:353)    -> ``Int8Engine.set_act_mode``
  ``Int8Engine::set_calib(ranges)``   (int8_engine.cuh:362)    -> ``Int8Engine.set_calib``
  ``Int8Engine::alloc_scratch(n)``    (int8_engine.cuh:807)    -> ``Int8Engine.alloc_scratch``
  ``Int8Engine::set_stream``          (int8_engine.cuh:771)    -> ``Int8Engine.set_stream``
  ``Int8Engine::forward(x, n,c,h,w, logits)`` (int8_engine.cuh:429) -> ``Int8Engine.forward``

Where the reference returns ``false`` plus a message, this mirror raises
``Ptq8Error`` carrying the same message; nothing exits the process.  There is
no CPU fallback: if ``libptq8.so`` is missing, importing the engine fails.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path
from typing import List, Optional, Sequence, Tuple

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libptq8.so"
_lib = None

PASS_CENTER_TAP = 1
PASS_DECOMPOSE = 2
PASS_POSITIONAL = 4
PASS_ALL = PASS_CENTER_TAP | PASS_DECOMPOSE | PASS_POSITIONAL
ACT_ABSMAX = 0
ACT_MINMAX = 1
NORM_DIV = 0   # 8-bit input: (px - mean*255) / (std*255)          (ref_e2e.py:272-274)
NORM_MUL = 1   # 8-bit input: ((px/255)*255 - mean*255) * (1/(std*255))  (main.cpp:245-261)

# every symbol include/ptq8.h declares
EXPORTS = (
    "ptq8_abi_version", "ptq8_model_load", "ptq8_model_free", "ptq8_model_info", "ptq8_model_conv",
    "ptq8_model_block", "ptq8_model_weights", "ptq8_model_codes", "ptq8_load_ptqc", "ptq8_act_scale", "ptq8_quantize_weight", "ptq8_quantize_device",
    "ptq8_quantize_device_noalloc",
    "ptq8_engine_create", "ptq8_engine_destroy", "ptq8_engine_last_error", "ptq8_engine_build",
    "ptq8_engine_set_act_mode", "ptq8_engine_set_calib", "ptq8_engine_set_input_shape",
    "ptq8_engine_alloc_scratch", "ptq8_engine_set_stream", "ptq8_engine_set_max_ctas", "ptq8_engine_stream", "ptq8_engine_forward",
    "ptq8_engine_forward_device", "ptq8_engine_forward_async",
    "ptq8_engine_set_input_norm", "ptq8_engine_forward_u8", "ptq8_engine_forward_u8_async",
    "ptq8_engine_forward_device_u8", "ptq8_engine_input_buffer", "ptq8_engine_logits_buffer", "ptq8_engine_run", "ptq8_engine_copy_logits",
    "ptq8_engine_sync", "ptq8_engine_check_device_error", "ptq8_engine_set_wait_test", "ptq8_engine_tensor_info",
    "ptq8_engine_dump", "ptq8_engine_dump_range",
    "ptq8_engine_n_launches", "ptq8_engine_weight_bytes", "ptq8_engine_passes_log", "ptq8_engine_profile",
    "ptq8_load", "ptq8_forward", "ptq8_forward_debug", "ptq8_capture_graph", "ptq8_destroy", "ptq8_last_error",
)


class Opts(ctypes.Structure):
    """ptq8_opts of include/ptq8.h."""
    _fields_ = [("device", ctypes.c_int), ("w_bits", ctypes.c_int), ("a_bits", ctypes.c_int),
                ("act_mode", ctypes.c_int), ("passes", ctypes.c_int), ("max_batch", ctypes.c_int)]


DUMP_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int8), ctypes.c_int,
                           ctypes.c_int, ctypes.c_int, ctypes.c_int)


class Ptq8Error(RuntimeError):
    def __init__(self, msg: str, status: int = 1):
        super().__init__(msg)
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libptq8.so (built by ``python -m ptq_int8_lab_b200.build``); fail loudly if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise Ptq8Error(f"{_LIB_PATH} not found: build it with `python -m ptq_int8_lab_b200.build`")
    L = ctypes.CDLL(str(_LIB_PATH))
    c_int, c_size, c_char_p, c_void_p = ctypes.c_int, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_void_p
    P = ctypes.POINTER
    sig = {
        "ptq8_abi_version": (c_int, []),
        "ptq8_model_load": (c_void_p, [c_char_p, c_char_p, c_size]),
        "ptq8_model_free": (None, [c_void_p]),
        "ptq8_model_info": (c_int, [c_void_p, P(c_int)]),
        "ptq8_model_conv": (c_int, [c_void_p, c_int, P(c_int)]),
        "ptq8_model_block": (c_int, [c_void_p, c_int, P(c_int), c_int, P(c_int), P(c_int), P(c_int), P(c_int)]),
        "ptq8_model_weights": (c_int, [c_void_p, c_int, P(P(ctypes.c_float)), P(c_size), P(P(ctypes.c_float))]),
        "ptq8_model_codes": (c_int, [c_void_p, c_int, P(P(ctypes.c_int8)), P(c_size), P(P(ctypes.c_float)),
                                     P(c_int)]),
        "ptq8_load_ptqc": (c_int, [c_char_p, c_size, P(ctypes.c_float), c_size, c_char_p, c_size]),
        "ptq8_act_scale": (ctypes.c_double, [ctypes.c_float, ctypes.c_float, c_int, c_int]),
        "ptq8_quantize_weight": (c_int, [P(ctypes.c_float), c_int, c_int, c_int, P(ctypes.c_int8), P(ctypes.c_float)]),
        "ptq8_quantize_device": (c_int, [c_int, P(ctypes.c_float), c_size, ctypes.c_float, ctypes.c_float, c_int,
                                         P(ctypes.c_int8)]),
        "ptq8_quantize_device_noalloc": (c_int, [c_int, P(ctypes.c_float), c_size, ctypes.c_float, ctypes.c_float,
                                                 c_int, P(ctypes.c_int8), c_char_p, c_size]),
        "ptq8_engine_create": (c_void_p, [c_int]),
        "ptq8_engine_destroy": (None, [c_void_p]),
        "ptq8_engine_last_error": (c_char_p, [c_void_p]),
        "ptq8_engine_build": (c_int, [c_void_p, c_void_p, c_int, c_int, P(c_int), c_int, c_int]),
        "ptq8_engine_set_act_mode": (c_int, [c_void_p, c_int]),
        "ptq8_engine_set_calib": (c_int, [c_void_p, P(ctypes.c_float), c_size]),
        "ptq8_engine_set_input_shape": (c_int, [c_void_p, c_int, c_int, c_int]),
        "ptq8_engine_alloc_scratch": (c_int, [c_void_p, c_int]),
        "ptq8_engine_set_stream": (c_int, [c_void_p, c_void_p]),
        "ptq8_engine_set_max_ctas": (c_int, [c_void_p, c_int]),
        "ptq8_engine_stream": (c_void_p, [c_void_p]),
        "ptq8_engine_forward": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
        "ptq8_engine_forward_device": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
        "ptq8_engine_forward_async": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
        "ptq8_engine_set_input_norm": (c_int, [c_void_p, c_int, P(ctypes.c_float), P(ctypes.c_float)]),
        "ptq8_engine_forward_u8": (c_int, [c_void_p, c_void_p, c_int, c_size, c_void_p]),
        "ptq8_engine_forward_u8_async": (c_int, [c_void_p, c_void_p, c_int, c_size, c_void_p]),
        "ptq8_engine_forward_device_u8": (c_int, [c_void_p, c_void_p, c_int, c_size, c_void_p]),
        "ptq8_engine_input_buffer": (c_void_p, [c_void_p]),
        "ptq8_engine_logits_buffer": (c_void_p, [c_void_p]),
        "ptq8_engine_run": (c_int, [c_void_p, c_int, c_int]),
        "ptq8_engine_copy_logits": (c_int, [c_void_p, c_int, c_void_p]),
        "ptq8_engine_sync": (c_int, [c_void_p]),
        "ptq8_engine_check_device_error": (c_int, [c_void_p]),
        "ptq8_engine_set_wait_test": (c_int, [c_void_p, ctypes.c_longlong, c_int]),
        "ptq8_engine_tensor_info": (c_int, [c_void_p, c_int, c_int, P(c_int)]),
        "ptq8_engine_dump": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_size]),
        "ptq8_engine_dump_range": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size]),
        "ptq8_engine_n_launches": (c_int, [c_void_p]),
        "ptq8_engine_weight_bytes": (c_int, [c_void_p, P(c_size), P(c_size), P(c_int)]),
        "ptq8_engine_profile": (c_int, [c_void_p, c_int, c_int, P(ctypes.c_float), P(ctypes.c_double),
                                        P(ctypes.c_double), P(c_int), c_int, P(c_int)]),
        "ptq8_engine_passes_log": (c_int, [c_void_p, c_char_p, c_size]),
        "ptq8_load": (c_int, [c_char_p, c_char_p, c_char_p, P(Opts), P(c_void_p), c_char_p, c_size]),
        "ptq8_forward": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
        "ptq8_forward_debug": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, DUMP_FN, c_void_p]),
        "ptq8_capture_graph": (c_int, [c_void_p, c_int]),
        "ptq8_destroy": (None, [c_void_p]),
        "ptq8_last_error": (c_char_p, [c_void_p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


# --------------------------------------------------------------------------- model files

class Model:
    """A loaded PTQW / PTQ2 model (owns the native handle)."""

    def __init__(self, handle: int, path: str):
        self._h = handle
        self.path = path
        info = (ctypes.c_int * 11)()
        lib().ptq8_model_info(handle, info)
        (self.n_conv, self.n_block, self.stem_pool, self.fc_in, self.fc_out, self.n_depthwise,
         self.n_grouped, self.n_relu6, self.n_residual2, fmt, self.n_conv_per_block) = list(info)
        self.format = {1: "PTQW", 2: "PTQ2", 3: "PTQ8"}[fmt]

    @classmethod
    def load(cls, path) -> "Model":
        err = ctypes.create_string_buffer(1024)
        h = lib().ptq8_model_load(str(path).encode(), err, len(err))
        if not h:
            raise Ptq8Error(err.value.decode(errors="replace"), 2)
        return cls(h, str(path))

    def conv(self, i: int) -> dict:
        m = (ctypes.c_int * 10)()
        if lib().ptq8_model_conv(self._h, i, m):
            raise IndexError(i)
        keys = ("cout", "cin", "kh", "kw", "sh", "sw", "ph", "pw", "relu", "groups")
        return dict(zip(keys, list(m)))

    def block(self, i: int) -> dict:
        cap = 16
        cs = (ctypes.c_int * cap)()
        n, ds, st, res = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        if lib().ptq8_model_block(self._h, i, cs, cap, ctypes.byref(n), ctypes.byref(ds), ctypes.byref(st),
                                  ctypes.byref(res)):
            raise IndexError(i)
        return dict(convs=list(cs)[:n.value], ds=ds.value, stride=st.value, residual=res.value)

    def weights(self, i: int) -> Tuple[np.ndarray, np.ndarray]:
        w = ctypes.POINTER(ctypes.c_float)()
        b = ctypes.POINTER(ctypes.c_float)()
        n = ctypes.c_size_t()
        if lib().ptq8_model_weights(self._h, i, ctypes.byref(w), ctypes.byref(n), ctypes.byref(b)):
            raise IndexError(i)
        nb = self.fc_out if i == -1 else self.conv(i)["cout"]
        wa = np.ctypeslib.as_array(w, shape=(n.value,)).copy() if n.value else np.zeros(0, np.float32)  # PTQ8: none
        return wa, np.ctypeslib.as_array(b, shape=(nb,)).copy()

    def codes(self, i: int):
        """(codes [cout, K] int8, f32 scales [cout], bits) stored by a PTQ8 package; None for PTQ2/PTQW."""
        c = ctypes.POINTER(ctypes.c_int8)()
        s = ctypes.POINTER(ctypes.c_float)()
        n, b = ctypes.c_size_t(), ctypes.c_int()
        if lib().ptq8_model_codes(self._h, i, ctypes.byref(c), ctypes.byref(n), ctypes.byref(s), ctypes.byref(b)):
            raise IndexError(i)
        if b.value == 0:
            return None
        cout = self.conv(i)["cout"]
        return (np.ctypeslib.as_array(c, shape=(n.value,)).reshape(cout, -1).copy(),
                np.ctypeslib.as_array(s, shape=(cout,)).copy(), b.value)

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            _lib.ptq8_model_free(h)


def load_ptqc(path, n_expected: int) -> List[Tuple[float, float]]:
    """Strict PTQC read: exact size, n == n_expected, finite, lo <= hi."""
    out = np.zeros(2 * max(n_expected, 1), dtype=np.float32)
    err = ctypes.create_string_buffer(1024)
    rc = lib().ptq8_load_ptqc(str(path).encode(), n_expected, _fptr(out), out.size, err, len(err))
    if rc:
        raise Ptq8Error(err.value.decode(errors="replace"), rc)
    return [(float(out[2 * i]), float(out[2 * i + 1])) for i in range(n_expected)]


def load_layer_plan(path, n_conv: int) -> List[int]:
    """Per-conv weight bits from a layer-plan JSON (mixed_check.py:62-81 schema)."""
    doc = json.loads(Path(path).read_text(encoding="utf-8"))
    layers = doc.get("layers") if isinstance(doc, dict) else None
    if not isinstance(layers, list) or len(layers) != n_conv:
        raise Ptq8Error(f"{path}: 'layers' must list {n_conv} convs in engine order")
    bits = []
    for i, e in enumerate(layers):
        b = int(e.get("bits", 0))
        if b not in (4, 8):
            raise Ptq8Error(f"{path}: layer {i} bits={b} (only 4 / 8)")
        if e.get("scheme", "per_channel") != "per_channel":
            raise Ptq8Error(f"{path}: layer {i} scheme {e.get('scheme')!r}: only per_channel weights run on the engine")
        bits.append(b)
    return bits


def act_scale(lo: float, hi: float, bits: int = 8, mode: int = ACT_ABSMAX) -> float:
    return float(lib().ptq8_act_scale(lo, hi, bits, mode))


def quantize_weight(w: np.ndarray, bits: int = 8) -> Tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, dtype=np.float32)
    cout = w.shape[0]
    k = w.size // cout
    codes = np.empty(w.shape, dtype=np.int8)
    scale = np.empty(cout, dtype=np.float32)
    rc = lib().ptq8_quantize_weight(_fptr(w), cout, k, bits, codes.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)),
                                    _fptr(scale))
    if rc:
        raise Ptq8Error("quantize_weight: invalid arguments", rc)
    return codes, scale


def quantize_device(x: np.ndarray, lo: float, hi: float, mode: int = ACT_ABSMAX, device: int = 0) -> np.ndarray:
    """int8 codes of x computed by the engine's device quantizer (epilogue code path)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size, dtype=np.int8)
    rc = lib().ptq8_quantize_device(device, _fptr(x), x.size, lo, hi, mode,
                                    out.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)))
    if rc:
        raise Ptq8Error("ptq8_quantize_device failed", rc)
    return out


# --------------------------------------------------------------------------- engine

class Int8Engine:
    """sm_100a int8 engine; one per device per host thread."""

    def __init__(self, device: int = 0):
        self._h = lib().ptq8_engine_create(device)
        self.device = device
        self.model: Optional[Model] = None

    def _check(self, rc: int):
        if rc:
            raise Ptq8Error(lib().ptq8_engine_last_error(self._h).decode(errors="replace"), rc)

    def build(self, model: Model, w_bits: int = 8, a_bits: int = 8, layer_bits: Optional[Sequence[int]] = None,
              passes: int = 0) -> "Int8Engine":
        self.model = model          # keep alive: the engine holds a pointer to it
        lb = None
        n = 0
        if layer_bits is not None:
            n = len(layer_bits)
            lb = (ctypes.c_int * n)(*[int(b) for b in layer_bits])
        self._check(lib().ptq8_engine_build(self._h, model._h, w_bits, a_bits, lb, n, passes))
        return self

    def set_act_mode(self, mode: int):
        self._check(lib().ptq8_engine_set_act_mode(self._h, mode))

    def set_calib(self, ranges: Sequence[Tuple[float, float]]):
        a = np.ascontiguousarray(np.asarray(ranges, dtype=np.float32).reshape(-1))
        self._check(lib().ptq8_engine_set_calib(self._h, _fptr(a), len(ranges)))

    def set_input_shape(self, c: int, h: int, w: int):
        self._check(lib().ptq8_engine_set_input_shape(self._h, c, h, w))

    def alloc_scratch(self, max_batch: int):
        self._check(lib().ptq8_engine_alloc_scratch(self._h, max_batch))
        self.max_batch = max_batch

    def set_stream(self, stream_ptr: int):
        self._check(lib().ptq8_engine_set_stream(self._h, ctypes.c_void_p(stream_ptr)))

    def set_max_ctas(self, max_ctas: int):
        """Cap the persistent grid of every tensor-core conv (0: one CTA per SM)."""
        self._check(lib().ptq8_engine_set_max_ctas(self._h, max_ctas))

    @property
    def stream(self) -> int:
        return lib().ptq8_engine_stream(self._h) or 0

    def forward(self, x: np.ndarray) -> np.ndarray:
        """Host fp32 NCHW in, host fp32 logits out (H2D + graph + D2H, synchronous)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, c, h, w = x.shape
        out = np.empty((n, self.model.fc_out), dtype=np.float32)
        self._check(lib().ptq8_engine_forward(self._h, x.ctypes.data, n, c, h, w, out.ctypes.data))
        return out

    def forward_host_ptr(self, x_ptr: int, n: int, c: int, h: int, w: int, out_ptr: int):
        """Same as forward() on raw host pointers (pinned buffers from the caller)."""
        self._check(lib().ptq8_engine_forward(self._h, ctypes.c_void_p(x_ptr), n, c, h, w, ctypes.c_void_p(out_ptr)))

    def forward_async(self, x_ptr: int, n: int, out_ptr: int):
        """Pipelined host-buffer forward on raw (pinned) host pointers: enqueue and return;
        sync() waits.  The next call's input copy overlaps this call's forward."""
        self._check(lib().ptq8_engine_forward_async(self._h, ctypes.c_void_p(x_ptr), n, ctypes.c_void_p(out_ptr)))

    def forward_device(self, x_ptr: int, n: int, logits_ptr: int):
        self._check(lib().ptq8_engine_forward_device(self._h, ctypes.c_void_p(x_ptr), n, ctypes.c_void_p(logits_ptr)))

    def set_input_norm(self, mode: int = NORM_DIV, mean=None, std=None):
        """Normalisation of 8-bit input (NORM_DIV / NORM_MUL; mean/std per channel, or
        None for the CIFAR-10 constants)."""
        if (mean is None) != (std is None):
            raise Ptq8Error("mean and std: both given or both None")
        if mean is None:
            self._check(lib().ptq8_engine_set_input_norm(self._h, mode, None, None))
            return
        m = np.ascontiguousarray(mean, dtype=np.float32)
        sd = np.ascontiguousarray(std, dtype=np.float32)
        self._check(lib().ptq8_engine_set_input_norm(self._h, mode, _fptr(m), _fptr(sd)))

    def forward_u8(self, x: np.ndarray, n: int = 0, record_bytes: int = 0, img_bytes: int = 3072) -> np.ndarray:
        """8-bit pixels in, host fp32 logits out; synchronous.  x: uint8 [n][c][h][w]
        (record_bytes 0), or a byte array whose first byte is image 0's first pixel, with
        image i at i * record_bytes (e.g. a raw CIFAR-10 batch file from its second byte)."""
        x = np.ascontiguousarray(x, dtype=np.uint8)
        if record_bytes == 0:
            n = x.shape[0]
        elif n <= 0 or x.size < (n - 1) * record_bytes + img_bytes:
            raise Ptq8Error(f"{n} records of {record_bytes} bytes do not fit in {x.size} bytes")
        out = np.empty((n, self.model.fc_out), dtype=np.float32)
        self._check(lib().ptq8_engine_forward_u8(self._h, x.ctypes.data, n, record_bytes, out.ctypes.data))
        return out

    def forward_u8_async(self, x_ptr: int, n: int, record_bytes: int, out_ptr: int):
        """Pipelined 8-bit forward on raw (pinned) host pointers; sync() waits."""
        self._check(lib().ptq8_engine_forward_u8_async(self._h, ctypes.c_void_p(x_ptr), n, record_bytes,
                                                       ctypes.c_void_p(out_ptr)))

    def forward_device_u8(self, x_ptr: int, n: int, record_bytes: int, logits_ptr: int):
        self._check(lib().ptq8_engine_forward_device_u8(self._h, ctypes.c_void_p(x_ptr), n, record_bytes,
                                                        ctypes.c_void_p(logits_ptr)))

    def input_buffer(self) -> int:
        return lib().ptq8_engine_input_buffer(self._h) or 0

    def logits_buffer(self) -> int:
        return lib().ptq8_engine_logits_buffer(self._h) or 0

    def run(self, n: int, use_graph: bool = True):
        self._check(lib().ptq8_engine_run(self._h, n, 1 if use_graph else 0))

    def copy_logits(self, n: int, dst_ptr: int):
        self._check(lib().ptq8_engine_copy_logits(self._h, n, ctypes.c_void_p(dst_ptr)))

    def sync(self):
        self._check(lib().ptq8_engine_sync(self._h))

    def n_launches(self) -> int:
        return lib().ptq8_engine_n_launches(self._h)

    def weight_bytes(self) -> dict:
        """Conv weight bytes in device memory, the same weights as int8 bytes, packed W4 convs."""
        dev, i8, npk = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int()
        self._check(lib().ptq8_engine_weight_bytes(self._h, ctypes.byref(dev), ctypes.byref(i8), ctypes.byref(npk)))
        return {"device_bytes": dev.value, "int8_bytes": i8.value, "packed_w4_convs": npk.value}

    def profile(self, n: int, iters: int = 5) -> List[dict]:
        """Per-step device time (ms) and algorithmic work (see ptq8_engine_profile)."""
        cap = 512
        ms = (ctypes.c_float * cap)()
        macs = (ctypes.c_double * cap)()
        byts = (ctypes.c_double * cap)()
        kind = (ctypes.c_int * cap)()
        ns = ctypes.c_int()
        self._check(lib().ptq8_engine_profile(self._h, n, iters, ms, macs, byts, kind, cap, ctypes.byref(ns)))
        return [dict(step=i, ms=float(ms[i]), macs=float(macs[i]), bytes=float(byts[i]), kind=int(kind[i]))
                for i in range(ns.value)]

    def passes_log(self) -> str:
        buf = ctypes.create_string_buffer(1 << 16)
        lib().ptq8_engine_passes_log(self._h, buf, len(buf))
        return buf.value.decode()

    def tensor_info(self, what: int, index: int = 0) -> Tuple[int, int, int, int]:
        s = (ctypes.c_int * 4)()
        self._check(lib().ptq8_engine_tensor_info(self._h, what, index, s))
        return tuple(s)

    def dump_codes(self, conv: int, n: int, n0: int = 0) -> np.ndarray:
        """int8 input codes of conv `conv` for images [n0, n0+n) of the last forward: NHWC
        (stem: im2col rows)."""
        _, h, w, ld = self.tensor_info(0, conv)
        out = np.empty((n, h, w, ld), dtype=np.int8)
        self._check(lib().ptq8_engine_dump_range(self._h, 0, conv, n0, n, out.ctypes.data, out.nbytes))
        return out

    def dump_final(self, n: int, n0: int = 0) -> np.ndarray:
        """fp32 map fed to the pooling head for images [n0, n0+n) of the last forward, NHWC."""
        _, h, w, c = self.tensor_info(1)
        out = np.empty((n, h, w, c), dtype=np.float32)
        self._check(lib().ptq8_engine_dump_range(self._h, 1, 0, n0, n, out.ctypes.data, out.nbytes))
        return out

    def check_device_error(self):
        """Raise Ptq8Error (status PTQ8_ERR_TIMEOUT) if a bounded device wait ran out."""
        self._check(lib().ptq8_engine_check_device_error(self._h))

    def set_wait_test(self, wait_limit_cycles: int = 0, stall_first_load: bool = False):
        """Failure-detection test hook (see ptq8_engine_set_wait_test)."""
        self._check(lib().ptq8_engine_set_wait_test(self._h, int(wait_limit_cycles), 1 if stall_first_load else 0))

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            if getattr(self, "_one_call", False):
                _lib.ptq8_destroy(h)
            else:
                _lib.ptq8_engine_destroy(h)


def load_one_call(model_path, calib_path, plan_path=None, max_batch: int = 0, device: int = 0, w_bits: int = 8,
                  act_mode: int = ACT_ABSMAX, passes: int = 0) -> Int8Engine:
    """The one-call interface: ptq8_load (model + PTQC + layer plan + build + calib +
    scratch in one call; the engine owns its model), wrapped as an Int8Engine."""
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(1024)
    opts = Opts(device, w_bits, 8, act_mode, passes, max_batch)
    rc = lib().ptq8_load(str(model_path).encode(), str(calib_path).encode(),
                         str(plan_path).encode() if plan_path else None, ctypes.byref(opts), ctypes.byref(h), err,
                         len(err))
    if rc:
        raise Ptq8Error(err.value.decode(errors="replace"), rc)
    e = Int8Engine.__new__(Int8Engine)
    e._h = h.value
    e._one_call = True
    e.device = device
    e.model = Model.load(model_path)   # shape metadata (fc_out) for forward()
    e.max_batch = max_batch
    return e


def open_engine(model_path, calib_path, plan_path=None, max_batch: int = 256, device: int = 0,
                w_bits: int = 8, passes: int = 0) -> Int8Engine:
    """Convenience: Model.load + load_ptqc + build + set_calib + alloc_scratch."""
    m = Model.load(model_path)
    ranges = load_ptqc(calib_path, m.n_conv)
    bits = load_layer_plan(plan_path, m.n_conv) if plan_path else None
    e = Int8Engine(device)
    e.build(m, w_bits=w_bits, a_bits=8, layer_bits=bits, passes=passes)
    e.set_calib(ranges)
    e.alloc_scratch(max_batch)
    return e
