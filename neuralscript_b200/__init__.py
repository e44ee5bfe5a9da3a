"""NeuralScript B200 backend: Python host-side bindings.

The product is the native library ``lib/libns_b200.so`` (engine + sm_100a
kernels, C-ABI in ``include/ns_b200.h`` and ``include/ns_b200_ops.h``) and one
``lib/libns_<model>.so`` per model exporting the unchanged NeuralScript
``ns_runtime.h`` ABI. This module only loads them with ctypes and mirrors the
reference's host API (src/codegen/codegen.cpp:916-1126): the same call names,
argument meaning and 0 / -1 return codes, raising ``RuntimeError`` where the
ABI returns -1. There is no Python or CPU fallback: if the library is
missing, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import List, Optional, Tuple

import numpy as np

from . import spec as spec_mod
from .spec import CONFIGS, parse

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "lib")
CORE_LIB = os.path.join(LIB_DIR, "libns_b200.so")

PRECISION = {"fp32": 0, "tf32": 1, "bf16": 2}


def build(jobs: int = 8) -> None:
    """Compile the kernels (sm_100a) and the per-model libraries in place."""
    subprocess.run(["make", "-s", "-C", os.path.join(HERE, "csrc"), f"-j{jobs}"], check=True)


class _WeightDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("offset", C.c_size_t), ("count", C.c_size_t)]


class _Layout(C.Structure):
    _fields_ = [("num_weights", C.c_size_t), ("desc", C.POINTER(_WeightDesc))]


_f32p = C.POINTER(C.c_float)
_lib = None


def lib() -> C.CDLL:
    """The core library (loaded once); raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(CORE_LIB):
        raise RuntimeError(f"{CORE_LIB} missing: run neuralscript_b200.build() (the B200 path has no fallback)")
    L = C.CDLL(CORE_LIB)
    sig = {
        "nsb_runtime_init": (C.c_void_p, [C.c_char_p, C.c_void_p, C.c_size_t]),
        "nsb_eval_infer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
        "nsb_model_output_numel": (C.c_size_t, [C.c_void_p, C.c_size_t]),
        "nsb_model_weight_count": (C.c_size_t, [C.c_void_p]),
        "nsb_spec_weight_count": (C.c_size_t, [C.c_char_p]),
        "nsb_model_get_weights": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
        "nsb_spec_layout": (C.POINTER(_Layout), [C.c_char_p]),
        "nsb_free": (None, [C.c_void_p]),
        "nsb_save_checkpoint": (C.c_int, [C.c_void_p, C.c_char_p]),
        "nsb_load_checkpoint": (C.c_int, [C.c_void_p, C.c_char_p]),
        "nsb_expert_count": (C.c_size_t, [C.c_void_p]),
        "nsb_expert_birth": (C.c_size_t, [C.c_void_p, C.c_int]),
        "nsb_expert_merge": (C.c_size_t, [C.c_void_p, C.c_int, C.c_int]),
        "nsb_expert_kill": (C.c_size_t, [C.c_void_p, C.c_int]),
        "nsb_runtime_train_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, _f32p, C.c_float]),
        "nsb_runtime_train_step_idx": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, _f32p, C.c_float]),
        "nsb_objective_loss": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, _f32p]),
        "nsb_set_precision": (C.c_int, [C.c_void_p, C.c_int]),
        "nsb_get_precision": (C.c_int, [C.c_void_p]),
        "nsb_eval_infer_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
        "nsb_train_step_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, _f32p,
                                            C.c_float, C.c_void_p]),
        "nsb_last_launch_count": (C.c_longlong, [C.c_void_p]),
        "nsb_model_get_gradients": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
        "nsb_model_get_input_gradient": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
        "nsb_region_timing": (C.c_int, [C.c_void_p, C.c_int]),
        "nsb_region_count": (C.c_int, [C.c_void_p]),
        "nsb_region_get": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_double),
                                     C.POINTER(C.c_longlong)]),
        "nsb_dist_unique_id": (C.c_int, [C.c_void_p]),
        "nsb_dist_init": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int]),
        "nsb_last_error": (C.c_char_p, []),
        "nsb_version": (C.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return lib().nsb_last_error().decode()


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {last_error()}")


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def spec_layout_shapes(spec_text: str):
    """[(name, offset, count, (rows, cols))] of a spec's weight blob."""
    return parse(spec_text).layout()


def spec_layout(spec_text: str) -> List[Tuple[str, int, int]]:
    lay = lib().nsb_spec_layout(spec_text.encode())
    if not lay:
        raise RuntimeError(f"bad spec: {last_error()}")
    L = lay.contents
    return [(L.desc[i].name.decode(), L.desc[i].offset, L.desc[i].count) for i in range(L.num_weights)]


class Model:
    """A NeuralScript model on the current CUDA device (one per process and
    GPU for data parallelism). Mirrors ns_runtime.h: weights are one fp32
    blob in layout order; inputs/outputs are host arrays."""

    def __init__(self, spec_text: str, weights: np.ndarray, precision: Optional[str] = None):
        self.spec_text = spec_text
        self.spec = parse(spec_text)
        w = np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
        self._last_rows = 0
        self._h = lib().nsb_runtime_init(spec_text.encode(), _ptr(w), w.size)
        if not self._h:
            raise RuntimeError(f"ns_runtime_init failed: {last_error()}")
        if precision is not None:
            self.set_precision(precision)

    @property
    def handle(self) -> C.c_void_p:
        return C.c_void_p(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().nsb_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_precision(self, mode: str) -> None:
        _check(lib().nsb_set_precision(self._h, PRECISION[mode]), "set_precision")

    @property
    def precision(self) -> str:
        return {v: k for k, v in PRECISION.items()}[lib().nsb_get_precision(self._h)]

    def output_numel(self, input_numel: int) -> int:
        return lib().nsb_model_output_numel(self._h, input_numel)

    def weight_count(self) -> int:
        return lib().nsb_model_weight_count(self._h)

    def infer(self, x: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
        """ns_eval_infer with host buffers; `out` (float32, contiguous) may be
        a caller-owned buffer, e.g. page-locked memory."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        n = self.output_numel(x.size)
        if out is None:
            out = np.empty(n, np.float32)
        if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < n:
            raise ValueError("infer: out must be a contiguous float32 array of at least %d elements" % n)
        _check(lib().nsb_eval_infer(self._h, _ptr(x), _ptr(out), x.size), "ns_eval_infer")
        return out.reshape(-1)[:n].reshape(-1, self.spec_out_cols)

    @property
    def spec_out_cols(self) -> int:
        return spec_mod.out_cols(self.spec)

    def train_step(self, x: np.ndarray, labels: np.ndarray, lr: float) -> float:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        y = np.ascontiguousarray(labels, dtype=np.float32).reshape(-1)
        loss = C.c_float(0)
        _check(lib().nsb_runtime_train_step(self._h, _ptr(x), _ptr(y), x.size, C.byref(loss), lr),
               "ns_runtime_train_step")
        self._last_rows = x.size // self.spec.in_cols
        return loss.value

    def train_step_idx(self, x: np.ndarray, targets: np.ndarray, lr: float) -> float:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        t = np.ascontiguousarray(targets, dtype=np.int32).reshape(-1)
        loss = C.c_float(0)
        _check(lib().nsb_runtime_train_step_idx(self._h, _ptr(x), _ptr(t), x.size, C.byref(loss), lr),
               "train_step_idx")
        self._last_rows = x.size // self.spec.in_cols
        return loss.value

    def objective(self, x: np.ndarray, labels: np.ndarray) -> float:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        y = np.ascontiguousarray(labels, dtype=np.float32).reshape(-1)
        loss = C.c_float(0)
        _check(lib().nsb_objective_loss(self._h, _ptr(x), _ptr(y), x.size, C.byref(loss)), "ns_objective_loss")
        return loss.value

    def get_weights(self) -> np.ndarray:
        out = np.empty(self.weight_count(), np.float32)
        _check(lib().nsb_model_get_weights(self._h, _ptr(out), out.size), "ns_model_get_weights")
        return out

    def get_gradients(self) -> np.ndarray:
        """Gradients of the last train step, in weight-blob layout."""
        out = np.empty(self.weight_count(), np.float32)
        _check(lib().nsb_model_get_gradients(self._h, _ptr(out), out.size), "get_gradients")
        return out

    def get_input_gradient(self) -> np.ndarray:
        """dLoss/dx of the last train step, [rows, input width] (specs with a
        `grad input` statement)."""
        rows = self._last_rows
        out = np.empty(rows * self.spec.in_cols, np.float32)
        _check(lib().nsb_model_get_input_gradient(self._h, _ptr(out), out.size), "get_input_gradient")
        return out.reshape(rows, self.spec.in_cols)

    def layout(self):
        return spec_layout(self.spec_text)

    def save(self, path: str) -> None:
        _check(lib().nsb_save_checkpoint(self._h, path.encode()), "ns_save_checkpoint")

    def load(self, path: str) -> None:
        _check(lib().nsb_load_checkpoint(self._h, path.encode()), "ns_load_checkpoint")

    def expert_count(self) -> int:
        return lib().nsb_expert_count(self._h)

    def expert_birth(self, n: int) -> int:
        return lib().nsb_expert_birth(self._h, n)

    def expert_merge(self, a: int, b: int) -> int:
        return lib().nsb_expert_merge(self._h, a, b)

    def expert_kill(self, k: int) -> int:
        return lib().nsb_expert_kill(self._h, k)

    # device-resident fast paths (torch tensors on this model's device)
    def infer_device(self, x, out, stream: int = 0) -> None:
        _check(lib().nsb_eval_infer_device(self._h, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), x.numel(),
                                           C.c_void_p(stream)), "eval_infer_device")

    def train_step_device(self, x, labels=None, targets=None, lr: float = 0.0, stream: int = 0,
                          want_loss: bool = True) -> float:
        loss = C.c_float(0)
        lp = C.c_void_p(labels.data_ptr()) if labels is not None else None
        tp = C.c_void_p(targets.data_ptr()) if targets is not None else None
        _check(lib().nsb_train_step_device(self._h, C.c_void_p(x.data_ptr()), lp, tp, x.numel(),
                                           C.byref(loss) if want_loss else None, lr, C.c_void_p(stream)),
               "train_step_device")
        self._last_rows = x.numel() // self.spec.in_cols
        return loss.value

    def region_timing(self, enable: bool = True) -> None:
        _check(lib().nsb_region_timing(self._h, 1 if enable else 0), "region_timing")

    def regions(self):
        """{label: (total_ms, count)} of the regions timed since enabling."""
        out = {}
        for i in range(lib().nsb_region_count(self._h)):
            lab, ms, n = C.c_char_p(), C.c_double(), C.c_longlong()
            lib().nsb_region_get(self._h, i, C.byref(lab), C.byref(ms), C.byref(n))
            out[lab.value.decode()] = (ms.value, n.value)
        return out

    def last_launch_count(self) -> int:
        return lib().nsb_last_launch_count(self._h)

    def dist_init(self, rank: int, world: int, uid: bytes, timeout_ms: int = 60000) -> None:
        buf = C.create_string_buffer(uid, 128)
        _check(lib().nsb_dist_init(self._h, rank, world, buf, timeout_ms), "dist_init")


def dist_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(lib().nsb_dist_unique_id(buf), "dist_unique_id")
    return buf.raw


class RuntimeLib:
    """The drop-in ABI: a per-model library exporting ns_runtime.h, called by
    the reference's own entry-point names."""

    def __init__(self, name: str):
        lib()  # the engine must be resident first
        path = os.path.join(LIB_DIR, f"libns_{name}.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} missing: run neuralscript_b200.build()")
        L = C.CDLL(path)
        sig = {
            "ns_runtime_init": (C.c_void_p, [C.c_void_p, C.c_size_t]),
            "ns_eval_infer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
            "ns_model_output_numel": (C.c_size_t, [C.c_void_p, C.c_size_t]),
            "ns_model_weight_count": (C.c_size_t, [C.c_void_p]),
            "ns_weight_count_static": (C.c_size_t, []),
            "ns_model_get_weights": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
            "ns_model_layout": (C.POINTER(_Layout), [C.c_void_p]),
            "ns_free": (None, [C.c_void_p]),
            "ns_save_checkpoint": (C.c_int, [C.c_void_p, C.c_char_p]),
            "ns_load_checkpoint": (C.c_int, [C.c_void_p, C.c_char_p]),
            "ns_expert_count": (C.c_size_t, [C.c_void_p]),
            "ns_expert_birth": (C.c_size_t, [C.c_void_p, C.c_int]),
            "ns_expert_merge": (C.c_size_t, [C.c_void_p, C.c_int, C.c_int]),
            "ns_expert_kill": (C.c_size_t, [C.c_void_p, C.c_int]),
            "ns_runtime_train_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, _f32p, C.c_float]),
            "ns_objective_loss": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, _f32p]),
        }
        for n, (res, args) in sig.items():
            f = getattr(L, n)
            f.restype = res
            f.argtypes = args
        self.L = L
        self.name = name

    def __getattr__(self, item):
        return getattr(self.L, item)

