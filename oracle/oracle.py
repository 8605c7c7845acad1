"""ctypes access to the CPU parity oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker or the timed CPU reference.  The shipped
library (llama3pure_b200) never imports it.

Two backends with one interface:
  impl="port" -> oracle/liboracle.so        (restatement, l3p_oracle.c)
  impl="ref"  -> oracle/_ref/libl3p_ref.so  (the reference's own functions,
                 compiled in place from llama3pure-c-engine.c)
`fast=True` selects the -Ofast OpenMP builds used for timing.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MODE_F32 = 0
MODE_Q8 = 1

_LIBS: dict = {}


class OracleRope(C.Structure):
    _fields_ = [
        ("rope_theta", C.c_float),
        ("rope_theta_swa", C.c_float),
        ("rms_norm_eps", C.c_float),
        ("q_norm", C.POINTER(C.c_float)),
        ("k_norm", C.POINTER(C.c_float)),
    ]


class OracleCfg(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int),
        ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int),
        ("head_dim", C.c_int),
        ("seq_len", C.c_int),
        ("scale", C.c_float),
        ("is_gemma3", C.c_int),
        ("swa_window", C.c_int),
        ("swa_pattern", C.c_int),
    ]


def lib_path(impl: str, fast=False) -> str:
    """fast: False (exact IEEE build), True (-Ofast -march=x86-64-v3) or "v4"
    (-Ofast -march=x86-64-v4, reference harness only)."""
    if impl == "port":
        return os.path.join(HERE, "liboracle_fast.so" if fast else "liboracle.so")
    if impl == "ref":
        name = {False: "libl3p_ref.so", True: "libl3p_ref_fast.so", "v4": "libl3p_ref_fast_v4.so"}[fast]
        return os.path.join(HERE, "_ref", name)
    raise ValueError(impl)


def cpu_has_v4() -> bool:
    """The host CPU runs x86-64-v4 code (AVX-512 F, BW, CD, DQ, VL)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    return {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= flags
    except OSError:
        pass
    return False


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def ref_available(fast=False) -> bool:
    return os.path.exists(lib_path("ref", fast))


def build_port() -> None:
    """Compile the restatement (gcc is present wherever this repo runs)."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)


def _load(impl: str, fast):
    key = (impl, fast)
    if key in _LIBS:
        return _LIBS[key]
    path = lib_path(impl, fast)
    if not os.path.exists(path):
        if impl != "port":
            raise FileNotFoundError(f"{path} not built (needs the reference source; run `make -C oracle ref`)")
        build_port()
    lib = C.CDLL(path)
    pre = "l3po_" if impl == "port" else "l3pref_"
    fp = C.POINTER(C.c_float)
    sig = {
        "create": (C.c_void_p, [C.POINTER(OracleCfg), C.c_int]),
        "destroy": (None, [C.c_void_p]),
        "load_kv": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, fp, fp]),
        "decode": (C.c_int, [C.c_void_p, C.c_int, C.c_int, fp, fp, fp, fp, C.POINTER(C.c_longlong)]),
        "prefill": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, fp, fp, fp, fp, C.POINTER(C.c_longlong)]),
        "fp16_to_fp32": (C.c_float, [C.c_uint16]),
        "fp32_to_fp16": (C.c_uint16, [C.c_float]),
        "q8_quantize": (None, [fp, C.c_void_p, C.c_int]),
        "q8_dot": (C.c_float, [C.c_void_p, C.c_void_p, C.c_int]),
        "q8_accum": (None, [fp, C.c_void_p, C.c_float, C.c_int]),
        "softmax": (None, [fp, C.c_int]),
        "rope": (C.c_int, [C.POINTER(OracleCfg), C.POINTER(OracleRope), C.c_int, C.c_int, C.c_int, fp, fp]),
        "matvec": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int, fp, fp]),
    }
    fns = {}
    for name, (res, args) in sig.items():
        f = getattr(lib, pre + name)
        f.restype = res
        f.argtypes = args
        fns[name] = f
    if impl == "ref":
        lib.l3pref_threads.restype = C.c_int
        fns["threads"] = lib.l3pref_threads
    _LIBS[key] = (lib, fns)
    return _LIBS[key]


def _fptr(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_float))


class Oracle:
    """One attention context of the oracle: its own KV cache for n_layers."""

    def __init__(self, shape, mode: int = MODE_F32, impl: str = "port", fast=False,
                 n_layers: int | None = None, seq_len: int | None = None):
        self.shape = shape
        self.mode = mode
        self.impl = impl
        _, self.f = _load(impl, fast)
        cfg = OracleCfg(
            n_layers if n_layers is not None else shape.n_layers,
            shape.n_heads,
            shape.n_kv_heads,
            shape.head_dim,
            seq_len if seq_len is not None else shape.seq_len,
            0.0,
            shape.is_gemma3,
            shape.swa_window,
            shape.swa_pattern,
        )
        self.cfg = cfg
        self.ctx = self.f["create"](C.byref(cfg), mode)
        if not self.ctx:
            raise RuntimeError("oracle create failed")

    def close(self):
        if self.ctx:
            self.f["destroy"](self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_kv(self, layer: int, pos0: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        rc = self.f["load_kv"](self.ctx, layer, pos0, k.shape[1], _fptr(k), _fptr(v))
        if rc:
            raise RuntimeError(f"oracle load_kv rc={rc}")

    def decode(self, layer: int, pos: int, q: np.ndarray, k_row=None, v_row=None):
        q = np.ascontiguousarray(q, np.float32)
        out = np.empty(self.shape.n_heads * self.shape.head_dim, np.float32)
        sk = C.c_longlong(0)
        kr = None if k_row is None else np.ascontiguousarray(k_row, np.float32)
        vr = None if v_row is None else np.ascontiguousarray(v_row, np.float32)
        rc = self.f["decode"](self.ctx, layer, pos, _fptr(q), _fptr(kr), _fptr(vr), _fptr(out), C.byref(sk))
        if rc:
            raise RuntimeError(f"oracle decode rc={rc}")
        return out.reshape(self.shape.n_heads, self.shape.head_dim), int(sk.value)

    def prefill(self, layer: int, start_pos: int, q: np.ndarray, k: np.ndarray, v: np.ndarray):
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        n = q.shape[0]
        out = np.empty((n, self.shape.n_heads, self.shape.head_dim), np.float32)
        sk = C.c_longlong(0)
        rc = self.f["prefill"](self.ctx, layer, start_pos, n, _fptr(q), _fptr(k), _fptr(v), _fptr(out), C.byref(sk))
        if rc:
            raise RuntimeError(f"oracle prefill rc={rc}")
        return out, int(sk.value)


def primitives(impl: str = "port"):
    """The codec/softmax primitives of one backend, for exhaustive pinning."""
    return _load(impl, False)[1]


def threads(impl: str = "ref", fast=True) -> int:
    fns = _load(impl, fast)[1]
    return int(fns["threads"]()) if "threads" in fns else 1


def rope(shape, layer: int, pos0: int, q: np.ndarray, k: np.ndarray, rope_theta: float = 0.0,
         rope_theta_swa: float = 0.0, rms_norm_eps: float = 0.0, q_norm=None, k_norm=None,
         impl: str = "port", n_layers: int | None = None):
    """The pre-attention step (QK-norm, RoPE; q unscaled) of tokens at pos0..

    q: [n_tok][n_heads*head_dim], k: [n_tok][n_kv_heads*head_dim]; returns
    rotated copies.  q_norm / k_norm: [n_layers][head_dim] or None."""
    _, f = _load(impl, False)
    q = np.array(q, np.float32, order="C", copy=True)
    k = np.array(k, np.float32, order="C", copy=True)
    nl = n_layers if n_layers is not None else max(layer + 1, getattr(shape, "n_layers", 1))
    cfg = OracleCfg(nl, shape.n_heads, shape.n_kv_heads, shape.head_dim, max(pos0 + q.shape[0], 1), 0.0,
                    shape.is_gemma3, shape.swa_window, shape.swa_pattern)
    qn = None if q_norm is None else np.ascontiguousarray(q_norm, np.float32)
    kn = None if k_norm is None else np.ascontiguousarray(k_norm, np.float32)
    rc_ = OracleRope(rope_theta, rope_theta_swa, rms_norm_eps, _fptr(qn), _fptr(kn))
    rc = f["rope"](C.byref(cfg), C.byref(rc_), layer, pos0, q.shape[0], _fptr(q), _fptr(k))
    if rc:
        raise RuntimeError(f"oracle rope rc={rc}")
    return q, k


W_F32, W_F16, W_Q4_0, W_Q4_1, W_Q5_0, W_Q5_1 = 0, 1, 2, 3, 6, 7
W_Q8_0, W_Q2_K, W_Q3_K, W_Q4_K, W_Q5_K, W_Q6_K = 8, 10, 11, 12, 13, 14
W_IQ4_NL, W_BF16 = 20, 29
W_BLOCK = {W_F32: (1, 4), W_F16: (1, 2), W_BF16: (1, 2), W_Q4_0: (32, 18), W_Q4_1: (32, 20), W_Q5_0: (32, 22),
           W_Q5_1: (32, 24), W_IQ4_NL: (32, 18), W_Q8_0: (32, 34), W_Q2_K: (256, 84), W_Q3_K: (256, 110),
           W_Q4_K: (256, 144), W_Q5_K: (256, 176), W_Q6_K: (256, 210)}  # values, bytes per block


def w_row_bytes(wtype: int, cols: int) -> int:
    n, b = W_BLOCK[wtype]
    return cols // n * b


def matvec(wtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, impl: str = "port") -> np.ndarray:
    """out[rows] = W x for GGUF weight rows (uint8 [rows][row bytes]), the
    reference's dequantise-then-dot path (matmul_quantized, c:2091)."""
    _, f = _load(impl, False)
    w = np.ascontiguousarray(w, np.uint8)
    assert w.size == rows * w_row_bytes(wtype, cols)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(rows, np.float32)
    rc = f["matvec"](wtype, w.ctypes.data, rows, cols, _fptr(x), _fptr(out))
    if rc:
        raise RuntimeError(f"oracle matvec rc={rc}")
    return out
