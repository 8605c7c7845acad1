"""Python host binding of libllama3pure_attn.so (the C ABI in
include/llama3pure_attn.h), used by the tests and the benchmark.

It mirrors the reference's seam one to one: `AttnContext.step` is the engine's
attention block (KV append + decode, llama3pure-c-engine.c:3299-3359),
`prefill` its prompt loop (c:3499-3613).  Host methods take numpy arrays;
`*_dev` methods take torch CUDA tensors (or raw device addresses) and enqueue
on a stream.  There is no CPU fallback: if the shared library is missing the
import raises.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

from .build import LIB_PATH

L3P_OK = 0
ERRORS = {
    -1: "L3P_E_INVAL",
    -2: "L3P_E_RANGE",
    -3: "L3P_E_CUDA",
    -4: "L3P_E_NOMEM",
    -5: "L3P_E_TIMEOUT",
    -6: "L3P_E_UNSUPPORTED",
}

# Every symbol include/llama3pure_attn.h declares.
EXPORTS = (
    "l3p_attn_create",
    "l3p_attn_destroy",
    "l3p_attn_last_error",
    "l3p_attn_check",
    "l3p_attn_set_stream",
    "l3p_attn_kv_append",
    "l3p_attn_kv_append_dev",
    "l3p_attn_decode",
    "l3p_attn_decode_dev",
    "l3p_attn_step",
    "l3p_attn_step_dev",
    "l3p_attn_decode_layers_dev",
    "l3p_attn_decode_partial_dev",
    "l3p_attn_lse_merge_dev",
    "l3p_attn_prefill",
    "l3p_attn_prefill_dev",
    "l3p_attn_load_kv",
    "l3p_attn_read_kv",
    "l3p_attn_load_kv_q8",
    "l3p_attn_read_kv_q8",
    "l3p_attn_kv_device_ptr",
    "l3p_attn_launch_count",
    "l3p_attn_device_arch",
    "l3p_attn_set_overlap",
    "l3p_attn_set_host_server",
    "l3p_attn_decode_plan",
    "l3p_attn_set_rope",
    "l3p_attn_rope_dev",
    "l3p_attn_step_raw",
    "l3p_attn_step_raw_dev",
    "l3p_attn_prefill_raw",
    "l3p_attn_prefill_raw_dev",
    "l3p_attn_set_wo",
    "l3p_attn_wo",
    "l3p_attn_wo_dev",
    "l3p_attn_step_raw_wo",
    "l3p_attn_seq_group_export",
    "l3p_attn_seq_group_import",
    "l3p_attn_decode_seq_dev",
    "l3p_attn_tp_group_export",
    "l3p_attn_tp_group_import",
    "l3p_attn_wo_allreduce_dev",
    "l3p_attn_decode_noalloc",
    "l3p_attn_noalloc_last_error",
)


class AttnConfig(C.Structure):
    """Mirror of l3p_attn_config."""

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
        ("device", C.c_int),
        ("kv_head_begin", C.c_int),
        ("kv_head_count", C.c_int),
        ("seq_begin", C.c_int),
        ("seq_count", C.c_int),
        ("kv_format", C.c_int),
    ]


class RopeConfig(C.Structure):
    """Mirror of l3p_attn_rope_config."""

    _fields_ = [
        ("rope_theta", C.c_float),
        ("rope_theta_swa", C.c_float),
        ("rms_norm_eps", C.c_float),
        ("q_norm", C.c_void_p),
        ("k_norm", C.c_void_p),
    ]


class AttnError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


_LIB = None


def load_library(path: str = LIB_PATH):
    """Load libllama3pure_attn.so and declare its signatures.  Raises if the
    library has not been built (there is no fallback implementation)."""
    global _LIB
    if _LIB is not None and path == LIB_PATH:
        return _LIB
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(the CUDA path is the only implementation)"
        )
    lib = C.CDLL(path)
    vp, fp, i = C.c_void_p, C.c_void_p, C.c_int
    sig = {
        "l3p_attn_create": (i, [C.POINTER(AttnConfig), C.POINTER(C.c_void_p)]),
        "l3p_attn_destroy": (None, [vp]),
        "l3p_attn_last_error": (C.c_char_p, [vp]),
        "l3p_attn_check": (i, [vp]),
        "l3p_attn_set_stream": (i, [vp, vp]),
        "l3p_attn_kv_append": (i, [vp, i, i, fp, fp]),
        "l3p_attn_kv_append_dev": (i, [vp, i, i, fp, fp, vp]),
        "l3p_attn_decode": (i, [vp, i, i, fp, fp]),
        "l3p_attn_decode_dev": (i, [vp, i, i, fp, fp, vp]),
        "l3p_attn_step": (i, [vp, i, i, fp, fp, fp, fp]),
        "l3p_attn_step_dev": (i, [vp, i, i, fp, fp, fp, fp, vp]),
        "l3p_attn_decode_layers_dev": (i, [vp, i, i, i, fp, fp, vp]),
        "l3p_attn_decode_partial_dev": (i, [vp, i, i, fp, fp, fp, vp]),
        "l3p_attn_lse_merge_dev": (i, [vp, i, i, i, i, fp, fp, fp, vp]),
        "l3p_attn_prefill": (i, [vp, i, i, i, fp, fp, fp, fp]),
        "l3p_attn_prefill_dev": (i, [vp, i, i, i, fp, fp, fp, fp, vp]),
        "l3p_attn_load_kv": (i, [vp, i, i, i, fp, fp]),
        "l3p_attn_read_kv": (i, [vp, i, i, i, fp, fp]),
        "l3p_attn_load_kv_q8": (i, [vp, i, i, i, fp, fp]),
        "l3p_attn_read_kv_q8": (i, [vp, i, i, i, fp, fp]),
        "l3p_attn_kv_device_ptr": (i, [vp, i, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
        "l3p_attn_launch_count": (C.c_longlong, [vp]),
        "l3p_attn_device_arch": (i, [i, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "l3p_attn_set_overlap": (i, [vp, i]),
        "l3p_attn_set_host_server": (i, [vp, i, C.c_longlong]),
        "l3p_attn_decode_plan": (i, [vp, i, i, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "l3p_attn_set_rope": (i, [vp, C.POINTER(RopeConfig)]),
        "l3p_attn_rope_dev": (i, [vp, i, i, i, fp, fp, fp, fp, vp]),
        "l3p_attn_step_raw": (i, [vp, i, i, fp, fp, fp, fp]),
        "l3p_attn_step_raw_dev": (i, [vp, i, i, fp, fp, fp, fp, vp]),
        "l3p_attn_prefill_raw": (i, [vp, i, i, i, fp, fp, fp, fp]),
        "l3p_attn_prefill_raw_dev": (i, [vp, i, i, i, fp, fp, fp, fp, vp]),
        "l3p_attn_set_wo": (i, [vp, i, i, vp, i]),
        "l3p_attn_wo": (i, [vp, i, fp, fp]),
        "l3p_attn_wo_dev": (i, [vp, i, fp, fp, vp]),
        "l3p_attn_step_raw_wo": (i, [vp, i, i, fp, fp, fp, fp]),
        "l3p_attn_seq_group_export": (i, [vp, i, i, vp]),
        "l3p_attn_seq_group_import": (i, [vp, vp]),
        "l3p_attn_decode_seq_dev": (i, [vp, i, i, fp, fp, vp]),
        "l3p_attn_tp_group_export": (i, [vp, i, i, i, vp]),
        "l3p_attn_tp_group_import": (i, [vp, vp]),
        "l3p_attn_wo_allreduce_dev": (i, [vp, i, fp, fp, vp]),
        "l3p_attn_decode_noalloc": (i, [C.POINTER(AttnConfig), i, i, fp, fp, fp, fp, vp]),
        "l3p_attn_noalloc_last_error": (C.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if path == LIB_PATH:
        _LIB = lib
    return lib


def _host(a: np.ndarray | None):
    if a is None:
        return None
    if a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError("host arrays must be C-contiguous float32")
    return a.ctypes.data


def _dev(t) -> int | None:
    """Device address of a torch CUDA tensor (or pass-through int)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not t.is_cuda or t.dtype.itemsize != 4 or not t.is_contiguous():
        raise TypeError("device tensors must be contiguous 32-bit CUDA tensors")
    return t.data_ptr()


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the default stream torch reports as 0


def _stream(s) -> int | None:
    """cudaStream_t for the C ABI.  None selects the context's own stream;
    torch's default stream (handle 0) is passed as cudaStreamLegacy so that it
    is not mistaken for None."""
    if s is None:
        return None
    h = s if isinstance(s, int) else s.cuda_stream  # torch.cuda.Stream
    return h if h != 0 else CUDA_STREAM_LEGACY


def _dev_stream(s) -> int | None:
    """Stream of a *_dev call: the given one, else torch's current stream when
    torch drives CUDA in this process (the device tensors were produced there,
    so the call is ordered after them), else the context's own stream."""
    if s is not None:
        return _stream(s)
    torch = sys.modules.get("torch")
    if torch is not None and torch.cuda.is_initialized():
        return _stream(torch.cuda.current_stream())
    return None


class AttnContext:
    """One l3p_attn_ctx: the device KV cache of `n_layers` for the KV heads
    and positions this process owns."""

    def __init__(self, n_layers: int, n_heads: int, n_kv_heads: int, head_dim: int, seq_len: int,
                 scale: float = 0.0, is_gemma3: int = 0, swa_window: int = 0, swa_pattern: int = 0,
                 device: int = 0, kv_head_begin: int = 0, kv_head_count: int = 0, seq_begin: int = 0,
                 seq_count: int = 0, kv_format: int = 0, lib=None):
        self.lib = lib or load_library()
        self.cfg = AttnConfig(n_layers, n_heads, n_kv_heads, head_dim, seq_len, scale, is_gemma3,
                              swa_window, swa_pattern, device, kv_head_begin, kv_head_count, seq_begin,
                              seq_count, kv_format)
        self.kv_format = kv_format
        self.n_heads, self.n_kv_heads, self.head_dim = n_heads, n_kv_heads, head_dim
        self.kv_head_begin = kv_head_begin
        self.kv_head_count = kv_head_count or (n_kv_heads - kv_head_begin)
        self.kv_mul = n_heads // n_kv_heads
        self.wo_dim = 0  # rows of the wo weights once set_wo has run
        h = C.c_void_p()
        rc = self.lib.l3p_attn_create(C.byref(self.cfg), C.byref(h))
        if rc != L3P_OK:
            raise AttnError(rc, "l3p_attn_create failed")
        self.h = h

    @classmethod
    def for_shape(cls, shape, **kw) -> "AttnContext":
        kw.setdefault("n_layers", shape.n_layers)
        kw.setdefault("seq_len", shape.seq_len)
        return cls(n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads, head_dim=shape.head_dim,
                   is_gemma3=shape.is_gemma3, swa_window=shape.swa_window, swa_pattern=shape.swa_pattern, **kw)

    # -- lifecycle -----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.l3p_attn_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _ok(self, rc: int, what: str) -> None:
        if rc != L3P_OK:
            msg = self.lib.l3p_attn_last_error(self.h)
            raise AttnError(rc, f"{what}: {msg.decode() if msg else ''}")

    @property
    def owned_rows(self) -> tuple[int, int]:
        """q-head rows this context writes: [row_lo, row_hi)."""
        return self.kv_head_begin * self.kv_mul, (self.kv_head_begin + self.kv_head_count) * self.kv_mul

    def check(self) -> None:
        self._ok(self.lib.l3p_attn_check(self.h), "check")

    def set_stream(self, stream) -> None:
        self._ok(self.lib.l3p_attn_set_stream(self.h, _stream(stream)), "set_stream")

    def set_overlap(self, enable: bool) -> None:
        """Programmatic dependent launch for decode (see l3p_attn_set_overlap)."""
        self._ok(self.lib.l3p_attn_set_overlap(self.h, int(bool(enable))), "set_overlap")

    def set_host_server(self, enable: bool, idle_us: int = 0) -> None:
        """Serve step()/decode() through a resident grid (see
        l3p_attn_set_host_server)."""
        self._ok(self.lib.l3p_attn_set_host_server(self.h, int(bool(enable)), int(idle_us)), "set_host_server")

    def launch_count(self) -> int:
        return int(self.lib.l3p_attn_launch_count(self.h))

    def decode_plan(self, pos: int, n_slices: int = 1) -> tuple[int, int]:
        """(CTAs per KV-head group, CTAs per cluster) of a decode launch at pos."""
        ns, cs = C.c_int(), C.c_int()
        self._ok(self.lib.l3p_attn_decode_plan(self.h, pos, n_slices, C.byref(ns), C.byref(cs)), "decode_plan")
        return ns.value, cs.value

    def set_rope(self, rope_theta: float = 0.0, rope_theta_swa: float = 0.0, rms_norm_eps: float = 0.0,
                 q_norm: np.ndarray | None = None, k_norm: np.ndarray | None = None) -> None:
        """RoPE tables and QK-norm weights ([n_layers][head_dim] float32) for
        the pre-attention entry points (l3p_attn_set_rope)."""
        qn = None if q_norm is None else np.ascontiguousarray(q_norm, np.float32)
        kn = None if k_norm is None else np.ascontiguousarray(k_norm, np.float32)
        rc = RopeConfig(rope_theta, rope_theta_swa, rms_norm_eps, _host(qn), _host(kn))
        self._ok(self.lib.l3p_attn_set_rope(self.h, C.byref(rc)), "set_rope")

    def set_wo(self, layer: int, wtype: int, rows: np.ndarray) -> None:
        """attn_output.weight of `layer`: uint8 GGUF rows [dim][row bytes]."""
        if rows.dtype != np.uint8 or not rows.flags.c_contiguous:
            raise TypeError("weight rows must be C-contiguous uint8")
        self._ok(self.lib.l3p_attn_set_wo(self.h, layer, wtype, rows.ctypes.data, rows.shape[0]), "set_wo")
        self.wo_dim = rows.shape[0]

    # -- host-pointer entry points ---------------------------------------------
    def load_kv(self, layer: int, pos0: int, k: np.ndarray, v: np.ndarray) -> None:
        self._ok(self.lib.l3p_attn_load_kv(self.h, layer, pos0, k.shape[1], _host(k), _host(v)), "load_kv")

    def read_kv(self, layer: int, pos0: int, n_pos: int):
        k = np.zeros((self.n_kv_heads, n_pos, self.head_dim), np.float32)
        v = np.zeros_like(k)
        self._ok(self.lib.l3p_attn_read_kv(self.h, layer, pos0, n_pos, _host(k), _host(v)), "read_kv")
        return k, v

    def load_kv_q8(self, layer: int, pos0: int, k_blocks: np.ndarray, v_blocks: np.ndarray) -> None:
        """Q8_0 cache from the reference's 34-byte blocks, uint8
        [n_kv_heads][n_pos][head_dim/32*34]."""
        for a in (k_blocks, v_blocks):
            if a.dtype != np.uint8 or not a.flags.c_contiguous:
                raise TypeError("block arrays must be C-contiguous uint8")
        self._ok(self.lib.l3p_attn_load_kv_q8(self.h, layer, pos0, k_blocks.shape[1], k_blocks.ctypes.data,
                                              v_blocks.ctypes.data), "load_kv_q8")

    def read_kv_q8(self, layer: int, pos0: int, n_pos: int):
        """The Q8_0 cache as the reference's 34-byte blocks."""
        k = np.zeros((self.n_kv_heads, n_pos, self.head_dim // 32 * 34), np.uint8)
        v = np.zeros_like(k)
        self._ok(self.lib.l3p_attn_read_kv_q8(self.h, layer, pos0, n_pos, k.ctypes.data, v.ctypes.data), "read_kv_q8")
        return k, v

    def kv_append(self, layer: int, pos: int, k_row: np.ndarray, v_row: np.ndarray) -> None:
        self._ok(self.lib.l3p_attn_kv_append(self.h, layer, pos, _host(k_row), _host(v_row)), "kv_append")

    def decode(self, layer: int, pos: int, q: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        if out is None:
            out = np.zeros((self.n_heads, self.head_dim), np.float32)
        self._ok(self.lib.l3p_attn_decode(self.h, layer, pos, _host(q), _host(out)), "decode")
        return out

    def step(self, layer: int, pos: int, q: np.ndarray, k_row: np.ndarray, v_row: np.ndarray,
             out: np.ndarray | None = None) -> np.ndarray:
        if out is None:
            out = np.zeros((self.n_heads, self.head_dim), np.float32)
        self._ok(self.lib.l3p_attn_step(self.h, layer, pos, _host(q), _host(k_row), _host(v_row), _host(out)), "step")
        return out

    def prefill(self, layer: int, start_pos: int, q: np.ndarray, k: np.ndarray, v: np.ndarray,
                out: np.ndarray | None = None) -> np.ndarray:
        n = q.shape[0]
        if out is None:
            out = np.zeros((n, self.n_heads, self.head_dim), np.float32)
        self._ok(self.lib.l3p_attn_prefill(self.h, layer, start_pos, n, _host(q), _host(k), _host(v), _host(out)),
                 "prefill")
        return out

    def step_raw(self, layer: int, pos: int, q: np.ndarray, k_row: np.ndarray, v_row: np.ndarray,
                 out: np.ndarray | None = None) -> np.ndarray:
        """step() with q, k before QK-norm and RoPE."""
        if out is None:
            out = np.zeros((self.n_heads, self.head_dim), np.float32)
        self._ok(self.lib.l3p_attn_step_raw(self.h, layer, pos, _host(q), _host(k_row), _host(v_row), _host(out)),
                 "step_raw")
        return out

    def prefill_raw(self, layer: int, start_pos: int, q: np.ndarray, k: np.ndarray, v: np.ndarray,
                    out: np.ndarray | None = None) -> np.ndarray:
        """prefill() with q, k before QK-norm and RoPE."""
        n = q.shape[0]
        if out is None:
            out = np.zeros((n, self.n_heads, self.head_dim), np.float32)
        self._ok(self.lib.l3p_attn_prefill_raw(self.h, layer, start_pos, n, _host(q), _host(k), _host(v),
                                               _host(out)), "prefill_raw")
        return out

    def wo(self, layer: int, x: np.ndarray) -> np.ndarray:
        out = np.zeros(max(self.wo_dim, 1), np.float32)
        self._ok(self.lib.l3p_attn_wo(self.h, layer, _host(x), _host(out)), "wo")
        return out

    def step_raw_wo(self, layer: int, pos: int, q: np.ndarray, k_row: np.ndarray, v_row: np.ndarray) -> np.ndarray:
        out = np.zeros(max(self.wo_dim, 1), np.float32)
        self._ok(self.lib.l3p_attn_step_raw_wo(self.h, layer, pos, _host(q), _host(k_row), _host(v_row), _host(out)),
                 "step_raw_wo")
        return out

    # -- device-pointer entry points -------------------------------------------
    def kv_device_ptr(self, layer: int) -> tuple[int, int]:
        k, v = C.c_void_p(), C.c_void_p()
        self._ok(self.lib.l3p_attn_kv_device_ptr(self.h, layer, C.byref(k), C.byref(v)), "kv_device_ptr")
        return k.value, v.value

    def kv_append_dev(self, layer, pos, k, v, stream=None) -> None:
        self._ok(self.lib.l3p_attn_kv_append_dev(self.h, layer, pos, _dev(k), _dev(v), _dev_stream(stream)),
                 "kv_append_dev")

    def decode_dev(self, layer, pos, q, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_decode_dev(self.h, layer, pos, _dev(q), _dev(out), _dev_stream(stream)), "decode_dev")

    def step_dev(self, layer, pos, q, k_row, v_row, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_step_dev(self.h, layer, pos, _dev(q), _dev(k_row), _dev(v_row), _dev(out),
                                            _dev_stream(stream)), "step_dev")

    def decode_layers_dev(self, layer0, n_layers, pos, q, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_decode_layers_dev(self.h, layer0, n_layers, pos, _dev(q), _dev(out),
                                                     _dev_stream(stream)), "decode_layers_dev")

    def decode_partial_dev(self, layer, pos, q, part_o, part_ml, stream=None) -> None:
        self._ok(self.lib.l3p_attn_decode_partial_dev(self.h, layer, pos, _dev(q), _dev(part_o), _dev(part_ml),
                                                      _dev_stream(stream)), "decode_partial_dev")

    def lse_merge_dev(self, n_parts, rows_per_part, row_begin, n_rows, parts_o, parts_ml, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_lse_merge_dev(self.h, n_parts, rows_per_part, row_begin, n_rows, _dev(parts_o),
                                                 _dev(parts_ml), _dev(out), _dev_stream(stream)), "lse_merge_dev")

    def prefill_dev(self, layer, start_pos, n_tok, q, k, v, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_prefill_dev(self.h, layer, start_pos, n_tok, _dev(q), _dev(k), _dev(v), _dev(out),
                                               _dev_stream(stream)), "prefill_dev")

    def seq_group_export(self, n_parts: int, part: int) -> bytes:
        """This member's 64-byte exchange-region handle (share it with the group)."""
        h = (C.c_ubyte * 64)()
        self._ok(self.lib.l3p_attn_seq_group_export(self.h, n_parts, part, C.byref(h)), "seq_group_export")
        return bytes(h)

    def seq_group_import(self, handles) -> None:
        """Map the members' regions: `handles` in member order."""
        buf = b"".join(handles)
        self._ok(self.lib.l3p_attn_seq_group_import(self.h, C.c_char_p(buf)), "seq_group_import")

    def decode_seq_dev(self, layer, pos, q, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_decode_seq_dev(self.h, layer, pos, _dev(q), _dev(out), _dev_stream(stream)),
                 "decode_seq_dev")

    def tp_group_export(self, n_members: int, member: int, dim: int) -> bytes:
        h = (C.c_ubyte * 64)()
        self._ok(self.lib.l3p_attn_tp_group_export(self.h, n_members, member, dim, C.byref(h)), "tp_group_export")
        return bytes(h)

    def tp_group_import(self, handles) -> None:
        self._ok(self.lib.l3p_attn_tp_group_import(self.h, C.c_char_p(b"".join(handles))), "tp_group_import")

    def wo_allreduce_dev(self, layer, x, xout, stream=None) -> None:
        self._ok(self.lib.l3p_attn_wo_allreduce_dev(self.h, layer, _dev(x), _dev(xout), _dev_stream(stream)),
                 "wo_allreduce_dev")

    def wo_dev(self, layer, x, xout, stream=None) -> None:
        self._ok(self.lib.l3p_attn_wo_dev(self.h, layer, _dev(x), _dev(xout), _dev_stream(stream)), "wo_dev")

    def rope_dev(self, layer, pos0, n_tok, q, k, q_out, k_out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_rope_dev(self.h, layer, pos0, n_tok, _dev(q), _dev(k), _dev(q_out), _dev(k_out),
                                            _dev_stream(stream)), "rope_dev")

    def step_raw_dev(self, layer, pos, q, k_row, v_row, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_step_raw_dev(self.h, layer, pos, _dev(q), _dev(k_row), _dev(v_row), _dev(out),
                                                _dev_stream(stream)), "step_raw_dev")

    def prefill_raw_dev(self, layer, start_pos, n_tok, q, k, v, out, stream=None) -> None:
        self._ok(self.lib.l3p_attn_prefill_raw_dev(self.h, layer, start_pos, n_tok, _dev(q), _dev(k), _dev(v),
                                                   _dev(out), _dev_stream(stream)), "prefill_raw_dev")


def decode_noalloc(cfg: AttnConfig, layer: int, pos: int, k_cache, v_cache, q, out, stream=None, lib=None) -> None:
    """l3p_attn_decode_noalloc: decode over a caller-owned layer cache without
    any device allocation (the split partials use the library's fixed scratch
    array; overlapping calls race)."""
    lib = lib or load_library()
    rc = lib.l3p_attn_decode_noalloc(C.byref(cfg), layer, pos, _dev(k_cache), _dev(v_cache), _dev(q), _dev(out),
                                     _dev_stream(stream))
    if rc != L3P_OK:
        msg = lib.l3p_attn_noalloc_last_error()
        raise AttnError(rc, f"decode_noalloc: {msg.decode() if msg else ''}")
