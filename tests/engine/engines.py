"""ctypes driver of the engine builds of tests/engine/Makefile (TEST
INFRASTRUCTURE ONLY): the reference C engine as it is (exact IEEE build and
its own -Ofast release build), and the same engine wired to
libllama3pure_attn.so.  Each build holds one model at a time."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libl3p_engine_ref.so")
WIRED_SO = os.path.join(ROOT, "oracle", "_ref", "libl3p_engine_wired.so")
OFAST_SO = os.path.join(ROOT, "oracle", "_ref", "libl3p_engine_ofast.so")


class EngineCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
                                      "vocab_size", "seq_len", "is_gemma3", "swa_window")] + [
        ("rope_theta", C.c_float), ("rope_theta_swa", C.c_float), ("rms_norm_eps", C.c_float),
        ("seed", C.c_ulonglong)]


# synthetic models: (dim, hidden, layers, heads, kv heads, head_dim, vocab, seq_len, gemma, swa_window, theta, theta_swa, eps)
MODELS = {
    "llama_hd64": (512, 1408, 3, 8, 2, 64, 512, 160, 0, 0, 500000.0, 10000.0, 1e-5),
    "llama_hd128": (1024, 2048, 2, 8, 2, 128, 512, 160, 0, 0, 500000.0, 10000.0, 1e-5),
    "gemma_hd256": (512, 1024, 7, 4, 1, 256, 512, 160, 1, 24, 1000000.0, 10000.0, 1e-6),
}


def available(wired: bool, ofast: bool = False) -> bool:
    return os.path.exists(WIRED_SO if wired else OFAST_SO if ofast else REF_SO)


class Engine:
    def __init__(self, wired: bool, ofast: bool = False):
        self.lib = C.CDLL(WIRED_SO if wired else OFAST_SO if ofast else REF_SO)
        self.lib.l3pe_init.argtypes = [C.POINTER(EngineCfg)]
        self.lib.l3pe_init.restype = C.c_int
        self.lib.l3pe_run.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        self.lib.l3pe_run.restype = C.c_int

    def run(self, model: str, prompt: list[int], n_gen: int, seed: int = 1):
        m = MODELS[model]
        cfg = EngineCfg(*m[:10], *m[10:], seed)
        rc = self.lib.l3pe_init(C.byref(cfg))
        if rc:
            raise RuntimeError(f"l3pe_init rc={rc}")
        p = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(n_gen, np.int32)
        logits = np.zeros((n_gen, m[6]), np.float32)
        rc = self.lib.l3pe_run(p.ctypes.data, len(prompt), n_gen, toks.ctypes.data, logits.ctypes.data)
        if rc:
            raise RuntimeError(f"l3pe_run rc={rc}")
        return toks, logits


def prompt_for(model: str, n: int, seed: int = 5) -> list[int]:
    g = np.random.default_rng(seed)
    return [int(t) for t in g.integers(0, MODELS[model][6], n)]
