"""The C-ABI library without a GPU: it builds for sm_100a, loads, exports
every symbol include/*.h declares, and rejects bad configurations before
touching the device."""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

from llama3pure_b200 import attn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(l3p_\w+)\s*\(", text))
    return names


def test_header_declares_the_bound_symbols():
    assert _declared_symbols() == set(attn.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", attn.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (l3p_\w+)", out))
    assert _declared_symbols() <= exported
    # nothing else of ours leaks out of the shared object
    assert {s for s in exported if s.startswith("l3p")} == _declared_symbols()


def test_library_is_compiled_for_sm100a_only():
    from llama3pure_b200.build import ARCH_FLAGS

    assert ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


@pytest.mark.gpu
def test_runtime_reports_sm100_kernels(lib):
    """The CUDA runtime's own view of the loaded image: SASS for sm_100,
    compiled from the compute_100 virtual architecture."""
    binary, ptx = C.c_int(0), C.c_int(-1)
    assert lib.l3p_attn_device_arch(0, C.byref(binary), C.byref(ptx)) == 0
    assert binary.value == 100
    assert ptx.value == 100


def _cfg(**kw):
    base = dict(n_layers=2, n_heads=8, n_kv_heads=2, head_dim=128, seq_len=64, scale=0.0, is_gemma3=0,
                swa_window=0, swa_pattern=0, device=0, kv_head_begin=0, kv_head_count=0, seq_begin=0,
                seq_count=0, kv_format=0)
    base.update(kw)
    return attn.AttnConfig(**base)


@pytest.mark.parametrize(
    "kw,code",
    [
        (dict(n_heads=6, n_kv_heads=4), -1),      # heads not a multiple of KV heads
        (dict(head_dim=96), -6),                  # no kernel for this head_dim
        (dict(kv_head_begin=1, kv_head_count=2), -1),  # shard past the last KV head
        (dict(seq_begin=60, seq_count=8), -1),    # shard past the capacity
        (dict(n_layers=0), -1),
        (dict(kv_format=2), -1),                  # no such cache format
    ],
)
def test_create_rejects_bad_config_without_device(lib, kw, code):
    h = C.c_void_p()
    assert lib.l3p_attn_create(C.byref(_cfg(**kw)), C.byref(h)) == code
    assert not h.value


def test_null_arguments_are_errors(lib):
    assert lib.l3p_attn_create(None, None) == -1
    assert lib.l3p_attn_decode(None, 0, 0, None, None) == -1
    assert lib.l3p_attn_check(None) == -1
    assert lib.l3p_attn_launch_count(None) == -1
    lib.l3p_attn_destroy(None)
