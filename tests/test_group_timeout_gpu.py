"""Failure detection of the NVLink groups without a GPU fault.

A member that never arrives: two processes share one GPU; the second exports
and maps its exchange region but never calls the group's decode or wo.  The
first member's merge kernel must give up after its bounded wait (about a
second), record the timeout in the context's error word -- l3p_attn_check
returns L3P_E_TIMEOUT -- and leave the context usable: a plain decode right
after matches the oracle.  Only one kernel waits (nothing runs on the other
side), so no two waiting kernels share the GPU.
"""
import os
import tempfile

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.synth import CONFIGS, decode_inputs, tolerance_ok

pytestmark = pytest.mark.gpu


def _has_gpu():
    try:
        import torch

        return torch.cuda.device_count() >= 1
    except Exception:
        return False


def _worker(rank, port, kind, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from llama3pure_b200.attn import AttnContext, AttnError
    from llama3pure_b200.synth import wo_input, wo_weights

    torch.cuda.set_device(0)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=120))
    sh = CONFIGS["llama32_1b_decode"].with_(n_layers=1)
    k, v, q = decode_inputs(sh, 0)
    result = {}
    b, e = (0, sh.seq_len // 2) if rank == 0 else (sh.seq_len // 2, sh.seq_len)
    seq_kw = dict(seq_begin=b, seq_count=e - b) if kind == "seq" else {}
    with AttnContext.for_shape(sh, **seq_kw) as ctx:
        cols = sh.n_heads * sh.head_dim
        if kind == "seq":
            h = ctx.seq_group_export(2, rank)
        else:
            ctx.set_wo(0, 8, wo_weights(8, 256, cols, seed=1))
            h = ctx.tp_group_export(2, rank, 256)
        hs = [None, None]
        dist.all_gather_object(hs, h)
        if kind == "seq":
            ctx.seq_group_import(hs)
        else:
            ctx.tp_group_import(hs)
        if rank == 0:
            dq = torch.from_numpy(q.reshape(-1).copy()).cuda()
            if kind == "seq":
                ctx.load_kv(0, b, np.ascontiguousarray(k[:, b:e]), np.ascontiguousarray(v[:, b:e]))
                dout = torch.zeros_like(dq)
                ctx.decode_seq_dev(0, sh.pos, dq, dout)
            else:
                dy = torch.zeros(256, device="cuda")
                ctx.wo_allreduce_dev(0, torch.from_numpy(wo_input(cols, 2)).cuda(), dy)
            try:
                ctx.check()
                result["code"] = 0
            except AttnError as err:
                result["code"] = err.code
            if kind == "tp":
                # the same context keeps working: its plain projection
                result["after"] = ctx.wo(0, wo_input(cols, 3))
        dist.barrier()  # the other member leaves only after the waiter has given up
    if rank == 0 and kind == "seq":
        # the context is gone with its group; a fresh one on the same GPU works
        with AttnContext.for_shape(sh) as ctx2:
            ctx2.load_kv(0, 0, k, v)
            result["after"] = ctx2.decode(0, sh.pos, q)
    if rank == 0:
        np.save(os.path.join(out_dir, "result.npy"), result, allow_pickle=True)
    dist.destroy_process_group()


@pytest.mark.skipif(not _has_gpu(), reason="needs a GPU")
@pytest.mark.parametrize("kind", ["seq", "tp"])
def test_a_member_that_never_arrives_times_out(kind):
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(29800 + (kind == "tp"), kind, d), nprocs=2, join=True)
        res = np.load(os.path.join(d, "result.npy"), allow_pickle=True).item()
    assert res["code"] == -5  # L3P_E_TIMEOUT
    if kind == "tp":
        from llama3pure_b200.synth import wo_input, wo_weights

        cols = CONFIGS["llama32_1b_decode"].n_heads * CONFIGS["llama32_1b_decode"].head_dim
        want = O.matvec(8, wo_weights(8, 256, cols, seed=1), 256, cols, wo_input(cols, 3))
        ok, ma, mr = tolerance_ok(res["after"], want)
        assert ok, f"wo after the timeout: max_abs={ma:.3e} max_rel={mr:.3e}"
    if kind == "seq":
        sh = CONFIGS["llama32_1b_decode"].with_(n_layers=1)
        k, v, q = decode_inputs(sh, 0)
        o = O.Oracle(sh, O.MODE_F32, "port", n_layers=1)
        o.load_kv(0, 0, k, v)
        want, _ = o.decode(0, sh.pos, q)
        o.close()
        ok, ma, mr = tolerance_ok(res["after"], want)
        assert ok, f"decode after the timeout: max_abs={ma:.3e} max_rel={mr:.3e}"
