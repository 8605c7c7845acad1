"""Sequence groups over NVLink (l3p_attn_seq_group_* / l3p_attn_decode_seq_dev)
on two GPUs, one process each.

Each member owns half of the positions; one decode_seq launch pair per layer
computes its partial triple, publishes it, waits for the other member's and
merges both, reading the peer's over NVLink.  The merged output on every
member must equal the oracle's decode over the whole range within
|gpu - ref| <= 1e-4 + 1e-4*|ref| -- including a position whose range lies
entirely in the first member (the second contributes an empty partial) and a
Gemma sliding window that straddles the split.  Needs two GPUs; skipped
otherwise.
"""
import os
import tempfile

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.synth import CONFIGS, GEMMA_SWA, decode_inputs, tolerance_ok

pytestmark = pytest.mark.gpu

CASES = {
    "l8b_end": (CONFIGS["llama31_8b_decode_8k"].with_(seq_len=4096, pos=4095, n_layers=2), 1),
    "l8b_first_half_only": (CONFIGS["llama31_8b_decode_8k"].with_(seq_len=4096, pos=1000, n_layers=2), 0),
    "gemma_window_straddles": (GEMMA_SWA.with_(seq_len=4096, pos=2200, n_layers=1), 0),
}


def _n_gpus():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _worker(rank, world, port, case, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from llama3pure_b200.attn import AttnContext

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    sh, layer = CASES[case]
    k, v, q = decode_inputs(sh, layer, ctx=sh.seq_len)
    b, e = sh.seq_len * rank // world, sh.seq_len * (rank + 1) // world
    results = []
    with AttnContext.for_shape(sh, device=rank, seq_begin=b, seq_count=e - b) as ctx:
        ctx.load_kv(layer, b, np.ascontiguousarray(k[:, b:e]), np.ascontiguousarray(v[:, b:e]))
        h = ctx.seq_group_export(world, rank)
        hs = [None] * world
        dist.all_gather_object(hs, h)
        ctx.seq_group_import(hs)
        dq = torch.from_numpy(q.reshape(-1).copy()).cuda()
        for overlap in (False, True):
            ctx.set_overlap(overlap)
            outs = []
            for _ in range(3):  # repeated steps: epochs advance, slots are reused
                dout = torch.zeros_like(dq)
                ctx.decode_seq_dev(layer, sh.pos, dq, dout)
                outs.append(dout)
            ctx.check()
            results += [o.cpu().numpy() for o in outs]
        dist.barrier()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack(results))
    dist.destroy_process_group()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("case", list(CASES))
def test_seq_group_over_nvlink_matches_the_whole_range(case):
    import torch.multiprocessing as mp

    sh, layer = CASES[case]
    k, v, q = decode_inputs(sh, layer, ctx=sh.seq_len)
    o = O.Oracle(sh, O.MODE_F32, "port", n_layers=layer + 1)
    o.load_kv(layer, 0, k, v)
    want, _ = o.decode(layer, sh.pos, q)
    o.close()
    port = 29600 + list(CASES).index(case)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, port, case, d), nprocs=2, join=True)
        for rank in range(2):
            got = np.load(os.path.join(d, f"rank{rank}.npy"))
            for i, g in enumerate(got):
                ok, ma, mr = tolerance_ok(g.reshape(want.shape), want)
                assert ok, f"{case} rank {rank} step {i}: max_abs={ma:.3e} max_rel={mr:.3e}"
