"""Tensor-parallel wo over NVLink (l3p_attn_tp_group_* /
l3p_attn_wo_allreduce_dev) on two GPUs, one process each.

Each member owns half of the KV heads, hence half of wo's columns; one call
per layer writes its partial projection into both members' memory and adds
the partials in member order.  Both members must hold the same bits, equal to
the reference's matmul_quantized over all columns (the oracle's matvec)
within |gpu - ref| <= 1e-4 + 1e-4*|ref|, for every weight type and over
several steps (the two exchange slots alternate).  Needs two GPUs.
"""
import os
import tempfile

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.synth import CONFIGS, tolerance_ok, wo_input, wo_weights

pytestmark = pytest.mark.gpu

SH = CONFIGS["llama31_8b_decode_8k"].with_(seq_len=32, n_layers=2)
DIM = 4096
STEPS = 5


def _n_gpus():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _worker(rank, world, port, wtype, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from llama3pure_b200.attn import AttnContext

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    cols = SH.n_heads * SH.head_dim
    per = SH.n_kv_heads // world
    w = wo_weights(wtype, DIM, cols, seed=3)
    res = []
    with AttnContext.for_shape(SH, device=rank, kv_head_begin=rank * per, kv_head_count=per) as ctx:
        ctx.set_wo(1, wtype, w)
        h = ctx.tp_group_export(world, rank, DIM)
        hs = [None] * world
        dist.all_gather_object(hs, h)
        ctx.tp_group_import(hs)
        for overlap in (False, True):
            ctx.set_overlap(overlap)
            outs = []
            for step in range(STEPS):
                x = torch.from_numpy(wo_input(cols, seed=100 + step)).cuda()
                y = torch.zeros(DIM, device="cuda")
                ctx.wo_allreduce_dev(1, x, y)
                outs.append(y)
            ctx.check()
            res += [o.cpu().numpy() for o in outs]
        dist.barrier()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack(res))
    dist.destroy_process_group()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("wtype", [O.W_Q8_0, O.W_Q2_K, O.W_Q3_K, O.W_Q4_K, O.W_Q5_K, O.W_Q6_K, O.W_Q4_0, O.W_Q4_1,
                                   O.W_Q5_0, O.W_Q5_1, O.W_IQ4_NL, O.W_F32, O.W_F16, O.W_BF16])
def test_wo_allreduce_over_nvlink(wtype):
    import torch.multiprocessing as mp

    cols = SH.n_heads * SH.head_dim
    w = wo_weights(wtype, DIM, cols, seed=3)
    wants = [O.matvec(wtype, w, DIM, cols, wo_input(cols, seed=100 + s)) for s in range(STEPS)] * 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, 29700 + wtype, wtype, d), nprocs=2, join=True)
        r0 = np.load(os.path.join(d, "rank0.npy"))
        r1 = np.load(os.path.join(d, "rank1.npy"))
    np.testing.assert_array_equal(r0.view(np.uint32), r1.view(np.uint32))  # same bits on both members
    for i, (g, want) in enumerate(zip(r0, wants)):
        ok, ma, mr = tolerance_ok(g, want)
        assert ok, f"type {wtype} call {i}: max_abs={ma:.3e} max_rel={mr:.3e}"
