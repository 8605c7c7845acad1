"""Sharded attention on one GPU: contexts owning a KV-head slice or a
sequence slice, combined exactly as the multi-GPU path combines them (rows
concatenated; partial triples LSE-merged on the device)."""
import numpy as np
import pytest

import oracle as O
from llama3pure_b200.attn import AttnContext
from llama3pure_b200.shard import plan_shards
from llama3pure_b200.synth import CONFIGS, AttnShape, decode_inputs, tolerance_ok

pytestmark = pytest.mark.gpu


def _oracle(sh, k, v, q):
    o = O.Oracle(sh, O.MODE_F32, "port", n_layers=1, seq_len=k.shape[1])
    o.load_kv(0, 0, k, v)
    out, _ = o.decode(0, sh.pos, q)
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_shards_concatenate_to_full(world):
    sh = CONFIGS["llama31_8b_decode_8k"].with_(pos=2047, seq_len=2048)
    k, v, q = decode_inputs(sh, 0)
    got = np.zeros((sh.n_heads, sh.head_dim), np.float32)
    for s in plan_shards(sh.n_kv_heads, sh.seq_len, world):
        with AttnContext.for_shape(sh, n_layers=1, kv_head_begin=s.kv_head_begin,
                                   kv_head_count=s.kv_head_count) as ctx:
            ctx.load_kv(0, 0, k, v)
            ctx.decode(0, sh.pos, q, out=got)  # writes only its own rows
    ok, ma, mr = tolerance_ok(got, _oracle(sh, k, v, q))
    assert ok, (ma, mr)


@pytest.mark.parametrize("name,seq_parts", [("gemma_2b_decode", 2), ("gemma_2b_decode", 4),
                                            ("llama31_8b_decode_8k", 2)])
def test_sequence_shards_lse_merge_to_full(name, seq_parts):
    import torch

    sh = CONFIGS[name]
    k, v, q = decode_inputs(sh, 0)
    world = seq_parts * (sh.n_kv_heads if sh.n_kv_heads < 8 else 1)
    shards = [s for s in plan_shards(sh.n_kv_heads, sh.seq_len, world, seq_parts=seq_parts) if s.head_group == 0]
    dq = torch.from_numpy(q).cuda()
    parts_o = torch.zeros((seq_parts, sh.n_heads, sh.head_dim), device="cuda")
    parts_ml = torch.zeros((seq_parts, sh.n_heads, 2), device="cuda")
    ctxs = []
    for s in shards:
        ctx = AttnContext.for_shape(sh, n_layers=1, kv_head_begin=s.kv_head_begin, kv_head_count=s.kv_head_count,
                                    seq_begin=s.seq_begin, seq_count=s.seq_count)
        ctx.load_kv(0, 0, k, v)
        ctx.decode_partial_dev(0, sh.pos, dq, parts_o[s.seq_part], parts_ml[s.seq_part])
        ctxs.append(ctx)
    out = torch.zeros((sh.n_heads, sh.head_dim), device="cuda")
    r0 = shards[0].kv_head_begin * sh.kv_mul
    r1 = (shards[0].kv_head_begin + shards[0].kv_head_count) * sh.kv_mul
    ctxs[0].lse_merge_dev(seq_parts, sh.n_heads, r0, r1 - r0, parts_o, parts_ml, out)
    torch.cuda.synchronize()
    for c in ctxs:
        c.check()
        c.close()
    want = _oracle(sh, k, v, q)
    ok, ma, mr = tolerance_ok(out.cpu().numpy()[r0:r1], want[r0:r1])
    assert ok, (ma, mr)


def test_partial_of_empty_shard_is_neutral():
    import torch

    sh = AttnShape("empty", 1, 4, 1, 128, 64, pos=10, seed=50)
    k, v, q = decode_inputs(sh, 0, ctx=64)
    with AttnContext.for_shape(sh, seq_begin=32, seq_count=32) as ctx:
        ctx.load_kv(0, 0, k, v)
        po = torch.full((4, 128), 7.0, device="cuda")
        pml = torch.zeros((4, 2), device="cuda")
        ctx.decode_partial_dev(0, sh.pos, torch.from_numpy(q).cuda(), po, pml)
        torch.cuda.synchronize()
        ctx.check()
    assert np.isneginf(pml[:, 0].cpu().numpy()).all()
    assert (pml[:, 1].cpu().numpy() == 0).all()
    assert (po.cpu().numpy() == 0).all()
