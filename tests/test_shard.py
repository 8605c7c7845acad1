"""Host-side multi-GPU logic on CPU: shard planning, the LSE merge of
sequence-split partials, and the same merge across two gloo ranks."""
import os
import socket

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.shard import lse_merge_np, partial_attention_np, plan_shards
from llama3pure_b200.synth import CONFIGS, AttnShape, decode_inputs, tolerance_ok


@pytest.mark.parametrize("name", ["llama31_8b_decode_8k", "llama31_8b_decode_128k", "gemma_2b_decode"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_every_head_and_position_once(name, world):
    sh = CONFIGS[name]
    shards = plan_shards(sh.n_kv_heads, sh.seq_len, world)
    cover = np.zeros((sh.n_kv_heads, sh.seq_len), np.int32)
    for s in shards:
        cover[s.kv_head_begin:s.kv_head_begin + s.kv_head_count, s.seq_begin:s.seq_begin + s.seq_count] += 1
    assert (cover == 1).all()
    # heads first: Llama's 8 KV heads give every rank its own head group up to 8 ranks
    if sh.n_kv_heads == 8:
        assert all(s.seq_count == sh.seq_len for s in shards)


def test_plan_explicit_sequence_split():
    shards = plan_shards(8, 131072, 8, seq_parts=2)
    assert {(s.kv_head_count, s.seq_count) for s in shards} == {(2, 65536)}


def _reference(sh, k, v, q):
    o = O.Oracle(sh, O.MODE_F32, "port", n_layers=1)
    o.load_kv(0, 0, k, v)
    out, _ = o.decode(0, sh.pos, q)
    return out


@pytest.mark.parametrize("parts", [1, 2, 3, 7])
def test_lse_merge_of_sequence_partials_matches_oracle(parts):
    sh = AttnShape("merge", 1, 8, 2, 64, 300, pos=299, seed=21)
    k, v, q = decode_inputs(sh, 0)
    want = _reference(sh, k, v, q)
    bounds = np.linspace(0, sh.pos + 1, parts + 1).astype(int)
    po, pml = zip(*[partial_attention_np(q, k, v, sh.scale, bounds[i], bounds[i + 1], sh.kv_mul)
                    for i in range(parts)])
    got = lse_merge_np(np.stack(po), np.stack(pml))
    ok, ma, mr = tolerance_ok(got, want)
    assert ok, (ma, mr)


def test_lse_merge_ignores_empty_partials():
    sh = AttnShape("merge", 1, 4, 1, 64, 50, pos=49, seed=22)
    k, v, q = decode_inputs(sh, 0)
    want = _reference(sh, k, v, q)
    full = partial_attention_np(q, k, v, sh.scale, 0, 50, sh.kv_mul)
    empty = partial_attention_np(q, k, v, sh.scale, 50, 50, sh.kv_mul)
    got = lse_merge_np(np.stack([empty[0], full[0]]), np.stack([empty[1], full[1]]))
    assert tolerance_ok(got, want)[0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    sh = AttnShape("gloo", 1, 8, 1, 64, 257, pos=256, seed=23)
    k, v, q = decode_inputs(sh, 0)
    shard = plan_shards(sh.n_kv_heads, sh.pos + 1, world)[rank]
    o, ml = partial_attention_np(q, k, v, sh.scale, shard.seq_begin, shard.seq_begin + shard.seq_count, sh.kv_mul)
    go = [torch.zeros(o.shape) for _ in range(world)]
    gml = [torch.zeros(ml.shape) for _ in range(world)]
    dist.all_gather(go, torch.from_numpy(o))
    dist.all_gather(gml, torch.from_numpy(ml))
    merged = lse_merge_np(np.stack([t.numpy() for t in go]), np.stack([t.numpy() for t in gml]))
    if rank == 0:
        np.save(result_path, merged)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_sequence_split_merge(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    res = str(tmp_path / "merged.npy")
    mp.start_processes(_gloo_rank, args=(world, _free_port(), res), nprocs=world, join=True, start_method="spawn")
    sh = AttnShape("gloo", 1, 8, 1, 64, 257, pos=256, seed=23)
    k, v, q = decode_inputs(sh, 0)
    want = _reference(sh, k, v, q)
    ok, ma, mr = tolerance_ok(np.load(res), want)
    assert ok, (ma, mr)
