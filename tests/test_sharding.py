"""Batch sharding over ranks (no GPU): the request partition, rank-local page pools,
and a world-size-2 ``gloo`` run of the sharded decode checked against the whole batch.

The decode of each rank is the numpy oracle here (CPU); on GPUs ``bench.py`` runs
``mla_decode`` on the same rank-local inputs.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import recipes
from oracle import mla_oracle as orc
from triton_mla.sharding import balance_requests, contiguous_requests, rank_local_batch


def test_contiguous_requests_cover_in_order():
    for batch, world in [(32, 1), (32, 8), (5, 8), (0, 3), (37, 4)]:
        shards = contiguous_requests(batch, world)
        assert len(shards) == world
        assert sum(shards, []) == list(range(batch))
        sizes = [len(s) for s in shards]
        assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_balance_requests_is_a_balanced_partition(world):
    rng = np.random.default_rng(world)
    for _ in range(20):
        lens = rng.integers(1, 16385, size=int(rng.integers(1, 300))).tolist()
        shards = balance_requests(lens, world)
        flat = sorted(sum(shards, []))
        assert flat == list(range(len(lens))), "every request on exactly one rank"
        assert all(s == sorted(s) for s in shards)
        loads = [sum(lens[i] for i in s) for s in shards]
        assert max(loads) <= sum(lens) / world + max(lens), "LPT bound"
        assert shards == balance_requests(lens, world), "deterministic"


def test_balance_requests_on_the_ragged_baseline_config():
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(1, 16385, (256,), generator=g).tolist()
    for world in (2, 4, 8):
        loads = [sum(lens[i] for i in s) for s in balance_requests(lens, world)]
        assert max(loads) / (sum(lens) / world) < 1.01


def _case(seed=3):
    lens = [300, 0, 1000, 17, 640, 129, 64, 5]
    return recipes.paged_case(lens, 16, 16, seed=seed), lens


def _oracle(q, kv, lens, bt, scale):
    return orc.mla_decode_ref(q.float().numpy(), kv.float().numpy(), lens.numpy(), bt.numpy(),
                              softmax_scale=scale, dtype=np.float64)


@pytest.mark.parametrize("world", [2, 3])
def test_rank_local_batches_reproduce_the_whole_batch(world):
    case, lens = _case()
    full_out, full_lse = _oracle(case["q"], case["kv"], case["seqlens"], case["block_table"], case["scale"])
    seen = []
    for reqs in balance_requests(lens, world):
        q, kv, sl, bt = rank_local_batch(case["q"], case["kv"], case["seqlens"], case["block_table"], reqs)
        need = sum((lens[i] + 15) // 16 for i in reqs)
        assert kv.shape[0] == max(need, 1), "the rank's pool holds only its requests' pages"
        if not reqs:
            continue
        out, lse = _oracle(q, kv, sl, bt, case["scale"])
        np.testing.assert_allclose(out, full_out[reqs], rtol=0, atol=1e-12)
        valid = np.asarray([lens[i] for i in reqs]) > 0
        np.testing.assert_allclose(lse[valid], full_lse[reqs][valid], rtol=0, atol=1e-12)
        seen += reqs
    assert sorted(seen) == [i for i in range(len(lens))]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        case, lens = _case(seed=11)  # every rank builds the same global batch from the seed
        reqs = balance_requests(lens, world)[rank]
        q, kv, sl, bt = rank_local_batch(case["q"], case["kv"], case["seqlens"], case["block_table"], reqs)
        out, lse = _oracle(q, kv, sl, bt, case["scale"])
        gathered = [None] * world
        dist.all_gather_object(gathered, (reqs, out, lse))
        # the bench's timing rule: every rank contributes its time, the job reports the max
        t = torch.tensor([float(10 + rank)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full_out, full_lse = _oracle(case["q"], case["kv"], case["seqlens"], case["block_table"], case["scale"])
            out_all = np.zeros_like(full_out)
            lse_all = np.full_like(full_lse, np.nan)
            for r_reqs, r_out, r_lse in gathered:
                out_all[r_reqs] = r_out
                lse_all[r_reqs] = r_lse
            np.testing.assert_allclose(out_all, full_out, rtol=0, atol=1e-12)
            valid = np.asarray(lens) > 0
            np.testing.assert_allclose(lse_all[valid], full_lse[valid], rtol=0, atol=1e-12)
            assert float(t.item()) == 10.0 + world - 1
            open(os.path.join(result_dir, "ok"), "w").close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_world_size_two_sharded_decode(tmp_path):
    """Two ranks (processes, gloo on CPU) each decode their share of one batch; the
    gathered rows equal the decode of the whole batch and the reported time is the max."""
    ctx_port = _free_port()
    mp.start_processes(_rank_main, args=(2, ctx_port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "ok").exists()
