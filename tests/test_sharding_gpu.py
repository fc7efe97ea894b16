"""The sharded decode on two GPUs: one process per GPU over NCCL, each rank decoding its
token-balanced share of one batch from its own compact page pool (no collective on the data
path).  The rows gathered on rank 0 equal the oracle's and, bit for bit, the one-GPU decode of
the whole batch with the same split count.  Skipped on a machine with fewer than two GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import recipes
from oracle import mla_oracle as orc
from triton_mla import mla_decode
from triton_mla.sharding import balance_requests, rank_local_batch

pytestmark = pytest.mark.gpu

LENS = [4096, 1, 0, 2500, 777, 64, 3000, 129, 1500, 2048]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    try:
        case = recipes.paged_case(LENS, 128, 64, seed=12)  # the same global batch on every rank
        reqs = balance_requests(LENS, world)[rank]
        q, kv, sl, bt = rank_local_batch(case["q"], case["kv"], case["seqlens"], case["block_table"], reqs)
        out, lse = mla_decode(q.to(device), kv.to(device), sl.to(device), bt.to(device),
                              softmax_scale=case["scale"], num_splits=2, return_lse=True)
        torch.cuda.synchronize(device)
        gathered = [None] * world
        dist.all_gather_object(gathered, (reqs, out.float().cpu().numpy(), lse.cpu().numpy()))
        if rank == 0:
            full_out, full_lse = mla_decode(case["q"].to(device), case["kv"].to(device), case["seqlens"].to(device),
                                            case["block_table"].to(device), softmax_scale=case["scale"],
                                            num_splits=2, return_lse=True)
            full_out, full_lse = full_out.float().cpu().numpy(), full_lse.cpu().numpy()
            out_all = np.full_like(full_out, np.nan)
            lse_all = np.full_like(full_lse, np.nan)
            for r_reqs, r_out, r_lse in gathered:
                out_all[r_reqs] = r_out
                lse_all[r_reqs] = r_lse
            # bit-identical to the one-GPU decode of the whole batch (requests are independent)
            assert np.array_equal(out_all, full_out)
            assert np.array_equal(lse_all, full_lse)
            ref_out, ref_lse = orc.mla_decode_ref(case["q"].float().numpy(), case["kv"].float().numpy(),
                                                  case["seqlens"].numpy(), case["block_table"].numpy(),
                                                  softmax_scale=case["scale"], dtype=np.float64)
            assert np.abs(out_all - ref_out).max() <= 2e-2
            valid = np.asarray(LENS) > 0
            assert np.abs(lse_all[valid] - ref_lse[valid]).max() <= 1e-3
            assert np.all(out_all[~valid] == 0) and np.all(np.isneginf(lse_all[~valid]))
            open(os.path.join(result_dir, "ok"), "w").close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_decode_matches_the_whole_batch(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "ok").exists()
