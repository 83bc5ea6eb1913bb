"""Host logic of the sequence-parallel path on CPU: the cross-rank state exchange (all-gather,
exclusive prefix and suffix sums, async handles) with the gloo backend, world sizes 2 and 3."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from linatt_b200.sequence_parallel import exclusive_prefix_sum, exclusive_suffix_sum, gather_states

        x = torch.full((3, 4, 5), float(rank + 1))
        x[0, 0, 0] = 100.0 * (rank + 1)
        for async_op in (False, True):
            stacked = gather_states(x, async_op=async_op).wait()
            assert stacked.shape == (world, 3, 4, 5)
            for r in range(world):
                assert float(stacked[r, 1, 1, 1]) == r + 1
            pre = exclusive_prefix_sum(stacked, rank)
            suf = exclusive_suffix_sum(stacked, rank)
            exp_pre = sum(r + 1 for r in range(rank))
            exp_suf = sum(r + 1 for r in range(rank + 1, world))
            if rank == 0:
                assert pre is None
            else:
                assert float(pre[1, 1, 1]) == exp_pre and float(pre[0, 0, 0]) == 100.0 * exp_pre
            if rank == world - 1:
                assert suf is None
            else:
                assert float(suf[2, 3, 4]) == exp_suf and float(suf[0, 0, 0]) == 100.0 * exp_suf
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world", [2, 3])
def test_state_exchange_prefix_suffix_gloo(world):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_single_rank_falls_back_to_the_local_op_without_a_group():
    """Without an initialised process group sp_kata_attn is parallel_kata_attn (which refuses CPU
    tensors: there is no CPU path)."""
    from linatt_b200.sequence_parallel import sp_kata_attn

    q = torch.randn(1, 8, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        sp_kata_attn(q, q, q, num_groups=4)
