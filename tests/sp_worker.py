"""Worker of the multi-GPU sequence-parallel parity test (launched by tests/test_gpu_sp.py with
torchrun): every rank runs sp_kata_attn forward + backward on its shard; rank 0 gathers the shards
and compares them with the single-GPU kernels over the whole sequence (relative L2 < 1e-2)."""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from linatt_b200.parallel_kata_attn import parallel_kata_attn
    from linatt_b200.sequence_parallel import sp_kata_attn

    B, T, H, D, M = 1, 1024 * world, 2, 128, 4
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(B, T, H, D, generator=g) / D ** 0.5 for _ in range(3))
    do = torch.randn(B, T, H, D, generator=g)
    q, k, v, do = (x.bfloat16().to(dev) for x in (q, k, v, do))
    sl = slice(rank * T // world, (rank + 1) * T // world)
    leaves = [x[:, sl].clone().requires_grad_(True) for x in (q, k, v)]
    o = sp_kata_attn(*leaves, num_groups=M)
    o.backward(do[:, sl])
    mine = torch.stack([o.detach().float()] + [x.grad.float() for x in leaves])
    allp = [torch.empty_like(mine) for _ in range(world)] if rank == 0 else None
    dist.gather(mine, allp, dst=0)
    ok = True
    if rank == 0:
        got = torch.cat(allp, dim=2)  # (4, B, T, H, D)
        fl = [x.clone().requires_grad_(True) for x in (q, k, v)]
        fo = parallel_kata_attn(*fl, num_groups=M)
        fo.backward(do)
        ref = torch.stack([fo.detach().float()] + [x.grad.float() for x in fl])
        for i, name in enumerate(("o", "dq", "dk", "dv")):
            e = float((got[i] - ref[i]).norm() / ref[i].norm())
            print(f"{name} rel-L2 {e:.3e}", flush=True)
            ok = ok and e < 1e-2
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and flag.item() == 1:
        print("SP_OK", flush=True)
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
