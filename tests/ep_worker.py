"""One rank of the NCCL expert-parallel check (run by tests/test_gpu_ep.py under torchrun).

Every rank builds the same seeded layer, keeps its expert slice and its token
shard, runs ``ExpertParallelMoE`` over NCCL, and compares with the single-GPU
fused layer on the same tokens (bit-exact: the same kernels see every row).
Rank 0 prints EP_OK when all ranks agree."""
from __future__ import annotations

import importlib
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    e4b = importlib.import_module("experts4bit-qlora_b200")
    E, H, I, k, T = 8, 256, 256, 2, 384
    g = torch.Generator().manual_seed(0)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    mod = e4b.Experts4bit.from_float(gate_up.cuda(), down.cuda())
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    logits = torch.randn(T, E, generator=g).cuda()
    w, idx = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    sizes = [T // world + (1 if r < T % world else 0) for r in range(world)]
    t0 = sum(sizes[:rank])
    t1 = t0 + sizes[rank]
    layer = e4b.ExpertParallelMoE.from_module(mod)
    got = layer(x[t0:t1], idx[t0:t1], w[t0:t1])
    got2 = layer(x[t0:t1], idx[t0:t1], w[t0:t1], micro_batches=3)  # comm stream overlapping compute
    ref = e4b.ops.moe_forward(x[t0:t1].contiguous(), idx[t0:t1].contiguous(), w[t0:t1].contiguous(),
                              mod.gate_up_proj.data, mod.gate_up_absmax, mod.down_proj.data, mod.down_absmax, E, I)
    ok = torch.tensor([1 if torch.equal(got, ref) and torch.equal(got2, ref) else 0], device="cuda")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if rank == 0 and int(ok.item()) == 1:
        print("EP_OK", flush=True)
    dist.destroy_process_group()
    return 0 if int(ok.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
