"""Helper launched by tests/test_gpu_multi.py under torchrun: runs a reduced
projection chain column-sharded over the ranks (CUDA graph; gathers by NCCL, or
fused into the projections over NVLink peer memory when argv[2] is "p2p", or
the whole step in one persistent kernel when it is "persistent") and
writes the final output bits of rank 0 to the path given as argv[1]."""

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from klab_b200.chain import ChainShape, ProjectionChain  # noqa: E402


def main():
    out_path = sys.argv[1]
    mode = sys.argv[2] if len(sys.argv) > 2 else "nccl"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    shape = ChainShape(layers=4, hidden=1024, kv=256, ffn=3584)
    persistent = mode == "persistent"
    gather = "p2p" if mode in ("p2p", "persistent") else "nccl"
    chain = ProjectionChain(shape, rank=rank, world=world, group=group, seed=11, gather=gather,
                            persistent=persistent)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    x = torch.randn((1, shape.hidden), generator=gen, device="cuda").to(torch.bfloat16)
    eager = chain.forward_eager(x).clone()
    out = chain.capture(x)
    for _ in range(3):
        chain.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), eager.view(torch.int16)), "graph replay differs from eager"
    from klab_b200 import _native

    assert _native.device_status() == 0, "a bounded wait gave up"
    if rank == 0:
        np.save(out_path, out.view(torch.int16).cpu().numpy())
    chain.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
