"""Worker of tests/test_slab_gpu.py::test_nccl_ranks_reproduce_the_whole_mesh.

Launched under torch.distributed.run, one rank per GPU: each rank builds its
slab of the global mesh, runs SlabOperator.apply (boundary layers, NCCL
exchange of the shared planes on a second stream overlapped with the
interior) twice, and saves its f for the parent test to compare with the CPU
oracle on the whole mesh.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def main(out_dir, nex, ney, nez, seed):
    import torch
    import torch.distributed as dist
    from tensoroperations_b200.sem3d import to_device
    from tensoroperations_b200.slab import SlabOperator, SlabPartition, slab_problem

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        part = SlabPartition(nex, ney, nez, 5, world, rank)
        prob = slab_problem(part, np.float32, seed)
        u, f, arrays, ibool = to_device(prob, dev)
        plan = prob.plan()
        op = SlabOperator(part, plan, plan.fields(u, f, arrays, ibool), f, dev)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            op.apply(stream)
            op.apply(stream)  # a second application must give the same f
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"f{rank}.npy"), np.stack([x.cpu().numpy() for x in f]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    out, nex, ney, nez, seed = sys.argv[1], *map(int, sys.argv[2:6])
    main(out, nex, ney, nez, seed)
