"""Worker of tests/test_slab_gpu.py::test_nccl_ranks_reproduce_the_whole_mesh.

Launched under torch.distributed.run, one rank per GPU: each rank builds its
slab of the global mesh and either runs SlabOperator.apply (boundary layers,
NCCL exchange of the shared planes on a second stream overlapped with the
interior) twice and saves f ("apply", f32), or runs three power-iteration
steps (NCCL all-reduce of the owner-counted sum of squares) and saves u
("power", f64); the parent test compares with the CPU oracle on the whole
mesh.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def main(out_dir, nex, ney, nez, seed, mode="apply", ngll=5):
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
        dtype = np.float32 if mode == "apply" else np.float64
        part = SlabPartition(nex, ney, nez, ngll, world, rank)
        prob = slab_problem(part, dtype, seed)
        u, f, arrays, ibool = to_device(prob, dev)
        plan = prob.plan()
        op = SlabOperator(part, plan, plan.fields(u, f, arrays, ibool), f, dev, u=u)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            if mode == "apply":
                op.apply(stream)
                op.apply(stream)  # a second application must give the same f
            else:
                for _ in range(3):
                    op.power_step(stream)
                op.power_u(stream)
        torch.cuda.synchronize()
        out = f if mode == "apply" else u
        np.save(os.path.join(out_dir, f"{'f' if mode == 'apply' else 'u'}{rank}.npy"),
                np.stack([x.cpu().numpy() for x in out]))
        op.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    out, nex, ney, nez, seed = sys.argv[1], *map(int, sys.argv[2:6])
    mode = sys.argv[6] if len(sys.argv) > 6 else "apply"
    ngll = int(sys.argv[7]) if len(sys.argv) > 7 else 5
    main(out, nex, ney, nez, seed, mode, ngll)
