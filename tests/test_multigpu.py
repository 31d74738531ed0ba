"""Multi-GPU paths on real GPUs (skipped with fewer than two devices).

The DiT step over two GPUs against the reference model's latent, with the same bar as one
GPU, in both layouts (heads: NCCL all_gather_into_tensor of each attention's head outputs
before the o-proj; tokens: all_to_all_single into and out of the head-parallel attention,
the rest split by token rows), issued op by op and replayed as a captured CUDA graph."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_l2

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, q, shard):
    import datetime
    import sys
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from anima_attn.dit import AnimaDiT, DiTConfig, StepGraph, make_weights
        g = np.load(os.path.join(GOLDEN, "dit_small.npz"))
        blocks, side, wseed, iseed = (int(v) for v in g["meta"])
        rng = np.random.default_rng(iseed)
        x = rng.standard_normal((1, 16, side, side), dtype=np.float32)
        cc = rng.standard_normal((1, 512, 1024), dtype=np.float32)
        cu = rng.standard_normal((1, 512, 1024), dtype=np.float32)
        cfg = DiTConfig(blocks=blocks)
        model = AnimaDiT(cfg, make_weights(cfg, seed=wseed, device="cuda"), rank=rank,
                         world=world, group=dist.group.WORLD, shard=shard)
        T = lambda a: torch.from_numpy(a).cuda()
        args = (float(g["sigma"]), float(g["sigma_next"]))
        with torch.no_grad():
            out = model.euler_cfg_step(T(x), *args, T(cc), T(cu), float(g["cfg"])).cpu().numpy()
            graph = StepGraph(model, T(x), *args, T(cc), T(cu), float(g["cfg"]))
            gout = graph().cpu().numpy()
            del graph  # holds NCCL calls: released before the process group
        if rank == 0:
            q.put((rel_l2(out, g["x_next"]), rel_l2(gout, g["x_next"])))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("shard", ["tokens", "heads"])
def test_dit_step_two_gpus(shard):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200 + (0 if shard == "tokens" else 3)
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, shard)) for r in range(2)]
    for p in procs:
        p.start()
    r_eager, r_graph = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert r_eager <= 1e-2 and r_graph <= 1e-2
