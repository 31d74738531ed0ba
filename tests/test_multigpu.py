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


def _rank(rank, world, port, q, shard, peer_gather=True, peer_a2a=True):
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
                         world=world, group=dist.group.WORLD, shard=shard,
                         peer_gather=peer_gather, peer_a2a=peer_a2a)
        assert model.peer_gather == (peer_gather and shard == "heads")
        assert model.peer_a2a == (peer_a2a and shard == "tokens")
        T = lambda a: torch.from_numpy(a).cuda()
        args = (float(g["sigma"]), float(g["sigma_next"]))
        with torch.no_grad():
            out = model.euler_cfg_step(T(x), *args, T(cc), T(cu), float(g["cfg"])).cpu().numpy()
            graph = StepGraph(model, T(x), *args, T(cc), T(cu), float(g["cfg"]))
            gout = graph().cpu().numpy()
            del graph  # holds NCCL calls: released before the process group
        torch.cuda.synchronize()
        model.close()  # peer mappings of the gather buffers
        if rank == 0:
            q.put((rel_l2(out, g["x_next"]), rel_l2(gout, g["x_next"])))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("shard,peer", [("tokens", True), ("tokens", False), ("heads", True),
                                        ("heads", False)])
def test_dit_step_two_gpus(shard, peer):
    """heads with peer (peer_gather): the attention kernel stores every head output into both
    ranks' gather buffers over NVLink (anima_attn_fwd_gather), a one-element all-reduce
    orders the ranks; without it, an NCCL all_gather_into_tensor.  tokens with peer
    (peer_a2a): the projection GEMM stores each head's operand rows into its owner's buffers
    and the attention each output row into its token owner's buffer; without it, two NCCL
    all_to_all_single per attention."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200 + {("tokens", True): 0, ("tokens", False): 9,
                                          ("heads", True): 3, ("heads", False): 6}[(shard, peer)]
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, shard, peer, peer))
             for r in range(2)]
    for p in procs:
        p.start()
    r_eager, r_graph = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert r_eager <= 1e-2 and r_graph <= 1e-2


def _gather_rank(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import anima_attn
        from anima_attn.peer import GatherBuffers
        B, H, hl, S, D = 2, 4, 2, 1000, 128  # ragged S: a partial unit and a partial key tile
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        qh, kh, vh = (torch.randn(B * hl, S, D, device="cuda", generator=g).half()
                      for _ in range(3))
        gb = GatherBuffers((B, S, H, D), torch.float16, "cuda", dist.group.WORLD, rank, world)
        for i in range(2):  # both buffers, twice each
            for _ in range(2):
                mine = gb.bufs[i][:, :, rank * hl:(rank + 1) * hl]
                anima_attn.attention_core(qh, kh, vh, B, hl, out=mine, out_dtype=torch.float16,
                                          peers=gb.destinations(i, rank * hl * D))
                gb.barrier()
        local = anima_attn.attention_core(qh, kh, vh, B, hl, out_dtype=torch.float16)
        full = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device="cuda")
        dist.all_gather_into_tensor(full, local.contiguous())
        ref = full.permute(1, 2, 0, 3, 4).reshape(B, S, H, D)
        torch.cuda.synchronize()
        ok = all(torch.equal(gb.bufs[i], ref) for i in range(2))
        status = anima_attn.status()
        gb.close()
        q.put((rank, ok, status))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_attention_epilogue_gather_equals_nccl_all_gather():
    """anima_attn_fwd_gather on two GPUs: each rank's attention stores its 2 heads into both
    ranks' [B, S, 4, D] buffers (peer mappings by CUDA IPC); after the barrier both buffers
    equal the NCCL all-gather of the same attention's local outputs, bit for bit."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 80
    procs = [ctx.Process(target=_gather_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == [(0, True, 0), (1, True, 0)]


def _scatter_rank(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import anima_attn
        from anima_attn import ops
        from anima_attn.peer import PeerBuffers
        B, L, side, H, hl, K, D = 2, 1024, 32, 4, 2, 256, 128
        n = B * L // world                       # token rows per rank
        g = torch.Generator(device="cuda").manual_seed(7)  # same values on both ranks
        x = torch.randn(B * L, K, device="cuda", generator=g).half()
        w = (torch.randn(3 * H * D, K, device="cuda", generator=g) / K ** 0.5).half()
        qw = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
        kw = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
        fr = anima_attn.rope_freqs_3d(1, side, side, device="cuda")
        op = ((B * hl, L, D), torch.float16)
        pb = PeerBuffers({"q": op, "k": op, "v": op, "o": ((n, H * D), torch.float16)}, "cuda",
                         dist.group.WORLD, rank, world)
        dest = [(pb.ptr("q", d), pb.ptr("k", d), pb.ptr("v", d)) for d in range(world)]
        ops.qkv_projection_scatter(x[rank * n:(rank + 1) * n].contiguous(), w, B, L, hl, rank * n,
                                   dest, 3, 0, qw, kw, fr, 1e-6)
        pb.barrier()
        # reference: this rank's heads projected from all rows by the local kernel
        w_mine = torch.cat([w[c * H * D + rank * hl * D:c * H * D + (rank + 1) * hl * D]
                            for c in range(3)]).contiguous()
        ref = ops.qkv_projection(x.view(B, L, K), w_mine, hl, 3, 0, qw, kw, fr, 1e-6)
        ok_proj = all(torch.allclose(pb.local[c].float(), r.float(), rtol=0, atol=2e-2)
                      for c, r in zip("qkv", ref))
        # attention on this rank's heads, output rows to their owners
        anima_attn.attention_core(pb.local["q"], pb.local["k"], pb.local["v"], B, hl,
                                  out_dtype=torch.float16,
                                  scatter=(pb.ptrs("o"), n, H * D, rank * hl))
        pb.barrier()
        # reference: every head's attention from the local projections of all heads
        qa, ka, va = ops.qkv_projection(x.view(B, L, K), w, H, 3, 0, qw, kw, fr, 1e-6)
        full = anima_attn.attention_core(qa, ka, va, B, H, out_dtype=torch.float16)  # [B,L,H,D]
        mine = full.reshape(B * L, H * D)[rank * n:(rank + 1) * n]
        ok_attn = torch.allclose(pb.local["o"].float(), mine.float(), rtol=0, atol=2e-2)
        torch.cuda.synchronize()
        status = anima_attn.status()
        pb.close()
        q.put((rank, bool(ok_proj), bool(ok_attn), status))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_projection_and_attention_scatter_equal_local_computation():
    """The tokens layout's two all-to-alls folded into kernels, on two GPUs: each rank
    projects its half of the token rows for all 4 heads (anima_qkv_projection_scatter) and
    every head's rows land in the owning rank's q/k/v buffers, equal to the local projection
    of all rows for its 2 heads; each rank's attention of its heads stores every output row
    into its token owner's [rows, 4 x 128] buffer (anima_attn_fwd_scatter_rows), equal to the
    owner's rows of an all-head attention computed locally."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29990 + os.getpid() % 8
    procs = [ctx.Process(target=_scatter_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == [(0, True, True, 0), (1, True, True, 0)]
