"""The all-gather fused into the consuming GEMM across two GPUs: a weight's
row shards live in CUDA-IPC heaps (``parallel.nvlink.PeerRowShards``) and the
gathered-B GEMM reads the peer's rows over NVLink inside its own TMA loads;
the product equals all-gather + matmul."""

import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rdzv():
    """A file rendezvous for the spawned ranks: no TCP port to collide with."""
    return "file://" + os.path.join(tempfile.mkdtemp(prefix="vagus_rdzv_"), "store")


def _ag_gemm_worker(rank, world, rdzv, q):
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world))
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world,
                                device_id=torch.device(f"cuda:{rank}"), timeout=datetime.timedelta(seconds=120))
        from vagus_b200 import ops
        from vagus_b200.parallel.nvlink import PeerRowShards
        errs = []
        for rows, cols, n in ((520, 1024, 1040), (256, 512, 500)):
            w = PeerRowShards(dist.group.WORLD, rows, cols)
            for it in range(2):                 # republished shards are read fresh
                g = torch.Generator(device="cuda").manual_seed(10 * it + rank)
                shard = torch.randn(rows, cols, device="cuda", generator=g).bfloat16()
                w.local().copy_(shard)
                w.publish()
                x = torch.randn(3, 100, cols, device="cuda", generator=g).bfloat16()
                y = w.linear(x, n)
                full = torch.empty(world * rows, cols, device="cuda", dtype=torch.bfloat16)
                dist.all_gather_into_tensor(full, shard)
                ref = x.float() @ full[:n].float().T
                errs.append(("ag_gemm", rows, ((y.float() - ref).norm() / ref.norm()).item()))
                w.publish()                     # nobody rewrites a shard a peer may still read
            torch.cuda.synchronize()
            w.close()
        errs.append(("error_word", 0, float(ops.native().error_word())))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gathered_weight_gemm_matches_allgather():
    """The all-gather fused into the GEMM (TMA loads of the peers' row shards)
    equals all-gather + matmul."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rdzv()
    procs = [ctx.Process(target=_ag_gemm_worker, args=(r, world, rdzv, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in results:
        assert not isinstance(errs, str), f"rank {rank}: {errs}"
        for kind, i, e in errs:
            assert e <= (1e-2 if kind == "ag_gemm" else 0.0), (rank, kind, i, e)
