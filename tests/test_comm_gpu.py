"""NVLink peer-to-peer collectives (ops/csrc/comm.cu) against NCCL, on two
GPUs: raw all-gather / reduce-scatter over several epochs (slot reuse),
FSDP2 with the custom collectives installed against FSDP2 on NCCL, the fused
Muon scatter, and the all-reduce (raw and as DDP's bucket hook)."""

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


def _worker(rank, world, rdzv, q):
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world))
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world,
                                device_id=torch.device(f"cuda:{rank}"), timeout=datetime.timedelta(seconds=120))
        from vagus_b200 import ops
        from vagus_b200.parallel.nvlink import NvlinkAllGather, NvlinkHeap, NvlinkReduceScatter
        heap = NvlinkHeap(dist.group.WORLD, ag_cap=1 << 20, rs_cap=4 << 20)
        ag, rs = NvlinkAllGather(heap), NvlinkReduceScatter(heap)
        errs = []
        for it in range(5):
            g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
            n = 1000 + 37 * it
            shard = torch.randn(n, device="cuda", generator=g).bfloat16()
            out = torch.empty(world * n, device="cuda", dtype=torch.bfloat16)
            out[rank * n:(rank + 1) * n].copy_(shard)
            ag(out, out[rank * n:(rank + 1) * n], dist.group.WORLD)
            ref = torch.empty_like(out)
            dist.all_gather_into_tensor(ref, shard)
            errs.append(("ag", it, (out.float() - ref.float()).abs().max().item()))
            full = torch.randn(world * n, device="cuda", generator=g)
            for op in (dist.ReduceOp.AVG, dist.ReduceOp.SUM):
                o = torch.empty(n, device="cuda")
                rs(o, full, dist.group.WORLD, op)
                r = torch.empty(n, device="cuda")
                dist.reduce_scatter_tensor(r, full.clone(), op=op)
                errs.append(("rs", it, (o - r).abs().max().item()))
        torch.cuda.synchronize()
        errs.append(("error_word", 0, float(ops.native().error_word())))

        # FSDP2 with the NVLink collectives == FSDP2 on NCCL
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.fsdp import fully_shard
        from vagus_b200.parallel.nvlink import use_nvlink_collectives
        mesh = init_device_mesh("cuda", (world,))

        def make():
            torch.manual_seed(0)
            m = torch.nn.Sequential(torch.nn.Linear(256, 512, bias=False), torch.nn.GELU(),
                                    torch.nn.Linear(512, 256, bias=False)).cuda()
            for layer in m:
                if isinstance(layer, torch.nn.Linear):
                    fully_shard(layer, mesh=mesh)
            fully_shard(m, mesh=mesh)
            return m

        grads = []
        for nv in (False, True):
            m = make()
            if nv:
                use_nvlink_collectives(m)
            x = torch.randn(64, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(rank))
            m(x).pow(2).mean().backward()
            grads.append([p.grad.full_tensor() for p in m.parameters()])
        for a, b in zip(*grads):
            errs.append(("fsdp", 0, (a - b).abs().max().item()))
        heap.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nvlink_collectives_match_nccl():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rdzv()
    procs = [ctx.Process(target=_worker, args=(r, world, rdzv, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in results:
        assert not isinstance(errs, str), f"rank {rank}: {errs}"
        for kind, it, e in errs:
            tol = 0.0 if kind in ("ag", "error_word") else 1e-5
            assert e <= tol, (rank, kind, it, e)


def _muon_worker(rank, world, rdzv, q):
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world))
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world,
                                device_id=torch.device(f"cuda:{rank}"), timeout=datetime.timedelta(seconds=120))
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Shard, distribute_tensor
        from vagus_b200 import ops
        from vagus_b200.optim.muon import muon_update_sharded
        mesh = init_device_mesh("cuda", (world,))
        shapes = [(256, 512)] * 3 + [(512, 256)] * 2 + [(128, 384)]
        g = torch.Generator().manual_seed(0)
        full_p = [torch.randn(s, generator=g) for s in shapes]
        full_g = [torch.randn(s, generator=g) for s in shapes]
        results = []
        exchanges = {}
        for use in (None, exchanges):
            P = [distribute_tensor(t.clone().cuda(), mesh, [Shard(0)]) for t in full_p]
            Gr = [distribute_tensor(t.clone().cuda(), mesh, [Shard(0)]) for t in full_g]
            M = [distribute_tensor(torch.zeros(s, device="cuda"), mesh, [Shard(0)]) for s in shapes]
            for _ in range(3):          # three epochs: both slots and a reuse
                muon_update_sharded(P, Gr, M, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True,
                                    ns_steps=5, eps=1e-7, exchanges=use)
            torch.cuda.synchronize()
            results.append([p.to_local().clone() for p in P])
        errs = [("muon", i, (a - b).abs().max().item()) for i, (a, b) in enumerate(zip(*results))]
        errs.append(("fused_used", 0, 0.0 if exchanges else 1.0))
        errs.append(("error_word", 0, float(ops.native().error_word())))
        for ex in exchanges.values():
            ex.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_muon_fused_scatter_matches_allgather():
    """The sharded Muon step with the momentum row shards pushed to the
    matrices' owners and the Newton-Schulz product scattered back to the row
    owners from the GEMM epilogue equals the all-gather path bit for bit
    (a bucket of three matrices over two ranks exercises the zero padding)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rdzv()
    procs = [ctx.Process(target=_muon_worker, args=(r, world, rdzv, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in results:
        assert not isinstance(errs, str), f"rank {rank}: {errs}"
        for kind, i, e in errs:
            assert e == 0.0, (rank, kind, i, e)


def _allreduce_worker(rank, world, rdzv, q):
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world),
                          NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world,
                                device_id=torch.device(f"cuda:{rank}"), timeout=datetime.timedelta(seconds=120))
        from vagus_b200 import ops
        from vagus_b200.parallel import wrap_ddp
        from vagus_b200.parallel.nvlink import NvlinkAllReduce
        ar = NvlinkAllReduce(dist.group.WORLD, 8 << 20)
        errs = []
        g = torch.Generator(device="cuda").manual_seed(rank)
        for it, (n, dt, op) in enumerate([(1, torch.float32, dist.ReduceOp.SUM), (7, torch.float32, dist.ReduceOp.AVG),
                                           (4099, torch.bfloat16, dist.ReduceOp.AVG),
                                           (1 << 20, torch.float32, dist.ReduceOp.AVG),
                                           (123457, torch.float32, dist.ReduceOp.SUM),
                                           (1 << 20, torch.bfloat16, dist.ReduceOp.SUM)]):
            x = torch.randn(n, device="cuda", generator=g).to(dt)
            ref = x.clone()
            dist.all_reduce(ref, op=op)
            ar(x, op)
            tol = 1e-5 if dt == torch.float32 else 2e-2
            errs.append(("ar", it, ((x.float() - ref.float()).abs().max() / ref.float().abs().max().clamp(min=1)).item(),
                         tol))
        big = torch.randn(3 << 20, device="cuda")                   # beyond the slot: NCCL fallback
        ref = big.clone()
        dist.all_reduce(ref)
        ar(big, dist.ReduceOp.SUM)
        errs.append(("fallback", 0, (big - ref).abs().max().item(), 1e-5))
        errs.append(("fallback_used", 0, 0.0 if ar.calls["nccl"] == 1 else 1.0, 0.0))
        torch.cuda.synchronize()

        # DDP with the NVLink bucket all-reduce == DDP on NCCL
        def trace(comm):
            torch.manual_seed(0)
            m = torch.nn.Sequential(torch.nn.Linear(256, 1024), torch.nn.GELU(), torch.nn.Linear(1024, 256)).cuda()
            ddp = wrap_ddp(m, torch.device(f"cuda:{rank}"), comm)
            opt = torch.optim.SGD(ddp.parameters(), lr=0.1)
            out = []
            for step in range(3):
                xb = torch.randn(32, 256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(step * 7 + rank))
                opt.zero_grad()
                ddp(xb).pow(2).mean().backward()
                out.append(torch.cat([p.grad.flatten() for p in m.parameters()]).clone())
                opt.step()
            used = ddp.nvlink_allreduce.calls["nvlink"] if ddp.nvlink_allreduce is not None else 0
            return out, used
        a, _ = trace("nccl")
        b, used = trace("nvlink")
        for i, (x, y) in enumerate(zip(a, b)):
            errs.append(("ddp", i, ((x - y).abs().max() / y.abs().max()).item(), 1e-5))
        errs.append(("ddp_hook_used", 0, 0.0 if used > 0 else 1.0, 0.0))
        errs.append(("error_word", 0, float(ops.native().error_word()), 0.0))
        ar.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nvlink_all_reduce_and_ddp_hook_match_nccl():
    """The two-shot NVLink all-reduce equals NCCL's (fp32 / bf16, sum /
    average, ragged sizes, several epochs over both slots, a too-large
    tensor through the NCCL fallback), and DDP with it as the bucket
    communication hook produces the gradients DDP on NCCL does."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rdzv()
    procs = [ctx.Process(target=_allreduce_worker, args=(r, world, rdzv, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in results:
        assert not isinstance(errs, str), f"rank {rank}: {errs}"
        for kind, it, e, tol in errs:
            assert e <= tol, (rank, kind, it, e)
