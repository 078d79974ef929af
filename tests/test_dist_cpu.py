"""Multi-process parity on CPU (gloo, world size 2): FSDP2 (shard 2) and
DDP give the same loss and gradient-norm traces for fp32 AdamW and Muon
(the FSDP path runs the sharded Newton-Schulz with its all-gathers)."""

import os
import socket

import torch
import torch.multiprocessing as mp

MODEL = dict(vocab_size=300, dim=64, layer_count=2, head_dim=32, context_len=64, ffn_hidden_dim=128)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(mode, opt_name, rank, steps=3):
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel as DDP
    from vagus_b200.models import build_model
    from vagus_b200.models.losses import make_ce
    from vagus_b200.optim import build_optimizer
    from vagus_b200.parallel import LMLoss, apply_fsdp, build_mesh, unwrap
    from vagus_b200.train.main import StepRunner
    torch.manual_seed(0)
    model = build_model("TransformerPP", MODEL)
    ce = make_ce("full")
    dev = torch.device("cpu")
    mesh = None
    if mode == "fsdp":
        mesh = build_mesh(2, dev, 2)
        model = LMLoss(model, ce)
        apply_fsdp(model, mesh, "float32", "float32")
    else:
        model = DDP(model)
    args = dict(lr=1e-2, weight_decay=0.1) if opt_name == "adamw" else \
        dict(lr=2e-2, weight_decay=0.1, adamw=dict(lr=1e-2, weight_decay=0.1))
    opt = build_optimizer(opt_name, unwrap(model), args)
    runner = StepRunner(model, opt, ce, dev, grad_accum_steps=2, grad_clip=1.0, is_fsdp=mode == "fsdp",
                        is_dist=True, mesh=mesh)
    g = torch.Generator().manual_seed(123 + rank)
    batches = []
    for _ in range(steps * 2):
        t = torch.randint(0, 300, (2, 33), generator=g)
        batches.append((t[:, :-1], t[:, 1:]))
    it = iter(batches)
    out = []
    for _ in range(steps):
        loss, _z, gn = runner.step(it)
        out.append((loss.item(), float(gn)))
    dist.barrier()
    return out


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank))
        from vagus_b200.parallel import setup_distributed
        setup_distributed("cpu", timeout_s=120)
        import torch.distributed as dist
        res = {}
        for opt_name in ("adamw", "muon"):
            res[opt_name] = {m: _run(m, opt_name, rank) for m in ("ddp", "fsdp")}
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


def test_fsdp_matches_ddp_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, res in results.items():
        assert not isinstance(res, str), res
        for opt_name, tol in (("adamw", 1e-5), ("muon", 2e-3)):
            for (la, ga), (lb, gb) in zip(res[opt_name]["ddp"], res[opt_name]["fsdp"]):
                assert abs(la - lb) <= tol * max(1.0, abs(la)), (opt_name, la, lb)
                assert abs(ga - gb) <= tol * max(1.0, abs(ga)) * 10, (opt_name, ga, gb)


def _layout_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank))
        from vagus_b200.parallel import setup_distributed
        setup_distributed("cpu", timeout_s=120)
        import torch.distributed as dist
        from torch.distributed.fsdp import FSDPModule
        from torch.distributed.fsdp._fully_shard._fsdp_api import AllGather
        from vagus_b200.models import build_model
        from vagus_b200.models.losses import make_ce
        from vagus_b200.parallel import LMLoss, apply_fsdp, build_mesh
        from vagus_b200.parallel.nvlink import unit_gather_layout

        class Recorder(AllGather):
            def __init__(self):
                self.inputs = []

            def allocate(self, size, *, dtype, device):
                return torch.empty(*size, dtype=dtype, device=device)

            def __call__(self, output_tensor, input_tensor, group, async_op=False):
                self.inputs.append(input_tensor.detach().clone())
                dist.all_gather_into_tensor(output_tensor, input_tensor, group=group)
                self.outputs = getattr(self, "outputs", []) + [output_tensor.detach().clone()]
                return None

        torch.manual_seed(0)
        model = LMLoss(build_model("TransformerPP", dict(MODEL, vocab_size=301)), make_ce("full"))
        apply_fsdp(model, build_mesh(world, torch.device("cpu"), world), "float32", "float32")
        blk = model.module.blocks[0]
        rec = Recorder()
        blk.set_custom_all_gather(rec)
        assert isinstance(blk, FSDPModule)
        layout = unit_gather_layout(blk)
        t = torch.randint(0, 301, (2, 33))
        model(t[:, :-1], t[:, 1:])                    # one forward: the block's parameters are gathered
        flat = rec.inputs[0]
        errs = []
        assert sum(e["numel"] for e in layout) == flat.numel()
        assert any(e["shape"][0] % world for e in layout)       # an uneven shard is among them
        for e in layout:
            name = e["name"]
            local = e["param"].to_local().detach().reshape(-1)       # this rank's (unpadded) shard
            got = flat[e["offset"]:e["offset"] + local.numel()]
            errs.append((name, (got - local).abs().max().item() if local.numel() else 0.0))
            assert e["rows"] == -(-e["shape"][0] // world), e
        # every rank's staging slot is its flat input: owner r's rows of a weight
        # start at slot_r + offset, which is what the in-place GEMM reads
        slots = rec.outputs[0].view(world, -1)
        for e in layout:
            if len(e["shape"]) != 2:
                continue
            rows, cols = e["rows"], e["shape"][1]
            w = torch.cat([slots[r, e["offset"]:e["offset"] + rows * cols].view(rows, cols) for r in range(world)])
            full = e["param"].full_tensor().detach()
            errs.append((e["name"] + " (from slots)", (w[:e["shape"][0]] - full).abs().max().item()))
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


def test_unit_gather_layout_matches_fsdp_all_gather_input():
    """The layout that a GEMM reading weight shards in place relies on: each
    parameter's shard sits at the predicted offset of the flat all-gather
    input FSDP2 hands to a custom all-gather (3 ranks: 64-row weights are
    split 22 / 22 / 20 and padded)."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_layout_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, errs in results.items():
        assert not isinstance(errs, str), errs
        assert errs and all(e == 0.0 for _, e in errs), (rank, errs)


def _hook_worker(rank, port, q):
    try:
        import torch.distributed as dist
        from torch.nn.parallel import DistributedDataParallel as DDP
        from vagus_b200.parallel.nvlink import NvlinkAllReduce
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
        ar = object.__new__(NvlinkAllReduce)        # no heaps on CPU: every bucket takes the fallback
        ar.group, ar.world, ar.rank, ar.slot, ar.calls = dist.group.WORLD, 2, rank, 0, {"nvlink": 0, "nccl": 0}
        torch.manual_seed(0)
        lin = torch.nn.Linear(8, 4)
        ref = torch.nn.Linear(8, 4)
        ref.load_state_dict(lin.state_dict())
        ddp, ddp_ref = DDP(lin), DDP(ref)
        ddp.register_comm_hook(None, ar.ddp_hook)  # DDP's own signature check runs here
        x = torch.randn(5, 8, generator=torch.Generator().manual_seed(rank))
        ddp(x).square().sum().backward()
        ddp_ref(x).square().sum().backward()
        err = max((a.grad - b.grad).abs().max().item() for a, b in zip(lin.parameters(), ref.parameters()))
        dist.destroy_process_group()
        q.put((rank, err, ar.calls["nccl"]))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e), 0))


def test_nvlink_allreduce_ddp_hook_registers_and_averages():
    """The NVLink all-reduce's DDP hook passes DDP's hook check and, on
    buffers it cannot take (CPU here), averages through the process group:
    gradients equal DDP's built-in all-reduce."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_hook_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
    for rank, err, calls in res:
        assert not isinstance(err, str), err
        assert err <= 1e-6 and calls >= 1, (rank, err, calls)
