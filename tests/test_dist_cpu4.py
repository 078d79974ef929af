"""Four gloo ranks on CPU emulating a 2-node x 2-GPU job: HSDP (2 x 2) and
FSDP2 (shard 4) loss / gradient-norm traces equal DDP's (fp32; and bf16 HSDP
vs DDP under bf16 autocast within 1e-3); the sharded Muon
step is bit-identical to the same step on replicated parameters, buckets
that do not divide by the world included; and train() under HSDP writes
checkpoints from which a resumed run reproduces the straight run exactly."""

import os
import shutil
import socket

import torch
import torch.multiprocessing as mp

from vagus_b200.data.prepare import synthetic_store

MODEL = dict(vocab_size=300, dim=64, layer_count=2, head_dim=32, context_len=64, ffn_hidden_dim=128)
WORLD = 4


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _env(rank, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                      LOCAL_RANK=str(rank))


def _trace(mode, opt_name, rank, steps=3, bf16=False):
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
    if mode == "ddp":
        model = DDP(model)
    else:
        mesh = build_mesh(2 if mode == "hsdp" else 4, dev, WORLD)
        model = LMLoss(model, ce)
        apply_fsdp(model, mesh, "bfloat16" if bf16 else "float32", "float32")
    args = dict(lr=1e-2, weight_decay=0.1) if opt_name == "adamw" else \
        dict(lr=2e-2, weight_decay=0.1, adamw=dict(lr=1e-2, weight_decay=0.1))
    opt = build_optimizer(opt_name, unwrap(model), args)
    amp = torch.autocast("cpu", dtype=torch.bfloat16) if bf16 else None
    runner = StepRunner(model, opt, ce, dev, grad_accum_steps=2, grad_clip=1.0, is_fsdp=mode != "ddp",
                        is_dist=True, mesh=mesh, autocast=amp)
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


def _sharded_muon_bitwise():
    """muon_update_sharded on Shard(0) DTensors == the same step on Replicate
    DTensors (every rank orthogonalises everything), bit for bit."""
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor
    from vagus_b200.optim.muon import muon_update_sharded
    mesh = init_device_mesh("cpu", (WORLD,))
    shapes = [(8, 16)] * 3 + [(16, 8)] * 5 + [(12, 20)]       # buckets of 3, 5 and 1 matrices
    g = torch.Generator().manual_seed(0)
    full_p = [torch.randn(s, generator=g) for s in shapes]
    full_g = [torch.randn(s, generator=g) for s in shapes]
    results = []
    for place in (Shard(0), Replicate()):
        P = [distribute_tensor(t.clone(), mesh, [place]) for t in full_p]
        Gr = [distribute_tensor(t.clone(), mesh, [place]) for t in full_g]
        M = [distribute_tensor(torch.zeros(s), mesh, [place]) for s in shapes]
        for _ in range(2):
            muon_update_sharded(P, Gr, M, lr=0.02, momentum=0.95, weight_decay=0.01, nesterov=True, ns_steps=5,
                                eps=1e-7)
        results.append([p.full_tensor() for p in P])
    return max((a - b).abs().max().item() for a, b in zip(*results))


def _train_cfg(tmp, run, steps):
    from vagus_b200.train import main as tm
    return tm.TrainConfig(run_name="h", data_dir=os.path.join(tmp, "tok"), model_name="TransformerPP",
                          model_args=MODEL, optimizer_name="muon", optimizer_args=dict(lr=2e-2, adamw=dict(lr=1e-2)),
                          context_len=32, batch_size=2, grad_accum_steps=2, train_tokens=steps * WORLD * 2 * 2 * 32,
                          world_size=WORLD, shard_size=2, device="cpu", dtype="float32", fsdp_param_dtype="float32",
                          compile=False,
                          ce_impl="full", run_dir=os.path.join(tmp, run), log_interval=1, slow_interval=1000,
                          deadline_margin_s=None, recent_ckpt_minutes=1e9, permanent_ckpt_interval=3)


def _worker(rank, port, tmp, q):
    try:
        _env(rank, port)
        from vagus_b200.parallel import setup_distributed
        setup_distributed("cpu", timeout_s=120)
        import torch.distributed as dist
        res = {"traces": {o: {m: _trace(m, o, rank) for m in ("ddp", "hsdp", "fsdp")} for o in ("adamw", "muon")},
               "bf16": {m: _trace(m, "adamw", rank, bf16=True) for m in ("ddp", "hsdp")},
               "muon_bitwise": _sharded_muon_bitwise()}
        from vagus_b200.train import main as tm
        tm.train(_train_cfg(tmp, "a", 6), teardown=False)
        if rank == 0:
            os.makedirs(os.path.join(tmp, "b"))
            shutil.copy(os.path.join(tmp, "a", "ckpt-00000003.pt"), os.path.join(tmp, "b", "ckpt-00000003.pt"))
        dist.barrier()
        tm.train(_train_cfg(tmp, "b", 6), teardown=False)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


def test_hsdp_fsdp_ddp_parity_sharded_muon_and_resume(tmp_path):
    synthetic_store(tmp_path / "tok", tokens=60_000, vocab=300, seed=1)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path), q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=900) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    for rank, res in results.items():
        assert not isinstance(res, str), res
        assert res["muon_bitwise"] == 0.0, (rank, res["muon_bitwise"])
        for opt_name, tol in (("adamw", 1e-5), ("muon", 2e-3)):
            tr = res["traces"][opt_name]
            for mode in ("hsdp", "fsdp"):
                for (la, ga), (lb, gb) in zip(tr["ddp"], tr[mode]):
                    assert abs(la - lb) <= tol * max(1.0, abs(la)), (opt_name, mode, la, lb)
                    assert abs(ga - gb) <= tol * max(1.0, abs(ga)) * 10, (opt_name, mode, ga, gb)
        # bf16: HSDP's bf16 parameter all-gathers vs DDP under bf16 autocast
        for (la, _), (lb, _) in zip(res["bf16"]["ddp"], res["bf16"]["hsdp"]):
            assert abs(la - lb) <= 1e-3 * max(1.0, abs(la)), ("bf16", la, lb)
    a = torch.load(tmp_path / "a" / "ckpt-00000006.pt", weights_only=False)
    b = torch.load(tmp_path / "b" / "ckpt-00000006.pt", weights_only=False)
    assert a["step"] == b["step"] == 6 and a["tokens_seen"] == b["tokens_seen"]
    for k in a["model"]:
        assert torch.equal(a["model"][k], b["model"][k]), k
