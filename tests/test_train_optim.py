"""Optimizer (Newton-Schulz, Muon, coverage, schedules) and the trainer:
a short CPU run, checkpoints, resume == uninterrupted run, stop request."""

import shutil

import pytest
import torch

from vagus_b200.data.prepare import synthetic_store
from vagus_b200.models import build_model
from vagus_b200.optim import build_optimizer
from vagus_b200.optim.muon import newton_schulz
from vagus_b200.train import main as tm
from vagus_b200.train.schedule import build_schedule, cosine, linear, wsd


@pytest.mark.parametrize("scheme", ["jordan", "polar_express"])
def test_newton_schulz_orthogonalises(scheme):
    torch.manual_seed(0)
    for shape in [(64, 32), (32, 64), (48, 48)]:
        G = torch.randn(*shape, dtype=torch.float32)
        X = newton_schulz(G, steps=5, scheme=scheme).float()
        s = torch.linalg.svdvals(X)
        assert s.max() < 1.3 and s.min() > 0.5, (scheme, shape, s.min().item(), s.max().item())
        # same column space as G: X ~ U V^T
        U, _, Vh = torch.linalg.svd(G, full_matrices=False)
        cos = torch.nn.functional.cosine_similarity((U @ Vh).flatten(), X.flatten(), dim=0)
        assert cos > 0.95


def test_schedules():
    assert cosine(0.0, warmup=0.1) == pytest.approx(0.0, abs=1e-6)
    assert cosine(1.0, warmup=0.1, min_ratio=0.1) == pytest.approx(0.1, abs=1e-6)
    assert linear(0.55, warmup=0.1, min_ratio=0.0) == pytest.approx(0.5, abs=1e-6)
    assert wsd(0.5, warmup=0.01, decay=0.2) == pytest.approx(1.0)
    assert wsd(1.0, warmup=0.01, decay=0.2, min_ratio=0.0) == pytest.approx(0.0, abs=1e-6)
    f = build_schedule("wsd", {"warmup": 0.01, "decay": 0.2})
    assert 0.0 <= f(0.95) < 1.0
    with pytest.raises(Exception):
        build_schedule("nope", {})


MODEL = dict(vocab_size=500, dim=64, layer_count=2, head_dim=32, context_len=64, ffn_hidden_dim=128)


@pytest.mark.parametrize("name", ["adamw", "muon"])
def test_optimizer_covers_every_parameter_and_steps(name):
    torch.manual_seed(0)
    m = build_model("TransformerPP", MODEL)
    args = dict(lr=1e-2, weight_decay=0.0) if name == "adamw" else dict(lr=2e-2, adamw=dict(lr=1e-2))
    opt = build_optimizer(name, m, args)
    x = torch.randint(0, 500, (2, 33))
    losses = []
    for _ in range(5):
        opt.zero_grad()
        logits = m(x[:, :-1])
        loss = torch.nn.functional.cross_entropy(logits.flatten(0, 1).float(), x[:, 1:].flatten())
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0]
    for g in opt.param_groups:
        assert "base_lr" in g


def _config(tmp_path, run, steps, **kw):
    data = tmp_path / "tok"
    if not data.exists():
        synthetic_store(data, tokens=60_000, vocab=500, seed=1)
    base = dict(run_name="t", data_dir=str(data), model_name="TransformerPP", model_args=MODEL,
                optimizer_name="muon", optimizer_args=dict(lr=2e-2, adamw=dict(lr=1e-2)),
                context_len=32, batch_size=2, grad_accum_steps=2, train_tokens=steps * 2 * 2 * 32,
                device="cpu", dtype="float32", compile=False, ce_impl="full", run_dir=str(tmp_path / run),
                log_interval=1, slow_interval=1000, deadline_margin_s=None, recent_ckpt_minutes=1e9)
    base.update(kw)
    return tm.TrainConfig(**base)


def test_train_checkpoints_and_exact_resume(tmp_path):
    run_a = tm.train(_config(tmp_path, "a", 6, permanent_ckpt_interval=3))
    assert (run_a / "ckpt-00000003.pt").exists() and (run_a / "ckpt-00000006.pt").exists()
    assert (run_a / "model-final.pt").exists() and (run_a / "config.yaml").exists()
    # resume a copy of the step-3 checkpoint and finish: same weights as the straight run
    run_b = tmp_path / "b"
    run_b.mkdir()
    shutil.copy(run_a / "ckpt-00000003.pt", run_b / "ckpt-00000003.pt")
    tm.train(_config(tmp_path, "b", 6, permanent_ckpt_interval=3))
    a = torch.load(run_a / "ckpt-00000006.pt", weights_only=False)
    b = torch.load(run_b / "ckpt-00000006.pt", weights_only=False)
    assert a["step"] == b["step"] == 6 and a["tokens_seen"] == b["tokens_seen"]
    for k in a["model"]:
        assert torch.equal(a["model"][k], b["model"][k]), k


def test_stop_request_checkpoints_and_exits(tmp_path, monkeypatch):
    calls = {"n": 0}
    real = tm.StepRunner.step

    def step(self, batches):
        calls["n"] += 1
        if calls["n"] == 2:
            tm.request_stop()
        return real(self, batches)

    monkeypatch.setattr(tm.StepRunner, "step", step)
    run = tm.train(_config(tmp_path, "s", 10))
    state = torch.load(run / "recent.pt", weights_only=False)
    assert state["step"] == 2
    assert not (run / "model-final.pt").exists()


def test_refuses_to_overwrite_a_run_without_checkpoints(tmp_path):
    (tmp_path / "x").mkdir()
    (tmp_path / "x" / "junk.txt").write_text("x")
    with pytest.raises(FileExistsError):
        tm.train(_config(tmp_path, "x", 2))


def test_from_yaml_with_model_recipe(tmp_path):
    (tmp_path / "m.yaml").write_text("model_name: TransformerPP\nmodel_args: {dim: 64}\n")
    (tmp_path / "t.yaml").write_text("model_recipe: m.yaml\nrun_name: r\ndata_dir: d\nbatch_size: 4\n")
    cfg = tm.TrainConfig.from_yaml(tmp_path / "t.yaml", ["batch_size=8"])
    assert cfg.model_args == {"dim": 64} and cfg.batch_size == 8
    with pytest.raises(TypeError):
        tm.TrainConfig.from_yaml(tmp_path / "t.yaml", ["nonsense_key=1"])


def test_registry_record(tmp_path):
    import json
    from vagus_b200.registry import write_record
    run = tm.train(_config(tmp_path, "r", 3))
    assert (run / "metrics.jsonl").exists()
    path = write_record(run, tmp_path / "registry", incidents=["none"], note="unit")
    rec = json.loads(path.read_text())
    assert set(rec) >= {"run", "recipe", "data", "results", "incidents", "archive"}
    assert rec["results"]["final_step"] == 3 and rec["results"]["loss_tail5"] is not None
    assert any(a["file"] == "model-final.pt" for a in rec["archive"])
    assert (run / "SHA256SUMS").read_text().count("\n") == len(rec["archive"])


def test_muon_exchange_eligibility_and_layout():
    """The fused Newton-Schulz scatter takes a bucket only when every rank can
    place its rows: even row split, dims multiples of 8, and for tall matrices
    (processed transposed, scattered by 32-column chunks) rows / world a
    multiple of 32; receive blocks are 256-byte aligned."""
    from vagus_b200.parallel.nvlink import MuonExchange
    cuda = torch.device("cuda")
    assert MuonExchange.eligible((1024, 1024), 8, cuda)
    assert MuonExchange.eligible((2816, 1024), 8, cuda)          # tall: 352 rows per rank
    assert not MuonExchange.eligible((4160, 1024), 8, cuda)      # tall: 520 rows per rank
    assert MuonExchange.eligible((1024, 2816), 8, cuda)          # wide: row blocks of 128
    assert not MuonExchange.eligible((1000, 1024), 16, cuda)     # uneven split
    assert not MuonExchange.eligible((1024, 1024), 1, cuda)      # nothing to exchange
    assert not MuonExchange.eligible((1024, 1024), 2, torch.device("cpu"))
    assert MuonExchange.block_bytes(4, 128, 1024) == 4 * 128 * 1024 * 2
    assert MuonExchange.block_bytes(3, 10, 10) % 256 == 0


def test_unreadable_recent_checkpoint_falls_back(tmp_path):
    """Failure injection on the host: a truncated recent.pt is reported and
    skipped; the run resumes from the newest readable checkpoint and finishes
    with the same weights as the uninterrupted run."""
    run_a = tm.train(_config(tmp_path, "a", 6, permanent_ckpt_interval=3))
    run_b = tmp_path / "b"
    run_b.mkdir()
    shutil.copy(run_a / "ckpt-00000003.pt", run_b / "ckpt-00000003.pt")
    good = (run_a / "ckpt-00000006.pt").read_bytes()
    (run_b / "recent.pt").write_bytes(good[: len(good) // 3])          # torn file
    tm.train(_config(tmp_path, "b", 6, permanent_ckpt_interval=3))
    a = torch.load(run_a / "ckpt-00000006.pt", weights_only=False)
    b = torch.load(run_b / "ckpt-00000006.pt", weights_only=False)
    for k in a["model"]:
        assert torch.equal(a["model"][k], b["model"][k]), k


def test_walltime_deadline_stops_with_checkpoint(tmp_path, monkeypatch):
    """Failure injection on the host: a job end time already inside the
    deadline margin stops the run after its first step, by rank consensus,
    with the recent checkpoint written and no final model."""
    import time
    monkeypatch.setenv("SLURM_JOB_END_TIME", str(time.time() + 5.0))
    run = tm.train(_config(tmp_path, "d", 10, deadline_margin_s=60.0))
    state = torch.load(run / "recent.pt", weights_only=False)
    assert state["step"] == 1
    assert not (run / "model-final.pt").exists()


def _dead_rank_worker(rank, port, q):
    import datetime
    import os
    import time
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=10))
    t = torch.ones(4)
    dist.all_reduce(t)                       # one healthy step
    def report(msg):
        q.put((rank, msg))
        q.close()
        q.join_thread()                      # flushed before the hard exit below

    if rank == 1:
        report("left")
        os._exit(0)                          # this rank dies between steps, without a goodbye
    t0 = time.time()
    try:
        dist.all_reduce(t)
        report("no error")
    except Exception as e:                   # noqa: BLE001 -- the failure this test injects
        report(f"detected after {time.time() - t0:.1f}s: {type(e).__name__}")
    os._exit(0)


def test_dead_rank_is_detected_by_the_next_collective():
    """Failure injection among CPU ranks: a gloo rank that exits between
    steps makes the survivor's next collective fail with an error (within the
    process-group timeout) instead of hanging."""
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert out[1] == "left"
    assert out[0].startswith("detected"), out[0]


def test_collective_dry_run_switch():
    """The exposed-communication probe's switch: while on, the FSDP2 hooks
    return before touching their heap (None here) or any process group."""
    from vagus_b200.parallel import nvlink
    ag, rs = nvlink.NvlinkAllGather(None), nvlink.NvlinkReduceScatter(None)
    nvlink.set_dry_run(True)
    try:
        assert ag(torch.empty(4), torch.empty(2), None) is None
        assert rs(torch.empty(2), torch.empty(4), None, None) is None
    finally:
        nvlink.set_dry_run(False)
    with pytest.raises(AttributeError):
        ag(torch.empty(4), torch.empty(2), None)          # off again: the real path needs a heap
