"""Two-GPU training under FSDP2 with the NVLink collectives, through the
public ``train()`` entry point, and the collectives under host skew.

* Rank 0 sleeps 5 s on the host before an all-gather and a reduce-scatter
  (longer than any wait inside one CTA is allowed to take): the results still
  equal NCCL's and the device error word stays 0 -- the cross-GPU waits are
  bounded by the process group's timeout, not by the kernels' own 2 s.
* ``train()`` writes a recent checkpoint mid-run whose write on rank 0 takes
  5 s (the other rank waits at the host barrier after the write instead of
  racing into the next step's collectives), writes a permanent checkpoint at
  step 3, finishes, and a second run resumed from that checkpoint ends where
  the straight run ended.  The weight-gradient GEMMs accumulate with atomics,
  so runs agree to a tolerance, not bit for bit: the resumed run must sit as
  close to the straight run as a second straight run does.

Reference behaviour: ``infra/train/main.py:714-723`` (rank 0 writes, NCCL
waits for it)."""

import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

MODEL = dict(vocab_size=4096, dim=256, layer_count=2, head_count=2, key_head_dim=128, value_head_dim=128,
             ffn_hidden_dim=704, gate="scalar", chunk_size=64, context_len=256)
WORLD = 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _env(rank, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")


def _skew_worker(rank, port, q):
    try:
        _env(rank, port)
        from vagus_b200.parallel import setup_distributed
        setup_distributed("auto", timeout_s=120)
        import torch.distributed as dist
        from vagus_b200 import ops
        from vagus_b200.parallel.nvlink import NvlinkAllGather, NvlinkHeap, NvlinkReduceScatter
        heap = NvlinkHeap(dist.group.WORLD, ag_cap=1 << 20, rs_cap=4 << 20)
        ag, rs = NvlinkAllGather(heap), NvlinkReduceScatter(heap)
        errs = []
        n = 4099
        g = torch.Generator(device="cuda").manual_seed(rank)
        shard = torch.randn(n, device="cuda", generator=g).bfloat16()
        full = torch.randn(WORLD * n, device="cuda", generator=g)
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            time.sleep(5.0)                    # host skew: the peer's kernels wait on the GPU meanwhile
        out = torch.empty(WORLD * n, device="cuda", dtype=torch.bfloat16)
        out[rank * n:(rank + 1) * n].copy_(shard)
        ag(out, out[rank * n:(rank + 1) * n], dist.group.WORLD)
        o = torch.empty(n, device="cuda")
        rs(o, full, dist.group.WORLD, dist.ReduceOp.AVG)
        torch.cuda.synchronize()
        ref = torch.empty_like(out)
        dist.all_gather_into_tensor(ref, shard)
        r = torch.empty(n, device="cuda")
        dist.reduce_scatter_tensor(r, full.clone(), op=dist.ReduceOp.AVG)
        errs.append(("ag", (out.float() - ref.float()).abs().max().item()))
        errs.append(("rs", (o - r).abs().max().item()))
        errs.append(("error_word", float(ops.native().error_word())))
        heap.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


def _run(target, args, timeout=600):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, *args, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=timeout) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    for rank, res in results.items():
        assert not isinstance(res, str), f"rank {rank}: {res}"
    return results


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nvlink_collectives_survive_host_skew():
    results = _run(_skew_worker, (_port(),))
    for rank, errs in results.items():
        for kind, e in errs:
            tol = 1e-5 if kind == "rs" else 0.0
            assert e <= tol, (rank, kind, e)


def _train_cfg(tmp, run, steps, recent_minutes):
    from vagus_b200.train import main as tm
    return tm.TrainConfig(run_name="g", data_dir=os.path.join(tmp, "tok"), model_name="GDNLM", model_args=MODEL,
                          optimizer_name="muon", optimizer_args=dict(lr=2e-3, adamw=dict(lr=1e-3)),
                          context_len=256, batch_size=2, grad_accum_steps=2,
                          train_tokens=steps * WORLD * 2 * 2 * 256, world_size=WORLD, shard_size=WORLD,
                          device="auto", dtype="bfloat16", fsdp_comm="nvlink", compile=False, ce_impl="fused",
                          run_dir=os.path.join(tmp, run), log_interval=1, slow_interval=1000,
                          deadline_margin_s=None, recent_ckpt_minutes=recent_minutes, permanent_ckpt_interval=3)


def _train_worker(rank, port, tmp, q):
    try:
        _env(rank, port)
        from vagus_b200.parallel import setup_distributed
        setup_distributed("auto", timeout_s=300)
        import shutil

        import torch.distributed as dist
        from vagus_b200 import ops
        from vagus_b200.train import main as tm
        real_write = tm._write_checkpoint
        slow = {"left": 1}

        def slow_write(*a, **k):               # rank 0's first recent write takes 5 s
            if a[1] == "recent" and slow["left"]:
                slow["left"] -= 1
                time.sleep(5.0)
            return real_write(*a, **k)

        tm._write_checkpoint = slow_write
        tm.train(_train_cfg(tmp, "a", 6, recent_minutes=0.0), teardown=False)
        tm.train(_train_cfg(tmp, "a2", 6, recent_minutes=1e9), teardown=False)
        if rank == 0:
            os.makedirs(os.path.join(tmp, "b"))
            shutil.copy(os.path.join(tmp, "a", "ckpt-00000003.pt"), os.path.join(tmp, "b", "ckpt-00000003.pt"))
        dist.barrier()
        tm.train(_train_cfg(tmp, "b", 6, recent_minutes=1e9), teardown=False)
        if rank == 0:
            os.makedirs(os.path.join(tmp, "c"))
            shutil.copy(os.path.join(tmp, "a", "ckpt-00000003.pt"), os.path.join(tmp, "c", "ckpt-00000003.pt"))
        dist.barrier()
        # resume at step 3 with nothing left to train: the final checkpoint is the loaded state, saved again
        tm.train(_train_cfg(tmp, "c", 3, recent_minutes=1e9), teardown=False)
        torch.cuda.synchronize()
        word = ops.native().error_word()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, {"error_word": word, "slow_write_done": slow["left"] == 0}))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_train_nvlink_fsdp_slow_checkpoint_and_resume(tmp_path):
    from vagus_b200.data.prepare import synthetic_store
    synthetic_store(tmp_path / "tok", tokens=200_000, vocab=4096, seed=1)
    results = _run(_train_worker, (_port(), str(tmp_path)), timeout=900)
    for rank, res in results.items():
        assert res["error_word"] == 0, (rank, res)
    assert results[0]["slow_write_done"]
    assert (tmp_path / "a" / "recent.pt").exists()
    # load + save round trip: model and optimizer state bit for bit
    a3 = torch.load(tmp_path / "a" / "ckpt-00000003.pt", weights_only=False)
    c3 = torch.load(tmp_path / "c" / "ckpt-00000003.pt", weights_only=False)
    for k in a3["model"]:
        assert torch.equal(a3["model"][k], c3["model"][k]), ("round trip model", k)
    flat = lambda sd: {f"{k}/{n}": t for k, st in sd["optimizer"]["state"].items()   # noqa: E731
                       for n, t in st.items() if torch.is_tensor(t)}
    fa, fc = flat(a3), flat(c3)
    assert fa.keys() == fc.keys() and len(fa) > 0, ("round trip optimizer keys", sorted(fa)[:4], sorted(fc)[:4])
    for k in fa:
        assert torch.equal(fa[k], fc[k]), ("round trip optimizer", k)
    a = torch.load(tmp_path / "a" / "ckpt-00000006.pt", weights_only=False)
    a2 = torch.load(tmp_path / "a2" / "ckpt-00000006.pt", weights_only=False)
    b = torch.load(tmp_path / "b" / "ckpt-00000006.pt", weights_only=False)
    assert a["step"] == b["step"] == 6 and a["tokens_seen"] == b["tokens_seen"]
    for k in a["model"]:
        # the resumed run is as close to the straight run as a second straight run is
        x, x2, y = (t["model"][k].float() for t in (a, a2, b))
        noise = (x - x2).norm().item()
        assert (x - y).norm() <= 3 * noise + 1e-3 * max(1e-3, x.norm().item()), \
            (k, (x - y).norm().item(), (x2 - y).norm().item(), noise, _losses(tmp_path))


def _losses(tmp):
    """Per-step training loss of each run (diagnostic for a failed comparison)."""
    import json
    out = {}
    for run in ("a", "a2", "b"):
        f = tmp / run / "metrics.jsonl"
        if f.exists():
            rows = [json.loads(line) for line in f.read_text().splitlines() if line.strip()]
            out[run] = [(r.get("step"), r.get("loss")) for r in rows if "loss" in r]
    return out
