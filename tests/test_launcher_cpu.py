"""The SLURM per-node launcher (recipe/slurm/torchrun_node.sh) run the way
srun runs it, with the SLURM variables set by hand: torchrun starts two CPU
workers on gloo that train a tiny recipe to completion (final model written)."""

import os
import socket
import subprocess
from pathlib import Path

import yaml

from vagus_b200.data.prepare import synthetic_store

ROOT = Path(__file__).resolve().parents[1]
MODEL = dict(vocab_size=300, dim=64, layer_count=2, head_dim=32, context_len=64, ffn_hidden_dim=128)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_torchrun_node_launcher_trains_a_tiny_recipe(tmp_path):
    synthetic_store(tmp_path / "tok", tokens=40_000, vocab=300, seed=1)
    recipe = dict(run_name="launch", data_dir=str(tmp_path / "tok"), model_name="TransformerPP", model_args=MODEL,
                  optimizer_name="adamw", optimizer_args=dict(lr=1e-3), context_len=32, batch_size=2,
                  grad_accum_steps=1, train_tokens=4 * 2 * 2 * 32, world_size=2, shard_size=1, device="cpu",
                  dtype="float32", compile=False, ce_impl="full", run_dir=str(tmp_path / "run"), log_interval=1,
                  slow_interval=1000, deadline_margin_s=None, recent_ckpt_minutes=1e9)
    path = tmp_path / "tiny.yaml"
    path.write_text(yaml.safe_dump(recipe))
    env = {**os.environ, "VAGUS_B200_HOME": str(ROOT), "SLURM_NNODES": "1", "GPUS_PER_NODE": "2", "SLURM_NODEID": "0",
           "SLURM_JOB_ID": "cpu-test", "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_port()),
           "CUDA_VISIBLE_DEVICES": ""}
    p = subprocess.run(["bash", str(ROOT / "recipe" / "slurm" / "torchrun_node.sh"), str(path)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, (p.stdout[-2000:], p.stderr[-3000:])
    assert (tmp_path / "run" / "model-final.pt").exists()


def test_sigusr1_through_the_launcher_stops_with_a_checkpoint(tmp_path):
    """The walltime path: SIGUSR1 to the node launcher (what srun relays from
    the batch script's trap) reaches both workers through torchrun; they stop
    at a step boundary with a recent checkpoint before the planned end (no
    final model).  torchrun itself exits non-zero after a forwarded signal;
    the batch script tolerates that and re-queues the run."""
    import signal
    import time
    synthetic_store(tmp_path / "tok", tokens=200_000, vocab=300, seed=1)
    recipe = dict(run_name="walltime", data_dir=str(tmp_path / "tok"), model_name="TransformerPP",
                  model_args=MODEL, optimizer_name="adamw", optimizer_args=dict(lr=1e-3), context_len=32,
                  batch_size=2, grad_accum_steps=1, train_tokens=100_000 * 2 * 2 * 32, world_size=2, shard_size=1,
                  device="cpu", dtype="float32", compile=False, ce_impl="full", run_dir=str(tmp_path / "run"),
                  log_interval=1, slow_interval=100_000, deadline_margin_s=None, recent_ckpt_minutes=1e9)
    path = tmp_path / "long.yaml"
    path.write_text(yaml.safe_dump(recipe))
    env = {**os.environ, "VAGUS_B200_HOME": str(ROOT), "SLURM_NNODES": "1", "GPUS_PER_NODE": "2", "SLURM_NODEID": "0",
           "SLURM_JOB_ID": "cpu-test", "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_port()),
           "CUDA_VISIBLE_DEVICES": ""}
    proc = subprocess.Popen(["bash", str(ROOT / "recipe" / "slurm" / "torchrun_node.sh"), str(path)], env=env,
                            stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    metrics = tmp_path / "run" / "metrics.jsonl"
    try:
        t0 = time.time()
        while time.time() - t0 < 300:
            if metrics.exists() and len(metrics.read_text().splitlines()) >= 3:
                break
            if proc.poll() is not None:
                break
            time.sleep(0.5)
        assert proc.poll() is None, "the run ended before the signal"
        proc.send_signal(signal.SIGUSR1)           # bash exec'd torchrun: this is the agent's pid
        out, err = proc.communicate(timeout=300)
    finally:
        if proc.poll() is None:
            proc.kill()
    assert "stop signal received" in out and "final recent checkpoint" in out, (out[-2000:], err[-3000:])
    assert (tmp_path / "run" / "recent.pt").exists()
    assert not (tmp_path / "run" / "model-final.pt").exists()
    # the re-queued job: same recipe, resumes from recent.pt and finishes (a
    # shorter token budget here so it ends quickly)
    import torch
    done = torch.load(tmp_path / "run" / "recent.pt", weights_only=False)["step"]
    env["MASTER_PORT"] = str(_port())
    p = subprocess.run(["bash", str(ROOT / "recipe" / "slurm" / "torchrun_node.sh"), str(path),
                        f"train_tokens={(done + 2) * 2 * 2 * 32}"], env=env, capture_output=True, text=True,
                       timeout=600)
    assert p.returncode == 0, (p.stdout[-2000:], p.stderr[-3000:])
    assert f"resumed from recent.pt at step {done:,}" in p.stdout, p.stdout[-2000:]
    assert torch.load(tmp_path / "run" / "model-final.pt", weights_only=False)["step"] == done + 2


def test_chain_guard_finds_the_run_of_a_recipe_without_run_dir(tmp_path):
    """The batch script re-queues until <run>/model-final.pt exists; for a
    recipe that leaves run_dir unset it must look where train() writes
    (out_root/<run_name>-<commit8>), so its snippet runs the same resolver."""
    import re
    import sys
    from vagus_b200.train import main as tm
    synthetic_store(tmp_path / "tok", tokens=40_000, vocab=300, seed=1)
    recipe = dict(run_name="guard", data_dir=str(tmp_path / "tok"), model_name="TransformerPP", model_args=MODEL,
                  optimizer_name="adamw", optimizer_args=dict(lr=1e-3), context_len=32, batch_size=2,
                  train_tokens=2 * 2 * 32, device="cpu", dtype="float32", compile=False, ce_impl="full",
                  out_root=str(tmp_path / "runs"), log_interval=1, slow_interval=1000, deadline_margin_s=None)
    path = tmp_path / "guard.yaml"
    path.write_text(yaml.safe_dump(recipe))
    run = tm.train(tm.TrainConfig.from_yaml(str(path)))
    assert (run / "model-final.pt").exists()
    sbatch = (ROOT / "recipe" / "slurm" / "b200_train.sbatch").read_text()
    snippet = re.search(r"<<'PY'\n(.*?)\nPY\n", sbatch, re.S).group(1)
    p = subprocess.run([sys.executable, "-", str(path)], input=snippet, capture_output=True, text=True, timeout=120,
                       cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    assert Path(p.stdout.strip()) == run
