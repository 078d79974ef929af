"""The command-line pipeline a user runs, each step through its own argument
parser in a fresh process (CPU): synthetic token store -> train a recipe
with a key=value override -> evaluate the run -> write its registry record."""

import json
import subprocess
import sys
from pathlib import Path

import yaml

ROOT = Path(__file__).resolve().parents[1]


def _py(*args, cwd):
    p = subprocess.run([sys.executable, *args], capture_output=True, text=True, timeout=600, cwd=cwd,
                       env={"PATH": "/usr/bin:/bin", "CUDA_VISIBLE_DEVICES": "", "PYTHONPATH": str(ROOT),
                            "HOME": str(cwd)})
    assert p.returncode == 0, (args, p.stdout[-2000:], p.stderr[-3000:])
    return p.stdout


def test_data_train_eval_registry_clis(tmp_path):
    _py("-m", "vagus_b200.data", "synthetic", str(tmp_path / "tok"), "--tokens", "40000", "--vocab", "400",
        cwd=tmp_path)
    model = dict(vocab_size=400, dim=64, layer_count=2, head_count=2, key_head_dim=32, value_head_dim=32,
                 ffn_hidden_dim=128, context_len=128, gate="scalar", delta=True, chunk_size=16)
    train = dict(run_name="cli", data_dir=str(tmp_path / "tok"), model_name="GDNLM", model_args=model,
                 optimizer_name="muon", optimizer_args=dict(lr=2e-2, adamw=dict(lr=3e-3)), context_len=64,
                 batch_size=2, train_tokens=3 * 2 * 64, device="cpu", dtype="float32", compile=False,
                 ce_impl="full", run_dir=str(tmp_path / "run"), log_interval=1, slow_interval=1000,
                 deadline_margin_s=None)
    (tmp_path / "train.yaml").write_text(yaml.safe_dump(train))
    _py("-m", "vagus_b200.train.main", str(tmp_path / "train.yaml"), "train_tokens=512", cwd=tmp_path)
    run = tmp_path / "run"
    assert (run / "model-final.pt").exists() and (run / "metrics.jsonl").exists()
    steps = [json.loads(l) for l in (run / "metrics.jsonl").read_text().splitlines() if l.strip()]
    assert max(s.get("step", 0) for s in steps) == 4          # the override: 512 tokens / 128 per step
    ev = dict(eval_name="cli-eval", device="cpu", dtype="float32", run_dir=str(tmp_path / "eval"),
              registry_dir=str(tmp_path / "registry" / "eval"), n_boot=50,
              subjects=[{"run": str(run), "label": "m", "tokenizer_id": "mistral32k"}],
              tasks=[{"name": "holdout", "args": {"data_dir": str(tmp_path / "tok"), "n_seq": 2, "context_len": [64]}}])
    (tmp_path / "eval.yaml").write_text(yaml.safe_dump(ev))
    _py("-m", "vagus_b200.eval.main", str(tmp_path / "eval.yaml"), cwd=tmp_path)
    assert any((tmp_path / "eval").iterdir())
    out = _py("-m", "vagus_b200.registry", str(run), "--out", str(tmp_path / "registry"), "--note", "cli test",
              cwd=tmp_path)
    assert str(tmp_path / "registry") in out
