"""The meter examples and checkpoint probes run end to end on tiny models
(CPU): probe reports are well formed and agree with direct computation."""

import json
import math
import os
import socket
import subprocess
import sys

import pytest
import torch

from vagus_b200.data.prepare import synthetic_store
from vagus_b200.meter.examples import (bench_attention, bench_ce, bench_linear_attention, bench_rope,
                                       probe_attention_health, profile_step, saturation_curve, write_selectivity)
from vagus_b200.meter.examples._common import parse_ckpts
from vagus_b200.models import build_model

ARGS = dict(vocab_size=101, dim=64, layer_count=3, head_count=2, key_head_dim=16, value_head_dim=32, gate_rank=8,
            chunk_size=8, la_impl="torch", context_len=48, layer_pattern="gdn,gdn,softmax", softmax_head_dim=16,
            softmax_out_gate=True)


def _model(**over):
    torch.manual_seed(0)
    return build_model("GDNLM", {**ARGS, **over}).eval()


def _tokens(n=2, L=32):
    g = torch.Generator().manual_seed(1)
    return [torch.randint(0, 101, (2, L), generator=g) for _ in range(n)]


def test_parse_ckpts():
    assert parse_ckpts(["A=x.pt", "y.pt"]) == {"A": "x.pt", "m1": "y.pt"}


def test_saturation_curve_matches_layer_residuals():
    m, toks = _model(), _tokens()
    r = saturation_curve.probe(m, toks)
    assert r["key_dim"] == 16 and r["positions"][0] == 1 and r["positions"][-1] == 32
    assert len(r["layers"]) == 2 and 1 <= r["knee"] <= 32
    # position 1 from a blank state: nothing stored, rho = 1 exactly
    assert abs(r["rho"][0] - 1.0) < 1e-5
    direct = m.blocks[0].att.residuals(m.blocks[0].rmsnorm1(m.embedding(toks[0])))
    assert direct.shape == (2, 32, 2)
    assert "knee" in saturation_curve.render(r)


def test_write_selectivity_report():
    r = write_selectivity.probe(_model(), _tokens())
    assert r["tokens"] == 2 * 2 * 32 * 2 * 2                 # batches x B x L x H x delta layers
    assert -1.0 <= r["corr_w_rho"] <= 1.0 and r["write_gain"] > 0
    c = r["concentration"]
    assert 0.01 <= c["top1%"] <= c["top5%"] <= c["top10%"] <= c["top25%"] <= 1.0
    assert 0.0 < r["w_mean"] <= 1.0                          # |w| = beta for unit keys
    assert "write gain" in write_selectivity.render(r)


def test_write_selectivity_kalman_write():
    r = write_selectivity.probe(_model(write="kalman_iso", gate="vector"), _tokens(1))
    assert math.isfinite(r["corr_w_rho"]) and r["write_gain"] > 0


def test_attention_health_matches_max_logit():
    m, toks = _model(), _tokens(1)
    r = probe_attention_health.probe(m, toks)
    layer = r["layer2"]
    assert len(layer["gap"]) == 4 and all(g >= 0 for g in layer["gap"])
    assert all(0 <= s <= 1 for s in layer["sink"]) and 0 <= layer["gate_open"] <= 1
    x = m.embedding(toks[0])
    for blk in m.blocks[:2]:
        x = blk(x)
    want = float(m.blocks[2].att.max_attn_logit(m.blocks[2].rmsnorm1(x)))
    assert abs(r["attn_logit_max"] - want) < 1e-4
    if "ceiling" in layer:
        assert layer["max_cos"] <= 1.0 + 1e-5
    assert "entropy" in probe_attention_health.render(r)


def test_probes_without_their_layers_raise():
    with pytest.raises(ValueError):
        probe_attention_health.probe(_model(layer_pattern="gdn"), _tokens(1))


def test_probe_cli_on_a_checkpoint(tmp_path):
    synthetic_store(tmp_path / "tok", tokens=5_000, vocab=101, seed=3, shards=1, doc_len=97, bos=1)
    m = _model()
    torch.save({"model_name": "GDNLM", "model_args": ARGS, "model": m.state_dict()}, tmp_path / "m.pt")
    out = tmp_path / "r.json"
    res = saturation_curve.main(["--ckpt", f"A={tmp_path / 'm.pt'}", "--data", str(tmp_path / "tok"),
                                 "--context-len", "32", "--batch", "2", "--batches", "1", "--device", "cpu",
                                 "--json", str(out)])
    assert json.loads(out.read_text())["A"]["knee"] == res["A"]["knee"]


def test_benchmarks_run_on_cpu(capsys):
    bench_attention.main(["--B", "1", "--H", "2", "--L", "32", "--dh", "16", "--iters", "2"])
    bench_ce.main(["--T", "64", "--D", "32", "--V", "50", "--iters", "2"])
    bench_rope.main(["--B", "1", "--L", "16", "--H", "2", "--dh", "16", "--iters", "2"])
    bench_linear_attention.main(["--B", "1", "--L", "64", "--H", "2", "--dk", "16", "--dv", "16", "--iters", "1",
                                 "--modes", "kda", "gla", "deltanet"])
    r = bench_linear_attention.main(["--decode", "--B", "1", "--H", "2", "--dk", "16", "--dv", "16", "--prefill", "16",
                                     "--steps", "3", "--iters", "1", "--modes", "gdn", "kda"])
    assert set(r) == {"gdn/torch", "kda/torch"} and all(v["decode_ms_per_token"] > 0 for v in r.values())
    r = bench_attention.main(["--decode", "--B", "1", "--H", "2", "--dh", "16", "--prefill", "16", "--steps", "3",
                              "--iters", "1", "--kv-heads", "1"])
    assert r["d16"]["prefill_ms"] > 0
    out = capsys.readouterr().out
    assert "FAILED" not in out and "sdpa" in out and "fused" in out and "us/token" in out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_bench_dist_gloo_two_ranks():
    env = {**os.environ, "CUDA_VISIBLE_DEVICES": ""}
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "-m", "vagus_b200.meter.examples.bench_dist", "--mib", "0.0625", "--iters", "2", "--dtype", "float32"]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert p.returncode == 0, p.stderr[-2000:]
    assert "nccl all-gather" in p.stdout and "bus GB/s" in p.stdout


def test_profile_step_on_cpu(tmp_path):
    args = dict(ARGS, layer_pattern="gdn,softmax", layer_count=2)
    r = profile_step.main(["--args", json.dumps(args), "--batch", "2", "--seq", "32", "--steps", "1", "--warmup", "1",
                           "--out", str(tmp_path)])
    assert any(p.endswith(".trace.json") for p in r["traces"].values())
    assert profile_step.family("gemm_kernel<256, false, false>") == "gemm"
    assert profile_step.family("gdr_bwd_scan_tc<256>") == "delta-rule"


def test_compare_agreement_is_leafwise():
    from vagus_b200.meter.compare import agreement, compare
    a = (torch.ones(3), {"s": torch.zeros(2)})
    b = (torch.ones(3) * 1.5, {"s": torch.zeros(2)})
    ag = agreement(b, a)
    assert ag.leaves == 2 and abs(ag.max_abs - 0.5) < 1e-12 and abs(ag.max_rel - 0.5) < 1e-12
    assert agreement((torch.ones(3),), a).max_abs == float("inf")          # structure differs
    assert agreement(torch.ones(2), torch.ones(3)).max_rel == float("inf")  # shape differs
    x = torch.randn(64, 64)
    res = compare({"mm": lambda t: t @ t, "mm2": lambda t: (t @ t) * (1 + 1e-3)}, (x,), warmup=1, iters=3,
                  verbose=False)
    assert res["mm"].vs_ref is None and 5e-4 < res["mm2"].vs_ref.max_rel < 2e-3
    assert len(res["mm"].samples) == 3


def test_dist_job_time_is_the_slowest_rank_per_iteration():
    from vagus_b200.meter.core import BenchResult
    from vagus_b200.meter.dist import job_time, render_dist_table

    def r(s):
        return BenchResult("f", "cpu", len(s), sum(s) / len(s), 0.0, min(s), max(s), 0.0, None, False, samples=s)
    res = {0: r([1.0, 5.0, 1.0]), 1: r([4.0, 1.0, 1.0])}
    assert job_time(res) == (4.0 + 5.0 + 1.0) / 3
    assert "job step" in render_dist_table(res)
