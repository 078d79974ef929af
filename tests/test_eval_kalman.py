"""Kalman-delta scans (fp64 oracles) and the evaluation harness end to end
on a tiny checkpoint trained here (record layout, determinism, pairing)."""

import json

import pytest
import torch

from vagus_b200.eval.main import EvalConfig, evaluate
from vagus_b200.eval.pairs import paired
from vagus_b200.models.kalman import kalman_gain_diag, kalman_gain_iso, mobius_scan

@pytest.fixture(autouse=True)
def _fp64_default(request):
    """fp64 default dtype for the scan oracles of this module only (restored
    after each test, so modules collected after this one keep fp32)."""
    prev = torch.get_default_dtype()
    if "trained" not in request.fixturenames:
        torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(prev)


def _pos(*shape):
    return torch.rand(*shape) + 0.1


def test_mobius_parallel_and_blocked_match_recurrent():
    torch.manual_seed(0)
    B, L, H = 2, 300, 3
    A, Bq, C, D = _pos(B, L, H), _pos(B, L, H), _pos(B, L, H), _pos(B, L, H)
    x0 = _pos(B, H)
    ref = mobius_scan(A, Bq, C, D, x0, impl="recurrent")
    par = mobius_scan(A, Bq, C, D, x0, impl="parallel", block=None)
    blk = mobius_scan(A, Bq, C, D, x0, impl="parallel", block=64)
    assert torch.allclose(par, ref, rtol=1e-10, atol=1e-12)
    assert torch.allclose(blk, ref, rtol=1e-10, atol=1e-12)
    long = mobius_scan(_pos(1, 1024, 1), _pos(1, 1024, 1), _pos(1, 1024, 1), _pos(1, 1024, 1), _pos(1, 1),
                       impl="parallel", block=None)
    assert torch.isfinite(long).all()


def test_iso_gain_matches_hand_recurrence():
    torch.manual_seed(1)
    B, L, H, dk = 1, 20, 2, 8
    k = torch.randn(B, L, H, dk)
    alpha = torch.rand(B, L, H, dk) * 0.5 + 0.5
    omega, r = _pos(B, L, H), _pos(B, L, H)
    c0 = _pos(B, H)
    beta, c_fin = kalman_gain_iso(k, alpha, omega, r, c0, info_scale=1.0)
    # precision c, prior variance bhat = a / c_prev + omega, gain = bhat / (r + bhat |k|^2)
    c = c0.clone()
    for t in range(L):
        a = alpha[:, t].square().mean(-1)
        kn2 = k[:, t].square().sum(-1)
        bhat = a / c + omega[:, t]
        assert torch.allclose(beta[:, t], bhat / (r[:, t] + bhat * kn2), rtol=1e-10)
        m = kn2 / dk / r[:, t]
        c = ((1 + m * omega[:, t]) * c + m * a) / (omega[:, t] * c + a)
    assert torch.allclose(c_fin, c, rtol=1e-10)


def test_diag_gain_shapes_and_positivity():
    torch.manual_seed(2)
    B, L, H, dk = 1, 12, 2, 4
    k = torch.randn(B, L, H, dk)
    alpha = torch.rand(B, L, H, dk) * 0.5 + 0.5
    kappa, p = kalman_gain_diag(k, alpha, _pos(B, L, H, dk), _pos(B, L, H), _pos(B, H, dk), info_scale=1.0)
    assert kappa.shape == (B, L, H, dk) and p.shape == (B, H, dk) and (p > 0).all()


def test_paired_statistics():
    a = [1.0, 2.0, 3.0, 4.0]
    b = [1.5, 2.5, 3.5, 4.5]
    r = paired(a, b, n_boot=200, seed=0)
    assert r["mean_diff"] == pytest.approx(0.5)
    assert r["frac_positive"] == pytest.approx(1.0) and r["n"] == 4
    assert r["ci95"][0] <= 0.5 <= r["ci95"][1]


@pytest.fixture(scope="module")
def trained(tmp_path_factory):
    torch.set_default_dtype(torch.float32)
    from vagus_b200.data.prepare import synthetic_store
    from vagus_b200.train import main as tm
    root = tmp_path_factory.mktemp("ev")
    data = root / "tok"
    synthetic_store(data, tokens=40_000, vocab=400, seed=4, doc_len=200, bos=1)
    model = dict(vocab_size=400, dim=64, layer_count=2, head_count=2, key_head_dim=32, value_head_dim=32,
                 ffn_hidden_dim=128, context_len=128, gate="scalar", delta=True, chunk_size=16)
    cfg = tm.TrainConfig(run_name="e", data_dir=str(data), model_name="GDNLM", model_args=model,
                         optimizer_name="adamw", optimizer_args=dict(lr=3e-3), context_len=64, batch_size=2,
                         train_tokens=4 * 2 * 64, device="cpu", dtype="float32", compile=False, ce_impl="full",
                         run_dir=str(root / "run"), log_interval=1, slow_interval=1000, deadline_margin_s=None)
    run = tm.train(cfg)
    return root, data, run


def _eval(root, data, run, name):
    tasks = [{"name": "holdout", "args": {"data_dir": str(data), "n_seq": 3, "context_len": [64]}}]
    subj = [{"run": str(run), "label": lab, "tokenizer_id": "mistral32k"} for lab in ("a", "b")]
    cfg = EvalConfig(eval_name=name, subjects=subj,
                     tasks=tasks, device="cpu", dtype="float32", run_dir=str(root / name),
                     registry_dir=str(root / "registry"), n_boot=50)
    return evaluate(cfg)


def test_eval_record_and_determinism(trained):
    torch.set_default_dtype(torch.float32)
    root, data, run = trained
    d1 = _eval(root, data, run, "e1")
    d2 = _eval(root, data, run, "e2")
    r1 = json.loads((d1 / "results.json").read_text())
    r2 = json.loads((d2 / "results.json").read_text())
    assert set(r1["holdout"]["subjects"]) == {"a", "b"}
    assert r1["holdout"]["subjects"]["a"]["items"] == r2["holdout"]["subjects"]["a"]["items"]
    assert "b" in r1["holdout"]["pairs"]
    meta = json.loads((d1 / "meta.json").read_text())
    assert meta["reference"] == "a" and len(meta["subjects"]) == 2
    assert (root / "registry" / "e1.json").exists()
    with pytest.raises(Exception):
        _eval(root, data, run, "e1")          # refuses to overwrite an existing record


def test_every_eval_recipe_loads_and_validates():
    """Each shipped eval recipe parses into an EvalConfig whose tasks are
    registered and accept the recipe's arguments (the reference's own eval
    recipes use the same schema and load the same way)."""
    from pathlib import Path
    recipes = sorted((Path(__file__).resolve().parent.parent / "recipe" / "eval").glob("*.yaml"))
    assert len(recipes) >= 7
    for path in recipes:
        cfg = EvalConfig.from_yaml(path)
        cfg.validate()
        assert cfg.subjects and cfg.tasks, path.name
    bad = EvalConfig(eval_name="x", subjects=["a.pt"], tasks=[{"name": "holdout", "args": {"nope": 1}}])
    with pytest.raises(TypeError):
        bad.validate()


def test_draw_pattern_is_the_documented_one(trained):
    """Draws consumes the generator exactly as documented: a token-weighted
    shard by rng.choice(p=...), then rng.integers(0, shard - length - slack);
    a document draw weights shards by their documents."""
    import numpy as np
    from vagus_b200.eval.core import Draws, open_store
    _, data, _ = trained
    store = open_store(data)
    d = Draws(store, np.random.default_rng(7))
    got = [d.window(64, slack=1) for _ in range(5)]
    r = np.random.default_rng(7)
    w = np.asarray(store.shard_tokens, dtype=np.float64)
    w /= w.sum()
    want = []
    for _ in range(5):
        s = int(r.choice(len(w), p=w))
        want.append((s, int(r.integers(0, store.shard_tokens[s] - 64 - 1))))
    assert got == want
    s, i, doc = Draws(store, np.random.default_rng(3)).document(10)
    assert len(doc) >= 10 and np.array_equal(doc, store.doc(s, i))


def test_generation_recall_and_saturation_tasks_run(trained):
    """The other three tasks end to end on the tiny trained subject: records
    have the documented items, and a second run draws the same items."""
    root, data, run = trained
    tasks = [{"name": "degeneration", "args": {"data_dir": str(data), "n_prompts": 3, "prompt_tokens": 8,
                                               "new_tokens": 12, "seeds": 2, "batch_size": 2}},
             {"name": "recall_probe", "args": {"data_dir": str(data), "lengths": [64], "kv_pairs": [4], "n": 3,
                                               "pool": [10, 390], "seps": [5, 6], "batch_size": 2}},
             {"name": "saturation", "args": {"data_dir": str(data), "n_seqs": 2, "length": 96, "batch_size": 2,
                                             "tail_from": 64, "edges": [1, 8, 32], "marks": [16, 48]}}]
    outs = []
    for name in ("t1", "t2"):
        cfg = EvalConfig(eval_name=name, subjects=[{"run": str(run), "label": "a", "tokenizer_id": "mistral32k"}],
                         tasks=tasks, device="cpu", dtype="float32", run_dir=str(root / name), registry_dir=None)
        outs.append(json.loads((evaluate(cfg) / "results.json").read_text()))
    for r in outs:
        deg = r["degeneration"]["subjects"]["a"]["items"]
        assert len(deg["rep4_floor"]) == 3 and len(deg["rep4_greedy"]) == 3 and len(deg["rep4_sampled"]) == 6
        rec = r["recall_probe"]["subjects"]["a"]
        assert set(rec["items"]) == {"acc_L64_p4", "logprob_L64_p4", "copy_L64_p4"}
        sat = r["saturation"]["subjects"]["a"]
        assert len(sat["items"]["bucket_mean"]) == 2 * 3          # layers x buckets
    assert outs[0]["recall_probe"]["subjects"]["a"]["items"] == outs[1]["recall_probe"]["subjects"]["a"]["items"]
    assert outs[0]["degeneration"]["subjects"]["a"]["items"] == outs[1]["degeneration"]["subjects"]["a"]["items"]
    assert (root / "t1" / "samples" / "degeneration" / "a.jsonl").exists()
