"""Stream-state generator and sampling (CPU, fp32): greedy == full forward,
split prefill, state export / load mid-generation, stop ids and capacity,
sampling knobs, checkpoint formats (full, slim, bf16 slim)."""

import pytest
import torch

from vagus_b200.inference.generator import Generator
from vagus_b200.inference.sampling import SamplingConfig, sample
from vagus_b200.models import build_model
from vagus_b200.models.io import SLIM_KEYS, export_slim, load_model

GDN = dict(vocab_size=300, dim=64, layer_count=2, head_count=2, key_head_dim=32, value_head_dim=32,
           ffn_hidden_dim=128, context_len=128, gate="scalar", delta=True, chunk_size=16,
           layer_pattern="gdn,softmax", softmax_head_dim=32)
TPP = dict(vocab_size=300, dim=64, layer_count=2, head_dim=32, context_len=128, ffn_hidden_dim=128)


@pytest.fixture(params=[("GDNLM", GDN), ("TransformerPP", TPP)], ids=["gdn_hybrid", "tpp"])
def model(request):
    torch.manual_seed(0)
    name, args = request.param
    m = build_model(name, args).eval()
    m.model_name, m.model_args = name, args
    return m


def _greedy_reference(m, ids, n):
    seq = ids.clone()
    with torch.no_grad():
        for _ in range(n):
            nxt = m(seq)[:, -1].argmax(-1)
            seq = torch.cat([seq, nxt[:, None]], 1)
    return seq[:, ids.shape[1]:]


def test_greedy_matches_full_forward_and_split_prefill(model):
    ids = torch.randint(2, 300, (2, 9))
    g = Generator(model)
    out = g.generate_ids(ids, SamplingConfig(max_new_tokens=6, temperature=0), max_len=64)
    assert torch.equal(out, _greedy_reference(model, ids, 6))
    g.reset(2, 64)
    g.prefill_ids(ids[:, :4])
    g.prefill_ids(ids[:, 4:])
    assert torch.equal(g.gen_ids(SamplingConfig(max_new_tokens=6, temperature=0)), out)


def test_export_load_mid_generation(model):
    ids = torch.randint(2, 300, (1, 7))
    cfg = SamplingConfig(max_new_tokens=5, temperature=0.8, top_k=20, seed=3)
    g = Generator(model)
    g.reset(1, 64)
    g.prefill_ids(ids)
    first = g.gen_ids(SamplingConfig(max_new_tokens=3, temperature=0))
    state = g.export_state()
    cont = g.gen_ids(cfg)
    g2 = Generator(model)
    g2.load_state(state)
    assert g2.stream_len == g.stream_len - cont.shape[1]
    assert torch.equal(g2.gen_ids(cfg), cont) and first.shape == (1, 3)


def test_stop_ids_and_capacity(model):
    ids = torch.randint(2, 300, (1, 5))
    g = Generator(model)
    g.reset(1, 64)
    g.prefill_ids(ids)
    t = g.gen_ids(SamplingConfig(max_new_tokens=1, temperature=0))
    g.reset(1, 64)
    g.prefill_ids(ids)
    out = g.gen_ids(SamplingConfig(max_new_tokens=10, temperature=0, stop_ids=(int(t[0, 0]),)))
    assert out.shape[1] == 1 and g.stop_reason == "stop_id"
    g.reset(1, 8)
    g.prefill_ids(ids)
    out = g.gen_ids(SamplingConfig(max_new_tokens=10, temperature=0))
    assert g.stop_reason == "capacity" and g.fed_len == 8  # the pending token is not fed yet


def test_sampling_knobs():
    logits = torch.tensor([[4.0, 3.0, 1.0, -2.0]])
    assert sample(logits, SamplingConfig(temperature=0)).item() == 0
    rng = torch.Generator().manual_seed(0)
    picks = {sample(logits, SamplingConfig(top_k=2), rng).item() for _ in range(200)}
    assert picks <= {0, 1} and len(picks) == 2
    picks = {sample(logits, SamplingConfig(top_p=0.5), rng).item() for _ in range(50)}
    assert picks == {0}                       # the mass before token 1 already exceeds 0.5


def test_checkpoint_formats(tmp_path, model):
    full = {"step": 3, "tokens_seen": 99, "model_name": model.model_name, "model_args": model.model_args,
            "tokenizer": {"id": "mistral32k", "sha256": "x"}, "model": model.state_dict(), "optimizer": {}}
    torch.save(full, tmp_path / "ckpt.pt")
    m2, meta = load_model(tmp_path / "ckpt.pt")
    assert meta["step"] == 3
    for (k, a), (_, b) in zip(model.state_dict().items(), m2.state_dict().items()):
        assert torch.equal(a, b), k
    slim = export_slim(tmp_path / "ckpt.pt", tmp_path / "slim.pt", dtype=torch.bfloat16)
    s = torch.load(slim, weights_only=False)
    assert set(s) == set(SLIM_KEYS)
    assert all(v.dtype == torch.bfloat16 for v in s["model"].values() if v.is_floating_point())
    m3, _ = load_model(slim, dtype=torch.float32)
    ids = torch.randint(2, 300, (1, 6))
    with torch.no_grad():
        assert (m3(ids) - model(ids)).abs().max() < 0.1
