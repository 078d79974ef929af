# Models: Decodable protocol, streaming generation == stateless forward,
# hybrids, optimizer coverage, FLOP model, metric hooks, config round-trip.
import pytest
import torch
from torch import nn

from vagus_b200.inference import Generator, SamplingConfig
from vagus_b200.models import build_model
from vagus_b200.models.attention import SoftmaxAttention
from vagus_b200.models.block import Block
from vagus_b200.models.cache import WithCache, missing_members
from vagus_b200.models.decodable import Decodable, missing_decodable
from vagus_b200.models.gdn import GatedDeltaNet
from vagus_b200.models.mixer import Mixer, missing_mixer
from vagus_b200.models.parallel_mixer import ParallelMixer
from vagus_b200.optim import build_optimizer
from vagus_b200.train.metrics import MetricCtx

ARGS = dict(vocab_size=101, dim=64, layer_count=3, head_count=2, key_head_dim=16, value_head_dim=32, gate_rank=8,
            chunk_size=8, la_impl="torch", context_len=48)
PAR = dict(layer_kinds=["gdn", "parallel", "gdn"], softmax_head_dim=16, softmax_rope=False)
MUON = dict(lr=1e-3, momentum=0.95, weight_decay=0.1, adamw=dict(lr=1e-3, weight_decay=0.1))


def build(**over):
    torch.manual_seed(0)
    return build_model("GDNLM", {**ARGS, **over}).eval()


def ref_greedy(model, ids, n):
    with torch.no_grad():
        for _ in range(n):
            ids = torch.cat([ids, model(ids)[:, -1].argmax(-1, keepdim=True)], 1)
    return ids


def test_protocol_and_stream_len():
    m = build()
    assert isinstance(m, Decodable) and missing_decodable(m) == []
    assert m.max_stream_len is None
    assert build(layer_pattern="gdn,softmax").max_stream_len == 48
    assert build(layer_pattern="gdn,gdn,softmax").kinds == ["gdn", "gdn", "softmax"]


@pytest.mark.parametrize("pattern", ["gdn", "gdn,softmax"])
def test_generation_matches_full_forward(pattern):
    m = build(layer_pattern=pattern)
    g = Generator(m)
    ids = torch.randint(2, 101, (2, 7))
    cfg = SamplingConfig(max_new_tokens=10, temperature=0, stop_ids=())
    out = g.generate_ids(ids, cfg, max_len=64)
    assert torch.equal(out, ref_greedy(m, ids, 10)[:, 7:])
    g.reset(2, max_len=64)
    g.prefill_ids(ids[:, :3])
    g.prefill_ids(ids[:, 3:])
    snap = g.export_state()
    a = g.gen_ids(cfg)
    h = Generator(m)
    h.load_state(snap)
    assert torch.equal(a, h.gen_ids(cfg)) and torch.equal(a, out)


def test_pure_model_runs_past_context_len():
    m = build()
    ids = torch.randint(2, 101, (1, 3 * ARGS["context_len"]))
    assert m(ids).shape == (1, ids.shape[1], 101)


def test_optimizer_coverage_and_gate_routing():
    m = build()
    groups = m.param_groups()
    n_gate = sum(1 for blk in m.blocks for _ in blk.att.gate_projections)
    assert n_gate == 9
    muon_ids = {id(p) for p in groups["muon"]}
    assert all(id(p) not in muon_ids for blk in m.blocks for p in blk.att.gate_projections)
    names = {id(p): n for n, p in m.named_parameters()}
    nd = {names[id(p)] for p in groups["adamw_no_decay"]}
    assert any("A_log" in n for n in nd) and any("dt_bias" in n for n in nd)
    opt = build_optimizer("muon", m, MUON)
    assert sum(len(g["params"]) for g in opt.param_groups) == sum(1 for _ in m.parameters())
    assert len(build(gate_proj_optimizer="muon").param_groups()["muon"]) == len(groups["muon"]) + n_gate


def test_train_step_bf16_autocast_cpu():
    m = build().train()
    ids = torch.randint(2, 101, (2, 20))
    with torch.autocast("cpu", dtype=torch.bfloat16):
        h = m(ids[:, :-1], return_hidden=True)
        loss = torch.nn.functional.cross_entropy((h @ m.head.weight.T).float().flatten(0, 1), ids[:, 1:].flatten())
    loss.backward()
    assert all(p.grad is not None for p in m.parameters())


def test_metric_hook_and_flops():
    m = build(layer_pattern="gdn,gdn,softmax")
    ctx = MetricCtx(model=m, last_batch=torch.randint(2, 101, (2, 30)))
    out = m.metric_hooks()["slow"][0](ctx)
    gates = {"gdn/state_rms_max", "gdn/alpha_mean", "gdn/mem_len_median", "gdn/mem_len_max", "gdn/beta_mean"}
    assert set(out) == gates | {"attn_logit_max"}
    assert 0 < out["gdn/alpha_mean"] < 1 and out["gdn/mem_len_max"] >= out["gdn/mem_len_median"] > 1
    assert m.metric_hooks()["slow"][0](MetricCtx(model=m)) == {}
    per_head = 3 * (6 * 16 * 32 + 2 * 8 * (3 * 16 + 2 * 32))
    assert m.attn_flops_per_token(2048) == 2 * 2 * per_head + 12 * 64 * 2048
    m0 = build(gate="none", delta=False)
    assert m0.attn_flops_per_token(2048) == 3 * 2 * 3 * (4 * 16 * 32 + 2 * 8 * (16 + 32))
    assert set(m0.metric_hooks()["slow"][0](ctx)) == {"gdn/state_rms_max"}
    assert set(build(gate="scalar").metric_hooks()["slow"][0](ctx)) == gates


def test_config_roundtrip():
    m = build(layer_pattern="gdn,softmax", gate="scalar")
    m2 = type(m).from_config(m.config)
    assert m2.kinds == m.kinds and [p.shape for p in m2.parameters()] == [p.shape for p in m.parameters()]


def test_mixer_protocol():
    m = build(layer_pattern="gdn,softmax")
    assert isinstance(m, WithCache) and missing_members(WithCache, m) == []
    for blk in m.blocks:
        assert missing_members(WithCache, blk) == [] and isinstance(blk.att, Mixer) and missing_mixer(blk.att) == []
    assert sorted(Mixer.__protocol_attrs__) == ["__call__", "decode_step", "export_cache", "forward", "load_cache",
                                               "reset_cache"]
    assert isinstance(m.blocks[0].att, GatedDeltaNet) and isinstance(m.blocks[1].att, SoftmaxAttention)
    with pytest.raises(TypeError, match="not a Mixer"):
        Block(dim=16, mixer=nn.Linear(16, 16), layer_count=1)


def test_checkpoint_fqns():
    m = build(layer_kinds=["gdn", "parallel", "softmax"], softmax_head_dim=16, softmax_out_gate=True)
    keys = set(m.state_dict())
    for k in ("embedding.weight", "head.weight", "rms_head.gamma", "blocks.0.rmsnorm1.gamma", "blocks.0.rmsnorm2.gamma",
              "blocks.0.ffn.l1.weight", "blocks.0.ffn.l2.weight", "blocks.0.att.wq.weight", "blocks.0.att.wk.weight",
              "blocks.0.att.wv.weight", "blocks.0.att.wg.weight", "blocks.0.att.wo.weight", "blocks.0.att.wa1.weight",
              "blocks.0.att.wa2.weight", "blocks.0.att.wb.weight", "blocks.0.att.A_log", "blocks.0.att.dt_bias",
              "blocks.0.att.o_norm.gamma", "blocks.0.att.conv_q.conv.weight", "blocks.1.att.att.wq.weight",
              "blocks.1.att.la.wq.weight", "blocks.1.att.att_norm.gamma", "blocks.1.att.la_norm.gamma",
              "blocks.1.att.wo.weight", "blocks.2.att.q_norm.gamma", "blocks.2.att.k_norm.gamma",
              "blocks.2.att.wg.weight"):
        assert k in keys, k
    assert not any("rope" in k or "cache" in k or k.endswith(".state") for k in keys)


def test_decay_init_range_reaches_the_mixer():
    narrow = build(A_init_range=(1.0, 2.0), dt_init_range=(1e-2, 2e-2))
    wide = build(A_init_range=(0.5, 32.0), dt_init_range=(5e-4, 1.5e-1))

    def rest_tau(m):
        att = m.blocks[0].att
        b = att.dt_bias.view(att.head_count, att.key_head_dim)
        return 1.0 / (att.A_log.exp()[:, None] * torch.nn.functional.softplus(b))

    for m, (lo, hi) in ((narrow, (1.0, 2.0)), (wide, (0.5, 32.0))):
        A = m.blocks[0].att.A_log.exp()
        assert (A >= lo - 1e-4).all() and (A <= hi + 1e-4).all()
    assert rest_tau(wide).log10().std() > 2 * rest_tau(narrow).log10().std()
    assert type(wide).from_config(wide.config).config["A_init_range"] == (0.5, 32.0)
    assert (build(**PAR, A_init_range=(0.5, 32.0)).blocks[1].att.la.A_log.exp() <= 32.0 + 1e-4).all()


def test_layer_kinds_and_parallel_shapes():
    m = build(**PAR)
    assert m.kinds == ["gdn", "parallel", "gdn"] and m.rope is None and m.max_stream_len is None
    par = m.blocks[1].att
    assert isinstance(par, ParallelMixer)
    assert par.att.head_count == 2 and par.att.in_dim == 64 and par.att.out_width == 32
    assert par.la.head_count == 1 and par.la.out_width == 32
    assert not hasattr(par.att, "wo") and not hasattr(par.la, "wo") and par.wo.weight.shape == (64, 64)
    with pytest.raises(AssertionError, match="layer_kinds"):
        build(layer_kinds=["gdn", "parallel"])
    with pytest.raises(AssertionError, match="parallel_width"):
        build(layer_kinds=["gdn", "parallel", "gdn"], softmax_head_dim=64)
    assert build(layer_kinds=["gdn", "parallel", "gdn"], softmax_head_dim=16).max_stream_len == 48


@pytest.mark.parametrize("kinds", [["gdn", "parallel", "gdn"], ["softmax", "gdn", "parallel"]])
def test_parallel_generation_matches_full_forward(kinds):
    m = build(**{**PAR, "layer_kinds": kinds})
    g = Generator(m)
    ids = torch.randint(2, 101, (2, 7))
    cfg = SamplingConfig(max_new_tokens=10, temperature=0, stop_ids=())
    out = g.generate_ids(ids, cfg, max_len=64)
    assert torch.equal(out, ref_greedy(m, ids, 10)[:, 7:])
    g.reset(2, max_len=64)
    g.prefill_ids(ids[:, :3])
    g.prefill_ids(ids[:, 3:])
    snap = g.export_state()
    assert set(snap["cache"]["blocks"][kinds.index("parallel")]["att"]) == {"att", "la"}
    a = g.gen_ids(cfg)
    h = Generator(m)
    h.load_state(snap)
    assert torch.equal(a, h.gen_ids(cfg)) and torch.equal(a, out)


@pytest.mark.parametrize("pattern", ["gdn,softmax", "gdn,parallel"])
def test_softmax_out_gate(pattern):
    m = build(layer_pattern=pattern, softmax_out_gate=True, softmax_head_dim=16)
    att = m.blocks[1].att if pattern == "gdn,softmax" else m.blocks[1].att.att
    assert att.out_gate and att.wg.weight.shape == (att.out_width, att.in_dim)
    assert any(p is att.wg.weight for p in m.param_groups()["muon"])
    ids = torch.randint(2, 101, (2, 7))
    ref = m(ids)
    m.reset_cache(2, 64)
    out = torch.cat([m.decode_step(ids[:, :4]), m.decode_step(ids[:, 4:])], 1)
    assert torch.allclose(out, ref, atol=1e-5)


def test_transformer_pp_generation_and_flops():
    torch.manual_seed(0)
    m = build_model("TransformerPP", dict(vocab_size=101, dim=64, head_dim=16, context_len=32, layer_count=2,
                                          qk_norm=True)).eval()
    g = Generator(m, start_id=1, stop_ids=(1,))
    ids = torch.randint(2, 101, (2, 5))
    cfg = SamplingConfig(max_new_tokens=8, temperature=0, stop_ids=())
    out = g.generate_ids(ids, cfg)
    start = torch.ones(2, 1, dtype=torch.long)
    assert torch.equal(out, ref_greedy(m, torch.cat([start, ids], 1), 8)[:, 6:])
    assert m.attn_flops_per_token(2048) == 12 * 2 * 64 * 2048
    assert m.max_stream_len == 32
    assert set(m.metric_hooks()["slow"][0](MetricCtx(model=m, last_batch=ids))) == {"attn_logit_max"}


def test_packed_attention_layer_gating(monkeypatch):
    """Which softmax-attention layers and inputs take the packed q / k / v path
    (``ops.attention_layer``): CUDA input in bf16 (or under bf16 autocast), no
    short conv or output gate, head dims 64 / 128, GEMM-sized projections.
    Checked on a stand-in for a CUDA tensor and for the extension, since only
    the predicate runs."""
    from types import SimpleNamespace
    from vagus_b200 import ops
    from vagus_b200.models.rope import RoPE
    import importlib
    attn_ops = importlib.import_module("vagus_b200.ops.attention")   # the module, not the function ops.attention
    monkeypatch.setattr(attn_ops, "native", lambda: SimpleNamespace(attn_fwd=None))

    def x_like(B, L, D, cuda=True, dtype=torch.bfloat16):
        return SimpleNamespace(is_cuda=cuda, dtype=dtype, shape=(B, L, D), dim=lambda: 3)

    def layer(dim=512, H=8, Hk=None, vm=1, **kw):
        return SoftmaxAttention(dim, H, Hk, vm, rope=RoPE(dim, dim // H, 256), **kw)

    assert ops.attention_layer_ok(layer(), x_like(2, 256, 512))
    assert ops.attention_layer_ok(layer(Hk=2, qk_norm=True), x_like(2, 256, 512))
    assert ops.attention_layer_ok(layer(H=4), x_like(2, 256, 512))                 # head dim 128
    assert not ops.attention_layer_ok(layer(), x_like(2, 256, 512, cuda=False))
    assert not ops.attention_layer_ok(layer(), x_like(2, 256, 512, dtype=torch.float32))
    assert not ops.attention_layer_ok(layer(short_conv_size=4), x_like(2, 256, 512))
    assert not ops.attention_layer_ok(layer(out_gate=True), x_like(2, 256, 512))
    assert not ops.attention_layer_ok(layer(H=16), x_like(2, 256, 512))            # head dim 32
    assert not ops.attention_layer_ok(layer(), x_like(1, 64, 512))                 # 64 tokens: below a GEMM tile
