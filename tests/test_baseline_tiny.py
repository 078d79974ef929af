"""The plumbing configuration of the benchmark set, end to end on CPU: a
tiny GDN LM (vocab 4096, d_model 128, 2 layers, 2 heads x 64, SwiGLU 384,
fp32) under DDP on two gloo ranks, one train step with AdamW on embeddings /
norms and Muon (5 Newton-Schulz steps) on the 2-D weights, on uniform token
ids from seed 0 (batch 4 x seq 256), then 32 tokens of greedy generation that
match the full-forward greedy continuation."""

import os
import socket

import torch
import torch.multiprocessing as mp

ARGS = dict(vocab_size=4096, dim=128, layer_count=2, head_count=2, key_head_dim=64, value_head_dim=64,
            ffn_hidden_dim=384, gate="scalar", delta=True, chunk_size=64, context_len=512, la_impl="torch")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank))
        from vagus_b200.parallel import setup_distributed
        setup_distributed("cpu", timeout_s=120)
        import torch.distributed as dist
        from torch.nn.parallel import DistributedDataParallel as DDP
        from vagus_b200.inference.generator import Generator
        from vagus_b200.inference.sampling import SamplingConfig
        from vagus_b200.models import build_model
        from vagus_b200.models.losses import make_ce
        from vagus_b200.optim import build_optimizer
        from vagus_b200.parallel import unwrap
        from vagus_b200.train.main import StepRunner
        torch.manual_seed(0)
        model = DDP(build_model("GDNLM", ARGS))
        opt = build_optimizer("muon", unwrap(model), dict(lr=2e-2, ns_steps=5, adamw=dict(lr=3e-3)))
        ce = make_ce("full")
        runner = StepRunner(model, opt, ce, torch.device("cpu"), grad_accum_steps=1, grad_clip=1.0, is_dist=True)
        g = torch.Generator().manual_seed(0)
        tokens = torch.randint(0, 4096, (world, 4, 257), generator=g)[rank]      # each rank its own batch
        loss, _z, gn = runner.step(iter([(tokens[:, :-1], tokens[:, 1:])]))
        m = unwrap(model).eval()
        # parameters are identical on both ranks after the DDP step
        flat = torch.cat([p.detach().flatten() for p in m.parameters()])
        other = flat.clone()
        dist.broadcast(other, src=0)
        prompt = torch.randint(0, 4096, (1, 16), generator=torch.Generator().manual_seed(1))   # same on both ranks
        gen = Generator(m).generate_ids(prompt, SamplingConfig(max_new_tokens=32, temperature=0.0), max_len=64)
        ids = prompt
        with torch.no_grad():
            for _ in range(32):
                ids = torch.cat([ids, m(ids)[:, -1].argmax(-1, keepdim=True)], 1)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, dict(loss=loss.item(), gn=float(gn), same_params=bool(torch.equal(flat, other)),
                          gen=gen.tolist(), greedy=ids[:, 16:].tolist())))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


def test_tiny_gdn_ddp_gloo_step_and_generation():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, r in res.items():
        assert not isinstance(r, str), r
        assert abs(r["loss"] - torch.log(torch.tensor(4096.0)).item()) < 0.5      # random init: ~ln V
        assert r["same_params"], rank
        assert len(r["gen"][0]) == 32 and r["gen"] == r["greedy"], rank
    assert res[0]["gen"] == res[1]["gen"]
