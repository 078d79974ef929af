"""All-gather and reduce-scatter bus bandwidth per message size: NCCL
against this framework's NVLink peer-to-peer kernels (``parallel.nvlink``,
CUDA-IPC heaps, one kernel per collective), timed on every rank with the
barrier-aligned ``meter.dist`` and reported as the slowest rank.

    timeout -k 60 600 torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node 8 \\
        -m vagus_b200.meter.examples.bench_dist --mib 1 16 64 256

Bus bandwidth follows the usual convention: (world - 1) / world x the
gathered (all-gather) or input (reduce-scatter) bytes per second.  Without
CUDA the NCCL rows run on gloo and the NVLink rows are skipped.

Parity: reference ``infra/meter/examples/bench_dist.py``.
"""

from __future__ import annotations

import argparse
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from ..dist import dist_bench


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--mib", type=float, nargs="+", default=[1, 16, 64, 256],
                    help="gathered / reduced tensor size per collective (MiB)")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dist.init_process_group("nccl" if cuda else "gloo", timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda") if cuda else torch.device("cpu")
    dt = getattr(torch, a.dtype)
    esize = torch.tensor([], dtype=dt).element_size()
    heap = None
    if cuda:
        from ...parallel.nvlink import NvlinkAllGather, NvlinkHeap, NvlinkReduceScatter, same_host
        if same_host(None):
            top = int(max(a.mib) * 2 ** 20)
            heap = NvlinkHeap(None, top // world + 256, top + 256)
            ag, rs = NvlinkAllGather(heap), NvlinkReduceScatter(heap)
    rows = []
    for mib in a.mib:
        n = int(mib * 2 ** 20) // esize // world * world
        full = torch.randn(n, device=dev).to(dt)
        shard = full[rank * (n // world):(rank + 1) * (n // world)].clone()
        out_full, out_shard = torch.empty_like(full), torch.empty_like(shard)
        cases = {"nccl all-gather": lambda: dist.all_gather_into_tensor(out_full, shard),
                 "nccl reduce-scatter": lambda: dist.reduce_scatter_tensor(out_shard, full)}
        if heap is not None:
            cases["nvlink all-gather"] = lambda: ag(out_full, shard, None)
            cases["nvlink reduce-scatter"] = lambda: rs(out_shard, full, None, dist.ReduceOp.SUM)
        for name, fn in cases.items():
            res = dist_bench(fn, name=name, iters=a.iters)
            if rank == 0:
                worst = max(r.mean_ms for r in res.values())
                bus = (world - 1) / world * n * esize / (worst * 1e-3) / 1e9
                rows.append((mib, name, worst, bus))
    if rank == 0:
        print(f"world {world}  dtype {a.dtype}")
        print(f"{'MiB':>8}  {'collective':<22} {'ms (slowest rank)':>18} {'bus GB/s':>9}")
        for mib, name, ms, bus in rows:
            print(f"{mib:8.1f}  {name:<22} {ms:18.3f} {bus:9.1f}")
    if heap is not None:
        dist.barrier()
        heap.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
