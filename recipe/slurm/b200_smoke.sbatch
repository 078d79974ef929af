#!/bin/bash
# Node smoke gate before a long run: the kernel and CPU test suites, the
# 2-GPU collective test, the headline benchmark at 1 and 8 GPUs and a short
# hybrid training smoke through the real trainer.
#SBATCH --job-name=vagus-b200-smoke
#SBATCH --nodes=1
#SBATCH --gres=gpu:8
#SBATCH --time=01:00:00
#SBATCH --output=logs/%x-%j.out
set -euo pipefail
python -c "import __graft_entry__ as g; g.build(); g.smoke()"
python -m pytest tests -x -q
python bench.py --steps 4 --warmup 3
timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \
    --master-port 29511 bench.py --gpus 8 --steps 4 --warmup 3
export MASTER_ADDR=127.0.0.1 MASTER_PORT=29512 GPUS_PER_NODE=8 SLURM_NNODES=1 SLURM_NODEID=0
recipe/slurm/torchrun_node.sh recipe/train/hax1_340M_smoke.yaml run_dir=runs/smoke-$SLURM_JOB_ID
