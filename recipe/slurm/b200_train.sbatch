#!/bin/bash
# Training on whole 8 x B200 nodes.  Usage:
#   sbatch --nodes=N recipe/slurm/b200_train.sbatch recipe/train/<run>.yaml [key=value ...]
# The job re-queues itself (chain guard) until the run's final permanent
# checkpoint exists; a SIGUSR1 two minutes before the walltime makes every
# rank write a recent checkpoint and exit cleanly.
#SBATCH --job-name=vagus-b200
#SBATCH --ntasks-per-node=1
#SBATCH --gres=gpu:8
#SBATCH --cpus-per-task=64
#SBATCH --time=24:00:00
#SBATCH --signal=B:USR1@120
#SBATCH --output=logs/%x-%j.out
set -euo pipefail
RECIPE=$1; shift
export MASTER_ADDR=$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n 1)
export MASTER_PORT=${MASTER_PORT:-29511}
export GPUS_PER_NODE=8
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
export OMP_NUM_THREADS=8
forward() { echo "walltime signal: forwarding to the workers"; kill -USR1 "$SRUN_PID" 2>/dev/null || true; }
trap forward USR1
srun --kill-on-bad-exit=1 recipe/slurm/torchrun_node.sh "$RECIPE" "$@" &
SRUN_PID=$!
wait "$SRUN_PID" || true
wait "$SRUN_PID" 2>/dev/null || true
# chain guard: resubmit while the run has not written model-final.pt
RUN=$(python - "$RECIPE" "$@" <<'PY'
import sys
from vagus_b200.train.main import TrainConfig, resolve_run_dir
print(resolve_run_dir(TrainConfig.from_yaml(sys.argv[1], sys.argv[2:])))
PY
)
if [ -n "$RUN" ] && [ ! -f "$RUN/model-final.pt" ]; then
  echo "run not finished: resubmitting"; sbatch --nodes="$SLURM_NNODES" "$0" "$RECIPE" "$@"
fi
