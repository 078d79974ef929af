#!/bin/bash
# Per-node launcher: one srun task per node runs this script and torchrun
# starts the node's 8 GPU workers (one process per B200).  The batch script
# exports MASTER_ADDR / MASTER_PORT (rendezvous on the first node).
#
#   srun --kill-on-bad-exit=1 recipe/slurm/torchrun_node.sh <train recipe> [key=value ...]
#
# --shutdown_timeout gives the workers time to write their recent checkpoint
# after a SIGTERM / SIGUSR1 (walltime forwarding) before the agent kills them.
cd "${VAGUS_B200_HOME:-$HOME/vagus-b200}" || exit 1
exec python -m torch.distributed.run \
    --nnodes "${SLURM_NNODES:-1}" --nproc_per_node "${GPUS_PER_NODE:-8}" --node_rank "${SLURM_NODEID:-0}" \
    --rdzv_backend c10d --rdzv_endpoint "$MASTER_ADDR:$MASTER_PORT" --rdzv_id "${SLURM_JOB_ID:-local}" \
    --shutdown_timeout 900 \
    -m vagus_b200.train.main "$@"
