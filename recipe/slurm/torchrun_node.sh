#!/bin/bash
# Per-node launcher: one srun task per node runs this script and torchrun
# starts the node's 8 GPU workers (one process per B200).  The batch script
# exports MASTER_ADDR / MASTER_PORT (rendezvous on the first node).
#
#   srun --kill-on-bad-exit=1 recipe/slurm/torchrun_node.sh <train recipe> [key=value ...]
#
# --signals-to-handle adds SIGUSR1 (the walltime warning the batch script
# forwards) to the signals torchrun passes on to its workers, whose handler
# makes the trainer stop at the next step boundary with a checkpoint (torchrun
# then exits non-zero; the batch script ignores srun's status and re-queues).
cd "${VAGUS_B200_HOME:-$HOME/vagus-b200}" || exit 1
exec python -m torch.distributed.run \
    --nnodes "${SLURM_NNODES:-1}" --nproc-per-node "${GPUS_PER_NODE:-8}" --node-rank "${SLURM_NODEID:-0}" \
    --rdzv-backend c10d --rdzv-endpoint "$MASTER_ADDR:$MASTER_PORT" --rdzv-id "${SLURM_JOB_ID:-local}" \
    --signals-to-handle SIGTERM,SIGINT,SIGHUP,SIGQUIT,SIGUSR1 \
    -m vagus_b200.train.main "$@"
