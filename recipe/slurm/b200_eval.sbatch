#!/bin/bash
# Evaluation of finished runs on one B200: sbatch recipe/slurm/b200_eval.sbatch recipe/eval/<name>.yaml
#SBATCH --job-name=vagus-b200-eval
#SBATCH --nodes=1
#SBATCH --gres=gpu:1
#SBATCH --time=04:00:00
#SBATCH --output=logs/%x-%j.out
set -euo pipefail
python -m vagus_b200.eval.main "$@"
