#!/bin/bash
# Launch one process per GPU on one node (torchrun), or under SLURM (srun sets SLURM_* and
# every task runs this script with one GPU).  Usage:
#   examples/run_job.sh <script.py or --config file.yaml> [n_gpus]
set -euo pipefail
TARGET=${1:?script or --config}
NGPU=${2:-$(nvidia-smi -L | wc -l)}
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
if [[ -n "${SLURM_PROCID:-}" ]]; then
  export RANK=$SLURM_PROCID WORLD_SIZE=$SLURM_NTASKS LOCAL_RANK=${SLURM_LOCALID:-0}
  export MASTER_ADDR=${MASTER_ADDR:-127.0.0.1} MASTER_PORT=${MASTER_PORT:-29500}
  if [[ "$TARGET" == --config ]]; then exec python -m maloq_b200.cli.main --config "$2"; fi
  exec python "$TARGET"
fi
if [[ "$TARGET" == --config ]]; then
  exec python -m torch.distributed.run --standalone --nproc-per-node "${3:-$NGPU}" -m maloq_b200.cli.main --config "$2"
fi
exec python -m torch.distributed.run --standalone --nproc-per-node "$NGPU" "$TARGET"
