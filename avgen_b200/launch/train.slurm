#!/bin/bash
# Multi-node training launcher for avgen_b200 on 8xB200 nodes.
#
#   sbatch --nodes 4 --gpus-per-node 8 avgen_b200/launch/train.slurm run.yaml [key=value ...]
#
# One torchrun agent per node, one rank per GPU, c10d rendezvous on the first
# node, up to 3 elastic restarts (each resumes from the latest complete
# checkpoint when checkpoint.resume=latest). The NCCL flight recorder is on so a
# hung collective leaves a per-rank trace behind instead of nothing.
#SBATCH --job-name=avgen_b200
#SBATCH --ntasks-per-node=1
#SBATCH --exclusive
#SBATCH --output=logs/%x-%j.out
set -euo pipefail

CONFIG="${1:?usage: sbatch train.slurm <config.yaml> [key=value ...]}"
shift || true

NODES="${SLURM_JOB_NUM_NODES:-1}"
GPUS="${SLURM_GPUS_ON_NODE:-8}"
HEAD="$(scontrol show hostnames "${SLURM_JOB_NODELIST}" | head -n 1)"
PORT="$(( 29500 + SLURM_JOB_ID % 10000 ))"

export OMP_NUM_THREADS="${OMP_NUM_THREADS:-8}"
export TORCH_NCCL_TRACE_BUFFER_SIZE="${TORCH_NCCL_TRACE_BUFFER_SIZE:-4000}"
export TORCH_NCCL_DUMP_ON_TIMEOUT=1
export TORCH_NCCL_ASYNC_ERROR_HANDLING=1
export NCCL_DEBUG="${NCCL_DEBUG:-WARN}"
# NVLink SHARP (in-switch reduction) for NCCL collectives inside a node
export NCCL_NVLS_ENABLE="${NCCL_NVLS_ENABLE:-1}"

mkdir -p logs
echo "avgen_b200: ${NODES} node(s) x ${GPUS} GPU(s); rendezvous ${HEAD}:${PORT}; config ${CONFIG} $*"

srun --kill-on-bad-exit=1 torchrun \
  --nnodes "${NODES}" --nproc-per-node "${GPUS}" \
  --rdzv-backend c10d --rdzv-endpoint "${HEAD}:${PORT}" --rdzv-id "${SLURM_JOB_ID}" \
  --max-restarts 3 \
  -m avgen_b200.cli.main train --config "${CONFIG}" "$@"
