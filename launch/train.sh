#!/bin/bash
#SBATCH --job-name=pan2_train
#SBATCH --nodes=1
#SBATCH --ntasks-per-node=1
#SBATCH --gres=gpu:8
#SBATCH --cpus-per-task=128
#SBATCH --output=logs/%x_%j.out
#SBATCH --error=logs/%x_%j.err
#SBATCH --open-mode=append
#SBATCH --no-requeue
#
# Train on one or more nodes of 8 B200s, one process per GPU:
#   sbatch launch/train.sh [CONFIG] [train.py options...]
#   bash   launch/train.sh config/pretrain_29B_720p.yaml --output_dir /runs/a   (interactive, one node)
# CONFIG defaults to config/pretrain_29B_720p.yaml (config/sft_29B_720p.yaml for SFT).  PAN_ROOT is the
# repository when the script is not run from it; GPUS_PER_NODE overrides the GPU count.
set -euo pipefail
CONFIG=config/pretrain_29B_720p.yaml
if [[ $# -gt 0 && $1 != -* ]]; then CONFIG=$1; shift; fi

root=""
for d in "${PAN_ROOT:-}" "${SLURM_SUBMIT_DIR:-}" "$(cd "$(dirname "$0")/.." 2>/dev/null && pwd)" "$PWD"; do
    [[ -n $d && -f $d/train.py ]] && { root=$(cd "$d" && pwd); break; }
done
[[ -n $root ]] || { echo "cannot find the repository (no train.py); set PAN_ROOT" >&2; exit 1; }
cd "$root"
[[ -f $CONFIG ]] || { echo "config not found: $CONFIG" >&2; exit 1; }
mkdir -p logs

export PYTORCH_CUDA_ALLOC_CONF=${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}
export HF_HUB_OFFLINE=${HF_HUB_OFFLINE:-1}
export TORCH_NCCL_ASYNC_ERROR_HANDLING=${TORCH_NCCL_ASYNC_ERROR_HANDLING:-1}
# multi-node over AWS EFA (libfabric): set PAN_NET=efa, or leave it to auto-detect the EFA devices
if [[ ${PAN_NET:-auto} == efa || ( ${PAN_NET:-auto} == auto && -d /sys/class/infiniband && \
      -n $(ls /sys/class/infiniband 2>/dev/null | grep -m1 efa) ) ]]; then
    export FI_PROVIDER=${FI_PROVIDER:-efa}
    export FI_EFA_USE_DEVICE_RDMA=${FI_EFA_USE_DEVICE_RDMA:-1}
    export FI_EFA_FORK_SAFE=${FI_EFA_FORK_SAFE:-1}
fi
# the CUDA extension is built in-tree once; every rank imports the same .so
python -c "import torch, pan2_b200._C" 2>/dev/null || python setup.py build_ext --inplace

GPUS_PER_NODE=${GPUS_PER_NODE:-$(nvidia-smi -L 2>/dev/null | wc -l)}
if [[ -n ${SLURM_JOB_ID:-} && ${SLURM_NNODES:-1} -gt 1 ]]; then
    head=$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n 1)
    export MASTER_ADDR=$(srun --nodes=1 --ntasks=1 -w "$head" hostname -I | awk '{print $1}')
    export MASTER_PORT=${MASTER_PORT:-29505}
    srun --ntasks-per-node=1 bash -c "torchrun --nnodes=$SLURM_NNODES --node_rank=\$SLURM_NODEID \
        --nproc-per-node=$GPUS_PER_NODE --rdzv-backend=c10d --rdzv-endpoint=$MASTER_ADDR:$MASTER_PORT \
        train.py --config $CONFIG $(printf '%q ' "$@")"
else
    torchrun --standalone --local-addr 127.0.0.1 --nnodes=1 --nproc-per-node="$GPUS_PER_NODE" \
        train.py --config "$CONFIG" "$@"
fi
