#!/bin/bash
#SBATCH --job-name=pan2_generate
#SBATCH --nodes=1
#SBATCH --ntasks-per-node=1
#SBATCH --gres=gpu:8
#SBATCH --cpus-per-task=128
#SBATCH --output=logs/%x_%j.out
#SBATCH --error=logs/%x_%j.err
#
# Generate the videos of a prompt file on one node:
#   bash launch/generate.sh <CHECKPOINT> [OUTPUT_DIR] [PROMPTS_JSON]
# SP_SIZE ranks share each prompt (Ulysses sequence parallel); the GPUS / SP_SIZE groups shard the
# prompt list.  SP_SIZE=1 gives one independent worker per GPU.  Sampler settings come from the
# variables below (any can be overridden from the environment); finished videos whose saved settings
# match are skipped on rerun.
set -euo pipefail
root=""
for d in "${PAN_ROOT:-}" "${SLURM_SUBMIT_DIR:-}" "$(cd "$(dirname "$0")/.." 2>/dev/null && pwd)" "$PWD"; do
    [[ -n $d && -f $d/generate.py ]] && { root=$(cd "$d" && pwd); break; }
done
[[ -n $root ]] || { echo "cannot find the repository (no generate.py); set PAN_ROOT" >&2; exit 1; }
cd "$root"

CHECKPOINT=${1:?usage: generate.sh <CHECKPOINT> [OUTPUT_DIR] [PROMPTS_JSON]}
OUTPUT_DIR=${2:-${OUTPUT_DIR:-outputs/$(date +%Y%m%d_%H%M%S)}}
PROMPTS_JSON=${3:-${PROMPTS_JSON:?set PROMPTS_JSON or pass it as the third argument}}
TRAINING_CONFIG=${TRAINING_CONFIG:-config/sft_29B_720p.yaml}
NUM_STEPS=${NUM_STEPS:-50}
FLOW_SHIFT=${FLOW_SHIFT:-9}
GUIDANCE_SCALE=${GUIDANCE_SCALE:-2.5}
TASK=${TASK:-auto}
VIDEO_HEIGHT=${VIDEO_HEIGHT:-704}
VIDEO_WIDTH=${VIDEO_WIDTH:-1248}
FPS=${FPS:-24}
VIDEO_LENGTH=${VIDEO_LENGTH:-241}
SEED=${SEED:-123}
GPUS=${GPUS:-$(nvidia-smi -L 2>/dev/null | wc -l)}
SP_SIZE=${SP_SIZE:-$GPUS}
EXTRA_ARGS=${EXTRA_ARGS:-}
NEG=()
[[ -n ${NEGATIVE_PROMPT_FILE:-} ]] && NEG=(--negative_prompt_file "$NEGATIVE_PROMPT_FILE")
mkdir -p "$OUTPUT_DIR" logs
export PYTORCH_CUDA_ALLOC_CONF=${PYTORCH_CUDA_ALLOC_CONF:-expandable_segments:True}
export HF_HUB_OFFLINE=${HF_HUB_OFFLINE:-1}
python -c "import torch, pan2_b200._C" 2>/dev/null || python setup.py build_ext --inplace

torchrun --standalone --local-addr 127.0.0.1 --nnodes=1 --nproc-per-node="$GPUS" generate.py \
    --task "$TASK" --prompt_json "$PROMPTS_JSON" --output_dir "$OUTPUT_DIR" --sp_size "$SP_SIZE" \
    --checkpoint_path "$CHECKPOINT" --training_config "$TRAINING_CONFIG" \
    --num_inference_steps "$NUM_STEPS" --flow_shift "$FLOW_SHIFT" --guidance_scale "$GUIDANCE_SCALE" \
    --video_height "$VIDEO_HEIGHT" --video_width "$VIDEO_WIDTH" --fps "$FPS" --video_length "$VIDEO_LENGTH" \
    --seed "$SEED" --dtype bf16 --i2v_skip_first_latent_cfg true "${NEG[@]}" \
    --skip_existing true --save_settings true $EXTRA_ARGS
