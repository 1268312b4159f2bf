#!/bin/bash
# Profiling of reversible ViT-B/16 on 8 GPUs: 12 layers, hidden 768, 12 heads, CIFAR-10 at
# 224 x 224, global batch 512 = 16 x 32 (Vit/scripts/exp-profiling/run_profiling.sh).
source "$(dirname "$0")/common.sh"
DATASET=${DATASET:-cifar-10}
exec $RUN "$ROOT/main.py" --model vit --par-mode pp --reversible --exp-mode=profiling \
  --dataset "$DATASET" --dataset-dir "$DATASET_DIR" --num-hidden-layers 12 --hidden-size 768 \
  --num-attention-heads 12 --num-classes 10 --batch-size 512 --microbatch-size 16 --num-microbatches 32 \
  --num-epochs 1 --autocast-dtype "$DTYPE" --lr 1e-7 $EXTRA
