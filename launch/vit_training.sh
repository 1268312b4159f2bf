#!/bin/bash
# Training of reversible ViT-B/16 on CIFAR-10 for 15 epochs on 8 GPUs, lr 1e-5, seed 1
# (Vit/scripts/exp-training/run_training.sh).
source "$(dirname "$0")/common.sh"
DATASET=${DATASET:-cifar-10}
exec $RUN "$ROOT/main.py" --model vit --par-mode pp --reversible --exp-mode=training \
  --dataset "$DATASET" --dataset-dir "$DATASET_DIR" --num-hidden-layers 12 --hidden-size 768 \
  --num-attention-heads 12 --num-classes 10 --batch-size 512 --microbatch-size 16 --num-microbatches 32 \
  --num-epochs 15 --autocast-dtype "$DTYPE" --lr 1e-5 --seed 1 --save-checkpoint $EXTRA
