#!/bin/bash
# Reconstruction error of reversible ViT-B/16 on 8 GPUs (Vit/scripts/exp-actv_err/run_actv_err.sh).
source "$(dirname "$0")/common.sh"
DATASET=${DATASET:-cifar-10}
exec $RUN "$ROOT/main.py" --model vit --par-mode pp --reversible --exp-mode=actv-err \
  --dataset "$DATASET" --dataset-dir "$DATASET_DIR" --num-hidden-layers 12 --hidden-size 768 \
  --num-attention-heads 12 --num-classes 10 --batch-size 512 --microbatch-size 16 --num-microbatches 32 \
  --num-epochs 1 --autocast-dtype "$DTYPE" --lr 1e-7 $EXTRA
