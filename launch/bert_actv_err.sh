#!/bin/bash
# Reconstruction error of reversible BERT with PaReprop on 8 GPUs (per-stage MSE / cosine of
# the reconstructed stage inputs; BERT/scripts/exp-actv_err/run_actv_err.sh).
source "$(dirname "$0")/common.sh"
DATASET=${DATASET:-imdb}
exec $RUN "$ROOT/main.py" --par-mode pp --reversible --is_pareprop --exp-mode=actv-err \
  --dataset "$DATASET" --dataset-dir "$DATASET_DIR" --num-hidden-layers 24 --hidden-size 768 \
  --num-attention-heads 12 --max-position-embeddings 512 --batch-size 512 --microbatch-size 16 \
  --num-microbatches 32 --num-epochs 1 --autocast-dtype "$DTYPE" --lr 1e-7 $EXTRA
