#!/bin/bash
# Profiling of reversible BERT with PaReprop on one node of 8 GPUs: 24 layers, hidden 768,
# 12 heads, seq 512, global batch 512 = 16 x 32 (BERT/scripts/exp-profiling/run_profiling.sh).
# The reference ran fp32 (DTYPE=fp32); the default here is the bf16 kernel path.
source "$(dirname "$0")/common.sh"
DATASET=${DATASET:-imdb}
exec $RUN "$ROOT/main.py" --par-mode pp --reversible --is_pareprop --exp-mode=profiling \
  --dataset "$DATASET" --dataset-dir "$DATASET_DIR" --num-hidden-layers 24 --hidden-size 768 \
  --num-attention-heads 12 --max-position-embeddings 512 --batch-size 512 --microbatch-size 16 \
  --num-microbatches 32 --num-epochs 1 --autocast-dtype "$DTYPE" --lr 1e-7 $EXTRA
