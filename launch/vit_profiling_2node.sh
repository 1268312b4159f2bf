#!/bin/bash
# Profiling of reversible ViT over 2 nodes x 7 GPUs: 28 layers, hidden 768, 12 heads,
# global batch 2800 = 50 x 56 (Vit/scripts/exp-profiling/run_profiling2.sh).  Run once per
# node with NNODES=2, NODE_RANK and MASTER_ADDR set.
NPROC=${NPROC:-7}
NNODES=${NNODES:-2}
source "$(dirname "$0")/common.sh"
DATASET=${DATASET:-cifar-10}
exec $RUN "$ROOT/main.py" --model vit --par-mode pp --reversible --exp-mode=profiling --p2p group \
  --dataset "$DATASET" --dataset-dir "$DATASET_DIR" --num-hidden-layers 28 --hidden-size 768 \
  --num-attention-heads 12 --num-classes 10 --batch-size 2800 --microbatch-size 50 --num-microbatches 56 \
  --num-epochs 1 --autocast-dtype "$DTYPE" --lr 1e-7 $EXTRA
