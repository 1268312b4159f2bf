#!/bin/bash
# Profiling of reversible BERT over 2 nodes x 5 GPUs: 20 layers, hidden 768, 12 heads, seq 512,
# global batch 2000 = 50 x 40 (BERT/scripts/exp-profiling/run_profiling2.sh).  Run once per
# node with NNODES=2, NODE_RANK and MASTER_ADDR set (c10d rendezvous).  Stage messages use
# NCCL point-to-point groups across nodes.
NPROC=${NPROC:-5}
NNODES=${NNODES:-2}
source "$(dirname "$0")/common.sh"
DATASET=${DATASET:-imdb}
exec $RUN "$ROOT/main.py" --par-mode pp --reversible --exp-mode=profiling --p2p group \
  --dataset "$DATASET" --dataset-dir "$DATASET_DIR" --num-hidden-layers 20 --hidden-size 768 \
  --num-attention-heads 12 --max-position-embeddings 512 --batch-size 2000 --microbatch-size 50 \
  --num-microbatches 40 --num-epochs 1 --autocast-dtype "$DTYPE" --lr 1e-7 $EXTRA
