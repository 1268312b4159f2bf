#!/bin/bash
# Training throughput of reversible BERT-Large (seq 512, global batch 512, bf16, synthetic
# data) at PP = 1, 2, 4, 8 for this framework and, with REF=1, for the installed reference
# (bench.py --impl reference), one JSON line per run.  Set NS="1 2" etc. to choose the sizes.
ROOT="$(cd "$(dirname "$0")/.." && pwd)"
NS=${NS:-"1 2 4 8"}
STEPS=${STEPS:-6}
WARMUP=${WARMUP:-3}
for n in $NS; do
  for impl in revpp ${REF:+reference}; do
    if [ "$n" -eq 1 ]; then
      python "$ROOT/bench.py" --gpus 1 --steps "$STEPS" --warmup "$WARMUP" --impl "$impl" $EXTRA
    else
      timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$n" \
        --master-addr 127.0.0.1 --master-port $((29600 + n)) "$ROOT/bench.py" --gpus "$n" \
        --steps "$STEPS" --warmup "$WARMUP" --impl "$impl" $EXTRA
    fi
  done
done
