# Shared settings of the launch scripts (sourced).  Override any of them from the environment:
#   NPROC (GPUs per node), NNODES, NODE_RANK, MASTER_ADDR, MASTER_PORT, DATASET_DIR, DTYPE, EXTRA
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)"
NPROC=${NPROC:-8}
NNODES=${NNODES:-1}
NODE_RANK=${NODE_RANK:-0}
MASTER_ADDR=${MASTER_ADDR:-127.0.0.1}
MASTER_PORT=${MASTER_PORT:-29500}
DATASET_DIR=${DATASET_DIR:-/dataset}
DTYPE=${DTYPE:-bf16}
if [ "$NNODES" -gt 1 ]; then
  RUN="python -m torch.distributed.run --nnodes=$NNODES --nproc-per-node=$NPROC --rdzv-backend=c10d \
--rdzv-id=${RDZV_ID:-revpp} --rdzv-endpoint=$MASTER_ADDR:$MASTER_PORT"
else
  RUN="python -m torch.distributed.run --nnodes=1 --nproc-per-node=$NPROC --master-addr=$MASTER_ADDR \
--master-port=$MASTER_PORT"
fi
