#!/usr/bin/env bash
# Launch training: one process per GPU through torch.distributed.run.
#   NGPU=8 MODULE=llama3 CONFIG=llama3_8b ./run_train.sh [--section.key value ...]
# COMM_MODE=fake_backend or local_tensor runs a single process that simulates NGPU ranks
# (configuration and sharding dry run, no collectives executed).
set -euo pipefail
NGPU=${NGPU:-8}
MODULE=${MODULE:-llama3}
CONFIG=${CONFIG:-llama3_debugmodel}
LOG_RANK=${LOG_RANK:-0}
COMM_MODE=${COMM_MODE:-}
MASTER_PORT=${MASTER_PORT:-29500}

if [[ -n "$COMM_MODE" ]]; then
  NGPU="$NGPU" LOCAL_RANK=0 exec python -m torchtitan_b200.train --module "$MODULE" --config "$CONFIG" \
    --comm.mode "$COMM_MODE" --training.steps 1 "$@"
fi
exec python -m torch.distributed.run --nnodes=1 --nproc-per-node="$NGPU" --master-addr 127.0.0.1 \
  --master-port "$MASTER_PORT" --local-ranks-filter "$LOG_RANK" --role rank --tee 3 \
  -m torchtitan_b200.train --module "$MODULE" --config "$CONFIG" "$@"
