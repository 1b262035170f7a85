#!/usr/bin/env bash
# Launch a training run: one process per GPU, torch.distributed over NCCL.
#
#   deploy/launch.sh <gpus_per_node> <config.toml> [train.py arguments...]
#
# Single node (the default): torchrun on this host with the rendezvous on 127.0.0.1.
# Several nodes: set NODES="host0 host1 ..." (the first is the rendezvous host) and run this script
# on every node with NODE_RANK set, or run it inside an LSF job, where the allocated hosts are read
# from LSB_MCPU_HOSTS and the per-node commands are started with blaunch.
#
# Environment set for every rank: PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True (activation
# sizes vary between crops; expandable segments stop the caching allocator from fragmenting),
# OMP_NUM_THREADS=4 (dataloader workers each get a few host threads), NCCL_DEBUG=WARN unless set.
# MIA_TRAIN (repository root, default: this script's parent) and PYTHON (default: python3) may be
# overridden.
set -euo pipefail

GPUS=${1:?usage: launch.sh <gpus_per_node> <config.toml> [train.py arguments...]}
CONFIG=${2:?usage: launch.sh <gpus_per_node> <config.toml> [train.py arguments...]}
shift 2
ROOT=${MIA_TRAIN:-$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)}
PY=${PYTHON:-python3}
EXTRA=("$@")

env_exports() {
  cat <<ENV
export PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True
export OMP_NUM_THREADS=\${OMP_NUM_THREADS:-4}
export NCCL_DEBUG=\${NCCL_DEBUG:-WARN}
ENV
}

if [[ -n "${LSB_MCPU_HOSTS:-}" && -n "${LSB_JOBID:-}" ]]; then
  read -r -a fields <<< "$LSB_MCPU_HOSTS"
  hosts=()
  for ((i = 0; i < ${#fields[@]}; i += 2)); do hosts+=("${fields[i]}"); done
  port=$((29400 + LSB_JOBID % 1000))
  echo "launch: LSF job $LSB_JOBID, ${#hosts[@]} node(s) x $GPUS GPU(s), rendezvous ${hosts[0]}:$port"
  cmd="cd '$ROOT' && $(env_exports | tr '\n' ';') exec $PY -m torch.distributed.run --nnodes=${#hosts[@]} \
--nproc-per-node=$GPUS --rdzv-backend=c10d --rdzv-id=$LSB_JOBID --rdzv-endpoint=${hosts[0]}:$port \
src/train.py --config '$CONFIG' ${EXTRA[*]:-}"
  exec blaunch -z "${hosts[*]}" bash -c "$cmd"
fi

cd "$ROOT"
eval "$(env_exports)"
if [[ -n "${NODES:-}" ]]; then
  read -r -a hosts <<< "$NODES"
  : "${NODE_RANK:?set NODE_RANK (0..$((${#hosts[@]} - 1))) on every node}"
  port=${MASTER_PORT:-29400}
  echo "launch: node $NODE_RANK of ${#hosts[@]} x $GPUS GPU(s), rendezvous ${hosts[0]}:$port"
  exec "$PY" -m torch.distributed.run --nnodes="${#hosts[@]}" --node-rank="$NODE_RANK" --nproc-per-node="$GPUS" \
    --rdzv-backend=c10d --rdzv-id="${RUN_ID:-mia}" --rdzv-endpoint="${hosts[0]}:$port" \
    src/train.py --config "$CONFIG" "${EXTRA[@]}"
fi
port=${MASTER_PORT:-29500}
echo "launch: 1 node x $GPUS GPU(s), rendezvous 127.0.0.1:$port"
exec "$PY" -m torch.distributed.run --nnodes=1 --nproc-per-node="$GPUS" --master-addr 127.0.0.1 \
  --master-port "$port" src/train.py --config "$CONFIG" "${EXTRA[@]}"
