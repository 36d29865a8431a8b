#!/usr/bin/env bash
# Detached multi-node launcher: one torchrun per host over ssh, logs and pid files
# per host, plus status / stop / sync.  Counterpart of the reference's
# scripts/launch_multinode*_detached.sh, status_*.sh, stop_*.sh and sync_*.sh.
#
#   HOSTS="node0 node1" NPROC=8 MASTER_ADDR=10.0.0.1 \
#     examples/launch_multinode.sh start examples/train_qlora.py --model qwen2.5-32b --mode gather
#   HOSTS="node0 node1" examples/launch_multinode.sh status
#   HOSTS="node0 node1" examples/launch_multinode.sh stop
#   HOSTS="node0 node1" examples/launch_multinode.sh sync        # rsync this repository to REMOTE_DIR
#
# The first host is node rank 0 and must be reachable at MASTER_ADDR:MASTER_PORT.
# DRY_RUN=1 prints every remote command instead of running it.
set -euo pipefail

HOSTS=${HOSTS:-localhost}
NPROC=${NPROC:-8}
MASTER_ADDR=${MASTER_ADDR:-127.0.0.1}
MASTER_PORT=${MASTER_PORT:-29500}
REMOTE_DIR=${REMOTE_DIR:-$(cd "$(dirname "$0")/.." && pwd)}
PYTHON=${PYTHON:-python}
RUN_ID=${RUN_ID:-zeroq_${MASTER_PORT}}
LOG_DIR=${LOG_DIR:-/tmp}
RUN_TIMEOUT=${RUN_TIMEOUT:-86400}
# NCCL settings passed to every rank (extend with NCCL_EXTRA="K=V K2=V2")
NCCL_ENV=${NCCL_ENV:-"NCCL_ASYNC_ERROR_HANDLING=1 TORCH_NCCL_BLOCKING_WAIT=0"}
NCCL_EXTRA=${NCCL_EXTRA:-}
DRY_RUN=${DRY_RUN:-0}

SSH_OPTS=(-o BatchMode=yes -o StrictHostKeyChecking=accept-new -o ServerAliveInterval=10
          -o ServerAliveCountMax=3 -T)

read -r -a HOST_LIST <<< "$HOSTS"
NNODES=${#HOST_LIST[@]}

remote() {  # remote <host> <command string>
  local host=$1; shift
  if [[ "$DRY_RUN" == "1" ]]; then
    echo "[$host] $*"
  elif [[ "$host" == "localhost" || "$host" == "127.0.0.1" ]]; then
    bash -c "$*"
  else
    ssh "${SSH_OPTS[@]}" "$host" "$*"
  fi
}

files_for() {  # files_for <node rank> -> "<log> <pid>"
  echo "$LOG_DIR/${RUN_ID}_node$1.log $LOG_DIR/${RUN_ID}_node$1.pid"
}

cmd_start() {
  [[ $# -ge 1 ]] || { echo "usage: $0 start <script.py> [args...]" >&2; exit 2; }
  local script=$1; shift
  local args
  args=$(printf '%q ' "$@")
  for i in "${!HOST_LIST[@]}"; do
    read -r log pid <<< "$(files_for "$i")"
    # setsid: the launcher leads its own process group (pgid = recorded pid), so
    # stop can signal torchrun and its workers without touching anything else
    local run="cd $REMOTE_DIR && env $NCCL_ENV $NCCL_EXTRA setsid nohup timeout -k 60 $RUN_TIMEOUT \
$PYTHON -m torch.distributed.run --nnodes $NNODES --node-rank $i --nproc-per-node $NPROC \
--master-addr $MASTER_ADDR --master-port $MASTER_PORT $script $args > $log 2>&1 < /dev/null & echo \$! > $pid"
    remote "${HOST_LIST[$i]}" "$run"
    echo "node $i (${HOST_LIST[$i]}): log $log"
  done
}

cmd_status() {
  for i in "${!HOST_LIST[@]}"; do
    read -r log pid <<< "$(files_for "$i")"
    remote "${HOST_LIST[$i]}" "if [ -f $pid ] && kill -0 \$(cat $pid) 2>/dev/null; then \
echo 'node $i: running (pid '\$(cat $pid)')'; else echo 'node $i: not running'; fi; \
[ -f $log ] && tail -n 3 $log || true"
  done
}

cmd_stop() {
  for i in "${!HOST_LIST[@]}"; do
    read -r log pid <<< "$(files_for "$i")"
    # the recorded pid leads the launcher's own process group (see start)
    remote "${HOST_LIST[$i]}" "if [ -f $pid ]; then p=\$(cat $pid); \
kill -TERM -- -\$p 2>/dev/null || true; rm -f $pid; echo 'node $i: stopped'; \
else echo 'node $i: no pid file'; fi"
  done
}

cmd_sync() {
  for i in "${!HOST_LIST[@]}"; do
    local host=${HOST_LIST[$i]}
    [[ "$host" == "localhost" || "$host" == "127.0.0.1" ]] && continue
    if [[ "$DRY_RUN" == "1" ]]; then
      echo "[$host] rsync -az --exclude .git $REMOTE_DIR/ $host:$REMOTE_DIR/"
    else
      rsync -az --exclude .git "$REMOTE_DIR/" "$host:$REMOTE_DIR/"
    fi
  done
}

sub=${1:-}
shift || true
case "$sub" in
  start) cmd_start "$@" ;;
  status) cmd_status ;;
  stop) cmd_stop ;;
  sync) cmd_sync ;;
  *) echo "usage: $0 {start <script> [args]|status|stop|sync}" >&2; exit 2 ;;
esac
