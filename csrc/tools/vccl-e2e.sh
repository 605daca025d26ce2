#!/usr/bin/env bash
# SPDX-License-Identifier: Apache-2.0
# Single-node bring-up check: run vccl-bench with --check for every op at
# 1, 2, 4 and 8 ranks (one forked rank per GPU), each run on a fresh
# VCCL_COMM_ID port so a previous run's socket cannot collide with it.  On a
# node without GPUs it checks the host data plane at 1, 2 and 4 ranks
# (VCCL_E2E_HOST_RANKS raises the count).
#
#   csrc/tools/vccl-e2e.sh [max bytes] [iters]          (defaults 64M, 20)
#
# Inside the bring-up kit (`make kit`) the script sits next to vccl-bench and
# uses that one; in the source tree it uses the built one.
set -euo pipefail
self=$(cd "$(dirname "$0")" && pwd)
if [ -x "$self/vccl-bench" ]; then
  bench=$self/vccl-bench
else
  bench=$(cd "$self/../.." && pwd)/vkccl_b200/_native/bin/vccl-bench
fi
max=${1:-64M}
iters=${2:-20}
ngpu=$( (nvidia-smi -L 2>/dev/null || true) | wc -l)
port=${VCCL_PORT:-5555}
export VCCL_SOCKET_ADDR=${VCCL_SOCKET_ADDR:-127.0.0.1}
# Without GPUs (or with VCCL_E2E_HOST=1) the same checks run on host buffers
# over the host data plane, one forked rank per slot.
mode=()
if [ "$ngpu" -eq 0 ] || [ "${VCCL_E2E_HOST:-0}" = 1 ]; then
  mode=(--host)
  ngpu=${VCCL_E2E_HOST_RANKS:-4}
fi
status=0
for n in 1 2 4 8; do
  [ "$n" -le "$ngpu" ] || continue
  for op in allreduce allgather reducescatter broadcast; do
    port=$((port + 1))
    if ! VCCL_COMM_ID=127.0.0.1:$port "$bench" --launch "$n" "${mode[@]}" --op "$op" -b 8 -e "$max" -f 4 \
         --iters "$iters" --check > /tmp/vccl-e2e-$n-$op.log 2>&1; then
      echo "FAIL n=$n $op ${mode[*]} (see /tmp/vccl-e2e-$n-$op.log)"; status=1
    else
      echo "ok   n=$n $op ${mode[*]}"
    fi
  done
done
exit $status
