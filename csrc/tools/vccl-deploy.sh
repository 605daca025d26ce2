#!/usr/bin/env bash
# SPDX-License-Identifier: Apache-2.0
# Copy a built libvccl.so (and the tools) to a node, keeping a backup and
# swapping atomically so running jobs keep their mapped copy.
#
#   csrc/tools/vccl-deploy.sh <host> [<remote dir>]     (default /opt/vkccl_b200)
set -euo pipefail
host=${1:?usage: vccl-deploy.sh <host> [<remote dir>]}
dest=${2:-/opt/vkccl_b200}
here=$(cd "$(dirname "$0")/../.." && pwd)
lib=$here/vkccl_b200/_native/libvccl.so
[ -f "$lib" ] || { echo "build first: make -j" >&2; exit 1; }
stamp=$(date +%Y%m%d%H%M%S)
ssh "$host" "mkdir -p '$dest/bin'"
scp -q "$lib" "$host:$dest/libvccl.so.new.$stamp"
scp -q "$here"/vkccl_b200/_native/bin/* "$host:$dest/bin/"
ssh "$host" "cd '$dest' && { [ -f libvccl.so ] && cp -p libvccl.so libvccl.so.bak.$stamp || true; } && mv -f libvccl.so.new.$stamp libvccl.so"
echo "deployed to $host:$dest (backup libvccl.so.bak.$stamp if there was one)"
