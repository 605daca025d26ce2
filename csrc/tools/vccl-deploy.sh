#!/usr/bin/env bash
# SPDX-License-Identifier: Apache-2.0
# Copy a built libvccl.so (and the tools) to a node, keeping a backup and
# swapping atomically so running jobs keep their mapped copy (the
# reference's tools/deploy.sh does the same for its library alone).
#
#   csrc/tools/vccl-deploy.sh <host> [<remote dir>]     (default /opt/vkccl_b200)
#
# The remote user is VCCL_SSH_USER (default root) unless <host> names one
# (user@host); VCCL_SSH and VCCL_SCP replace the ssh and scp commands (for
# example to add -i <key> or a jump host).  Consumers can instead point
# VCCL_LIBRARY at any copy of the library without deploying it.
set -euo pipefail
host=${1:?usage: vccl-deploy.sh <host> [<remote dir>]}
dest=${2:-/opt/vkccl_b200}
case $host in
  *@*) target=$host ;;
  *) target=${VCCL_SSH_USER:-root}@$host ;;
esac
ssh_cmd=${VCCL_SSH:-ssh}
scp_cmd=${VCCL_SCP:-scp}
here=$(cd "$(dirname "$0")/../.." && pwd)
lib=$here/vkccl_b200/_native/libvccl.so
[ -f "$lib" ] || { echo "build first: make -j" >&2; exit 1; }
stamp=$(date +%Y%m%d%H%M%S)
$ssh_cmd "$target" "mkdir -p '$dest/bin'"
$scp_cmd -q "$lib" "$target:$dest/libvccl.so.new.$stamp"
$scp_cmd -q "$here"/vkccl_b200/_native/bin/* "$target:$dest/bin/"
$ssh_cmd "$target" "cd '$dest' && { [ -f libvccl.so ] && cp -p libvccl.so libvccl.so.bak.$stamp || true; } && mv -f libvccl.so.new.$stamp libvccl.so"
echo "deployed to $target:$dest"
echo "roll back: $ssh_cmd $target \"cd '$dest' && mv -f libvccl.so.bak.$stamp libvccl.so\" (if a previous library existed)"
