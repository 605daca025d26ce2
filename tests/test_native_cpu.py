# SPDX-License-Identifier: Apache-2.0
"""Native control-plane suites (CPU; no GPU needed).

test_bootstrap: the reference's stray-client rendezvous test.
test_control:   lifecycle / split / ops / abort / host failure detection.
"""

import os
import subprocess

from conftest import BIN


def _run(name, timeout=300):
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_DEBUG="ERROR")
    p = subprocess.run([os.path.join(BIN, name)], env=env, capture_output=True, text=True, timeout=timeout)
    assert p.returncode == 0, p.stdout + p.stderr
    return p.stdout


def test_bootstrap_rejects_stray_client():
    assert "bootstrap-reject: OK" in _run("test_bootstrap")


def test_control_plane_suite():
    assert "control-plane: OK" in _run("test_control")


def test_control_plane_under_sanitizers():
    """Threaded bootstrap rounds, fd exchange and abort under TSan and ASan/UBSan; the host data
    plane's collectives, its sender thread and an abort racing a waiting all-reduce likewise."""
    import shutil

    if shutil.which("g++") is None:
        import pytest

        pytest.skip("no host C++ compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    subprocess.run(["make", "-s", "sanitize"], cwd=root, check=True, capture_output=True, timeout=600)
    for name in ("test_bootstrap_threads_tsan", "test_bootstrap_threads_asan"):
        out = _run(name, timeout=300)
        assert "bootstrap-threads: OK" in out
    for name in ("test_hostplane_threads_tsan", "test_hostplane_threads_asan"):
        out = _run(name, timeout=300)
        assert "hostplane-threads: OK" in out


def test_gemm_index_arithmetic():
    """Tile orders, split-K coverage, epilogue stage slots and split plans (host build of the device math)."""
    assert "tiling: OK" in _run("test_tiling")


def test_tuning_tables():
    """VCCL_TUNING_FILE parsing and rule lookup."""
    assert "tuning: OK" in _run("test_tuning")


def test_bring_up_kit(tmp_path):
    """`make kit` packs the library, tools, native tests, headers and the bring-up script; unpacked
    elsewhere, the tools find the library through their rpath."""
    import glob
    import platform
    import tarfile

    root = os.path.dirname(BIN)
    subprocess.run(["make", "kit"], cwd=os.path.dirname(os.path.dirname(root)), check=True,
                   capture_output=True, timeout=600)
    tar = os.path.join(root, f"vccl-e2e-kit-{platform.machine()}.tar.gz")
    with tarfile.open(tar) as t:
        names = set(t.getnames())
        for want in ("kit/libvccl.so", "kit/bin/vccl-bench", "kit/bin/vccl-info", "kit/bin/test_collectives",
                     "kit/bin/test_dmabuf", "kit/bin/vccl-e2e.sh", "kit/include/vccl.h"):
            assert want in names, want
        t.extractall(tmp_path, filter="data")
    # the kit is a user artefact; the test leaves none behind in the tree
    subprocess.run(["rm", "-rf", os.path.join(root, "kit"), tar], check=True)
    p = subprocess.run([str(tmp_path / "kit" / "bin" / "vccl-bench"), "--help"], capture_output=True, text=True,
                       timeout=60)
    # it loaded (libvccl.so found next to bin/, else the loader exits 127) and printed its usage
    assert p.returncode != 127 and "usage: vccl-bench" in (p.stdout + p.stderr), p.stderr
    assert glob.glob(str(tmp_path / "kit" / "include" / "vccl*.h"))


def test_deploy_script_with_fake_ssh(tmp_path):
    """csrc/tools/vccl-deploy.sh against a stand-in ssh/scp (VCCL_SSH / VCCL_SCP, the reference's
    override names) that act on a local directory: the library and tools land in place, the user
    defaults to root, and a second deploy keeps the previous library as a backup."""
    repo = os.path.dirname(os.path.dirname(os.path.dirname(BIN)))
    log = tmp_path / "log"
    ssh = tmp_path / "fake-ssh"
    ssh.write_text(f'#!/bin/sh\necho "ssh $1" >> {log}\nshift\nsh -c "$1"\n')
    scp = tmp_path / "fake-scp"
    scp.write_text('#!/bin/sh\n[ "$1" = -q ] && shift\nn=$#\ni=0\nsrcs=""\n'
                   'for a in "$@"; do i=$((i+1)); if [ $i -lt $n ]; then srcs="$srcs $a"; else dst=${a#*:}; fi; done\n'
                   f'echo "scp $dst" >> {log}\ncp $srcs "$dst"\n')
    ssh.chmod(0o755)
    scp.chmod(0o755)
    dest = tmp_path / "node"
    env = dict(os.environ, VCCL_SSH=str(ssh), VCCL_SCP=str(scp))
    script = os.path.join(repo, "csrc", "tools", "vccl-deploy.sh")
    for _ in range(2):
        p = subprocess.run(["bash", script, "node1", str(dest)], env=env, capture_output=True, text=True, timeout=120)
        assert p.returncode == 0, p.stdout + p.stderr
    assert (dest / "libvccl.so").is_file() and (dest / "bin" / "vccl-bench").is_file()
    assert any(f.name.startswith("libvccl.so.bak.") for f in dest.iterdir())
    assert "ssh root@node1" in log.read_text()


def test_vccl_info_without_gpu():
    """vccl-info on a node without GPUs: the advertised address, the IPv4 interfaces, and the note
    that communicators use the host data plane (reference: tools/vccl_info.cc surveys the node)."""
    p = subprocess.run([os.path.join(BIN, "vccl-info")], env=dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1"),
                       capture_output=True, text=True, timeout=60)
    assert p.returncode == 0, p.stderr
    assert "bootstrap / host data plane address: 127.0.0.1" in p.stdout
    assert "lo=127.0.0.1" in p.stdout
    assert "host data plane" in p.stdout.splitlines()[-1] or "device(s)" in p.stdout


def test_bring_up_script_on_host_plane():
    """csrc/tools/vccl-e2e.sh on a node without GPUs: vccl-bench --check for every op at 1, 2 and 4
    ranks over the host data plane (the reference's kit/vccl-e2e.sh bring-up role)."""
    import random

    repo = os.path.dirname(os.path.dirname(os.path.dirname(BIN)))
    env = dict(os.environ, VCCL_E2E_HOST="1", VCCL_PORT=str(20000 + random.randint(0, 20000)),
               VCCL_DEBUG="ERROR")
    p = subprocess.run(["bash", os.path.join(repo, "csrc", "tools", "vccl-e2e.sh"), "64K", "5"], env=env,
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout + p.stderr
    assert p.stdout.count("ok ") == 12, p.stdout


def test_registration_cache_protocol():
    """Registration cache: simulated ranks with their own address layouts run random call sequences
    (reuse, slices, reallocation at the same address, a rank unable to take part, application
    windows); every rank plans alike, every cached call has one window per buffer at one offset on
    every rank over the current allocation, entries never overlap or exceed the capacity; a skewed-
    offset negative control (csrc/tests/test_regcache.cc)."""
    assert "regcache: OK" in _run("test_regcache")


def test_collective_index_arithmetic():
    """Coverage and staging bounds of the staged, pipelined-NVLS and window kernels' splits, with a
    negative control for re-split rounds (csrc/tests/test_coll_index.cc)."""
    assert "all checks passed" in _run("test_coll_index")


def _run_dmabuf(args, extra_env):
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_DEBUG="ERROR", **extra_env)
    return subprocess.run([os.path.join(BIN, "test_dmabuf")] + args, env=env, capture_output=True, text=True,
                          timeout=300)


def test_dmabuf_registration_control_plane():
    """vcclCommRegisterDmaBuf's CPU-mapping route on 1 to 3 device-less forked ranks: a memfd, and a
    real dmabuf from /dev/udmabuf where the kernel has it, all-reduced and all-gathered in place
    (reference: tests/test_dmabuf.cc)."""
    for n in (1, 2, 3):
        # several device-less ranks move the mappings' bytes over the host data plane
        p = _run_dmabuf([str(n), "memfd"], {"VCCL_NO_DEVICE": "1"})
        assert p.returncode == 0 and f"dmabuf (memfd, {n} ranks): OK" in p.stdout, p.stdout + p.stderr
        p = _run_dmabuf([str(n), "udmabuf"], {"VCCL_NO_DEVICE": "1"})
        assert p.returncode in (0, 77), p.stdout + p.stderr
