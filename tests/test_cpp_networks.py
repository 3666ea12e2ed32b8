"""The C++ mirror of the reference's networks/ API (include/spo_networks.hpp) without a
GPU: it compiles warning-free against the C ABI, links against libspo_cuda.so, lays out
parameters exactly as the Python mirror does, and reports capacity errors (before
anything is enqueued) and the library's own errors as spo::networks::Error."""

import os
import shutil
import subprocess

import pytest

from spo_mojo_b200 import ffi
from spo_mojo_b200.workloads import NetSpec

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    assert os.path.exists(ffi.LIB_PATH), "build libspo_cuda.so first (python -m spo_mojo_b200.build)"
    out = str(tmp_path_factory.mktemp("cpp") / "networks_host_checks")
    libdir = os.path.dirname(ffi.LIB_PATH)
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "cpp", "networks_host_checks.cpp"), "-o", out,
           "-L", libdir, "-lspo_cuda", "-Wl,-rpath," + libdir,
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


@pytest.fixture(scope="module")
def output(program):
    r = subprocess.run([program], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout.splitlines()


def test_every_host_check_passes(output):
    fails = [line for line in output if line.startswith("FAIL")]
    assert not fails, fails
    oks = {line.split()[1] for line in output if line.startswith("ok ")}
    assert {"actor_capacity_message", "linear_forward_short_output", "linear_backward_short_dy",
            "adam_step_zero_is_refused_by_the_library", "global_clip_scale_known_answer"} <= oks


def test_layout_matches_the_python_mirror(output):
    layouts = [line for line in output if line.startswith("layout")]
    assert len(layouts) == 3
    for line in layouts:
        head, tail = line[len("layout "):].split(" : ")
        dims = tuple(int(v) for v in head.split())
        nums = tail.split()
        total = int(nums[-1])
        pairs = [(int(nums[i]), int(nums[i + 1])) for i in range(0, len(nums) - 2, 2)]
        offs, want_total = NetSpec(dims).offsets()
        assert pairs == [tuple(o) for o in offs] and total == want_total, (dims, pairs, offs)


def test_golden_program_builds(tmp_path):
    """tests/cpp/networks_golden.cpp (the reference's actor-backward goldens through the C++
    mirror; it needs a GPU to run) compiles warning-free and links."""
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    out = str(tmp_path / "networks_golden")
    libdir = os.path.dirname(ffi.LIB_PATH)
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "cpp", "networks_golden.cpp"), "-o", out,
           "-L", libdir, "-lspo_cuda", "-Wl,-rpath," + libdir,
           "-L", os.path.join(CUDA, "lib64"), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    usage = subprocess.run([out], capture_output=True, text=True, timeout=60)
    assert usage.returncode == 1 and "usage" in usage.stderr
