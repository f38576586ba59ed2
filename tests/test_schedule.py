"""The decode kernel's weight-stream schedule, checked on the CPU.

tests/cpp/schedule_test.cu compiles whispereacp_b200/csrc/schedule.h (host
code: the per-CTA lists of units the producer warp streams through its
shared-memory ring) and builds schedules for op lists shaped like the
decoder's at tiny.en, base.en, small.en, medium.en and large-v3 sizes: the
few-row form (fused cross query, fc2 split into K parts, the 2-token prompt),
the batched mma.sync form (several row tiles, tiles larger than a stage) and
the tensor-core form (K splits, one and two row groups, the tcgen05 logits).
It checks that every unit is 16-byte aligned and fits a stage (the bulk
copy's rules), that all CTAs' units together read each weight matrix, the
token table and each window's cross keys exactly as often as the ops consume
them -- the basis of the bench's algorithmic bytes -- and that each op's L2
prefetches go to one CTA each.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(ROOT, "tests", "cpp", "schedule_test.cu")


def test_the_weight_stream_schedule_reads_every_byte_as_often_as_the_ops_do(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc is not installed")
    program = os.path.join(str(tmp_path), "schedule_test")
    build = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O1", "-ccbin", "g++",
                            "--expt-relaxed-constexpr", "-o", program, SOURCE], capture_output=True, text=True)
    if build.returncode != 0:
        pytest.fail(build.stderr)
    run = subprocess.run([program], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
