"""Sharded full-array reductions over 2 GPUs of one node (one process per
GPU, NCCL all_reduce of the per-GPU partials) against the whole-array
oracle.  Skipped when fewer than 2 GPUs are visible."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("n_total", [(1 << 24) + 5, 3])
def test_two_gpu_sharded_reductions_match_oracle(tmp_path, n_total):
    out = tmp_path / "result.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", str(HERE / "_sharded_worker.py"), str(out),
           str(n_total)]
    proc = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    got = json.loads(out.read_text())
    assert got["world"] == 2
    x = orc.uniform_f32(n_total, seed=99)
    xi = orc.uniform_i32(n_total, seed=99, lo=-1000, hi=1000)
    exact, abs_sum = orc.sum_f32_exact(x)
    v, idx = orc.argmax_f32(x)
    for r in got["results"]:
        assert abs(r["sum_f32"] - exact) <= 1e-5 * abs_sum
        assert r["sum_i32"] == orc.sum_i32(xi)
        assert r["argmax_packed"] == orc.argmax_packed_key(v, idx)
        t = r["typed"]
        assert t["u32"] == orc.sum_u32(xi.view(np.uint32))
        assert t["e4m3"] == orc.sum_typed_exact("e4m3", (xi & 0x7E).astype(np.uint8))[0]  # exact
        h_exact, h_abs = orc.sum_typed_exact("f16", (xi & 0x3BFF).astype(np.uint16))
        assert abs(t["f16"] - h_exact) <= 1e-6 * h_abs
        for dtype, arr in (("u32", xi.view(np.uint32)), ("f16", (xi & 0x3BFF).astype(np.uint16)),
                           ("f64", x.astype(np.float64))):
            i, _ = orc.argmax_typed(dtype, arr)
            assert t[f"argmax_{dtype}"][1] == i, dtype
    # batched steps with launch overlap: the same results as the plain calls
    for r in got["results"]:
        for b in got["batched"]:
            assert b == [r["sum_f32"], r["sum_i32"], r["argmax_packed"]]
    # order-fixed sums: bit-identical to the single-array restatement
    want_f32, _ = orc.sum_ordered("f32", x)
    want_bf16, _ = orc.sum_ordered("bf16", orc.f32_to_bf16(x))
    for r in got["ordered"]:
        assert np.float64(r["f32"]).view(np.uint64) == np.float64(want_f32).view(np.uint64)
        assert np.float64(r["bf16"]).view(np.uint64) == np.float64(want_bf16).view(np.uint64)


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_argmax_past_32_bit_indices(tmp_path):
    """2^32 + 2^20 + 7 elements: the partial records are gathered (the packed
    key has no room for the index) and the lowest index of the maximum,
    past 2^32 on rank 1, wins for f32 and bf16."""
    out = tmp_path / "wide.json"
    n_total = (1 << 32) + (1 << 20) + 7
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", str(HERE / "_sharded_wide_worker.py"), str(out),
           str(n_total)]
    proc = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    got = json.loads(out.read_text())
    assert got["world"] == 2
    for r in got["results"]:
        assert r["f32"] == [1000.0, (1 << 32) + 50]
        assert r["bf16"] == [1000.0, (1 << 32) + 50]


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_rank_leaving_between_steps(tmp_path):
    """Rank 1 leaves after step 1 (announced, nothing in flight); rank 0
    raises RankFailure on the host before launching step 2, within a second,
    and then aborts its communicator (NCCL's abort measured 1.2 s on B200)."""
    out = tmp_path / "leave.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", str(HERE / "_sharded_leave_worker.py"), str(out)]
    proc = subprocess.run(["timeout", "-k", "30", "180"] + cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    got = json.loads(out.read_text())
    x = orc.uniform_f32(1 << 24, seed=5)
    exact, abs_sum = orc.sum_f32_exact(x)
    assert abs(got["first"] - exact) <= 1e-5 * abs_sum
    assert got["outcome"] == "RankFailure" and got["elapsed"] < 1.0
    assert got["abort_s"] is not None and got["abort_s"] < 30.0
