"""Host-side failure injection and dispatch checks on CPU: the library is
pointed (FLIGHT4S_CUDA_DRIVER) at a fake CUDA driver that records launches
and returns injected errors; each scenario runs in its own process."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def fake_driver(tmp_path_factory):
    out = tmp_path_factory.mktemp("fake") / "libfakecuda.so"
    cuda_inc = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
    subprocess.run(["gcc", "-O1", "-fPIC", "-shared", f"-I{cuda_inc}", str(HERE / "fake_driver" / "fake_cuda.c"),
                    "-o", str(out)], check=True)
    return out


SCENARIOS = {
    "launch_records_geometry": {},
    "launch_error_propagates": {"FAKE_CUDA_FAIL": "cuLaunchKernelEx=719"},
    "out_of_memory": {"FAKE_CUDA_FAIL": "cuMemAlloc=2"},
    "pop_mismatch": {"FAKE_CUDA_POP_MISMATCH": "1"},
    "push_failure": {"FAKE_CUDA_FAIL": "cuCtxPushCurrent=201"},
    "jit_error_log": {"FAKE_CUDA_FAIL": "cuModuleLoadDataEx=218"},
    "invalid_arguments_never_reach_driver": {},
    "hotpath_dispatch": {},
    "host_ordered_pipeline": {},
}


@pytest.mark.parametrize("scenario", sorted(SCENARIOS))
def test_scenario(fake_driver, scenario):
    env = {k: v for k, v in os.environ.items() if not k.startswith("FAKE_CUDA_")}
    env.update(FLIGHT4S_CUDA_DRIVER=str(fake_driver), **SCENARIOS[scenario])
    proc = subprocess.run([sys.executable, str(HERE / "_fake_driver_scenarios.py"), scenario, str(fake_driver)],
                          env=env, capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
