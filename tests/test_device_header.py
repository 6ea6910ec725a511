"""include/flight4s_b200_device.cuh compiles under NVRTC for sm_100a with
only its own directory on the include path (no GPU needed)."""
from pathlib import Path

import pytest

from _nvrtc import ROOT, compile_cubin

KERNELS = Path(__file__).resolve().parent / "device" / "intrinsics_kernels.cu"


def test_header_compiles_under_nvrtc():
    pytest.importorskip("cuda.bindings.nvrtc")
    cubin = compile_cubin(KERNELS)
    assert len(cubin) > 1000


def test_header_is_self_contained():
    text = (ROOT / "include" / "flight4s_b200_device.cuh").read_text()
    assert "#include" not in text.split("*/", 1)[1]
