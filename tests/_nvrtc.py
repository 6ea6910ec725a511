"""NVRTC compilation of tests/device/*.cu against include/ (the way the
reference compiles its generated kernels), for the device-header tests."""
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def compile_cubin(source_path: Path, arch: str = "sm_100a") -> bytes:
    """CUBIN of one source file; raises RuntimeError with NVRTC's log."""
    from cuda.bindings import nvrtc
    src = source_path.read_bytes()
    err, prog = nvrtc.nvrtcCreateProgram(src, source_path.name.encode(), 0, [], [])
    if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        raise RuntimeError(f"nvrtcCreateProgram: {err}")
    opts = [f"--gpu-architecture={arch}".encode(), f"-I{ROOT / 'include'}".encode(), b"-std=c++17"]
    try:
        (err,) = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            _, size = nvrtc.nvrtcGetProgramLogSize(prog)
            log = b" " * size
            nvrtc.nvrtcGetProgramLog(prog, log)
            raise RuntimeError(f"NVRTC compile failed: {log.decode(errors='replace')}")
        _, size = nvrtc.nvrtcGetCUBINSize(prog)
        cubin = b" " * size
        (err,) = nvrtc.nvrtcGetCUBIN(prog, cubin)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            raise RuntimeError(f"nvrtcGetCUBIN: {err}")
        return bytes(cubin)
    finally:
        nvrtc.nvrtcDestroyProgram(prog)
