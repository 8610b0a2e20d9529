"""Build the in-tree native libraries of fugatensor_b200.

    python -m fugatensor_b200.build        (or: python fugatensor_b200/build.py)

Produces, next to this file:
  libfgt.so   the C-ABI backend (include/fgt.h): planner, kernel generator,
              NVRTC compilation for sm_100a, driver-API launches, NCCL (dlopen).
  _native     the Python extension (pybind11) over libfgt's prepared programs:
              the engine's cache-hit dispatch (CUDA graph replay).
The device template library (csrc/fgt_device.cuh) is embedded into libfgt.so
as text for NVRTC, and is also compiled once by nvcc for sm_100a here so
that a template error is caught at build time rather than at first use.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
LIB = PKG / "libfgt.so"

CPP_SOURCES = ["fgt_graph.cpp", "fgt_plan.cpp", "fgt_codegen.cpp", "fgt_runtime.cpp"]
CU_SOURCES = ["fgt_noalloc.cu"]
HEADERS = ["fgt_internal.h", "fgt_plan.h", "fgt_driver.h", "fgt_device.cuh"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError("build step failed: " + " ".join(map(str, cmd)) + "\n" + proc.stdout)
    return proc.stdout


def _embed_device_library() -> Path:
    text = (CSRC / "fgt_device.cuh").read_text()
    delim = "FGTDEV"
    assert f"){delim}\"" not in text
    out = BUILD / "fgt_device_src.cpp"
    body = ("// generated from csrc/fgt_device.cuh by build.py\n"
            f"extern const char* const fgt_device_library_source;\n"
            f"const char* const fgt_device_library_source = R\"{delim}(\n{text}\n){delim}\";\n")
    if not out.exists() or out.read_text() != body:
        out.write_text(body)
    return out


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _check_device_library():
    """nvcc compile of the device library for sm_100a (build-time check)."""
    probe = BUILD / "fgt_device_check.cu"
    probe.write_text(
        '#include "fgt_device.cuh"\n'
        'extern "C" __global__ void fgt_device_check(const float* x, float* y, const fgt_u16* h, long long n) {\n'
        '  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;\n'
        '  if (i * 4 + 3 >= n) return;\n'
        '  float v[4]; fgt_vload(v, x + i * 4);\n'
        '  float a = fgt_fmax(v[0], v[1]) + fgt_rnd_bf16(v[2]) + fgt_f16_to_f32(h[i]) + fgt_i64_to_bf16v(i);\n'
        '  a += fgt_f64_to_f32_odd((double)v[3]) + (float)fgt_ifloordiv<int>((int)i, 3, -2147483647 - 1);\n'
        '  a += fgt_arg_better_f<true>(v[0], 0, v[1], 1) ? 1.0f : 0.0f;\n'
        '  a += fgt_shfl_xor(a, 1);\n'
        '  float o[4] = {a, a, a, a}; fgt_vstore(y + i * 4, o);\n'
        '}\n')
    obj = BUILD / "fgt_device_check.o"
    if _stale(obj, [CSRC / "fgt_device.cuh", probe]):
        _run([str(CUDA / "bin" / "nvcc"), *GENCODE, "-lineinfo", "-O3", "-fmad=false", "-std=c++17",
              f"-I{CSRC}", "-c", str(probe), "-o", str(obj)])


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    embedded = _embed_device_library()
    _check_device_library()
    deps = [CSRC / f for f in CPP_SOURCES + HEADERS] + [ROOT / "include" / "fgt.h", embedded]
    objs = []
    for src in CPP_SOURCES + [embedded]:
        src = Path(src) if isinstance(src, Path) else CSRC / src
        obj = BUILD / (src.stem + ".o")
        if _stale(obj, [src] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "fgt.h"]):
            _run(["g++", "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wno-unused-function", f"-I{ROOT / 'include'}",
                  f"-I{CSRC}", f"-I{CUDA / 'include'}", f'-DFGT_CUDA_LIB_DIR="{CUDA / "lib64"}"', "-c", str(src),
                  "-o", str(obj)])
        objs.append(obj)
    # statically compiled kernels (nvcc, sm_100a)
    for src in CU_SOURCES:
        src = CSRC / src
        obj = BUILD / (src.stem + ".o")
        if _stale(obj, [src, CSRC / "fgt_device.cuh", CSRC / "fgt_driver.h", ROOT / "include" / "fgt.h"]):
            _run([str(CUDA / "bin" / "nvcc"), *GENCODE, "-lineinfo", "-O3", "-fmad=false", "-std=c++17",
                  "-Xcompiler", "-fPIC", f"-I{ROOT / 'include'}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)])
        objs.append(obj)
    if _stale(LIB, objs + deps):
        _run(["g++", "-shared", "-o", str(LIB), *map(str, objs), f"-L{CUDA / 'lib64'}", "-lcudart_static",
              "-lrt", "-ldl", "-lpthread", f"-Wl,-rpath,{CUDA / 'lib64'}", "-Wl,--no-undefined"])
    native = _build_native()
    if verbose:
        print(f"built {LIB}")
        print(f"built {native}")
    return LIB


def _build_native() -> Path:
    """The pybind11 extension _native, linked to libfgt.so beside it."""
    import sysconfig
    import pybind11
    out = PKG / ("_native" + sysconfig.get_config_var("EXT_SUFFIX"))
    src = CSRC / "fgt_native.cpp"
    if _stale(out, [src, LIB, ROOT / "include" / "fgt.h"]):
        _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", f"-I{pybind11.get_include()}",
              f"-I{sysconfig.get_paths()['include']}", f"-I{ROOT / 'include'}", str(src), "-o", str(out),
              f"-L{PKG}", "-lfgt", "-Wl,-rpath,$ORIGIN"])
    return out


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
