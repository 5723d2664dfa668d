"""In-tree build of the native libraries (no JIT cache, nothing installed).

  sion_b200/libfelix_b200.so   kernels (sm_100a) + C ABI + felix:: C++ API
  sion_b200/_sion.<abi>.so     sion:: LibTorch wrappers + Python module

Usage: python -m sion_b200.build [--force]
Both artefacts are rebuilt only when a source is newer than the output.
nvcc cross-compiles for sm_100a without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import re
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INC = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfelix_b200.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["felix_c.cu", "sgemm_sm100.cu", "hgemm_sm100.cu", "flash_attn_sm100.cu",
              "topk_sm100.cu", "flash_attn_bwd_sm100.cu"]
CPP_SOURCES = ["felix_api.cpp"]
HEADERS = ["sm100_ptx.cuh", "felix_internal.h"]

NVCC_FLAGS = [
    "-std=c++20", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def _ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def ext_path() -> str:
    return os.path.join(PKG, "_sion" + _ext_suffix())


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> str:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


# The attention forward kernel moves registers between its warpgroups with
# setmaxnreg; the split is computed for a launch count of 168 registers per
# thread (flash_attn_sm100.cu kRegsLaunch). The host refuses to launch a build
# whose count differs; this check reports it at build time instead.
FA_REGS_LAUNCH = 168


def check_attention_registers(ptxas_log: str) -> None:
    """Raise if ptxas gave the register-split forward kernel another count."""
    cur = None
    for line in ptxas_log.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            cur = m.group(1)
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m and cur and "flash_attn_fwd_kernel" in cur:
            if int(m.group(1)) != FA_REGS_LAUNCH:
                raise RuntimeError(
                    f"{cur}: ptxas used {m.group(1)} registers per thread; the attention "
                    f"kernel's setmaxnreg split assumes {FA_REGS_LAUNCH} (build with "
                    f"-DFELIX_FA_REGSPLIT=0 or adjust kRegsLaunch)")


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, h) for h in HEADERS]
    for d, _, fs in os.walk(INC):
        hs += [os.path.join(d, f) for f in fs]
    return hs


def build_felix(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for s in CU_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + hdrs):
            extra = ["-Xptxas", "-v"] if s == "flash_attn_sm100.cu" else []
            jobs.append([NVCC, *NVCC_FLAGS, *extra, f"-I{INC}", "-c", src, "-o", obj])
    for s in CPP_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + hdrs):
            jobs.append(["g++", "-std=c++20", "-O2", "-fPIC",
                         f"-I{INC}", f"-I{CUDA_HOME}/include",
                         "-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        logs = list(ex.map(_run, jobs))
    for job, log in zip(jobs, logs):
        if "-Xptxas" in job:
            check_attention_registers(log)
    if force or jobs or _newer(LIB, objs):
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
              "-cudart", "static", "-o", LIB, *objs, "-ldl"])
    return LIB


def build_ext(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    out = ext_path()
    src = os.path.join(CSRC, "sion_torch.cpp")
    if not (force or _newer(out, [src, LIB] + _headers())):
        return out
    os.makedirs(BUILD, exist_ok=True)
    incs = cpp_extension.include_paths(device_type="cuda") if "device_type" in \
        cpp_extension.include_paths.__code__.co_varnames else cpp_extension.include_paths(cuda=True)
    libdirs = cpp_extension.library_paths(device_type="cuda") if "device_type" in \
        cpp_extension.library_paths.__code__.co_varnames else cpp_extension.library_paths(cuda=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    py_inc = sysconfig.get_paths()["include"]
    cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_sion",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-I{INC}", f"-I{py_inc}", f"-I{CUDA_HOME}/include"]
    cmd += [f"-I{i}" for i in incs]
    cmd += [src, "-o", out, f"-L{PKG}", "-lfelix_b200", "-Wl,-rpath,$ORIGIN"]
    cmd += [f"-L{d}" for d in libdirs]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_felix(force)
    build_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIB)
    print(ext_path())
