"""Build recipe for libmvb200.so (sm_100a) — nvcc, in-tree.

The shared library is written to ``lib/libmvb200.so`` beside this file so it
travels with the source tree to the GPU host; nothing is installed into
site-packages and there is no JIT cache.  ``build_native()`` recompiles only
the objects whose sources (or shared headers) changed.

Run directly to build:  python <package-dir>/build.py [--force] [--verbose]
"""

from __future__ import annotations

import concurrent.futures as _cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG_DIR), "include")
LIB_DIR = os.path.join(PKG_DIR, "lib")
OBJ_DIR = os.path.join(LIB_DIR, "obj")
LIB_PATH = os.path.join(LIB_DIR, "libmvb200.so")

SOURCES = ["kv_write.cu", "decode_fma.cu", "decode_mma.cu", "decode_stream.cu", "decode_sched.cu", "capi.cu",
           "decode_noalloc.cu", "gather.cu", "rope_write.cu", "step_metadata.cu", "prefill_mma.cu"]
HEADERS = ["mvb_common.cuh", "decode_common.cuh", "mma_tile.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmvb200.so")
    return cand


def _deps_mtime() -> float:
    paths = [os.path.join(CSRC, h) for h in HEADERS]
    paths.append(os.path.join(INCLUDE, "mini_vllm_b200.h"))
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, verbose: bool, force: bool) -> str:
    obj = os.path.join(OBJ_DIR, os.path.splitext(src)[0] + ".o")
    src_path = os.path.join(CSRC, src)
    if (
        not force
        and os.path.exists(obj)
        and os.path.getmtime(obj) >= max(os.path.getmtime(src_path), _deps_mtime())
    ):
        return obj
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-c", src_path, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build_native(force: bool = False, verbose: bool = False) -> str:
    """Compile every CUDA source for sm_100a and link ``lib/libmvb200.so``."""
    os.makedirs(OBJ_DIR, exist_ok=True)
    with _cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, force), SOURCES))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < newest:
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-Xlinker", "-soname=libmvb200.so", "-o", LIB_PATH, *objs,
               "-lrt", "-ldl", "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link of libmvb200.so failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


TRACE_LIB_PATH = os.path.join(LIB_DIR, "libmvb200_trace.so")


def build_trace(force: bool = False) -> str:
    """Link ``lib/libmvb200_trace.so``: the library with the stream decode
    compiled with ``-DMVB_STREAM_TRACE`` (per-warp %globaltimer stamps and the
    ``mvb_trace_clear`` / ``mvb_trace_read`` calls; ``bench.py --op trace``
    loads it).  The other objects are the product's."""
    build_native(force=force)
    src = os.path.join(CSRC, "decode_stream.cu")
    obj = os.path.join(OBJ_DIR, "decode_stream_trace.o")
    if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), _deps_mtime()):
        cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-DMVB_STREAM_TRACE", "-I", INCLUDE, "-c", src, "-o", obj]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for the trace build of decode_stream.cu:\n{res.stdout}\n{res.stderr}")
    objs = [obj if s_ == "decode_stream.cu" else os.path.join(OBJ_DIR, os.path.splitext(s_)[0] + ".o")
            for s_ in SOURCES]
    if force or not os.path.exists(TRACE_LIB_PATH) or os.path.getmtime(TRACE_LIB_PATH) < max(
            os.path.getmtime(o) for o in objs):
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-Xlinker", "-soname=libmvb200_trace.so", "-o", TRACE_LIB_PATH,
               *objs, "-lrt", "-ldl", "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link of libmvb200_trace.so failed:\n{res.stdout}\n{res.stderr}")
    return TRACE_LIB_PATH

TORCH_BINDING_SRC = os.path.join(CSRC, "torch_binding.cpp")
TORCH_BINDING_PATH = os.path.join(LIB_DIR, "_mvb_torch.so")


def build_torch_binding(force: bool = False) -> str:
    """Compile the direct Python binding of the per-step calls (g++ against
    torch's headers; links ``libmvb200.so`` from the same directory)."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    lib = build_native(force=force)
    deps = [TORCH_BINDING_SRC, os.path.join(INCLUDE, "mini_vllm_b200.h"), lib]
    if (not force and os.path.exists(TORCH_BINDING_PATH)
            and os.path.getmtime(TORCH_BINDING_PATH) >= max(os.path.getmtime(d) for d in deps)):
        return TORCH_BINDING_PATH
    torch_lib = cpp_extension.library_paths()[0]
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           "-DTORCH_EXTENSION_NAME=_mvb_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
    for inc in cpp_extension.include_paths() + [os.path.join(cuda_home, "include"),
                                               sysconfig.get_paths()["include"], INCLUDE]:
        cmd += ["-I", inc]
    cmd += [TORCH_BINDING_SRC, "-o", TORCH_BINDING_PATH,
            "-L", torch_lib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            "-L", LIB_DIR, "-lmvb200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed for torch_binding.cpp:\n{res.stdout}\n{res.stderr}")
    return TORCH_BINDING_PATH


if __name__ == "__main__":
    print(build_native(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
    print(build_torch_binding(force="--force" in sys.argv))
