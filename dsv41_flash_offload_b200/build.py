"""Build the sm_100a C-ABI library libdsv41_b200.so in-tree with nvcc.

    python -m dsv41_flash_offload_b200.build [--verbose]

nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3, one object per source file (compiled in
parallel under _build/), then one link; the CUDA runtime is linked statically so the library only
needs the driver (and coexists with torch's own runtime).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdsv41_b200.so")
SOURCES = ["capi.cu", "permute.cu", "transform.cu", "gemv.cu", "gemm.cu", "noalloc.cu", "ep_peer.cu", "router.cu"]
HEADERS = ["common.cuh", "internal.h", "gemm.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for p in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc"):
        if p and os.path.exists(p):
            return p
    return "nvcc"


def nvcc_version(nvcc: str) -> str:
    out = subprocess.run([nvcc, "--version"], capture_output=True, text=True).stdout
    for line in out.splitlines():
        if "release" in line:
            return line.split("release")[-1].strip().split(",")[0]
    return "unknown"


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(HERE, "..", "include", "dsv41_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False, defines=(),
          lib_path: str = LIB) -> str:
    """Build the library (when a source is newer than it, or `force`). `defines` are extra -D flags
    (the kernels' compile-time launch-shape switches) and `lib_path` the output, for variants."""
    if not force and lib_path == LIB and not defines and not needs_build():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    nvcc = nvcc_path()
    ver = nvcc_version(nvcc)
    flags = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", f'-DDSV41_NVCC_VERSION="{ver}"',
             *[f"-D{d}" for d in defines]]
    if ptxas_verbose:
        flags.insert(0, "-Xptxas=-v")
    tag = os.path.splitext(os.path.basename(lib_path))[0]
    objdir = os.path.join(HERE, "_build", tag)
    os.makedirs(objdir, exist_ok=True)

    def compile_one(src):
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc, *flags, "-c", "-o", obj, os.path.join(CSRC, src)]
        if verbose:
            print(" ".join(cmd), flush=True)
        return obj, subprocess.run(cmd, capture_output=True, text=True)

    # one nvcc per source file, in parallel, then one link step
    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    for _, r in results:
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc failed building libdsv41_b200.so")
        if verbose or ptxas_verbose:
            sys.stderr.write(r.stderr)
    link = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", lib_path + ".tmp"] + [o for o, _ in results]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed linking libdsv41_b200.so")
    os.replace(lib_path + ".tmp", lib_path)
    return lib_path


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB)
