"""Build the in-tree CUDA library ``_lib/liborthocache_b200.so`` for sm_100a.

Each ``csrc/*.cu`` translation unit is compiled by ``nvcc`` in parallel and
linked into one shared library whose exported symbols are the C ABI of
``include/orthocache_b200.h``.  Objects are kept beside the library and a
translation unit is recompiled only when it or a header changed.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(OUT_DIR, "liborthocache_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build orthocache_gpu_b200")
    return p


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(f) <= t for f in _deps())


def build(force: bool = False, verbose: bool = False, jobs: int | None = None, out_dir: str | None = None,
          defines: tuple = ()) -> str:
    """Compile (if needed) and return the path of the shared library.

    ``out_dir`` / ``defines`` build a variant elsewhere (e.g. with OC_TRACE,
    the diagnostics timeline) without touching the in-tree library.
    """
    out = out_dir or OUT_DIR
    lib_path = os.path.join(out, os.path.basename(LIB))
    if not force and up_to_date(lib_path):
        return lib_path
    os.makedirs(out, exist_ok=True)
    extra = [f"-D{d}" for d in defines]
    cc = nvcc()
    objs = []

    headers = [f for f in _deps() if not f.endswith(".cu")]
    newest_header = max(os.path.getmtime(f) for f in headers)

    def compile_one(src):
        obj = os.path.join(out, os.path.basename(src)[:-3] + ".o")
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header):
            return obj
        cmd = [cc, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = lib_path + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib_path)
    return lib_path


BINDING = os.path.join(OUT_DIR, "oc_torch.so")


def build_binding(force: bool = False, verbose: bool = False) -> str:
    """Compile the pybind11 binding csrc/oc_torch.cpp (C++, no GPU code) into _lib/oc_torch.so.

    It links liborthocache_b200.so from the same directory (rpath $ORIGIN).
    """
    src = os.path.join(CSRC, "oc_torch.cpp")
    deps = [src, LIB, os.path.join(ROOT, "include", "orthocache_b200.h")]
    if not force and os.path.exists(BINDING) and all(os.path.getmtime(d) <= os.path.getmtime(BINDING) for d in deps):
        return BINDING
    from torch.utils import cpp_extension
    tmp = os.path.join(OUT_DIR, "oc_torch_build")
    os.makedirs(tmp, exist_ok=True)
    cpp_extension.load(name="oc_torch", sources=[src], build_directory=tmp, verbose=verbose,
                       extra_cflags=["-O2"], extra_ldflags=[f"-L{OUT_DIR}", "-lorthocache_b200",
                                                           "'-Wl,-rpath,$$ORIGIN:$$ORIGIN/..'"],
                       is_python_module=True)
    shutil.copy2(os.path.join(tmp, "oc_torch.so"), BINDING + ".tmp")
    os.replace(BINDING + ".tmp", BINDING)
    return BINDING


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_binding(force="--force" in sys.argv))
