"""In-tree build of libaexis_cuda.so for sm_100a (nvcc, no JIT cache).

The library is plain CUDA C++ behind a C ABI (include/aexis_cuda.h); torch is
not linked. Objects go to aiimage_b200/_build/, the shared library next to this
file so it travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libaexis_cuda.so")
SOURCES = ["abi.cu", "k_gemv.cu", "k_gemv_stream.cu", "k_gemv_mma.cu", "k_misc.cu", "k_decoder.cu", "k_noalloc.cu", "k_gemm_tc.cu", "k_topk.cu", "k_batch.cu", "k_decoder_persist.cu", "k_batch_attn.cu", "k_recurrent.cu", "k_sample.cu", "k_kvstate.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xptxas", "-v",
         "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: cannot build libaexis_cuda")


def _deps() -> list[str]:
    inc = os.path.join(ROOT, "include", "aexis_cuda.h")
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))] + [inc]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, obj: str, log: str) -> None:
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stderr[-4000:]}")


def build_native(force: bool = False, jobs: int | None = None) -> str:
    """Compile and link libaexis_cuda.so if any source is newer than it."""
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps()
    headers = [d for d in deps if d.endswith((".h", ".cuh"))]
    todo = []
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            todo.append((src, obj, obj + ".log"))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda a: _compile(*a), todo))
    if force or todo or _stale(LIB, objs):
        # --no-undefined: a declaration without a definition fails here, not at load time.
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--no-undefined", "-o", LIB, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError("link failed:\n" + res.stderr[-4000:])
    return LIB


if __name__ == "__main__":
    print(build_native(force=True))
