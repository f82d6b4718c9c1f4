"""Build libcvattn.so (sm_100a) in-tree with nvcc.

Usage:  python cosyvoice.cpp_b200/build.py [--force] [-j N]

Objects go to cosyvoice.cpp_b200/_build/ (git-ignored); the shared library is
written next to the Python bindings, cosyvoice.cpp_b200/cvattn/libcvattn.so,
so it travels with the repository snapshot to the GPU box.  The CUDA runtime
is linked statically; the driver API (tensor maps) is reached through
cudaGetDriverEntryPoint, so the library needs only libcuda at run time.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "cvattn", "libcvattn.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          "--expt-relaxed-constexpr", f"-I{INCLUDE}"]

# ggml type ids of the decode K types (one object per K type)
K_TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q4_1": 3, "q5_0": 6, "q5_1": 7, "q8_0": 8}


def _units():
    units = []
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INCLUDE, "cvattn.h"))
    for src in ("kv_append.cu", "decode.cu", "flash_tc.cu", "capi.cpp", "decode_noalloc.cu"):
        obj = os.path.join(BUILD, src.replace(".", "_") + ".o")
        units.append((os.path.join(CSRC, src), obj, []))
    for name, tid in K_TYPES.items():
        for stem in ("decode_inst", "flash_inst", "flash_pipe_inst", "decode_tc_inst", "decode_pipe_inst",
                     "decode_stream_inst", "decode_mma_inst"):
            if stem == "decode_tc_inst" and name == "f32":
                continue  # the tensor-core decode covers block-quantized and f16 K only
            if stem in ("decode_pipe_inst", "decode_stream_inst", "decode_mma_inst") and name in ("f32", "f16"):
                continue  # the persistent decodes cover block-quantized K only
            obj = os.path.join(BUILD, f"{stem}_{name}.o")
            units.append((os.path.join(CSRC, f"{stem}.cu"), obj, [f"-DCVATTN_KT={tid}"]))
    return units, headers


def _stale(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, obj: str, defs: list[str], verbose: bool) -> str:
    cmd = [NVCC, *ARCH, *CFLAGS, *defs, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, *CFLAGS, *defs, "-x", "cu", "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src} {defs}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    units, headers = _units()
    todo = [(s, o, d) for (s, o, d) in units if force or _stale(o, [s, *headers])]
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    logs = []
    if todo:
        with ThreadPoolExecutor(max_workers=jobs) as ex:
            for log in ex.map(lambda u: _compile(*u, verbose), todo):
                logs.append(log)
    objs = [o for (_, o, _) in units]
    if force or todo or _stale(OUT, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", OUT, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write("".join(logs))
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true", help="print ptxas register / spill info")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))


if __name__ == "__main__":
    main()
