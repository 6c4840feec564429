"""Build liblaya_b200.so in-tree with nvcc for sm_100a.

    python laya-inference-engine_b200/build.py [--force]

Every .cu under csrc/ is compiled to an object in _build/ (in parallel, only
when its sources changed) and linked into laya_b200/liblaya_b200.so.  nvcc
cross-compiles without a GPU.
"""
import argparse
import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "laya_b200" / "liblaya_b200.so"
BUILD = HERE / "_build"
INCLUDE = HERE.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def _digest(src):
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for p in sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))):
        h.update(p.read_bytes())
    h.update(src.read_bytes())
    return h.hexdigest()[:16]


def _compile(src, force):
    obj = BUILD / f"{src.stem}.o"
    stamp = BUILD / f"{src.stem}.stamp"
    dig = _digest(src)
    if not force and obj.exists() and stamp.exists() and stamp.read_text() == dig:
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    stamp.write_text(dig)
    return obj


def build(force=False, verbose=False):
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), sources))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp),
           *map(str, objs), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, OUT)
    if verbose:
        print(f"built {OUT}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    try:
        build(force=args.force, verbose=True)
    except RuntimeError as exc:
        print(exc, file=sys.stderr)
        sys.exit(1)
