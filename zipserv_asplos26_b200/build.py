"""Build the in-tree native library zipserv_asplos26_b200/_lib/libzipserv_b200.so.

    python -m zipserv_asplos26_b200.build [--verbose] [--ptxas-info]

Compiles the CUDA kernels for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) together with the host encoder and the C
ABI into one shared library with a static CUDA runtime, so it loads with
ctypes on any machine that has the NVIDIA driver (and on a CPU-only machine
for packing). Object files are cached under _lib/obj and rebuilt when a
source or header changes.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libzipserv_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["zipserv_cuda.cu"]  # includes zipgemm.cu, decompress.cu, capi_cuda.cu
HOST_SOURCES = ["packer.cpp", "capi_host.cpp"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH") or "/usr/local/cuda"
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else (shutil.which("nvcc") or "nvcc")


def _headers_digest() -> str:
    # Every header and every .cu (zipserv_cuda.cu includes the other .cu files).
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.cu"))
                   + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    stamp_path = obj_dir / "stamp.json"
    stamp = json.loads(stamp_path.read_text()) if stamp_path.exists() else {}
    headers = _headers_digest()
    common = ["-std=c++17", "-O3", "-Xcompiler", "-fPIC,-pthread", f"-I{INCLUDE}", f"-I{CSRC}"]
    objects = []
    changed = force or stamp.get("headers") != headers or not LIB_PATH.exists()
    new_stamp = {"headers": headers}
    for name in CUDA_SOURCES + HOST_SOURCES:
        src = CSRC / name
        obj = obj_dir / (name + ".o")
        digest = hashlib.sha256(src.read_bytes()).hexdigest()
        new_stamp[name] = digest
        objects.append(obj)
        if not force and obj.exists() and stamp.get(name) == digest and stamp.get("headers") == headers:
            continue
        changed = True
        cmd = [nvcc(), *common, "-c", str(src), "-o", str(obj)]
        if name.endswith(".cu"):
            cmd += [*ARCH, "-lineinfo", "--expt-relaxed-constexpr"]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
        else:
            cmd += ["-x", "cu", *ARCH]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    if changed:
        cmd = [nvcc(), *ARCH, "--shared", "-cudart", "static", "-Xcompiler", "-fPIC,-pthread",
               *map(str, objects), "-o", str(LIB_PATH)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    stamp_path.write_text(json.dumps(new_stamp, indent=1))
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(args.verbose, args.ptxas_info, args.force or args.ptxas_info))


if __name__ == "__main__":
    main()
