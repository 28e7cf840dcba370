"""Build every native library of the package in place (no JIT cache).

    python speech-mac_b200/phonon_b200/build.py

libphonon_cuda.so             nvcc, -gencode arch=compute_100a,code=sm_100a
libphonon_transformer_cuda.so gcc -std=c17, links libphonon_cuda.so
libphonon_synth.so            gcc -std=c17 (seeded synthetic inputs)
"""
import os
import shlex
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    print("+", " ".join(shlex.quote(c) for c in cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target, sources):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(s).stat().st_mtime > t for s in sources)


def build_cuda(force=False):
    out = PKG / "libphonon_cuda.so"
    srcs = [CSRC / "phonon_cuda.cu", *sorted(CSRC.glob("*.cuh")), INCLUDE / "phonon_cuda.h"]
    if force or _stale(out, srcs):
        _run([NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", f"-I{INCLUDE}", "-shared", "-o", str(out),
              str(CSRC / "phonon_cuda.cu")])
    return out


def build_dropin(force=False):
    out = PKG / "libphonon_transformer_cuda.so"
    srcs = [CSRC / "phonon_transformer_cuda.c", INCLUDE / "phonon_transformer.h",
            INCLUDE / "phonon_q8.h", INCLUDE / "phonon_pack.h", INCLUDE / "phonon_cuda.h",
            PKG / "libphonon_cuda.so"]
    if force or _stale(out, srcs):
        _run(["gcc", "-std=c17", "-O2", "-fPIC", "-Wall", "-Wextra", "-Werror", f"-I{INCLUDE}",
              "-shared", "-o", str(out), str(CSRC / "phonon_transformer_cuda.c"),
              f"-L{PKG}", "-lphonon_cuda", "-Wl,-rpath,$ORIGIN", "-lpthread", "-lm"])
    return out


def build_synth(force=False):
    out = PKG / "libphonon_synth.so"
    srcs = [CSRC / "phonon_synth.c", CSRC / "phonon_synth.h"]
    if force or _stale(out, srcs):
        _run(["gcc", "-std=c17", "-O2", "-fPIC", "-Wall", "-Wextra", "-Werror", "-shared", "-o",
              str(out), str(CSRC / "phonon_synth.c"), "-lm"])
    return out


def build_all(force=False):
    build_synth(force)
    build_cuda(force)
    build_dropin(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
