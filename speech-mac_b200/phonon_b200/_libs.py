"""Locations and loaders of the in-tree native libraries.

Every library is built in place (see build.py) so that it travels with the
source tree. Loaders fail loudly when a library is missing: there is no
fallback path.
"""
import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent              # speech-mac_b200/
CSRC = ROOT / "csrc"
REPO = ROOT.parent
INCLUDE = REPO / "include"
SYNTH_SO = PKG / "libphonon_synth.so"
CUDA_SO = PKG / "libphonon_cuda.so"
DROPIN_SO = PKG / "libphonon_transformer_cuda.so"

_cache = {}


def _load(path, mode=0):
    key = str(path)
    if key not in _cache:
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} is not built: run __graft_entry__.build()")
        _cache[key] = C.CDLL(key, mode=mode)
    return _cache[key]


def load_synth():
    return _load(SYNTH_SO)


def load_cuda():
    return _load(CUDA_SO, mode=C.RTLD_GLOBAL)


def load_dropin():
    load_cuda()
    return _load(DROPIN_SO)
