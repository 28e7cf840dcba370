"""The C-ABI boundary without a GPU: every entry point declared in include/*.h
is exported by the built libraries, and the drop-in headers compile against a
reference caller."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
INCLUDE = ROOT / "include"
PKG = ROOT / "speech-mac_b200" / "phonon_b200"


def declared(header):
    text = re.sub(r"/\*.*?\*/", "", (INCLUDE / header).read_text(), flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(phonon_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def exported(so):
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], check=True, capture_output=True,
                         text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_cuda_library_exports_header():
    so = PKG / "libphonon_cuda.so"
    assert so.exists(), "run __graft_entry__.build()"
    missing = set(declared("phonon_cuda.h")) - exported(so)
    assert not missing, missing
    C.CDLL(str(so))  # loads without a GPU


def test_dropin_exports_reference_api():
    so = PKG / "libphonon_transformer_cuda.so"
    assert so.exists()
    names = set(declared("phonon_transformer.h")) | set(declared("phonon_q8.h"))
    missing = names - exported(so)
    assert not missing, missing
    assert "phonon_flow_stack_step_cancel" in names and "phonon_q8_matvec" in names


def test_synth_library_loads():
    from phonon_b200 import synth
    assert synth.Generator(0).next_u64() != 0


def test_tensor_view_layout():
    """PhononTensorView matches src/phonon_pack.h:10-19 on LP64."""
    from oracle.oracle import PhononTensorView
    assert C.sizeof(PhononTensorView) == 4 + 4 + 8 * 8 + 8 + 8 + 8
    assert PhononTensorView.data.offset == 72


@pytest.mark.parametrize("test", ["test_phonon_q8.c"])
def test_reference_test_compiles_against_dropin(tmp_path, test):
    """Where the speech-mac tree exists, its own Q8 test links unchanged
    against the drop-in headers and library (linked, not run: no GPU)."""
    from oracle.oracle import reference_root
    src = reference_root() / "tests" / test
    if not src.exists():
        pytest.skip("speech-mac tree not present")
    exe = tmp_path / "t"
    subprocess.run(["gcc", "-std=c17", "-O1", f"-I{INCLUDE}", str(src), "-o", str(exe),
                    f"-L{PKG}", "-lphonon_transformer_cuda", "-lphonon_cuda",
                    f"-Wl,-rpath,{PKG}"], check=True)
    assert exe.exists()
