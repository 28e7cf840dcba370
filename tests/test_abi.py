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


# Engine sources that build on Linux (audio_queue_playback.c needs AudioToolbox,
# speech_stream.c the playback header, phonon_math.c NEON and sha256.c
# CommonCrypto; the first two reference nothing of the path).
ENGINE = ["english_normalize", "phonon_conv", "phonon_mimi", "phonon_pack", "phonon_pcm",
          "phonon_prompt_plan", "phonon_sampler", "phonon_tokenizer", "phonon_voice", "speech",
          "speech_cli", "speech_error", "speech_main", "utf8", "wav_writer"]


def test_engine_links_against_dropin(tmp_path):
    """Every symbol that speech-mac's engine sources take from
    src/phonon_transformer.c or src/phonon_q8.c is exported by
    libphonon_transformer_cuda.so, so the engine links with those two files
    replaced by the drop-in (nm over objects compiled here; no GPU)."""
    from oracle.oracle import reference_root
    src = reference_root() / "src"
    if not (src / "phonon_transformer.c").exists():
        pytest.skip("speech-mac tree not present")
    shim = ROOT / "oracle" / "shim"

    def obj(name):
        out = tmp_path / f"{name}.o"
        subprocess.run(["gcc", "-std=c17", "-O1", "-c", f"-I{shim}", f"-I{src}", "-DPHONON_PACK_TEST_API",
                        str(src / f"{name}.c"), "-o", str(out)], check=True)
        return out

    def syms(path, *flags):
        r = subprocess.run(["nm", *flags, str(path)], capture_output=True, text=True, check=True)
        return {ln.split()[-1] for ln in r.stdout.splitlines() if ln.strip()}

    path_defs = set()
    for name in ("phonon_transformer", "phonon_q8"):
        r = subprocess.run(["nm", "--defined-only", "--extern-only", str(obj(name))], capture_output=True,
                           text=True, check=True)
        path_defs |= {ln.split()[-1] for ln in r.stdout.splitlines() if ln.split()[1] == "T"}
    needed = set()
    for name in ENGINE:
        needed |= syms(obj(name), "-u") & path_defs
    exported = syms(PKG / "libphonon_transformer_cuda.so", "-D", "--defined-only")
    assert needed, "no engine symbol taken from the path?"
    assert not needed - exported, sorted(needed - exported)
    assert {"phonon_flow_condition", "phonon_flow_output_norm", "phonon_flow_embed_latent"} <= needed


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
