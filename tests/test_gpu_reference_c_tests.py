"""The reference's own C tests, run unchanged against the drop-in library.

oracle/Makefile (`make -C oracle dropin`, run by __graft_entry__.build() where
the speech-mac tree exists) compiles speech-mac's tests/test_phonon_q8.c and
tests/test_phonon_transformer.c and links them against
libphonon_transformer_cuda.so in place of src/phonon_transformer.c and
src/phonon_q8.c; the engine sources the transformer test also needs (pack
reader, sampler, voice) compile where they lie. The binaries travel with the
repository, so this test reads nothing of the reference tree. With none of
the PHONON_* asset variables set, test_phonon_transformer.c runs its
model-free sections (tests/test_phonon_transformer.c:538-860): primitives and
their hex pins, KV cache contracts, linears (the bf16 and Q8_0 cancellation
pins and fp16 scale edge cases), conditioning, voice projection, prefix
assembly, and layer / stack / prefill contracts, every numerical call on the
GPU."""
import os
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REF_BIN = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


@pytest.mark.parametrize("name,expect", [("test_phonon_q8_dropin", "phonon Q8 kernel tests passed"),
                                         ("test_phonon_transformer_dropin", "phonon transformer primitives: ok")])
def test_reference_c_test_passes_against_dropin(cuda_ok, name, expect):
    exe = REF_BIN / name
    if not exe.exists():
        pytest.skip(f"{exe} not built (make -C oracle dropin needs the speech-mac tree once)")
    env = {k: v for k, v in os.environ.items() if not k.startswith("PHONON_")}
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=env)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stderr
    assert expect in r.stdout
