"""Extract the speech-mac model-free pins into tests/golden/pins.json.

Run in a checkout that has the reference tree ($PHONON_REFERENCE_ROOT, else a
`reference` directory beside the repository):

    python tests/golden/make_golden.py [REF_ROOT]

The reference's C tests are read as TEXT; nothing of the reference is
executed. Every vector keeps a pointer to the file and line range it came
from. The output is a small committed fixture so that the tests run where the
reference tree does not exist.
"""
import json
import re
import struct
import sys
from pathlib import Path

HEX_FLOAT = r"[-+]?0x[0-9a-fA-F.]+p[-+]?\d+f?|[-+]?0x0\.0p\+0f|[-+]?\d+\.\d*(?:e[-+]?\d+)?f?|[-+]?\d+f?"


def parse_floats(text):
    """Parse a C initializer of float literals (decimal or hex) into floats."""
    out = []
    for tok in re.findall(HEX_FLOAT, text):
        t = tok.rstrip("fF")
        out.append(float.fromhex(t) if "0x" in t.lower() else float(t))
    return out


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def block(text, start_pat, end_pat="};"):
    i = text.index(start_pat)
    j = text.index(end_pat, i)
    return text[i + len(start_pat):j], text[:i].count("\n") + 1, text[:j].count("\n") + 1


def main():
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from oracle.oracle import reference_root
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_root()
    pins = {}

    # --- GELU (tests/test_phonon_transformer.c) ---
    t = (ref / "tests/test_phonon_transformer.c").read_text()
    src, a, _ = block(t, "float neon_gelu[] = {")
    dst, _, b = block(t, "const float neon_expected[] = {")
    pins["gelu_hex"] = {
        "source": f"tests/test_phonon_transformer.c:{a}-{b}",
        "input": parse_floats(src),
        "expected_bits": [f32_bits(v) for v in parse_floats(dst)],
    }
    pins["gelu_closed_form"] = {
        "source": "tests/test_phonon_transformer.c:552-555",
        "input": [-1.0, 0.0, 1.0],
        "expected": [-0.15865526, 0.0, 0.8413447],
        "atol": 1e-6,
    }
    # RoPE pinned HF values
    pos_txt, a, _ = block(t, "const size_t rope_positions[] = {")
    exp_txt, _, b = block(t, "const float rope_expected[3][2] = {", "};")
    pins["rope_hf"] = {
        "source": f"tests/test_phonon_transformer.c:{a}-{b + 10}",
        "positions": [int(x) for x in re.findall(r"\d+", pos_txt)],
        "row_init": {"2": 1.0, "3": -0.5},
        "expected": [parse_floats(x) for x in re.findall(r"\{([^{}]*)\}", exp_txt)],
        "atol": 3e-7,
        "theta": 10000.0,
    }

    # --- LayerNorm regression (tests/phonon_layer_norm_regression.inc, test_speech.c) ---
    inc = (ref / "tests/phonon_layer_norm_regression.inc").read_text()
    body, a, b = block(inc, "layer_norm_regression_bits[512] = {")
    bits = [int(x, 16) for x in re.findall(r"0x([0-9a-fA-F]+)U", body)]
    assert len(bits) == 512, len(bits)
    sp = (ref / "tests/test_speech.c").read_text()
    m = re.search(r"CHECK\(first == UINT32_C\((0x[0-9a-fA-F]+)\)\)", sp)
    pins["layer_norm_regression"] = {
        "source": f"tests/phonon_layer_norm_regression.inc:{a}-{b}; tests/test_speech.c:109-119",
        "input_bits": bits,
        "expected_first_bits": int(m.group(1), 16),
        "epsilon": 1e-5,
    }

    # --- attention regression (tests/test_speech.c:120-169) ---
    cases_txt, a, b = block(sp, "} cases[] = {", "};")
    cases = []
    for c in re.findall(r"\{(\d+),\s*(\d+),\s*(\d+),\s*UINT32_C\((0x[0-9a-fA-F]+)\)\}", cases_txt):
        cases.append({"count": int(c[0]), "middle": float(c[1]), "tail": float(c[2]),
                      "expected_bits": int(c[3], 16)})
    pins["attention_regression"] = {
        "source": f"tests/test_speech.c:{a}-{b + 30}",
        "layout": "query[0]=8; k[0]=2; k[(n-1)*64]=tail; k[512*64]=middle if nonzero; "
                  "v[0]=v[(n-1)*64]=0.01; stride 64; all other entries 0",
        "cases": cases,
    }

    # --- SLEEF math (tests/test_phonon_math.c) ---
    mt = (ref / "tests/test_phonon_math.c").read_text()
    def arr(name):
        body, a, b = block(mt, name)
        return parse_floats(body), a, b
    silu_in, a, _ = arr("float silu[] = {")
    silu_out, _, _ = arr("const float expected_silu[] = {")
    ph, _, _ = arr("const float phases[] = {")
    ecos, _, _ = arr("const float expected_cos[] = {")
    esin, _, _ = arr("const float expected_sin[] = {")
    ein, _, _ = arr("float exponentials[] = {")
    eout, _, b = arr("const float expected_exp[] = {")
    pins["sleef_math"] = {
        "source": f"tests/test_phonon_math.c:{a}-{b}",
        "silu_input": silu_in, "silu_expected_bits": [f32_bits(v) for v in silu_out],
        "phases": ph, "cos_expected_bits": [f32_bits(v) for v in ecos],
        "sin_expected_bits": [f32_bits(v) for v in esin],
        "exp_input": ein, "exp_expected_bits": [f32_bits(v) for v in eout],
    }

    # --- Q8 known answers (tests/test_phonon_q8.c), linear edge cases ---
    pins["q8_known_answers"] = {
        "source": "tests/test_phonon_q8.c:9-55",
        "dot_two_blocks": {"scales": [0x3800, 0x4000], "values": "block0[i]=i-16, block1[i]=1",
                           "input": "64 ones", "expected": 56.0},
        "matvec_rows": {"matrix": "[b0,b1],[b1,b0]", "expected": [56.0, 56.0]},
        "matvec_asymmetric": {"scales": [0x3800, 0x4000, 0x3800, 0x4000],
                              "values": [1, 2, -1, 3], "input": "32 ones then 32 twos",
                              "expected": [272.0, 368.0]},
        "subnormal_scale": {"scale": 0x0001, "values": "32 ones", "input": "32 ones",
                            "expected_bits": f32_bits(2.0 ** -19)},
    }
    pins["linear_edges"] = {
        "source": "tests/test_phonon_transformer.c:608-662",
        "bf16_2x2": {"weights": [0x3F80, 0xC000, 0x4000, 0x3F00], "input": [3.0, 2.0],
                     "expected": [-1.0, 7.0]},
        "cancellation": {"input": "i%4==0 ? 1e8 : (i%4==2 ? -1e8 : 1), 32 columns",
                         "weights": "all ones, 2 rows (bf16 0x3f80 or q8 scale 0x3c00 q=1)",
                         "bias": [0.0, 0.25], "expected_accelerate": [0.0, 0.25]},
        "q8_scale_edges": {"scales": [0x0001, 0x8000], "values": "all ones",
                           "input": "32 ones", "expected": [2.0 ** -19, 0.0],
                           "rejected_scales": [0x7C00, 0x7E00]},
    }
    pins["kv_layout"] = {
        "source": "tests/test_phonon_transformer.c:586-607",
        "capacity": 2, "layer": 8, "position": 1, "key": "k[i]=i", "value": "v[i]=-i",
        "flat_index": (8 * 2 + 1) * 512 + 7, "expected": 7.0,
    }
    # --- flow head (tests/test_phonon_sampler.c): a nonzero synthetic head whose
    # weights, condition and state follow formulas in the test; the expected
    # velocity comes from an independent PyTorch evaluation quoted there.
    t = (ref / "tests/test_phonon_sampler.c").read_text()
    exp, a, b = block(t, "const float expected[32] = {")
    lo = t.index("static void test_nonzero_flow_head_against_independent_reference(void) {")
    pins["flow_head_synthetic"] = {
        "source": f"tests/test_phonon_sampler.c:{t[:lo].count(chr(10)) + 1}-{b + 7}",
        "expected": parse_floats(exp),
        "atol": 2e-4,
        "s": 0.0, "t": 1.0,
    }
    out = Path(__file__).with_name("pins.json")
    out.write_text(json.dumps(pins, indent=1, sort_keys=True) + "\n")
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
