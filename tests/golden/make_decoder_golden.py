"""Generate tests/golden/decoder_cases.npz from the reference decoder (oracle/_ref).

Run after ``make -C oracle dropin REF=<reference checkout>``:

    python tests/golden/make_decoder_golden.py

For every pin case of oracle/qkn_decoder_oracle.py (PIN_CASES: Qwen3 with one and two
layers, Gemma 2 and Gemma 3 settings, SmolVLM) the seeded model, its prompt and its
teacher-forced token stream are written to a file and run by oracle/_ref/qkn_weights_emul
(the reference's common/decoder/qkn_decoder.c) or oracle/_ref/smolvlm_weights_emul
(exports/smolvlm/decoder.c), with the kernels of tmzt/smol-genius and attention over
bf16 K / fp16 V -- and its per-step greedy tokens and final normalised hidden states
are stored with the prompt and the stream.  The weights are not stored:
they are regenerated from the case's seed.
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
from qkn_decoder_oracle import PIN_CASES, pin_case, read_reference_steps, write_weights_file  # noqa: E402

REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def _binary(name):
    return os.path.join(REF_DIR, "smolvlm_weights_emul" if PIN_CASES[name].get("smolvlm") else "qkn_weights_emul")


def main() -> None:
    for name in PIN_CASES:
        if not os.path.exists(_binary(name)):
            sys.exit(f"{_binary(name)} is missing: run make -C oracle dropin REF=<reference checkout>")
    cases = {}
    with tempfile.TemporaryDirectory() as d:
        for name in PIN_CASES:
            m, prompt, feed = pin_case(name)
            inp, out = os.path.join(d, "model.bin"), os.path.join(d, "steps.bin")
            write_weights_file(inp, m, prompt, feed)
            subprocess.run([_binary(name), inp, out], check=True)
            tokens, xs = read_reference_steps(out, len(feed), m.H)
            cases[f"{name}/prompt"] = np.asarray(prompt, np.int32)
            cases[f"{name}/feed"] = np.asarray(feed, np.int32)
            cases[f"{name}/tokens"] = tokens.astype(np.int32)
            cases[f"{name}/x"] = xs.astype(np.float32)
    path = os.path.join(HERE, "decoder_cases.npz")
    np.savez_compressed(path, **cases)
    print(f"wrote {path}: {len(PIN_CASES)} cases")


if __name__ == "__main__":
    main()
