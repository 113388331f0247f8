"""Generate tests/golden/siglip_cases.npz from the reference SigLIP encoder (oracle/_ref).

Run after ``make -C oracle dropin REF=<reference checkout>``:

    python tests/golden/make_siglip_golden.py

For every pin case of oracle/siglip_oracle.py (SIGLIP_PIN_CASES) the seeded encoder and
its two seeded images are written to a file and run by oracle/_ref/siglip_weights_ref --
siglip_forward of tmzt/smol-genius (common/vision/siglip.c) with its kernels -- and the
encoder output is stored.  Weights and images regenerate from the case's seeds.
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
from siglip_oracle import SIGLIP_PIN_CASES, siglip_pin_case  # noqa: E402

BIN = os.path.join(ROOT, "oracle", "_ref", "siglip_weights_ref")


def main() -> None:
    if not os.path.exists(BIN):
        sys.exit(f"{BIN} is missing: run make -C oracle dropin REF=<reference checkout>")
    cases = {}
    with tempfile.TemporaryDirectory() as d:
        for name in SIGLIP_PIN_CASES:
            m, images = siglip_pin_case(name)
            inp, out = os.path.join(d, "model.bin"), os.path.join(d, "out.bin")
            m.write_weights_file(inp, images)
            subprocess.run([BIN, inp, out], check=True)
            cases[f"{name}/out"] = np.fromfile(out, np.float32).reshape(len(images), m.n_pos, m.H)
    path = os.path.join(HERE, "siglip_cases.npz")
    np.savez_compressed(path, **cases)
    print(f"wrote {path}: {len(SIGLIP_PIN_CASES)} cases")


if __name__ == "__main__":
    main()
