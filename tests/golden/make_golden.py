"""Regenerate the golden fixtures (tests/golden/*.npz) from the float64 CPU oracle.

    python tests/golden/make_golden.py

The oracle (oracle/torch_ref.py) restates the reference's step and is pinned by the
reference's own known-answer tests (tests/test_oracle_kats.py). The reference itself
cannot run here (it needs warp-lang 1.15.0, which is not installable offline), so these
fixtures freeze the oracle's answers on small seeded cases.
"""

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, os.path.dirname(HERE))

import numpy as np  # noqa: E402

from golden.cases import CASES, run_oracle  # noqa: E402


def main():
    for name, spec in CASES.items():
        out = run_oracle(spec)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print(name, float(out["loss"]))


if __name__ == "__main__":
    main()
