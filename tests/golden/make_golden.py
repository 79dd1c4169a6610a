"""Writes the golden fixtures of tests/golden from the C oracle.

    python tests/golden/make_golden.py [name ...]

Run it only when the canonical arithmetic changes on purpose; the tests
compare the oracle and the CUDA path against these files.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from golden import cases  # noqa: E402


def main(names=None) -> None:
    """Writes every fixture, or only those named on the command line."""
    for name, (cfg, seed) in cases.DECODE_CASES.items():
        if names and name not in names:
            continue
        np.savez(cases.HERE / f"{name}.npz", **cases.run_oracle_decode(cfg, seed))
        print("wrote", name)
    for name, (k, sd, seed) in cases.GEMV_CASES.items():
        if names and name not in names:
            continue
        np.savez(cases.HERE / f"{name}.npz", **cases.run_oracle_gemv(k, sd, seed))
        print("wrote", name)


if __name__ == "__main__":
    main(sys.argv[1:])
