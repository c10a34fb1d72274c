"""Generates tests/golden/member_windows.json by running the REFERENCE's own window-budget designs
(`knee.window_budget.member_windows`, src/knee/window_budget.py:57-123).

Run here (the reference is importable on CPU; the GPU box only reads the committed JSON):

    PYTHONPATH=<reference>/src python tests/golden/make_windows.py

Every case records the sorted window indices of one (design, member, seed) at one study geometry:
2 slots x 24 windows (the benchmark's two crop windows of 26 slices) and the submission's 8 slots x
11 windows.
"""
from __future__ import annotations

import json
from pathlib import Path

from knee.window_budget import member_windows   # the reference

HERE = Path(__file__).resolve().parent
DESIGNS = ["full", "parx", "par", "mod3", "mod4", "mod4x3", "q8f4", "scale"]
GEOMETRIES = [(2, 24), (8, 11)]


def main() -> None:
    cases = []
    for n_slots, per in GEOMETRIES:
        for design in DESIGNS:
            for seed in range(3):
                for member in range(4):
                    idx = member_windows(design, member, n_slots, per, seed=seed)
                    cases.append({"design": design, "member": member, "seed": seed, "n_slots": n_slots,
                                  "per": per, "windows": [int(v) for v in idx]})
    (HERE / "member_windows.json").write_text(json.dumps(cases, separators=(",", ":")))
    print(len(cases), "cases")


if __name__ == "__main__":
    main()
