"""Generate tests/golden/block_choices.json from the reference's own heuristics.

    python tests/golden/make_block_choices.py <path to the reference checkout>

The reference's `choose_block` (bf/fp32.py:212-221) and `choose_qgroup_block`
(bf/fp32_qgroup.py:217-225) are public helpers that callers report; this package
keeps them (gpu_algo_b200/bf/).  The reference modules import CuPy at the top,
which is not installed here, so CuPy is replaced by an empty module for the
import: neither function touches it.  The JSON records the block each function
picks over a grid of (k, d[, qpb]) and is read by tests/test_bf_helpers.py.
"""
from __future__ import annotations

import importlib
import json
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
KS = (1, 2, 4, 8, 10, 16, 32, 64, 100, 128, 200, 256, 512, 1024)
DS = (1, 8, 33, 96, 128, 300, 960, 1024, 4096)
QPBS = (1, 2, 4, 8, 16)


def main(argv: list[str]) -> int:
    ref = argv[1] if len(argv) > 1 else os.environ.get("GPU_ALGO_REFERENCE")
    if not ref:
        print("usage: make_block_choices.py <reference checkout> (or $GPU_ALGO_REFERENCE)",
              file=sys.stderr)
        return 2
    sys.modules.setdefault("cupy", types.ModuleType("cupy"))
    sys.path.insert(0, ref)
    fp32 = importlib.import_module("bf.fp32")
    qgroup = importlib.import_module("bf.fp32_qgroup")
    out = {
        "choose_block": [[k, d, fp32.choose_block(k, d)] for k in KS for d in DS],
        "choose_qgroup_block": [[k, d, q, qgroup.choose_qgroup_block(k, d, q)]
                                for k in KS for d in DS for q in QPBS],
    }
    with open(os.path.join(HERE, "block_choices.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
        f.write("\n")
    print(f"wrote block_choices.json ({len(out['choose_block'])} + "
          f"{len(out['choose_qgroup_block'])} cases)")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
