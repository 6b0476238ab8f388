"""Writes checkpoint_inventory.json: inventory SHA-256 values computed by the
reference's own build_inventory (src/minifield_training/core/parameters.py:58-152).

Run from the repository root in a container that has the reference checked
out at REFERENCE_SRC (the path is an argument, not read at test time):

    python tests/golden/make_checkpoint_golden.py /path/to/reference/src
"""

import json
import os
import sys

CASES = [
    {"shapes": {"weight": [2]}, "format_id": "synthetic/1", "decayed": []},
    {"shapes": {"conv.weight": [8, 1, 3]}, "format_id": "synthetic/strided", "decayed": []},
    {"shapes": {"a.matrix": [37, 53], "b.matrix": [64, 16], "c.vector": [61], "d.frozen": [9, 7]},
     "format_id": "synthetic/mixed", "decayed": ["a.matrix", "b.matrix"], "frozen": ["d.frozen"],
     "quantization_profile": "int8-channel-absmax-v1", "quantized": ["a.matrix"], "source_dtype": "float16"},
]


def main(src):
    sys.path.insert(0, src)
    from minifield_training.core import parameters

    out = []
    for case in CASES:
        inv = parameters.build_inventory(
            {k: tuple(v) for k, v in case["shapes"].items()}, format_id=case["format_id"],
            decayed_names=frozenset(case["decayed"]), frozen_names=frozenset(case.get("frozen", [])),
            quantization_profile=case.get("quantization_profile"),
            quantized_names=frozenset(case.get("quantized", [])),
            source_dtype=case.get("source_dtype", "bfloat16"))
        out.append(dict(case, sha256=inv.sha256, parameter_count=inv.parameter_count))
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "checkpoint_inventory.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(path)


if __name__ == "__main__":
    main(sys.argv[1])
