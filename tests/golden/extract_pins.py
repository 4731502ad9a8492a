"""Extract the reference's recorded oracle statistics into reference_pins.json.

The reference (CHNJZ/dsa) ran its FP32 oracle (``tools/review.py:115-178``)
on seeded inputs for each of its 16 shapes and for the public adversarial
families, and wrote ``reference_max`` (max |oracle|) and ``ref_sq``
(sum oracle^2) for output, softmax_max and softmax_sum into
``validation/accuracy-all16/*/result.json`` and
``validation/public/*/result.json``. Those numbers pin both the input
generator and the oracle arithmetic. This script copies them (and nothing
else) into a small committed fixture.

Usage: python tests/golden/extract_pins.py <path-to-reference-checkout>
"""
import glob
import json
import os
import sys


def main(root):
    pins = []
    seen = set()
    for pattern in ("validation/accuracy-all16/*/result.json", "validation/public/*/result.json"):
        for path in sorted(glob.glob(os.path.join(root, pattern))):
            data = json.load(open(path))
            if "accuracy" not in data:
                continue
            metrics = data["accuracy"]["metrics"]
            model = sorted(metrics)[0]
            key = (data["case"], tuple(data["shape"]), data["seed"], data["family"])
            if key in seen:
                continue
            seen.add(key)
            pins.append({
                "case": data["case"],
                "shape": data["shape"],
                "seed": data["seed"],
                "family": data["family"],
                "source": os.path.relpath(path, root),
                "stats": {k: {"reference_max": v["reference_max"], "ref_sq": v["ref_sq"],
                              "elements": v["elements"]} for k, v in metrics[model].items()},
            })
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_pins.json")
    with open(out, "w") as f:
        json.dump(pins, f, indent=1)
    print(f"wrote {len(pins)} pins to {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else ".")
