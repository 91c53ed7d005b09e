"""Writes tests/golden/reference_prototypes.json: every function ork-driver's public headers declare
(include/ork_npu.h and include/ork/*.h of the reference tree), with its normalised return and parameter
types. tests/test_abi.py checks that every symbol this library exports under a name of that list has
exactly that prototype. Run where the reference tree is present: REF=<reference tree> python
tests/golden/make_reference_prototypes.py (without REF: BASELINE.json's reference_path)."""
import glob
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from cproto import prototypes  # noqa: E402

def reference_tree():
    ref = os.environ.get("REF")
    if not ref:
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        with open(os.path.join(root, "BASELINE.json")) as f:
            ref = json.load(f)["reference_path"]
    return ref


def main():
    REF = reference_tree()
    files = [os.path.join(REF, "include", "ork_npu.h")] + sorted(glob.glob(os.path.join(REF, "include", "ork", "*.h")))
    protos = prototypes([open(f).read() for f in files])
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_prototypes.json")
    with open(out, "w") as f:
        json.dump({"source": [os.path.relpath(x, REF) for x in files], "prototypes": protos}, f, indent=0,
                  sort_keys=True)
    print(f"{len(protos)} prototypes -> {out}")


if __name__ == "__main__":
    main()
