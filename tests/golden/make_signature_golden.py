"""Golden shape signatures, made by running tgc's own hash. Run once where tgc's source tree
is available (it is not on the GPU hosts):

    TGC_REFERENCE=<path to tgc's source tree> python tests/golden/make_signature_golden.py

Writes signatures.json: tgc.runtime.cache.shape_signature of every graph under graphs/ and of
the fuzz graphs in fuzz.json (loaded with tgc.ir.serialize.loads), and of tgc's
isomorphism.renamed copy of each workload graph (the hash must not see names).
"""

from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
if not os.environ.get("TGC_REFERENCE"):
    sys.exit("set TGC_REFERENCE to the root of tgc's source tree")
sys.path.insert(0, os.environ["TGC_REFERENCE"])

from tgc.ir.isomorphism import renamed  # noqa: E402
from tgc.ir.serialize import loads  # noqa: E402
from tgc.runtime.cache import shape_signature  # noqa: E402


def main() -> None:
    out = {"graphs": {}, "renamed": {}, "fuzz": {}}
    gdir = os.path.join(HERE, "graphs")
    for name in sorted(os.listdir(gdir)):
        with open(os.path.join(gdir, name)) as f:
            g = loads(f.read())
        out["graphs"][name] = shape_signature(g)
        out["renamed"][name] = shape_signature(renamed(g, prefix="r"))
    with open(os.path.join(HERE, "fuzz.json")) as f:
        fz = json.load(f)
    for cfg, d in fz.items():
        out["fuzz"][cfg] = [shape_signature(loads(t)) for t in d["graphs"]]
    with open(os.path.join(HERE, "signatures.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"{len(out['graphs'])} graph signatures written")


if __name__ == "__main__":
    main()
