"""Golden fixtures for the graph fuzzer, made by running tgc's own generator and interpreter.
Run once where tgc's source tree is available (it is not on the GPU hosts):

    TGC_REFERENCE=<path to tgc's source tree> python tests/golden/make_fuzz_golden.py

Writes
  fuzz.json   for each generator configuration, tgc.verify.fuzz.generate(config, seed) printed
              by tgc.ir.serialize.dumps, seeds 0..count-1 (tgcb.fuzz.generate must print the
              same text)
  fuzz.npz    tgc.verify.reference.run of every such graph on
              tgc.verify.fuzz.feeds_for(graph, seed) (random_feeds, positive=True)
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REFERENCE = os.environ.get("TGC_REFERENCE")
if not REFERENCE:
    sys.exit("set TGC_REFERENCE to the root of tgc's source tree")
sys.path.insert(0, REFERENCE)

from tgc.ir.serialize import dumps  # noqa: E402
from tgc.verify.fuzz import GeneratorConfig, feeds_for, generate  # noqa: E402
from tgc.verify.reference import run  # noqa: E402

# name -> (GeneratorConfig keyword arguments, seeds)
CONFIGS = {
    "default": ({}, 60),
    "wide": ({"nodes": 16, "inputs": 3, "rows": 48, "columns": 200, "reduction_chance": 0.25}, 30),
}


def main() -> None:
    texts, arrays = {}, {}
    for name, (kwargs, count) in CONFIGS.items():
        config = GeneratorConfig(**kwargs)
        texts[name] = {"config": kwargs, "graphs": []}
        for seed in range(count):
            graph = generate(config, seed=seed)
            texts[name]["graphs"].append(dumps(graph))
            for i, out in enumerate(run(graph, feeds_for(graph, seed=seed))):
                arrays[f"{name}/{seed}/{i}"] = out.numpy()
    with open(os.path.join(HERE, "fuzz.json"), "w") as f:
        json.dump(texts, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "fuzz.npz"), **arrays)
    print(f"{sum(c for _, c in CONFIGS.values())} fuzz graphs written")


if __name__ == "__main__":
    main()
