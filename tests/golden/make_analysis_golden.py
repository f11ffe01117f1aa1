"""Golden outputs of tgc's attention and normalisation analyses, made by running tgc itself.
Run once where tgc's source tree is available (it is not on the GPU hosts):

    TGC_REFERENCE=<path to tgc's source tree> python tests/golden/make_analysis_golden.py

Writes analysis.npz: tgc.analysis.attention.streaming_attention / naive_attention on
random_head inputs, and tgc.analysis.normalisation layer_norm / rms_norm / batch_norm on
random_rows inputs (with a non-trivial gain and offset drawn from a seeded generator).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
if not os.environ.get("TGC_REFERENCE"):
    sys.exit("set TGC_REFERENCE to the root of tgc's source tree")
sys.path.insert(0, os.environ["TGC_REFERENCE"])

from tgc.analysis import attention as A  # noqa: E402
from tgc.analysis import normalisation as N  # noqa: E402

HEADS = [  # (sequence, width, block, seed, scale)
    (256, 64, 128, 0, 1.0),
    (300, 32, 50, 1, 1.0),
    (192, 128, 64, 2, 1.0),
    (200, 16, 7, 3, 8.0),
]
ROWS = [(48, 512, 0.5, 0), (37, 300, 0.0, 1)]


def main() -> None:
    out = {}
    for s, w, blk, seed, scale in HEADS:
        q, k, v = A.random_head(A.AttentionShape(s, w), seed=seed, scale=scale)
        tag = f"attn/{s}_{w}_{blk}_{seed}_{scale}"
        out[f"{tag}/streaming"] = A.streaming_attention(q, k, v, blk).numpy()
        out[f"{tag}/naive"] = A.naive_attention(q, k, v).numpy()
    for rows, width, offset, seed in ROWS:
        x, _, _ = N.random_rows(N.NormShape(rows, width), seed=seed, offset=offset)
        g = torch.Generator().manual_seed(100 + seed)
        gain = torch.rand(width, generator=g) + 0.5
        shift = torch.randn(width, generator=g)
        tag = f"norm/{rows}_{width}_{offset}_{seed}"
        out[f"{tag}/gain"] = gain.numpy()
        out[f"{tag}/shift"] = shift.numpy()
        out[f"{tag}/layer"] = N.layer_norm(x, gain, shift).numpy()
        out[f"{tag}/rms"] = N.rms_norm(x, gain).numpy()
        out[f"{tag}/batch"] = N.batch_norm(x, gain, shift).numpy()
        mean = torch.randn(width, generator=g)
        var = torch.rand(width, generator=g) + 0.1
        out[f"{tag}/mean"] = mean.numpy()
        out[f"{tag}/var"] = var.numpy()
        out[f"{tag}/batch_running"] = N.batch_norm(x, gain, shift, running=(mean, var)).numpy()
    np.savez_compressed(os.path.join(HERE, "analysis.npz"), **out)
    print(f"{len(out)} arrays written")


if __name__ == "__main__":
    main()
