#!/usr/bin/env python3
"""Regenerate tests/golden/golden.npz from the reference's own shader sources.

Needs oracle/_ref/libglsl_ref.so (make -C oracle ref, which reads the reference
tree's shaders/*.comp.glsl).  For every case of cases.py the shader is dispatched on
the host exactly as the bench driver records it, and the output region is stored
together with a digest of the inputs (so a drift of the seeded generator is caught
instead of silently comparing different inputs).

    python tests/golden/make_golden.py
"""
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))

from cases import CASES, build, input_digest, output_of  # noqa: E402
from oracle import GlslRef  # noqa: E402


def main():
    ref = GlslRef()
    outs, meta = {}, {}
    for name in CASES:
        c = build(name)
        meta[name] = input_digest(c)
        pushes = c["push"] if isinstance(c["push"][0], list) else [c["push"]]
        for p in pushes:
            ref.dispatch(c["shader"], p, c["blob"], c["feat"], c["aux"], c["groups"])
        outs[name] = output_of(c)
    np.savez_compressed(HERE / "golden.npz", **outs)
    (HERE / "golden_inputs.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "golden.npz", {k: v.shape for k, v in outs.items()})


if __name__ == "__main__":
    main()
