"""Shared helpers of the parity tests: tolerances of BASELINE.json's north star and
the comparison / routing-agreement statistics."""
from __future__ import annotations

import numpy as np

MAX_ABS = 2e-2       # max |gpu - oracle| over fp16 outputs
REL_L2 = 1e-3        # ||gpu - oracle||_2 / ||oracle||_2
TIE_MARGIN = 1e-3    # routing may differ only where the oracle's top-2 logit margin is below this


def err_stats(got, ref):
    g = np.asarray(got, dtype=np.float32).ravel()
    r = np.asarray(ref, dtype=np.float32).ravel()
    d = np.abs(g - r)
    rel = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
    return float(d.max()) if d.size else 0.0, rel, int((g != r).sum())


def assert_close(got, ref, what="", max_abs=MAX_ABS, rel_l2=REL_L2):
    m, rel, nd = err_stats(got, ref)
    assert np.isfinite(np.asarray(got, dtype=np.float32)).all(), f"{what}: non-finite values"
    assert m <= max_abs and rel <= rel_l2, f"{what}: max_abs {m:.3g} rel_l2 {rel:.3g} ({nd} differ)"
    return m, rel, nd


def routing_agreement(gpu_assign, ref_assign, margin):
    """(hard mismatches, tie mismatches): a mismatch is a tie when the oracle's top-2
    margin is below TIE_MARGIN."""
    diff = np.asarray(gpu_assign) != np.asarray(ref_assign)
    ties = np.asarray(margin) < TIE_MARGIN
    return int((diff & ~ties).sum()), int((diff & ties).sum())


def checkpoint_of(L, blob, split_qkv=False):
    """Named tensors (default convention of export.py) holding the blob's weights."""
    from prism_inference_b200 import export
    names = export.default_names(L)
    ck = {}
    from prism_inference_b200 import layout
    for lname, (w, b) in layout.unpack_weights(L, blob).items():
        p = names[lname]
        if split_qkv and lname.endswith(".qkv"):
            D = L.dim
            for j, x in enumerate("qkv"):
                ck[f"{p[:-4]}.{x}.weight"] = w.reshape(3 * D, D)[j * D:(j + 1) * D].astype(np.float32)
                ck[f"{p[:-4]}.{x}.bias"] = b[j * D:(j + 1) * D].astype(np.float32)
        else:
            ck[f"{p}.weight"] = w.astype(np.float32)
            ck[f"{p}.bias"] = b.astype(np.float32)
    return ck
