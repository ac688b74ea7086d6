"""Error figures of the parity tests: max abs and max rel error per compared
quantity, printed and, when DITCH_PARITY_REPORT names a file, appended to it
as JSON lines (one per quantity) so a run can commit the numbers it saw.

max_rel is the max abs error over the largest magnitude of the reference
vector (the scale the bound uses); max_elem_rel is the largest
|got - want| / |want| over the elements with |want| above 1 % of that scale.
"""
import json
import os

import numpy as np


def errors(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    scale = float(np.abs(want).max()) if want.size else 0.0
    big = np.abs(want) > 0.01 * scale
    elem = float((err[big] / np.abs(want[big])).max()) if big.any() else 0.0
    return {"max_abs": float(err.max()) if err.size else 0.0, "max_rel": float(err.max() / scale) if scale else 0.0,
            "max_elem_rel": elem, "ref_max_abs": scale}


def record(case, quantity, got, want, bound=None, **extra):
    """Returns the error figures (and records them)."""
    e = errors(got, want)
    line = {"case": case, "quantity": quantity, **e, **extra}
    if bound is not None:
        line["bound"] = float(bound)
    print(json.dumps(line))
    path = os.environ.get("DITCH_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(line) + "\n")
    return e


def record_value(case, quantity, got, want, **extra):
    """A scalar (KL, cosine): abs and rel difference."""
    got, want = float(got), float(want)
    line = {"case": case, "quantity": quantity, "got": got, "want": want, "abs": abs(got - want),
            "rel": abs(got - want) / abs(want) if want else 0.0, **extra}
    print(json.dumps(line))
    path = os.environ.get("DITCH_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(line) + "\n")
    return line
