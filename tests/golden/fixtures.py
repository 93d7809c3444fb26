"""Loader for the golden vectors written by make_golden.py."""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "manifest.json")) as _f:
    MANIFEST = json.load(_f)


def names(op: str | None = None):
    return sorted(k for k, v in MANIFEST.items() if op is None or v["op"] == op)


def load(name: str):
    """Returns (meta, arrays); arrays stored only as a digest + head are
    returned under ``<key>__head`` and must be checked through ``meta``."""
    meta = MANIFEST[name]
    with np.load(os.path.join(HERE, name + ".npz")) as z:
        arrays = {k: z[k] for k in z.files}
    return meta, arrays
