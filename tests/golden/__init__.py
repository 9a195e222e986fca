# SPDX-License-Identifier: Apache-2.0
"""Golden outputs of the reference's own code (see make_golden.py)."""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load() -> dict:
    with np.load(os.path.join(HERE, "golden.npz")) as z:
        return {k: z[k] for k in z.files}


def meta() -> dict:
    with open(os.path.join(HERE, "golden.json")) as f:
        return json.load(f)
