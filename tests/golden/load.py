"""Lazy loader for the committed golden vectors."""
from functools import lru_cache
from pathlib import Path

import numpy as np

PATH = Path(__file__).resolve().parent / "golden.npz"


@lru_cache(maxsize=1)
def golden():
    with np.load(PATH) as z:
        return {k: z[k] for k in z.files}
