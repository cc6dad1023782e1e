"""Imports the reference's own Python (BHUHD/minixmax-h3) — TEST INFRASTRUCTURE.

Only the CPU pin tests and tests/golden/make_golden.py use this, to check the
oracle restatement against the reference and to regenerate the committed
golden fixtures.  The reference tree is not present on GPU boxes, where
``load()`` returns None and those tests skip.
"""
from __future__ import annotations

import os
import sys
from types import SimpleNamespace
from typing import Optional

# The reference checkout sits beside this repository (``../reference``);
# H3B_REFERENCE_ROOT overrides the location.
_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_ROOT = os.environ.get("H3B_REFERENCE_ROOT", os.path.join(os.path.dirname(_REPO), "reference"))
REF_SRC = os.path.join(REF_ROOT, "Ref2VA-910C-FastAPI-INT8-CANN9.1.0", "runtime", "src")


def load() -> Optional[SimpleNamespace]:
    """Returns the reference modules on the hot path, or None if absent."""
    if not os.path.isdir(os.path.join(REF_SRC, "h3_npu")):
        return None
    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    from h3_npu.model import dit
    from h3_npu.modules import linear
    from h3_npu.ops import attention, float8_cast, hadamard, int8_convrot, nvfp4, rope, ulysses
    from h3_npu.runtime import dist

    return SimpleNamespace(dit=dit, linear=linear, attention=attention, float8_cast=float8_cast,
                           hadamard=hadamard, int8_convrot=int8_convrot, nvfp4=nvfp4, rope=rope, ulysses=ulysses, dist=dist)
