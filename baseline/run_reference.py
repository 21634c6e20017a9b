"""Reference arm of bench.py: runs the unmodified reference trainer staged under
`baseline/_ref` (git-ignored) for the same metric and config.  Until the staging exists this
reports why it is unavailable."""
from __future__ import annotations

import os

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def run_reference(args) -> dict:
    if not os.path.exists(os.path.join(REF, "train_gpt.py")):
        return {"impl": "reference", "unavailable": "baseline/_ref is not staged on this machine"}
    from .reference_driver import drive, drive_track2
    if getattr(args, "track", 1) == 2:
        if not os.path.exists(os.path.join(REF, "train_gpt_medium.py")):
            return {"impl": "reference", "unavailable": "baseline/_ref/train_gpt_medium.py is not staged on this machine"}
        return drive_track2(args, REF)
    return drive(args, REF)
