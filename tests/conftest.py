"""Shared test setup: import paths and the ``gpu`` marker."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "laya-inference-engine_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

