"""Data roots: $RF_DATA (default <repo>/data) expanded in config strings (code/kva/paths.py:16-36)."""
import os
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
DATA = Path(os.environ.get("RF_DATA", REPO / "data"))


def expand(value):
    """Expand $RF_DATA / ${RF_DATA} (and other environment variables) in strings, recursively."""
    if isinstance(value, str):
        return os.path.expandvars(value.replace("$RF_DATA", str(DATA)).replace("${RF_DATA}", str(DATA)))
    if isinstance(value, dict):
        return {k: expand(v) for k, v in value.items()}
    if isinstance(value, list):
        return [expand(v) for v in value]
    return value
