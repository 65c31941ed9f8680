"""Data roots: $RF_DATA (default <repo>/data) expanded in config strings (code/kva/paths.py:16-36)."""
import os
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
DATA = Path(os.environ.get("RF_DATA", REPO / "data"))


def expand(value):
    """Expand $RF_DATA / ${RF_DATA} (and other environment variables) in strings, recursively. The reference's
    $KVA_DATA names the same root unless it is set in the environment, so its config files load unchanged."""
    if isinstance(value, str):
        for var in ("RF_DATA",) + (() if "KVA_DATA" in os.environ else ("KVA_DATA",)):
            value = value.replace("${" + var + "}", str(DATA)).replace("$" + var, str(DATA))
        return os.path.expandvars(value)
    if isinstance(value, dict):
        return {k: expand(v) for k, v in value.items()}
    if isinstance(value, list):
        return [expand(v) for v in value]
    return value
