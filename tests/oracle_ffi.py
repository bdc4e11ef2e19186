"""Re-export of the oracle bindings (oracle/ffi.py) for the tests."""
import sys
from pathlib import Path

_ORACLE = Path(__file__).resolve().parents[1] / "oracle"
if str(_ORACLE) not in sys.path:
    sys.path.insert(0, str(_ORACLE))

from ffi import *  # noqa: E402,F401,F403
from ffi import Oracle, Reference, reference_available, rel_l2  # noqa: E402,F401
