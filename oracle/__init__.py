"""CPU oracle (test infrastructure only; see kolibri_oracle.py)."""
from .kolibri_oracle import *  # noqa: F401,F403
