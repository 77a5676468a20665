"""CPU oracle package -- test infrastructure only (see mtp_oracle.py)."""
from .mtp_oracle import *  # noqa: F401,F403
