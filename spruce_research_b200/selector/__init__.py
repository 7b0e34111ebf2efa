"""Flat-gate selector drop-ins (reference: selector/gate.py)."""
from .gate import FlatGate, load_gate  # noqa: F401
