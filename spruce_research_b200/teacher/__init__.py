"""Selector feature pooling drop-ins (reference: teacher/chunked_extract.py)."""
from .chunked_extract import _group_avg_tokens, _proto_pool_seq, pool_selector_features  # noqa: F401
