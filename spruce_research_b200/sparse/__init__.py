"""Block-sparse prefill attention drop-in (reference: sparse/attention.py)."""
from .attention import SPARSE_PREFILL_ATTENTION, register_sparse_prefill_attention, sparse_prefill_attention_forward  # noqa: F401,E501
