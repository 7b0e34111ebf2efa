"""Block-sparse prefill attention drop-in (reference: sparse/attention.py)."""
from .attention import SPARSE_PREFILL_ATTENTION, register_sparse_prefill_attention, sparse_prefill_attention_forward  # noqa: F401,E501
from .summaries import (KVSummaryTable, build_kv_summary_table, residual_attention_density,  # noqa: F401
                        token_validity_from_attention_mask)
