"""B200-native SPRUCE sparse-prefill hot path (sm_100a CUDA behind a C ABI).

Reference-named drop-ins:
  kernels.sparse_prefill   triton_sparse_prefill_attention_forward, adapters, registration
  kernels.direct_index     direct_index_sparse_triton
  sparse.attention         sparse_prefill_attention_forward
  teacher.chunked_extract  _proto_pool_seq, _group_avg_tokens
  selector.gate            FlatGate, load_gate
  export_selected_blocks   selected_ids_to_blocks, selected_mask_to_blocks
  interfaces.validator     validate_selected_blocks
  route_overrides          charged_route_density
Per-layer pipeline: pipeline.SparsePrefillLayer; multi-GPU split: sharding.
"""
__version__ = "0.1.0"
