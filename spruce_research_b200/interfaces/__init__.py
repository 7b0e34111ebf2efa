"""The frozen selected_blocks contract (reference: interfaces/)."""
from .validator import LOCAL_WINDOW, PAD_VALUE, validate_selected_blocks  # noqa: F401
from .residual_summaries import (ResidualTreeLayout, build_residual_summary_nodes,  # noqa: F401
                                 build_residual_tree_layout, residual_frontier_for_row,
                                 validate_residual_summary_nodes)
