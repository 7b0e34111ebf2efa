"""The frozen selected_blocks contract (reference: interfaces/)."""
from .validator import LOCAL_WINDOW, PAD_VALUE, validate_selected_blocks  # noqa: F401
