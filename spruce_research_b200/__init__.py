"""B200-native SPRUCE sparse-prefill hot path (sm_100a CUDA behind a C ABI)."""
__version__ = "0.1.0"
