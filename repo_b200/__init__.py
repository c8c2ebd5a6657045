"""B200-native CubicSplat render/optimise hot path (sm_100a CUDA behind a C ABI)."""
__version__ = "0.1.0"
