"""B200-native (sm_100a) LLMY looped hybrid block: kernels behind a C ABI, PyTorch host."""
__all__ = ["kernels"]
