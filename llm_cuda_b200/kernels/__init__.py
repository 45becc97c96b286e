"""CUDA kernel entry points (RoPE+append, paged decode, LSE merge)."""
