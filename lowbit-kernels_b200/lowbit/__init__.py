"""lowbit (B200): INT4 weight-only (W4A16) kernels for sm_100a behind the lowbit operator surface."""
