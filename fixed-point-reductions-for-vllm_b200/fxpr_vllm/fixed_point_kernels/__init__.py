"""B200 CUDA kernels of the fixed-point reduction hot path (host launchers)."""
