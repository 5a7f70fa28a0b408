"""Performance tools: standalone decode-step and kernel timing (CUDA events), used for profiling."""
