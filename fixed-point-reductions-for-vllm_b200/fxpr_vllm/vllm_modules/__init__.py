"""vLLM glue: runtime config, quantisation method, attention backend, RMSNorm, sampler."""
