"""vLLM v1 attention hook: decoder adapter, plugin backend and registration."""
