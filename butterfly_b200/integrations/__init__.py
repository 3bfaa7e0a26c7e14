"""Model integrations (layer swap) for the compressed Butterfly kernels."""
