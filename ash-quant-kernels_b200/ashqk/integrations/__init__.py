"""Integrations of the B200 kernels with serving frameworks (imported on demand)."""
