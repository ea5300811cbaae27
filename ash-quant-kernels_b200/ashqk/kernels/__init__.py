"""Kernel-level entry points, module paths as in the reference (ashqk/kernels/)."""
