"""Operators of the decode hot path (drop-ins for starkv_serve/kernels/*)."""
