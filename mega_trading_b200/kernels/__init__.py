"""Operator modules mirroring ``mega_trading.kernels`` (same names and signatures)."""
