"""B200-native (sm_100a) implementation of duoan/mega-trading's transformer-op hot path.

``mega_trading_b200.kernels.triton_attention`` and ``mega_trading_b200.kernels.triton_ops``
mirror the reference modules ``mega_trading.kernels.triton_attention`` / ``triton_ops``;
``mega_trading_b200.install`` rebinds the reference model's operator aliases to them.
"""

__version__ = "0.1.0"
