"""B200-native delta-attention hot path (prefill + decode) behind the
reference's attention plug-in surface."""

__version__ = "0.1.0"
