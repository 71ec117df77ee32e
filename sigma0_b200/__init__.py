"""sigma0_b200: a B200-native framework for limit-order-book sequence models."""
__version__ = "0.1.0"
