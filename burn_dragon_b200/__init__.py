"""B200-native BDH / Dragon training and inference."""

__version__ = "0.1.0"
