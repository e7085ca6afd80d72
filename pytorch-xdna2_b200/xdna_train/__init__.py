"""B200-native training backend with torch-xdna2's plugin surface."""
__version__ = "0.1.0"
