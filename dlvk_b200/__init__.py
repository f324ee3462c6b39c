"""dlvk_b200: a B200-native (sm_100a) deep-learning framework with the
capabilities and public API of DLVK."""
__version__ = "0.1.0"
