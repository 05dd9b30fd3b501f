"""pan2_b200: a B200-native (sm_100a) training and inference framework for PAN 2's video MMDiT."""
__version__ = "0.1.0"
