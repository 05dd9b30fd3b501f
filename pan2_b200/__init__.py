"""pan2_b200: a B200-native (sm_100a) training and inference framework for PAN 2's video MMDiT."""
import torch as _torch  # noqa: F401  (loads libtorch, which the compiled extension pan2_b200._C links)

__version__ = "0.1.0"
