"""phung5_b200 — a B200-native (sm_100a) speculative-decoding LLM serving engine."""
import torch  # noqa: F401  (loads libc10/libtorch before the native extension)

__version__ = "0.1.0"
