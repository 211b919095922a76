"""phung5_b200 — a B200-native (sm_100a) speculative-decoding LLM serving engine."""
__version__ = "0.1.0"
