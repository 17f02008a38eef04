"""B200-native LoopSpec decode engine (pipelined self-speculative decoding on looped transformers)."""

from .config import ModelConfig, PRESETS, get_config, parse_loopspec_flags  # noqa: F401

__version__ = "0.1.0"
