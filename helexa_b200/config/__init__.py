from .model_config import FULL, LINEAR, ModelConfig
from .presets import PRESETS, get_preset

__all__ = ["ModelConfig", "FULL", "LINEAR", "PRESETS", "get_preset"]
