from .decoder import DecoderConfig, DecoderLM, DecoderLayer, RMSNorm, PRESETS, get_config

__all__ = ["DecoderConfig", "DecoderLM", "DecoderLayer", "RMSNorm", "PRESETS", "get_config"]
