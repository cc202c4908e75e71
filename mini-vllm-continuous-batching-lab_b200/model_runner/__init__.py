from .base import AttentionGroup, AttentionMetadata, ModelConfig

__all__ = ["AttentionGroup", "AttentionMetadata", "ModelConfig"]
