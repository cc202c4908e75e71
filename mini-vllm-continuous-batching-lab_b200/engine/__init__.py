from .step_metadata import StepMetadata, StepMetadataBuilder

__all__ = ["StepMetadata", "StepMetadataBuilder"]
