"""Module-level API: QuantizedLinearInt8 / QuantizedLinearInt4 and quantize_model_*."""
