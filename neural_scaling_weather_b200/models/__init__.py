"""Model definitions."""

from .swin import SwinTransformer, TimeStepper, get_model, load_model  # noqa: F401
