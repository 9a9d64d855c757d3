"""flash_attn.layers: the rotary embedding layer (plain torch)."""
from . import rotary

__all__ = ["rotary"]
