"""flash_attn.layers -> fable_attn.layers."""
from . import rotary  # noqa: F401
