"""flash_attn.layers.rotary -> fable_attn.layers.rotary."""
from fable_attn.layers.rotary import *  # noqa: F401,F403
from fable_attn.layers.rotary import RotaryEmbedding, apply_rotary_emb  # noqa: F401
