"""flash_attn.flash_attn_interface -> fable_attn.flash_attn_interface (FA-2 order)."""
from fable_attn.flash_attn_interface import *  # noqa: F401,F403
from fable_attn.flash_attn_interface import flash_attn_combine, flash_attn_with_kvcache  # noqa: F401
