"""flash_attn_interface (FA-3 argument order) -> fable_attn.fa3_interface."""
from fable_attn.fa3_interface import *  # noqa: F401,F403
from fable_attn.fa3_interface import (  # noqa: F401
    flash_attn_func, flash_attn_qkvpacked_func, flash_attn_varlen_func, flash_attn_with_kvcache,
    flash_attn_combine, get_scheduler_metadata,
)
