"""flash_attn import name backed by fable_attn (FA-2 argument order)."""
from fable_attn import FLASH_ATTN_API_VERSION as __version__  # noqa: F401
from fable_attn.flash_attn_interface import (  # noqa: F401
    flash_attn_func,
    flash_attn_qkvpacked_func,
    flash_attn_kvpacked_func,
    flash_attn_varlen_func,
    flash_attn_varlen_qkvpacked_func,
    flash_attn_varlen_kvpacked_func,
    flash_attn_combine,
    flash_attn_with_kvcache,
)
from . import bert_padding, flash_attn_interface, layers  # noqa: F401,E402
