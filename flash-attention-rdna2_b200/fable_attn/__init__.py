"""fable_attn — exact FlashAttention for NVIDIA B200 (sm_100a) behind the flash-attn API.

    import fable_attn; fable_attn.install_as_flash_attn()   # `import flash_attn` now resolves here
or directly:
    from fable_attn import flash_attn_func

Forward, backward, varlen, paged-KV decode and split merge all run on hand-written CUDA
kernels (fable_attn._C over libfable_attn.so, whose C ABI is include/fable_attn.h).
"""
import sys

from .flash_attn_interface import (
    flash_attn_func,
    flash_attn_qkvpacked_func,
    flash_attn_kvpacked_func,
    flash_attn_varlen_func,
    flash_attn_varlen_qkvpacked_func,
    flash_attn_varlen_kvpacked_func,
    flash_attn_combine,
    flash_attn_with_kvcache,
)
from . import bert_padding
from . import torch_op

torch_op.register()



def device_error(clear=False):
    """Error bits the kernels recorded on the current device (0 = none): a pipeline wait that gave
    up (the kernel unwound and its outputs are not valid), a paged-K/V entry outside the cache, or
    a rotary position outside its table.  Synchronises with the device; clear=True resets them."""
    from . import _C
    return int(_C.device_error(bool(clear)))


__all__ = [
    "device_error", "flash_attn_func", "flash_attn_qkvpacked_func", "flash_attn_kvpacked_func", "flash_attn_varlen_func",
    "flash_attn_varlen_qkvpacked_func", "flash_attn_varlen_kvpacked_func", "flash_attn_combine",
    "flash_attn_with_kvcache", "bert_padding", "install_as_flash_attn",
]

__version__ = "0.2.0"

# Version announced when installed under the flash_attn name: libraries gate features on it
# (window_size, softcap need >= 2.4), so the drop-in reports the FA-2 API level it covers, with a
# local suffix that keeps the implementation visible (reference package/fable_attn/__init__.py:54).
FLASH_ATTN_API_VERSION = "2.8.3+fable." + __version__


def install_as_flash_attn():
    """Register this package under the module names foreign code imports:
    flash_attn (FA-2 order), flash_attn.flash_attn_interface, flash_attn.bert_padding,
    flash_attn.layers(.rotary), and flash_attn_interface (FA-3 order).  FA-2 and FA-3 stay on
    separate names because their positional orders differ."""
    from . import flash_attn_interface as _fi
    from . import fa3_interface as _fi3
    from . import bert_padding as _bp
    from . import layers as _layers
    from .layers import rotary as _rotary

    me = sys.modules[__name__]
    me.__dict__.setdefault("_fable_own_version", __version__)
    me.__version__ = FLASH_ATTN_API_VERSION
    _fi.__version__ = FLASH_ATTN_API_VERSION
    sys.modules["flash_attn"] = me
    sys.modules["flash_attn.flash_attn_interface"] = _fi
    sys.modules["flash_attn.bert_padding"] = _bp
    sys.modules["flash_attn.layers"] = _layers
    sys.modules["flash_attn.layers.rotary"] = _rotary
    sys.modules["flash_attn_interface"] = _fi3
    return me
