"""B200 (sm_100a) FlashAttention forward behind the reference's Python API.

Same public surface as the reference package
(src/flash_attention_sm75/__init__.py:1-4): ``flash_attention_forward`` and
``__version__``; ``flash_attention_forward_kvcache`` (Nq != Nk),
``flash_attention_forward_host`` (host buffers, copies overlapped with compute),
``flash_attention_varlen_forward`` (packed variable-length batches),
``flash_attention_forward_padded`` (padded batches with per-entry row ranges)
and ``flash_attention`` / ``flash_attention_padded`` / ``flash_attention_varlen``
(forward + backward) are additions.
"""
from .ops import (flash_attention, flash_attention_forward, flash_attention_forward_host,
                  flash_attention_forward_kvcache, flash_attention_forward_padded,
                  flash_attention_padded, flash_attention_varlen, flash_attention_varlen_forward)

__version__ = "0.1.0"
__all__ = ["flash_attention_forward", "flash_attention_forward_kvcache",
           "flash_attention_forward_host", "flash_attention_varlen_forward",
           "flash_attention_forward_padded", "flash_attention", "flash_attention_padded",
           "flash_attention_varlen"]
