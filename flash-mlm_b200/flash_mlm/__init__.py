"""flash-mlm on B200: fused masked-language-model attention forward (sm_100a).

Drop-in for the reference package's public API
(src/flash_mlm/__init__.py:59-68).  The attention, pack and unpack work runs in
hand-written CUDA kernels (libflashmlm.so); calling them without a CUDA device
or without the built library raises instead of falling back.
"""

from flash_mlm.host.cache import InferenceCache, PackMetadata, PackingCache
from flash_mlm.host.host import flash_attn_mlm, flash_attn_mlm_compressed, flash_attn_mlm_precompressed
from flash_mlm.host.host_utils import build_pack_metadata, unpack_from_kernel
from flash_mlm._lib import check_device_errors

__all__ = [
    "PackMetadata",
    "PackingCache",
    "InferenceCache",
    "build_pack_metadata",
    "unpack_from_kernel",
    "flash_attn_mlm",
    "flash_attn_mlm_compressed",
    "flash_attn_mlm_precompressed",
]
