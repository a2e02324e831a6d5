from flash_mlm.host.host import flash_attn_mlm, flash_attn_mlm_compressed, flash_attn_mlm_precompressed
from flash_mlm.host.cache import InferenceCache, PackMetadata, PackingCache
from flash_mlm.host.host_utils import build_pack_metadata, unpack_from_kernel

__all__ = [
    "flash_attn_mlm",
    "flash_attn_mlm_compressed",
    "flash_attn_mlm_precompressed",
    "PackMetadata",
    "build_pack_metadata",
    "unpack_from_kernel",
    "InferenceCache",
    "PackingCache",
]
