"""B200-native ZipServ: TCA-TBE lossless bf16 compression, ZipGEMM and
compressed-KV decode attention for sm_100a.

Kernels live in libzipserv_b200.so (built in-tree by build_lib.py); Python
modules here are thin torch-facing wrappers over its C ABI."""
from .codec import Compressed, analyze_exponents, compress, compress_host, decompress, to_device, zipgemm  # noqa: F401

__all__ = ["Compressed", "analyze_exponents", "compress", "compress_host", "decompress", "to_device", "zipgemm"]
from .attention import compress_kv, decode_attention, flash_attn_with_kvcache, pad_kv_by_kv_head  # noqa: E402,F401

__all__ += ["compress_kv", "decode_attention", "flash_attn_with_kvcache", "pad_kv_by_kv_head"]
from . import store  # noqa: E402,F401  (save / load of compressed matrices)
