"""B200-native ZipServ: TCA-TBE lossless bf16 compression, ZipGEMM and
compressed-KV decode attention for sm_100a.

Kernels live in libzipserv_b200.so (built in-tree by build_lib.py); Python
modules here are thin torch-facing wrappers over its C ABI."""
from .codec import Compressed, analyze_exponents, compress, compress_host, decompress, to_device, zipgemm  # noqa: F401

__all__ = ["Compressed", "analyze_exponents", "compress", "compress_host", "decompress", "to_device", "zipgemm"]
from .attention import (compress_kv, decode_attention, decode_attention_dense, flash_attn_with_kvcache,  # noqa: E402,F401
                        pad_kv_by_kv_head, pad_kv_token_major)

__all__ += ["compress_kv", "decode_attention", "decode_attention_dense", "flash_attn_with_kvcache", "pad_kv_by_kv_head",
            "pad_kv_token_major"]
from . import store  # noqa: E402,F401  (save / load of compressed matrices)
