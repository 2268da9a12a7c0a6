"""B200-native ZipServ: TCA-TBE lossless bf16 compression, ZipGEMM and
compressed-KV decode attention for sm_100a.

Kernels live in libzipserv_b200.so (built in-tree by build_lib.py); Python
modules here are thin torch-facing wrappers over its C ABI."""
from .codec import Compressed, analyze_exponents, compress, decompress, zipgemm  # noqa: F401

__all__ = ["Compressed", "analyze_exponents", "compress", "decompress", "zipgemm"]
