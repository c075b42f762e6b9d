"""futon_b200 — B200-native encoder forward pass for futon packs.

The CUDA kernels, the native tokenizer and the C ABI live in
libfuton_cuda.so (sources in csrc/, headers include/futon_cuda.h and
include/futon_tokenizer.h); this package is the host-side mirror of the
reference's native Provider over it.
"""
from ._lib import CanceledError, FutonError, FutonLibraryError, device_count
from .pack import Pack, PackConfig, PackError, load_pack, write_pack
from .provider import CancelFlag, Model, Options, Provider, new, pack_ids
from .tokenizer import Tokenizer, TokenizerConfig

__all__ = [
    "CanceledError", "CancelFlag", "FutonError", "FutonLibraryError", "Model", "Options", "Pack",
    "PackConfig", "PackError", "Provider", "Tokenizer", "TokenizerConfig", "device_count",
    "load_pack", "new", "pack_ids", "write_pack",
]
