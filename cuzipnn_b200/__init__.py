"""B200-native ZipNN lossless tensor compression: the API of cuZipNN (ruihe774/cuZipNN,
src/cuzipnn/__init__.py) on hand-written sm_100a kernels, with rANS as the entropy coder."""

from ._codec import (
    compress_tensor,
    compress_tensor_with_crc32,
    compress_tensors,
    decompress_tensor,
    decompress_tensors,
    hash_tensor_with_crc32,
    last_decode_status,
)
from ._shard import compress_shard, decompress_shard, gather_index, plan_shards

__all__ = [
    "compress_tensor",
    "compress_tensor_with_crc32",
    "compress_tensors",
    "decompress_tensor",
    "decompress_tensors",
    "hash_tensor_with_crc32",
    "last_decode_status",
    "plan_shards",
    "compress_shard",
    "decompress_shard",
    "gather_index",
]
