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
from ._shard import (
    assemble_chunk_ranges,
    compress_chunk_range,
    compress_shard,
    decompress_chunk_range,
    decompress_shard,
    gather_chunk_ranges,
    gather_index,
    plan_chunk_ranges,
    plan_shards,
    split_chunk_range,
)

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
    "plan_chunk_ranges",
    "compress_chunk_range",
    "gather_chunk_ranges",
    "assemble_chunk_ranges",
    "split_chunk_range",
    "decompress_chunk_range",
]
