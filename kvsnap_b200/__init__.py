"""kvsnap_b200: a B200-native data plane for kvsnap's KV-cache snapshots.

Modules:
  dataplane   TorchBlockDataPlane, CudaPool, PinnedAllocation (drop-in for kvsnap.connector.dataplane),
              PendingDigests, DigestCache, CorruptBlockError
  blobs       write_blobs, read_and_restore: KVSBLOB1 files between pinned memory and disk
  native_io   NativeIO, get_io_backend (drop-in for kvsnap.store.native_io's native backend)
  crc32c      crc32c (drop-in for kvsnap.store.crc32c)
  reshard     TP regroup of head shards between tensor-parallel sizes
  build       builds _native/_cuda_native.so and _native/_io_native.so in-tree
"""
__version__ = "0.1.0"
