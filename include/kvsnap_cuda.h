/*
 * kvsnap_cuda.h: the C ABI of kvsnap_b200/_native/_cuda_native.so.
 *
 * Two groups of entry points, all extern "C", plain pointers and sizes, no
 * torch types. Every int-returning call returns 0 on success and -1 on error,
 * with the message in the calling thread's kvsnap_cuda_error().
 *
 * 1. The pinned-pool ABI, version 2: the same symbols, argument meaning and
 *    error behaviour as the reference's csrc/dataplane/cuda_pool.cpp, which
 *    kvsnap/connector/dataplane.py:47-60 binds with ctypes. A build of this
 *    library dropped in as kvsnap/_native/_cuda_native<EXT_SUFFIX>.so (or named
 *    by KVSNAP_CUDA_LIBRARY) serves the reference's CudaPool unchanged.
 *
 * 2. The data-plane kernels (kvsnap_dp_*), sm_100a CUDA. They replace the
 *    reference's restore kernel (kvsnap/connector/copy_kernel.py:23-49), its
 *    torch save gather (kvsnap/connector/dataplane.py:409-427) and its host
 *    checksums (csrc/dataplane/io.cpp:27-47 CRC32C, hashlib SHA-256 in
 *    kvsnap/store/store.py:616-629 and kvsnap/connector/volatile.py:141-151).
 *    Tables passed to them (spans, block ids, addresses) live in device memory
 *    (or mapped pinned memory); packed-block addresses may be device memory or
 *    pinned host memory from cudaHostAlloc, which the kernels read and write in
 *    place over the host link.
 */
#ifndef KVSNAP_CUDA_H
#define KVSNAP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- 1. pinned pool (ABI 2) ------------------------------------------------ */

/* Thread-local text of the last error (reference cuda_pool.cpp:50). */
const char* kvsnap_cuda_error(void);
/* Returns 2 (reference cuda_pool.cpp:52; checked at dataplane.py:64-66). */
int kvsnap_pool_abi_version(void);
/* A pinned arena of `capacity` bytes on `device` plus its own non-blocking copy
   stream; NULL on error (reference cuda_pool.cpp:53-62). */
void* kvsnap_pool_create(size_t capacity, int device);
/* Frees the pool; if its stream cannot be drained the pinned memory is kept
   (quarantined) instead of freed (reference cuda_pool.cpp:63, 30-38). */
void kvsnap_pool_destroy(void* pool);
/* Drains the copy stream, then frees; on a failed drain the pool stays intact
   and -1 is returned (reference cuda_pool.cpp:66-74). */
int kvsnap_pool_close_checked(void* pool);
/* The copy stream's handle, borrowed (reference cuda_pool.cpp:78-85). */
int kvsnap_pool_copy_stream(void* pool, uintptr_t* stream);
/* First-fit reservation. Fails with a message containing "pinned capacity
   exhausted" when it cannot fit (reference cuda_pool.cpp:86-104). Start offsets
   are rounded up to 16 bytes so every allocation suits 16-byte vector access. */
int kvsnap_pool_reserve(void* pool, size_t size, uint64_t* id, void** ptr);
/* One async copy between device memory and an allocation on the copy stream;
   a device-to-host copy first waits for `producer_stream` (reference
   cuda_pool.cpp:107-133). */
int kvsnap_pool_copy(void* pool, uint64_t id, size_t host_offset, void* device_ptr, size_t size, int to_host,
                     uintptr_t producer_stream);
/* `height` rows of `width` bytes, strided on both sides (reference cuda_pool.cpp:139-169). */
int kvsnap_pool_copy_2d(void* pool, uint64_t id, size_t host_offset, size_t host_pitch, void* device_ptr,
                        size_t device_pitch, size_t width, size_t height, int to_host, uintptr_t producer_stream);
/* Block until the allocation's last copy completes (reference cuda_pool.cpp:170-177). */
int kvsnap_pool_wait(void* pool, uint64_t id);
/* 1 when idle, 0 while a copy is in flight, -1 on error (reference cuda_pool.cpp:178-189). */
int kvsnap_pool_ready(void* pool, uint64_t id);
/* Wait, then return the bytes to the arena (reference cuda_pool.cpp:190-199). */
int kvsnap_pool_release(void* pool, uint64_t id);
/* Extension (no reference counterpart): kvsnap_pool_copy queued on `stream`
   (0: the pool's copy stream) instead of the pool's stream, with no producer
   fence: the caller orders its own stream. Lets a restore's host-to-device
   copies run beside a save's device-to-host copies (the host link is full
   duplex). The allocation's completion event is recorded on `stream`. */
int kvsnap_pool_copy_on(void* pool, uint64_t id, size_t host_offset, void* device_ptr, size_t size, int to_host,
                        uintptr_t stream);
/* Extension (no reference counterpart): record the allocation's completion
   event on `stream` (0: the pool's copy stream) now, so wait/ready/release
   also fence kernels queued there that read or write the allocation in place. */
int kvsnap_pool_mark(void* pool, uint64_t id, uintptr_t stream);
/* Extension (no reference counterpart): n copies in one call, entry k moving
   sizes[k] bytes between allocation ids[k] at host_offsets[k] and device
   address device_ptrs[k], queued in order on `stream` (0: the pool's copy
   stream) with no producer fence. Every entry is checked before any is
   queued; each allocation's completion event is recorded after the last copy.
   Consecutive entries whose host and device ranges both continue the previous
   one's move in one copy.
   Replaces n kvsnap_pool_copy_on calls (one per block of a host-tier
   snapshot, reference volatile.py:281-307) with one. */
int kvsnap_pool_copy_many(void* pool, int64_t n, const uint64_t* ids, const uint64_t* host_offsets,
                          const uint64_t* device_ptrs, const uint64_t* sizes, int to_host, uintptr_t stream);
/* Extension: kvsnap_pool_wait for each of n allocations, in one call. */
int kvsnap_pool_wait_many(void* pool, int64_t n, const uint64_t* ids);

/* Extension for the cross-owner host tier (replaces the socket copy of
   kvsnap/connector/vllm.py:524-534 and connector/volatile.py:87-138): a pool
   whose arena is POSIX shared memory named `name` (one path component that
   starts with '/', created with mode 0600, so only this user's processes open
   it), registered with CUDA as pinned and mapped memory. It behaves as
   kvsnap_pool_create's; destroying it unlinks the name, and the mappings other
   processes made stay valid until they close them. NULL on error (a name
   already in use included). */
void* kvsnap_pool_create_shared(size_t capacity, int device, const char* name);
/* Extension: the arena's first byte and its capacity, so an owner can tell
   other processes where an allocation lies in its shared arena. */
int kvsnap_pool_arena(void* pool, void** base, size_t* capacity);
/* Map another process's shared arena read-only into this one and register it
   with CUDA (pinned, mapped, read-only) on `device`, so that its blocks serve
   as restore sources in place: *base and *size receive the mapping. */
int kvsnap_shared_open(const char* name, int device, void** base, size_t* size);
/* Unregister and unmap a mapping from kvsnap_shared_open. The caller first
   waits for every copy and kernel that reads it. */
int kvsnap_shared_close(void* base, size_t size);

/* ---- 2. data-plane kernels --------------------------------------------------- */

#define KVSNAP_DP_ABI_VERSION 1

/* Status bits a kernel ORs into its status word instead of faulting. */
#define KVSNAP_DP_MISALIGNED 1u      /* an address or size broke the vector width */
#define KVSNAP_DP_BAD_BLOCK 2u       /* a block id outside its cache */
#define KVSNAP_DP_CRC_MISMATCH 4u    /* a block's CRC32C differed from the expected one */
#define KVSNAP_DP_BAD_CUT 8u         /* KVSNAP_DP_PAIRS or _SPLIT* met spans that do not cut that way */

/* OR into a `vec` argument when every packed address is device memory: the
   kernels then cut each unit into 4 segments, move whole 128-byte lines
   coalesced, each group of 8 lanes 1 KiB of its segment a step, and CRC each
   lane's bytes in its registers through per-lane tables (HBM-friendly),
   instead of 16 bytes a lane in 512-byte steps (host-link friendly).
   Needs vec 16. */
#define KVSNAP_DP_HBM 0x100
/* With KVSNAP_DP_HBM, a hint when every span is small (up to 8 KiB, e.g. a
   tensor-parallel shard's): each warp then takes contiguous units and folds
   the CRCs of a block's consecutive spans as one run. Results are the same
   with or without it. */
#define KVSNAP_DP_RUNS 0x200
/* With KVSNAP_DP_RUNS, a hint when every span has one size S of 2 or 4 KiB
   (a TP-8 or TP-16 shard's) and nspans is even: each unit is then a pair of
   consecutive spans, so each lane owns 2 * S / 32 contiguous packed bytes and
   a unit's CRC is placed once per 2 * S. A pair whose spans differ sets
   KVSNAP_DP_BAD_CUT and is skipped. Results are the same with or without
   it. */
#define KVSNAP_DP_PAIRS 0x400
/* With KVSNAP_DP_HBM, without KVSNAP_DP_RUNS: each unit is one of 2 (SPLIT2)
   or 4 (SPLIT4) equal pieces of a span, so that large spans (a Qwen3-8B
   layer's 32 KiB) move in 16 KiB units, which measured faster. Every span
   must cut into pieces that are a multiple of 4 KiB; one that does not sets
   KVSNAP_DP_BAD_CUT and is skipped. The last block of a gather with
   valid_tokens > 0 is not split. Results are the same with or without it. */
#define KVSNAP_DP_SPLIT2 0x800
#define KVSNAP_DP_SPLIT4 0x1000
#define KVSNAP_DP_SPLIT_MASK 0x1800
/* With KVSNAP_DP_HBM and crc_out: add this call's share of each block's CRC
   to crc_out as it stands (not cleared first) and leave it raw (no finish
   step). A save that moves each block in several calls, a range of spans at
   a time, ends with kvsnap_dp_crc32c_finish. */
#define KVSNAP_DP_CRC_ACCUMULATE 0x2000

/*
 * One registered layer view, i.e. one span of every packed block. A packed
 * block is the spans back to back in registration order (layer-name order,
 * reference dataplane.py:226); span s of cache block b lives at
 * base + b * pitch and is `bytes` long, dense, copied in storage order
 * (dataplane.py:283-305). 64 bytes.
 */
typedef struct kvsnap_span {
    int64_t base;         /* device address of block 0 of this view */
    int64_t pitch;        /* bytes between consecutive blocks */
    int64_t offset;       /* byte offset of the span inside a packed block */
    int64_t bytes;        /* span bytes per block */
    int64_t token_pitch;  /* bytes between consecutive token slots (tail zeroing) */
    int32_t tokens;       /* token slots per block (the block size) */
    int32_t row_bytes;    /* contiguous bytes of one (head, token) row */
    int64_t nblocks;      /* blocks in this cache, for in-kernel bounds checks */
    uint32_t crc_shift;   /* x^(8 * bytes after this span) mod P, filled by kvsnap_dp_plan */
    uint32_t flags;       /* reserved, 0 */
} kvsnap_span;

int kvsnap_dp_abi_version(void);

/* Fill `offset` and `crc_shift` of a host span array in registration order;
   writes the packed block size to *block_bytes. Host-only, no CUDA. */
int kvsnap_dp_plan(kvsnap_span* spans, int nspans, uint64_t* block_bytes);

/* CRC32C of a host buffer with a prior value: the host library's semantics
   (reference io.cpp:39-44), exported here for self-checks. Host-only. */
uint32_t kvsnap_dp_crc32c_host(const void* data, size_t size, uint32_t prior);

/*
 * Save gather (replaces dataplane.py:388-437 and its host hashing). For each
 * i < n and span s: copy the span of cache block blocks[i] to
 * targets[i] + spans[s].offset. In block n-1, token slots >= valid_tokens are
 * written as zeros when valid_tokens > 0 (dataplane.py:262-272, 433-436).
 * When crc_out is not NULL, crc_out[i] receives the CRC32C of packed block i
 * as written (zeros included). `vec` is 16 or 8: the alignment every address,
 * pitch, offset and span size meets. `ctas` 0 picks a default. status (device
 * word, may be NULL) receives KVSNAP_DP_* bits.
 */
int kvsnap_dp_gather(const kvsnap_span* spans, int nspans, uint64_t block_bytes, const int64_t* blocks,
                     const int64_t* targets, int64_t n, int32_t valid_tokens, uint32_t* crc_out,
                     uint32_t* status, int vec, int ctas, uintptr_t stream);

/*
 * Restore scatter (replaces copy_kernel.py:23-49 and the loader-thread CRC
 * check, store.py:717-718). For each i < n and span s: copy
 * sources[i] + spans[s].offset to the span of cache block blocks[i]. When
 * crc_out is not NULL it receives the CRC32C of each source block; when
 * expect is not NULL as well, a block whose CRC differs sets
 * KVSNAP_DP_CRC_MISMATCH in *status (its bytes are already written: callers
 * that must not write unverified bytes verify first with kvsnap_dp_crc32c).
 * A non-NULL `gate` is read by every CTA first: when *gate is non-zero the
 * kernel writes nothing.
 */
int kvsnap_dp_scatter(const kvsnap_span* spans, int nspans, uint64_t block_bytes, const int64_t* sources,
                      const int64_t* blocks, int64_t n, uint32_t* crc_out, const uint32_t* expect,
                      const uint32_t* gate, uint32_t* status, int vec, int ctas, uintptr_t stream);

/* CRC32C of n packed blocks of block_bytes at addrs[i] (device or pinned host).
   With expect not NULL, mismatches set KVSNAP_DP_CRC_MISMATCH in *status. */
int kvsnap_dp_crc32c(const int64_t* addrs, int64_t n, uint64_t block_bytes, uint32_t* crc_out,
                     const uint32_t* expect, uint32_t* status, int vec, int ctas, uintptr_t stream);

/* SHA-256 of n packed blocks of block_bytes at addrs[i]; digest i is the 32
   big-endian bytes at out + 32 * i, the bytes of hashlib.sha256(block).digest()
   (the store's content id, store.py:623). One lane hashes one block. */
int kvsnap_dp_sha256(const int64_t* addrs, int64_t n, uint64_t block_bytes, uint8_t* out, uintptr_t stream);

/* The same hash, one part of every block at a time, so that the bytes of only
   one part need to be in device memory at once. Call it for parts in order:
   bytes [done_bytes, done_bytes + part_bytes) of each block of total_bytes,
   that part starting at addrs[i]. state holds 8 words a block between calls
   (n * 32 bytes, device memory): the first part (done_bytes 0) starts from
   the SHA-256 initial value, later ones from state. Parts before the last
   must be whole 64-byte chunks; the last part (done_bytes + part_bytes ==
   total_bytes) pads and writes the digests to out as kvsnap_dp_sha256 does,
   the others write state. */
int kvsnap_dp_sha256_part(const int64_t* addrs, int64_t n, uint64_t part_bytes, uint64_t done_bytes,
                          uint64_t total_bytes, uint32_t* state, uint8_t* out, uintptr_t stream);

/* Land one column of n packed blocks from a device slot where each block goes:
   bytes [0, len) at src + i * src_stride are copied to targets[i] + offset,
   for i < n. Targets may be pinned host memory (written over the host link by
   the SMs, one 4 KiB piece a warp step) or device memory. No counterpart in
   the reference: its save copies whole chunks with cudaMemcpyAsync
   (kvsnap/connector/dataplane.py:418-427); a bounded save's columns are too
   small for the copy engine (256 KiB copies to scattered per-block targets ran
   at 30 GB/s on B200, this kernel at 52.6 with 16 CTAs). src, src_stride,
   offset, len and every target must be multiples of 16 bytes: a block that
   is not sets KVSNAP_DP_MISALIGNED in *status and is skipped. `ctas` 0 picks 16. */
int kvsnap_dp_land(const void* src, int64_t src_stride, const int64_t* targets, int64_t offset, int64_t n,
                   int64_t len, uint32_t* status, int ctas, uintptr_t stream);

/* Land one column of n packed blocks whose targets lie at one pitch: bytes
   [0, len) at src + i * src_stride are copied to dst + i * dst_pitch, for
   i < n, as one copy-engine transfer (cudaMemcpy2DAsync, device to host) on
   `stream`. dst is pinned host memory. A bounded save's column is n small
   pieces, so when its targets are evenly spaced (blocks reserved back to back,
   or one buffer) this moves the column at the copy engine's rate while the SMs
   gather the next one; otherwise kvsnap_dp_land. No counterpart in the
   reference, whose save copies whole chunks with cudaMemcpyAsync
   (kvsnap/connector/dataplane.py:418-427). */
int kvsnap_dp_land_strided(const void* src, int64_t src_stride, void* dst, int64_t dst_pitch, int64_t n,
                           int64_t len, uintptr_t stream);

/* Finish raw CRC accumulators that KVSNAP_DP_HBM gathers or scatters left
   under KVSNAP_DP_CRC_ACCUMULATE: crc[i] becomes block i's CRC32C; with
   expect not NULL, mismatches set KVSNAP_DP_CRC_MISMATCH in *status. */
int kvsnap_dp_crc32c_finish(uint32_t* crc, const uint32_t* expect, int64_t n, uint64_t block_bytes,
                            uint32_t* status, uintptr_t stream);

/*
 * The reference restore kernel's exact interface (copy_kernel.py:43-49): all
 * six tables are device int64 arrays; job j copies layer_words[l] 8-byte words
 * of layer l = j % n_layers from sources[b] + layer_offsets[l] to
 * layer_bases[l] + blocks[b] * layer_pitches[l], b = j / n_layers. No checksums.
 */
int kvsnap_dp_copy_host_blocks(const int64_t* sources, const int64_t* blocks, int64_t n_blocks,
                               const int64_t* layer_offsets, const int64_t* layer_bases,
                               const int64_t* layer_pitches, const int64_t* layer_words, int64_t n_layers,
                               int ctas, uintptr_t stream);

/*
 * Tensor-parallel regroup (no reference counterpart: the reference treats a
 * restore at another TP size as a miss, kvsnap/connector/vllm.py:9-14). This
 * rank's cache holds H heads a layer; the snapshot was saved by `groups` times
 * as many ranks, shard q holding heads [q*H/groups, (q+1)*H/groups). For each
 * block i and span s, every (head, token) row of cache block blocks[i] is read
 * from shard q's packed block at shards[i*groups + q] + src_spans[s].offset.
 * src_spans describe one shard's packed layout (the same spans with H/groups
 * heads; offsets from kvsnap_dp_plan). Shard addresses may be this GPU's
 * memory or a peer's mapped with kvsnap_dp_ipc_open: the kernel reads them
 * with plain loads over NVLink. The caller orders producer and consumer ranks.
 */
int kvsnap_dp_regroup(const kvsnap_span* dst_spans, const kvsnap_span* src_spans, int nspans, const int64_t* shards,
                      int groups, const int64_t* blocks, int64_t n, uint32_t* status, int ctas, uintptr_t stream);

/* Device memory from cudaMalloc, shareable with other processes through
   kvsnap_dp_ipc_export (memory from torch's expandable segments is not). */
int kvsnap_dp_device_alloc(size_t size, int device, void** ptr);
int kvsnap_dp_device_free(void* ptr);
/* A 64-byte CUDA IPC handle for an allocation made by kvsnap_dp_device_alloc. */
int kvsnap_dp_ipc_export(void* ptr, void* handle);
/* Map another process's allocation into this one on `device` (peer access enabled lazily). */
int kvsnap_dp_ipc_open(const void* handle, int device, void** ptr);
int kvsnap_dp_ipc_close(void* ptr);

/*
 * Verified restore scatter that allocates nothing. No counterpart in the
 * reference. For callers that cannot allocate device memory: a serving worker
 * whose KV cache was sized to fill the GPU has no room left for a CRC buffer,
 * and host code that must not enter an allocator (which may synchronise the
 * device) cannot ask for one. The per-block CRC32C accumulators and one gate
 * word live in one fixed scratch array inside this library,
 * (KVSNAP_DP_STATIC_MAX_BLOCKS + 64) x 4 bytes, held on every GPU that loads
 * the library until the process exits. The caller passes inputs and outputs.
 *
 * Check before write: every source block's CRC32C is computed and compared
 * with expect[i] first; the scatter then runs gated on that verdict. On a
 * mismatch nothing is written to the cache and KVSNAP_DP_CRC_MISMATCH is set
 * in *status (other bits as kvsnap_dp_scatter sets them). `vec` takes the same
 * flags as kvsnap_dp_scatter (KVSNAP_DP_HBM and its unit cuts for sources in
 * device memory). Sources in pinned host memory cross the host link twice,
 * once for the check and once for the copy.
 *
 * n above the maximum is rejected with an error and nothing is launched.
 * Every call looks up the scratch's device address (cudaGetSymbolAddress, no
 * allocation); make the first call on a device before any stream capture,
 * since it may load the module. Every call shares the scratch and clears what
 * it uses at its start: calls whose work overlaps on the GPU race on it and
 * must not be issued concurrently.
 */
#define KVSNAP_DP_STATIC_MAX_BLOCKS 65536
int kvsnap_dp_scatter_verify_static(const kvsnap_span* spans, int nspans, uint64_t block_bytes,
                                    const int64_t* sources, const int64_t* blocks, int64_t n,
                                    const uint32_t* expect, uint32_t* status, int vec, int ctas, uintptr_t stream);

#ifdef __cplusplus
}
#endif
#endif /* KVSNAP_CUDA_H */
