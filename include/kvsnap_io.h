/*
 * kvsnap_io.h: the C ABI of kvsnap_b200/_native/_io_native.so (host only).
 *
 * Same symbols, argument meaning and errno-style results as the reference's
 * csrc/dataplane/io.cpp, which kvsnap/store/native_io.py:59-65 binds with
 * ctypes (ABI version 1). Unlike the pool library, these return an errno value
 * (0 on success), never -1 (reference io.cpp:50).
 */
#ifndef KVSNAP_IO_H
#define KVSNAP_IO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Returns 1 (reference io.cpp:48; checked at native_io.py:69). */
int kvsnap_io_abi_version(void);
/* CRC32C (Castagnoli, reflected 0x82F63B78) continuing from `prior`
   (reference io.cpp:39-44). */
uint32_t kvsnap_crc32c_extend(const void* data, size_t size, uint32_t prior);
/* kvsnap_crc32c_extend(data, size, 0) (reference io.cpp:45-47). */
uint32_t kvsnap_crc32c(const void* data, size_t size);
/* Write all of data at offset, retrying EINTR and short writes; fdatasync when
   durable. EINVAL for a negative or overflowing offset (reference io.cpp:51-69). */
int kvsnap_pwrite_all(int fd, const void* data, size_t size, int64_t offset, int durable);
/* Read exactly size bytes at offset; EIO at end of file (reference io.cpp:71-81). */
int kvsnap_pread_all(int fd, void* data, size_t size, int64_t offset);
/* A transfer pool that runs at most `workers` (1..64) transfers and at most
   max_bytes at once; NULL on bad arguments (reference io.cpp:130-133, which
   runs them on that many worker threads). Here each transfer runs on its
   caller's thread once admitted: the call waits for its result either way. */
void* kvsnap_io_pool_create(size_t workers, size_t max_bytes);
void kvsnap_io_pool_destroy(void* pool);
/* Run one pread (write=0) or pwrite (write=1) through the pool and wait for
   it: EINVAL for bad arguments, EMSGSIZE above the pool's byte limit,
   ECANCELED when the pool is destroyed before admitting it (reference
   io.cpp:135-154). Destroying the pool waits for admitted transfers. */
int kvsnap_io_pool_transfer(void* pool, int fd, void* data, size_t size, int64_t offset, int write, int durable);

#ifdef __cplusplus
}
#endif
#endif /* KVSNAP_IO_H */
