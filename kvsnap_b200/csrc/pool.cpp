// Pinned host arena with a copy stream: the pool half of _cuda_native.so.
//
// Implements the reference's pinned-pool C ABI version 2 (kvsnap
// csrc/dataplane/cuda_pool.cpp:50-199, bound by kvsnap/connector/dataplane.py:38-131)
// with the same symbols, argument meaning and failure rules:
//   * every entry returns 0 / -1 with the text in a thread-local error string;
//   * a device-to-host copy first makes the copy stream wait for the producer;
//   * an allocation's completion authority is its event, and when an enqueue or
//     an event record fails the allocation falls back to draining the stream,
//     so memory a DMA may still touch is never handed out again;
//   * a pool whose stream cannot be drained keeps (quarantines) its memory.
// Written against the CUDA runtime API only, so tests can compile it against a
// fake runtime (tests/native/fake_cudart.h) and drive its failure paths on a CPU.
#include <cuda_runtime_api.h>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <map>
#include <vector>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>

#include "kvsnap_internal.h"

namespace {

thread_local std::string g_error;

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void cuda(cudaError_t rc) {
    if (rc != cudaSuccess) throw Failure(cudaGetErrorString(rc));
}

// Start offsets are kept at 16-byte multiples: the data-plane kernels move
// 16-byte vectors in and out of pinned allocations.
constexpr size_t kAlign = 16;

struct Slot {
    size_t offset = 0, size = 0;
    cudaEvent_t done = nullptr;   // completion of the last work queued on this slot
    bool queued = false;          // some copy or kernel was queued on it
    bool done_valid = false;      // `done` was recorded after that work
    bool foreign = false;         // that work ran on a stream other than the pool's
};

struct Arena {
    char* base = nullptr;
    size_t capacity = 0;
    int device = 0;
    std::string shared;          // the POSIX shared-memory name of a shared arena, else empty
    bool registered = false;     // the shared mapping is registered with CUDA
    cudaStream_t stream = nullptr;
    std::map<uint64_t, Slot> slots;
    std::map<size_t, size_t> used;   // live ranges, offset -> size, in address order
    uint64_t next_id = 1;
    bool drained = false;
    std::mutex mutex;

    ~Arena() {
        cudaSetDevice(device);
        // Memory the device may still be copying into stays allocated for
        // the life of the process rather than being reused.
        if (!drained && stream && cudaStreamSynchronize(stream) != cudaSuccess) return;
        for (auto& kv : slots)
            if (kv.second.done) cudaEventDestroy(kv.second.done);
        if (stream) cudaStreamDestroy(stream);
        if (shared.empty()) {
            if (base) cudaFreeHost(base);
            return;
        }
        // A shared arena: other processes' mappings stay valid after the name goes.
        if (registered) cudaHostUnregister(base);
        if (base) munmap(base, capacity);
        shm_unlink(shared.c_str());
    }

    Slot& slot(uint64_t id) {
        auto it = slots.find(id);
        if (it == slots.end()) throw Failure("unknown pinned allocation");
        return it->second;
    }

    // Wait until nothing queued on `s` can still touch its bytes. Without a valid
    // event the work's stream must drain; work on a foreign stream drains the device.
    void settle(Slot& s) {
        if (!s.queued) return;
        if (s.done_valid)
            cuda(cudaEventSynchronize(s.done));
        else
            cuda(s.foreign ? cudaDeviceSynchronize() : cudaStreamSynchronize(stream));
    }

    // Make the copy stream wait for everything queued on `producer` so far.
    void after_producer(uintptr_t producer) {
        cudaEvent_t fence = nullptr;
        cuda(cudaEventCreateWithFlags(&fence, cudaEventDisableTiming));
        cudaError_t rc = cudaEventRecord(fence, reinterpret_cast<cudaStream_t>(producer));
        if (rc == cudaSuccess) rc = cudaStreamWaitEvent(stream, fence, 0);
        cudaEventDestroy(fence);
        cuda(rc);
    }

    // Mark the slot busy before enqueueing, so a failed enqueue or record
    // leaves "drain the whole stream" as its only completion authority.
    void begin(Slot& s) {
        s.queued = true;
        s.done_valid = false;
        s.foreign = false;
    }

    void end(Slot& s) {
        cuda(cudaEventRecord(s.done, stream));
        s.done_valid = true;
    }
};

template <typename F>
int guarded(F&& body) {
    try {
        body();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

Arena* live(void* pool) {
    if (!pool) throw Failure("pinned pool is not open");
    return static_cast<Arena*>(pool);
}

}  // namespace

void kvsnap_internal_set_error(const char* message) { g_error = message; }

extern "C" const char* kvsnap_cuda_error() { return g_error.c_str(); }

extern "C" int kvsnap_pool_abi_version() { return 2; }

extern "C" void* kvsnap_pool_create(size_t capacity, int device) {
    try {
        if (capacity == 0) throw Failure("pool capacity must be positive");
        auto arena = std::make_unique<Arena>();
        arena->capacity = capacity;
        arena->device = device;
        cuda(cudaSetDevice(device));
        void* base = nullptr;
        // Portable: usable from every device's context; mapped: kernels read
        // and write it in place through its (unified) host address.
        cuda(cudaHostAlloc(&base, capacity, cudaHostAllocPortable | cudaHostAllocMapped));
        arena->base = static_cast<char*>(base);
        cuda(cudaStreamCreateWithFlags(&arena->stream, cudaStreamNonBlocking));
        return arena.release();
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

namespace {

void check_shared_name(const char* name) {
    if (!name || name[0] != '/' || std::strlen(name) < 2 || std::strlen(name) > 200 || std::strchr(name + 1, '/'))
        throw Failure("a shared arena name is one path component that starts with '/'");
}

std::string os_error(const char* what) { return std::string(what) + ": " + std::strerror(errno); }

}  // namespace

extern "C" void* kvsnap_pool_create_shared(size_t capacity, int device, const char* name) {
    try {
        if (capacity == 0) throw Failure("pool capacity must be positive");
        check_shared_name(name);
        auto arena = std::make_unique<Arena>();
        arena->capacity = capacity;
        arena->device = device;
        cuda(cudaSetDevice(device));
        const int fd = shm_open(name, O_CREAT | O_EXCL | O_RDWR, 0600);
        if (fd < 0) throw Failure(os_error("shm_open"));
        arena->shared = name;     // from here the destructor unlinks the name
        const bool sized = ftruncate(fd, static_cast<off_t>(capacity)) == 0;
        void* base = sized ? mmap(nullptr, capacity, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0) : MAP_FAILED;
        const std::string failed = sized ? os_error("mmap") : os_error("ftruncate");
        close(fd);
        if (base == MAP_FAILED) throw Failure(failed);
        arena->base = static_cast<char*>(base);
        // Portable: every device's context; mapped: kernels use it in place at its host address.
        cuda(cudaHostRegister(base, capacity, cudaHostRegisterPortable | cudaHostRegisterMapped));
        arena->registered = true;
        cuda(cudaStreamCreateWithFlags(&arena->stream, cudaStreamNonBlocking));
        return arena.release();
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

namespace {

// Map the named segment and register it with CUDA: read-only where the platform
// registers read-only host memory, else read-write (this process still only reads it).
void* map_shared(const char* name, bool read_only, size_t* bytes, cudaError_t* registered) {
    const int fd = shm_open(name, read_only ? O_RDONLY : O_RDWR, 0);
    if (fd < 0) throw Failure(os_error("shm_open"));
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        const std::string failed = os_error("fstat");
        close(fd);
        throw Failure(failed);
    }
    *bytes = static_cast<size_t>(st.st_size);
    void* mapped = mmap(nullptr, *bytes, read_only ? PROT_READ : PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    const std::string failed = os_error("mmap");
    close(fd);
    if (mapped == MAP_FAILED) throw Failure(failed);
    const unsigned flags = cudaHostRegisterPortable | cudaHostRegisterMapped | (read_only ? cudaHostRegisterReadOnly : 0u);
    *registered = cudaHostRegister(mapped, *bytes, flags);
    if (*registered != cudaSuccess) munmap(mapped, *bytes);
    return mapped;
}

}  // namespace

extern "C" int kvsnap_shared_open(const char* name, int device, void** base, size_t* size) {
    return guarded([&] {
        check_shared_name(name);
        if (!base || !size) throw Failure("opening a shared arena needs outputs");
        cuda(cudaSetDevice(device));
        size_t bytes = 0;
        cudaError_t rc = cudaSuccess;
        void* mapped = map_shared(name, true, &bytes, &rc);
        if (rc != cudaSuccess) {
            cudaGetLastError();                      // the read-only attempt's error is not this call's result
            mapped = map_shared(name, false, &bytes, &rc);
            cuda(rc);
        }
        *base = mapped;
        *size = bytes;
    });
}

extern "C" int kvsnap_shared_close(void* base, size_t size) {
    return guarded([&] {
        if (!base || !size) throw Failure("closing a shared arena needs its mapping");
        cuda(cudaHostUnregister(base));
        if (munmap(base, size) != 0) throw Failure(os_error("munmap"));
    });
}

extern "C" void kvsnap_pool_destroy(void* pool) { delete static_cast<Arena*>(pool); }

extern "C" int kvsnap_pool_close_checked(void* pool) {
    return guarded([&] {
        if (!pool) return;
        Arena* a = static_cast<Arena*>(pool);
        cuda(cudaSetDevice(a->device));
        cuda(cudaStreamSynchronize(a->stream));
        a->drained = true;
        delete a;
    });
}

extern "C" int kvsnap_pool_arena(void* pool, void** base, size_t* capacity) {
    return guarded([&] {
        if (!pool || !base || !capacity) throw Failure("arena query requires a live pool and outputs");
        Arena* a = static_cast<Arena*>(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        *base = a->base;
        *capacity = a->capacity;
    });
}

extern "C" int kvsnap_pool_copy_stream(void* pool, uintptr_t* stream) {
    return guarded([&] {
        if (!pool || !stream) throw Failure("copy stream requires a live pool and an output");
        Arena* a = static_cast<Arena*>(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        cuda(cudaSetDevice(a->device));
        *stream = reinterpret_cast<uintptr_t>(a->stream);
    });
}

extern "C" int kvsnap_pool_reserve(void* pool, size_t size, uint64_t* id, void** ptr) {
    return guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        if (size == 0 || size > a->capacity) throw Failure("pinned capacity exhausted");
        // First fit over the live ranges in address order (ids are not ordered by address).
        size_t at = 0;
        for (const auto& range : a->used) {
            if (range.first >= at && range.first - at >= size) break;
            size_t end = range.first + range.second;
            at = (end + kAlign - 1) / kAlign * kAlign;
        }
        if (at > a->capacity || size > a->capacity - at) throw Failure("pinned capacity exhausted");
        cuda(cudaSetDevice(a->device));
        Slot s;
        s.offset = at;
        s.size = size;
        cuda(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
        *id = a->next_id++;
        *ptr = a->base + at;
        a->slots.emplace(*id, s);
        a->used.emplace(at, size);
    });
}

extern "C" int kvsnap_pool_copy(void* pool, uint64_t id, size_t host_offset, void* device_ptr, size_t size,
                                int to_host, uintptr_t producer_stream) {
    return guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        Slot& s = a->slot(id);
        if (host_offset > s.size || size > s.size - host_offset)
            throw Failure("copy outside pinned allocation");
        cuda(cudaSetDevice(a->device));
        if (to_host) a->after_producer(producer_stream);
        char* host = a->base + s.offset + host_offset;
        a->begin(s);
        if (to_host)
            cuda(cudaMemcpyAsync(host, device_ptr, size, cudaMemcpyDeviceToHost, a->stream));
        else
            cuda(cudaMemcpyAsync(device_ptr, host, size, cudaMemcpyHostToDevice, a->stream));
        a->end(s);
    });
}

extern "C" int kvsnap_pool_copy_2d(void* pool, uint64_t id, size_t host_offset, size_t host_pitch,
                                   void* device_ptr, size_t device_pitch, size_t width, size_t height,
                                   int to_host, uintptr_t producer_stream) {
    return guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        Slot& s = a->slot(id);
        if (width == 0 || height == 0 || host_pitch < width || device_pitch < width)
            throw Failure("invalid 2D copy geometry");
        // Last row ends at host_offset + (height - 1) * host_pitch + width.
        if (host_pitch > 0 && height - 1 > (SIZE_MAX - width) / host_pitch)
            throw Failure("2D copy outside pinned allocation");
        const size_t extent = (height - 1) * host_pitch + width;
        if (host_offset > s.size || extent > s.size - host_offset)
            throw Failure("2D copy outside pinned allocation");
        cuda(cudaSetDevice(a->device));
        if (to_host) a->after_producer(producer_stream);
        char* host = a->base + s.offset + host_offset;
        a->begin(s);
        if (to_host)
            cuda(cudaMemcpy2DAsync(host, host_pitch, device_ptr, device_pitch, width, height,
                                   cudaMemcpyDeviceToHost, a->stream));
        else
            cuda(cudaMemcpy2DAsync(device_ptr, device_pitch, host, host_pitch, width, height,
                                   cudaMemcpyHostToDevice, a->stream));
        a->end(s);
    });
}

extern "C" int kvsnap_pool_copy_on(void* pool, uint64_t id, size_t host_offset, void* device_ptr, size_t size,
                                   int to_host, uintptr_t stream) {
    return guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        Slot& s = a->slot(id);
        if (host_offset > s.size || size > s.size - host_offset)
            throw Failure("copy outside pinned allocation");
        cuda(cudaSetDevice(a->device));
        cudaStream_t on = stream ? reinterpret_cast<cudaStream_t>(stream) : a->stream;
        char* host = a->base + s.offset + host_offset;
        a->begin(s);
        s.foreign = on != a->stream;
        if (to_host)
            cuda(cudaMemcpyAsync(host, device_ptr, size, cudaMemcpyDeviceToHost, on));
        else
            cuda(cudaMemcpyAsync(device_ptr, host, size, cudaMemcpyHostToDevice, on));
        cuda(cudaEventRecord(s.done, on));
        s.done_valid = true;
    });
}

extern "C" int kvsnap_pool_mark(void* pool, uint64_t id, uintptr_t stream) {
    return guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        Slot& s = a->slot(id);
        cuda(cudaSetDevice(a->device));
        cudaStream_t on = stream ? reinterpret_cast<cudaStream_t>(stream) : a->stream;
        a->begin(s);
        s.foreign = on != a->stream;
        cuda(cudaEventRecord(s.done, on));
        s.done_valid = true;
    });
}

extern "C" int kvsnap_pool_copy_many(void* pool, int64_t n, const uint64_t* ids, const uint64_t* host_offsets,
                                     const uint64_t* device_ptrs, const uint64_t* sizes, int to_host,
                                     uintptr_t stream) {
    return guarded([&] {
        if (n < 0 || (n > 0 && (!ids || !host_offsets || !device_ptrs || !sizes)))
            throw Failure("invalid copy list");
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        // Every entry is checked before anything is queued.
        std::vector<Slot*> slots(static_cast<size_t>(n));
        for (int64_t k = 0; k < n; ++k) {
            Slot& s = a->slot(ids[k]);
            if (host_offsets[k] > s.size || sizes[k] > s.size - host_offsets[k])
                throw Failure("copy outside pinned allocation");
            slots[static_cast<size_t>(k)] = &s;
        }
        if (n == 0) return;
        cuda(cudaSetDevice(a->device));
        cudaStream_t on = stream ? reinterpret_cast<cudaStream_t>(stream) : a->stream;
        for (Slot* s : slots) {
            a->begin(*s);
            s->foreign = on != a->stream;
        }
        // Entries whose host and device ranges both continue the previous one's
        // (blocks reserved one after another land next to each other in the
        // arena) move in one copy: fewer DMA descriptors for the same bytes.
        for (int64_t k = 0; k < n;) {
            char* host = a->base + slots[static_cast<size_t>(k)]->offset + host_offsets[k];
            const uint64_t device = device_ptrs[k];
            uint64_t bytes = sizes[k];
            int64_t j = k + 1;
            for (; j < n; ++j) {
                const char* next = a->base + slots[static_cast<size_t>(j)]->offset + host_offsets[j];
                if (next != host + bytes || device_ptrs[j] != device + bytes) break;
                bytes += sizes[j];
            }
            void* dev = reinterpret_cast<void*>(static_cast<uintptr_t>(device));
            if (to_host)
                cuda(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, on));
            else
                cuda(cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, on));
            k = j;
        }
        for (Slot* s : slots) {
            if (s->done_valid) continue;      // listed twice: recorded already, after every copy
            cuda(cudaEventRecord(s->done, on));
            s->done_valid = true;
        }
    });
}

extern "C" int kvsnap_pool_wait_many(void* pool, int64_t n, const uint64_t* ids) {
    return guarded([&] {
        if (n < 0 || (n > 0 && !ids)) throw Failure("invalid allocation list");
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        for (int64_t k = 0; k < n; ++k) a->slot(ids[k]);
        if (n == 0) return;
        cuda(cudaSetDevice(a->device));
        for (int64_t k = 0; k < n; ++k) a->settle(a->slot(ids[k]));
    });
}

extern "C" int kvsnap_pool_wait(void* pool, uint64_t id) {
    return guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        Slot& s = a->slot(id);
        cuda(cudaSetDevice(a->device));
        a->settle(s);
    });
}

extern "C" int kvsnap_pool_ready(void* pool, uint64_t id) {
    int idle = 0;
    int rc = guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        Slot& s = a->slot(id);
        cuda(cudaSetDevice(a->device));
        if (!s.queued) {
            idle = 1;
            return;
        }
        cudaError_t q = s.done_valid ? cudaEventQuery(s.done) : cudaStreamQuery(a->stream);
        if (q == cudaSuccess)
            idle = 1;
        else if (q != cudaErrorNotReady)
            cuda(q);
    });
    return rc < 0 ? -1 : idle;
}

extern "C" int kvsnap_pool_release(void* pool, uint64_t id) {
    return guarded([&] {
        Arena* a = live(pool);
        std::lock_guard<std::mutex> lock(a->mutex);
        Slot& s = a->slot(id);
        cuda(cudaSetDevice(a->device));
        a->settle(s);   // blocking: the bytes are idle before they go back to the arena
        cuda(cudaEventDestroy(s.done));
        a->used.erase(s.offset);
        a->slots.erase(id);
    });
}
