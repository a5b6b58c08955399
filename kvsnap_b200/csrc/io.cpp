// Host CRC32C and file I/O: _io_native.so.
//
// The reference's csrc/dataplane/io.cpp ABI version 1 (bound by
// kvsnap/store/native_io.py:59-65), rebuilt:
//   * CRC32C over three interleaved SSE4.2 streams, joined with GF(2)
//     shift-multiplications, so the crc32 instruction's latency is hidden;
//     a byte table where SSE4.2 is absent. Same values as the reference
//     (io.cpp:16-47), pinned by tests/test_io_native.py;
//   * pread / pwrite loops with EINTR, short-transfer and EOF handling;
//   * a bounded worker pool that admits at most a byte budget in flight.
#include <cerrno>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <future>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include <unistd.h>

#if defined(__x86_64__)
#include <nmmintrin.h>
#endif

#include "kvsnap_io.h"

namespace {

constexpr uint32_t kPoly = 0x82F63B78u;

struct ByteTable {
    uint32_t t[256];
    ByteTable() {
        for (uint32_t v = 0; v < 256; ++v) {
            uint32_t r = v;
            for (int k = 0; k < 8; ++k) r = (r >> 1) ^ (kPoly & (0u - (r & 1u)));
            t[v] = r;
        }
    }
};
const ByteTable kTable;

// Reflected GF(2) product mod P (bit 31 = x^0).
uint32_t mulmod(uint32_t a, uint32_t b) {
    uint32_t p = 0;
    for (int k = 31; k >= 0; --k) {
        p ^= b & (0u - ((a >> k) & 1u));
        b = (b >> 1) ^ (kPoly & (0u - (b & 1u)));
    }
    return p;
}

// x^(8n) mod P: appending n zero bytes to a raw CRC register multiplies it by this.
uint32_t xpow8n(uint64_t n) {
    uint32_t result = 1u << 31, square = 1u << 23;
    for (; n; n >>= 1) {
        if (n & 1u) result = mulmod(result, square);
        square = mulmod(square, square);
    }
    return result;
}

uint32_t raw_bytes(uint32_t reg, const uint8_t* p, size_t n) {
    while (n--) reg = kTable.t[(reg ^ *p++) & 0xFFu] ^ (reg >> 8);
    return reg;
}

#if defined(__x86_64__)
constexpr size_t kLane = 8192;   // bytes per interleaved stream per round
const uint32_t kShift1 = xpow8n(kLane);
const uint32_t kShift2 = xpow8n(2 * kLane);

__attribute__((target("sse4.2"))) uint32_t raw_sse42(uint32_t reg, const uint8_t* p, size_t n) {
    while (n >= 3 * kLane) {
        uint64_t a = reg, b = 0, c = 0;
        for (size_t i = 0; i < kLane; i += 8) {
            uint64_t wa, wb, wc;
            std::memcpy(&wa, p + i, 8);
            std::memcpy(&wb, p + kLane + i, 8);
            std::memcpy(&wc, p + 2 * kLane + i, 8);
            a = _mm_crc32_u64(a, wa);
            b = _mm_crc32_u64(b, wb);
            c = _mm_crc32_u64(c, wc);
        }
        // raw(reg, A||B||C) = A' * x^(8*2L) + B' * x^(8*L) + C'.
        reg = mulmod(static_cast<uint32_t>(a), kShift2) ^ mulmod(static_cast<uint32_t>(b), kShift1) ^
              static_cast<uint32_t>(c);
        p += 3 * kLane;
        n -= 3 * kLane;
    }
    uint64_t r = reg;
    for (; n >= 8; n -= 8, p += 8) {
        uint64_t w;
        std::memcpy(&w, p, 8);
        r = _mm_crc32_u64(r, w);
    }
    uint32_t r32 = static_cast<uint32_t>(r);
    while (n--) r32 = _mm_crc32_u8(r32, *p++);
    return r32;
}
#endif

}  // namespace

extern "C" int kvsnap_io_abi_version() { return 1; }

extern "C" uint32_t kvsnap_crc32c_extend(const void* data, size_t size, uint32_t prior) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
#if defined(__x86_64__)
    if (__builtin_cpu_supports("sse4.2")) return ~raw_sse42(~prior, p, size);
#endif
    return ~raw_bytes(~prior, p, size);
}

extern "C" uint32_t kvsnap_crc32c(const void* data, size_t size) { return kvsnap_crc32c_extend(data, size, 0); }

namespace {
bool bad_range(size_t size, int64_t offset) {
    return offset < 0 || size > static_cast<uint64_t>(INT64_MAX - offset);
}
}  // namespace

extern "C" int kvsnap_pwrite_all(int fd, const void* data, size_t size, int64_t offset, int durable) {
    if (bad_range(size, offset)) return EINVAL;
    const char* p = static_cast<const char*>(data);
    for (size_t done = 0; done < size;) {
        ssize_t n = pwrite(fd, p + done, size - done, offset + static_cast<int64_t>(done));
        if (n < 0) {
            if (errno == EINTR) continue;
            return errno;
        }
        if (n == 0) return EIO;
        done += static_cast<size_t>(n);
    }
    if (durable) {
        int rc;
        do rc = fdatasync(fd);
        while (rc < 0 && errno == EINTR);
        if (rc < 0) return errno;
    }
    return 0;
}

extern "C" int kvsnap_pread_all(int fd, void* data, size_t size, int64_t offset) {
    if (bad_range(size, offset)) return EINVAL;
    char* p = static_cast<char*>(data);
    for (size_t done = 0; done < size;) {
        ssize_t n = pread(fd, p + done, size - done, offset + static_cast<int64_t>(done));
        if (n < 0) {
            if (errno == EINTR) continue;
            return errno;
        }
        if (n == 0) return EIO;   // end of file before `size` bytes
        done += static_cast<size_t>(n);
    }
    return 0;
}

namespace {

struct Request {
    int fd = -1, write = 0, durable = 0;
    void* data = nullptr;
    size_t size = 0;
    int64_t offset = 0;
    std::promise<int> result;
};

class Workers {
  public:
    Workers(size_t count, size_t budget) : budget_(budget) {
        try {
            for (size_t i = 0; i < count; ++i) threads_.emplace_back([this] { serve(); });
        } catch (...) {
            stop();
            throw;
        }
    }
    ~Workers() { stop(); }

    int submit(int fd, void* data, size_t size, int64_t offset, int write, int durable) {
        auto request = std::make_shared<Request>();
        request->fd = fd;
        request->data = data;
        request->size = size;
        request->offset = offset;
        request->write = write;
        request->durable = durable;
        std::future<int> done = request->result.get_future();
        {
            std::unique_lock<std::mutex> lock(mutex_);
            room_.wait(lock, [&] { return stopping_ || size <= budget_ - in_flight_; });
            if (stopping_) return ECANCELED;
            in_flight_ += size;
            queue_.push_back(std::move(request));
        }
        ready_.notify_one();
        return done.get();
    }

    size_t budget() const { return budget_; }

  private:
    void serve() {
        for (;;) {
            std::shared_ptr<Request> request;
            {
                std::unique_lock<std::mutex> lock(mutex_);
                ready_.wait(lock, [&] { return stopping_ || !queue_.empty(); });
                if (queue_.empty()) return;   // stopping and drained
                request = std::move(queue_.front());
                queue_.pop_front();
            }
            int rc = request->write
                         ? kvsnap_pwrite_all(request->fd, request->data, request->size, request->offset,
                                             request->durable)
                         : kvsnap_pread_all(request->fd, request->data, request->size, request->offset);
            {
                std::lock_guard<std::mutex> lock(mutex_);
                in_flight_ -= request->size;
            }
            room_.notify_all();
            request->result.set_value(rc);
        }
    }

    void stop() {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            stopping_ = true;
        }
        ready_.notify_all();
        room_.notify_all();
        for (auto& t : threads_)
            if (t.joinable()) t.join();
    }

    const size_t budget_;
    size_t in_flight_ = 0;
    bool stopping_ = false;
    std::mutex mutex_;
    std::condition_variable ready_, room_;
    std::deque<std::shared_ptr<Request>> queue_;
    std::vector<std::thread> threads_;
};

}  // namespace

extern "C" void* kvsnap_io_pool_create(size_t workers, size_t max_bytes) {
    if (workers == 0 || workers > 64 || max_bytes == 0) return nullptr;
    try {
        return new Workers(workers, max_bytes);
    } catch (...) {
        return nullptr;
    }
}

extern "C" void kvsnap_io_pool_destroy(void* pool) { delete static_cast<Workers*>(pool); }

extern "C" int kvsnap_io_pool_transfer(void* pool, int fd, void* data, size_t size, int64_t offset, int write,
                                       int durable) {
    if (!pool || (!data && size) || (write != 0 && write != 1)) return EINVAL;
    Workers* w = static_cast<Workers*>(pool);
    if (size > w->budget()) return EMSGSIZE;
    try {
        return w->submit(fd, data, size, offset, write, durable);
    } catch (...) {
        return ENOMEM;
    }
}
