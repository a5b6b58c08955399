// Host CRC32C and file I/O: _io_native.so.
//
// The reference's csrc/dataplane/io.cpp ABI version 1 (bound by
// kvsnap/store/native_io.py:59-65), rebuilt:
//   * CRC32C over three interleaved SSE4.2 streams, joined with GF(2)
//     shift-multiplications, so the crc32 instruction's latency is hidden;
//     a byte table where SSE4.2 is absent. Same values as the reference
//     (io.cpp:16-47), pinned by tests/test_io_native.py;
//   * pread / pwrite loops with EINTR, short-transfer and EOF handling;
//   * a transfer pool that runs at most `workers` transfers and a byte budget
//     at once, each on its caller's thread.
#include <cerrno>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>

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

// Every byte of [offset, offset + size) moved by positional reads or writes,
// resuming after signals and short transfers. A read that meets end of file, or
// a write that makes no progress, is EIO; other failures return their errno.
// A negative offset, or a range past INT64_MAX, is EINVAL before any call.
template <bool kWrite>
int move_all(int fd, char* bytes, size_t size, int64_t offset) {
    if (offset < 0 || size > static_cast<uint64_t>(INT64_MAX - offset)) return EINVAL;
    size_t moved = 0;
    while (moved < size) {
        const off_t at = static_cast<off_t>(offset + static_cast<int64_t>(moved));
        const ssize_t n = kWrite ? pwrite(fd, bytes + moved, size - moved, at) : pread(fd, bytes + moved, size - moved, at);
        if (n > 0) {
            moved += static_cast<size_t>(n);
        } else if (n == 0) {
            return EIO;
        } else if (errno != EINTR) {
            return errno;
        }
    }
    return 0;
}

int sync_data(int fd) {
    for (;;) {
        if (fdatasync(fd) == 0) return 0;
        if (errno != EINTR) return errno;
    }
}

}  // namespace

extern "C" int kvsnap_pwrite_all(int fd, const void* data, size_t size, int64_t offset, int durable) {
    const int rc = move_all<true>(fd, const_cast<char*>(static_cast<const char*>(data)), size, offset);
    return rc || !durable ? rc : sync_data(fd);
}

extern "C" int kvsnap_pread_all(int fd, void* data, size_t size, int64_t offset) {
    return move_all<false>(fd, static_cast<char*>(data), size, offset);
}

namespace {

// The transfer pool. Its C ABI is synchronous: a caller hands over one read or
// write and waits for its result. So no work is handed to other threads: each
// caller runs its own transfer once the gate admits it, and the gate bounds
// what the pool allows at once: `slots` transfers and `budget` bytes in
// flight. Destroying the gate turns away every waiter (ECANCELED) and waits
// for the transfers already admitted.
class Gate {
  public:
    Gate(size_t slots, size_t budget) : free_slots_(slots), budget_(budget), room_(budget) {}

    ~Gate() {
        std::unique_lock<std::mutex> hold(mu_);
        closing_ = true;
        changed_.notify_all();
        changed_.wait(hold, [&] { return running_ == 0 && waiting_ == 0; });
    }

    size_t budget() const { return budget_; }

    int run(int fd, char* bytes, size_t size, int64_t offset, bool write, bool durable) {
        {
            std::unique_lock<std::mutex> hold(mu_);
            ++waiting_;
            changed_.wait(hold, [&] { return closing_ || (free_slots_ > 0 && size <= room_); });
            --waiting_;
            if (closing_) {
                changed_.notify_all();
                return ECANCELED;
            }
            --free_slots_;
            room_ -= size;
            ++running_;
        }
        const int rc = write ? kvsnap_pwrite_all(fd, bytes, size, offset, durable)
                             : kvsnap_pread_all(fd, bytes, size, offset);
        {
            std::lock_guard<std::mutex> hold(mu_);
            ++free_slots_;
            room_ += size;
            --running_;
        }
        changed_.notify_all();
        return rc;
    }

  private:
    std::mutex mu_;
    std::condition_variable changed_;
    size_t free_slots_;
    const size_t budget_;
    size_t room_;
    size_t running_ = 0, waiting_ = 0;
    bool closing_ = false;
};

}  // namespace

extern "C" void* kvsnap_io_pool_create(size_t workers, size_t max_bytes) {
    if (workers < 1 || workers > 64 || max_bytes == 0) return nullptr;
    return new (std::nothrow) Gate(workers, max_bytes);
}

extern "C" void kvsnap_io_pool_destroy(void* pool) { delete static_cast<Gate*>(pool); }

extern "C" int kvsnap_io_pool_transfer(void* pool, int fd, void* data, size_t size, int64_t offset, int write,
                                       int durable) {
    if (!pool || (!data && size) || (write != 0 && write != 1)) return EINVAL;
    Gate* gate = static_cast<Gate*>(pool);
    if (size > gate->budget()) return EMSGSIZE;
    return gate->run(fd, static_cast<char*>(data), size, offset, write == 1, durable != 0);
}
