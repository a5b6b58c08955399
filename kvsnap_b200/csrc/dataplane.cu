// sm_100a data-plane kernels of _cuda_native.so: save gather, restore scatter,
// CRC32C and SHA-256 of packed snapshot blocks.
//
// Reference behaviour reproduced (paths in the kvsnap source tree):
//   * packed block = the registered layer spans back to back in layer-name
//     order, each span a dense block copied in storage order
//     (kvsnap/connector/dataplane.py:221-249, 283-305);
//   * save: gather a request's blocks into packed blocks and zero the token
//     slots past the last computed token of the last block
//     (dataplane.py:262-272, 388-437);
//   * restore: copy each packed (block, layer) span into its cache row
//     (kvsnap/connector/copy_kernel.py:23-49);
//   * checksums: CRC32C, reflected Castagnoli 0x82F63B78 with inverted
//     register and output (csrc/dataplane/io.cpp:16-47), and the content id
//     SHA-256 (FIPS 180-4) of each packed block (kvsnap/store/store.py:623).
//
// CRC32C on a GPU. A CRC is linear over GF(2): for a raw register (no
// inversions) raw(0, A||B) = raw(0, A) * x^(8|B|) + raw(0, B) mod P. So each
// warp CRCs its own (block, span) unit, the 32 lanes each keep a partial
// register over the 16-byte vectors they load (coalesced: lane j takes bytes
// 16j..16j+15 of every 512-byte step), the partials are moved into place by
// multiplying with x^(8k) mod P and XOR-reduced over the warp, the span's
// result is moved to its place in the packed block the same way, and units of
// one block meet in one word through atomicXor. Bytes are folded in with
// slicing-by-16 tables in shared memory (T_k[v] = raw CRC of byte v followed
// by k zero bytes), built at compile time.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "kvsnap_cuda.h"
#include "kvsnap_internal.h"

namespace {

constexpr uint32_t kPoly = 0x82F63B78u;

// ---- GF(2) arithmetic, reflected (bit 31 = coefficient of x^0) --------------

__host__ __device__ constexpr uint32_t gf_mulmod(uint32_t a, uint32_t b) {
    uint32_t p = 0;
    for (int k = 31; k >= 0; --k) {
        p ^= b & (0u - ((a >> k) & 1u));
        b = (b >> 1) ^ (kPoly & (0u - (b & 1u)));
    }
    return p;
}

// x^(-8n) mod P: n bytes of division by x (x is a unit: P has a constant term).
// In the reflected form bit 31 of a product by x is set exactly when P was
// added, which makes each step invertible.
__host__ __device__ constexpr uint32_t gf_xpow_neg8n(int n) {
    uint32_t r = 1u << 31;
    for (int k = 0; k < 8 * n; ++k) r = (r >> 31) ? ((r ^ kPoly) << 1) | 1u : r << 1;
    return r;
}

__host__ __device__ constexpr uint32_t gf_xpow8n(uint64_t n) {
    uint32_t result = 1u << 31, square = 1u << 23;   // x^0, x^8
    for (; n; n >>= 1) {
        if (n & 1u) result = gf_mulmod(result, square);
        square = gf_mulmod(square, square);
    }
    return result;
}

// Tables: slots 0..15 hold T_0..T_15, slots 16..19 T_492..T_495 (moving a lane's
// register 496 bytes ahead), slots 20..23 T_244..T_247 (the same for 8-byte
// vectors).
// Slots 24..27 hold T_124..T_127 (a word, then the 124 bytes to the same word of
// the next 128-byte line: the segment kernels' chains).
struct CrcTables {
    uint32_t t[28][256];
};

constexpr CrcTables make_tables() {
    CrcTables r{};
    for (uint32_t v = 0; v < 256; ++v) {
        uint32_t x = v;
        for (int k = 0; k < 8; ++k) x = (x >> 1) ^ (kPoly & (0u - (x & 1u)));
        r.t[0][v] = x;
    }
    for (int k = 1; k < 16; ++k)
        for (int v = 0; v < 256; ++v) r.t[k][v] = (r.t[k - 1][v] >> 8) ^ r.t[0][r.t[k - 1][v] & 0xFFu];
    for (int j = 0; j < 4; ++j) {
        const uint32_t far16 = gf_xpow8n(492 + j), far8 = gf_xpow8n(244 + j);
        for (int v = 0; v < 256; ++v) {
            r.t[16 + j][v] = gf_mulmod(r.t[0][v], far16);
            r.t[20 + j][v] = gf_mulmod(r.t[0][v], far8);
        }
    }
    const uint32_t line = gf_xpow8n(124);
    for (int j = 0; j < 4; ++j) {
        for (int v = 0; v < 256; ++v) r.t[24 + j][v] = gf_mulmod(r.t[j][v], line);
    }
    return r;
}

// x^(8 * v * 256^k) mod P for every byte value v of byte k of a 64-bit n, so that
// x^(8n) takes one GF(2) multiply a nonzero byte of n after the first (the
// kernel prologues' placement factors: one or two multiplies, not one a set bit).
struct Pow8 {
    uint32_t p[8][256];
};

constexpr Pow8 make_pow8() {
    Pow8 r{};
    uint32_t step = 1u << 23;                     // x^8
    for (int k = 0; k < 8; ++k) {
        uint32_t acc = 1u << 31;                  // x^0
        for (int v = 0; v < 256; ++v) {
            r.p[k][v] = acc;
            acc = gf_mulmod(acc, step);
        }
        step = acc;                               // x^(8 * 256^(k + 1))
    }
    return r;
}

__device__ const CrcTables g_tables = make_tables();
__device__ const Pow8 g_pow8 = make_pow8();

__device__ __forceinline__ uint32_t dev_xpow8n(uint64_t n) {
    uint32_t r = g_pow8.p[0][n & 255u];
    for (int k = 1; (n >>= 8) != 0; ++k)
        if (n & 255u) r = gf_mulmod(r, g_pow8.p[k][n & 255u]);
    return r;
}

// ---- vectors ------------------------------------------------------------------

template <int VEC>
struct Vec;
template <>
struct Vec<16> {
    using T = uint4;
    static constexpr int kTables = 20;
    __device__ static T zero() { return make_uint4(0, 0, 0, 0); }
    __device__ static T load(const char* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }
    __device__ static void store(char* p, T v) { *reinterpret_cast<uint4*>(p) = v; }
    __device__ static uint32_t word(const T& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
    __device__ static void set_word(T& v, int i, uint32_t w) {
        if (i == 0) v.x = w; else if (i == 1) v.y = w; else if (i == 2) v.z = w; else v.w = w;
    }
};
template <>
struct Vec<8> {
    using T = uint2;
    static constexpr int kTables = 12;
    __device__ static T zero() { return make_uint2(0, 0); }
    __device__ static T load(const char* p) { return __ldcs(reinterpret_cast<const uint2*>(p)); }
    __device__ static void store(char* p, T v) { *reinterpret_cast<uint2*>(p) = v; }
    __device__ static uint32_t word(const T& v, int i) { return i == 0 ? v.x : v.y; }
    __device__ static void set_word(T& v, int i, uint32_t w) {
        if (i == 0) v.x = w; else v.y = w;
    }
};

// Shared-memory copy of the tables one vector width needs: T_0..T_{VEC-1}, then
// the four "far" tables for moving a register 32*VEC - VEC bytes ahead.
template <int VEC>
__device__ __forceinline__ void load_tables(uint32_t* tb) {
    const uint32_t* g = &g_tables.t[0][0];
    for (int i = threadIdx.x; i < Vec<VEC>::kTables * 256; i += blockDim.x) {
        const int slot = i >> 8, v = i & 255;
        const int src = slot < VEC ? slot : (VEC == 16 ? 16 : 20) + (slot - VEC);
        tb[i] = g[src * 256 + v];
    }
}

#define KV_T(slot, byte) tb[(slot) * 256 + (byte)]

// One Horner step of a lane's register: r <- r * x^(8*32*VEC) + raw(0, v).
__device__ __forceinline__ uint32_t crc_step(const uint32_t* tb, uint32_t r, uint4 v) {
    const uint32_t far = KV_T(19, r & 255) ^ KV_T(18, (r >> 8) & 255) ^ KV_T(17, (r >> 16) & 255) ^ KV_T(16, r >> 24);
    const uint32_t w = v.x ^ far;
    return KV_T(15, w & 255) ^ KV_T(14, (w >> 8) & 255) ^ KV_T(13, (w >> 16) & 255) ^ KV_T(12, w >> 24) ^
           KV_T(11, v.y & 255) ^ KV_T(10, (v.y >> 8) & 255) ^ KV_T(9, (v.y >> 16) & 255) ^ KV_T(8, v.y >> 24) ^
           KV_T(7, v.z & 255) ^ KV_T(6, (v.z >> 8) & 255) ^ KV_T(5, (v.z >> 16) & 255) ^ KV_T(4, v.z >> 24) ^
           KV_T(3, v.w & 255) ^ KV_T(2, (v.w >> 8) & 255) ^ KV_T(1, (v.w >> 16) & 255) ^ KV_T(0, v.w >> 24);
}

__device__ __forceinline__ uint32_t crc_step(const uint32_t* tb, uint32_t r, uint2 v) {
    const uint32_t far = KV_T(11, r & 255) ^ KV_T(10, (r >> 8) & 255) ^ KV_T(9, (r >> 16) & 255) ^ KV_T(8, r >> 24);
    const uint32_t w = v.x ^ far;
    return KV_T(7, w & 255) ^ KV_T(6, (w >> 8) & 255) ^ KV_T(5, (w >> 16) & 255) ^ KV_T(4, w >> 24) ^
           KV_T(3, v.y & 255) ^ KV_T(2, (v.y >> 8) & 255) ^ KV_T(1, (v.y >> 16) & 255) ^ KV_T(0, v.y >> 24);
}

#undef KV_T

__device__ __forceinline__ uint32_t warp_xor(uint32_t v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) v ^= __shfl_xor_sync(0xFFFFFFFFu, v, d);
    return v;
}

__device__ __forceinline__ void flag(uint32_t* status, uint32_t bits) {
    if (status) atomicOr(status, bits);
}

// Zero the bytes of a vector at span offset `at` whose token slot is >= valid.
template <int VEC>
__device__ typename Vec<VEC>::T mask_tail(typename Vec<VEC>::T v, int64_t at, const kvsnap_span& sp, int valid) {
    if (sp.row_bytes % VEC == 0) {   // the vector lies inside one (head, token) row
        const int64_t token = (at / sp.token_pitch) % sp.tokens;
        return token >= valid ? Vec<VEC>::zero() : v;
    }
    for (int w = 0; w < VEC / 4; ++w) {
        uint32_t word = Vec<VEC>::word(v, w);
        for (int b = 0; b < 4; ++b) {
            const int64_t token = ((at + 4 * w + b) / sp.token_pitch) % sp.tokens;
            if (token >= valid) word &= ~(0xFFu << (8 * b));
        }
        Vec<VEC>::set_word(v, w, word);
    }
    return v;
}

// One warp moves (STORE) and/or checksums `len` bytes from src to dst. The
// span is front-padded with zeros to a whole number of 32*VEC-byte steps, which
// leaves a zero-initialised raw CRC unchanged. Returns the lane's register:
// its vectors' raw CRC as if the unit ended at the lane's last vector + 32*VEC
// - (lane+1)*VEC; the caller multiplies by x^(8*VEC*(31-lane)).
template <int VEC, bool STORE, bool CRC>
__device__ __forceinline__ uint32_t warp_unit(const uint32_t* tb, const char* __restrict__ src,
                                              char* __restrict__ dst, int64_t len, int lane, bool tail,
                                              const kvsnap_span& sp, int valid) {
    using V = typename Vec<VEC>::T;
    constexpr int kStep = 32 * VEC;
    constexpr int kUnroll = 4;
    const int64_t steps = (len + kStep - 1) / kStep;
    const int64_t first = (int64_t)lane * VEC - (steps * kStep - len);
    uint32_t r = 0;
    int64_t t = 0;
    for (; t + kUnroll <= steps; t += kUnroll) {
        V v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t at = first + (t + u) * kStep;
            v[u] = at >= 0 ? Vec<VEC>::load(src + at) : Vec<VEC>::zero();
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t at = first + (t + u) * kStep;
            if (at >= 0) {
                if (tail) v[u] = mask_tail<VEC>(v[u], at, sp, valid);
                if (STORE) Vec<VEC>::store(dst + at, v[u]);
            }
        }
        if (CRC) {
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) r = crc_step(tb, r, v[u]);
        }
    }
    for (; t < steps; ++t) {
        const int64_t at = first + t * kStep;
        V v = Vec<VEC>::zero();
        if (at >= 0) {
            v = Vec<VEC>::load(src + at);
            if (tail) v = mask_tail<VEC>(v, at, sp, valid);
            if (STORE) Vec<VEC>::store(dst + at, v);
        }
        if (CRC) r = crc_step(tb, r, v);
    }
    return r;
}

enum Mode { kGather = 0, kScatter = 1 };

struct SpanArgs {
    const kvsnap_span* spans;
    int nspans;
    const int64_t* blocks;   // cache block ids
    const int64_t* packed;   // packed block addresses: gather targets / scatter sources
    int64_t n;
    int32_t valid;           // gather: token slots kept in the last block (0: all)
    uint32_t* crc;           // raw XOR accumulators, zeroed before launch, or null
    const uint32_t* gate;    // scatter: skip all writes when *gate != 0
    uint32_t* status;
    int split = 0;           // grid-stride segment kernels: units are 1 / 2^split of a span (KVSNAP_DP_SPLIT*)
    int place = 0;           // grid-stride segment kernels: placement tables follow the line buffers
    int spans_at = -1;       // segment kernels: byte offset of a shared-memory copy of the span table, or -1
    int clean = 0;           // segment kernels, set in the kernel: the table passed the checks every unit needs
};

template <int VEC, int MODE>
__global__ void __launch_bounds__(256) span_kernel(SpanArgs a) {
    __shared__ uint32_t tb[Vec<VEC>::kTables * 256];
    const bool crc = a.crc != nullptr;
    if (crc) load_tables<VEC>(tb);
    __syncthreads();
    if (MODE == kScatter && a.gate && *a.gate) return;
    const int lane = threadIdx.x & 31;
    const uint32_t lane_shift = crc ? dev_xpow8n((uint64_t)VEC * (31 - lane)) : 0;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t units = a.n * a.nspans;
    for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < units; u += warps) {
        const int64_t i = u / a.nspans;
        const kvsnap_span sp = a.spans[u - i * a.nspans];
        const int64_t block = a.blocks[i];
        if (block < 0 || block >= sp.nblocks) {
            if (lane == 0) flag(a.status, KVSNAP_DP_BAD_BLOCK);
            continue;
        }
        const int64_t packed = a.packed[i] + sp.offset;
        const int64_t cache = sp.base + block * sp.pitch;
        if ((packed | cache | sp.bytes) & (VEC - 1)) {
            if (lane == 0) flag(a.status, KVSNAP_DP_MISALIGNED);
            continue;
        }
        const char* src = reinterpret_cast<const char*>(MODE == kGather ? cache : packed);
        char* dst = reinterpret_cast<char*>(MODE == kGather ? packed : cache);
        const bool tail = MODE == kGather && a.valid > 0 && i == a.n - 1;
        uint32_t r;
        if (crc)
            r = warp_unit<VEC, true, true>(tb, src, dst, sp.bytes, lane, tail, sp, a.valid);
        else
            r = warp_unit<VEC, true, false>(tb, src, dst, sp.bytes, lane, tail, sp, a.valid);
        if (crc) {
            r = warp_xor(gf_mulmod(r, gf_mulmod(lane_shift, sp.crc_shift)));
            if (lane == 0) atomicXor(&a.crc[i], r);
        }
    }
}

// ---- segment-lane kernels, for packed blocks in device memory -------------------
//
// When both sides of a copy are HBM, the L1 data pipe (global and shared
// wavefronts together) and the latency of the loads in flight, not DRAM
// alone, bound a CRC'ing copy. Three things keep the wavefronts per byte low:
//   * every global load and store moves whole 128-byte lines, 8 lanes a line
//     (fully coalesced);
//   * each lane folds the bytes it loaded, in stream order, so nothing goes
//     through shared memory but the table lookups;
//   * the lookups go to per-lane copies of the tables, so none conflicts.
// A unit of `len` bytes is front-padded with zeros to 4 equal segments of S
// bytes, S a multiple of 1 KiB (a zero prefix leaves a zero-started raw CRC as
// is). Lanes 8r..8r+7 own segment r: in step t, load j of lane (r, s) moves
// 16-byte slot s of line 8t + j of segment r, so each load instruction moves
// four whole lines, each step 1 KiB of every segment straight through, and
// every lane's bytes arrive in its own registers in stream order: nothing is
// transposed through shared memory.
// A lane keeps four independent CRC chains, one per 32-bit word of its
// 16-byte slot: chain k folds word k of a line and then the 124 bytes up to
// the same word of the next line, which is slicing-by-4 with T_124..T_127.
// Four chains give the lookup latency four times the work to hide behind. At
// the end of a unit, Horner over the chains, ((c0 x^32 + c1) x^32 + c2) x^32
// + c3, and the lane's place, x^(8 * (16 * (7 - s) + S * (3 - r))), sum over
// the warp to raw(unit) * x^(8 * 124), a constant factor that the finish step
// divides out. The four tables are replicated once per lane (entry (k, v) of
// lane l lies in bank l), so the lookups never conflict. One CTA per SM holds
// 128 KiB of them.
constexpr int kRepWords = 4 * 256 * 32;                 // replicated T_124..T_127
constexpr int kSegLine = 128;                           // bytes of a line
constexpr int kSegStepLines = 8;                        // lines of each segment a step moves
constexpr int kSegStep = 4 * kSegStepLines * kSegLine;  // bytes a warp moves per step (4 KiB)
// Warps a CTA and steps of loads in flight a warp: build-time tuning knobs.
// kSegWarps sizes the register budget and the largest shared-memory layout; a
// launch may use fewer warps (the kernels read their count from blockDim). On
// B200, with two steps in flight, twelve warps measured fastest for runs of
// spans of at most 8 KiB (fewer leave small spans' per-unit work exposed);
// ten (KVSNAP_SEG_BULK_WARPS) for grid-stride units of 16 KiB, where 8, 9, 11
// and 12 warps measured 1 to 6 % slower. More than twelve leave the copying
// kernels too few registers (at 14 or 16 they spill); the whole-block CRC,
// which only loads, fits 16 warps in 128 registers (KVSNAP_SEG_CRC_WARPS).
#ifndef KVSNAP_SEG_WARPS
#define KVSNAP_SEG_WARPS 12
#endif
#ifndef KVSNAP_SEG_BULK_WARPS
#define KVSNAP_SEG_BULK_WARPS 10
#endif
#ifndef KVSNAP_SEG_DEPTH
#define KVSNAP_SEG_DEPTH 2
#endif
constexpr int kSegWarps = KVSNAP_SEG_WARPS;
constexpr int kSegBulkWarps = KVSNAP_SEG_BULK_WARPS;
static_assert(kSegBulkWarps >= 1 && kSegBulkWarps <= kSegWarps, "bulk launches use at most kSegWarps warps");
constexpr int kSegDepth = KVSNAP_SEG_DEPTH;
constexpr int kSegThreads = 32 * kSegWarps;

// Replicated layout, 256 bytes an entry so one byte permute forms an address:
// entry v of T_{127-(2h+p)} for lane l lies at byte h*65536 + v*256 + p*128 + 4l,
// which puts every lane in its own bank whatever v is. The layout is built at
// compile time into a 128 KiB image in global memory, and each CTA copies it
// with asynchronous 16-byte copies, all of a thread's in flight at once.
struct alignas(16) RepImage {
    uint32_t w[kRepWords];
};

constexpr RepImage make_rep_image() {
    const CrcTables t = make_tables();
    RepImage r{};
    for (int i = 0; i < kRepWords; ++i) {
        const int h = i >> 14, v = (i >> 6) & 255, p = (i >> 5) & 1;
        r.w[i] = t.t[27 - (2 * h + p)][v];   // slot 27 - q holds T_{127-q}
    }
    return r;
}

__device__ const RepImage g_rep = make_rep_image();

// Each thread waits for its own copies here; the prologue's closing barrier makes them visible
// to the CTA.
__device__ __forceinline__ void load_rep_tables(uint32_t* tb) {
    const uint32_t to = static_cast<uint32_t>(__cvta_generic_to_shared(tb));
    const uint4* from = reinterpret_cast<const uint4*>(g_rep.w);
    for (int i = threadIdx.x; i < kRepWords / 4; i += blockDim.x)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(to + 16u * uint32_t(i)), "l"(from + i)
                     : "memory");
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// The replicated T_124..T_127 and one plain copy of T_0..T_3.
__device__ __forceinline__ void load_seg_tables(uint32_t* tb, uint32_t* t4) {
    load_rep_tables(tb);
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) t4[i] = g_tables.t[i >> 8][i & 255];
}

// The factor the segment kernels leave on every block's raw CRC, inverted.
constexpr uint32_t kSegUnscale = gf_xpow_neg8n(124);

// The replicated tables as a lane sees them: the shared base and 4 * lane.
struct RepTables {
    const char* t;
    uint32_t l4;
    __device__ __forceinline__ uint32_t at(int offset, uint32_t x, uint32_t sel) const {
        // __byte_perm(x, l4, 0x55b4) = (byte b of x) << 8 | 4 * lane
        return *reinterpret_cast<const uint32_t*>(t + offset + __byte_perm(x, l4, sel));
    }
};

// r <- raw(r, the 4 bytes of w then 124 zero bytes), little-endian byte order:
// T_127[x0] ^ T_126[x1] ^ T_125[x2] ^ T_124[x3] for x = r ^ w.
__device__ __forceinline__ uint32_t crc_word(const RepTables& tl, uint32_t r, uint32_t w) {
    const uint32_t x = r ^ w;
    return tl.at(0, x, 0x5504) ^ tl.at(128, x, 0x5514) ^ tl.at(65536, x, 0x5524) ^ tl.at(65536 + 128, x, 0x5534);
}

struct Chains {
    uint32_t c[4] = {0, 0, 0, 0};
    __device__ __forceinline__ void fold(const RepTables& tl, uint4 v) {
        c[0] = crc_word(tl, c[0], v.x);
        c[1] = crc_word(tl, c[1], v.y);
        c[2] = crc_word(tl, c[2], v.z);
        c[3] = crc_word(tl, c[3], v.w);
    }
};

// Segment bytes S for a unit of `len` bytes: whole steps of 8 lines.
__device__ __forceinline__ int64_t seg_bytes(int64_t len) { return (len + kSegStep - 1) / kSegStep * (kSegStep / 4); }

// Bytes of one step of one segment.
constexpr int kSegStepSeg = kSegStepLines * kSegLine;

// The place of lane (row, slot)'s bytes in a unit of 4 segments of `seg` bytes,
// as the exponent n of x^(8n) that puts them there.
__host__ __device__ constexpr uint64_t lane_place(int64_t seg, int lane) {
    return uint64_t(16 * (7 - (lane & 7))) + uint64_t(seg) * uint64_t(3 - (lane >> 3));
}

// Token-slot test of the save's last block: the bytes at span offset `at` belong
// to token slot (at / token_pitch) % tokens, which is >= valid exactly when
// at mod (token_pitch * tokens) >= valid * token_pitch. A 16-byte vector lies in
// one (head, token) row when row_bytes is a multiple of 16; otherwise the
// general byte-wise mask applies.
struct TailMask {
    uint32_t group = 0, keep = 0;
    bool rows = false;
    TailMask() = default;
    __device__ TailMask(const kvsnap_span& sp, int valid) {
        const int64_t g = sp.token_pitch * sp.tokens;
        rows = sp.row_bytes % 16 == 0 && g > 0 && g <= INT32_MAX && sp.bytes <= INT32_MAX;
        if (rows) {
            group = uint32_t(g);
            keep = uint32_t(valid) * uint32_t(sp.token_pitch);
        }
    }
    __device__ __forceinline__ uint4 apply(uint4 v, int64_t at, const kvsnap_span& sp, int valid) const {
        if (rows) return uint32_t(at) % group >= keep ? make_uint4(0, 0, 0, 0) : v;
        return mask_tail<16>(v, at, sp, valid);
    }
};

// Loads bypass L1 and ask L2 for whole 256-byte sectors: eight lanes cover a
// 128-byte line and a lane's next line follows in the same segment, so the
// second half of each sector is read by the next step.
__device__ __forceinline__ uint4 seg_load(const char* src, int64_t at) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (at >= 0)
        asm volatile("ld.global.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(src + at));
    return v;
}

// The same load at an address known to be inside the source (no front padding).
__device__ __forceinline__ uint4 seg_load_line(const char* p) {
    uint4 v;
    asm("ld.global.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

// Both sides are streamed: a session is far larger than L2, so nothing a
// gather or scatter touches is read again from L2.
__device__ __forceinline__ void seg_store(char* dst, int64_t at, uint4 v) {
    __stcs(reinterpret_cast<uint4*>(dst + at), v);
}

// r * x^32 mod P: four zero bytes through slicing-by-4 (T_0..T_3, one shared copy).
__device__ __forceinline__ uint32_t mul_x32(const uint32_t* t4, uint32_t r) {
    return t4[768 + (r & 255)] ^ t4[512 + ((r >> 8) & 255)] ^ t4[256 + ((r >> 16) & 255)] ^ t4[r >> 24];
}

// A lane's four chains, combined: ((c0 x^32 + c1) x^32 + c2) x^32 + c3.
__device__ __forceinline__ uint32_t combine_chains(const Chains& r, const uint32_t* t4) {
    uint32_t h = mul_x32(t4, r.c[0]) ^ r.c[1];
    h = mul_x32(t4, h) ^ r.c[2];
    return mul_x32(t4, h) ^ r.c[3];
}

// x^(8 * lane_place(S, lane)), which moves a lane's chains to their place in a
// unit of 4 segments of S bytes; recomputed only when S changes.
// With `after` > 0 (a piece of a split span, `after` pieces of 4 * S bytes
// following it), times x^(8 * 4 * S * after), cached per value of `after`.
struct LaneShift {
    int64_t seg = -1;
    uint32_t k = 0, k1 = 0, k2 = 0, k3 = 0;
    uint32_t known = 0;          // bit a: the factor for after = a is cached
    __device__ __forceinline__ uint32_t factor(int64_t s, int lane, int after = 0) {
        if (s != seg) {
            seg = s;
            k = dev_xpow8n(lane_place(s, lane));
            known = 1;
        }
        if (after == 0) return k;
        if (!(known >> after & 1)) {
            const uint32_t f = gf_mulmod(k, dev_xpow8n(uint64_t(4 * s) * uint64_t(after)));
            if (after == 1) k1 = f; else if (after == 2) k2 = f; else k3 = f;
            known |= 1u << after;
        }
        return after == 1 ? k1 : after == 2 ? k2 : k3;
    }
};

// r * x^(8*m) for the m = `bytes` the table tx was built for (four lookups,
// as mul_x32 with T_k[v] * x^(8m-32)), or by a GF(2) multiply for any other m.
struct AppendBytes {
    const uint32_t* tx;
    int64_t bytes;
    __device__ __forceinline__ uint32_t apply(uint32_t r, int64_t m) const {
        if (m == bytes) return mul_x32(tx, r);
        return gf_mulmod(r, dev_xpow8n(uint64_t(m)));
    }
};

// Builds tx[k*256 + v] = T_k[v] * x^(8m - 32) (m >= 4), the table of AppendBytes.
__device__ __forceinline__ void load_append_table(uint32_t* tx, int64_t m) {
    const uint32_t f = dev_xpow8n(uint64_t(m - 4));
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) tx[i] = gf_mulmod(g_tables.t[i >> 8][i & 255], f);
}

// ---- placing a unit by table ------------------------------------------------------
//
// Without runs every unit ends with two products: each lane's segment value by
// its placement factor F_l = x^(8 * lane_place(seg, l)), and the warp's sum by the
// unit's shift x^(8 * bytes after it in its block). A GF(2) multiply loop is 32
// dependent steps; both products go through shared tables instead, built once
// a CTA, when the unit has the segment size and a position the tables hold.
//
// Window table (8 KiB): win[(4j + v)*32 + l] = (v << 2j) * F_l. A lane's
// product is the XOR of sixteen lookups, one a 2-bit window of its value, each
// in the lane's own bank.
// Shift table: sh[33r + l] = shift_r * x^l for row r = (span << split) +
// piece, shift_r = x^(8 * bytes after that unit in its block). Bit k of a value
// stands for x^(31-k), so for a warp-uniform y, y * shift_r = XOR over lanes l
// of (bit 31-l of y) * sh[33r + l]: one lookup a lane and a warp XOR.
//
// The tables are used only where the CTA's shared memory stays within
// kSegCarveBytes. The SM splits 256 KiB between shared memory and L1 in steps;
// above 196 KiB of shared memory (less 1 KiB the CTA reserves) L1 falls from
// 60 to 28 KiB, too little for the loads a CTA keeps in flight: the same
// kernel with 200 KiB requested measured 13 % slower.
constexpr int kWinWords = 16 * 4 * 32;
constexpr int kShiftPitch = 33;          // words a position: 32, and one so rows start in other banks
constexpr int kSegCarveBytes = 195 * 1024;

__host__ __device__ constexpr int place_bytes(int positions) { return (kWinWords + positions * kShiftPitch) * 4; }

// r * x, reflected: one step of a GF(2) multiply loop.
__device__ __forceinline__ uint32_t gf_mulx(uint32_t r) { return (r >> 1) ^ (kPoly & (0u - (r & 1u))); }

struct Placement {
    const char* win = nullptr;      // the window table + 4 * lane; null: no tables
    const uint32_t* sh = nullptr;   // the shift table
    int64_t seg = -1;               // the segment size the window table was built for
    int split = 0;                  // log2 of the units a span: rows are (span << split) + piece
};

// Window table for segment size seg. Window j of lane l covers bits 2j and
// 2j+1, which stand for x^(31-2j) and x^(30-2j) times F_l.
__device__ void build_windows(uint32_t* win, int64_t seg) {
    for (int e = threadIdx.x; e < 16 * 32; e += blockDim.x) {
        const int j = e >> 5, l = e & 31;
        uint32_t b1 = dev_xpow8n(lane_place(seg, l));
        for (int k = 0; k < 30 - 2 * j; ++k) b1 = gf_mulx(b1);
        const uint32_t b0 = gf_mulx(b1);
        win[(4 * j + 0) * 32 + l] = 0u;
        win[(4 * j + 1) * 32 + l] = b0;
        win[(4 * j + 2) * 32 + l] = b1;
        win[(4 * j + 3) * 32 + l] = b0 ^ b1;
    }
}

// Shift table rows 0..count-1; shift_of(r) gives row r's x^(8 * bytes after its unit).
template <class ShiftOf>
__device__ void build_shifts(uint32_t* sh, int count, ShiftOf shift_of) {
    for (int s = threadIdx.x; s < count; s += blockDim.x) {
        uint32_t b = shift_of(s);
        for (int l = 0; l < 32; ++l) {
            sh[kShiftPitch * s + l] = b;
            b = gf_mulx(b);
        }
    }
}

// a * F_lane through the window table (win already offset by 4 * lane).
__device__ __forceinline__ uint32_t window_mul(const char* win, uint32_t a) {
    uint32_t r = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j)
        r ^= *reinterpret_cast<const uint32_t*>(win + 512 * j + 128 * ((a >> (2 * j)) & 3u));
    return r;
}

// ---- a warp's stream of units --------------------------------------------------
//
// A warp takes its units as one stream of 4 KiB steps, so the loads of the
// next units' first steps are in flight while the current unit finishes: small
// units (a TP shard's 4 or 8 KiB spans) pay no load latency of their own. The
// load side runs kSegDepth steps ahead of the fold side and hands each unit's
// description over through a ring in shared memory.
//
// Small spans (RUNS): a warp takes a contiguous range of units, mostly
// consecutive spans of one packed block, and folds their CRCs as one run.
// Each lane keeps a Horner sum of its segments' values over the run,
// multiplying by x^(8 * bytes of the next unit): four lookups in a shared
// table when that is the span size the table was built for. Placing the lanes
// and the run in the block then costs two GF(2) multiplies and one atomic per
// run, not per unit. The caller asks for this with KVSNAP_DP_RUNS when its
// spans are small; otherwise units are placed one by one and dealt to warps
// grid-stride, which measured faster for 32 KiB spans.

// One unit as the warp's stream carries it (the same in every lane).
struct alignas(16) SegUnit {
    const char* src;
    char* dst;
    int64_t seg;         // bytes of each of the unit's 4 segments, a multiple of kSegStepSeg
    int64_t pad;         // zero bytes in front of the unit
    int64_t block;       // the packed block it belongs to (its CRC accumulator)
    uint32_t shift;      // x^(8 * bytes after the unit in its packed block)
    int32_t steps;       // seg / kSegStepSeg
    int32_t span;        // position of the unit in its block (span, pair or piece), for runs and the tail mask
    int32_t after;       // pieces after this one in its span (a split span), else 0
    int64_t alt;         // the cache-side base of segments 2 and 3: the second span of a pair, less
                         // its size; else the same base as segments 0 and 1
};
// The load side is at most kSegDepth steps, so at most kSegDepth + 1 units
// (it moves on to the next unit as soon as it issues a unit's last step),
// ahead of the unit being folded: kSegDepth + 2 entries never collide.
constexpr int kRing = kSegDepth + 2 <= 4 ? 4 : 8;
static_assert(kRing >= kSegDepth + 2 && (kRing & (kRing - 1)) == 0, "ring of unit descriptions");

// Dynamic shared memory of a segment kernel of `warps` warps, in order: the
// replicated tables, T_0..T_3 (the chain combine), for runs the append table,
// then the unit rings (a launch without a CRC holds only the rings). The
// replicated tables start the layout so that their base is a constant: each
// lookup addresses a constant plus its byte-permuted index. It is sized to the launch: shared memory and L1
// split one 256 KiB array a SM, and what L1 keeps holds the loads in flight
// (a 200 KiB layout, which leaves 28 KiB of L1 instead of 60, measured 13 %
// slower).
__host__ __device__ constexpr int seg_ring_bytes(int warps) { return warps * kRing * int(sizeof(SegUnit)); }
__host__ __device__ constexpr int seg_smem_bytes(int warps, bool runs) {
    return seg_ring_bytes(warps) + (runs ? 2 : 1) * 4 * 256 * 4 + kRepWords * 4;
}
constexpr int kSegSmemTotal = seg_smem_bytes(kSegWarps, true);
static_assert(kSegSmemTotal <= 227 * 1024, "segment kernels exceed the shared memory of a CTA");
// Rows of placement tables a grid-stride CTA of `warps` warps can hold after its other shared memory.
__host__ __device__ constexpr int place_rows(int warps) {
    return (kSegCarveBytes - seg_smem_bytes(warps, false) - kWinWords * 4) / (kShiftPitch * 4);
}
constexpr int kSegSmemMax = kSegSmemTotal > kSegCarveBytes ? kSegSmemTotal : kSegCarveBytes;
static_assert(kSegSmemMax <= 227 * 1024, "segment kernels exceed the shared memory of a CTA");

// A warp's view of that layout.
struct SegSmem {
    SegUnit* ring;       // its unit ring
    uint32_t* t4;        // T_0..T_3
    uint32_t* tx;        // the append table (runs only)
    uint32_t* tb;        // the replicated tables
    __device__ SegSmem(uint4* smem, int warp, bool runs, bool crc) {
        tb = reinterpret_cast<uint32_t*>(smem);
        t4 = tb + kRepWords;
        tx = t4 + 4 * 256;
        ring = reinterpret_cast<SegUnit*>(crc ? t4 + (runs ? 2 : 1) * 4 * 256 : tb) + warp * kRing;
    }
};

// (block, span) units of a gather or scatter: unit u is span u % nspans of
// packed block u / nspans, walked as (block, span) steps so that no unit costs
// a 64-bit division. RANGE: warp w of W takes the contiguous units
// [u*w/W, u*(w+1)/W), whose neighbours are mostly the next span of the same
// block (runs); otherwise warp w takes units w, w + W, ..., so that
// concurrent warps move neighbouring bytes.
template <int MODE, bool RANGE, int WIDTH = 1>
struct SpanUnits {
    static_assert(WIDTH == 1 || (RANGE && WIDTH == 2), "units of two spans walk contiguous ranges");
    static constexpr int width = WIDTH;    // spans a unit: 2 for pairs, else 1
    SpanArgs a;
    int64_t i, left;     // packed block of the cursor, and units left to walk
    int64_t di;          // block step (grid-stride)
    int s, ds;           // span of the cursor, and its step (grid-stride)
    int p, dp;           // piece of the cursor in its span, and its step (grid-stride)
    int split;           // log2 of the units a span (grid-stride only), else 0
    int64_t held = -1, held_block = 0, held_packed = 0;   // packed block `held`'s cache id and address
    __device__ SpanUnits(const SpanArgs& args, int64_t w, int64_t warps) : a(args) {
        split = RANGE ? 0 : args.split;
        const int per_block = args.nspans / width << split;
        const int64_t count = args.n * per_block;
        const int64_t begin = RANGE ? count * w / warps : w;
        i = begin / per_block;
        const int at = int(begin - i * per_block);
        s = (at >> split) * width;
        p = at & ((1 << split) - 1);
        const int64_t spans_step = warps >> split;   // the grid stride in whole spans, and dp pieces
        dp = int(warps & ((1 << split) - 1));
        di = spans_step / args.nspans;
        ds = int(spans_step - di * args.nspans);
        left = RANGE ? count * (w + 1) / warps - begin : (begin < count ? (count - begin + warps - 1) / warps : 0);
    }
    __device__ __forceinline__ void step() {
        --left;
        if (RANGE) {
            if ((s += width) == a.nspans) {
                s = 0;
                ++i;
            }
        } else {
            i += di;
            s += ds;
            if ((p += dp) >> split) {
                p -= 1 << split;
                ++s;
            }
            if (s >= a.nspans) {
                s -= a.nspans;
                ++i;
            }
        }
    }
    __device__ __forceinline__ bool next(SegUnit& out, int lane) {
        for (; left > 0; step()) {
            const kvsnap_span& sp = a.spans[s];
            if (i != held) {     // a block's units are mostly consecutive: its table entries are read once
                held_block = a.blocks[i];
                held_packed = a.packed[i];
                held = i;
            }
            const int64_t block = held_block;
            if (block < 0 || block >= sp.nblocks) {
                if (lane == 0) flag(a.status, KVSNAP_DP_BAD_BLOCK);
                continue;
            }
            int64_t bytes = sp.bytes >> split;
            const int64_t packed = held_packed + sp.offset + p * bytes;
            const int64_t cache = sp.base + block * sp.pitch + p * bytes;
            // A clean table (every span 16-byte aligned, whole steps a piece, pairs adjacent and equal)
            // leaves a unit only its block bounds and packed address to check.
            if (!a.clean && split && (bytes << split != sp.bytes || bytes % kSegStep)) {
                if (lane == 0) flag(a.status, KVSNAP_DP_BAD_CUT);
                continue;
            }
            int64_t second = cache;      // the cache-side base of lines 16..31
            uint32_t shift = sp.crc_shift;
            if (width == 2) {            // the pair's second span follows in the packed block
                const kvsnap_span& sq = a.spans[s + 1];
                uint32_t bad = 0;
                if (!a.clean && (sq.bytes != bytes || sq.offset != sp.offset + bytes || (2 * bytes) % kSegStep))
                    bad |= KVSNAP_DP_BAD_CUT;
                if (block >= sq.nblocks) bad |= KVSNAP_DP_BAD_BLOCK;
                const int64_t other = sq.base + block * sq.pitch;
                if (!a.clean && (other & 15)) bad |= KVSNAP_DP_MISALIGNED;
                if (bad) {
                    if (lane == 0) flag(a.status, bad);
                    continue;
                }
                second = other - bytes;
                shift = sq.crc_shift;
                bytes *= 2;
            }
            if ((a.clean ? packed : packed | cache | bytes) & 15) {
                if (lane == 0) flag(a.status, KVSNAP_DP_MISALIGNED);
                continue;
            }
            out.src = reinterpret_cast<const char*>(MODE == kGather ? cache : packed);
            out.dst = reinterpret_cast<char*>(MODE == kGather ? packed : cache);
            out.alt = second;
            out.seg = seg_bytes(bytes);
            out.pad = 4 * out.seg - bytes;
            out.block = i;
            out.shift = shift;
            out.steps = int32_t(out.seg / kSegStepSeg);
            out.span = s / width;
            out.after = (1 << split) - 1 - p;
            step();
            return true;
        }
        return false;
    }
};

// 64 KiB pieces of packed blocks in device memory (the CRC of whole blocks).
constexpr int64_t kSegPiece = 64 << 10;
// Warp w of W takes units w, w + W, ..., walked as (block, piece) steps so
// that no unit costs a 64-bit division. Without `shifts` (the launcher built a
// shift table) no unit computes its shift either.
struct PieceUnits {
    const int64_t* addrs;
    int64_t n, block_bytes, pieces;
    uint32_t* status;
    int64_t i, p;        // block and piece of the cursor
    int64_t di, dp;      // the grid stride, in blocks and pieces
    bool shifts;
    __device__ PieceUnits(const int64_t* a, int64_t count, int64_t bytes, uint32_t* st, int64_t w, int64_t warps,
                          bool with_shifts)
        : addrs(a), n(count), block_bytes(bytes), pieces((bytes + kSegPiece - 1) / kSegPiece), status(st),
          shifts(with_shifts) {
        i = w / pieces;
        p = w - i * pieces;
        di = warps / pieces;
        dp = warps - di * pieces;
    }
    __device__ __forceinline__ void step() {
        i += di;
        if ((p += dp) >= pieces) {
            p -= pieces;
            ++i;
        }
    }
    __device__ __forceinline__ bool next(SegUnit& out, int lane) {
        for (; i < n; step()) {
            const int64_t at = p * kSegPiece, len = min(kSegPiece, block_bytes - at);
            const int64_t base = addrs[i] + at;
            if ((base | len) & 15) {
                if (lane == 0) flag(status, KVSNAP_DP_MISALIGNED);
                continue;
            }
            out.src = reinterpret_cast<const char*>(base);
            out.dst = nullptr;
            out.alt = base;
            out.seg = seg_bytes(len);
            out.pad = 4 * out.seg - len;
            out.block = i;
            out.shift = shifts ? dev_xpow8n(uint64_t(block_bytes - at - len)) : 0u;
            out.after = 0;
            out.steps = int32_t(out.seg / kSegStepSeg);
            out.span = int32_t(p);
            step();
            return true;
        }
        return false;
    }
};

// One warp's stream: every unit's bytes moved (STORE) and CRC'd (CRC; the
// unit's share XORed into crc_out[block]), the last block's tail masked (TAIL).
// Lane (r, s) = (l >> 3, l & 7) moves, in step t, the 16-byte slot s of lines
// 8t + j of segment r, j = 0..7; `ring` holds the warp's unit descriptions.
// ALT (runs): the cache side of lines 16..31, the loads' (1, gather) or the
// stores' (2, scatter), is addressed from the unit's `alt` base.
template <bool STORE, bool CRC, bool TAIL, bool RUNS, int ALT = 0, class Units>
__device__ __forceinline__ void warp_stream(Units units, const RepTables& tl, const uint32_t* t4,
                                            const AppendBytes& append, SegUnit* ring, int lane,
                                            uint32_t* crc_out, const kvsnap_span* spans, int valid,
                                            const Placement& pl = Placement{}) {
    const int row = lane >> 3, slot = lane & 7;
    SegUnit L;                                   // the unit the load side is in
    if (!units.next(L, lane)) return;
    int lk = 0, lt = 0;                          // its ring entry and next step
    bool loading = true;
    if (lane == 0) ring[0] = L;
    __syncwarp();
    SegUnit P = L;                               // the unit being stored and folded
    int pk = 0, pt = 0;
    Chains r;
    LaneShift place;
    // The run of units being folded together: one packed block, consecutive
    // positions, one segment size. acc is the lane's Horner sum over it.
    bool run = false;
    int64_t run_block = 0, run_seg = 0;
    int32_t run_pos = 0;
    uint32_t run_shift = 0, acc = 0;
    auto flush = [&]() {
        const uint32_t x = gf_mulmod(warp_xor(gf_mulmod(acc, place.factor(run_seg, lane))), run_shift);
        if (lane == 0) atomicXor(&crc_out[run_block], x);
    };

    // The load side's next step: its base and offset (lane-specific) for loads j = 0..7
    // at first + j * kSegLine; then the load side moves on.
    const char* lbase = nullptr;
    int64_t lfirst = 0;
    auto load_addr = [&]() {
        lbase = ALT == 1 && row >= 2 ? reinterpret_cast<const char*>(L.alt) : L.src;
        lfirst = row * L.seg + 16 * slot - L.pad + int64_t(lt) * kSegStepSeg;
    };
    auto load_move = [&]() {
        if (++lt == L.steps) {
            lt = 0;
            loading = units.next(L, lane);
            if (loading) {
                lk = (lk + 1) & (kRing - 1);
                if (lane == 0) ring[lk] = L;
            }
        }
    };
    auto load_next = [&](uint4(&v)[8]) -> bool {
        if (!loading) return false;
        load_addr();
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = seg_load(lbase, lfirst + j * kSegLine);
        load_move();
        return true;
    };
    // Store, fold and refill one step: for each j, line j is masked (TAIL),
    // stored, folded into the chains, and its register refilled with the load
    // side's next step, so the loads go out while the step is folded.
    auto step = [&](uint4(&v)[8]) -> bool {
        const int64_t first = row * P.seg + 16 * slot - P.pad + int64_t(pt) * kSegStepSeg;
        char* sbase = ALT == 2 && row >= 2 ? reinterpret_cast<char*>(P.alt) : P.dst;
        TailMask mask;
        kvsnap_span sp{};
        if (TAIL) {
            sp = spans[P.span];
            mask = TailMask(sp, valid);
        }
        const bool refill = loading;
        if (refill) load_addr();
        if (!TAIL && P.pad == 0 && (!refill || L.pad == 0)) {
            // No front padding on either side (every unit of a whole number of 4 KiB steps): each
            // side's eight lines are one base plus constant offsets, with no per-line test. On
            // B200 this path moved 4 and 8 KiB spans 4 to 5 % faster at 132 CTAs. Issuing each
            // refill before its line is folded (a copy of the line kept) measured 8 % slower.
            char* const sd = sbase + first;
            const char* const ls = lbase + lfirst;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (STORE) __stcs(reinterpret_cast<uint4*>(sd + j * kSegLine), v[j]);
                if (CRC) r.fold(tl, v[j]);
                if (refill) v[j] = seg_load_line(ls + j * kSegLine);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int64_t at = first + j * kSegLine;     // the front padding can cover whole segments
                if (TAIL && at >= 0) v[j] = mask.apply(v[j], at, sp, valid);
                if (STORE && at >= 0) seg_store(sbase, at, v[j]);
                if (CRC) r.fold(tl, v[j]);
                if (refill) v[j] = seg_load(lbase, lfirst + j * kSegLine);
            }
        }
        if (refill) load_move();
        return refill;
    };
    // After a step: at the end of a unit, its CRC share goes out and the next unit comes in.
    auto advance = [&]() {
        if (++pt < P.steps) return;
        if (CRC && !RUNS) {
            const uint32_t h = combine_chains(r, t4);
            uint32_t x;
            if (pl.win) {   // by table; the shift row holds the piece's place in its span
                const uint32_t y = warp_xor(P.seg == pl.seg ? window_mul(pl.win, h) : gf_mulmod(h, place.factor(P.seg, lane)));
                const int row = (P.span << pl.split) + ((1 << pl.split) - 1 - P.after);
                x = warp_xor((y >> (31 - lane)) & 1u ? pl.sh[kShiftPitch * row + lane] : 0u);
            } else {
                x = gf_mulmod(warp_xor(gf_mulmod(h, place.factor(P.seg, lane, P.after))), P.shift);
            }
            if (lane == 0) atomicXor(&crc_out[P.block], x);
            r = Chains{};
        }
        if (CRC && RUNS) {
            const uint32_t h = combine_chains(r, t4);
            if (run && P.block == run_block && P.span == run_pos + 1 && P.seg == run_seg) {
                acc = append.apply(acc, 4 * P.seg - P.pad) ^ h;
            } else {
                if (run) flush();
                run = true;
                run_block = P.block;
                run_seg = P.seg;
                acc = h;
            }
            run_pos = P.span;
            run_shift = P.shift;
            r = Chains{};
        }
        pt = 0;
        pk = (pk + 1) & (kRing - 1);
        __syncwarp();
        P = ring[pk];                            // stale once the stream has ended; then unused
        __syncwarp();
    };

    uint4 v[kSegDepth][8];
    int pending = 0;
#pragma unroll
    for (int d = 0; d < kSegDepth; ++d)
        if (load_next(v[d])) ++pending;
    while (pending > 0) {
#pragma unroll
        for (int d = 0; d < kSegDepth; ++d) {
            if (pending > 0) {                   // slot d holds the oldest step in flight
                if (!step(v[d])) --pending;
                advance();
            }
        }
    }
    if (CRC && RUNS && run) flush();
}

// TAIL: every unit belongs to the save's last block, whose token slots from
// `valid` on are written as zeros. The launcher gives that block a launch of
// its own, so the common kernel carries none of the masking code.
// Shared memory: unit rings, then (with a CRC) the tables, and in the
// grid-stride path the placement tables when the launcher sized for them.
template <int MODE, bool TAIL, bool RUNS, bool PAIRS = false>
__global__ void __launch_bounds__(kSegThreads, 1) span_kernel_hbm(SpanArgs a) {
    static_assert(!PAIRS || RUNS, "pairs of spans fold in runs");
    extern __shared__ uint4 smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, per_cta = blockDim.x >> 5;
    const bool crc = a.crc != nullptr;
    const SegSmem sm(smem, warp, RUNS, crc);
    SegUnit* ring = sm.ring;
    uint32_t *t4 = sm.t4, *tx = sm.tx, *tb = sm.tb;
    // Runs are folded with the first unit's size (a pair: two spans); units of other sizes take the multiply.
    const int64_t first_bytes = (PAIRS ? 2 : 1) * a.spans[0].bytes;
    const int64_t span_bytes = first_bytes >= 4 ? first_bytes : 4;
    Placement pl;
    if (crc) {
        load_seg_tables(tb, t4);
        if (RUNS) load_append_table(tx, span_bytes);
        if (!RUNS && !TAIL && a.place) {   // the launcher sized shared memory for the placement tables
            uint32_t* win = reinterpret_cast<uint32_t*>(smem + seg_smem_bytes(per_cta, false) / 16);
            const kvsnap_span* spans = a.spans;
            const int split = a.split;
            const int64_t seg = seg_bytes(spans[0].bytes >> split);   // the windows: the first unit's size
            build_windows(win, seg);
            build_shifts(win + kWinWords, a.nspans << split, [spans, split](int r) {
                const kvsnap_span& sp = spans[r >> split];
                const int after = (1 << split) - 1 - (r & ((1 << split) - 1));   // pieces after it in its span
                return after ? gf_mulmod(sp.crc_shift, dev_xpow8n(uint64_t(sp.bytes >> split) * uint64_t(after)))
                             : sp.crc_shift;
            });
            pl = Placement{reinterpret_cast<const char*>(win) + 4 * lane, win + kWinWords, seg, split};
        }
    }
    // The span table each unit's description reads, copied where the launcher made room for it:
    // small units (a TP shard's) look it up every other step.
    SpanArgs b = a;
    if (a.spans_at >= 0) {
        uint4* to = reinterpret_cast<uint4*>(reinterpret_cast<char*>(smem) + a.spans_at);
        const uint4* from = reinterpret_cast<const uint4*>(a.spans);
        for (int k = threadIdx.x; k < a.nspans * int(sizeof(kvsnap_span) / 16); k += blockDim.x) to[k] = from[k];
        b.spans = reinterpret_cast<const kvsnap_span*>(to);
    }
    // The table checks that hold for every unit, made once a CTA (TP shards' small units would
    // otherwise repeat them every other step).
    int ok = 1;
    for (int k = threadIdx.x; k < a.nspans; k += blockDim.x) {
        const kvsnap_span& sp = a.spans[k];
        if ((sp.base | sp.pitch | sp.offset | sp.bytes) & 15) ok = 0;
        if (a.split && ((sp.bytes >> a.split) << a.split != sp.bytes || (sp.bytes >> a.split) % kSegStep)) ok = 0;
        if (PAIRS && (k & 1)) {
            const kvsnap_span& sq = a.spans[k - 1];
            if (sp.bytes != sq.bytes || sp.offset != sq.offset + sq.bytes || (2 * sp.bytes) % kSegStep) ok = 0;
        }
    }
    b.clean = __syncthreads_and(ok);
    if (MODE == kScatter && a.gate && *a.gate) return;
    const RepTables tl{reinterpret_cast<const char*>(tb), 4u * lane};
    const AppendBytes append{tx, span_bytes};
    const int64_t w = (int64_t)blockIdx.x * per_cta + warp, warps = (int64_t)gridDim.x * per_cta;
    if (!crc)
        warp_stream<true, false, TAIL, false>(SpanUnits<MODE, false>(b, w, warps), tl, t4, append, ring, lane,
                                              nullptr, b.spans, b.valid);
    else
        warp_stream<true, true, TAIL, RUNS, RUNS ? (MODE == kGather ? 1 : 2) : 0>(
            SpanUnits<MODE, RUNS, PAIRS ? 2 : 1>(b, w, warps), tl, t4, append, ring, lane, b.crc, b.spans, b.valid,
            pl);
}

// `place`: the launcher sized shared memory for placement tables with a shift row a piece.
#ifndef KVSNAP_SEG_CRC_WARPS
#define KVSNAP_SEG_CRC_WARPS 16
#endif
// Warps of the whole-block CRC, which only loads (its own register budget):
// 12, 14 and 16 measured 0.69, 0.73 and 0.78 of the HBM copy rate.
constexpr int kSegCrcWarps = KVSNAP_SEG_CRC_WARPS;
static_assert(seg_smem_bytes(kSegCrcWarps, false) + kWinWords * 4 <= kSegCarveBytes, "CRC kernel shared memory");

__global__ void __launch_bounds__(32 * kSegCrcWarps, 1) crc_kernel_hbm(const int64_t* addrs, int64_t n,
                                                                 int64_t block_bytes, uint32_t* crc,
                                                                 uint32_t* status, int place) {
    extern __shared__ uint4 smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, per_cta = blockDim.x >> 5;
    const SegSmem sm(smem, warp, false, true);
    SegUnit* ring = sm.ring;
    uint32_t *t4 = sm.t4, *tx = sm.tx, *tb = sm.tb;     // tx: unused without runs
    load_seg_tables(tb, t4);
    Placement pl;
    const int64_t pieces = (block_bytes + kSegPiece - 1) / kSegPiece;
    if (place) {   // windows for whole pieces; row p: x^(8 * bytes after piece p in its block)
        uint32_t* win = reinterpret_cast<uint32_t*>(smem + seg_smem_bytes(per_cta, false) / 16);
        build_windows(win, seg_bytes(kSegPiece));
        build_shifts(win + kWinWords, int(pieces), [block_bytes](int p) {
            const int64_t at = int64_t(p) * kSegPiece;
            return dev_xpow8n(uint64_t(block_bytes - at - min(kSegPiece, block_bytes - at)));
        });
        pl = Placement{reinterpret_cast<const char*>(win) + 4 * lane, win + kWinWords, seg_bytes(kSegPiece), 0};
    }
    __syncthreads();
    const RepTables tl{reinterpret_cast<const char*>(tb), 4u * lane};
    const AppendBytes append{tx, kSegPiece};
    const PieceUnits units(addrs, n, block_bytes, status, (int64_t)blockIdx.x * per_cta + warp,
                           (int64_t)gridDim.x * per_cta, !place);
    warp_stream<false, true, false, false>(units, tl, t4, append, ring, lane, crc, nullptr, 0, pl);
}

// CRC32C of whole packed blocks, in pieces of kPiece bytes per warp.
constexpr int64_t kPiece = 64 << 10;

template <int VEC>
__global__ void __launch_bounds__(256) crc_kernel(const int64_t* addrs, int64_t n, int64_t block_bytes,
                                                  uint32_t* crc, uint32_t* status) {
    __shared__ uint32_t tb[Vec<VEC>::kTables * 256];
    load_tables<VEC>(tb);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const uint32_t lane_shift = dev_xpow8n((uint64_t)VEC * (31 - lane));
    const int64_t pieces = (block_bytes + kPiece - 1) / kPiece;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    kvsnap_span none{};
    for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n * pieces; u += warps) {
        const int64_t i = u / pieces, p = u - i * pieces;
        const int64_t at = p * kPiece, len = min(kPiece, block_bytes - at);
        const int64_t base = addrs[i] + at;
        if ((base | len) & (VEC - 1)) {
            if (lane == 0) flag(status, KVSNAP_DP_MISALIGNED);
            continue;
        }
        uint32_t r = warp_unit<VEC, false, true>(tb, reinterpret_cast<const char*>(base), nullptr, len, lane,
                                                 false, none, 0);
        const uint32_t after = dev_xpow8n((uint64_t)(block_bytes - at - len));
        r = warp_xor(gf_mulmod(r, gf_mulmod(lane_shift, after)));
        if (lane == 0) atomicXor(&crc[i], r);
    }
}

// crc[i] <- crc[i] * unscale ^ (~0 ^ ~0 * x^(8*block_bytes)): the factor a
// kernel left on the raw CRC divided out, then the inverted register and
// output of the standard CRC32C, once per block; then the comparison.
__global__ void finish_kernel(uint32_t* crc, const uint32_t* expect, int64_t n, uint32_t unscale,
                              uint32_t init_term, uint32_t* status) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t value = gf_mulmod(crc[i], unscale) ^ init_term;
    crc[i] = value;
    if (expect && value != expect[i]) flag(status, KVSNAP_DP_CRC_MISMATCH);
}

// ---- SHA-256 (FIPS 180-4) -----------------------------------------------------

__constant__ uint32_t kSha256K[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }
__device__ __forceinline__ uint32_t be32(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// Message words of chunk c of a block at p (bytes, block_bytes long), big-endian,
// SHA-256 padding included: chunks [0, full) are data, the last one or two carry
// the remaining bytes, 0x80, zeros and the bit length.
__device__ __forceinline__ void sha256_words(const unsigned char* p, bool aligned, int64_t c, int64_t full,
                                             int rest, uint64_t bits, uint32_t w[16]) {
    if (c < full) {
        if (aligned) {
            const uint4* q = reinterpret_cast<const uint4*>(p + 64 * c);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint4 v = __ldcs(q + k);
                w[4 * k + 0] = be32(v.x);
                w[4 * k + 1] = be32(v.y);
                w[4 * k + 2] = be32(v.z);
                w[4 * k + 3] = be32(v.w);
            }
        } else {
            for (int j = 0; j < 16; ++j) {
                const unsigned char* b = p + 64 * c + 4 * j;
                w[j] = (uint32_t(b[0]) << 24) | (uint32_t(b[1]) << 16) | (uint32_t(b[2]) << 8) | b[3];
            }
        }
        return;
    }
    const int k = int(c - full);                     // 0, or 1 when the tail needs two chunks
    const unsigned char* tail = p + 64 * full;
    for (int j = 0; j < 16; ++j) {
        uint32_t word = 0;
        for (int q = 0; q < 4; ++q) {
            const int at = 64 * k + 4 * j + q;
            const uint32_t byte = at < rest ? tail[at] : (at == rest ? 0x80u : 0u);
            word = (word << 8) | byte;
        }
        w[j] = word;
    }
    if (k == (rest < 56 ? 0 : 1)) {
        w[14] = uint32_t(bits >> 32);
        w[15] = uint32_t(bits);
    }
}

// SHA-256 with the work of one block split over two warps on two SM
// sub-partitions. One lane of each hashes one block, 32 blocks a warp pair:
// the schedule warp loads each 64-byte chunk and expands it into the 64 words
// W[t] + K[t] in a shared-memory ring; the compress warp runs only the 64
// rounds, reading those words. Per block the rounds are a serial chain and
// their integer issue rate bounds the hash time, so the compress warp gets a
// sub-partition to itself. The two warps hand ring slots over with named
// barriers (bar.arrive / bar.sync, 64 threads): both run the same number of
// chunks, so every wait is matched. The schedule warp keeps the loads of the
// next kShaPrefetch chunks in flight, so that its loads (from device memory,
// or over the host link for blocks in pinned memory) do not hold the rounds up.
//
// A launch hashes one part of every block: bytes [done, done + part) of a
// block of `total` bytes, starting at addrs[i]. The first part starts from the
// initial hash value, later ones from the 8 state words the previous part
// left; the last part pads (with the whole block's bit length) and writes the
// digest. A whole-block hash is the one part [0, total).
#ifndef KVSNAP_SHA_SLOTS
#define KVSNAP_SHA_SLOTS 3
#endif
#ifndef KVSNAP_SHA_PREFETCH
#define KVSNAP_SHA_PREFETCH 1
#endif
#ifndef KVSNAP_SHA_PAIRS
#define KVSNAP_SHA_PAIRS 2
#endif
constexpr int kShaPairs = KVSNAP_SHA_PAIRS;       // warp pairs a CTA
constexpr int kShaSlots = KVSNAP_SHA_SLOTS;       // ring slots a pair
constexpr int kShaPrefetch = KVSNAP_SHA_PREFETCH; // chunks a schedule lane has loads in flight for
constexpr int kShaSlotWords = 64 * 32;
static_assert(1 + 2 * kShaSlots * kShaPairs <= 16, "a CTA has 16 named barriers, and barrier 0 is __syncthreads'");

struct ShaPart {
    const int64_t* addrs;    // where each block's part starts
    int64_t n;
    int64_t part;            // bytes of each block in this part
    int64_t total;           // bytes of a whole block (the length the padding records)
    int first, last;         // the part starts / ends the blocks
    uint32_t* state;         // 8 words a block between parts
    uint8_t* out;            // 32 bytes a block, written by the last part
};

__device__ __forceinline__ void named_arrive(int id) { asm volatile("bar.arrive %0, 64;" ::"r"(id) : "memory"); }
__device__ __forceinline__ void named_sync(int id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }

// a + c issued as a multiply-add (`one` is 1 at run time, so the compiler
// cannot fold it into an add): it runs on the FMA pipe and leaves the integer
// ALU, which the rotations and logic ops keep busy, to them.
__device__ __forceinline__ uint32_t fadd(uint32_t a, uint32_t one, uint32_t c) {
    uint32_t d;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(one), "r"(c));
    return d;
}

__device__ __forceinline__ void be_words(const uint4 (&v)[4], uint32_t w[16]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        w[4 * k + 0] = be32(v[k].x);
        w[4 * k + 1] = be32(v[k].y);
        w[4 * k + 2] = be32(v[k].z);
        w[4 * k + 3] = be32(v[k].w);
    }
}

__global__ void __launch_bounds__(64 * kShaPairs) sha256_kernel(ShaPart a, uint32_t one) {
    extern __shared__ uint32_t ring[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = warp >> 1;
    // Warps 0,1 / 2,3 form pairs; even warps compress and odd warps schedule, so
    // within a CTA the compress warps sit on sub-partitions 0 and 2.
    const bool compress = (warp & 1) == 0;
    const int64_t first = ((int64_t)blockIdx.x * kShaPairs + pair) * 32;
    if (first >= a.n) return;                        // the whole pair idles together
    const int64_t i = first + lane;
    const bool live = i < a.n;
    uint32_t* slots = ring + pair * kShaSlots * kShaSlotWords;
    const int full_id = 1 + pair * 2 * kShaSlots;    // barrier ids: FULL[s], EMPTY[s] per pair
    const int empty_id = full_id + kShaSlots;
    const int64_t full = a.part / 64;
    const int rest = int(a.part - full * 64);
    const int64_t chunks = full + (a.last ? (rest < 56 ? 1 : 2) : 0);

    if (!compress) {
        const unsigned char* p = reinterpret_cast<const unsigned char*>(a.addrs[live ? i : a.n - 1]);
        const bool aligned = (reinterpret_cast<uintptr_t>(p) & 15) == 0;
        const uint64_t bits = uint64_t(a.total) * 8;
        const uint4* q = reinterpret_cast<const uint4*>(p);
        uint4 next[kShaPrefetch][4];
        if (aligned) {
#pragma unroll
            for (int u = 0; u < kShaPrefetch; ++u)
                if (u < full) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) next[u][k] = __ldcs(q + 4 * u + k);
                }
        }
        for (int64_t base = 0; base < chunks; base += kShaPrefetch) {
#pragma unroll
            for (int u = 0; u < kShaPrefetch; ++u) {
                const int64_t c = base + u;
                if (c >= chunks) break;
                uint32_t w[16];
                if (aligned && c < full) {
                    // This chunk's words, then the loads of the chunk kShaPrefetch on in flight under the expansion.
                    be_words(next[u], w);
                    if (c + kShaPrefetch < full) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) next[u][k] = __ldcs(q + 4 * (c + kShaPrefetch) + k);
                    }
                } else {
                    sha256_words(p, aligned, c, full, rest, bits, w);
                }
                const int s = int(c % kShaSlots);
                if (c >= kShaSlots) named_sync(empty_id + s);
                uint32_t* slot = slots + s * kShaSlotWords + lane;
#pragma unroll
                for (int t = 0; t < 64; ++t) {
                    if (t >= 16) {
                        const uint32_t x = w[(t + 1) & 15], y = w[(t + 14) & 15];
                        w[t & 15] += (rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3)) + w[(t + 9) & 15] +
                                     (rotr(y, 17) ^ rotr(y, 19) ^ (y >> 10));
                    }
                    slot[t * 32] = w[t & 15] + kSha256K[t];
                }
                named_arrive(full_id + s);
            }
        }
        // Match the compress warp's last releases, so every barrier generation completes.
        for (int64_t c = chunks > kShaSlots ? chunks - kShaSlots : 0; c < chunks; ++c)
            named_sync(empty_id + int(c % kShaSlots));
        return;
    }
    uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    if (!a.first && live) {
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = a.state[8 * i + j];
    }
    for (int64_t c = 0; c < chunks; ++c) {
        const int s = int(c % kShaSlots);
        named_sync(full_id + s);
        const uint32_t* slot = slots + s * kShaSlotWords + lane;
        uint32_t a0 = h[0], b = h[1], cc = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
#pragma unroll
        for (int t = 0; t < 64; ++t) {
            // The round, reassociated so the new e is one three-input add after
            // Sigma1 and Ch: e' = (d + h + W + K) + Sigma1(e) + Ch(e,f,g), with
            // d + h + W + K formed off the critical path from values known rounds
            // earlier. T1 = (h + W + K) + Ch + Sigma1 goes to the FMA pipe, beside
            // the rotations on the ALU; placing e' there too lengthened the chain
            // (34.8 and 36.2 ms a session instead of 33.9 in a variant sweep).
            const uint32_t hk = k + slot[t * 32];
            const uint32_t dhk = d + hk;
            const uint32_t ch = (e & f) ^ (~e & g);
            const uint32_t s1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
            const uint32_t e_new = dhk + ch + s1;
            const uint32_t t1 = fadd(s1, one, fadd(ch, one, hk));
            const uint32_t s0 = rotr(a0, 2) ^ rotr(a0, 13) ^ rotr(a0, 22);
            const uint32_t maj = (a0 & b) ^ (a0 & cc) ^ (b & cc);
            const uint32_t a_new = t1 + s0 + maj;
            k = g;
            g = f;
            f = e;
            e = e_new;
            d = cc;
            cc = b;
            b = a0;
            a0 = a_new;
        }
        named_arrive(empty_id + s);
        h[0] += a0; h[1] += b; h[2] += cc; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += k;
    }
    if (!live) return;
    if (a.last) {
        uint32_t* o = reinterpret_cast<uint32_t*>(a.out + 32 * i);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = be32(h[j]);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) a.state[8 * i + j] = h[j];
    }
}

// ---- landing a column of packed blocks -------------------------------------------
//
// The bounded staged save moves each block a column at a time, so its copies
// to the targets are small (a few hundred KiB each). The SMs store them
// instead of the copy engine: a warp moves one 4 KiB piece of one block a step,
// 16 bytes a lane, eight loads in flight before the eight stores.
__global__ void __launch_bounds__(256) land_kernel(const char* src, int64_t stride, const int64_t* targets,
                                                   int64_t offset, int64_t n, int64_t len, uint32_t* status) {
    const int lane = threadIdx.x & 31;
    const int64_t pieces = (len + 4095) / 4096;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n * pieces; u += warps) {
        const int64_t i = u / pieces, p = u - i * pieces;
        const int64_t target = targets[i] + offset;
        if (target & 15) {
            if (lane == 0 && p == 0) flag(status, KVSNAP_DP_MISALIGNED);
            continue;
        }
        const char* from = src + i * stride + p * 4096;
        char* to = reinterpret_cast<char*>(target) + p * 4096;
        const int64_t left = len - p * 4096;
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int64_t at = int64_t(k * 32 + lane) * 16;
            if (at < left) v[k] = __ldcs(reinterpret_cast<const uint4*>(from + at));
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int64_t at = int64_t(k * 32 + lane) * 16;
            if (at < left) __stcs(reinterpret_cast<uint4*>(to + at), v[k]);
        }
    }
}

// ---- the reference restore kernel's interface ------------------------------------

__global__ void __launch_bounds__(256) copy_host_blocks_kernel(const int64_t* sources, const int64_t* blocks,
                                                               int64_t n_blocks, const int64_t* offsets,
                                                               const int64_t* bases, const int64_t* pitches,
                                                               const int64_t* words, int64_t n_layers) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t j = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); j < n_blocks * n_layers;
         j += warps) {
        const int64_t b = j / n_layers, l = j - b * n_layers;
        const char* src = reinterpret_cast<const char*>(sources[b] + offsets[l]);
        char* dst = reinterpret_cast<char*>(bases[l] + blocks[b] * pitches[l]);
        const int64_t len = words[l] * 8;
        if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | len) & 15) == 0) {
            for (int64_t at = 16 * lane; at < len; at += 512)
                *reinterpret_cast<uint4*>(dst + at) = __ldcs(reinterpret_cast<const uint4*>(src + at));
        } else {
            for (int64_t at = 8 * lane; at < len; at += 256)
                *reinterpret_cast<uint2*>(dst + at) = __ldcs(reinterpret_cast<const uint2*>(src + at));
        }
    }
}

// ---- tensor-parallel regroup ---------------------------------------------------------
//
// Restore at TP size T of a snapshot saved at TP size T*g: each of this rank's
// cache blocks takes its heads from g source shards, shard q holding heads
// [q*H/g, (q+1)*H/g) of every layer. The shards' packed blocks may sit in
// this GPU's memory or a peer GPU's (mapped over NVLink with CUDA IPC); the
// kernel reads them with plain loads, so the transfer over NVLink is fused with
// the interleave into the cache rows. Plain loads only, no waits on other GPUs:
// the host orders the ranks before and after the launch.

// Byte offset of row (head, token) inside a dense [H, N, C] block span whose
// token slots are `token_pitch` bytes apart: head-major when a token slot is
// one row, token-major otherwise.
__device__ __forceinline__ int64_t row_at(const kvsnap_span& sp, int64_t head, int64_t token) {
    const int64_t heads = sp.bytes / (int64_t(sp.tokens) * sp.row_bytes);
    const int64_t head_pitch = sp.token_pitch == sp.row_bytes ? int64_t(sp.tokens) * sp.row_bytes : sp.row_bytes;
    (void)heads;
    return head * head_pitch + token * sp.token_pitch;
}

struct RegroupArgs {
    const kvsnap_span* dst;      // this rank's registered spans (the cache)
    const kvsnap_span* src;      // one shard's packed layout: same spans, heads / groups
    int nspans;
    const int64_t* shards;       // shard q of block i at shards[i * groups + q]
    int groups;
    const int64_t* blocks;       // this rank's cache block ids
    int64_t n;
    uint32_t* status;
};

__global__ void __launch_bounds__(256) regroup_kernel(RegroupArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t units = a.n * a.nspans;
    for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < units; u += warps) {
        const int64_t i = u / a.nspans;
        const int s = int(u - i * a.nspans);
        const kvsnap_span d = a.dst[s], sp = a.src[s];
        const int64_t block = a.blocks[i];
        if (block < 0 || block >= d.nblocks) {
            if (lane == 0) flag(a.status, KVSNAP_DP_BAD_BLOCK);
            continue;
        }
        const int64_t rows_per_shard = sp.bytes / sp.row_bytes;   // heads/g x tokens
        const int64_t shard_heads = rows_per_shard / sp.tokens;
        const int64_t row = d.row_bytes;
        char* cache = reinterpret_cast<char*>(d.base + block * d.pitch);
        if ((row & 15) || (reinterpret_cast<uintptr_t>(cache) & 15) || sp.row_bytes != row) {
            if (lane == 0) flag(a.status, KVSNAP_DP_MISALIGNED);
            continue;
        }
        const int64_t vecs_per_row = row / 16;
        const int64_t total = a.groups * rows_per_shard * vecs_per_row;
        for (int64_t v = lane; v < total; v += 32) {
            const int64_t q = v / (rows_per_shard * vecs_per_row);
            const int64_t rest = v - q * rows_per_shard * vecs_per_row;
            const int64_t r = rest / vecs_per_row, k = rest - r * vecs_per_row;
            const int64_t h = r / sp.tokens, t = r - h * sp.tokens;     // head within the shard, token
            const char* shard = reinterpret_cast<const char*>(a.shards[i * a.groups + q]);
            const uint4 x = *reinterpret_cast<const uint4*>(shard + sp.offset + row_at(sp, h, t) + 16 * k);
            *reinterpret_cast<uint4*>(cache + row_at(d, q * shard_heads + h, t) + 16 * k) = x;
        }
    }
}

// ---- host side ----------------------------------------------------------------------

struct Fail {
    const char* what;
};

void check(cudaError_t rc) {
    if (rc != cudaSuccess) throw Fail{cudaGetErrorString(rc)};
}

template <typename F>
int guarded(F&& body) {
    try {
        body();
        return 0;
    } catch (const Fail& f) {
        kvsnap_internal_set_error(f.what);
        return -1;
    }
}

// Make the stream's device current and return its SM count.
int enter_stream(uintptr_t stream) {
    int device = 0;
    if (stream) {
        check(cudaStreamGetDevice(reinterpret_cast<cudaStream_t>(stream), &device));
        check(cudaSetDevice(device));
    } else {
        check(cudaGetDevice(&device));
    }
    int sms = 0;
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    return sms;
}

// Raise a kernel's dynamic shared memory limit on the current device, once per
// (kernel, device): the attribute belongs to the kernel's instance on that device.
void configure_once(const void* fn, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int device = 0;
    check(cudaGetDevice(&device));
    std::lock_guard<std::mutex> hold(mu);
    if (done.count({fn, device})) return;
    check(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.insert({fn, device});
}

int grid_for(int64_t warps_of_work, int ctas, int sms) {
    if (ctas > 0) return ctas;
    int64_t want = (warps_of_work + 7) / 8;   // 8 warps a CTA
    int64_t cap = 4LL * sms;
    return int(want < 1 ? 1 : (want > cap ? cap : want));
}

uint32_t init_term(uint64_t block_bytes) { return ~0u ^ gf_mulmod(~0u, gf_xpow8n(block_bytes)); }

// unscale: kSegUnscale after the segment kernels, 1 (x^0) after the others.
void finish(uint32_t* crc, const uint32_t* expect, int64_t n, uint64_t block_bytes, uint32_t* status,
            cudaStream_t s, uint32_t unscale = 1u << 31) {
    finish_kernel<<<int((n + 255) / 256), 256, 0, s>>>(crc, expect, n, unscale, init_term(block_bytes), status);
    check(cudaGetLastError());
}

}  // namespace

extern "C" int kvsnap_dp_abi_version() { return KVSNAP_DP_ABI_VERSION; }

extern "C" uint32_t kvsnap_dp_crc32c_host(const void* data, size_t size, uint32_t prior) {
    // Bytewise, from the tables: a self-check of the device tables' generator.
    static const CrcTables tables = make_tables();
    const unsigned char* p = static_cast<const unsigned char*>(data);
    uint32_t r = ~prior;
    for (size_t i = 0; i < size; ++i) r = tables.t[0][(r ^ p[i]) & 0xFFu] ^ (r >> 8);
    return ~r;
}

extern "C" int kvsnap_dp_plan(kvsnap_span* spans, int nspans, uint64_t* block_bytes) {
    return guarded([&] {
        if (!spans || nspans <= 0 || !block_bytes) throw Fail{"plan needs at least one span"};
        uint64_t total = 0;
        for (int s = 0; s < nspans; ++s) {
            if (spans[s].bytes <= 0) throw Fail{"span without bytes"};
            spans[s].offset = int64_t(total);
            total += uint64_t(spans[s].bytes);
        }
        for (int s = 0; s < nspans; ++s)
            spans[s].crc_shift = gf_xpow8n(total - uint64_t(spans[s].offset) - uint64_t(spans[s].bytes));
        *block_bytes = total;
    });
}

namespace {

// Room for a shared-memory copy of the span table after a segment kernel's `bytes`, when it keeps
// the launch within kSegCarveBytes (the L1 the loads in flight need); returns the launch's bytes.
static_assert(sizeof(kvsnap_span) % 16 == 0, "the span table is copied in 16-byte vectors");
int with_span_table(SpanArgs& a, int bytes, int nspans) {
    const int at = (bytes + 15) / 16 * 16;
    const int end = at + nspans * int(sizeof(kvsnap_span));
    // The copy loads the table in 16-byte vectors: only a 16-byte aligned table is copied.
    if (end > kSegCarveBytes || (reinterpret_cast<uintptr_t>(a.spans) & 15)) return bytes;
    a.spans_at = at;
    return end;
}

// The gather or scatter launches; throws Fail on a bad request or a CUDA error.
template <int MODE>
void spans_launch(const kvsnap_span* spans, int nspans, uint64_t block_bytes, const int64_t* blocks,
                  const int64_t* packed, int64_t n, int32_t valid, uint32_t* crc, const uint32_t* expect,
                  const uint32_t* gate, uint32_t* status, int vec, int ctas, uintptr_t stream) {
    {
        const bool hbm = (vec & KVSNAP_DP_HBM) != 0;
        const bool runs = (vec & KVSNAP_DP_RUNS) != 0, pairs = (vec & KVSNAP_DP_PAIRS) != 0;
        const int split = (vec & KVSNAP_DP_SPLIT_MASK) / KVSNAP_DP_SPLIT2;   // log2 of the pieces a span
        const bool accumulate = (vec & KVSNAP_DP_CRC_ACCUMULATE) != 0;
        vec &= ~(KVSNAP_DP_HBM | KVSNAP_DP_RUNS | KVSNAP_DP_PAIRS | KVSNAP_DP_SPLIT_MASK | KVSNAP_DP_CRC_ACCUMULATE);
        if (accumulate && (!hbm || expect)) throw Fail{"KVSNAP_DP_CRC_ACCUMULATE needs KVSNAP_DP_HBM and no expect"};
        if (split && (!hbm || runs || split > 2)) throw Fail{"split spans need KVSNAP_DP_HBM, without KVSNAP_DP_RUNS"};
        if (n < 0 || nspans <= 0 || !spans) throw Fail{"invalid span table"};
        if (pairs && (!hbm || !runs)) throw Fail{"pairs of spans need KVSNAP_DP_HBM and KVSNAP_DP_RUNS"};
        if (pairs && nspans % 2) throw Fail{"pairs of spans need an even span count"};
        if (vec != 16 && vec != 8) throw Fail{"vector width must be 16 or 8"};
        if (hbm && vec != 16) throw Fail{"the device-memory kernels need 16-byte alignment"};
        if (n == 0) return;
        if (!blocks || !packed) throw Fail{"block and address tables are required"};
        if (expect && !crc) throw Fail{"verifying needs a CRC output"};
        const int sms = enter_stream(stream);
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        if (crc && !accumulate) check(cudaMemsetAsync(crc, 0, sizeof(uint32_t) * size_t(n), s));
        SpanArgs a{spans, nspans, blocks, packed, n, valid, crc, gate, status, split};
        if (hbm) {
            // Without a CTA count, the segment kernels run on all SMs but one in nine (132 of 148):
            // with 12 warps a CTA, B200 moved every span size fastest at 128 to 136 CTAs, and 3 to
            // 10 % slower from 140 CTAs on (4, 8, 16 and 32 KiB spans alike).
            const int cap = ctas > 0 ? ctas : (sms - sms / 9 > 0 ? sms - sms / 9 : 1);
            auto grid_of = [&](int64_t blocks_of_work, int warps) {
                const int64_t want = ((blocks_of_work * nspans << split) + warps - 1) / warps;
                return ctas > 0 ? ctas : int(want < cap ? want : cap);
            };

            int64_t body = n;
            if constexpr (MODE == kGather) {
                if (valid > 0) {   // the last block, masked, in a launch of its own
                    body = n - 1;
                    SpanArgs last{spans, nspans, blocks + body, packed + body, 1, valid, crc ? crc + body : nullptr,
                                  gate, status};
                    int bytes = crc ? seg_smem_bytes(kSegWarps, false) : seg_ring_bytes(kSegWarps);
                    bytes = with_span_table(last, bytes, nspans);
                    configure_once(reinterpret_cast<const void*>(span_kernel_hbm<MODE, true, false>), kSegSmemMax);
                    span_kernel_hbm<MODE, true, false><<<grid_of(1, kSegWarps), kSegThreads, bytes, s>>>(last);
                    check(cudaGetLastError());
                }
            }
            if (body > 0) {
                a.n = body;
                auto kernel = !runs ? span_kernel_hbm<MODE, false, false>
                              : pairs ? span_kernel_hbm<MODE, false, true, true> : span_kernel_hbm<MODE, false, true>;
                // A launch on fewer CTAs than SMs keeps more loads in flight a CTA: at 132 of 148 SMs, 12
                // warps moved Qwen3-8B spans at 0.93 of the HBM copy rate where 10 reached 0.91; a launch
                // asked for on every SM takes 10 warps, which measured fastest there.
                const int warps = runs || cap < sms ? kSegWarps : kSegBulkWarps;
                // Grid-stride units are placed by table when the rows fit within kSegCarveBytes.
                const int rows = nspans << split;
                a.place = crc && !runs && rows <= place_rows(warps);
                int bytes = !crc ? seg_ring_bytes(warps) : seg_smem_bytes(warps, runs) + (a.place ? place_bytes(rows) : 0);
                bytes = with_span_table(a, bytes, nspans);
                configure_once(reinterpret_cast<const void*>(kernel), kSegSmemMax);
                kernel<<<grid_of(body, warps), 32 * warps, bytes, s>>>(a);
                check(cudaGetLastError());
            }
            if (crc && !accumulate) finish(crc, expect, n, block_bytes, status, s, kSegUnscale);
            return;
        }
        const int grid = grid_for(n * nspans, ctas, sms);
        if (vec == 16)
            span_kernel<16, MODE><<<grid, 256, 0, s>>>(a);
        else
            span_kernel<8, MODE><<<grid, 256, 0, s>>>(a);
        check(cudaGetLastError());
        if (crc) finish(crc, expect, n, block_bytes, status, s);
    }
}

template <int MODE>
int launch_spans(const kvsnap_span* spans, int nspans, uint64_t block_bytes, const int64_t* blocks,
                 const int64_t* packed, int64_t n, int32_t valid, uint32_t* crc, const uint32_t* expect,
                 const uint32_t* gate, uint32_t* status, int vec, int ctas, uintptr_t stream) {
    return guarded([&] {
        spans_launch<MODE>(spans, nspans, block_bytes, blocks, packed, n, valid, crc, expect, gate, status, vec,
                           ctas, stream);
    });
}

}  // namespace

extern "C" int kvsnap_dp_gather(const kvsnap_span* spans, int nspans, uint64_t block_bytes, const int64_t* blocks,
                                const int64_t* targets, int64_t n, int32_t valid_tokens, uint32_t* crc_out,
                                uint32_t* status, int vec, int ctas, uintptr_t stream) {
    if (valid_tokens < 0) {
        kvsnap_internal_set_error("valid_tokens must be non-negative");
        return -1;
    }
    return launch_spans<kGather>(spans, nspans, block_bytes, blocks, targets, n, valid_tokens, crc_out, nullptr,
                                 nullptr, status, vec, ctas, stream);
}

extern "C" int kvsnap_dp_scatter(const kvsnap_span* spans, int nspans, uint64_t block_bytes,
                                 const int64_t* sources, const int64_t* blocks, int64_t n, uint32_t* crc_out,
                                 const uint32_t* expect, const uint32_t* gate, uint32_t* status, int vec,
                                 int ctas, uintptr_t stream) {
    return launch_spans<kScatter>(spans, nspans, block_bytes, blocks, sources, n, 0, crc_out, expect, gate,
                                  status, vec, ctas, stream);
}

namespace {

// CRC32C of n whole packed blocks into crc_out (cleared first), then the finish
// step. The kernels report bad addresses in `status`; the comparison with
// `expect` reports into `verdict` (the same word for kvsnap_dp_crc32c).
void crc_blocks(const int64_t* addrs, int64_t n, uint64_t block_bytes, uint32_t* crc_out, const uint32_t* expect,
                uint32_t* status, uint32_t* verdict, int vec, int ctas, cudaStream_t s, int sms) {
    const bool hbm = (vec & KVSNAP_DP_HBM) != 0;
    vec &= ~(KVSNAP_DP_HBM | KVSNAP_DP_RUNS | KVSNAP_DP_PAIRS | KVSNAP_DP_SPLIT_MASK);   // whole blocks: no use
    check(cudaMemsetAsync(crc_out, 0, sizeof(uint32_t) * size_t(n), s));
    if (hbm && vec == 16) {
        configure_once(reinterpret_cast<const void*>(crc_kernel_hbm), kSegSmemMax);
        const int64_t pieces = (int64_t(block_bytes) + kSegPiece - 1) / kSegPiece;
        const int64_t want = (n * pieces + kSegCrcWarps - 1) / kSegCrcWarps;
        const int grid = ctas > 0 ? ctas : int(want < sms ? want : sms);
        const int place = pieces <= place_rows(kSegCrcWarps);     // pieces are placed by table
        const int bytes = seg_smem_bytes(kSegCrcWarps, false) + (place ? place_bytes(int(pieces)) : 0);
        crc_kernel_hbm<<<grid, 32 * kSegCrcWarps, bytes, s>>>(addrs, n, int64_t(block_bytes), crc_out, status,
                                                               place);
        check(cudaGetLastError());
        finish(crc_out, expect, n, block_bytes, verdict, s, kSegUnscale);
        return;
    }
    const int64_t pieces = (int64_t(block_bytes) + kPiece - 1) / kPiece;
    const int grid = grid_for(n * pieces, ctas, sms);
    if (vec == 16)
        crc_kernel<16><<<grid, 256, 0, s>>>(addrs, n, int64_t(block_bytes), crc_out, status);
    else
        crc_kernel<8><<<grid, 256, 0, s>>>(addrs, n, int64_t(block_bytes), crc_out, status);
    check(cudaGetLastError());
    finish(crc_out, expect, n, block_bytes, verdict, s);
}

}  // namespace

extern "C" int kvsnap_dp_crc32c(const int64_t* addrs, int64_t n, uint64_t block_bytes, uint32_t* crc_out,
                                const uint32_t* expect, uint32_t* status, int vec, int ctas, uintptr_t stream) {
    return guarded([&] {
        const int width = vec & ~(KVSNAP_DP_HBM | KVSNAP_DP_RUNS | KVSNAP_DP_PAIRS | KVSNAP_DP_SPLIT_MASK);
        if (n < 0 || width != 16 && width != 8) throw Fail{"invalid CRC request"};
        if (n == 0) return;
        if (!addrs || !crc_out || block_bytes == 0) throw Fail{"CRC needs addresses, output and a block size"};
        const int sms = enter_stream(stream);
        crc_blocks(addrs, n, block_bytes, crc_out, expect, status, status, vec, ctas,
                   reinterpret_cast<cudaStream_t>(stream), sms);
    });
}

namespace {

void sha_launch(const int64_t* addrs, int64_t n, uint64_t part, uint64_t done, uint64_t total, uint32_t* state,
                uint8_t* out, uintptr_t stream) {
    if (n < 0 || done > total || part > total - done) throw Fail{"invalid digest request"};
    if (n == 0) return;
    const bool last = done + part == total;
    if (!addrs) throw Fail{"digests need addresses"};
    if (!last && (part % 64 || !state)) throw Fail{"a digest part before the last needs whole 64-byte chunks and a state"};
    if (done && (done % 64 || !state)) throw Fail{"a digest part after the first needs a state at a chunk boundary"};
    if (last && !out) throw Fail{"digests need an output"};
    if (last && (reinterpret_cast<uintptr_t>(out) & 3)) throw Fail{"digest output must be 4-byte aligned"};
    if (state && (reinterpret_cast<uintptr_t>(state) & 3)) throw Fail{"digest state must be 4-byte aligned"};
    enter_stream(stream);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    constexpr int smem = kShaPairs * kShaSlots * kShaSlotWords * int(sizeof(uint32_t));
    configure_once(reinterpret_cast<const void*>(sha256_kernel), smem);
    const ShaPart a{addrs, n, int64_t(part), int64_t(total), done == 0, last, state, out};
    const int64_t per_cta = 32 * kShaPairs;
    sha256_kernel<<<int((n + per_cta - 1) / per_cta), 64 * kShaPairs, smem, s>>>(a, 1u);
    check(cudaGetLastError());
}

}  // namespace

extern "C" int kvsnap_dp_sha256(const int64_t* addrs, int64_t n, uint64_t block_bytes, uint8_t* out,
                                uintptr_t stream) {
    return guarded([&] { sha_launch(addrs, n, block_bytes, 0, block_bytes, nullptr, out, stream); });
}

extern "C" int kvsnap_dp_sha256_part(const int64_t* addrs, int64_t n, uint64_t part_bytes, uint64_t done_bytes,
                                     uint64_t total_bytes, uint32_t* state, uint8_t* out, uintptr_t stream) {
    return guarded([&] { sha_launch(addrs, n, part_bytes, done_bytes, total_bytes, state, out, stream); });
}

extern "C" int kvsnap_dp_land(const void* src, int64_t src_stride, const int64_t* targets, int64_t offset,
                              int64_t n, int64_t len, uint32_t* status, int ctas, uintptr_t stream) {
    return guarded([&] {
        if (n < 0 || len < 0 || offset < 0 || src_stride < 0) throw Fail{"invalid landing request"};
        if (n == 0 || len == 0) return;
        if (!src || !targets) throw Fail{"landing needs a source and targets"};
        if (n > 1 && src_stride < len) throw Fail{"landing source blocks overlap (stride below the length)"};
        if ((reinterpret_cast<uintptr_t>(src) | uint64_t(src_stride) | uint64_t(offset) | uint64_t(len)) & 15)
            throw Fail{"landing needs 16-byte aligned sources, strides, offsets and lengths"};
        const int sms = enter_stream(stream);
        const int64_t pieces = n * ((len + 4095) / 4096);
        const int64_t want = (pieces + 7) / 8;
        const int grid = ctas > 0 ? ctas : int(want < 16 ? want : (16 < sms ? 16 : sms));
        land_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
            static_cast<const char*>(src), src_stride, targets, offset, n, len, status);
        check(cudaGetLastError());
    });
}

extern "C" int kvsnap_dp_land_strided(const void* src, int64_t src_stride, void* dst, int64_t dst_pitch, int64_t n,
                                      int64_t len, uintptr_t stream) {
    return guarded([&] {
        if (n < 0 || len < 0 || src_stride < 0 || dst_pitch < 0) throw Fail{"invalid landing request"};
        if (n == 0 || len == 0) return;
        if (!src || !dst) throw Fail{"landing needs a source and a destination"};
        if (n > 1 && (src_stride < len || dst_pitch < len))
            throw Fail{"landing rows overlap (a stride or pitch below the length)"};
        enter_stream(stream);
        // One copy-engine transfer for the whole column: n rows of len bytes.
        check(cudaMemcpy2DAsync(dst, size_t(n > 1 ? dst_pitch : len), src, size_t(n > 1 ? src_stride : len),
                                size_t(len), size_t(n), cudaMemcpyDeviceToHost, reinterpret_cast<cudaStream_t>(stream)));
    });
}

extern "C" int kvsnap_dp_crc32c_finish(uint32_t* crc, const uint32_t* expect, int64_t n, uint64_t block_bytes,
                                       uint32_t* status, uintptr_t stream) {
    return guarded([&] {
        if (n < 0) throw Fail{"invalid CRC finish request"};
        if (n == 0) return;
        if (!crc) throw Fail{"CRC finish needs the accumulators"};
        enter_stream(stream);
        finish(crc, expect, n, block_bytes, status, reinterpret_cast<cudaStream_t>(stream), kSegUnscale);
    });
}

extern "C" int kvsnap_dp_copy_host_blocks(const int64_t* sources, const int64_t* blocks, int64_t n_blocks,
                                          const int64_t* layer_offsets, const int64_t* layer_bases,
                                          const int64_t* layer_pitches, const int64_t* layer_words,
                                          int64_t n_layers, int ctas, uintptr_t stream) {
    return guarded([&] {
        if (n_blocks < 0 || n_layers < 0) throw Fail{"negative table size"};
        if (n_blocks == 0 || n_layers == 0) return;
        const int sms = enter_stream(stream);
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        const int grid = grid_for(n_blocks * n_layers, ctas, sms);
        copy_host_blocks_kernel<<<grid, 256, 0, s>>>(sources, blocks, n_blocks, layer_offsets, layer_bases,
                                                     layer_pitches, layer_words, n_layers);
        check(cudaGetLastError());
    });
}

extern "C" int kvsnap_dp_regroup(const kvsnap_span* dst_spans, const kvsnap_span* src_spans, int nspans,
                                 const int64_t* shards, int groups, const int64_t* blocks, int64_t n,
                                 uint32_t* status, int ctas, uintptr_t stream) {
    return guarded([&] {
        if (n < 0 || nspans <= 0 || groups <= 0 || !dst_spans || !src_spans) throw Fail{"invalid regroup request"};
        if (n == 0) return;
        if (!shards || !blocks) throw Fail{"regroup needs shard and block tables"};
        const int sms = enter_stream(stream);
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        RegroupArgs a{dst_spans, src_spans, nspans, shards, groups, blocks, n, status};
        regroup_kernel<<<grid_for(n * nspans, ctas, sms), 256, 0, s>>>(a);
        check(cudaGetLastError());
    });
}

extern "C" int kvsnap_dp_device_alloc(size_t size, int device, void** ptr) {
    return guarded([&] {
        if (!ptr || size == 0) throw Fail{"device allocation needs a size and an output"};
        check(cudaSetDevice(device));
        check(cudaMalloc(ptr, size));
    });
}

extern "C" int kvsnap_dp_device_free(void* ptr) {
    return guarded([&] { check(cudaFree(ptr)); });
}

extern "C" int kvsnap_dp_ipc_export(void* ptr, void* handle) {
    return guarded([&] {
        if (!ptr || !handle) throw Fail{"IPC export needs a device pointer and a 64-byte output"};
        cudaIpcMemHandle_t h;
        check(cudaIpcGetMemHandle(&h, ptr));
        memcpy(handle, &h, sizeof(h));
    });
}

extern "C" int kvsnap_dp_ipc_open(const void* handle, int device, void** ptr) {
    return guarded([&] {
        if (!handle || !ptr) throw Fail{"IPC open needs a handle and an output"};
        cudaIpcMemHandle_t h;
        memcpy(&h, handle, sizeof(h));
        check(cudaSetDevice(device));
        check(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    });
}

extern "C" int kvsnap_dp_ipc_close(void* ptr) {
    return guarded([&] { check(cudaIpcCloseMemHandle(ptr)); });
}

// ---- verified restore scatter that allocates nothing -----------------------------------
//
// For callers that cannot allocate device memory. The per-block CRC32C
// accumulators and one gate word live in this file-scope array instead of a
// caller buffer: words [0, kStaticMaxBlocks) hold the CRCs, word kStaticGate
// the verdict that gates the scatter. In host code `g_static_scratch` is a
// host-side stand-in, not a device address; every call looks the device
// address up with cudaGetSymbolAddress, with the stream's device current, and
// passes that pointer to the kernels.
constexpr int64_t kStaticMaxBlocks = KVSNAP_DP_STATIC_MAX_BLOCKS;
constexpr int64_t kStaticGate = kStaticMaxBlocks;
__device__ __align__(256) uint32_t g_static_scratch[kStaticMaxBlocks + 64];

namespace {

// The verdict of the check, copied into the caller's status word after the gated scatter.
__global__ void report_gate_kernel(const uint32_t* gate, uint32_t* status) {
    if (threadIdx.x == 0 && *gate) atomicOr(status, *gate);
}

}  // namespace

extern "C" int kvsnap_dp_scatter_verify_static(const kvsnap_span* spans, int nspans, uint64_t block_bytes,
                                               const int64_t* sources, const int64_t* blocks, int64_t n,
                                               const uint32_t* expect, uint32_t* status, int vec, int ctas,
                                               uintptr_t stream) {
    return guarded([&] {
        if (n < 0 || n > kStaticMaxBlocks) throw Fail{"kvsnap_dp_scatter_verify_static: more blocks than its fixed "
                                                      "scratch holds (KVSNAP_DP_STATIC_MAX_BLOCKS)"};
        if (!expect || !status) throw Fail{"kvsnap_dp_scatter_verify_static needs expected CRCs and a status word"};
        if (n == 0) return;
        if (!spans || nspans <= 0 || !sources || !blocks || block_bytes == 0)
            throw Fail{"kvsnap_dp_scatter_verify_static needs spans, sources, block ids and a block size"};
        const int sms = enter_stream(stream);   // the stream's device is current from here on
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        void* address = nullptr;
        check(cudaGetSymbolAddress(&address, g_static_scratch));
        uint32_t* scratch = static_cast<uint32_t*>(address);
        uint32_t* gate = scratch + kStaticGate;
        // 1. CRC32C of every source block into the scratch; a mismatch sets the gate.
        check(cudaMemsetAsync(gate, 0, sizeof(uint32_t), s));
        crc_blocks(sources, n, block_bytes, scratch, expect, status, gate, vec, ctas, s, sms);
        // 2. The scatter, which writes nothing when the gate is set.
        spans_launch<kScatter>(spans, nspans, block_bytes, blocks, sources, n, 0, nullptr, nullptr, gate, status, vec,
                               ctas, stream);
        // 3. The verdict into the caller's status.
        report_gate_kernel<<<1, 32, 0, s>>>(gate, status);
        check(cudaGetLastError());
    });
}
