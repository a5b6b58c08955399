/*
 * ORACLE (test infrastructure only; never linked into the product library).
 *
 * Plain-C restatement of kvsnap's CRC32C, the checksum its store keeps per
 * snapshot block:
 *   - Castagnoli polynomial, reflected form 0x82F63B78;
 *   - register starts at ~prior, output is ~register (reference
 *     csrc/dataplane/io.cpp:16-25 `portable_crc`, io.cpp:39-47
 *     `kvsnap_crc32c_extend` / `kvsnap_crc32c`);
 *   - the same value as the byte-table Python path (reference
 *     kvsnap/store/crc32c.py:5-27).
 *
 * Pinned by tests/test_oracle_golden.py against the reference's known vectors
 * (tests/unit/test_native_io.py:99-103, tests/unit/test_store.py:41-44,
 * csrc/dataplane/io_test.cpp:9-10) and against the reference io.cpp compiled
 * from its own source into oracle/_ref.
 *
 * Also holds the GF(2) arithmetic the tests use to check the CUDA path's way of
 * combining partial CRCs (x^(8n) mod P in the reflected representation); that
 * part is ordinary polynomial algebra over GF(2), stated from the definition.
 */
#include <stddef.h>
#include <stdint.h>

#define ORACLE_POLY 0x82F63B78u

/* One bit at a time, straight from the definition of a reflected CRC. */
uint32_t oracle_crc32c_bitwise(const void* data, size_t size, uint32_t prior) {
    const uint8_t* p = (const uint8_t*)data;
    uint32_t reg = ~prior;
    for (size_t i = 0; i < size; ++i) {
        reg ^= p[i];
        for (int bit = 0; bit < 8; ++bit)
            reg = (reg & 1u) ? (reg >> 1) ^ ORACLE_POLY : (reg >> 1);
    }
    return ~reg;
}

static uint32_t table[256];
static int table_ready = 0;

static void build_table(void) {
    for (uint32_t v = 0; v < 256; ++v) {
        uint32_t r = v;
        for (int bit = 0; bit < 8; ++bit)
            r = (r & 1u) ? (r >> 1) ^ ORACLE_POLY : (r >> 1);
        table[v] = r;
    }
    table_ready = 1;
}

/* Byte-table form, the same recurrence as the reference's Python fallback. */
uint32_t oracle_crc32c(const void* data, size_t size, uint32_t prior) {
    if (!table_ready) build_table();
    const uint8_t* p = (const uint8_t*)data;
    uint32_t reg = ~prior;
    for (size_t i = 0; i < size; ++i)
        reg = table[(reg ^ p[i]) & 0xFFu] ^ (reg >> 8);
    return ~reg;
}

/* CRC32C of n blocks of block_bytes each, laid out back to back. */
void oracle_crc32c_blocks(const void* data, size_t nblocks, size_t block_bytes, uint32_t* out) {
    const uint8_t* p = (const uint8_t*)data;
    for (size_t b = 0; b < nblocks; ++b) out[b] = oracle_crc32c(p + b * block_bytes, block_bytes, 0);
}

/*
 * Reflected GF(2) polynomials: bit 31 holds the x^0 coefficient, bit 0 the
 * x^31 coefficient. Product a*b mod P, computed by walking a's coefficients
 * from x^0 upward while b is multiplied by x each step.
 */
uint32_t oracle_gf_mulmod(uint32_t a, uint32_t b) {
    uint32_t product = 0;
    for (int k = 31; k >= 0; --k) {
        if (a & (1u << k)) product ^= b;
        b = (b & 1u) ? (b >> 1) ^ ORACLE_POLY : (b >> 1);
    }
    return product;
}

/* x^(8*nbytes) mod P: the operator that appends nbytes zero bytes to a raw CRC register. */
uint32_t oracle_xpow8n(uint64_t nbytes) {
    uint32_t result = 1u << 31;          /* x^0 */
    uint32_t square = 1u << 23;          /* x^8: one byte */
    while (nbytes) {
        if (nbytes & 1u) result = oracle_gf_mulmod(result, square);
        square = oracle_gf_mulmod(square, square);
        nbytes >>= 1;
    }
    return result;
}

/* CRC32C of A||B from crc(A), crc(B) and |B|, for the combining rule the CUDA path relies on. */
uint32_t oracle_crc32c_combine(uint32_t crc_a, uint32_t crc_b, uint64_t len_b) {
    return oracle_gf_mulmod(oracle_xpow8n(len_b), crc_a) ^ crc_b;
}
