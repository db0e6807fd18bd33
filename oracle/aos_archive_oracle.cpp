// CPU oracle for the adapter archive path: BLAKE3 and `.aos` archive
// validation.  TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench's CPU leg):
// the product hashes on the GPU (adapter-os_b200/csrc/blake3.cu) and parses
// archives in adapter-os_b200/csrc/aos_archive.cu.
//
// BLAKE3 comes to the reference through the `blake3` crate (Cargo.lock:
// version 1.8.3), which is not under the reference tree.  This file restates
// the published BLAKE3 function (hash mode, 32-byte output): the compression
// function with 7 rounds of the G mixing function and the message
// permutation, 1024-byte chunks of 64-byte blocks, and the left-balanced
// binary tree of parent nodes.  The reference calls it as B3Hash::hash /
// B3Hash::hash_multi (crates/adapteros-infra-common/src/hash.rs:22-36).
// Pinned by the empty-input digest of crates/adapteros-model-hub/src/
// integrity.rs:465-470 and by the segment hashes that the reference's own
// archives under test_data/adapters carry in their index entries.
//
// Archive rules restated from crates/adapteros-aos/src/writer.rs:
// header parse 407-446 (magic, index offset 64, reserved bytes zero),
// segment index 449-558 (flag bit 0, bounds, 80-byte entries, overlaps,
// per-segment BLAKE3), scope hash 31-37 (first 16 bytes of BLAKE3 of the
// scope path), segment selection 585-620.
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

const uint32_t kIV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                         0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
const int kPerm[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};
constexpr uint32_t CHUNK_START = 1, CHUNK_END = 2, PARENT = 4, ROOT = 8;

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

inline void g(uint32_t* s, int a, int b, int c, int d, uint32_t x, uint32_t y) {
    s[a] = s[a] + s[b] + x;
    s[d] = rotr(s[d] ^ s[a], 16);
    s[c] = s[c] + s[d];
    s[b] = rotr(s[b] ^ s[c], 12);
    s[a] = s[a] + s[b] + y;
    s[d] = rotr(s[d] ^ s[a], 8);
    s[c] = s[c] + s[d];
    s[b] = rotr(s[b] ^ s[c], 7);
}

// compression function; out[0..8] is the next chaining value
void compress(const uint32_t cv[8], const uint32_t block[16], uint64_t counter, uint32_t len, uint32_t flags,
              uint32_t out[16]) {
    uint32_t s[16] = {cv[0], cv[1], cv[2], cv[3], cv[4], cv[5], cv[6], cv[7],
                      kIV[0], kIV[1], kIV[2], kIV[3], (uint32_t)counter, (uint32_t)(counter >> 32), len, flags};
    uint32_t m[16];
    memcpy(m, block, sizeof m);
    for (int r = 0; r < 7; ++r) {
        g(s, 0, 4, 8, 12, m[0], m[1]);
        g(s, 1, 5, 9, 13, m[2], m[3]);
        g(s, 2, 6, 10, 14, m[4], m[5]);
        g(s, 3, 7, 11, 15, m[6], m[7]);
        g(s, 0, 5, 10, 15, m[8], m[9]);
        g(s, 1, 6, 11, 12, m[10], m[11]);
        g(s, 2, 7, 8, 13, m[12], m[13]);
        g(s, 3, 4, 9, 14, m[14], m[15]);
        if (r < 6) {
            uint32_t t[16];
            for (int i = 0; i < 16; ++i) t[i] = m[kPerm[i]];
            memcpy(m, t, sizeof m);
        }
    }
    for (int i = 0; i < 8; ++i) {
        out[i] = s[i] ^ s[i + 8];
        out[i + 8] = s[i + 8] ^ cv[i];
    }
}

void load_block(const uint8_t* p, uint32_t n, uint32_t w[16]) {  // little-endian words, zero padded
    uint8_t b[64] = {0};
    memcpy(b, p, n);
    for (int i = 0; i < 16; ++i)
        w[i] = (uint32_t)b[4 * i] | (uint32_t)b[4 * i + 1] << 8 | (uint32_t)b[4 * i + 2] << 16 |
               (uint32_t)b[4 * i + 3] << 24;
}

// chaining value of chunk `idx` (bytes p[0..n), n <= 1024); root marks the
// last block of a one-chunk input
void chunk_cv(const uint8_t* p, uint64_t n, uint64_t idx, bool root, uint32_t cv[8]) {
    uint32_t h[8];
    memcpy(h, kIV, sizeof h);
    const uint64_t nb = n == 0 ? 1 : (n + 63) / 64;
    for (uint64_t b = 0; b < nb; ++b) {
        const uint32_t len = (uint32_t)(b + 1 < nb ? 64 : n - 64 * b);
        uint32_t w[16], out[16];
        load_block(p + 64 * b, len, w);
        uint32_t f = (b == 0 ? CHUNK_START : 0) | (b + 1 == nb ? CHUNK_END : 0);
        if (root && b + 1 == nb) f |= ROOT;
        compress(h, w, idx, len, f, out);
        memcpy(h, out, sizeof h);
    }
    memcpy(cv, h, sizeof h);
}

void parent_cv(const uint32_t* l, const uint32_t* r, bool root, uint32_t cv[8]) {
    uint32_t w[16], out[16];
    memcpy(w, l, 32);
    memcpy(w + 8, r, 32);
    compress(kIV, w, 0, 64, PARENT | (root ? ROOT : 0), out);
    memcpy(cv, out, 32);
}

uint64_t rd64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = v << 8 | p[i];
    return v;
}
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }

}  // namespace

extern "C" {

// BLAKE3 of data[0..len) into out[32].  The tree is reduced level by level,
// pairing nodes (2i, 2i+1) and carrying an odd last node up unchanged, which
// is the left-balanced tree of the BLAKE3 specification.
void oracle_blake3(const void* data, uint64_t len, uint8_t out[32]) {
    const uint8_t* p = (const uint8_t*)data;
    const uint64_t n = len == 0 ? 1 : (len + 1023) / 1024;
    uint32_t root[8];
    if (n == 1) {
        chunk_cv(p, len, 0, true, root);
    } else {
        std::vector<uint32_t> cv(8 * n);
        for (uint64_t c = 0; c < n; ++c)
            chunk_cv(p + 1024 * c, c + 1 < n ? 1024 : len - 1024 * c, c, false, &cv[8 * c]);
        uint64_t m = n;
        while (m > 2) {
            const uint64_t half = m / 2;
            for (uint64_t i = 0; i < half; ++i) parent_cv(&cv[16 * i], &cv[16 * i + 8], false, &cv[8 * i]);
            if (m & 1) memmove(&cv[8 * half], &cv[8 * (m - 1)], 32);
            m = half + (m & 1);
        }
        parent_cv(&cv[0], &cv[8], true, root);
    }
    for (int i = 0; i < 8; ++i)
        for (int b = 0; b < 4; ++b) out[4 * i + b] = (uint8_t)(root[i] >> (8 * b));
}

// The same digest through the incremental form of the specification: a
// stack of subtree chaining values, merged after each completed chunk while
// the chunk count has trailing zero bits, then folded into the last chunk
// from the top of the stack down.  Tests compare it with oracle_blake3 at
// sizes beyond the reference's fixtures.
void oracle_blake3_incremental(const void* data, uint64_t len, uint8_t out[32]) {
    const uint8_t* p = (const uint8_t*)data;
    const uint64_t n = len == 0 ? 1 : (len + 1023) / 1024;
    std::vector<uint32_t> stack;
    for (uint64_t c = 0; c + 1 < n; ++c) {
        uint32_t cv[8];
        chunk_cv(p + 1024 * c, 1024, c, false, cv);
        for (uint64_t total = c + 1; (total & 1) == 0; total >>= 1) {
            uint32_t merged[8];
            parent_cv(&stack[stack.size() - 8], cv, false, merged);
            stack.resize(stack.size() - 8);
            memcpy(cv, merged, 32);
        }
        stack.insert(stack.end(), cv, cv + 8);
    }
    uint32_t cv[8];
    chunk_cv(p + 1024 * (n - 1), len - 1024 * (n - 1), n - 1, n == 1, cv);
    while (!stack.empty()) {
        uint32_t merged[8];
        parent_cv(&stack[stack.size() - 8], cv, stack.size() == 8, merged);
        stack.resize(stack.size() - 8);
        memcpy(cv, merged, 32);
    }
    for (int i = 0; i < 8; ++i)
        for (int b = 0; b < 4; ++b) out[4 * i + b] = (uint8_t)(cv[i] >> (8 * b));
}

// Validation of an archive image, in the order of writer.rs:407-558.
// Returns 0, or the number of the first failed rule:
//   1 too small for the header   2 bad magic        3 index offset != 64
//   4 reserved bytes non-zero    5 flag bit 0 clear  6 index beyond file
//   7 index size not a multiple of 80               8 manifest beyond file
//   9 manifest overlaps index    10 unknown backend tag
//   11 segment overlaps index    12 segment overlaps manifest
//   13 segment beyond file       14 segment hash mismatch
// n_seg receives the number of index entries on success.
int oracle_aos_validate(const void* data, uint64_t len, uint32_t* n_seg) {
    const uint8_t* b = (const uint8_t*)data;
    if (len < 64) return 1;
    if (!(memcmp(b, "AOS\0", 4) == 0 || memcmp(b, "AOS2", 4) == 0)) return 2;
    const uint32_t flags = rd32(b + 4);
    const uint64_t io = rd64(b + 8), isz = rd64(b + 16), mo = rd64(b + 24), ms = rd64(b + 32);
    if (io != 64) return 3;
    for (int i = 40; i < 64; ++i)
        if (b[i]) return 4;
    if (!(flags & 1)) return 5;
    if (isz > len - io) return 6;
    const uint64_t iend = io + isz;
    if (isz % 80) return 7;
    if (ms > UINT64_MAX - mo || mo + ms > len) return 8;
    if (mo < iend) return 9;
    for (uint64_t e = 0; e < isz / 80; ++e) {
        const uint8_t* ent = b + io + 80 * e;
        const uint32_t tag = (uint32_t)ent[4] | (uint32_t)ent[5] << 8;
        if (tag > 3) return 10;
        const uint64_t off = rd64(ent + 8), n = rd64(ent + 16);
        if (n > UINT64_MAX - off) return 13;
        if (off < iend) return 11;
        if (off + n > mo) return 12;
        if (off + n > len) return 13;
        uint8_t h[32];
        oracle_blake3(b + off, n, h);
        if (memcmp(h, ent + 40, 32) != 0) return 14;
    }
    *n_seg = (uint32_t)(isz / 80);
    return 0;
}

}  // extern "C"
