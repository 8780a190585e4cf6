// som.cuh -- host side of the reference's .som container (crates/sosomodel/src/lib.rs:
// 32-34, :86-104; index.rs:118-139): every .som file (manifest, index, shard) is a
// 24-byte header -- magic "SOMODL01", CRC32C of the payload, version, payload length --
// then the payload (shards of version >= 2 put it at byte 64, so a mmap'd shard's weights
// are 64-byte aligned).  The checksum is CRC-32C (Castagnoli: reflected polynomial
// 0x1EDC6F41, init and final xor 0xFFFFFFFF), the `crc` crate's CRC_32_ISCSI; this is the
// published table method, eight bytes per step (slice-by-8).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>

namespace sb {
namespace som {

struct Crc32cTables {
    uint32_t t[8][256];
    Crc32cTables()
    {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = (c >> 1) ^ (0x82F63B78u & (0u - (c & 1u)));  // reflected 0x1EDC6F41
            t[0][i] = c;
        }
        for (uint32_t i = 0; i < 256; i++)
            for (int s = 1; s < 8; s++) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xffu];
    }
};

inline const Crc32cTables &crc_tables()
{
    static const Crc32cTables tabs;
    return tabs;
}

// Running CRC-32C state (pre-inverted), so that a shard can be checked piece by piece.
inline uint32_t crc32c_update(uint32_t crc, const uint8_t *p, size_t n)
{
    const Crc32cTables &T = crc_tables();
    while (n && ((uintptr_t)p & 7)) crc = (crc >> 8) ^ T.t[0][(crc ^ *p++) & 0xffu], n--;
    while (n >= 8) {
        uint64_t w;
        std::memcpy(&w, p, 8);  // little-endian hosts only (x86-64, aarch64)
        w ^= crc;
        crc = T.t[7][w & 0xff] ^ T.t[6][(w >> 8) & 0xff] ^ T.t[5][(w >> 16) & 0xff] ^ T.t[4][(w >> 24) & 0xff] ^
              T.t[3][(w >> 32) & 0xff] ^ T.t[2][(w >> 40) & 0xff] ^ T.t[1][(w >> 48) & 0xff] ^ T.t[0][w >> 56];
        p += 8, n -= 8;
    }
    while (n--) crc = (crc >> 8) ^ T.t[0][(crc ^ *p++) & 0xffu];
    return crc;
}

}  // namespace som
}  // namespace sb

extern "C" uint32_t sb_crc32c(const void *data, size_t n)
{
    if (!data && n) return 0u;
    return ~sb::som::crc32c_update(0xFFFFFFFFu, static_cast<const uint8_t *>(data), n);
}

// The payload of a .som file in memory: 1 and *payload / *len / *version set when the
// magic, the length and the CRC agree (parse_som, lib.rs:88-104, and for shards
// verify_shard, index.rs:118-139: payload at byte 24, or 64 from version 2 on), else 0.
extern "C" int sb_som_payload(const void *file, size_t file_len, int shard, const void **payload, size_t *len,
                              uint32_t *version)
{
    const uint8_t *d = static_cast<const uint8_t *>(file);
    if (!d || !payload || !len || file_len < 24 || std::memcmp(d, "SOMODL01", 8) != 0) return 0;
    uint32_t crc, ver;
    uint64_t plen;
    std::memcpy(&crc, d + 8, 4);
    std::memcpy(&ver, d + 12, 4);
    std::memcpy(&plen, d + 16, 8);
    const size_t off = (shard && ver >= 2) ? 64 : 24;
    if (plen > file_len || off > file_len - plen) return 0;
    if (~sb::som::crc32c_update(0xFFFFFFFFu, d + off, (size_t)plen) != crc) return 0;
    *payload = d + off;
    *len = (size_t)plen;
    if (version) *version = ver;
    return 1;
}
