// CRC-64/XZ (a.k.a. CRC-64/GO-ECMA): width 64, polynomial 0x42F0E1EBA9EA3693,
// reflected input and output, init 0xFFFFFFFFFFFFFFFF, xorout
// 0xFFFFFFFFFFFFFFFF, check("123456789") = 0x995DC9BBDF1939FA.
//
// Written from the published parameter set (Rocksoft model). The same
// parameters as the reference's module hash (csrc/hook.cpp:315-321) so module
// hashes in an archive mean the same thing in both projects. Slicing-by-8
// tables for ~2-4 GB/s on a host core.
#pragma once

#include <cstddef>
#include <cstdint>

namespace fb {

struct Crc64Tables {
  uint64_t t[8][256];
  constexpr Crc64Tables() : t{} {
    constexpr uint64_t kReflectedPoly = 0xC96C5795D7870F42ull;  // bit-reverse of 0x42F0E1EBA9EA3693
    for (int i = 0; i < 256; ++i) {
      uint64_t c = static_cast<uint64_t>(i);
      for (int b = 0; b < 8; ++b) c = (c & 1) ? (c >> 1) ^ kReflectedPoly : (c >> 1);
      t[0][i] = c;
    }
    for (int i = 0; i < 256; ++i)
      for (int s = 1; s < 8; ++s) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xFF];
  }
};

inline const Crc64Tables& crc64_tables() {
  static const Crc64Tables tables;
  return tables;
}

// Streaming update: state starts at ~0 and the final value is ~state.
inline uint64_t crc64_update(uint64_t state, const void* data, size_t len) {
  const auto& T = crc64_tables().t;
  const uint8_t* p = static_cast<const uint8_t*>(data);
  while (len >= 8) {
    uint64_t v;
    __builtin_memcpy(&v, p, 8);
    state ^= v;
    state = T[7][state & 0xFF] ^ T[6][(state >> 8) & 0xFF] ^ T[5][(state >> 16) & 0xFF] ^
            T[4][(state >> 24) & 0xFF] ^ T[3][(state >> 32) & 0xFF] ^
            T[2][(state >> 40) & 0xFF] ^ T[1][(state >> 48) & 0xFF] ^ T[0][state >> 56];
    p += 8;
    len -= 8;
  }
  while (len--) state = T[0][(state ^ *p++) & 0xFF] ^ (state >> 8);
  return state;
}

inline uint64_t crc64(const void* data, size_t len) {
  return ~crc64_update(~0ull, data, len);
}

}  // namespace fb
