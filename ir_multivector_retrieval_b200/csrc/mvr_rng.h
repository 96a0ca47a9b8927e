// mvr_rng.h — host-side RNG draws of the reference build path.
//
// The reference seeds every k-means with `Rng.init(seed)` over Zig std's
// DefaultPrng (src/util/rng.zig:25-27): Xoshiro256++ whose 256-bit state is
// four SplitMix64 outputs of the 64-bit seed. k-means++ consumes one
// `nextIndex(n)` (Lemire multiply-shift bounded integer, rng.zig:35-38) and
// then one `float(f64)` per weighted draw (rng.zig:69). The draws do not
// depend on the data, so the host generates them all up front and the GPU
// consumes them in order.
#pragma once
#include <cstdint>
#include <cstring>

namespace mvr {

struct Xoshiro256pp {
  uint64_t s[4];

  static uint64_t splitmix(uint64_t& x) {
    x += 0x9e3779b97f4a7c15ULL;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
  }
  static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

  explicit Xoshiro256pp(uint64_t seed) {
    uint64_t x = seed;
    for (auto& w : s) w = splitmix(x);
  }

  uint64_t next() {
    const uint64_t r = rotl(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return r;
  }

  // Uniform integer in [0, n): multiply-shift with rejection below
  // (2^64 - n) mod n.
  uint64_t below(uint64_t n) {
    uint64_t x = next();
    unsigned __int128 m = (unsigned __int128)x * n;
    uint64_t lo = (uint64_t)m;
    if (lo < n) {
      uint64_t t = 0 - n;
      if (t >= n) {
        t -= n;
        if (t >= n) t %= n;
      }
      while (lo < t) {
        x = next();
        m = (unsigned __int128)x * n;
        lo = (uint64_t)m;
      }
    }
    return (uint64_t)(m >> 64);
  }

  static int lz(uint64_t x) { return x ? __builtin_clzll(x) : 64; }

  // Uniform double in [0, 1): 52 random mantissa bits, exponent
  // -1 - (leading zeros of the draw), extended by further draws when the
  // top 12 bits are all zero.
  double unit_f64() {
    const uint64_t r = next();
    uint64_t z = (uint64_t)lz(r);
    if (z >= 12) {
      z = 12;
      for (;;) {
        const uint64_t more = (uint64_t)lz(next());
        z += more;
        if (more != 64) break;
        if (z >= 1022) {
          z = 1022;
          break;
        }
      }
    }
    const uint64_t bits = ((1022 - z) << 52) | (r & 0xFFFFFFFFFFFFFULL);
    double d;
    std::memcpy(&d, &bits, 8);
    return d;
  }
  // Random.float(f32) (Zig std): 23 random mantissa bits from the draw's low
  // bits, exponent -1 - (leading zeros of the draw), extended by further
  // draws when the top 41 bits are all zero.
  float unit_f32() {
    const uint64_t r = next();
    uint32_t z = (uint32_t)lz(r);
    if (z >= 41) {
      z = 41 + (uint32_t)lz(next());
      if (z == 41 + 64) {
        const uint32_t x = (uint32_t)next() | 0x7FFu;
        z += (uint32_t)__builtin_clz(x);
      }
    }
    const uint32_t bits = ((126u - z) << 23) | ((uint32_t)r & 0x7FFFFFu);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
  }
};


}  // namespace mvr
