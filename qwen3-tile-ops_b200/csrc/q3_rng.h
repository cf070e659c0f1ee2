// The random stream of numpy's np.random.default_rng(seed), host side: the
// reference's sampler draws with it (tools/engine.py: Request.rng =
// default_rng(params.seed), Sampler.sample -> rng.choice(V, p=probs)).
//
// Restated from the published algorithms (numpy 2.x; checked against numpy's
// own outputs in tests/test_sampling_cpu.py):
// * SeedSequence (M. E. O'Neill's seed_seq design as numpy adopted it): the
//   seed as little-endian 32-bit words, hashed into a 4-word pool with two
//   multiplicative hashes and a cross-mixing pass, then expanded with a second
//   hash into the words PCG64 is seeded from;
// * PCG64 = PCG-XSL-RR 128/64: a 128-bit LCG (state = state * mult + inc),
//   output = rotr64(hi ^ lo, hi >> 58) of the advanced state;
// * Generator.random() = (next64 >> 11) * 2^-53.
#pragma once

#include <stdint.h>

namespace q3rng {

constexpr uint32_t kInitA = 0x43b0d7e5u, kMultA = 0x931e8875u;
constexpr uint32_t kInitB = 0x8b51f9ddu, kMultB = 0x58f38dedu;
constexpr uint32_t kMixL = 0xca01f9ddu, kMixR = 0x4973f715u;
constexpr int kPool = 4;

struct SeedSeq {
  uint32_t pool[kPool];

  explicit SeedSeq(uint64_t seed) {
    uint32_t ent[2];
    int n = 0;
    ent[n++] = static_cast<uint32_t>(seed);
    if (seed >> 32) ent[n++] = static_cast<uint32_t>(seed >> 32);
    uint32_t hc = kInitA;
    auto hashmix = [&hc](uint32_t v) {
      v ^= hc;
      hc *= kMultA;
      v *= hc;
      v ^= v >> 16;
      return v;
    };
    auto mix = [](uint32_t x, uint32_t y) {
      uint32_t r = kMixL * x - kMixR * y;
      return r ^ (r >> 16);
    };
    for (int i = 0; i < kPool; ++i) pool[i] = hashmix(i < n ? ent[i] : 0u);
    for (int s = 0; s < kPool; ++s)
      for (int d = 0; d < kPool; ++d)
        if (s != d) pool[d] = mix(pool[d], hashmix(pool[s]));
  }

  // generate_state(n, uint64): 2n 32-bit words, paired low word first
  void state64(uint64_t *out, int n) const {
    uint32_t hc = kInitB;
    for (int i = 0; i < 2 * n; ++i) {
      uint32_t v = pool[i % kPool];
      v ^= hc;
      hc *= kMultB;
      v *= hc;
      v ^= v >> 16;
      if (i & 1) out[i / 2] |= static_cast<uint64_t>(v) << 32;
      else out[i / 2] = v;
    }
  }
};

struct Pcg64 {
  unsigned __int128 state = 0, inc = 0;
  static constexpr unsigned __int128 kMult =
      (static_cast<unsigned __int128>(0x2360ED051FC65DA4ull) << 64) | 0x4385DF649FCCF645ull;

  Pcg64() = default;
  explicit Pcg64(uint64_t seed) {
    uint64_t w[4];
    SeedSeq(seed).state64(w, 4);
    const unsigned __int128 init = (static_cast<unsigned __int128>(w[0]) << 64) | w[1];
    const unsigned __int128 seq = (static_cast<unsigned __int128>(w[2]) << 64) | w[3];
    state = 0;
    inc = (seq << 1) | 1u;
    step();
    state += init;
    step();
  }
  void step() { state = state * kMult + inc; }
  uint64_t next64() {
    step();
    const uint64_t hi = static_cast<uint64_t>(state >> 64), lo = static_cast<uint64_t>(state);
    const uint64_t x = hi ^ lo;
    const unsigned rot = static_cast<unsigned>(hi >> 58);
    return (x >> rot) | (x << ((64u - rot) & 63u));
  }
  double random() { return static_cast<double>(next64() >> 11) * (1.0 / 9007199254740992.0); }
};

}  // namespace q3rng
