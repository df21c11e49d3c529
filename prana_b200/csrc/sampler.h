// sampler.h -- the host sampler object behind prana_sampler (sampler.rs:6-20, 50-70).
#pragma once
#include <cstdint>

struct prana_sampler {
  bool greedy = true;
  float temp = 0.0f;
  uint64_t state = 1;

  // XorShift::next_u64 / next_f32 (sampler.rs:59-70)
  uint64_t next_u64() {
    uint64_t x = state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    state = x;
    return x * 0x2545F4914F6CDD1DULL;
  }
  float next_f32() { return (float)(next_u64() >> 40) / (float)(1ULL << 24); }
};
