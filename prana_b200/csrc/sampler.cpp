// sampler.cpp -- token sampling on the host (sampler.rs): greedy argmax or
// temperature sampling with the reference's xorshift64* stream, over logits
// the caller has on the host (prana_forward returns them).  Built with
// -ffp-contract=off and libm expf, so probabilities, the running subtraction
// and therefore the drawn ids are the reference's bit for bit.
#include <cmath>
#include <cstdint>
#include <memory>
#include <new>
#include <vector>

#include "../../include/prana_cuda.h"
#include "sampler.h"

namespace prana {
int fail(int code, const char* fmt, ...);
}
using prana::fail;

namespace {

// argmax (sampler.rs:40-48): the first maximum
uint32_t argmax(const float* v, size_t n) {
  size_t best = 0;
  for (size_t i = 0; i < n; i++)
    if (v[i] > v[best]) best = i;
  return (uint32_t)best;
}

// softmax (norms.rs:44-56): max (NaN-ignoring, as f32::max folds), exp of the
// differences, sequential f32 sum, multiply by 1 / sum
void softmax(std::vector<float>& v) {
  float mx = -INFINITY;
  for (float x : v) mx = std::fmax(mx, x);
  float sum = 0.0f;
  for (float& x : v) {
    x = expf(x - mx);
  }
  for (float x : v) sum += x;
  const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
  for (float& x : v) x *= inv;
}

}  // namespace

extern "C" {

// Sampler::new (sampler.rs:13-20): greedy when temperature <= 0
int prana_sampler_create(float temperature, uint64_t seed, prana_sampler** out) {
  if (!out) return fail(PRANA_E_INVALID, "null argument");
  prana_sampler* s = new (std::nothrow) prana_sampler();
  if (!s) return fail(PRANA_E_OOM, "host allocation failed");
  s->greedy = temperature <= 0.0f;  // as Sampler::new: a NaN temperature samples
  s->temp = temperature;
  s->state = seed ? seed : 1;  // XorShift::new: seed.max(1)
  *out = s;
  return PRANA_OK;
}

int prana_sampler_free(prana_sampler* s) {
  delete s;
  return PRANA_OK;
}

// Sampler::sample (sampler.rs:22-37)
int prana_sample(prana_sampler* s, const float* logits, size_t n, uint32_t* token) {
  if (!s || !logits || !token || !n) return fail(PRANA_E_INVALID, "null argument or empty logits");
  if (s->greedy) {
    *token = argmax(logits, n);
    return PRANA_OK;
  }
  try {
    std::vector<float> p(logits, logits + n);
    for (float& x : p) x = x / s->temp;
    softmax(p);
    float r = s->next_f32();
    for (size_t i = 0; i < n; i++) {
      r -= p[i];
      if (r <= 0.0f) {
        *token = (uint32_t)i;
        return PRANA_OK;
      }
    }
    *token = (uint32_t)(n - 1);  // float round-off: the last bucket
    return PRANA_OK;
  } catch (const std::bad_alloc&) {
    return fail(PRANA_E_OOM, "host allocation failed");
  }
}

// The generator's next uniform draw in [0, 1) (XorShift::next_f32), for
// callers that sample themselves; advances the stream like prana_sample does.
int prana_sampler_next_f32(prana_sampler* s, float* out) {
  if (!s || !out) return fail(PRANA_E_INVALID, "null argument");
  *out = s->next_f32();
  return PRANA_OK;
}

}  // extern "C"
