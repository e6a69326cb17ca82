// TEST INFRASTRUCTURE ONLY: the CPU checker of the render's start image.
//
// The reference draws its start image in Generator::generate
// (src/u15-generator.cc:394-417) with the C++ standard library's
// std::mt19937_64 engine and std::normal_distribution<float>, one draw per
// value of the channel-last [H][W][3] image in order, each scaled in double
// by GenConfig::init_noise_scale (src/u15-config.cc:106-122) and rounded to
// float. Those two files need the vpipe SDK to compile, so the steps are
// restated here over the same library types; orc_mt19937_64_nth exposes the
// raw engine for its known answer (the C++ standard's: the 10000th output of
// a default-seeded mt19937_64 is 9981545732273789042).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <random>

extern "C" {

void orc_init_noise(uint64_t seed, double noise_scale, float* out, long n)
{
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  for (long i = 0; i < n; ++i) out[i] = (float)(noise_scale * nd(rng));
}

uint64_t orc_mt19937_64_nth(uint64_t seed, long nth)
{
  std::mt19937_64 rng(seed);
  uint64_t v = 0;
  for (long i = 0; i < nth; ++i) v = rng();
  return v;
}

// mode 0: not a resolution mode (noise_scale itself); 1: "resolution" /
// "dynamic"; 2: "dynamic_sqrt" -- the three branches of the reference's rule.
double orc_init_noise_scale(int image_tokens, int mode, double noise_scale, double max_value,
                            int base_seq_len)
{
  if (mode == 0) return std::min(noise_scale, max_value);
  const double base = (double)(base_seq_len > 0 ? base_seq_len : 64);
  double s = std::sqrt((double)image_tokens / base) * noise_scale;
  if (mode == 2) s = std::sqrt(s);
  return std::min(s, max_value);
}

}  // extern "C"
