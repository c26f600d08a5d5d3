// Exposes the reference smoke's CPU restatement of the True2D forward
// (cpu_reference, native/cuda/orbit_wars_cuda_true2d_smoke.cpp:127-260) as C
// symbols, so the golden-fixture script can run the reference's own code.
// The reference file is compiled in place through the include path; its
// main() is renamed so this builds as a library. Test infrastructure only.
#define main orbit_wars_reference_true2d_smoke_main
#include "orbit_wars_cuda_true2d_smoke.cpp"
#undef main

#include <algorithm>

extern "C" size_t ref_true2d_smoke_weight_count(void) { return weight_count(); }
extern "C" size_t ref_true2d_smoke_games(void) { return kGameCount; }

// input: 2 x 64 x 7 f32; weights: one model; output: 2 x 64 x 24 f32.
extern "C" void ref_true2d_cpu_reference(const float* input, const float* weights, float* output) {
  std::vector<float> in(input, input + kGameCount * kRowCount * kInputFeatureCount);
  std::vector<float> w(weights, weights + weight_count());
  const std::vector<float> out = cpu_reference(in, w);
  std::copy(out.begin(), out.end(), output);
}
