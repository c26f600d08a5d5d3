// CPU oracle for the reference's True2D self-play policy forward and its
// legacy TrainableTransformer forward.
//
// TEST INFRASTRUCTURE ONLY: called by tests, the smoke entry and the bench's
// CPU-baseline leg as the checker; the product library never uses it.
//
// Restates, for any request batch, head count and model population:
//   True2DTransformer::forward_with_trace   crates/orbit-wars-core/src/true2d_model.rs:197-283
//   expand_to_pair_matrix_from_parts        true2d_model.rs:321-366
//   apply_matrix_layer                      true2d_model.rs:419-461
//   apply_attention_layer / full_self_attention_values  true2d_model.rs:463-544
//   collapse_pair_matrix / row_softmax / weighted_target_fraction  true2d_model.rs:546-647
//   deterministic_weight / seeded           true2d_model.rs:653-663, :159-169
//   TrainableTransformer::forward           crates/orbit-wars-core/src/model.rs:210-301
// Output layout per row: 12 x (target_fraction, send_fraction), as the
// reference's GPU ABI writes it (native/cuda/orbit_wars_cuda.cu:686-774).
//
// Pinned against the reference's own C++ restatement (cpu_reference in
// native/cuda/orbit_wars_cuda_true2d_smoke.cpp:127-260) by the golden fixture
// tests/golden/true2d_smoke_fixture.npz, produced from the reference source by
// tests/golden/make_true2d_golden.py.

#include <cmath>
#include <cstdint>
#include <cstddef>
#include <vector>
#include <limits>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr size_t kFeatures = 7;         // config.rs TRUE2D_INPUT_FEATURES
constexpr size_t kTargets = 12;         // config.rs TRUE2D_ACTION_TARGETS_PER_SOURCE
constexpr size_t kCellWeights = 12;     // TRUE2D_MATRIX_LAYER_PLANES
constexpr size_t kHeadWeights = 7;
constexpr size_t kSharedWeights = 6;
constexpr size_t kOutScalars = 5;
constexpr size_t kOutPerRow = kTargets * 2;

struct T2Layout {
  size_t rows, cells, layers, heads;
  size_t pair, src_emb, tgt_emb, pair_emb, bias, matrix, attn, tbias, sbias, scalars, total;
};

T2Layout layout(size_t layers, size_t rows, size_t heads) {
  T2Layout o{};
  o.rows = rows;
  o.cells = rows * rows;
  o.layers = layers;
  o.heads = heads;
  size_t c = 0;
  o.pair = c; c += kFeatures * 2;
  o.src_emb = c; c += rows;
  o.tgt_emb = c; c += rows;
  o.pair_emb = c; c += o.cells;
  o.bias = c; c += 1;
  o.matrix = c; c += layers * o.cells * kCellWeights;
  o.attn = c; c += heads * kHeadWeights + kSharedWeights;
  o.tbias = c; c += rows * kTargets;
  o.sbias = c; c += rows * kTargets;
  o.scalars = c; c += kOutScalars * kTargets;
  o.total = c;
  return o;
}

inline float sigmoidf_(float v) { return 1.0f / (1.0f + std::exp(-v)); }

void matrix_layer(const T2Layout& L, const float* lw, std::vector<float>& m) {
  for (size_t cell = 0; cell < L.cells; ++cell) {
    const float v = m[cell];
    const float* w = lw + cell * kCellWeights;
    const float ha = std::tanh(v * w[2] + w[3]);
    const float hb = std::tanh(v * w[4] + ha * w[5] + w[6]);
    const float g = sigmoidf_(v * w[7] + w[8]);
    const float u = hb * w[9] + ha * w[10] + w[11];
    const float r = v * (1.0f + w[0]) + w[1];
    m[cell] = std::tanh(r + g * u);
  }
}

void attention_layer(const T2Layout& L, const float* aw, std::vector<float>& m) {
  std::vector<float> ctx(L.cells, 0.0f);
  for (size_t qi = 0; qi < L.cells; ++qi) {
    float combined = 0.0f;
    for (size_t h = 0; h < L.heads; ++h) {
      const float* hw = aw + h * kHeadWeights;
      const float q = m[qi] * hw[0] + hw[1];
      float mx = -std::numeric_limits<float>::infinity();
      for (size_t kj = 0; kj < L.cells; ++kj) mx = std::fmax(mx, q * (m[kj] * hw[2] + hw[3]));
      float den = 0.0f, acc = 0.0f;
      for (size_t kj = 0; kj < L.cells; ++kj) {
        const float k = m[kj] * hw[2] + hw[3];
        const float v = m[kj] * hw[4] + hw[5];
        const float a = std::exp(q * k - mx);
        den += a;
        acc += a * v;
      }
      combined += acc / den * hw[6];
    }
    ctx[qi] = combined;
  }
  const float* s = aw + L.heads * kHeadWeights;
  for (size_t cell = 0; cell < L.cells; ++cell) {
    const float r = m[cell] * s[0] + ctx[cell] + s[1];
    const float hid = std::tanh(r * s[2] + s[3]);
    m[cell] = std::tanh(r + hid * s[4] + s[5]);
  }
}

void collapse(const T2Layout& L, const float* w, const std::vector<float>& m, float* out) {
  const size_t R = L.rows;
  std::vector<float> p(R);
  for (size_t s = 0; s < R; ++s) {
    float sends[kTargets];
    float send_sum = 0.0f;
    const float* row = m.data() + s * R;
    for (size_t a = 0; a < kTargets; ++a) {
      const float* sc = w + L.scalars + a * kOutScalars;
      const float* tb = w + L.tbias + a * R;
      const float* sb = w + L.sbias + a * R;
      // target softmax -> expected index fraction
      float mx = -std::numeric_limits<float>::infinity();
      for (size_t t = 0; t < R; ++t) mx = std::fmax(mx, row[t] * sc[0] + tb[t]);
      float den = 0.0f;
      for (size_t t = 0; t < R; ++t) {
        p[t] = std::exp(row[t] * sc[0] + tb[t] - mx);
        den += p[t];
      }
      float frac = 0.0f;
      if (R > 1)
        for (size_t t = 0; t < R; ++t) frac += (p[t] / den) * (static_cast<float>(t) / static_cast<float>(R - 1));
      frac = std::fmin(std::fmax(frac, 0.0f), 1.0f);
      // send softmax -> weighted value -> sigmoid
      mx = -std::numeric_limits<float>::infinity();
      for (size_t t = 0; t < R; ++t) mx = std::fmax(mx, row[t] * sc[1] + sb[t]);
      den = 0.0f;
      for (size_t t = 0; t < R; ++t) {
        p[t] = std::exp(row[t] * sc[1] + sb[t] - mx);
        den += p[t];
      }
      float logit = sc[4];
      for (size_t t = 0; t < R; ++t) logit += (p[t] / den) * row[t] * sc[2];
      sends[a] = sigmoidf_(logit * sc[3]);
      send_sum += sends[a];
      out[s * kOutPerRow + a * 2] = frac;
    }
    for (size_t a = 0; a < kTargets; ++a)
      out[s * kOutPerRow + a * 2 + 1] = send_sum > 1.0f ? sends[a] / send_sum : sends[a];
  }
}

void forward_one(const T2Layout& L, const float* w, const float* rows, float* out) {
  const size_t R = L.rows;
  std::vector<float> m(L.cells);
  const float* pw = w + L.pair;
  for (size_t s = 0; s < R; ++s) {
    for (size_t t = 0; t < R; ++t) {
      const float* xs = rows + s * kFeatures;
      const float* xt = rows + t * kFeatures;
      float v = 0.0f;
      for (size_t f = 0; f < kFeatures; ++f) v += xs[f] * pw[f];
      for (size_t f = 0; f < kFeatures; ++f) v += xt[f] * pw[kFeatures + f];
      v += w[L.src_emb + s] + w[L.tgt_emb + t] + w[L.pair_emb + s * R + t] + w[L.bias];
      m[s * R + t] = std::tanh(v);
    }
  }
  const size_t mid = L.layers / 2;  // attention_layer_index, true2d_model.rs:128-130
  const size_t per_layer = L.cells * kCellWeights;
  for (size_t l = 0; l < mid; ++l) matrix_layer(L, w + L.matrix + l * per_layer, m);
  attention_layer(L, w + L.attn, m);
  for (size_t l = mid; l < L.layers; ++l) matrix_layer(L, w + L.matrix + l * per_layer, m);
  collapse(L, w, m, out);
}

uint64_t mix_hash(uint64_t seed, uint64_t row, uint64_t column) {
  uint64_t x = seed ^ (row * 0x9E3779B97F4A7C15ull) ^ (column * 0xBF58476D1CE4E5B9ull);
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}

}  // namespace

extern "C" {

size_t owo_true2d_weight_count(size_t layers, size_t rows, size_t heads) {
  if (layers == 0 || rows < 2 || heads == 0) return 0;
  return layout(layers, rows, heads).total;
}

// deterministic_weight(seed, row, column) of true2d_model.rs:653-663: in [-1, 1].
float owo_deterministic_weight(uint64_t seed, uint64_t row, uint64_t column) {
  const uint64_t x = mix_hash(seed, row, column);
  const float normalized = static_cast<float>(static_cast<double>(x) / static_cast<double>(UINT64_MAX));
  return normalized * 2.0f - 1.0f;
}

// True2DTransformer::seeded: weight[i] = deterministic_weight(seed, 0, i) * 0.02.
void owo_true2d_seeded(uint64_t seed, float* weights, size_t count) {
  for (size_t i = 0; i < count; ++i) weights[i] = owo_deterministic_weight(seed, 0, i) * 0.02f;
}

// Batched True2D forward: request r uses model model_indices[r] of
// all_weights (models back to back). Returns 0 ok, 1 bad argument.
int owo_true2d_forward(const float* input_rows, const size_t* model_indices, const float* all_weights,
                       size_t model_count, float* output_rows, size_t request_count, size_t layers,
                       size_t rows, size_t heads, int threads) {
  if (input_rows == nullptr || all_weights == nullptr || output_rows == nullptr || layers == 0 ||
      rows < 2 || heads == 0 || model_count == 0)
    return 1;
  const T2Layout L = layout(layers, rows, heads);
  for (size_t r = 0; r < request_count; ++r)
    if (model_indices != nullptr && model_indices[r] >= model_count) return 1;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
  for (long long r = 0; r < static_cast<long long>(request_count); ++r) {
    const size_t model = model_indices != nullptr ? model_indices[r] : 0;
    forward_one(L, all_weights + model * L.total, input_rows + r * rows * kFeatures,
                output_rows + r * rows * kOutPerRow);
  }
  return 0;
}

// TrainableTransformer::forward (model.rs:210-301). Input per row: 2 features
// (owner_class, ship_log_percent) packed as the reference GPU ABI passes them;
// output per row: 2 values (target, send) -- the reference CPU repeats them
// over 12 targets (ActionOutput::repeated), the GPU ABI writes the pair.
// Weight layout: input_projection[2*d] + position[d] + layer_scales[L*d] + output[2*d]
// (native/cuda/README.md weight_layout).
int owo_trainable_forward(const float* input_rows, const float* weights, float* output_rows,
                          size_t games, size_t layers, size_t d_model, size_t heads, size_t rows) {
  if (input_rows == nullptr || weights == nullptr || output_rows == nullptr || games == 0 ||
      layers == 0 || d_model == 0 || heads == 0 || rows == 0 || d_model % heads != 0)
    return 1;
  const size_t d = d_model, hd = d / heads;
  const float* inp = weights;
  const float* pos = inp + 2 * d;
  const float* scales = pos + d;
  const float* outp = scales + layers * d;
  for (size_t g = 0; g < games; ++g) {
    std::vector<float> hid(rows * d), next(rows * d), scores(rows);
    for (size_t r = 0; r < rows; ++r) {
      const float f0 = input_rows[(g * rows + r) * 2];
      const float f1 = input_rows[(g * rows + r) * 2 + 1];
      const float p = static_cast<float>(r) / static_cast<float>(rows);
      for (size_t k = 0; k < d; ++k) {
        float v = p * pos[k];
        v += f0 * inp[k];
        v += f1 * inp[d + k];
        hid[r * d + k] = std::tanh(v);
      }
    }
    for (size_t l = 0; l < layers; ++l) {
      std::fill(next.begin(), next.end(), 0.0f);
      for (size_t h = 0; h < heads; ++h) {
        const size_t h0 = h * hd;
        for (size_t s = 0; s < rows; ++s) {
          float mx = -std::numeric_limits<float>::infinity();
          for (size_t t = 0; t < rows; ++t) {
            float dot = 0.0f;
            for (size_t c = 0; c < hd; ++c) dot += hid[s * d + h0 + c] * hid[t * d + h0 + c];
            scores[t] = dot / std::sqrt(static_cast<float>(hd));
            mx = std::fmax(mx, scores[t]);
          }
          float den = 0.0f;
          for (size_t t = 0; t < rows; ++t) {
            scores[t] = std::exp(scores[t] - mx);
            den += scores[t];
          }
          for (size_t t = 0; t < rows; ++t) {
            const float a = scores[t] / den;
            for (size_t c = 0; c < hd; ++c) next[s * d + h0 + c] += a * hid[t * d + h0 + c];
          }
        }
      }
      for (size_t r = 0; r < rows; ++r)
        for (size_t k = 0; k < d; ++k)
          hid[r * d + k] = std::tanh(hid[r * d + k] + next[r * d + k] * scales[l * d + k]);
    }
    for (size_t r = 0; r < rows; ++r) {
      // dense_projection(row, output, column, d) = sum_k row[k] * output[column*d+k] / sqrt(d)
      // (model.rs:398-406; GPU output_projection_kernel orbit_wars_cuda.cu:245-272).
      float t0 = 0.0f, t1 = 0.0f;
      for (size_t k = 0; k < d; ++k) {
        t0 += hid[r * d + k] * outp[k];
        t1 += hid[r * d + k] * outp[d + k];
      }
      const float sc = std::sqrt(static_cast<float>(d));
      output_rows[(g * rows + r) * 2] = sigmoidf_(t0 / sc);
      output_rows[(g * rows + r) * 2 + 1] = sigmoidf_(t1 / sc);
    }
  }
  return 0;
}

}  // extern "C"

extern "C" {

// v[i] = sinf((float)(i + 1) * step) * scale: the fixture formula of the
// reference smoke (orbit_wars_cuda_true2d_smoke.cpp:281, :286, :290),
// evaluated with the same C library so golden vectors regenerate exactly.
void owo_sinusoid_fill(float* out, size_t n, float step, float scale) {
  for (size_t i = 0; i < n; ++i) out[i] = std::sin(static_cast<float>(i + 1) * step) * scale;
}

}  // extern "C"
