// CPU oracle for the Orbit Wars entity-encoder policy forward.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker: tests, the smoke entry
// and the bench's CPU-baseline leg call it; the product library never links,
// loads or calls it.
//
// PARITY UNPINNED BY THE REFERENCE: TryDotAtwo/Orbit-Wars-2D-Transformer has
// no implementation of this network (no LayerNorm, GELU FFN, value head,
// key-padding mask, FP8 or Gumbel sampling anywhere in it). The math is the
// frozen encoder-policy spec restated in this file; an independent float64
// numpy restatement (tests/spec_numpy.py) cross-checks it. Conventions that do exist in
// the reference are followed:
//   - scaled, max-subtracted multi-head softmax attention:
//     crates/orbit-wars-core/src/model.rs:247-288
//   - request x rows x features contiguous f32 buffers:
//     crates/orbit-wars-trainer/src/cuda_true2d.rs:469-487
//   - status codes 0/1/2: native/cuda/orbit_wars_cuda.cu:12-14
//
// Three numeric modes: T = double is the "truth" used for parity; T = float is
// the plain fp32 CPU forward timed as the CPU baseline (OpenMP over states,
// weights pre-transposed so the inner loops vectorise); the recipe emulation
// (owo_policy_forward_emulated) is float64 with the bf16 / e4m3 rounding
// points of a precision path applied, which separates what the precision
// recipe itself loses from what a kernel's arithmetic loses. Padded entities
// never reach a valid output, so every mode computes the valid rows only.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <algorithm>
#include <limits>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

typedef struct OwoShape {
  int32_t n_entities;  // N
  int32_t features;    // F
  int32_t d_model;     // d
  int32_t heads;       // h
  int32_t ffn;         // f
  int32_t layers;      // L
  int32_t actions;     // P
} OwoShape;

}  // extern "C"

namespace {

struct Offsets {
  size_t we, be, lnf_g, lnf_b, wp, bp, wv, bv, total;
  struct Layer { size_t ln1g, ln1b, wqkv, bqkv, wo, bo, ln2g, ln2b, w1, b1, w2, b2; };
  std::vector<Layer> layer;
};

// Weight-blob layout: the f32 tensors in the order make_offsets lists them.
Offsets make_offsets(const OwoShape& s) {
  Offsets o;
  const size_t d = s.d_model, F = s.features, f = s.ffn, P = s.actions;
  size_t c = 0;
  o.we = c; c += d * F;
  o.be = c; c += d;
  o.layer.resize(s.layers);
  for (int l = 0; l < s.layers; ++l) {
    auto& L = o.layer[l];
    L.ln1g = c; c += d;
    L.ln1b = c; c += d;
    L.wqkv = c; c += 3 * d * d;
    L.bqkv = c; c += 3 * d;
    L.wo = c; c += d * d;
    L.bo = c; c += d;
    L.ln2g = c; c += d;
    L.ln2b = c; c += d;
    L.w1 = c; c += f * d;
    L.b1 = c; c += f;
    L.w2 = c; c += d * f;
    L.b2 = c; c += d;
  }
  o.lnf_g = c; c += d;
  o.lnf_b = c; c += d;
  o.wp = c; c += P * d;
  o.bp = c; c += P;
  o.wv = c; c += d;
  o.bv = c; c += 1;
  o.total = c;
  return o;
}

bool shape_ok(const OwoShape& s) {
  return s.n_entities > 0 && s.n_entities <= 4096 && s.features > 0 && s.d_model > 0 &&
         s.heads > 0 && s.d_model % s.heads == 0 && s.ffn > 0 && s.layers >= 0 && s.actions > 0;
}

// Transposed copy of W[out,in] -> Wt[in,out] in type T.
template <typename T>
std::vector<T> transpose(const float* w, size_t out, size_t in) {
  std::vector<T> t(out * in);
  for (size_t o = 0; o < out; ++o)
    for (size_t i = 0; i < in; ++i) t[i * out + o] = static_cast<T>(w[o * in + i]);
  return t;
}

template <typename T>
struct Prepared {
  OwoShape s;
  Offsets off;
  const float* w;
  std::vector<T> we_t, wp_t;
  std::vector<std::vector<T>> wqkv_t, wo_t, w1_t, w2_t;
  void init(const OwoShape& shape, const float* weights) {
    s = shape;
    off = make_offsets(shape);
    w = weights;
    const size_t d = s.d_model, F = s.features, f = s.ffn, P = s.actions;
    we_t = transpose<T>(w + off.we, d, F);
    wp_t = transpose<T>(w + off.wp, P, d);
    for (int l = 0; l < s.layers; ++l) {
      const auto& L = off.layer[l];
      wqkv_t.push_back(transpose<T>(w + L.wqkv, 3 * d, d));
      wo_t.push_back(transpose<T>(w + L.wo, d, d));
      w1_t.push_back(transpose<T>(w + L.w1, f, d));
      w2_t.push_back(transpose<T>(w + L.w2, d, f));
    }
  }
};

// y[rows,out] = x[rows,in] * Wt[in,out] + b
template <typename T>
void linear(const T* x, size_t rows, size_t in, const T* wt, size_t out, const float* b, T* y) {
  for (size_t r = 0; r < rows; ++r) {
    T* yr = y + r * out;
    for (size_t o = 0; o < out; ++o) yr[o] = static_cast<T>(b[o]);
    const T* xr = x + r * in;
    for (size_t i = 0; i < in; ++i) {
      const T xi = xr[i];
      const T* wrow = wt + i * out;
      for (size_t o = 0; o < out; ++o) yr[o] += xi * wrow[o];
    }
  }
}

template <typename T>
void layer_norm(const T* x, size_t rows, size_t d, const float* g, const float* b, T* y) {
  for (size_t r = 0; r < rows; ++r) {
    const T* xr = x + r * d;
    T mean = 0;
    for (size_t i = 0; i < d; ++i) mean += xr[i];
    mean /= static_cast<T>(d);
    T var = 0;
    for (size_t i = 0; i < d; ++i) {
      const T c = xr[i] - mean;
      var += c * c;
    }
    var /= static_cast<T>(d);
    const T inv = static_cast<T>(1) / std::sqrt(var + static_cast<T>(1e-5));
    T* yr = y + r * d;
    for (size_t i = 0; i < d; ++i) yr[i] = (xr[i] - mean) * inv * static_cast<T>(g[i]) + static_cast<T>(b[i]);
  }
}

template <typename T>
T gelu(T v) {
  return static_cast<T>(0.5) * v * (static_cast<T>(1) + std::erf(v * static_cast<T>(0.70710678118654752440)));
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
// as 1, 2, 3", SC'11), written from the paper's round definition.
void philox4x32_10(uint32_t ctr[4], uint32_t k0, uint32_t k1) {
  for (int round = 0; round < 10; ++round) {
    if (round > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * ctr[0];
    const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * ctr[2];
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    const uint32_t n0 = hi1 ^ ctr[1] ^ k0;
    const uint32_t n2 = hi0 ^ ctr[3] ^ k1;
    ctr[0] = n0;
    ctr[1] = lo1;
    ctr[2] = n2;
    ctr[3] = lo0;
  }
}

double gumbel_noise(uint64_t seed, uint32_t state, uint32_t entity, uint32_t action) {
  uint32_t c[4] = {action / 4u, entity, state, 0u};
  philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  const double u = (static_cast<double>(c[action % 4u]) + 0.5) * (1.0 / 4294967296.0);
  return -std::log(-std::log(u));
}

// One state's forward. Scratch vectors are per thread.
template <typename T>
void forward_state(const Prepared<T>& p, const float* feat, int count, size_t state_index,
                   int sample, uint64_t seed, float* logits, float* value, int32_t* actions,
                   std::vector<T>& x, std::vector<T>& a, std::vector<T>& qkv, std::vector<T>& o,
                   std::vector<T>& t, std::vector<T>& h, std::vector<T>& scores) {
  const OwoShape& s = p.s;
  const size_t N = s.n_entities, F = s.features, d = s.d_model, f = s.ffn, P = s.actions;
  const size_t H = s.heads, hd = d / H;
  const float* w = p.w;
  // padded entities (j >= count) never reach a valid output: only the valid rows are computed
  const size_t Nv = static_cast<size_t>(std::max(count, 0));
  // embedding
  std::vector<T> ft(N * F);
  for (size_t i = 0; i < N * F; ++i) ft[i] = static_cast<T>(feat[i]);
  linear<T>(ft.data(), Nv, F, p.we_t.data(), d, w + p.off.be, x.data());
  const T scale = static_cast<T>(1) / std::sqrt(static_cast<T>(hd));
  for (int l = 0; l < s.layers; ++l) {
    const auto& L = p.off.layer[l];
    layer_norm<T>(x.data(), Nv, d, w + L.ln1g, w + L.ln1b, a.data());
    linear<T>(a.data(), Nv, d, p.wqkv_t[l].data(), 3 * d, w + L.bqkv, qkv.data());
    // masked multi-head attention (keys j >= count masked)
    std::fill(o.begin(), o.end(), static_cast<T>(0));
    for (size_t hh = 0; hh < H; ++hh) {
      const size_t qo = hh * hd, ko = d + hh * hd, vo = 2 * d + hh * hd;
      for (size_t i = 0; i < Nv; ++i) {
        T mx = -std::numeric_limits<T>::infinity();
        for (int j = 0; j < count; ++j) {
          T dot = 0;
          for (size_t c = 0; c < hd; ++c) dot += qkv[i * 3 * d + qo + c] * qkv[j * 3 * d + ko + c];
          scores[j] = dot * scale;
          mx = std::max(mx, scores[j]);
        }
        T den = 0;
        for (int j = 0; j < count; ++j) {
          scores[j] = std::exp(scores[j] - mx);
          den += scores[j];
        }
        const T inv = static_cast<T>(1) / den;
        for (int j = 0; j < count; ++j) {
          const T pj = scores[j] * inv;
          for (size_t c = 0; c < hd; ++c) o[i * d + qo + c] += pj * qkv[j * 3 * d + vo + c];
        }
      }
    }
    linear<T>(o.data(), Nv, d, p.wo_t[l].data(), d, w + L.bo, t.data());
    for (size_t i = 0; i < Nv * d; ++i) x[i] += t[i];
    layer_norm<T>(x.data(), Nv, d, w + L.ln2g, w + L.ln2b, a.data());
    linear<T>(a.data(), Nv, d, p.w1_t[l].data(), f, w + L.b1, h.data());
    for (size_t i = 0; i < Nv * f; ++i) h[i] = gelu<T>(h[i]);
    linear<T>(h.data(), Nv, f, p.w2_t[l].data(), d, w + L.b2, t.data());
    for (size_t i = 0; i < Nv * d; ++i) x[i] += t[i];
  }
  layer_norm<T>(x.data(), Nv, d, w + p.off.lnf_g, w + p.off.lnf_b, a.data());
  // policy head on valid entities; padded entities are exactly 0 / -1
  std::vector<T> lg(P);
  for (size_t j = 0; j < N; ++j) {
    float* out = logits + j * P;
    if (static_cast<int>(j) >= count) {
      for (size_t q = 0; q < P; ++q) out[q] = 0.0f;
      actions[j] = -1;
      continue;
    }
    linear<T>(a.data() + j * d, 1, d, p.wp_t.data(), P, w + p.off.bp, lg.data());
    int best = 0;
    double best_v = -std::numeric_limits<double>::infinity();
    for (size_t q = 0; q < P; ++q) {
      out[q] = static_cast<float>(lg[q]);
      double score = static_cast<double>(lg[q]);
      if (sample) score += gumbel_noise(seed, static_cast<uint32_t>(state_index), static_cast<uint32_t>(j), static_cast<uint32_t>(q));
      if (score > best_v) {
        best_v = score;
        best = static_cast<int>(q);
      }
    }
    actions[j] = best;
  }
  // value head on the mean of valid entities
  T v = static_cast<T>(w[p.off.bv]);
  if (count > 0) {
    for (size_t c = 0; c < d; ++c) {
      T m = 0;
      for (int j = 0; j < count; ++j) m += a[j * d + c];
      m /= static_cast<T>(count);
      v += m * static_cast<T>(w[p.off.wv + c]);
    }
  }
  *value = static_cast<float>(v);
}

// ---------------------------------------------------------------- recipe emulation
// Float64 forward that rounds at the points where the bf16 / fp8 paths store
// a tensor in a narrow type, so that "the recipe's own error" (what any exact
// implementation of the precision recipe loses against the float64 truth) is
// measured apart from the kernels' arithmetic error. Rounding points:
//   kStoreBf16    features, QKV, softmax P, attention output, GELU output,
//                 bf16 LayerNorm outputs, logits (and value on the fp8 path)
//   kResidBf16    the residual stream between residual adds (the d = 256
//                 tensor-core paths keep it in bf16)
//   kQuantQkv .. kQuantDown  e4m3 operands of one block GEMM: per-token scale
//                 s = absmax/448 (1 for an all-zero row), q = e4m3(v/s) RNE
//                 saturating, the GEMM sums q_a*q_w*s_a*s_w exactly
// The weight blob is used as given (pass matrices already on the bf16 or
// per-channel e4m3 grid to exclude weight quantisation).
enum : unsigned {
  kStoreBf16 = 1u,
  kQuantQkv = 2u,
  kQuantOut = 4u,
  kQuantUp = 8u,
  kQuantDown = 16u,
  kValueBf16 = 32u,
  kResidBf16 = 64u,  // the residual stream is kept in bf16 between the residual adds
};

double round_bf16(double v) {
  float f = static_cast<float>(v);
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return f;  // inf / nan unchanged
  u += 0x7FFFu + ((u >> 16) & 1u);                  // round to nearest even on the upper 16 bits
  u &= 0xFFFF0000u;
  std::memcpy(&f, &u, 4);
  return f;
}

// e4m3 ("fn": no infinities, max 448, min normal 2^-6, subnormal step 2^-9),
// round to nearest even, saturating to +-448.
float round_e4m3(float v) {
  if (!(v == v)) return v;
  const float a = std::fabs(v);
  if (a == 0.0f) return v;
  float q;
  if (a >= 448.0f) {
    q = 448.0f;
  } else {
    int e;
    std::frexp(a, &e);          // a = m * 2^e, m in [0.5, 1): the binade's step is 2^(e-4)
    const int step_exp = std::max(e - 4, -9);
    const double scaled = std::ldexp(static_cast<double>(a), -step_exp);
    q = static_cast<float>(std::ldexp(std::nearbyint(scaled), step_exp));  // FE_TONEAREST: ties to even
    if (q > 448.0f) q = 448.0f;
  }
  return v < 0 ? -q : q;
}

// Per-token e4m3 operand: v -> q*s with s = absmax/448 computed in f32 like the kernels.
void quantize_rows(std::vector<double>& v, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; ++r) {
    double* row = v.data() + r * cols;
    float amax = 0.0f;
    for (size_t c = 0; c < cols; ++c) amax = std::max(amax, std::fabs(static_cast<float>(row[c])));
    const float s = amax > 0.0f ? amax * (1.0f / 448.0f) : 1.0f;
    const float inv = 1.0f / s;
    for (size_t c = 0; c < cols; ++c)
      row[c] = static_cast<double>(round_e4m3(static_cast<float>(row[c]) * inv)) * static_cast<double>(s);
  }
}

void round_all_bf16(std::vector<double>& v, size_t n) {
  for (size_t i = 0; i < n; ++i) v[i] = round_bf16(v[i]);
}

void forward_state_emu(const Prepared<double>& p, unsigned mode, const float* feat, int count, float* logits,
                       float* value, int32_t* actions) {
  const OwoShape& s = p.s;
  const size_t N = s.n_entities, F = s.features, d = s.d_model, f = s.ffn, P = s.actions;
  const size_t H = s.heads, hd = d / H;
  const float* w = p.w;
  const bool bf = (mode & kStoreBf16) != 0;
  const size_t Nv = static_cast<size_t>(std::max(count, 0));  // padded rows never reach a valid output
  std::vector<double> x(N * d), a(N * d), qkv(N * 3 * d), o(N * d), t(N * d), h(N * f), scores(N);
  std::vector<double> ft(N * F);
  for (size_t i = 0; i < N * F; ++i) ft[i] = bf ? round_bf16(feat[i]) : feat[i];
  linear<double>(ft.data(), Nv, F, p.we_t.data(), d, w + p.off.be, x.data());
  // The kernels form each residual sum in f32 (mode 0 is the plain float64
  // forward) and take its LayerNorm from that sum; the stream then keeps it in
  // f32, or in bf16 (kResidBf16), for the next residual add.
  auto sum_x = [&](double v) { return mode != 0 ? static_cast<double>(static_cast<float>(v)) : v; };
  auto keep_x = [&]() {
    if (mode & kResidBf16) round_all_bf16(x, Nv * d);
  };
  for (size_t i = 0; i < Nv * d; ++i) x[i] = sum_x(x[i]);
  auto ln_out = [&](const float* g, const float* b, bool quant) {
    layer_norm<double>(x.data(), Nv, d, g, b, a.data());
    if (quant) quantize_rows(a, Nv, d);
    else if (bf) round_all_bf16(a, Nv * d);
  };
  const double scale = 1.0 / std::sqrt(static_cast<double>(hd));
  if (s.layers > 0) {
    ln_out(w + p.off.layer[0].ln1g, w + p.off.layer[0].ln1b, (mode & kQuantQkv) != 0);
    keep_x();
  }
  for (int l = 0; l < s.layers; ++l) {
    const auto& L = p.off.layer[l];
    linear<double>(a.data(), Nv, d, p.wqkv_t[l].data(), 3 * d, w + L.bqkv, qkv.data());
    if (bf) round_all_bf16(qkv, Nv * 3 * d);
    std::fill(o.begin(), o.end(), 0.0);
    for (size_t hh = 0; hh < H && count > 0; ++hh) {
      const size_t qo = hh * hd, ko = d + hh * hd, vo = 2 * d + hh * hd;
      for (size_t i = 0; i < Nv; ++i) {
        double mx = -std::numeric_limits<double>::infinity();
        for (int j = 0; j < count; ++j) {
          double dot = 0;
          for (size_t c = 0; c < hd; ++c) dot += qkv[i * 3 * d + qo + c] * qkv[j * 3 * d + ko + c];
          scores[j] = dot * scale;
          mx = std::max(mx, scores[j]);
        }
        double den = 0;
        for (int j = 0; j < count; ++j) {
          scores[j] = std::exp(scores[j] - mx);
          den += scores[j];
          if (bf) scores[j] = round_bf16(scores[j]);  // P enters the PV product as bf16; the sum does not
        }
        for (int j = 0; j < count; ++j)
          for (size_t c = 0; c < hd; ++c) o[i * d + qo + c] += scores[j] * qkv[j * 3 * d + vo + c];
        for (size_t c = 0; c < hd; ++c) o[i * d + qo + c] /= den;
      }
    }
    if (bf) round_all_bf16(o, Nv * d);
    if (mode & kQuantOut) quantize_rows(o, Nv, d);
    linear<double>(o.data(), Nv, d, p.wo_t[l].data(), d, w + L.bo, t.data());
    for (size_t i = 0; i < Nv * d; ++i) x[i] = sum_x(x[i] + t[i]);
    ln_out(w + L.ln2g, w + L.ln2b, (mode & kQuantUp) != 0);
    keep_x();
    linear<double>(a.data(), Nv, d, p.w1_t[l].data(), f, w + L.b1, h.data());
    for (size_t i = 0; i < Nv * f; ++i) h[i] = gelu<double>(h[i]);
    if (bf) round_all_bf16(h, Nv * f);
    if (mode & kQuantDown) quantize_rows(h, Nv, f);
    linear<double>(h.data(), Nv, f, p.w2_t[l].data(), d, w + L.b2, t.data());
    for (size_t i = 0; i < Nv * d; ++i) x[i] = sum_x(x[i] + t[i]);
    if (l + 1 < s.layers) {
      ln_out(w + p.off.layer[l + 1].ln1g, w + p.off.layer[l + 1].ln1b, (mode & kQuantQkv) != 0);
      keep_x();
    } else {
      // final LN stays f32 (heads read y in f32)
      layer_norm<double>(x.data(), Nv, d, w + p.off.lnf_g, w + p.off.lnf_b, a.data());
    }
  }
  if (s.layers == 0) layer_norm<double>(x.data(), Nv, d, w + p.off.lnf_g, w + p.off.lnf_b, a.data());
  std::vector<double> lg(P);
  for (size_t j = 0; j < N; ++j) {
    float* out = logits + j * P;
    if (static_cast<int>(j) >= count) {
      for (size_t q = 0; q < P; ++q) out[q] = 0.0f;
      actions[j] = -1;
      continue;
    }
    linear<double>(a.data() + j * d, 1, d, p.wp_t.data(), P, w + p.off.bp, lg.data());
    int best = 0;
    double best_v = -std::numeric_limits<double>::infinity();
    for (size_t q = 0; q < P; ++q) {
      const double v = bf ? round_bf16(lg[q]) : lg[q];
      out[q] = static_cast<float>(v);
      if (v > best_v) {
        best_v = v;
        best = static_cast<int>(q);
      }
    }
    actions[j] = best;
  }
  double v = w[p.off.bv];
  if (count > 0) {
    for (size_t c = 0; c < d; ++c) {
      double m = 0;
      for (int j = 0; j < count; ++j) m += a[j * d + c];
      v += (m / count) * static_cast<double>(w[p.off.wv + c]);
    }
  }
  *value = static_cast<float>((mode & kValueBf16) ? round_bf16(v) : v);
}

template <typename T>
int run(const OwoShape* shape, const float* weights, size_t n_weights, const float* features,
        const int32_t* counts, int32_t batch, int threads, int sample, uint64_t seed,
        float* logits, float* value, int32_t* actions) {
  if (shape == nullptr || weights == nullptr || features == nullptr || counts == nullptr ||
      logits == nullptr || value == nullptr || actions == nullptr || batch < 0)
    return 1;
  if (!shape_ok(*shape)) return 1;
  Prepared<T> p;
  p.init(*shape, weights);
  if (n_weights != p.off.total) return 1;
  const size_t N = shape->n_entities, F = shape->features, d = shape->d_model, f = shape->ffn,
               P = shape->actions;
  for (int32_t b = 0; b < batch; ++b)
    if (counts[b] < 0 || counts[b] > shape->n_entities) return 1;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
  {
    std::vector<T> x(N * d), a(N * d), qkv(N * 3 * d), o(N * d), t(N * d), h(N * f), scores(N);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int32_t b = 0; b < batch; ++b) {
      forward_state<T>(p, features + static_cast<size_t>(b) * N * F, counts[b], static_cast<size_t>(b),
                       sample, seed, logits + static_cast<size_t>(b) * N * P, value + b,
                       actions + static_cast<size_t>(b) * N, x, a, qkv, o, t, h, scores);
    }
  }
  return 0;
}

}  // namespace

extern "C" {

size_t owo_policy_weight_count(const OwoShape* shape) {
  if (shape == nullptr || !shape_ok(*shape)) return 0;
  return make_offsets(*shape).total;
}

// Forward of `batch` states. accumulate_f64 != 0 selects the float64 truth
// mode, else plain fp32. threads <= 0 leaves the OpenMP default (all cores).
// sample != 0 selects Gumbel-max actions keyed by `seed`. Returns 0 on success,
// 1 on a bad argument.
int owo_policy_forward(const OwoShape* shape, const float* weights, size_t n_weights,
                       const float* features, const int32_t* counts, int32_t batch,
                       int accumulate_f64, int threads, int sample, uint64_t seed,
                       float* logits, float* value, int32_t* actions) {
  if (accumulate_f64)
    return run<double>(shape, weights, n_weights, features, counts, batch, threads, sample, seed,
                       logits, value, actions);
  return run<float>(shape, weights, n_weights, features, counts, batch, threads, sample, seed,
                    logits, value, actions);
}

// Float64 forward with the precision recipe's rounding points applied (mode:
// the kStoreBf16 / kQuant* / kValueBf16 bits above). Greedy actions only.
// Returns 0 on success, 1 on a bad argument.
int owo_policy_forward_emulated(const OwoShape* shape, const float* weights, size_t n_weights,
                                const float* features, const int32_t* counts, int32_t batch, unsigned mode,
                                int threads, float* logits, float* value, int32_t* actions) {
  if (shape == nullptr || weights == nullptr || features == nullptr || counts == nullptr ||
      logits == nullptr || value == nullptr || actions == nullptr || batch < 0 || !shape_ok(*shape))
    return 1;
  Prepared<double> p;
  p.init(*shape, weights);
  if (n_weights != p.off.total) return 1;
  for (int32_t b = 0; b < batch; ++b)
    if (counts[b] < 0 || counts[b] > shape->n_entities) return 1;
  const size_t N = shape->n_entities, F = shape->features, P = shape->actions;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
  for (int32_t b = 0; b < batch; ++b)
    forward_state_emu(p, mode, features + static_cast<size_t>(b) * N * F, counts[b],
                      logits + static_cast<size_t>(b) * N * P, value + b, actions + static_cast<size_t>(b) * N);
  return 0;
}

// Gumbel-max actions from given logits (the GPU's own): actions[b,j] =
// argmax_p(logits[b,j,p] + G(seed, state_base + b, j, p)) for j < counts[b],
// -1 otherwise; gap[b,j] = the top-two score difference (ties that a rounding
// may flip have a small gap). Returns 0, or 1 on a bad argument.
int owo_gumbel_argmax(const float* logits, const int32_t* counts, int32_t batch, int32_t n_entities,
                      int32_t n_actions, uint64_t seed, uint32_t state_base, int threads, int32_t* actions,
                      float* gap) {
  if (logits == nullptr || counts == nullptr || actions == nullptr || gap == nullptr || batch < 0 ||
      n_entities <= 0 || n_actions <= 0)
    return 1;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
  for (int32_t b = 0; b < batch; ++b) {
    for (int32_t j = 0; j < n_entities; ++j) {
      const size_t row = static_cast<size_t>(b) * n_entities + j;
      if (j >= counts[b]) {
        actions[row] = -1;
        gap[row] = INFINITY;
        continue;
      }
      double best = -INFINITY, second = -INFINITY;
      int arg = 0;
      for (int32_t p = 0; p < n_actions; ++p) {
        const double s = static_cast<double>(logits[row * n_actions + p]) +
                         gumbel_noise(seed, state_base + static_cast<uint32_t>(b), static_cast<uint32_t>(j),
                                      static_cast<uint32_t>(p));
        if (s > best) {
          second = best;
          best = s;
          arg = p;
        } else if (s > second) {
          second = s;
        }
      }
      actions[row] = arg;
      gap[row] = static_cast<float>(best - second);
    }
  }
  return 0;
}

// e4m3 rounding of one f32 value (for known-answer tests of the emulation).
float owo_round_e4m3(float v) { return round_e4m3(v); }

// Gumbel noise G for (seed, state, entity, action) as the spec defines it.
double owo_gumbel(uint64_t seed, uint32_t state, uint32_t entity, uint32_t action) {
  return gumbel_noise(seed, state, entity, action);
}

// Raw Philox4x32-10 block for known-answer tests.
void owo_philox4x32_10(const uint32_t counter[4], uint32_t k0, uint32_t k1, uint32_t out[4]) {
  uint32_t c[4] = {counter[0], counter[1], counter[2], counter[3]};
  philox4x32_10(c, k0, k1);
  for (int i = 0; i < 4; ++i) out[i] = c[i];
}

int owo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
