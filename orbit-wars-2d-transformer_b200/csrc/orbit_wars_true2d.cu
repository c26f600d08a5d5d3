// sm_100a implementation of the reference engine's GPU ABI
// (include/orbit_wars_cuda.h): the True2D self-play policy forward, the
// legacy TrainableTransformer forward and the identity copy.
//
// True2D forward per request (true2d_model.rs:197-283), three stages:
//   1. t2_expand_pre:  thread per (request, cell): expand (true2d_model.rs:321-366)
//                      then the pre-attention matrix layers (:419-461) with the
//                      cell value held in a register; weights of request r's
//                      model streamed from L2/HBM (12 floats per layer per cell,
//                      three 16-byte loads); tanh as one ex2.approx with the
//                      reciprocal on the FMA pipe, the gate's sigmoid as one
//                      ex2.approx and one rcp.approx.
//   2. attention (:463-544), CTA per request, attention FFN fused:
//      t2_attention_moments: the scores are rank one, so each query's softmax-
//                      weighted mean of the cell values follows from the
//                      request's Chebyshev moments and the query's modified
//                      Bessel values (O(cells x P) instead of cells^2 exponentials);
//      t2_attention:   one pass over keys in shared memory with the exact
//                      closed-form row max, for the requests the first kernel
//                      leaves (very large attention weights, over 4,096 cells).
//   3. t2_post_collapse: CTA per 4 rows of a request: post-attention matrix layers,
//                      then the 12-action collapse (:546-647), a thread per
//                      (row, action), from shared memory.
// The model population stays resident in HBM between calls (upload_population);
// all buffers live in one process-global workspace like the reference's
// (orbit_wars_cuda.cu:421-441), guarded by a mutex.

#include "orbit_wars_cuda.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <pthread.h>
#include <thread>
#include <vector>

#include "ow_common.cuh"
#include "ow_encode.cuh"

namespace {

constexpr int kOk = 0, kBad = 1, kRt = 2;  // orbit_wars_cuda.cu:12-14
constexpr size_t kFeatures = 7;
constexpr size_t kTargets = 12;
constexpr size_t kOutPerRow = 24;
constexpr size_t kCellWeights = 12;
constexpr size_t kHeadWeights = 7;
constexpr size_t kSharedWeights = 6;
constexpr size_t kOutScalars = 5;
constexpr size_t kMinRows = 2, kMaxRows = 128, kMaxHeads = 16;

OrbitWarsCudaStatus ok() { return {kOk, "ok"}; }
OrbitWarsCudaStatus bad(const char* m) { return {kBad, m}; }
OrbitWarsCudaStatus rt(const char* m) { return {kRt, m}; }
OrbitWarsCudaStatus from_cuda(cudaError_t e) { return e == cudaSuccess ? ok() : rt(cudaGetErrorString(e)); }

#define T2_TRY(expr)                               \
  do {                                             \
    const cudaError_t e_ = (expr);                 \
    if (e_ != cudaSuccess) return from_cuda(e_);   \
  } while (0)

struct T2Layout {
  size_t rows, cells, layers, heads;
  size_t pair, src_emb, tgt_emb, pair_emb, bias, matrix, attn, tbias, sbias, scalars, total;
};

// Weight-vector layout, true2d_model.rs:111-126 (order of the slices in :216-246).
T2Layout t2_layout(size_t layers, size_t rows, size_t heads) {
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

bool shape_ok(const OrbitWarsCudaTrue2DShape& s) {
  return s.layer_count > 0 && s.row_count >= kMinRows && s.row_count <= kMaxRows && s.head_count >= 1 &&
         s.head_count <= kMaxHeads;
}

// Device-side view of the layout (passed by value).
struct T2Dev {
  int rows, cells, layers, heads, mid;
  long long pair, src_emb, tgt_emb, pair_emb, bias, matrix, attn, tbias, sbias, scalars, total;
};

// Device copy of a model: the host layout with `pad` floats inserted before
// the matrix-layer section so each cell's 12 weights start on a 16-byte
// boundary (host offset 4239 for 64 rows is not), and the model stride
// rounded up to 4 floats.
size_t matrix_pad(const T2Layout& L) { return (4 - L.matrix % 4) % 4; }
size_t dev_total(const T2Layout& L) { return (L.total + matrix_pad(L) + 3) / 4 * 4; }

T2Dev dev_layout(const T2Layout& L) {
  T2Dev d{};
  const long long pad = static_cast<long long>(matrix_pad(L));
  d.rows = static_cast<int>(L.rows);
  d.cells = static_cast<int>(L.cells);
  d.layers = static_cast<int>(L.layers);
  d.heads = static_cast<int>(L.heads);
  d.mid = static_cast<int>(L.layers / 2);  // attention_layer_index, true2d_model.rs:128-130
  d.pair = L.pair; d.src_emb = L.src_emb; d.tgt_emb = L.tgt_emb; d.pair_emb = L.pair_emb; d.bias = L.bias;
  d.matrix = L.matrix + pad; d.attn = L.attn + pad; d.tbias = L.tbias + pad; d.sbias = L.sbias + pad;
  d.scalars = L.scalars + pad;
  d.total = static_cast<long long>(dev_total(L));
  return d;
}

__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

// One gated per-cell matrix layer, true2d_model.rs:419-461. VEC: the 12
// weights are 16-byte aligned (padded device layout) and read as three float4;
// otherwise (the reference's own layout) as scalars.
template <bool VEC>
__device__ __forceinline__ void load_cell_weights(const float* __restrict__ w12, float4& a, float4& b, float4& c) {
  if (VEC) {
    a = __ldg(reinterpret_cast<const float4*>(w12));
    b = __ldg(reinterpret_cast<const float4*>(w12) + 1);
    c = __ldg(reinterpret_cast<const float4*>(w12) + 2);
  } else {
    a = make_float4(__ldg(w12), __ldg(w12 + 1), __ldg(w12 + 2), __ldg(w12 + 3));
    b = make_float4(__ldg(w12 + 4), __ldg(w12 + 5), __ldg(w12 + 6), __ldg(w12 + 7));
    c = make_float4(__ldg(w12 + 8), __ldg(w12 + 9), __ldg(w12 + 10), __ldg(w12 + 11));
  }
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// tanh for the matrix layers, written from tanh|x| = 2 / (1 + e^(-2|x|)) - 1:
// one ex2.approx, and the reciprocal of d = 1 + e^(-2|x|) in [1, 2] on the FMA
// pipe, a quadratic fitted here by least squares for relative error on [1, 2]
// (1.2%) and then two Newton steps y += y (1 - d y) (1.1e-7). Absolute error a
// few 1e-7 everywhere; relative error grows as x -> 0 (the form cancels), which
// the matrix layers tolerate: their tanh values enter weighted sums and the
// next layer's affine maps, where absolute error is what carries. A Taylor
// branch for |x| < 1/4 on the cell's own tanh measured 5% slower and left the
// outputs where they were (3.3e-7 from the reference build).
__device__ __forceinline__ float tanh_cell(float x) {
  const float d = 1.0f + ex2_approx(fabsf(x) * (-2.0f * 1.4426950408889634f));
  float y = fmaf(fmaf(0.31368835f, d, -1.4250640f), d, 2.0995536f);
  y = fmaf(y, fmaf(-d, y, 1.0f), y);
  y = fmaf(y, fmaf(-d, y, 1.0f), y);
  return copysignf(fmaf(2.0f, y, -1.0f), x);
}

// logistic sigmoid 1 / (1 + e^-z) for the matrix layers' gate: one ex2.approx and one rcp.approx
__device__ __forceinline__ float sigmoid_cell(float z) {
  return rcp_approx(1.0f + ex2_approx(z * -1.4426950408889634f));
}

// a = (w0,w1,w2,w3) b = (w4,w5,w6,w7) c = (w8,w9,w10,w11)
__device__ __forceinline__ float matrix_cell_w(float v, const float4 a, const float4 b, const float4 c) {
  const float ha = tanh_cell(fmaf(v, a.z, a.w));
  const float hb = tanh_cell(fmaf(v, b.x, fmaf(ha, b.y, b.z)));
  const float g = sigmoid_cell(fmaf(v, b.w, c.x));
  const float u = fmaf(hb, c.y, fmaf(ha, c.z, c.w));
  const float r = fmaf(v, 1.0f + a.x, a.y);
  return tanh_cell(fmaf(g, u, r));
}

// The same cell for two requests of one model at once (the grouped kernels'
// request pairs): every FP32 step of tanh_cell, sigmoid_cell and
// matrix_cell_w as one packed f32x2 instruction, whose lanes round exactly as
// the scalar instruction does, so each lane's result is bit-identical to
// matrix_cell_w and a pair takes about half the issue slots (the MUFU
// operations stay scalar). The tanh keeps -d = -(1 + e) instead of d: round to
// nearest is symmetric, so -(1 + e) rounds to exactly the negated sum, and the
// quadratic's and the Newton steps' signs are turned to match, product for
// product.
__device__ __forceinline__ float2 f2s(float s) { return make_float2(s, s); }

__device__ __forceinline__ float2 tanh_cell2(float2 x) {
  const float2 t = ow::mul_f2(x, f2s(2.0f * 1.4426950408889634f));
  const float2 e = make_float2(ex2_approx(-fabsf(t.x)), ex2_approx(-fabsf(t.y)));
  const float2 nd = ow::sub_f2(f2s(-1.0f), e);
  float2 y = ow::fma_f2(ow::fma_f2(f2s(0.31368835f), nd, f2s(1.4250640f)), nd, f2s(2.0995536f));
  y = ow::fma_f2(y, ow::fma_f2(nd, y, f2s(1.0f)), y);
  y = ow::fma_f2(y, ow::fma_f2(nd, y, f2s(1.0f)), y);
  const float2 r = ow::fma_f2(f2s(2.0f), y, f2s(-1.0f));
  return make_float2(copysignf(r.x, x.x), copysignf(r.y, x.y));
}

__device__ __forceinline__ float2 sigmoid_cell2(float2 z) {
  const float2 t = ow::mul_f2(z, f2s(-1.4426950408889634f));
  const float2 d = ow::add_f2(f2s(1.0f), make_float2(ex2_approx(t.x), ex2_approx(t.y)));
  return make_float2(rcp_approx(d.x), rcp_approx(d.y));
}

__device__ __forceinline__ float2 matrix_cell_w2(float2 v, const float4 a, const float4 b, const float4 c) {
  const float2 ha = tanh_cell2(ow::fma_f2(v, f2s(a.z), f2s(a.w)));
  const float2 hb = tanh_cell2(ow::fma_f2(v, f2s(b.x), ow::fma_f2(ha, f2s(b.y), f2s(b.z))));
  const float2 g = sigmoid_cell2(ow::fma_f2(v, f2s(b.w), f2s(c.x)));
  const float2 u = ow::fma_f2(hb, f2s(c.y), ow::fma_f2(ha, f2s(c.z), f2s(c.w)));
  const float2 r = ow::fma_f2(v, f2s(1.0f + a.x), f2s(a.y));
  return tanh_cell2(ow::fma_f2(g, u, r));
}

template <bool VEC>
__device__ __forceinline__ float matrix_cell(float v, const float* __restrict__ w12) {
  float4 a, b, c;
  load_cell_weights<VEC>(w12, a, b, c);
  return matrix_cell_w(v, a, b, c);
}

__device__ __forceinline__ const float* model_of(const float* __restrict__ all_w, const size_t* __restrict__ idx,
                                                 int models, int r, long long total, int* err) {
  size_t m = idx != nullptr ? idx[r] : 0;
  if (m >= static_cast<size_t>(models)) {
    ow::record_error(err, ow::kErrBadModelIndex);
    m = 0;
  }
  return all_w + static_cast<long long>(m) * total;
}

// 1. expand + matrix layers [0, mid)
template <bool VEC>
__global__ void __launch_bounds__(256) t2_expand_pre(const float* __restrict__ x, const size_t* __restrict__ idx,
                                                     const float* __restrict__ all_w, int models, T2Dev L,
                                                     float* __restrict__ m, int* err) {
  const int r = blockIdx.y;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= L.cells) return;
  const float* w = model_of(all_w, idx, models, r, L.total, err);
  const int s = cell / L.rows, t = cell % L.rows;
  const float* xs = x + (static_cast<long long>(r) * L.rows + s) * kFeatures;
  const float* xt = x + (static_cast<long long>(r) * L.rows + t) * kFeatures;
  const float* pw = w + L.pair;
  float v = 0.0f;
#pragma unroll
  for (int f = 0; f < static_cast<int>(kFeatures); ++f) v = fmaf(xs[f], pw[f], v);
#pragma unroll
  for (int f = 0; f < static_cast<int>(kFeatures); ++f) v = fmaf(xt[f], pw[kFeatures + f], v);
  v += w[L.src_emb + s] + w[L.tgt_emb + t] + w[L.pair_emb + cell] + w[L.bias];
  v = tanhf(v);
  const float* mw = w + L.matrix + static_cast<long long>(cell) * kCellWeights;
  const long long per_layer = static_cast<long long>(L.cells) * kCellWeights;
  for (int l = 0; l < L.mid; ++l) v = matrix_cell<VEC>(v, mw + l * per_layer);
  m[static_cast<long long>(r) * L.cells + cell] = v;
}

// ---- collapse (true2d_model.rs:546-647) of one (row, action) by one thread
// Row stride of the collapse's shared arrays: one float of padding so that
// lanes reading the same column t of different rows hit different banks.
constexpr int kRowStride = kMaxRows + 1;

// Stages target_bias and send_bias of a model, times log2 e, into
// s_bias[2][kTargets][kRowStride] (callers synchronise before reading).
__device__ __forceinline__ void stage_collapse_bias(const float* __restrict__ w, const T2Dev& L, float* s_bias) {
  const float kLog2e = 1.4426950408889634f;
  for (int i = threadIdx.x; i < 2 * static_cast<int>(kTargets) * L.rows; i += blockDim.x) {
    const int which = i / (static_cast<int>(kTargets) * L.rows), rest = i % (static_cast<int>(kTargets) * L.rows);
    const int a = rest / L.rows, t = rest % L.rows;
    const float b = which == 0 ? w[L.tbias + rest] : w[L.sbias + rest];
    s_bias[(which * kTargets + a) * kRowStride + t] = b * kLog2e;
  }
}

// Action a of one row (row values mrow[0..rows), shared memory): the target
// softmax over rows of m_t * s0 + tb[a][t] gives the expected target index
// / (rows - 1), clamped to [0, 1] (frac); the send softmax of m_t * s1 + sb[a][t]
// weights the row values, and sigmoid((weighted * s2 + s4) * s3) is the send
// fraction before the row's normalisation (send). Scores are formed in log2
// units (biases staged times log2 e, one FMA each), so each exponential is one
// ex2.approx; a pass for the two maxima, then one for the four sums.
__device__ __forceinline__ void collapse_item(const float* mrow, const float* s_bias, int a, int rows,
                                              const float* __restrict__ sc, float& frac, float& send) {
  const float kLog2e = 1.4426950408889634f;
  const float* tb = s_bias + a * kRowStride;
  const float* sb = s_bias + (kTargets + a) * kRowStride;
  const float s0 = sc[0] * kLog2e, s1 = sc[1] * kLog2e;
  float tmax = -INFINITY, smax = -INFINITY;
  for (int t = 0; t < rows; ++t) {
    const float v = mrow[t];
    tmax = fmaxf(tmax, fmaf(v, s0, tb[t]));
    smax = fmaxf(smax, fmaf(v, s1, sb[t]));
  }
  float tden = 0.0f, tnum = 0.0f, sden = 0.0f, snum = 0.0f;
  for (int t = 0; t < rows; ++t) {
    const float v = mrow[t];
    const float et = ex2_approx(fmaf(v, s0, tb[t]) - tmax);
    tden += et;
    tnum = fmaf(et, static_cast<float>(t), tnum);
    const float es = ex2_approx(fmaf(v, s1, sb[t]) - smax);
    sden += es;
    snum = fmaf(es, v, snum);
  }
  frac = fminf(fmaxf(tnum / (tden * static_cast<float>(rows - 1)), 0.0f), 1.0f);
  const float logit = fmaf(snum / sden, sc[2], sc[4]);
  send = sigmoid_f(logit * sc[3]);
}

// ---- grouped matrix layers: requests of one model processed together
// A group is up to kGroup requests that use the same model: entry g of the
// group table holds (model, request 0, ..., request kGroup-1), -1 for an empty
// slot. A thread keeps its cell's value for every request of the group in
// registers and loads each layer's 12 weights once for all of them, so weight
// traffic drops by the group size; the arithmetic per request is that of
// matrix_cell, in the same order, so the results are unchanged.
constexpr int kGroup = 8;
static_assert(kGroup % 2 == 0, "request pairs");

// 1g. expand + matrix layers [0, mid) for one group; thread per cell.
__global__ void __launch_bounds__(256) t2_expand_pre_g(const float* __restrict__ x, const int* __restrict__ groups,
                                                       const float* __restrict__ all_w, int models, T2Dev L,
                                                       float* __restrict__ m, int* err) {
  const int* gr = groups + static_cast<long long>(blockIdx.y) * (kGroup + 1);
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= L.cells) return;
  const int model = gr[0];
  if (model < 0 || model >= models) {  // the host validates the indices; this only guards the table
    ow::record_error(err, ow::kErrBadModelIndex);
    return;
  }
  const float* w = all_w + static_cast<long long>(model) * L.total;
  const int s = cell / L.rows, t = cell % L.rows;
  const float* pw = w + L.pair;
  const float tail = w[L.src_emb + s] + w[L.tgt_emb + t] + w[L.pair_emb + cell] + w[L.bias];
  int req[kGroup];
  float v[kGroup];
#pragma unroll
  for (int i = 0; i < kGroup; ++i) {
    req[i] = gr[1 + i];
    float a = 0.0f;
    if (req[i] >= 0) {
      const float* xs = x + (static_cast<long long>(req[i]) * L.rows + s) * kFeatures;
      const float* xt = x + (static_cast<long long>(req[i]) * L.rows + t) * kFeatures;
#pragma unroll
      for (int f = 0; f < static_cast<int>(kFeatures); ++f) a = fmaf(xs[f], pw[f], a);
#pragma unroll
      for (int f = 0; f < static_cast<int>(kFeatures); ++f) a = fmaf(xt[f], pw[kFeatures + f], a);
    }
    a += tail;
    v[i] = tanhf(a);
  }
  const float* mw = w + L.matrix + static_cast<long long>(cell) * kCellWeights;
  const long long per_layer = static_cast<long long>(L.cells) * kCellWeights;
  for (int l = 0; l < L.mid; ++l) {
    float4 a, b, c;
    load_cell_weights<true>(mw + l * per_layer, a, b, c);
#pragma unroll
    for (int i = 0; i < kGroup; i += 2) {
      const float2 o = matrix_cell_w2(make_float2(v[i], v[i + 1]), a, b, c);
      v[i] = o.x;
      v[i + 1] = o.y;
    }
  }
#pragma unroll
  for (int i = 0; i < kGroup; ++i)
    if (req[i] >= 0) m[static_cast<long long>(req[i]) * L.cells + cell] = v[i];
}

// 3g. matrix layers [mid, layers) + collapse for one group: CTA = 4 rows of
// every request of the group (blockDim = 4 * rows, at most 512 threads).
// done (or nullptr): one word per CTA in mapped host memory, set to `epoch`
// once the CTA's outputs are visible to the host, so host threads can copy a
// group's requests while later groups still run.
__global__ void __launch_bounds__(512) t2_post_collapse_g(const int* __restrict__ groups,
                                                          const float* __restrict__ all_w, int models, T2Dev L,
                                                          const float* __restrict__ m, float* __restrict__ out,
                                                          int* err, unsigned* done, unsigned epoch) {
  constexpr int kRows = 4;  // rows of each request per CTA
  __shared__ float s_m[kGroup][kRows][kRowStride];
  __shared__ float s_bias[2][kTargets][kRowStride];  // target and send biases x log2 e
  __shared__ float s_send[kGroup][kRows][kTargets];
  __shared__ float s_frac[kGroup][kRows][kTargets];
  const int* gr = groups + static_cast<long long>(blockIdx.y) * (kGroup + 1);
  const int row0 = blockIdx.x * kRows;
  const int model = gr[0];
  if (model < 0 || model >= models) {
    if (threadIdx.x == 0) ow::record_error(err, ow::kErrBadModelIndex);
    return;
  }
  int req[kGroup];
#pragma unroll
  for (int i = 0; i < kGroup; ++i) req[i] = gr[1 + i];
  const float* w = all_w + static_cast<long long>(model) * L.total;
  const long long per_layer = static_cast<long long>(L.cells) * kCellWeights;
  stage_collapse_bias(w, L, &s_bias[0][0][0]);
  for (int i = threadIdx.x; i < kRows * L.rows; i += blockDim.x) {
    const int lr = i / L.rows, t = i % L.rows;
    const int row = row0 + lr;
    if (row >= L.rows) continue;
    const int cell = row * L.rows + t;
    float v[kGroup];
#pragma unroll
    for (int g = 0; g < kGroup; ++g)
      v[g] = req[g] >= 0 ? m[static_cast<long long>(req[g]) * L.cells + cell] : 0.0f;
    const float* mw = w + L.matrix + static_cast<long long>(cell) * kCellWeights;
    for (int l = L.mid; l < L.layers; ++l) {
      float4 a, b, c;
      load_cell_weights<true>(mw + l * per_layer, a, b, c);
#pragma unroll
      for (int g = 0; g < kGroup; g += 2) {
        const float2 o = matrix_cell_w2(make_float2(v[g], v[g + 1]), a, b, c);
        v[g] = o.x;
        v[g + 1] = o.y;
      }
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) s_m[g][lr][t] = v[g];
  }
  __syncthreads();
  // thread per (request, row, action)
  for (int item = threadIdx.x; item < kGroup * kRows * static_cast<int>(kTargets); item += blockDim.x) {
    const int g = item / (kRows * static_cast<int>(kTargets));
    const int rest = item % (kRows * static_cast<int>(kTargets));
    const int lr = rest / kTargets, a = rest % kTargets;
    const int row = row0 + lr;
    const int rq = gr[1 + g];  // the group table, not req[]: a runtime index would put req[] in local memory
    if (row >= L.rows || rq < 0) continue;
    collapse_item(s_m[g][lr], &s_bias[0][0][0], a, L.rows, w + L.scalars + a * kOutScalars, s_frac[g][lr][a],
                  s_send[g][lr][a]);
  }
  __syncthreads();
  // the row's send fractions normalised when they sum above 1
  if (threadIdx.x < kGroup * kRows) {
    const int g = threadIdx.x / kRows, lr = threadIdx.x % kRows;
    float sum = 0.0f;
    for (int a = 0; a < static_cast<int>(kTargets); ++a) sum += s_send[g][lr][a];
    const float norm = sum > 1.0f ? 1.0f / sum : 1.0f;
    for (int a = 0; a < static_cast<int>(kTargets); ++a) s_send[g][lr][a] *= norm;
  }
  __syncthreads();
  // each (request, row) output is 24 contiguous floats: six 16-byte stores of (target, send) pairs
  for (int item = threadIdx.x; item < kGroup * kRows * 6; item += blockDim.x) {
    const int g = item / (kRows * 6), lr = (item / 6) % kRows, q = item % 6;
    const int row = row0 + lr;
    const int rq = gr[1 + g];
    if (row >= L.rows || rq < 0) continue;
    const float4 v = make_float4(s_frac[g][lr][2 * q], s_send[g][lr][2 * q], s_frac[g][lr][2 * q + 1],
                                 s_send[g][lr][2 * q + 1]);
    reinterpret_cast<float4*>(out + (static_cast<long long>(rq) * L.rows + row) * kOutPerRow)[q] = v;
  }
  if (done != nullptr) {
    // every thread orders its own output stores before the barrier, then one
    // thread publishes the CTA's done word
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(done + blockIdx.y * gridDim.x + blockIdx.x) = epoch;
  }
}

// 2^x for x <= 0 on the FMA pipe: Cody-Waite style reduction x = n + f with
// n = rint(x) from the 1.5 * 2^23 shifter and f in [-1/2, 1/2], a degree-4
// polynomial for 2^f fitted here for minimum relative error on that interval
// (2.7e-6 in f32 Horner evaluation), then n added to the exponent field with an
// integer multiply-add. x is clamped to -125 first (2^-125 is far below any
// softmax term that matters). Nine FMA-pipe instructions, no MUFU.
__device__ __forceinline__ float exp2_poly(float x) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23: x + kShift rounds x to an integer in the low bits
  x = fmaxf(x, -125.0f);
  const float t = x + kShift;
  const float f = x - (t - kShift);
  float p = fmaf(9.570096619e-03f, f, 5.591785908e-02f);
  p = fmaf(p, f, 2.402474433e-01f);
  p = fmaf(p, f, 6.931217909e-01f);
  p = fmaf(p, f, 9.999992847e-01f);
  // bits(t) = bits(kShift) + n, and bits(kShift) << 23 wraps to 0, so bits(t) << 23 = n << 23
  return __uint_as_float(__float_as_uint(t) * 8388608u + __float_as_uint(p));
}

// 2. full scalar attention + attention FFN, CTA per request, in place on m.
//
// The scores of a head are rank one: q_i k_j with q_i = m_i wq + bq and
// k_j = m_j wk + bk, so softmax_j(q_i k_j) = softmax_j(a_i m_j) with
// a_i = q_i wk, and the head's weighted value is
//   wavg_i = wv E_i[m] + bv,   E_i[m] = sum_j m_j e^(a_i m_j) / sum_j e^(a_i m_j).
// Two kernels compute it.
//
// 2a. t2_attention_moments (the usual path). With c, h the centre and
// half-width of the request's cell values, x_j = (m_j - c) / h lies in
// [-1, 1] and b_i = a_i h. The generating function of the modified Bessel
// functions (Abramowitz & Stegun 9.6.34 with cos t = x) gives, for every real b,
//   e^(b x) = I_0(b) + 2 sum_{k>=1} I_k(b) T_k(x)          (T_k: Chebyshev)
// so with the request's Chebyshev moments mu_k = sum_j T_k(x_j) and
// nu_k = sum_j x_j T_k(x_j) = (mu_{k+1} + mu_{|k-1|}) / 2,
//   sum_j e^(b x_j)     = I_0 mu_0 + 2 sum_k I_k mu_k
//   sum_j x_j e^(b x_j) = I_0 nu_0 + 2 sum_k I_k nu_k
// and E_i[m] = c + h (second / first). The I_k(b_i) come from Miller's
// backward recurrence I_{k-1} = I_{k+1} + (2k / b) I_k started at k = P with
// arbitrary scale (the scale cancels in the ratio), in double precision.
// The series is cut at P = ceil(8.5 sqrt(|b|max) + 7): over |b| in [1e-12, 1e3]
// the dropped terms sum to at most 1e-16 of e^|b| (checked against tabulated
// e^-|b| I_k(|b|)), and every term of the first sum is at most e^|b| while the
// sum is at least e^|b| (a cell sits at each end of [-1, 1]), so the ratio is
// good to double rounding, far below the f32 rounding of a direct sum. Work per
// request and head: O(cells x P) for the moments and for the recurrences,
// instead of cells^2 exponentials. A request whose |b|max exceeds
// kMomentBetaMax on some head, or with more than 512 x 8 cells, is flagged for:
//
// 2b. t2_attention (direct): one pass over the keys in shared memory with the
// exact closed-form row max of the rank-1 scores; each of the THREADS threads
// owns QPT queries and, per key, the last NPOLY of them take their exponential
// from the FMA pipe (exp2_poly), the others from the MUFU (ex2.approx). The
// request's cell values are staged in shared memory first, so a grid of more
// than QPT x THREADS cells (several query chunks) reads the attention's
// inputs, not the outputs of an earlier chunk. Requests that 2a took return
// at once.
constexpr int kAttnThreads = 1024;
constexpr int kAttnQpt = 4;
constexpr int kAttnPoly = 1;
constexpr int kMomThreads = 512;
constexpr int kMomQpt = 8;
constexpr int kMomentMax = 192;              // highest Chebyshev order used by the recurrence
constexpr double kMomentBetaMax = 470.0;     // ceil(8.5 sqrt(470) + 7) = 192
constexpr double kMomentBetaLinear = 1e-6;   // below: first order in b, relative error O(b^2)

__device__ __forceinline__ int moment_order(double beta) {
  const int p = static_cast<int>(ceil(8.5 * sqrt(beta) + 7.0));
  return (p + 3) & ~3;  // a multiple of 4: the recurrence checks its scale every 4 steps
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// |b|max of a head: q is affine in m, so its largest magnitude sits at an end of [lo, hi]
__device__ __forceinline__ double head_beta_max(const float* hw, float lo, float hi, double mh) {
  const double qmax = fmax(fabs(static_cast<double>(fmaf(lo, hw[0], hw[1]))),
                           fabs(static_cast<double>(fmaf(hi, hw[0], hw[1]))));
  return qmax * fabs(static_cast<double>(hw[2])) * mh;
}

// E[m] for two queries from the moments (mu_k, nu_k), k = 0 .. P: Miller's
// backward recurrence from k = P (z_{P+1} = 0, z_P = 1) for each query, the two
// sums accumulated on the way down, rescaled together every four steps.
__device__ __forceinline__ void moment_pair(const double2* __restrict__ s_mn, int P, float m0, float m1, float wq,
                                            float bq, float wk, double mc, double mh, double& em0, double& em1) {
  double bb[2], step[2], z[2], z1[2], sf[2], sp[2];
  const float mq[2] = {m0, m1};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    bb[i] = static_cast<double>(fmaf(mq[i], wq, bq)) * static_cast<double>(wk) * mh;
    step[i] = fabs(bb[i]) >= kMomentBetaLinear ? 2.0 / bb[i] : 0.0;
    z[i] = 1.0;
    z1[i] = 0.0;
    sf[i] = 0.0;
    sp[i] = 0.0;
  }
  // k = P .. 1, four steps between scale checks (P is a multiple of 4)
  for (int k = P; k > 0; k -= 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const double2 mn = s_mn[k - u];
      const double kk = static_cast<double>(k - u);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        sf[i] = fma(z[i], mn.x, sf[i]);
        sp[i] = fma(z[i], mn.y, sp[i]);
        const double zn = fma(kk * step[i], z[i], z1[i]);
        z1[i] = z[i];
        z[i] = zn;
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (fabs(z[i]) > 1e180) {  // growth per step is at most 1 + 2P / 1e-6 < 4e8
        z[i] *= 1e-180;
        z1[i] *= 1e-180;
        sf[i] *= 1e-180;
        sp[i] *= 1e-180;
      }
    }
  }
  const double2 mn0 = s_mn[0];
  const double mu1 = s_mn[1].x, mu2 = s_mn[2].x;
  double em[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    double ratio;
    if (!(fabs(bb[i]) >= kMomentBetaLinear)) {
      // e^(b x) = 1 + b x + O(b^2): sum x e^(bx) / sum e^(bx) to first order (sum x^2 = (mu_0 + mu_2) / 2)
      ratio = fma(bb[i], 0.5 * (mn0.x + mu2), mn0.y) / fma(bb[i], mu1, mn0.x);
    } else {
      ratio = fma(z[i], mn0.y, 2.0 * sp[i]) / fma(z[i], mn0.x, 2.0 * sf[i]);
    }
    em[i] = fma(mh, ratio, mc);
  }
  em0 = em[0];
  em1 = em[1];
}

// 2a. CTA per request, THREADS threads of QPT cells each; direct[r] = 1 when
// the request is left to 2b, 0 when it is done here.
template <int THREADS, int QPT>
__global__ void __launch_bounds__(THREADS) t2_attention_moments(const size_t* __restrict__ idx,
                                                                const float* __restrict__ all_w, int models, T2Dev L,
                                                                float* __restrict__ m, int* err,
                                                                int* __restrict__ direct) {
  constexpr int kWarps = THREADS / 32;
  __shared__ float s_red[2][kWarps];
  __shared__ double2 s_mn[kMomentMax + 2];  // (mu_k, nu_k)
  __shared__ double s_part[kWarps][8];
  const int r = blockIdx.x;
  if (L.cells > THREADS * QPT) {
    if (threadIdx.x == 0) direct[r] = 1;
    return;
  }
  const float* w = model_of(all_w, idx, models, r, L.total, err);
  const float* aw = w + L.attn;
  float* mr = m + static_cast<long long>(r) * L.cells;
  float mv[QPT];
  float lo = INFINITY, hi = -INFINITY;
#pragma unroll
  for (int i = 0; i < QPT; ++i) {
    const int c = i * THREADS + threadIdx.x;
    mv[i] = c < L.cells ? mr[c] : 0.0f;
    if (c < L.cells) {
      lo = fminf(lo, mv[i]);
      hi = fmaxf(hi, mv[i]);
    }
  }
  hi = ow::warp_max(hi);
  lo = -ow::warp_max(-lo);
  if ((threadIdx.x & 31) == 0) {
    s_red[0][threadIdx.x >> 5] = hi;
    s_red[1][threadIdx.x >> 5] = lo;
  }
  __syncthreads();
  hi = s_red[0][0];
  lo = s_red[1][0];
  for (int i = 1; i < kWarps; ++i) {
    hi = fmaxf(hi, s_red[0][i]);
    lo = fminf(lo, s_red[1][i]);
  }
  // centre and half-width (exact in double: f32 sums and halves)
  const double mc = 0.5 * (static_cast<double>(lo) + static_cast<double>(hi));
  const double mh = 0.5 * (static_cast<double>(hi) - static_cast<double>(lo));
  bool take = true;  // the same in every thread
  for (int h = 0; h < L.heads; ++h) take = take && head_beta_max(aw + h * kHeadWeights, lo, hi, mh) <= kMomentBetaMax;
  if (threadIdx.x == 0) direct[r] = take ? 0 : 1;
  if (!take) return;
  float ctx[QPT];
#pragma unroll
  for (int i = 0; i < QPT; ++i) ctx[i] = 0.0f;
  for (int h = 0; h < L.heads; ++h) {
    const float* hw = aw + h * kHeadWeights;
    const float wq = hw[0], bq = hw[1], wk = hw[2], wv = hw[4], bv = hw[5], wo = hw[6];
    float wavg[QPT];
    if (!(mh > 0.0)) {
      // one cell value: every weight is equal, E[m] = that value
#pragma unroll
      for (int i = 0; i < QPT; ++i) wavg[i] = fmaf(lo, wv, bv);
    } else {
      const int P = moment_order(head_beta_max(hw, lo, hi, mh));  // mu_0 .. mu_{P+1}
      const double inv_h = 1.0 / mh;
      double x[QPT], tp[QPT], tc[QPT];
#pragma unroll
      for (int i = 0; i < QPT; ++i) {
        const bool valid = i * THREADS + static_cast<int>(threadIdx.x) < L.cells;
        x[i] = valid ? (static_cast<double>(mv[i]) - mc) * inv_h : 0.0;
        tp[i] = x[i];               // T_{-1} = T_1
        tc[i] = valid ? 1.0 : 0.0;  // T_0 (0 for a padding slot: its T_k stay 0)
      }
      __syncthreads();  // the previous head is done with s_mn and s_part
      for (int kb = 0; kb <= P + 1; kb += 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          double sum = 0.0;
#pragma unroll
          for (int i = 0; i < QPT; ++i) {
            sum += tc[i];
            const double tn = fma(2.0 * x[i], tc[i], -tp[i]);
            tp[i] = tc[i];
            tc[i] = tn;
          }
          sum = warp_sum_d(sum);
          if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5][u] = sum;
        }
        __syncthreads();
        if (threadIdx.x < 8 && kb + static_cast<int>(threadIdx.x) <= P + 1) {
          double mu = 0.0;
          for (int wi = 0; wi < kWarps; ++wi) mu += s_part[wi][threadIdx.x];
          s_mn[kb + threadIdx.x].x = mu;
        }
        __syncthreads();
      }
      for (int k = threadIdx.x; k <= P; k += THREADS) s_mn[k].y = k == 0 ? s_mn[1].x : 0.5 * (s_mn[k + 1].x + s_mn[k - 1].x);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < QPT; i += 2) {
        double e0, e1;
        moment_pair(s_mn, P, mv[i], mv[i + 1], wq, bq, wk, mc, mh, e0, e1);
        wavg[i] = static_cast<float>(fma(e0, static_cast<double>(wv), static_cast<double>(bv)));
        wavg[i + 1] = static_cast<float>(fma(e1, static_cast<double>(wv), static_cast<double>(bv)));
      }
    }
#pragma unroll
    for (int i = 0; i < QPT; ++i) ctx[i] = fmaf(wavg[i], wo, ctx[i]);
  }
  // attention FFN; each thread rewrites only the cells it read
  const float* s = aw + L.heads * kHeadWeights;
#pragma unroll
  for (int i = 0; i < QPT; ++i) {
    const int c = i * THREADS + threadIdx.x;
    if (c < L.cells) {
      const float rr = fmaf(mv[i], s[0], ctx[i] + s[1]);
      const float hid = tanhf(fmaf(rr, s[2], s[3]));
      mr[c] = tanhf(fmaf(hid, s[4], rr + s[5]));
    }
  }
}

// 2b. direct attention for the requests 2a flagged.
template <int THREADS, int QPT, int NPOLY>
__global__ void __launch_bounds__(THREADS) t2_attention(const size_t* __restrict__ idx,
                                                        const float* __restrict__ all_w, int models, T2Dev L,
                                                        float* __restrict__ m, int* err,
                                                        const int* __restrict__ direct) {
  constexpr int kAttnThreads = THREADS;
  constexpr int kQueriesPerThread = QPT;
  extern __shared__ float4 s_dyn[];
  float2* s_kv = reinterpret_cast<float2*>(s_dyn);        // [cells] (k * log2 e, v)
  float* s_m = reinterpret_cast<float*>(s_kv + L.cells);  // [cells] the attention's input
  __shared__ float s_red[2][32];
  const int r = blockIdx.x;
  if (direct[r] == 0) return;
  const float* w = model_of(all_w, idx, models, r, L.total, err);
  const float* aw = w + L.attn;
  float* mr = m + static_cast<long long>(r) * L.cells;
  const float kLog2e = 1.4426950408889634f;
  for (int c = threadIdx.x; c < L.cells; c += kAttnThreads) s_m[c] = mr[c];
  for (int base = 0; base < L.cells; base += kAttnThreads * kQueriesPerThread) {
    float mv[kQueriesPerThread], ctx[kQueriesPerThread];
    __syncthreads();  // s_m staged
#pragma unroll
    for (int i = 0; i < kQueriesPerThread; ++i) {
      const int c = base + i * kAttnThreads + threadIdx.x;
      mv[i] = c < L.cells ? s_m[c] : 0.0f;
      ctx[i] = 0.0f;
    }
    for (int h = 0; h < L.heads; ++h) {
      const float* hw = aw + h * kHeadWeights;
      const float wq = hw[0], bq = hw[1], wk = hw[2], bk = hw[3], wv = hw[4], bv = hw[5], wo = hw[6];
      __syncthreads();  // previous head / chunk done with s_kv
      float kmax = -INFINITY, kmin = INFINITY;
      for (int c = threadIdx.x; c < L.cells; c += kAttnThreads) {
        const float cv = s_m[c];
        const float k = fmaf(cv, wk, bk);
        s_kv[c] = make_float2(k * kLog2e, fmaf(cv, wv, bv));
        kmax = fmaxf(kmax, k);
        kmin = fminf(kmin, k);
      }
      kmax = ow::warp_max(kmax);
      kmin = -ow::warp_max(-kmin);
      if ((threadIdx.x & 31) == 0) {
        s_red[0][threadIdx.x >> 5] = kmax;
        s_red[1][threadIdx.x >> 5] = kmin;
      }
      __syncthreads();
      kmax = s_red[0][0];
      kmin = s_red[1][0];
      for (int i = 1; i < kAttnThreads / 32; ++i) {
        kmax = fmaxf(kmax, s_red[0][i]);
        kmin = fminf(kmin, s_red[1][i]);
      }
      float q[kQueriesPerThread], off[kQueriesPerThread], den[kQueriesPerThread], acc[kQueriesPerThread];
#pragma unroll
      for (int i = 0; i < kQueriesPerThread; ++i) {
        q[i] = fmaf(mv[i], wq, bq);
        // exact row max of the rank-1 scores q*k_j, in log2 units
        off[i] = (q[i] >= 0.0f ? q[i] * kmax : q[i] * kmin) * kLog2e;
        den[i] = 0.0f;
        acc[i] = 0.0f;
      }
#pragma unroll 4
      for (int j = 0; j < L.cells; ++j) {
        const float2 kv = s_kv[j];
#pragma unroll
        for (int i = 0; i < kQueriesPerThread; ++i) {
          const float x = fmaf(q[i], kv.x, -off[i]);
          const float e = i >= kQueriesPerThread - NPOLY ? exp2_poly(x) : ex2_approx(x);
          den[i] += e;
          acc[i] = fmaf(e, kv.y, acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < kQueriesPerThread; ++i) ctx[i] = fmaf(acc[i] / den[i], wo, ctx[i]);
    }
    const float* s = aw + L.heads * kHeadWeights;
#pragma unroll
    for (int i = 0; i < kQueriesPerThread; ++i) {
      const int c = base + i * kAttnThreads + threadIdx.x;
      if (c < L.cells) {
        const float rr = fmaf(mv[i], s[0], ctx[i] + s[1]);
        const float hid = tanhf(fmaf(rr, s[2], s[3]));
        mr[c] = tanhf(fmaf(hid, s[4], rr + s[5]));
      }
    }
  }
}

// Launches the attention for `n` requests: 2a over every request, then 2b,
// whose CTAs return at once for the requests 2a took. direct: n ints of scratch.
cudaError_t launch_t2_attention(const size_t* idx, const float* all_w, int models, const T2Dev& D, float* m, int* err,
                                int* direct, unsigned n, cudaStream_t stream) {
  t2_attention_moments<kMomThreads, kMomQpt><<<n, kMomThreads, 0, stream>>>(idx, all_w, models, D, m, err, direct);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem = static_cast<size_t>(D.cells) * (sizeof(float2) + sizeof(float));
  auto k = t2_attention<kAttnThreads, kAttnQpt, kAttnPoly>;
  e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  k<<<n, kAttnThreads, smem, stream>>>(idx, all_w, models, D, m, err, direct);
  return cudaGetLastError();
}

// 3. matrix layers [mid, layers) + collapse; CTA = 4 rows of one request.
constexpr int kRowsPerCta = 4;

template <bool VEC>
__global__ void __launch_bounds__(512) t2_post_collapse(const size_t* __restrict__ idx, const float* __restrict__ all_w,
                                                        int models, T2Dev L, const float* __restrict__ m,
                                                        float* __restrict__ out, int* err) {
  __shared__ float s_m[kRowsPerCta][kRowStride];
  __shared__ float s_bias[2][kTargets][kRowStride];  // target and send biases x log2 e
  __shared__ float s_send[kRowsPerCta][kTargets];
  const int r = blockIdx.y;
  const int row0 = blockIdx.x * kRowsPerCta;
  const float* w = model_of(all_w, idx, models, r, L.total, err);
  const long long per_layer = static_cast<long long>(L.cells) * kCellWeights;
  stage_collapse_bias(w, L, &s_bias[0][0][0]);
  for (int i = threadIdx.x; i < kRowsPerCta * L.rows; i += blockDim.x) {
    const int lr = i / L.rows, t = i % L.rows;
    const int row = row0 + lr;
    if (row >= L.rows) continue;
    const int cell = row * L.rows + t;
    float v = m[static_cast<long long>(r) * L.cells + cell];
    const float* mw = w + L.matrix + static_cast<long long>(cell) * kCellWeights;
    for (int l = L.mid; l < L.layers; ++l) v = matrix_cell<VEC>(v, mw + l * per_layer);
    s_m[lr][t] = v;
  }
  __syncthreads();
  // thread per (row, action)
  for (int item = threadIdx.x; item < kRowsPerCta * static_cast<int>(kTargets); item += blockDim.x) {
    const int lr = item / kTargets, a = item % kTargets;
    const int row = row0 + lr;
    if (row >= L.rows) continue;
    float frac;
    collapse_item(s_m[lr], &s_bias[0][0][0], a, L.rows, w + L.scalars + a * kOutScalars, frac, s_send[lr][a]);
    out[(static_cast<long long>(r) * L.rows + row) * kOutPerRow + a * 2] = frac;
  }
  __syncthreads();
  if (threadIdx.x < kRowsPerCta) {
    const int lr = threadIdx.x, row = row0 + lr;
    if (row < L.rows) {
      float sum = 0.0f;
      for (int a = 0; a < static_cast<int>(kTargets); ++a) sum += s_send[lr][a];
      const float norm = sum > 1.0f ? 1.0f / sum : 1.0f;
      for (int a = 0; a < static_cast<int>(kTargets); ++a)
        out[(static_cast<long long>(r) * L.rows + row) * kOutPerRow + a * 2 + 1] = s_send[lr][a] * norm;
    }
  }
}

// ---------------------------------------------------------------- legacy TrainableTransformer (model.rs:210-301)
// CTA per game: hidden [rows][d] in shared memory; per layer, per head, scaled
// max-subtracted softmax over rows; h = tanh(h + attn*scale); sigmoid heads.
__global__ void trainable_kernel(const float* __restrict__ in, const float* __restrict__ w, float* __restrict__ out,
                                 int rows, int d, int heads, int layers) {
  extern __shared__ float sm[];
  float* hid = sm;               // rows*d
  float* nxt = sm + rows * d;    // rows*d
  const int g = blockIdx.x;
  const float* inp = w;
  const float* pos = w + 2 * d;
  const float* scales = pos + d;
  const float* outp = scales + static_cast<long long>(layers) * d;
  for (int i = threadIdx.x; i < rows * d; i += blockDim.x) {
    const int r = i / d, k = i % d;
    const float f0 = in[(static_cast<long long>(g) * rows + r) * 2];
    const float f1 = in[(static_cast<long long>(g) * rows + r) * 2 + 1];
    const float p = static_cast<float>(r) / static_cast<float>(rows);
    hid[i] = tanhf(p * pos[k] + f0 * inp[k] + f1 * inp[d + k]);
  }
  __syncthreads();
  const int hd = d / heads;
  const float inv = 1.0f / sqrtf(static_cast<float>(hd));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int l = 0; l < layers; ++l) {
    for (int item = warp; item < heads * rows; item += nw) {
      const int h = item / rows, s = item % rows;
      float mx = -INFINITY;
      for (int t = 0; t < rows; ++t) {
        float part = 0.0f;
        for (int c = lane; c < hd; c += 32) part += hid[s * d + h * hd + c] * hid[t * d + h * hd + c];
        mx = fmaxf(mx, ow::warp_sum(part) * inv);
      }
      float den = 0.0f;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // hd <= 256 -> 8 per lane
      for (int t = 0; t < rows; ++t) {
        float part = 0.0f;
        for (int c = lane; c < hd; c += 32) part += hid[s * d + h * hd + c] * hid[t * d + h * hd + c];
        const float e = expf(ow::warp_sum(part) * inv - mx);
        den += e;
        for (int c = lane, i = 0; c < hd; c += 32, ++i) acc[i] = fmaf(e, hid[t * d + h * hd + c], acc[i]);
      }
      for (int c = lane, i = 0; c < hd; c += 32, ++i) nxt[s * d + h * hd + c] = acc[i] / den;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rows * d; i += blockDim.x)
      hid[i] = tanhf(hid[i] + nxt[i] * scales[static_cast<long long>(l) * d + (i % d)]);
    __syncthreads();
  }
  const float sc = sqrtf(static_cast<float>(d));
  for (int r = warp; r < rows; r += nw) {
    float t0 = 0.0f, t1 = 0.0f;
    for (int k = lane; k < d; k += 32) {
      t0 += hid[r * d + k] * outp[k];
      t1 += hid[r * d + k] * outp[d + k];
    }
    t0 = ow::warp_sum(t0);
    t1 = ow::warp_sum(t1);
    if (lane == 0) {
      out[(static_cast<long long>(g) * rows + r) * 2] = sigmoid_f(t0 / sc);
      out[(static_cast<long long>(g) * rows + r) * 2 + 1] = sigmoid_f(t1 / sc);
    }
  }
}

__global__ void copy_kernel(const float4* __restrict__ in, float4* __restrict__ out, size_t n4, const float* in_tail,
                            float* out_tail, size_t tail) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4; i += gridDim.x * blockDim.x)
    out[i] = in[i];
  if (blockIdx.x == 0 && threadIdx.x < tail) out_tail[threadIdx.x] = in_tail[threadIdx.x];
}

// ---------------------------------------------------------------- allocation-free forward
// Scratch of orbit_wars_cuda_true2d_forward_noalloc: a fixed device array
// every GPU that loads this library holds until exit (1 MiB). The first 256
// bytes hold the error word; the rest holds the per-request cell matrices and
// one path flag per request for the attention (game_count * (rows^2 + 1)
// floats at most kNoAllocCells).
constexpr size_t kNoAllocFloats = size_t(1) << 18;
constexpr size_t kNoAllocHeaderFloats = 64;
constexpr size_t kNoAllocCells = kNoAllocFloats - kNoAllocHeaderFloats;  // 262,080 cells
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

// Device address of g_noalloc_scratch on the current device. In host code
// the array's name is only a host-side stand-in, never a device address, so
// every call asks the runtime for it: a cached address would dangle after a
// device reset reloads the module. Once the module is loaded (the first call
// on a device, which is why that call must come before any stream capture)
// the lookup involves no allocation and no synchronisation.
cudaError_t noalloc_scratch_address(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = static_cast<float*>(p);
  return cudaSuccess;
}

// The reference's weight layout on the device, unpadded (scalar weight loads).
T2Dev ref_layout_dev(const T2Layout& L) {
  T2Dev d{};
  d.rows = static_cast<int>(L.rows);
  d.cells = static_cast<int>(L.cells);
  d.layers = static_cast<int>(L.layers);
  d.heads = static_cast<int>(L.heads);
  d.mid = static_cast<int>(L.layers / 2);
  d.pair = L.pair; d.src_emb = L.src_emb; d.tgt_emb = L.tgt_emb; d.pair_emb = L.pair_emb; d.bias = L.bias;
  d.matrix = L.matrix; d.attn = L.attn; d.tbias = L.tbias; d.sbias = L.sbias; d.scalars = L.scalars;
  d.total = static_cast<long long>(L.total);
  return d;
}

// ---------------------------------------------------------------- device decode
// The part of the engine's decoder that needs no geometry
// (crates/orbit-wars-core/src/decoder.rs:85-124, target_row_from_fraction
// :457-461), on the forward's outputs still in HBM. CTA per request, thread per
// (source row, target slot). Active rows are the rows whose planet id is not
// NO_PLANET_ID (-1), in row order (encoder.rs:14-26). A source is decoded only
// when it is active, owned by the player and on the map (flags, the encoder's
// row flags: kRowOwned set, kRowAbsent clear); then, per slot:
//   target_row = active[min(floor(clamp(target_fraction, 0, 1) * n_active), n_active - 1)],
//   skipped when it is the source row or its planet is absent from the map
//   (planet_by_id misses, decoder.rs:112-114);
//   send = clamp(send_fraction, 0, 1), skipped when send <= 0;
//   ship_count = floor(ships * send), skipped when < 1.
// target_rows[r][s][a] is the target row or -1 (skipped), ship_counts the count
// or 0. A non-finite output of a decoded source raises the device error word,
// as the decoder returns NonFiniteModelOutput.
__global__ void __launch_bounds__(512) t2_decode(const float* __restrict__ out, const int32_t* __restrict__ row_ids,
                                                 const uint8_t* __restrict__ flags, const float* __restrict__ ships,
                                                 int rows, int32_t* __restrict__ target_rows,
                                                 int32_t* __restrict__ ship_counts, int* err) {
  __shared__ int s_active[kMaxRows];
  __shared__ int s_n;
  const int r = blockIdx.x;
  const int32_t* ids = row_ids + static_cast<long long>(r) * rows;
  const uint8_t* fl = flags + static_cast<long long>(r) * rows;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int i = 0; i < rows; ++i)
      if (ids[i] != -1) s_active[n++] = i;
    s_n = n;
  }
  __syncthreads();
  const int n_active = s_n;
  for (int item = threadIdx.x; item < rows * static_cast<int>(kTargets); item += blockDim.x) {
    const int src = item / kTargets, a = item % kTargets;
    const long long o = (static_cast<long long>(r) * rows + src) * kTargets + a;
    int target = -1, count = 0;
    if (ids[src] != -1 && (fl[src] & (enc::kRowOwned | enc::kRowAbsent)) == enc::kRowOwned && n_active > 0) {
      const float* pair = out + (static_cast<long long>(r) * rows + src) * kOutPerRow + a * 2;
      const float tf = pair[0], sf = pair[1];
      if (!isfinite(tf) || !isfinite(sf)) {
        ow::record_error(err, ow::kErrNonFiniteOutput);
      } else {
        const int scaled = static_cast<int>(floorf(fminf(fmaxf(tf, 0.0f), 1.0f) * static_cast<float>(n_active)));
        const int trow = s_active[min(scaled, n_active - 1)];
        const float send = fminf(fmaxf(sf, 0.0f), 1.0f);
        if (trow != src && (fl[trow] & enc::kRowAbsent) == 0 && send > 0.0f) {
          const int c = static_cast<int>(floorf(ships[static_cast<long long>(r) * rows + src] * send));
          if (c >= 1) {
            target = trow;
            count = c;
          }
        }
      }
    }
    target_rows[o] = target;
    ship_counts[o] = count;
  }
}

#include "ow_t2_train.cuh"

// ---------------------------------------------------------------- process-global workspace
struct Workspace {
  std::mutex mu;
  // population
  float* weights = nullptr;
  size_t weights_cap = 0;  // floats
  size_t models = 0;
  OrbitWarsCudaTrue2DShape shape{0, 0, 0};
  bool resident = false;
  size_t request_capacity = 0;
  // per-call buffers
  float* in = nullptr;
  size_t in_cap = 0;
  float* out = nullptr;
  size_t out_cap = 0;
  float* m = nullptr;
  size_t m_cap = 0;
  size_t* idx = nullptr;
  size_t idx_cap = 0;
  int32_t* dec_ids = nullptr;  // device decode: row planet ids, row flags, ships; outputs
  uint8_t* dec_flags = nullptr;
  float* dec_ships = nullptr;
  int32_t* dec_rows = nullptr;
  int32_t* dec_counts = nullptr;
  size_t dec_cap = 0;
  // device encoder: game states packed into pinned memory, uploaded in one copy
  unsigned char* enc_host = nullptr;
  size_t enc_host_cap = 0;
  unsigned char* enc_dev = nullptr;
  size_t enc_dev_cap = 0;
  int32_t* enc_err = nullptr;
  size_t enc_err_cap = 0;
  std::vector<int32_t> host_err;
  // pinned staging of the host-buffer forward's input rows and output rows
  unsigned char* pin_out = nullptr;
  size_t pin_out_cap = 0;
  unsigned char* pin_map = nullptr;  // mapped pinned outputs (synchronous host-buffer forwards)
  size_t pin_map_cap = 0;
  unsigned* done_map = nullptr;  // mapped done words of the collapse CTAs, one per CTA
  size_t done_cap = 0;
  unsigned done_epoch = 0;       // the value this call's CTAs write (0 never)
  unsigned char* pin_meta = nullptr;  // model indices and the group table of a call
  size_t pin_meta_cap = 0;
  std::vector<cudaEvent_t> out_pieces;  // output download pieces (host-buffer forwards)
  // training step: one device arena and the pinned staging of the weights, kept between calls
  unsigned char* train_arena = nullptr;
  size_t train_cap = 0;
  unsigned char* train_pin = nullptr;
  size_t train_pin_cap = 0;
  int* groups = nullptr;  // model groups of the current call: (model, kGroup request indices) each
  size_t groups_cap = 0;
  std::vector<int> host_groups;
  int* err = nullptr;
  cudaStream_t stream = nullptr;
  // device timing (orbit_wars_cuda_true2d_profile_begin/_end): an event before
  // each kernel of run_forward and one after the last, names[i] = the kernel
  // launched after events[i] (nullptr for the closing event)
  std::vector<cudaEvent_t> prof_events;
  std::vector<const char*> prof_names;
  size_t prof_used = 0;
  bool prof_on = false;
};

Workspace& ws() {
  static Workspace* w = new Workspace();  // lives for the process, like the reference's
  return *w;
}

template <typename T>
cudaError_t ensure(T*& p, size_t& cap, size_t n) {
  if (n <= cap && p != nullptr) return cudaSuccess;
  if (p != nullptr) cudaFree(p);
  p = nullptr;
  cap = 0;
  const cudaError_t e = cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T));
  if (e == cudaSuccess) cap = n;
  return e;
}

cudaError_t ensure_common(Workspace& W) {
  if (W.stream == nullptr) {
    const cudaError_t e = cudaStreamCreateWithFlags(&W.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return e;
  }
  if (W.err == nullptr) {
    const cudaError_t e = cudaMalloc(&W.err, sizeof(int));
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Device buffers of the decode for rn = requests x rows (ids, flags, ships) and
// rn x 12 outputs.
cudaError_t ensure_decode(Workspace& W, size_t rn) {
  const size_t dn = rn * kTargets;
  if (dn <= W.dec_cap && W.dec_ids != nullptr) return cudaSuccess;
  for (void* q : {static_cast<void*>(W.dec_ids), static_cast<void*>(W.dec_flags), static_cast<void*>(W.dec_ships),
                  static_cast<void*>(W.dec_rows), static_cast<void*>(W.dec_counts)})
    if (q != nullptr) cudaFree(q);
  W.dec_ids = nullptr; W.dec_flags = nullptr; W.dec_ships = nullptr; W.dec_rows = nullptr; W.dec_counts = nullptr;
  W.dec_cap = 0;
  cudaError_t e = cudaMalloc(&W.dec_ids, rn * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMalloc(&W.dec_flags, rn);
  if (e == cudaSuccess) e = cudaMalloc(&W.dec_ships, rn * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&W.dec_rows, dn * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMalloc(&W.dec_counts, dn * sizeof(int32_t));
  if (e == cudaSuccess) W.dec_cap = dn;
  return e;
}

bool same_shape(const OrbitWarsCudaTrue2DShape& a, const OrbitWarsCudaTrue2DShape& b) {
  return a.layer_count == b.layer_count && a.row_count == b.row_count && a.head_count == b.head_count;
}

const char* device_error_text(int code) {
  switch (code) {
    case ow::kErrBadModelIndex: return "model index outside the population";
    case ow::kErrNonFiniteOutput: return "non-finite model output";
    default: return "device error";
  }
}

// Uploads `models` models into the resident population.
OrbitWarsCudaStatus upload(Workspace& W, const float* all_w, size_t models, const OrbitWarsCudaTrue2DShape& shape) {
  const T2Layout L = t2_layout(shape.layer_count, shape.row_count, shape.head_count);
  const size_t dt = dev_total(L), pad = matrix_pad(L);
  T2_TRY(ensure(W.weights, W.weights_cap, dt * models));
  // prefix (input pair .. expand bias) and the rest (matrix .. output scalars), one strided copy each
  T2_TRY(cudaMemcpy2DAsync(W.weights, dt * sizeof(float), all_w, L.total * sizeof(float), L.matrix * sizeof(float),
                           models, cudaMemcpyHostToDevice, W.stream));
  T2_TRY(cudaMemcpy2DAsync(W.weights + L.matrix + pad, dt * sizeof(float), all_w + L.matrix, L.total * sizeof(float),
                           (L.total - L.matrix) * sizeof(float), models, cudaMemcpyHostToDevice, W.stream));
  W.models = models;
  W.shape = shape;
  W.resident = true;
  return ok();
}

// memcpy split over up to 8 host threads (pageable <-> pinned staging).
// Host copies between pinned staging and the caller's buffers, split over a
// pool of worker threads started once (thread start-up would otherwise cost
// more than a few-MB copy). One copy at a time: the pool's own mutex orders
// callers. The pool is never destroyed; its idle workers end with the process.
// A child process forked after the pool started has no workers (and may hold
// a copy of a locked mutex): there every copy runs on the calling thread.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool* pool = new CopyPool();
    return *pool;
  }
  void copy(unsigned char* dst, const unsigned char* src, size_t bytes) {
    const size_t parts = std::min<size_t>(workers_ + 1, std::max<size_t>(1, bytes >> 19));
    if (parts <= 1 || forked_) {
      std::memcpy(dst, src, bytes);
      return;
    }
    struct Job {
      unsigned char* dst;
      const unsigned char* src;
      size_t bytes, per;
    } job{dst, src, bytes, ((bytes + parts - 1) / parts + 63) & ~size_t(63)};
    run_parts(
        [](void* c, size_t k) {
          const Job* j = static_cast<const Job*>(c);
          const size_t o = k * j->per;
          if (o < j->bytes) std::memcpy(j->dst + o, j->src + o, std::min(j->per, j->bytes - o));
        },
        &job, parts);
  }
  // fn(ctx, k) for k = 0 .. parts - 1 (at most the workers + 1): k = 0 on the
  // calling thread, the rest on workers; returns when all have returned. In a
  // forked child every part runs on the calling thread, in order.
  void run_parts(void (*fn)(void*, size_t), void* ctx, size_t parts) {
    parts = std::max<size_t>(1, std::min<size_t>(parts, workers_ + 1));
    if (parts == 1 || forked_) {
      for (size_t k = 0; k < parts; ++k) fn(ctx, k);
      return;
    }
    std::lock_guard<std::mutex> one(call_mu_);
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn_ = fn;
      ctx_ = ctx;
      parts_ = parts;
      pending_ = parts - 1;
      ++generation_;
    }
    cv_.notify_all();
    fn(ctx, 0);
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [&] { return pending_ == 0; });
  }
  size_t threads() const { return forked_ ? 1 : workers_ + 1; }

 private:
  CopyPool() {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    workers_ = std::min<size_t>(7, hw > 1 ? hw - 1 : 0);
    for (size_t k = 1; k <= workers_; ++k) std::thread([this, k] { run(k); }).detach();
    pthread_atfork(nullptr, nullptr, [] { forked_ = true; });
  }
  void run(size_t k) {
    uint64_t seen = 0;
    for (;;) {
      void (*fn)(void*, size_t);
      void* ctx;
      size_t parts;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return generation_ != seen; });
        seen = generation_;
        fn = fn_;
        ctx = ctx_;
        parts = parts_;
      }
      if (k < parts) {
        fn(ctx, k);
        std::lock_guard<std::mutex> lk(mu_);
        if (--pending_ == 0) done_.notify_one();
      }
    }
  }
  size_t workers_ = 0;
  std::mutex call_mu_, mu_;
  std::condition_variable cv_, done_;
  uint64_t generation_ = 0;
  void (*fn_)(void*, size_t) = nullptr;
  void* ctx_ = nullptr;
  size_t parts_ = 0, pending_ = 0;
  static inline volatile bool forked_ = false;
};

void par_copy(unsigned char* dst, const unsigned char* src, size_t bytes) { CopyPool::get().copy(dst, src, bytes); }

// Host side of a streamed output copy. The collapse CTAs publish one done word
// each (set to the call's epoch) in mapped memory after their outputs; the pool
// threads take the model groups in launch order, wait for a group's words and
// copy its requests' rows to the caller's buffer while later groups still run.
struct GroupCopy {
  const volatile unsigned* done;
  unsigned epoch;
  size_t per_group;          // collapse CTAs per group
  const int* table;          // kGroup + 1 ints per group: the model, then request indices (-1: none)
  size_t n_groups;
  const unsigned char* src;  // the mapped outputs
  unsigned char* dst;        // the caller's outputs
  size_t req_bytes;
  cudaStream_t stream;
  std::chrono::steady_clock::time_point deadline;
  std::atomic<size_t> next{0};
  std::atomic<int> stream_done{0};  // set by the calling thread once the stream has drained
  std::atomic<int> gave_up{0};      // some group's words never came: the caller copies everything
};

void group_copy(void* c, size_t k) {
  GroupCopy* j = static_cast<GroupCopy*>(c);
  for (;;) {
    const size_t g = j->next.fetch_add(1);
    if (g >= j->n_groups) return;
    for (size_t b = 0; b < j->per_group; ++b) {
      const volatile unsigned* w = j->done + g * j->per_group + b;
      for (unsigned spins = 1; *w != j->epoch; ++spins) {
        if (j->gave_up.load(std::memory_order_relaxed) != 0) return;
        if ((spins & 1023u) != 0) continue;
        // the calling thread watches the stream: once it has drained, a word
        // still unset belongs to a CTA that returned early (a device error)
        if (k == 0 && j->stream_done.load() == 0 && cudaStreamQuery(j->stream) != cudaErrorNotReady)
          j->stream_done.store(1);
        if ((j->stream_done.load() != 0 && *w != j->epoch) || std::chrono::steady_clock::now() > j->deadline) {
          j->gave_up.store(1);
          return;
        }
      }
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    const int* t = j->table + g * (kGroup + 1);
    for (int i = 1; i <= kGroup; ++i)
      if (t[i] >= 0) {
        const size_t o = static_cast<size_t>(t[i]) * j->req_bytes;
        std::memcpy(j->dst + o, j->src + o, j->req_bytes);
      }
  }
}

// Piece size for a staged transfer of `bytes`: four pieces, none under 512 KB.
size_t copy_piece(size_t bytes) { return std::max<size_t>(size_t(512) << 10, ((bytes + 3) / 4 + 4095) & ~size_t(4095)); }

cudaError_t ensure_pinned(unsigned char*& p, size_t& cap, size_t bytes) {
  if (bytes <= cap && p != nullptr) return cudaSuccess;
  if (p != nullptr) cudaFreeHost(p);
  p = nullptr;
  cap = 0;
  const cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&p), std::max<size_t>(bytes, 16), cudaHostAllocDefault);
  if (e == cudaSuccess) cap = bytes;
  return e;
}

// Waits for the stream and reports the device error word.
OrbitWarsCudaStatus finish(Workspace& W) {
  int herr = 0;
  T2_TRY(cudaMemcpyAsync(&herr, W.err, sizeof(int), cudaMemcpyDeviceToHost, W.stream));
  T2_TRY(cudaStreamSynchronize(W.stream));
  if (herr != 0) return rt(device_error_text(herr));
  return ok();
}

// Decode inputs and outputs of orbit_wars_cuda_true2d_decode_many_resident:
// host buffers, or (row_ids == nullptr) inputs already in W.dec_* (written by
// the device encoder).
struct DecodeIo {
  const int32_t* row_ids;
  const uint8_t* flags;
  const float* ships;
  int32_t* target_rows;
  int32_t* ship_counts;
};

// Runs the forward for `n` requests: inputs from the host buffer input_rows, or
// already in W.in when input_rows is nullptr (written by the device encoder).
OrbitWarsCudaStatus run_forward(Workspace& W, const float* input_rows, const size_t* model_indices, float* output_rows,
                                size_t n, const OrbitWarsCudaTrue2DShape& shape, const DecodeIo* dec = nullptr,
                                bool sync = true) {
  const T2Layout L = t2_layout(shape.layer_count, shape.row_count, shape.head_count);
  const T2Dev D = dev_layout(L);
  const size_t in_n = n * L.rows * kFeatures, out_n = n * L.rows * kOutPerRow, m_n = n * L.cells;
  if (input_rows != nullptr) T2_TRY(ensure(W.in, W.in_cap, in_n));
  T2_TRY(ensure(W.out, W.out_cap, out_n));
  T2_TRY(ensure(W.m, W.m_cap, m_n + n));  // cell matrices, then the attention's per-request path flags
  T2_TRY(ensure(W.idx, W.idx_cap, n));
  // device timing (profile_begin / profile_end): copies and kernels, one phase each
  const bool prof = W.prof_on && W.prof_used + 9 <= W.prof_events.size();
  auto mark = [&](const char* name) {
    if (prof) {
      cudaEventRecord(W.prof_events[W.prof_used], W.stream);
      W.prof_names[W.prof_used++] = name;
    }
  };
  const int models = static_cast<int>(W.models);
  // group the requests by model (counting sort; host-validated indices), kGroup per group
  std::vector<int>& gt = W.host_groups;
  gt.clear();
  {
    std::vector<int> start(static_cast<size_t>(models) + 1, 0), order(n);
    for (size_t r = 0; r < n; ++r) ++start[(model_indices != nullptr ? model_indices[r] : 0) + 1];
    for (int k = 0; k < models; ++k) start[k + 1] += start[k];
    std::vector<int> fill(start.begin(), start.end() - 1);
    for (size_t r = 0; r < n; ++r) order[fill[model_indices != nullptr ? model_indices[r] : 0]++] = static_cast<int>(r);
    for (int k = 0; k < models; ++k)
      for (int i = start[k]; i < start[k + 1]; i += kGroup) {
        gt.push_back(k);
        for (int j = 0; j < kGroup; ++j) gt.push_back(i + j < start[k + 1] ? order[i + j] : -1);
      }
  }
  const size_t n_groups = gt.size() / (kGroup + 1);
  T2_TRY(ensure(W.groups, W.groups_cap, gt.size()));
  // model indices and the group table go up from pinned memory too (a pageable
  // source would make each copy wait on the host); the previous call's copies
  // are done: every call that uses this staging ends synchronised
  const size_t idx_bytes = model_indices != nullptr ? n * sizeof(size_t) : 0, gt_bytes = gt.size() * sizeof(int);
  T2_TRY(ensure_pinned(W.pin_meta, W.pin_meta_cap, idx_bytes + gt_bytes));
  if (idx_bytes) std::memcpy(W.pin_meta, model_indices, idx_bytes);
  std::memcpy(W.pin_meta + idx_bytes, gt.data(), gt_bytes);
  mark("copy_rows_h2d");
  if (input_rows != nullptr) {
    T2_TRY(cudaMemsetAsync(W.err, 0, sizeof(int), W.stream));
    // host rows straight from the caller's (pageable) buffer: for the few MB of
    // rows a call carries, the driver's own staging measured faster than host
    // threads copying into pinned memory in pieces (129-139 against 155 us for
    // 1,024 requests)
    T2_TRY(cudaMemcpyAsync(W.in, input_rows, in_n * sizeof(float), cudaMemcpyHostToDevice, W.stream));
  }
  const size_t* didx = nullptr;
  if (model_indices != nullptr) {
    T2_TRY(cudaMemcpyAsync(W.idx, W.pin_meta, idx_bytes, cudaMemcpyHostToDevice, W.stream));
    didx = W.idx;
  }
  T2_TRY(cudaMemcpyAsync(W.groups, W.pin_meta + idx_bytes, gt_bytes, cudaMemcpyHostToDevice, W.stream));
  const dim3 g1((L.cells + 255) / 256, static_cast<unsigned>(n_groups));
  mark("t2_expand_pre");
  t2_expand_pre_g<<<g1, 256, 0, W.stream>>>(W.in, W.groups, W.weights, models, D, W.m, W.err);
  T2_TRY(cudaGetLastError());
  mark("t2_attention");
  T2_TRY(launch_t2_attention(didx, W.weights, models, D, W.m, W.err, reinterpret_cast<int*>(W.m + m_n),
                                  static_cast<unsigned>(n), W.stream));
  const dim3 g3((L.rows + kRowsPerCta - 1) / kRowsPerCta, static_cast<unsigned>(n_groups));
  const int threads3 = static_cast<int>(std::min<size_t>(512, std::max<size_t>(128, kRowsPerCta * L.rows)));
  mark("t2_post_collapse");
  // synchronous host-buffer forward without decode: the collapse writes the
  // outputs over PCIe into mapped pinned memory while it runs
  const bool mapped_out = output_rows != nullptr && dec == nullptr && sync;
  float* out_target = W.out;
  unsigned* done_dev = nullptr;
  if (mapped_out) {
    const size_t bytes = out_n * sizeof(float);
    if (bytes > W.pin_map_cap || W.pin_map == nullptr) {
      if (W.pin_map != nullptr) cudaFreeHost(W.pin_map);
      W.pin_map = nullptr;
      W.pin_map_cap = 0;
      T2_TRY(cudaHostAlloc(reinterpret_cast<void**>(&W.pin_map), bytes, cudaHostAllocMapped));
      W.pin_map_cap = bytes;
    }
    void* dp = nullptr;
    T2_TRY(cudaHostGetDevicePointer(&dp, W.pin_map, 0));
    out_target = static_cast<float*>(dp);
    const size_t words = static_cast<size_t>(g3.x) * g3.y;
    if (words > W.done_cap || W.done_map == nullptr) {
      if (W.done_map != nullptr) cudaFreeHost(W.done_map);
      W.done_map = nullptr;
      W.done_cap = 0;
      T2_TRY(cudaHostAlloc(reinterpret_cast<void**>(&W.done_map), words * sizeof(unsigned), cudaHostAllocMapped));
      std::memset(W.done_map, 0, words * sizeof(unsigned));
      W.done_cap = words;
    }
    if (++W.done_epoch == 0) {  // wrapped: clear the words so no stale one matches
      std::memset(W.done_map, 0, W.done_cap * sizeof(unsigned));
      W.done_epoch = 1;
    }
    void* dd = nullptr;
    T2_TRY(cudaHostGetDevicePointer(&dd, W.done_map, 0));
    done_dev = static_cast<unsigned*>(dd);
  }
  t2_post_collapse_g<<<g3, threads3, 0, W.stream>>>(W.groups, W.weights, models, D, W.m, out_target, W.err,
                                                    done_dev, W.done_epoch);
  T2_TRY(cudaGetLastError());
  mark(nullptr);
  if (dec != nullptr) {
    const size_t rn = n * L.rows, dn = n * L.rows * kTargets;
    if (dec->row_ids != nullptr) {
      T2_TRY(ensure_decode(W, rn));
      T2_TRY(cudaMemcpyAsync(W.dec_ids, dec->row_ids, rn * sizeof(int32_t), cudaMemcpyHostToDevice, W.stream));
      T2_TRY(cudaMemcpyAsync(W.dec_flags, dec->flags, rn, cudaMemcpyHostToDevice, W.stream));
      T2_TRY(cudaMemcpyAsync(W.dec_ships, dec->ships, rn * sizeof(float), cudaMemcpyHostToDevice, W.stream));
    }
    mark("t2_decode");
    t2_decode<<<static_cast<unsigned>(n), 512, 0, W.stream>>>(W.out, W.dec_ids, W.dec_flags, W.dec_ships,
                                                              D.rows, W.dec_rows, W.dec_counts, W.err);
    T2_TRY(cudaGetLastError());
    mark(nullptr);
    T2_TRY(cudaMemcpyAsync(dec->target_rows, W.dec_rows, dn * sizeof(int32_t), cudaMemcpyDeviceToHost, W.stream));
    T2_TRY(cudaMemcpyAsync(dec->ship_counts, W.dec_counts, dn * sizeof(int32_t), cudaMemcpyDeviceToHost, W.stream));
  }
  if (!sync) {
    if (output_rows != nullptr)
      T2_TRY(cudaMemcpyAsync(output_rows, W.out, out_n * sizeof(float), cudaMemcpyDeviceToHost, W.stream));
    return ok();
  }
  if (mapped_out) {
    // each group's rows go to the caller as soon as its CTAs are done; if a
    // wait ends without them (a device error, or a minute after the launches),
    // everything is copied once the stream has finished
    GroupCopy job;
    job.done = W.done_map;
    job.epoch = W.done_epoch;
    job.per_group = g3.x;
    job.table = gt.data();
    job.n_groups = n_groups;
    job.src = W.pin_map;
    job.dst = reinterpret_cast<unsigned char*>(output_rows);
    job.req_bytes = static_cast<size_t>(L.rows) * kOutPerRow * sizeof(float);
    job.stream = W.stream;
    job.deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    CopyPool& pool = CopyPool::get();
    pool.run_parts(group_copy, &job, pool.threads());
    const OrbitWarsCudaStatus st = finish(W);
    if (st.code == kOk && job.gave_up.load() != 0)
      par_copy(reinterpret_cast<unsigned char*>(output_rows), W.pin_map, out_n * sizeof(float));
    return st;
  }
  // outputs through pinned memory in pieces, an event after each piece's DMA:
  // host threads copy piece k out while piece k + 1 downloads
  if (output_rows != nullptr) {
    const size_t bytes = out_n * sizeof(float);
    T2_TRY(ensure_pinned(W.pin_out, W.pin_out_cap, bytes));
    const size_t piece = copy_piece(bytes), pieces = (bytes + piece - 1) / piece;
    while (W.out_pieces.size() < pieces) {
      cudaEvent_t ev;
      T2_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
      W.out_pieces.push_back(ev);
    }
    mark("copy_out_d2h");
    for (size_t k = 0; k < pieces; ++k) {
      const size_t o = k * piece;
      T2_TRY(cudaMemcpyAsync(W.pin_out + o, reinterpret_cast<const unsigned char*>(W.out) + o,
                             std::min(piece, bytes - o), cudaMemcpyDeviceToHost, W.stream));
      T2_TRY(cudaEventRecord(W.out_pieces[k], W.stream));
    }
    mark(nullptr);
    for (size_t k = 0; k < pieces; ++k) {
      T2_TRY(cudaEventSynchronize(W.out_pieces[k]));
      const size_t o = k * piece;
      par_copy(reinterpret_cast<unsigned char*>(output_rows) + o, W.pin_out + o, std::min(piece, bytes - o));
    }
  }
  return finish(W);
}

// ---------------------------------------------------------------- device encoder, host side
// AgentConfig::validate (crates/orbit-wars-core/src/config.rs:335-377) on the
// fields the encoder reads, plus the 64-row bound of EncodedState.
bool encoder_config_ok(const OrbitWarsEncoderConfig& c) {
  if (c.max_rows != c.initial_planet_slots + c.comet_slots + c.padding_slots) return false;
  if (c.max_rows == 0 || c.initial_planet_slots == 0 || c.max_rows > static_cast<size_t>(enc::kMaxRows)) return false;
  if (!(c.ship_log_pivot > 0.0f && c.ship_log_cap > c.ship_log_pivot)) return false;
  if (c.max_players != 4) return false;  // OWNER_CLASS_PLAYER_SLOTS
  const float cls[7] = {c.owner_class_own,     c.owner_class_enemy_1, c.owner_class_enemy_2,
                        c.owner_class_enemy_3, c.owner_class_neutral, c.owner_class_empty,
                        c.owner_class_absent_on_map};
  for (int i = 0; i < 7; ++i) {
    if (!std::isfinite(cls[i])) return false;
    for (int j = i + 1; j < 7; ++j)
      if (cls[i] == cls[j]) return false;
  }
  if (!(std::isfinite(c.board_size) && c.board_size > 0.0f)) return false;
  if (!(c.fleet_speed_max >= 1.0f)) return false;
  return true;
}

const char* encode_error_text(int code) {
  switch (code) {
    case enc::kInvalidConfig: return "encode failed: InvalidConfig";
    case enc::kInvalidOwnerClass: return "encode failed: InvalidOwnerClass";
    case enc::kMissingHome: return "encode failed: MissingHomePlanet";
    case enc::kRowOverflow: return "encode failed: RowOverflow";
    default: return "encode failed";
  }
}

bool offsets_ok(const size_t* off, size_t games, size_t* max_len) {
  if (off == nullptr || off[0] != 0) return false;
  size_t m = 0;
  for (size_t g = 0; g < games; ++g) {
    if (off[g + 1] < off[g]) return false;
    m = std::max(m, off[g + 1] - off[g]);
  }
  *max_len = m;
  return true;
}

// Validates the batch (before any device call), packs it into pinned memory,
// uploads it in one copy and launches the encoder into W.in (rows), W.dec_ids / dec_flags / dec_ships and
// W.enc_err, all on W.stream; W.err is cleared first.
OrbitWarsCudaStatus launch_encode(Workspace& W, const OrbitWarsGameBatch* games, const uint32_t* request_games,
                                  const int32_t* request_players, size_t n, const OrbitWarsEncoderConfig& cfg) {
  if (games == nullptr || request_games == nullptr || request_players == nullptr || n == 0 ||
      games->game_count == 0 || games->planets == nullptr || games->initial_planets == nullptr)
    return bad("invalid encode buffer");
  if (!encoder_config_ok(cfg)) return bad("invalid encoder config");
  const size_t G = games->game_count;
  const bool comets = games->comet_planet_ids != nullptr || games->comet_offsets != nullptr;
  size_t max_p = 0, max_i = 0, max_c = 0;
  if (!offsets_ok(games->planet_offsets, G, &max_p) || !offsets_ok(games->initial_offsets, G, &max_i) ||
      (comets && (games->comet_planet_ids == nullptr || !offsets_ok(games->comet_offsets, G, &max_c))))
    return bad("invalid game offsets");
  for (size_t r = 0; r < n; ++r)
    if (request_games[r] >= G) return bad("request game out of range");
  const size_t warp_bytes = enc::warp_smem_bytes(static_cast<int>(std::min<size_t>(max_p, 1 << 20)),
                                                 static_cast<int>(std::min<size_t>(max_i, 1 << 20)));
  constexpr size_t kSmemCap = 200 * 1024;
  if (max_p > 65535 || max_c > 65535 || warp_bytes > kSmemCap) return bad("game too large for the device encoder");
  const int warps = static_cast<int>(std::min<size_t>(enc::kWarps, kSmemCap / warp_bytes));
  T2_TRY(ensure_common(W));
  const size_t np = games->planet_offsets[G], ni = games->initial_offsets[G], nc = comets ? games->comet_offsets[G] : 0;
  auto up16 = [](size_t b) { return (b + 15) & ~size_t(15); };
  const size_t o_p = 0, o_i = o_p + up16(np * sizeof(enc::Planet)), o_c = o_i + up16(ni * sizeof(enc::Planet));
  const size_t o_po = o_c + up16(nc * sizeof(int32_t)), o_io = o_po + up16((G + 1) * 8), o_co = o_io + up16((G + 1) * 8);
  const size_t o_rg = o_co + up16((G + 1) * 8), o_rp = o_rg + up16(n * 4), total = o_rp + up16(n * 4);
  if (total > W.enc_host_cap) {
    if (W.enc_host != nullptr) cudaFreeHost(W.enc_host);
    W.enc_host = nullptr;
    W.enc_host_cap = 0;
    T2_TRY(cudaHostAlloc(reinterpret_cast<void**>(&W.enc_host), total, cudaHostAllocDefault));
    W.enc_host_cap = total;
  }
  T2_TRY(ensure(W.enc_dev, W.enc_dev_cap, total));
  T2_TRY(ensure(W.enc_err, W.enc_err_cap, n));
  unsigned char* h = W.enc_host;
  std::memcpy(h + o_p, games->planets, np * sizeof(enc::Planet));
  std::memcpy(h + o_i, games->initial_planets, ni * sizeof(enc::Planet));
  if (nc > 0) std::memcpy(h + o_c, games->comet_planet_ids, nc * sizeof(int32_t));
  std::memcpy(h + o_po, games->planet_offsets, (G + 1) * 8);
  std::memcpy(h + o_io, games->initial_offsets, (G + 1) * 8);
  if (comets) std::memcpy(h + o_co, games->comet_offsets, (G + 1) * 8);
  std::memcpy(h + o_rg, request_games, n * 4);
  std::memcpy(h + o_rp, request_players, n * 4);
  T2_TRY(cudaMemsetAsync(W.err, 0, sizeof(int), W.stream));
  T2_TRY(cudaMemcpyAsync(W.enc_dev, h, total, cudaMemcpyHostToDevice, W.stream));
  const size_t rn = n * cfg.max_rows;
  T2_TRY(ensure(W.in, W.in_cap, rn * kFeatures));
  T2_TRY(ensure_decode(W, rn));
  unsigned char* d = W.enc_dev;
  enc::Batch b{reinterpret_cast<const enc::Planet*>(d + o_p), reinterpret_cast<const unsigned long long*>(d + o_po),
               reinterpret_cast<const enc::Planet*>(d + o_i), reinterpret_cast<const unsigned long long*>(d + o_io),
               comets ? reinterpret_cast<const int32_t*>(d + o_c) : nullptr,
               comets ? reinterpret_cast<const unsigned long long*>(d + o_co) : nullptr,
               reinterpret_cast<const uint32_t*>(d + o_rg), reinterpret_cast<const int32_t*>(d + o_rp)};
  const enc::Cfg c{static_cast<int>(cfg.max_rows), static_cast<int>(cfg.initial_planet_slots),
                   static_cast<int>(cfg.comet_slots), static_cast<int>(cfg.max_players),
                   cfg.ship_log_pivot, cfg.ship_log_cap,
                   cfg.owner_class_own, cfg.owner_class_enemy_1, cfg.owner_class_enemy_2, cfg.owner_class_enemy_3,
                   cfg.owner_class_neutral, cfg.owner_class_empty, cfg.owner_class_absent_on_map,
                   cfg.board_size, cfg.fleet_speed_max};
  const enc::Out o{W.in, W.dec_ids, W.dec_flags, W.dec_ships, W.enc_err};
  const size_t smem = warp_bytes * warps;
  if (smem > 48 * 1024)
    T2_TRY(cudaFuncSetAttribute(enc::encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  const bool prof = W.prof_on && W.prof_used + 2 <= W.prof_events.size();
  if (prof) {
    cudaEventRecord(W.prof_events[W.prof_used], W.stream);
    W.prof_names[W.prof_used++] = "t2_encode";
  }
  const unsigned blocks = static_cast<unsigned>((n + warps - 1) / warps);
  enc::encode_kernel<<<blocks, warps * 32, smem, W.stream>>>(b, c, static_cast<int>(n), static_cast<int>(max_p),
                                                             static_cast<int>(max_i), warps, o);
  T2_TRY(cudaGetLastError());
  if (prof) {
    cudaEventRecord(W.prof_events[W.prof_used], W.stream);
    W.prof_names[W.prof_used++] = nullptr;
  }
  return ok();
}

// Copies the per-request encode errors back (after the stream is synchronised by
// the caller) and returns the first failing request's error.
OrbitWarsCudaStatus encode_result(Workspace& W, size_t n, int32_t* encode_errors) {
  int32_t* e = encode_errors;
  if (e == nullptr) {
    W.host_err.resize(n);
    e = W.host_err.data();
  }
  T2_TRY(cudaMemcpyAsync(e, W.enc_err, n * sizeof(int32_t), cudaMemcpyDeviceToHost, W.stream));
  T2_TRY(cudaStreamSynchronize(W.stream));
  for (size_t r = 0; r < n; ++r)
    if (e[r] != enc::kOk) return bad(encode_error_text(e[r]));
  return ok();
}


// ---------------------------------------------------------------- training step, host side

// One full-batch SGD step (orbit_wars_cuda.cu:2823-3330): samples are sorted by
// model (stable counting sort) and processed in chunks of at most
// batch_sample_count; every chunk runs forward with history, loss, backward and
// adds its gradients to the per-model sums; the update is applied once at the end.
OrbitWarsCudaStatus train_step(Workspace& W, const float* input_rows, const float* output_rows, const int* rewards,
                               const float* target_action_rewards, const size_t* model_indices, float* all_weights,
                               size_t sample_count, size_t model_count, const OrbitWarsCudaTrue2DShape& shape,
                               const OrbitWarsCudaTrue2DTrainingConfig& tc) {
  const T2Layout Ly = t2_layout(shape.layer_count, shape.row_count, shape.head_count);
  const T2Dev D = ref_layout_dev(Ly);
  const size_t rows = Ly.rows, cells = Ly.cells, layers = Ly.layers, heads = Ly.heads, total = Ly.total;
  const size_t n_out = 2 * rows * kTargets + kOutScalars * kTargets;
  const size_t cap = std::min<size_t>(std::min<size_t>(tc.batch_sample_count, sample_count), 65535);
  // order: samples sorted by model; counts per model over the whole call
  std::vector<int> count(model_count, 0), order(sample_count);
  for (size_t i = 0; i < sample_count; ++i) ++count[model_indices[i]];
  {
    std::vector<size_t> fill(model_count + 1, 0);
    for (size_t m = 0; m < model_count; ++m) fill[m + 1] = fill[m] + static_cast<size_t>(count[m]);
    for (size_t i = 0; i < sample_count; ++i) order[fill[model_indices[i]]++] = static_cast<int>(i);
  }
  // device buffers (freed on every exit path)
  // one device arena for every buffer of the step, kept between calls and
  // grown when a call needs more (the population's buffers are separate)
  const size_t ctas = (cells + 255) / 256;
  size_t need = 0;
  auto carve = [&](size_t bytes) {
    const size_t o = need;
    need += (std::max<size_t>(bytes, 4) + 255) & ~size_t(255);
    return o;
  };
  const size_t o_w = carve(model_count * total * sizeof(float)), o_g = carve(model_count * total * sizeof(float));
  const size_t o_count = carve(model_count * sizeof(int)), o_x = carve(cap * rows * kFeatures * sizeof(float));
  const size_t o_out = carve(cap * rows * kOutPerRow * sizeof(float)), o_tar = carve(cap * rows * kTargets * sizeof(float));
  const size_t o_rew = carve(cap * sizeof(int)), o_model = carve(cap * sizeof(int));
  const size_t o_mstart = carve((model_count + 1) * sizeof(int));
  const size_t o_hist = carve(cap * (layers + 2) * cells * sizeof(float));
  const size_t o_grad = carve(cap * (layers + 2) * cells * sizeof(float));
  const size_t o_attv = carve(cap * cells * sizeof(float)), o_attg = carve(cap * cells * sizeof(float));
  const size_t o_stats = carve(cap * heads * 3 * cells * sizeof(float));
  const size_t o_gpart = carve(cap * kTargets * cells * sizeof(float)), o_opart = carve(cap * n_out * sizeof(float));
  const size_t o_hpart = carve(cap * heads * 8 * sizeof(float)), o_igrad = carve(cap * heads * cells * sizeof(float));
  const size_t o_cpart = carve(model_count * cells * 16 * sizeof(float)), o_hcta = carve(cap * ctas * 8 * sizeof(float));
  if (need > W.train_cap || W.train_arena == nullptr) {
    if (W.train_arena != nullptr) cudaFree(W.train_arena);
    W.train_arena = nullptr;
    W.train_cap = 0;
    T2_TRY(cudaMalloc(reinterpret_cast<void**>(&W.train_arena), need));
    W.train_cap = need;
  }
  unsigned char* ab = W.train_arena;
  float* dw = reinterpret_cast<float*>(ab + o_w);
  float* dg = reinterpret_cast<float*>(ab + o_g);
  int* dcount = reinterpret_cast<int*>(ab + o_count);
  float* dx = reinterpret_cast<float*>(ab + o_x);
  float* dout = reinterpret_cast<float*>(ab + o_out);
  float* dtar = reinterpret_cast<float*>(ab + o_tar);
  int* drew = reinterpret_cast<int*>(ab + o_rew);
  int* dmodel = reinterpret_cast<int*>(ab + o_model);
  int* dmstart = reinterpret_cast<int*>(ab + o_mstart);
  float* hist = reinterpret_cast<float*>(ab + o_hist);
  float* grad = reinterpret_cast<float*>(ab + o_grad);
  float* attv = reinterpret_cast<float*>(ab + o_attv);
  float* attg = reinterpret_cast<float*>(ab + o_attg);
  float* stats = reinterpret_cast<float*>(ab + o_stats);
  float* gpart = reinterpret_cast<float*>(ab + o_gpart);
  float* opart = reinterpret_cast<float*>(ab + o_opart);
  float* hpart = reinterpret_cast<float*>(ab + o_hpart);
  float* igrad = reinterpret_cast<float*>(ab + o_igrad);
  float* cpart = reinterpret_cast<float*>(ab + o_cpart);
  float* hcta = reinterpret_cast<float*>(ab + o_hcta);
  // pinned staging of the weights, kept between calls
  const size_t wbytes = model_count * total * sizeof(float);
  if (wbytes > W.train_pin_cap || W.train_pin == nullptr) {
    if (W.train_pin != nullptr) cudaFreeHost(W.train_pin);
    W.train_pin = nullptr;
    W.train_pin_cap = 0;
    T2_TRY(cudaHostAlloc(reinterpret_cast<void**>(&W.train_pin), wbytes, cudaHostAllocDefault));
    W.train_pin_cap = wbytes;
  }
  cudaStream_t st = W.stream;
  // device timing (profile_begin / profile_end): copies and kernel phases
  auto mark = [&](const char* name) {
    if (W.prof_on && W.prof_used < W.prof_events.size()) {
      cudaEventRecord(W.prof_events[W.prof_used], st);
      W.prof_names[W.prof_used++] = name;
    }
  };
  mark("train_weights_h2d");
  // weights up in 16 MB pieces: a piece is copied into pinned memory by host
  // threads while the previous piece's DMA runs
  constexpr size_t kPiece = size_t(16) << 20;
  for (size_t o = 0; o < wbytes; o += kPiece) {
    const size_t b = std::min(kPiece, wbytes - o);
    par_copy(W.train_pin + o, reinterpret_cast<const unsigned char*>(all_weights) + o, b);
    T2_TRY(cudaMemcpyAsync(reinterpret_cast<unsigned char*>(dw) + o, W.train_pin + o, b, cudaMemcpyHostToDevice, st));
  }
  T2_TRY(cudaMemsetAsync(dg, 0, model_count * total * sizeof(float), st));
  T2_TRY(cudaMemcpyAsync(dcount, count.data(), model_count * sizeof(int), cudaMemcpyHostToDevice, st));
  // shared memory: the mid state (forward) and five per-cell vectors (backward) when they fit
  const size_t fwd_smem = cells * sizeof(float), bwd_smem = 5 * cells * sizeof(float);
  const int fwd_sm = fwd_smem <= 200 * 1024, bwd_sm = bwd_smem <= 200 * 1024;
  if (fwd_sm && fwd_smem > 48 * 1024)
    T2_TRY(cudaFuncSetAttribute(t2tr::fwd_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(fwd_smem)));
  if (bwd_sm && bwd_smem > 48 * 1024)
    T2_TRY(cudaFuncSetAttribute(t2tr::bwd_attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(bwd_smem)));
  // the prepared-term backward (512 threads, six floats per cell) where it fits
  const size_t prep_smem = 6 * cells * sizeof(float);
  const bool prep_sm = prep_smem <= 200 * 1024;
  const unsigned cb512 = static_cast<unsigned>((cells + 511) / 512);
  if (prep_sm && prep_smem > 48 * 1024)
    T2_TRY(cudaFuncSetAttribute(t2tr::bwd_attention_smem, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(prep_smem)));
  // staged chunk inputs in sorted order
  std::vector<float> hx(cap * rows * kFeatures), hout(cap * rows * kOutPerRow), htar(cap * rows * kTargets);
  std::vector<int> hrew(cap), hmodel(cap), hmstart(model_count + 1);
  t2tr::Tr t{};
  t.L = D;
  t.w = dw;
  t.g = dg;
  t.x = dx;
  t.out = dout;
  t.rewards = drew;
  t.tar = dtar;
  t.model = dmodel;
  t.mstart = dmstart;
  t.models = static_cast<int>(model_count);
  t.hist = hist;
  t.grad = grad;
  t.attv = attv;
  t.att_grad = attg;
  t.stats = stats;
  t.gpart = gpart;
  t.opart = opart;
  t.hpart = hpart;
  t.igrad = igrad;
  t.cpart = cpart;
  t.owner_own = tc.owner_class_own;
  t.owner_empty = tc.owner_class_empty;
  t.owner_absent = tc.owner_class_absent_on_map;
  t.reward_normalizer = tc.reward_normalizer;
  t.send_threshold = tc.send_threshold;
  t.learning_rate = tc.learning_rate;
  const unsigned cb = static_cast<unsigned>(ctas);
  const unsigned mid = static_cast<unsigned>(D.mid);
  for (size_t off = 0; off < sample_count; off += cap) {
    const size_t n = std::min(cap, sample_count - off);
    std::fill(hmstart.begin(), hmstart.end(), 0);
    for (size_t k = 0; k < n; ++k) {
      const size_t i = static_cast<size_t>(order[off + k]);
      std::memcpy(&hx[k * rows * kFeatures], input_rows + i * rows * kFeatures, rows * kFeatures * sizeof(float));
      std::memcpy(&hout[k * rows * kOutPerRow], output_rows + i * rows * kOutPerRow, rows * kOutPerRow * sizeof(float));
      std::memcpy(&htar[k * rows * kTargets], target_action_rewards + i * rows * kTargets, rows * kTargets * sizeof(float));
      hrew[k] = rewards[i];
      hmodel[k] = static_cast<int>(model_indices[i]);
      ++hmstart[model_indices[i] + 1];
    }
    for (size_t m = 0; m < model_count; ++m) hmstart[m + 1] += hmstart[m];
    mark("train_samples_h2d");
    T2_TRY(cudaMemcpyAsync(dx, hx.data(), n * rows * kFeatures * sizeof(float), cudaMemcpyHostToDevice, st));
    T2_TRY(cudaMemcpyAsync(dout, hout.data(), n * rows * kOutPerRow * sizeof(float), cudaMemcpyHostToDevice, st));
    T2_TRY(cudaMemcpyAsync(dtar, htar.data(), n * rows * kTargets * sizeof(float), cudaMemcpyHostToDevice, st));
    T2_TRY(cudaMemcpyAsync(drew, hrew.data(), n * sizeof(int), cudaMemcpyHostToDevice, st));
    T2_TRY(cudaMemcpyAsync(dmodel, hmodel.data(), n * sizeof(int), cudaMemcpyHostToDevice, st));
    T2_TRY(cudaMemcpyAsync(dmstart, hmstart.data(), (model_count + 1) * sizeof(int), cudaMemcpyHostToDevice, st));
    T2_TRY(cudaMemsetAsync(grad, 0, n * (layers + 2) * cells * sizeof(float), st));
    t.n = static_cast<int>(n);
    const dim3 gs(cb, static_cast<unsigned>(n)), gm(cb, static_cast<unsigned>(model_count));
    // forward with history
    mark("train_forward");
    t2tr::fwd_matrix<<<gs, 256, 0, st>>>(t, 0, static_cast<int>(mid), 1);
    t2tr::fwd_attention<<<gs, 256, fwd_sm ? fwd_smem : 0, st>>>(t, fwd_sm);
    t2tr::fwd_matrix<<<gs, 256, 0, st>>>(t, static_cast<int>(mid), static_cast<int>(layers), 0);
    // loss
    mark("train_loss");
    t2tr::loss_backward<<<dim3(static_cast<unsigned>(kTargets), static_cast<unsigned>(n)),
                          static_cast<unsigned>((rows + 31) / 32 * 32), 0, st>>>(t);
    t2tr::sum_actions<<<gs, 256, 0, st>>>(t);
    // backward
    mark("train_backward_matrix");
    for (int l = static_cast<int>(layers) - 1; l >= static_cast<int>(mid); --l) t2tr::bwd_matrix<<<gm, 256, 0, st>>>(t, l);
    mark("train_backward_attention");
    t2tr::bwd_apply<<<gm, 256, 0, st>>>(t);
    t2tr::reduce_shared<<<static_cast<unsigned>(model_count), 32, 0, st>>>(t);
    for (int h = 0; h < static_cast<int>(heads); ++h) {
      if (prep_sm) {
        t2tr::bwd_attention_smem<<<dim3(cb512, static_cast<unsigned>(n)), 512, prep_smem, st>>>(t, h, hcta);
        t2tr::sum_heads<<<gs, 256, 0, st>>>(t, h, hcta, static_cast<int>(cb512));
      } else {
        t2tr::bwd_attention<<<gs, 256, bwd_sm ? bwd_smem : 0, st>>>(t, h, hcta, bwd_sm);
        t2tr::sum_heads<<<gs, 256, 0, st>>>(t, h, hcta, static_cast<int>(ctas));
      }
    }
    t2tr::reduce_heads<<<static_cast<unsigned>(model_count), static_cast<unsigned>(heads * 8), 0, st>>>(t);
    mark("train_backward_matrix");
    for (int l = static_cast<int>(mid) - 1; l >= 0; --l) t2tr::bwd_matrix<<<gm, 256, 0, st>>>(t, l);
    mark("train_backward_expand_reduce");
    t2tr::bwd_expand<<<gm, 256, 0, st>>>(t);
    t2tr::reduce_expand<<<static_cast<unsigned>(model_count), 128, 0, st>>>(t);
    t2tr::reduce_output<<<dim3(static_cast<unsigned>((n_out + 127) / 128), static_cast<unsigned>(model_count)), 128, 0,
                          st>>>(t);
    T2_TRY(cudaGetLastError());
    mark(nullptr);
    // the host staging vectors are rewritten by the next chunk
    T2_TRY(cudaStreamSynchronize(st));
  }
  const long long all = static_cast<long long>(model_count) * static_cast<long long>(total);
  mark("train_sgd_d2h");
  t2tr::apply_sgd<<<static_cast<unsigned>((all + 255) / 256), 256, 0, st>>>(dw, dg, dcount, static_cast<int>(model_count),
                                                                          static_cast<long long>(total), tc.learning_rate);
  T2_TRY(cudaGetLastError());
  // weights down in pieces: each piece leaves pinned memory by host threads as soon as its DMA is done
  std::vector<cudaEvent_t> piece_ev;
  for (size_t o = 0; o < wbytes; o += kPiece) {
    const size_t b = std::min(kPiece, wbytes - o);
    T2_TRY(cudaMemcpyAsync(W.train_pin + o, reinterpret_cast<unsigned char*>(dw) + o, b, cudaMemcpyDeviceToHost, st));
    cudaEvent_t ev;
    T2_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    piece_ev.push_back(ev);
    T2_TRY(cudaEventRecord(ev, st));
  }
  mark(nullptr);
  cudaError_t e = cudaSuccess;
  for (size_t k = 0, o = 0; k < piece_ev.size(); ++k, o += kPiece) {
    if (e == cudaSuccess) e = cudaEventSynchronize(piece_ev[k]);
    if (e == cudaSuccess)
      par_copy(reinterpret_cast<unsigned char*>(all_weights) + o, W.train_pin + o, std::min(kPiece, wbytes - o));
    cudaEventDestroy(piece_ev[k]);
  }
  T2_TRY(e);
  T2_TRY(cudaStreamSynchronize(st));
  return ok();
}

}  // namespace

// ---------------------------------------------------------------- MUFU rate probe
// Throughput of the special-function pipe, the bound of the True2D matrix
// layers: one CTA of 1024 threads per SM, each thread running 8 independent
// chains of `op` (0: ex2.approx.ftz.f32 of the negated value, which keeps the
// chain in (0, 1]; 1: rcp.approx.ftz.f32 of 1 + v, which converges to 0.618:
// a bare rcp chain would alternate v and 1/v, and the assembler may fold
// rcp(rcp(v)) away), so the pipe, not a dependency, sets the pace. Each CTA
// records its clock64 span.
template <int OP>
__global__ void __launch_bounds__(1024, 1) mufu_rate_kernel(int iters, float* sink, long long* cycles) {
  float v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = 0.25f + 0.0625f * k + 1e-6f * threadIdx.x;
  __syncthreads();
  const long long c0 = clock64();
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (OP == 0)
        asm volatile("{\n\t.reg .f32 t;\n\tneg.f32 t, %1;\n\tex2.approx.ftz.f32 %0, t;\n\t}" : "=f"(v[k]) : "f"(v[k]));
      else
        asm volatile("{\n\t.reg .f32 t;\n\tadd.f32 t, %1, 0f3F800000;\n\trcp.approx.ftz.f32 %0, t;\n\t}"
                     : "=f"(v[k]) : "f"(v[k]));
    }
  }
  __syncthreads();
  const long long c1 = clock64();
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) acc += v[k];
  if (acc == -1.0f) sink[threadIdx.x] = acc;  // never true: keeps the chains live
  if (threadIdx.x == 0) cycles[blockIdx.x] = c1 - c0;
}

extern "C" {

OrbitWarsCudaStatus orbit_wars_cuda_status(void) {
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return from_cuda(e);
  if (n <= 0) return rt("no cuda devices");
  return {kOk, "cuda device available"};
}

OrbitWarsCudaStatus orbit_wars_cuda_encode_identity_batch(const float* input_rows, float* output_rows,
                                                          size_t game_count, size_t row_count, size_t feature_count) {
  if (input_rows == nullptr || output_rows == nullptr || game_count == 0 || row_count == 0 || feature_count == 0)
    return bad("invalid batch buffer");
  const size_t n = game_count * row_count * feature_count;
  const bool aligned = (reinterpret_cast<uintptr_t>(input_rows) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(output_rows) % 16 == 0);
  const size_t n4 = aligned ? n / 4 : 0;
  const size_t tail = n - n4 * 4;
  if (tail > 1024) {
    // unaligned large copy: plain device-to-device copy
    T2_TRY(cudaMemcpy(output_rows, input_rows, n * sizeof(float), cudaMemcpyDeviceToDevice));
    return from_cuda(cudaDeviceSynchronize());
  }
  const int blocks = static_cast<int>(std::min<size_t>((n4 + 255) / 256 + 1, 148 * 16));
  copy_kernel<<<blocks, 256>>>(reinterpret_cast<const float4*>(input_rows), reinterpret_cast<float4*>(output_rows), n4,
                               input_rows + n4 * 4, output_rows + n4 * 4, tail);
  T2_TRY(cudaGetLastError());
  return from_cuda(cudaDeviceSynchronize());
}

OrbitWarsCudaStatus orbit_wars_cuda_trainable_forward(const float* input_rows, const float* weights,
                                                      float* output_rows, size_t game_count,
                                                      OrbitWarsCudaTransformerShape shape) {
  if (input_rows == nullptr || weights == nullptr || output_rows == nullptr || game_count == 0)
    return bad("invalid trainable buffer");
  // orbit_wars_cuda.cu:281-285 shape rule (d in [8, 256], heads | d)
  if (shape.layer_count == 0 || shape.d_model < 8 || shape.d_model > 256 || shape.head_count == 0 ||
      shape.row_count == 0 || shape.d_model % shape.head_count != 0 || shape.row_count > 256)
    return bad("invalid transformer shape");
  const size_t d = shape.d_model, rows = shape.row_count, L = shape.layer_count;
  const size_t wcount = 2 * d + d + L * d + 2 * d;
  const size_t in_n = game_count * rows * 2, out_n = game_count * rows * 2;
  const size_t smem = 2 * rows * d * sizeof(float);
  if (smem > 200 * 1024) return bad("trainable shape too large for one CTA");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  T2_TRY(ensure_common(W));
  float *dw = nullptr, *din = nullptr, *dout = nullptr;
  T2_TRY(cudaMalloc(&dw, wcount * sizeof(float)));
  cudaError_t e = cudaMalloc(&din, in_n * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&dout, out_n * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpyAsync(dw, weights, wcount * sizeof(float), cudaMemcpyHostToDevice, W.stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(din, input_rows, in_n * sizeof(float), cudaMemcpyHostToDevice, W.stream);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(trainable_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) {
    trainable_kernel<<<static_cast<unsigned>(game_count), 256, smem, W.stream>>>(
        din, dw, dout, static_cast<int>(rows), static_cast<int>(d), static_cast<int>(shape.head_count),
        static_cast<int>(L));
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(output_rows, dout, out_n * sizeof(float), cudaMemcpyDeviceToHost, W.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(W.stream);
  cudaFree(dw);
  cudaFree(din);
  cudaFree(dout);
  return from_cuda(e);
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward(const float* input_rows, const float* weights, float* output_rows,
                                                   size_t game_count, OrbitWarsCudaTrue2DShape shape) {
  if (input_rows == nullptr || weights == nullptr || output_rows == nullptr || game_count == 0)
    return bad("invalid true2d buffer");
  if (!shape_ok(shape)) return bad("invalid true2d shape");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  T2_TRY(ensure_common(W));
  // single-model call: uploads that model (the resident population is replaced)
  OrbitWarsCudaStatus s = upload(W, weights, 1, shape);
  if (s.code != kOk) return s;
  W.resident = false;  // a single-model upload is not a population
  return run_forward(W, input_rows, nullptr, output_rows, game_count, shape);
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward_many(const float* input_rows, const size_t* model_indices,
                                                        const float* all_weights, float* output_rows,
                                                        size_t request_count, size_t model_count,
                                                        OrbitWarsCudaTrue2DShape shape) {
  if (input_rows == nullptr || model_indices == nullptr || all_weights == nullptr || output_rows == nullptr ||
      request_count == 0 || model_count == 0)
    return bad("invalid true2d many buffer");
  if (!shape_ok(shape)) return bad("invalid true2d shape");
  for (size_t r = 0; r < request_count; ++r)
    if (model_indices[r] >= model_count) return bad("model index out of range");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  T2_TRY(ensure_common(W));
  OrbitWarsCudaStatus s = upload(W, all_weights, model_count, shape);
  if (s.code != kOk) return s;
  W.request_capacity = std::max(W.request_capacity, request_count);
  return run_forward(W, input_rows, model_indices, output_rows, request_count, shape);
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_upload_population(const float* all_weights, size_t model_count,
                                                             size_t request_capacity,
                                                             OrbitWarsCudaTrue2DShape shape) {
  if (all_weights == nullptr || model_count == 0 || request_capacity == 0) return bad("invalid true2d population");
  if (!shape_ok(shape)) return bad("invalid true2d shape");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  T2_TRY(ensure_common(W));
  OrbitWarsCudaStatus s = upload(W, all_weights, model_count, shape);
  if (s.code != kOk) return s;
  // size the per-call buffers for the capacity up front (orbit_wars_cuda.cu:505-573)
  const T2Layout L = t2_layout(shape.layer_count, shape.row_count, shape.head_count);
  T2_TRY(ensure(W.in, W.in_cap, request_capacity * L.rows * kFeatures));
  T2_TRY(ensure(W.out, W.out_cap, request_capacity * L.rows * kOutPerRow));
  T2_TRY(ensure(W.m, W.m_cap, request_capacity * (L.cells + 1)));
  T2_TRY(ensure(W.idx, W.idx_cap, request_capacity));
  W.request_capacity = request_capacity;
  return from_cuda(cudaStreamSynchronize(W.stream));
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward_many_resident(const float* input_rows,
                                                                 const size_t* model_indices, float* output_rows,
                                                                 size_t request_count,
                                                                 OrbitWarsCudaTrue2DShape shape) {
  if (input_rows == nullptr || model_indices == nullptr || output_rows == nullptr || request_count == 0)
    return bad("invalid true2d resident buffer");
  if (!shape_ok(shape)) return bad("invalid true2d shape");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  if (!W.resident) return rt("true2d population is not loaded");  // orbit_wars_cuda.cu:2808-2813
  if (!same_shape(W.shape, shape)) return bad("true2d shape differs from the resident population");
  if (request_count > W.request_capacity) return rt("true2d request capacity exceeded");
  for (size_t r = 0; r < request_count; ++r)
    if (model_indices[r] >= W.models) return bad("model index out of range");
  return run_forward(W, input_rows, model_indices, output_rows, request_count, shape);
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_decode_many_resident(
    const float* input_rows, const size_t* model_indices, const int32_t* row_planet_ids, const uint8_t* row_flags,
    const float* source_ships, int32_t* target_rows, int32_t* ship_counts, float* output_rows, size_t request_count,
    OrbitWarsCudaTrue2DShape shape) {
  if (input_rows == nullptr || model_indices == nullptr || row_planet_ids == nullptr || row_flags == nullptr ||
      source_ships == nullptr || target_rows == nullptr || ship_counts == nullptr || request_count == 0)
    return bad("invalid true2d decode buffer");
  if (!shape_ok(shape)) return bad("invalid true2d shape");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  if (!W.resident) return rt("true2d population is not loaded");
  if (!same_shape(W.shape, shape)) return bad("true2d shape differs from the resident population");
  if (request_count > W.request_capacity) return rt("true2d request capacity exceeded");
  for (size_t r = 0; r < request_count; ++r)
    if (model_indices[r] >= W.models) return bad("model index out of range");
  const DecodeIo dec{row_planet_ids, row_flags, source_ships, target_rows, ship_counts};
  return run_forward(W, input_rows, model_indices, output_rows, request_count, shape, &dec);
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_decode_outputs(const float* output_rows, const int32_t* row_planet_ids,
                                                          const uint8_t* row_flags, const float* source_ships,
                                                          int32_t* target_rows, int32_t* ship_counts,
                                                          size_t request_count, size_t row_count) {
  if (output_rows == nullptr || row_planet_ids == nullptr || row_flags == nullptr || source_ships == nullptr ||
      target_rows == nullptr || ship_counts == nullptr || request_count == 0)
    return bad("invalid true2d decode buffer");
  if (row_count < kMinRows || row_count > kMaxRows) return bad("invalid row count");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  T2_TRY(ensure_common(W));
  const size_t out_n = request_count * row_count * kOutPerRow;
  T2_TRY(ensure(W.out, W.out_cap, out_n));
  T2_TRY(cudaMemsetAsync(W.err, 0, sizeof(int), W.stream));
  T2_TRY(cudaMemcpyAsync(W.out, output_rows, out_n * sizeof(float), cudaMemcpyHostToDevice, W.stream));
  const size_t rn = request_count * row_count, dn = rn * kTargets;
  T2_TRY(ensure_decode(W, rn));
  T2_TRY(cudaMemcpyAsync(W.dec_ids, row_planet_ids, rn * sizeof(int32_t), cudaMemcpyHostToDevice, W.stream));
  T2_TRY(cudaMemcpyAsync(W.dec_flags, row_flags, rn, cudaMemcpyHostToDevice, W.stream));
  T2_TRY(cudaMemcpyAsync(W.dec_ships, source_ships, rn * sizeof(float), cudaMemcpyHostToDevice, W.stream));
  t2_decode<<<static_cast<unsigned>(request_count), 512, 0, W.stream>>>(
      W.out, W.dec_ids, W.dec_flags, W.dec_ships, static_cast<int>(row_count), W.dec_rows, W.dec_counts, W.err);
  T2_TRY(cudaGetLastError());
  T2_TRY(cudaMemcpyAsync(target_rows, W.dec_rows, dn * sizeof(int32_t), cudaMemcpyDeviceToHost, W.stream));
  T2_TRY(cudaMemcpyAsync(ship_counts, W.dec_counts, dn * sizeof(int32_t), cudaMemcpyDeviceToHost, W.stream));
  return finish(W);
}

// config.rs:1-19 defaults of the fields the encoder reads.
void orbit_wars_encoder_config_default(OrbitWarsEncoderConfig* out) {
  if (out == nullptr) return;
  out->max_rows = 64;
  out->initial_planet_slots = 40;
  out->comet_slots = 20;
  out->padding_slots = 4;
  out->ship_log_pivot = 1000.0f;
  out->ship_log_cap = 100000.0f;
  out->max_players = 4;
  out->owner_class_own = 1.0f;
  out->owner_class_enemy_1 = 0.75f;
  out->owner_class_enemy_2 = 0.5f;
  out->owner_class_enemy_3 = 0.25f;
  out->owner_class_neutral = 0.0f;
  out->owner_class_empty = -0.5f;
  out->owner_class_absent_on_map = -1.0f;
  out->board_size = 100.0f;
  out->fleet_speed_max = 6.0f;
}

OrbitWarsCudaStatus orbit_wars_cuda_encode_states(const OrbitWarsGameBatch* games, const uint32_t* request_games,
                                                  const int32_t* request_players, size_t request_count,
                                                  const OrbitWarsEncoderConfig* config, float* input_rows,
                                                  int32_t* row_planet_ids, uint8_t* row_flags, float* row_ships,
                                                  int32_t* encode_errors) {
  if (config == nullptr || input_rows == nullptr || row_planet_ids == nullptr || row_flags == nullptr)
    return bad("invalid encode buffer");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  const OrbitWarsCudaStatus s = launch_encode(W, games, request_games, request_players, request_count, *config);
  if (s.code != kOk) return s;
  const size_t rn = request_count * config->max_rows;
  T2_TRY(cudaMemcpyAsync(input_rows, W.in, rn * kFeatures * sizeof(float), cudaMemcpyDeviceToHost, W.stream));
  T2_TRY(cudaMemcpyAsync(row_planet_ids, W.dec_ids, rn * sizeof(int32_t), cudaMemcpyDeviceToHost, W.stream));
  T2_TRY(cudaMemcpyAsync(row_flags, W.dec_flags, rn, cudaMemcpyDeviceToHost, W.stream));
  if (row_ships != nullptr)
    T2_TRY(cudaMemcpyAsync(row_ships, W.dec_ships, rn * sizeof(float), cudaMemcpyDeviceToHost, W.stream));
  return encode_result(W, request_count, encode_errors);
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_play_many_resident(
    const OrbitWarsGameBatch* games, const uint32_t* request_games, const int32_t* request_players,
    const size_t* model_indices, size_t request_count, const OrbitWarsEncoderConfig* config, int32_t* row_planet_ids,
    int32_t* target_rows, int32_t* ship_counts, int32_t* encode_errors, float* input_rows, float* output_rows,
    OrbitWarsCudaTrue2DShape shape) {
  if (config == nullptr || model_indices == nullptr || row_planet_ids == nullptr || target_rows == nullptr ||
      ship_counts == nullptr || request_count == 0)
    return bad("invalid true2d play buffer");
  if (!shape_ok(shape)) return bad("invalid true2d shape");
  if (config->max_rows != shape.row_count) return bad("encoder rows differ from the model rows");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  if (!W.resident) return rt("true2d population is not loaded");
  if (!same_shape(W.shape, shape)) return bad("true2d shape differs from the resident population");
  if (request_count > W.request_capacity) return rt("true2d request capacity exceeded");
  for (size_t r = 0; r < request_count; ++r)
    if (model_indices[r] >= W.models) return bad("model index out of range");
  OrbitWarsCudaStatus s = launch_encode(W, games, request_games, request_players, request_count, *config);
  if (s.code != kOk) return s;
  const size_t rn = request_count * shape.row_count;
  const DecodeIo dec{nullptr, nullptr, nullptr, target_rows, ship_counts};
  s = run_forward(W, nullptr, model_indices, output_rows, request_count, shape, &dec, false);
  if (s.code != kOk) return s;
  T2_TRY(cudaMemcpyAsync(row_planet_ids, W.dec_ids, rn * sizeof(int32_t), cudaMemcpyDeviceToHost, W.stream));
  if (input_rows != nullptr)
    T2_TRY(cudaMemcpyAsync(input_rows, W.in, rn * kFeatures * sizeof(float), cudaMemcpyDeviceToHost, W.stream));
  const OrbitWarsCudaStatus e = encode_result(W, request_count, encode_errors);
  const OrbitWarsCudaStatus f = finish(W);
  return e.code != kOk ? e : f;
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_train_full_attention(
    const float* input_rows, const float* output_rows, const int* rewards, const float* target_action_rewards,
    const size_t* model_indices, float* all_weights, size_t sample_count, size_t model_count,
    OrbitWarsCudaTrue2DShape shape, OrbitWarsCudaTrue2DTrainingConfig training_config) {
  // argument checks of orbit_wars_cuda.cu:2834-2850
  const OrbitWarsCudaTrue2DTrainingConfig& tc = training_config;
  const bool config_ok = tc.batch_sample_count > 0 && tc.learning_rate > 0.0f && tc.reward_normalizer > 0.0f &&
                         tc.send_threshold >= 0.0f && tc.send_threshold <= 1.0f;
  if (input_rows == nullptr || output_rows == nullptr || rewards == nullptr || target_action_rewards == nullptr ||
      model_indices == nullptr || all_weights == nullptr || sample_count == 0 || model_count == 0 ||
      !shape_ok(shape) || !config_ok)
    return bad("invalid true2d training batch");
  for (size_t i = 0; i < sample_count; ++i)
    if (model_indices[i] >= model_count) return bad("true2d training model index out of range");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  T2_TRY(ensure_common(W));
  return train_step(W, input_rows, output_rows, rewards, target_action_rewards, model_indices, all_weights,
                    sample_count, model_count, shape, tc);
}

// Allocation-free variant of orbit_wars_cuda_true2d_forward (no counterpart in
// the reference): device buffers in, device buffers out, scratch from the
// fixed device array above. Enqueued on `stream`; no cudaMalloc/cudaFree.
OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward_noalloc(const float* input_rows, const float* weights,
                                                           float* output_rows, size_t game_count,
                                                           OrbitWarsCudaTrue2DShape shape, void* stream) {
  if (input_rows == nullptr || weights == nullptr || output_rows == nullptr || game_count == 0)
    return bad("invalid true2d buffer");
  if (!shape_ok(shape)) return bad("invalid true2d shape");
  const T2Layout L = t2_layout(shape.layer_count, shape.row_count, shape.head_count);
  if (game_count > kNoAllocCells / (L.cells + 1))
    return bad("game_count x (row_count^2 + 1) exceeds the allocation-free scratch (262080 floats)");
  float* scratch = nullptr;
  T2_TRY(noalloc_scratch_address(&scratch));
  // The kernels' error word: with no index array and one model they record
  // nothing (a model index is the only device-side error of these three
  // kernels), so launch errors in the returned status are the whole story.
  // It is still cleared, since the array keeps the previous call's contents.
  int* err = reinterpret_cast<int*>(scratch);
  float* m = scratch + kNoAllocHeaderFloats;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  T2_TRY(cudaMemsetAsync(err, 0, sizeof(int), s));
  const T2Dev D = ref_layout_dev(L);
  const dim3 g1((L.cells + 255) / 256, static_cast<unsigned>(game_count));
  t2_expand_pre<false><<<g1, 256, 0, s>>>(input_rows, nullptr, weights, 1, D, m, err);
  T2_TRY(cudaGetLastError());
  T2_TRY(launch_t2_attention(nullptr, weights, 1, D, m, err, reinterpret_cast<int*>(m + game_count * L.cells),
                                  static_cast<unsigned>(game_count), s));
  const dim3 g3((L.rows + kRowsPerCta - 1) / kRowsPerCta, static_cast<unsigned>(game_count));
  const int threads3 = static_cast<int>(std::min<size_t>(512, std::max<size_t>(128, kRowsPerCta * L.rows)));
  t2_post_collapse<false><<<g3, threads3, 0, s>>>(nullptr, weights, 1, D, m, output_rows, err);
  return from_cuda(cudaGetLastError());
}

// Measured rate of the special-function pipe (no counterpart in the reference):
// one launch of mufu_rate_kernel per op on the current device, timed with
// CUDA events after a warm-up launch.
OrbitWarsCudaStatus orbit_wars_cuda_mufu_rate(int32_t op, double* ops_per_second, double* ops_per_clock_per_sm,
                                              double* sm_clock_mhz) {
  if ((op != 0 && op != 1) || ops_per_second == nullptr || ops_per_clock_per_sm == nullptr ||
      sm_clock_mhz == nullptr)
    return bad("op must be 0 (ex2) or 1 (rcp); outputs must not be null");
  int dev = 0;
  T2_TRY(cudaGetDevice(&dev));
  int sms = 0;
  T2_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  float* sink = nullptr;
  long long* cyc = nullptr;
  T2_TRY(cudaMalloc(&sink, 1024 * sizeof(float)));
  if (cudaMalloc(&cyc, sms * sizeof(long long)) != cudaSuccess) {
    cudaFree(sink);
    return rt("cudaMalloc failed");
  }
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  const int iters = 4096;
  auto launch = [&]() {
    if (op == 0) mufu_rate_kernel<0><<<sms, 1024>>>(iters, sink, cyc);
    else mufu_rate_kernel<1><<<sms, 1024>>>(iters, sink, cyc);
  };
  launch();  // warm-up
  cudaEventRecord(e0);
  launch();
  cudaEventRecord(e1);
  cudaError_t e = cudaEventSynchronize(e1);
  float ms = 0.0f;
  std::vector<long long> c(sms);
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  if (e == cudaSuccess) e = cudaMemcpy(c.data(), cyc, sms * sizeof(long long), cudaMemcpyDeviceToHost);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(sink);
  cudaFree(cyc);
  if (e != cudaSuccess) return from_cuda(e);
  const double ops_cta = 1024.0 * iters * 8.0;
  double mean_cyc = 0.0;
  for (long long v : c) mean_cyc += static_cast<double>(v);
  mean_cyc /= sms;
  *ops_per_second = ops_cta * sms / (ms * 1e-3);
  *ops_per_clock_per_sm = ops_cta / mean_cyc;
  *sm_clock_mhz = mean_cyc / (ms * 1e-3) / 1e6;  // cycles of the timed span over its event time (upper bound on launch gaps)
  return ok();
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_profile_begin(int32_t max_calls) {
  if (max_calls <= 0 || max_calls > 100000) return bad("max_calls must be in [1, 100000]");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  const size_t need = static_cast<size_t>(max_calls) * 12;  // encode, copies, forward kernels, decode
  while (W.prof_events.size() < need) {
    cudaEvent_t ev;
    T2_TRY(cudaEventCreate(&ev));
    W.prof_events.push_back(ev);
  }
  W.prof_names.assign(W.prof_events.size(), nullptr);
  W.prof_used = 0;
  W.prof_on = true;
  return ok();
}

OrbitWarsCudaStatus orbit_wars_cuda_true2d_profile_end(OrbitWarsCudaKernelTiming* out, int32_t capacity,
                                                       int32_t* count) {
  if (count == nullptr || (out == nullptr && capacity > 0)) return bad("null argument");
  Workspace& W = ws();
  std::lock_guard<std::mutex> lock(W.mu);
  W.prof_on = false;
  if (W.stream != nullptr) T2_TRY(cudaStreamSynchronize(W.stream));
  int32_t n = 0;
  for (size_t i = 0; i + 1 < W.prof_used; ++i) {
    const char* name = W.prof_names[i];
    if (name == nullptr) continue;  // closing event of a call: the next event opens another call
    float ms = 0.0f;
    T2_TRY(cudaEventElapsedTime(&ms, W.prof_events[i], W.prof_events[i + 1]));
    int32_t k = 0;
    while (k < n && std::strcmp(out[k].name, name) != 0) ++k;
    if (k == n) {
      if (n >= capacity) continue;
      out[n].name = name;
      out[n].launches = 0;
      out[n].total_ms = 0.0f;
      ++n;
    }
    out[k].launches += 1;
    out[k].total_ms += ms;
  }
  *count = n;
  W.prof_used = 0;
  return ok();
}

}  // extern "C"

