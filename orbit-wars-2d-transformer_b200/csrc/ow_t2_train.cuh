// True2D training step on the device: orbit_wars_cuda_true2d_train_full_attention
// (native/cuda/orbit_wars_cuda.cu:2823-3330 of the reference ABI).
//
// One call = one full-batch SGD step per model of the population:
//   w[m] -= learning_rate * (sum over m's samples of dLoss/dw) / (m's sample count)
// with the reference's loss (policy-gradient terms on the stored outputs):
//   target choice: softmax over target rows of cell * target_scale + target_bias,
//     weighted by reward + target_action_reward, against the stored choice
//     (orbit_wars_cuda.cu:1426-1525);
//   send choice: sigmoid of the send logit, weighted by the reward, against the
//     stored send fraction >= send_threshold, for sources whose target is
//     another on-map row (:1527-1597).
// The forward is the inference forward (true2d_model.rs:197-283) with every
// matrix state kept: state 0 = expand, states 1..mid = matrix layers before the
// attention layer, mid + 1 = attention + apply, mid + 2..layers + 1 = the rest.
//
// Layout of the work, B200 side:
//   * samples are sorted by model on the host, so one model's samples are a
//     contiguous segment [mstart[m], mstart[m+1]) of every per-sample buffer;
//   * per-cell backward kernels run a thread per (model, cell) over its model's
//     segment: the state gradients are written per sample, the 12 weight
//     gradients of a matrix-layer cell stay in registers and are added once to
//     the model's gradient (no atomics: every sum has a fixed order, so a call
//     is deterministic);
//   * the attention backward is O(cells^2) per (sample, head): a CTA holds the
//     whole mid state and the per-query statistics of its head in shared memory;
//   * reductions over cells or samples go through per-sample partial buffers.
// The arithmetic follows the reference's formulas; sums are taken in a
// different order, and the O(cells^2) attention loops use the fast exponential
// (__expf, a few ulp) and a reciprocal of each denominator, so results agree to
// f32 rounding, not bit for bit.
#pragma once

namespace t2tr {

constexpr float kOwnerEps = 1e-6f;  // TRUE2D_OWNER_CLASS_EPSILON
constexpr int kMaxHeadsTr = 16;

__device__ __forceinline__ bool owner_is(float a, float b) { return fabsf(a - b) <= kOwnerEps; }

// The training step's view of shapes and buffers (kernel parameter).
struct Tr {
  T2Dev L;                 // reference (unpadded) weight layout
  const float* w;          // [models][total]
  float* g;                // [models][total] gradient sums
  const float* x;          // [n][rows][7]      samples sorted by model
  const float* out;        // [n][rows][24]
  const int* rewards;      // [n]
  const float* tar;        // [n][rows][12]
  const int* model;        // [n] model of each sample
  const int* mstart;       // [models + 1] segments of the sorted samples
  int n, models;
  float* hist;             // [n][layers + 2][cells] matrix states
  float* grad;             // [n][layers + 2][cells] their gradients
  float* attv;             // [n][cells] combined attention context
  float* att_grad;         // [n][cells]
  float* stats;            // [n][heads][3][cells] per query: max score, 1 / denominator, weighted average
  float* gpart;            // [n][12][cells] final-state gradient per action
  float* opart;            // [n][2 * rows * 12 + 60] output-weight gradients per sample
  float* hpart;            // [n][heads][8] head-weight gradients per sample (7 used)
  float* igrad;            // [n][heads][cells] attention input gradient per head
  float* cpart;            // [models][cells][16] per-cell partials (shared layer / expand)
  float owner_own, owner_empty, owner_absent;
  float reward_normalizer, send_threshold, learning_rate;
};

__device__ __forceinline__ long long hoff(const Tr& t, int s, int state) {
  return (static_cast<long long>(s) * (t.L.layers + 2) + state) * t.L.cells;
}

__device__ __forceinline__ float sig(float v) { return 1.0f / (1.0f + expf(-v)); }

// reference matrix layer forward (orbit_wars_cuda.cu:123-143), weights w[0..11]
__device__ __forceinline__ float mat_fwd(float v, const float* w) {
  const float ha = tanhf(v * w[2] + w[3]);
  const float hb = tanhf(v * w[4] + ha * w[5] + w[6]);
  const float gt = sig(v * w[7] + w[8]);
  const float u = hb * w[9] + ha * w[10] + w[11];
  const float r = v * (1.0f + w[0]) + w[1];
  return tanhf(r + gt * u);
}

// ---------------------------------------------------------------- forward with history
// expand (state 0) and matrix layers [l0, l1): thread per (sample, cell)
__global__ void __launch_bounds__(256) fwd_matrix(Tr t, int l0, int l1, int with_expand) {
  const int s = blockIdx.y;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= t.L.cells) return;
  const float* w = t.w + static_cast<long long>(t.model[s]) * t.L.total;
  const int rows = t.L.rows, mid = t.L.mid;
  float v;
  if (with_expand) {
    const int src = cell / rows, tgt = cell % rows;
    const float* xs = t.x + (static_cast<long long>(s) * rows + src) * 7;
    const float* xt = t.x + (static_cast<long long>(s) * rows + tgt) * 7;
    const float* pw = w + t.L.pair;
    float a = 0.0f;
    for (int f = 0; f < 7; ++f) a += xs[f] * pw[f];
    for (int f = 0; f < 7; ++f) a += xt[f] * pw[7 + f];
    a += w[t.L.src_emb + src] + w[t.L.tgt_emb + tgt] + w[t.L.pair_emb + cell] + w[t.L.bias];
    v = tanhf(a);
    t.hist[hoff(t, s, 0) + cell] = v;
  } else {
    const int in_state = l0 < mid ? l0 : l0 + 1;
    v = t.hist[hoff(t, s, in_state) + cell];
  }
  for (int l = l0; l < l1; ++l) {
    const int out_state = (l < mid ? l : l + 1) + 1;
    v = mat_fwd(v, w + t.L.matrix + (static_cast<long long>(l) * t.L.cells + cell) * 12);
    t.hist[hoff(t, s, out_state) + cell] = v;
  }
}

// attention layer forward (orbit_wars_cuda.cu:1263-1334) + apply (:1336-1384):
// CTA per (sample, 256 query cells); the mid state of the sample in shared memory.
__global__ void __launch_bounds__(256) fwd_attention(Tr t, int use_smem) {
  extern __shared__ float sm[];  // [cells] when use_smem
  __shared__ float s_red[2][8];
  const int s = blockIdx.y;
  const int cells = t.L.cells, mid = t.L.mid;
  const float* w = t.w + static_cast<long long>(t.model[s]) * t.L.total;
  const float* hw = w + t.L.attn;
  const float* sw = hw + t.L.heads * 7;
  const float* mv = t.hist + hoff(t, s, mid);
  const float* s_v = mv;
  if (use_smem) {
    for (int i = threadIdx.x; i < cells; i += blockDim.x) sm[i] = mv[i];
    s_v = sm;
  }
  __syncthreads();
  // max and min of the mid state: the closed-form max of q * key over keys
  float lo = INFINITY, hi = -INFINITY;
  for (int i = threadIdx.x; i < cells; i += blockDim.x) {
    lo = fminf(lo, s_v[i]);
    hi = fmaxf(hi, s_v[i]);
  }
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if ((threadIdx.x & 31) == 0) {
    s_red[0][threadIdx.x >> 5] = lo;
    s_red[1][threadIdx.x >> 5] = hi;
  }
  __syncthreads();
  lo = s_red[0][0];
  hi = s_red[1][0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) {
    lo = fminf(lo, s_red[0][i]);
    hi = fmaxf(hi, s_red[1][i]);
  }
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= cells) return;
  const float cv = s_v[q];
  float ctx = 0.0f;
  for (int h = 0; h < t.L.heads; ++h) {
    const float qs = hw[h * 7 + 0], qb = hw[h * 7 + 1], ks = hw[h * 7 + 2], kb = hw[h * 7 + 3];
    const float vs = hw[h * 7 + 4], vb = hw[h * 7 + 5], os = hw[h * 7 + 6];
    const float query = cv * qs + qb;
    // keys are affine in the cell value: max_j query * key_j sits at an end of [lo, hi]
    const float k_lo = lo * ks + kb, k_hi = hi * ks + kb;
    const float mx = fmaxf(query * k_lo, query * k_hi);
    float den = 0.0f, wv = 0.0f;
    for (int j = 0; j < cells; ++j) {
      const float kv = s_v[j];
      const float a = __expf(query * (kv * ks + kb) - mx);
      den += a;
      wv += a * (kv * vs + vb);
    }
    const float wavg = wv / den;
    float* st = t.stats + (static_cast<long long>(s) * t.L.heads + h) * 3 * cells;
    st[q] = mx;
    st[cells + q] = 1.0f / den;  // kept as the reciprocal: the backward multiplies
    st[2 * cells + q] = wavg;
    ctx += wavg * os;
  }
  t.attv[static_cast<long long>(s) * cells + q] = ctx;
  const float res = cv * sw[0] + ctx + sw[1];
  const float fh = tanhf(res * sw[2] + sw[3]);
  t.hist[hoff(t, s, mid + 1) + q] = tanhf(res + fh * sw[4] + sw[5]);
}

// ---------------------------------------------------------------- loss
// CTA per (sample, action a), thread per target row t (blockDim = rows rounded
// up to a warp multiple). For every owned source row: the gradient of the
// final state row (per action, summed later in action order) and the
// output-weight gradient terms of this sample.
__global__ void __launch_bounds__(128) loss_backward(Tr t) {
  const int s = blockIdx.y, a = blockIdx.x;
  const int rows = t.L.rows, cells = t.L.cells;
  const int tr = threadIdx.x;
  const bool live = tr < rows;
  __shared__ int s_active[128];   // active rows in order
  __shared__ int s_nactive;
  __shared__ float s_red[4][4];
  const float* x = t.x + static_cast<long long>(s) * rows * 7;
  const float* w = t.w + static_cast<long long>(t.model[s]) * t.L.total;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int r = 0; r < rows; ++r)
      if (!owner_is(x[r * 7], t.owner_empty)) s_active[n++] = r;
    s_nactive = n;
  }
  __syncthreads();
  const int n_active = s_nactive;
  const float* fin = t.hist + hoff(t, s, t.L.layers + 1);
  float* gp = t.gpart + (static_cast<long long>(s) * 12 + a) * cells;
  const float reward_scale = static_cast<float>(t.rewards[s]) / t.reward_normalizer;
  const float* sc = w + t.L.scalars + a * 5;
  const float target_scale = sc[0], send_key_scale = sc[1], send_value_scale = sc[2];
  const float send_output_scale = sc[3], send_output_bias = sc[4];
  const float tb = live ? w[t.L.tbias + a * rows + tr] : 0.0f;
  const float sbv = live ? w[t.L.sbias + a * rows + tr] : 0.0f;
  float g_tb = 0.0f, g_sb = 0.0f;  // this thread's bias gradients (target row tr)
  float g_ts = 0.0f, g_sks = 0.0f, g_svs = 0.0f, g_sos = 0.0f, g_sob = 0.0f;  // scalar terms (thread 0 adds the per-source ones)
  const int nw = (blockDim.x + 31) >> 5;
  auto block_max = [&](float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) s_red[0][threadIdx.x >> 5] = v;
    __syncthreads();
    float r = s_red[0][0];
    for (int i = 1; i < nw; ++i) r = fmaxf(r, s_red[0][i]);
    return r;
  };
  auto block_sum2 = [&](float u, float v, float& su, float& sv) {
    for (int o = 16; o > 0; o >>= 1) {
      u += __shfl_xor_sync(0xffffffffu, u, o);
      v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
      s_red[1][threadIdx.x >> 5] = u;
      s_red[2][threadIdx.x >> 5] = v;
    }
    __syncthreads();
    su = 0.0f;
    sv = 0.0f;
    for (int i = 0; i < nw; ++i) {
      su += s_red[1][i];
      sv += s_red[2][i];
    }
  };
  for (int src = 0; src < rows; ++src) {
    float g_cell = 0.0f;
    const bool owned = owner_is(x[src * 7], t.owner_own) && n_active > 0;
    if (owned) {
      const float* o = t.out + (static_cast<long long>(s) * rows + src) * 24 + a * 2;
      const float trs = reward_scale + t.tar[(static_cast<long long>(s) * rows + src) * 12 + a];
      const float frac = fminf(fmaxf(o[0], 0.0f), 1.0f);
      int sel_i = static_cast<int>(floorf(frac * static_cast<float>(n_active)));
      if (sel_i >= n_active) sel_i = n_active - 1;
      const int sel = s_active[sel_i];
      const float cv = live ? fin[src * rows + tr] : 0.0f;
      const float score = cv * target_scale + tb;
      const float mx = block_max(live ? score : -INFINITY);
      const float e = live ? expf(score - mx) : 0.0f;
      float den, unused;
      block_sum2(e, 0.0f, den, unused);
      if (trs != 0.0f && live) {
        const float p = e / den;
        const float d_score = trs * (p - (tr == sel ? 1.0f : 0.0f));
        g_cell += d_score * target_scale;
        g_tb += d_score;
        g_ts += d_score * cv;
      }
      const bool send = !(reward_scale == 0.0f || sel == src || owner_is(x[sel * 7], t.owner_absent));
      if (send) {
        const float ss = cv * send_key_scale + sbv;
        const float smx = block_max(live ? ss : -INFINITY);
        const float att = live ? expf(ss - smx) : 0.0f;
        float sden, swv;
        block_sum2(att, att * cv, sden, swv);
        const float avg = swv / sden;
        const float logit = send_output_bias + avg * send_value_scale;
        const float sp = sig(logit * send_output_scale);
        const float sfrac = fminf(fmaxf(o[1], 0.0f), 1.0f);
        const float send_action = sfrac >= t.send_threshold ? 1.0f : 0.0f;
        const float d_ssl = reward_scale * (sp - send_action);
        const float d_sl = d_ssl * send_output_scale;
        const float d_avg = d_sl * send_value_scale;
        if (threadIdx.x == 0) {
          g_sos += d_ssl * logit;
          g_sob += d_sl;
          g_svs += d_sl * avg;
        }
        if (live) {
          const float pr = att / sden;
          const float d_ss = d_avg * pr * (cv - avg);
          g_cell += d_avg * pr + d_ss * send_key_scale;
          g_sb += d_ss;
          g_sks += d_ss * cv;
        }
      }
    }
    if (live) gp[src * rows + tr] = g_cell;
  }
  // per-sample output-weight gradients: biases by thread, scalars block-reduced
  float* op = t.opart + static_cast<long long>(s) * (2 * rows * 12 + 60);
  if (live) {
    op[a * rows + tr] = g_tb;
    op[rows * 12 + a * rows + tr] = g_sb;
  }
  float r_ts, r_sks;
  block_sum2(g_ts, g_sks, r_ts, r_sks);
  if (threadIdx.x == 0) {
    float* ps = op + 2 * rows * 12 + a * 5;
    ps[0] = r_ts;
    ps[1] = r_sks;
    ps[2] = g_svs;
    ps[3] = g_sos;
    ps[4] = g_sob;
  }
}

// final-state gradient: sum of the 12 actions' terms, in action order
__global__ void __launch_bounds__(256) sum_actions(Tr t) {
  const int s = blockIdx.y;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= t.L.cells) return;
  const float* gp = t.gpart + static_cast<long long>(s) * 12 * t.L.cells + cell;
  float g = 0.0f;
  for (int a = 0; a < 12; ++a) g += gp[static_cast<long long>(a) * t.L.cells];
  t.grad[hoff(t, s, t.L.layers + 1) + cell] = g;
}

// ---------------------------------------------------------------- backward
// matrix layer l (orbit_wars_cuda.cu:1961-2029 and :2031-2132): thread per
// (model, cell) over the model's samples; the input state's gradient is added,
// the 12 weight gradients summed in registers.
__global__ void __launch_bounds__(256) bwd_matrix(Tr t, int l) {
  const int m = blockIdx.y;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= t.L.cells) return;
  const int s0 = t.mstart[m], s1 = t.mstart[m + 1];
  if (s0 == s1) return;
  const float* w = t.w + static_cast<long long>(m) * t.L.total + t.L.matrix +
                   (static_cast<long long>(l) * t.L.cells + cell) * 12;
  float cw[12];
#pragma unroll
  for (int i = 0; i < 12; ++i) cw[i] = w[i];
  const int in_state = l < t.L.mid ? l : l + 1;
  float acc[12];
#pragma unroll
  for (int i = 0; i < 12; ++i) acc[i] = 0.0f;
  for (int s = s0; s < s1; ++s) {
    const float v = t.hist[hoff(t, s, in_state) + cell];
    const float next = t.hist[hoff(t, s, in_state + 1) + cell];
    const float d_next = t.grad[hoff(t, s, in_state + 1) + cell];
    const float ha = tanhf(v * cw[2] + cw[3]);
    const float hb = tanhf(v * cw[4] + ha * cw[5] + cw[6]);
    const float gt = sig(v * cw[7] + cw[8]);
    const float u = hb * cw[9] + ha * cw[10] + cw[11];
    const float d_pre = d_next * (1.0f - next * next);
    float d_cell = d_pre * (1.0f + cw[0]);
    const float d_gate_in = d_pre * u * gt * (1.0f - gt);
    d_cell += d_gate_in * cw[7];
    const float d_update = d_pre * gt;
    const float d_hb = d_update * cw[9];
    float d_ha = d_update * cw[10];
    const float d_hb_in = d_hb * (1.0f - hb * hb);
    d_cell += d_hb_in * cw[4];
    d_ha += d_hb_in * cw[5];
    const float d_ha_in = d_ha * (1.0f - ha * ha);
    d_cell += d_ha_in * cw[2];
    t.grad[hoff(t, s, in_state) + cell] += d_cell;
    acc[0] += d_pre * v;
    acc[1] += d_pre;
    acc[2] += d_ha_in * v;
    acc[3] += d_ha_in;
    acc[4] += d_hb_in * v;
    acc[5] += d_hb_in * ha;
    acc[6] += d_hb_in;
    acc[7] += d_gate_in * v;
    acc[8] += d_gate_in;
    acc[9] += d_update * hb;
    acc[10] += d_update * ha;
    acc[11] += d_update;
  }
  float* g = t.g + static_cast<long long>(m) * t.L.total + t.L.matrix + (static_cast<long long>(l) * t.L.cells + cell) * 12;
#pragma unroll
  for (int i = 0; i < 12; ++i) g[i] += acc[i];
}

// apply step of the attention layer (orbit_wars_cuda.cu:1829-1884, shared
// weights :1886-1959): thread per (model, cell); the six shared-weight terms
// go to cpart[m][cell][0..5] and are summed over cells by reduce_cells.
__global__ void __launch_bounds__(256) bwd_apply(Tr t) {
  const int m = blockIdx.y;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= t.L.cells) return;
  const int s0 = t.mstart[m], s1 = t.mstart[m + 1];
  float* cp = t.cpart + (static_cast<long long>(m) * t.L.cells + cell) * 16;
  float acc[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (s0 < s1) {
    const float* sw = t.w + static_cast<long long>(m) * t.L.total + t.L.attn + t.L.heads * 7;
    const int mid = t.L.mid;
    for (int s = s0; s < s1; ++s) {
      const float v = t.hist[hoff(t, s, mid) + cell];
      const float res = v * sw[0] + t.attv[static_cast<long long>(s) * t.L.cells + cell] + sw[1];
      const float fh = tanhf(res * sw[2] + sw[3]);
      const float next = t.hist[hoff(t, s, mid + 1) + cell];
      const float d_value = t.grad[hoff(t, s, mid + 1) + cell] * (1.0f - next * next);
      const float d_fin = d_value * sw[4] * (1.0f - fh * fh);
      const float d_res = d_value + d_fin * sw[2];
      t.grad[hoff(t, s, mid) + cell] += d_res * sw[0];
      t.att_grad[static_cast<long long>(s) * t.L.cells + cell] = d_res;
      acc[0] += d_res * v;
      acc[1] += d_res;
      acc[2] += d_fin * res;
      acc[3] += d_fin;
      acc[4] += d_value * fh;
      acc[5] += d_value;
    }
  }
#pragma unroll
  for (int i = 0; i < 6; ++i) cp[i] = acc[i];
}

// attention backward (orbit_wars_cuda.cu:2134-2263) for one head: CTA per
// (sample, 256 cells); the mid state, the attention gradient and the head's
// per-query statistics of the sample in shared memory (5 x cells floats).
// Writes the input gradient of this head to igrad and the head-weight terms
// summed over the CTA's cells to hpart (block-reduced here, summed over the
// CTAs of the sample by sum_heads).
__global__ void __launch_bounds__(256) bwd_attention(Tr t, int h, float* hcta, int use_smem) {
  extern __shared__ float sm[];
  const int cells = t.L.cells;
  __shared__ float s_red[8][8];
  const int s = blockIdx.y;
  const int m = t.model[s];
  const float* hw = t.w + static_cast<long long>(m) * t.L.total + t.L.attn + h * 7;
  const float qs = hw[0], qb = hw[1], ks = hw[2], kb = hw[3], vs = hw[4], vb = hw[5], os = hw[6];
  const float* mv = t.hist + hoff(t, s, t.L.mid);
  const float* st = t.stats + (static_cast<long long>(s) * t.L.heads + h) * 3 * cells;
  const float* ag = t.att_grad + static_cast<long long>(s) * cells;
  // the five per-cell vectors: staged in shared memory when they fit (5 x cells floats),
  // else read from global memory (L1 / L2)
  const float* s_v = mv;
  const float* s_dg = ag;
  const float* s_mx = st;
  const float* s_den = st + cells;
  const float* s_wa = st + 2 * cells;
  if (use_smem) {
    for (int i = threadIdx.x; i < cells; i += blockDim.x) {
      sm[i] = mv[i];
      sm[cells + i] = ag[i];
      sm[2 * cells + i] = st[i];
      sm[3 * cells + i] = st[cells + i];
      sm[4 * cells + i] = st[2 * cells + i];
    }
    s_v = sm;
    s_dg = sm + cells;
    s_mx = sm + 2 * cells;
    s_den = sm + 3 * cells;
    s_wa = sm + 4 * cells;
  }
  __syncthreads();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  float gq_s = 0.f, gq_b = 0.f, gk_s = 0.f, gk_b = 0.f, gv_s = 0.f, gv_b = 0.f, go = 0.f;
  if (c < cells) {
    const float cv = s_v[c];
    float input_g = 0.0f;
    const float d_att_c = s_dg[c];
    if (d_att_c != 0.0f) {
      const float qc = cv * qs + qb;
      const float mx = s_mx[c], den = s_den[c], wa = s_wa[c];
      const float d_wavg = d_att_c * os;
      float d_query = 0.0f;
      for (int j = 0; j < cells; ++j) {
        const float kv = s_v[j];
        const float key = kv * ks + kb;
        const float val = kv * vs + vb;
        const float p = __expf(qc * key - mx) * den;  // den holds 1 / denominator
        d_query += d_wavg * p * (val - wa) * key;
      }
      go = d_att_c * wa;
      gq_s = d_query * cv;
      gq_b = d_query;
      input_g += d_query * qs;
    }
    const float key_c = cv * ks + kb, val_c = cv * vs + vb;
    for (int i = 0; i < cells; ++i) {
      const float d_att = s_dg[i];
      if (d_att == 0.0f) continue;
      const float qv = s_v[i] * qs + qb;
      const float p = __expf(qv * key_c - s_mx[i]) * s_den[i];  // s_den holds 1 / denominator
      const float d_wavg = d_att * os;
      const float d_val = d_wavg * p;
      const float d_key = d_wavg * p * (val_c - s_wa[i]) * qv;
      gv_s += d_val * cv;
      gv_b += d_val;
      gk_s += d_key * cv;
      gk_b += d_key;
      input_g += d_val * vs + d_key * ks;
    }
    t.igrad[(static_cast<long long>(s) * t.L.heads + h) * cells + c] = input_g;
  }
  // block sums of the seven head-weight terms
  float v7[7] = {gq_s, gq_b, gk_s, gk_b, gv_s, gv_b, go};
#pragma unroll
  for (int k = 0; k < 7; ++k)
    for (int o = 16; o > 0; o >>= 1) v7[k] += __shfl_xor_sync(0xffffffffu, v7[k], o);
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int k = 0; k < 7; ++k) s_red[threadIdx.x >> 5][k] = v7[k];
  __syncthreads();
  if (threadIdx.x < 7) {
    float r = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) r += s_red[i][threadIdx.x];
    hcta[(static_cast<long long>(s) * gridDim.x + blockIdx.x) * 8 + threadIdx.x] = r;
  }
}

// The same attention backward with the per-cell terms prepared once per CTA in
// shared memory (6 x cells floats), 512 threads per CTA:
//   s_kv[j] = (key_j, value_j)
//   s_q[i]  = (query_i, max_i, d_att_i * out_scale / denominator_i, wavg_i)
// so that both O(cells^2) loops read one broadcast vector per step and spend
// one exponential, three multiply-adds and a subtraction on it:
//   d_query_c = s_q[c].z * sum_j e^(q_c k_j - max_c) (v_j - wavg_c) k_j
//   for key c: sum_v = sum_i s_q[i].z e^(q_i k_c - max_i)
//              sum_k = sum_i s_q[i].z e^(q_i k_c - max_i) (v_c - wavg_i) q_i
// and the value / key weight terms are sum_v, sum_k times (cell value, 1).
__global__ void __launch_bounds__(512) bwd_attention_smem(Tr t, int h, float* hcta) {
  extern __shared__ float4 smq[];
  const int cells = t.L.cells;
  __shared__ float s_red[16][8];
  const int s = blockIdx.y;
  const int m = t.model[s];
  const float* hw = t.w + static_cast<long long>(m) * t.L.total + t.L.attn + h * 7;
  const float qs = hw[0], qb = hw[1], ks = hw[2], kb = hw[3], vs = hw[4], vb = hw[5], os = hw[6];
  const float* mv = t.hist + hoff(t, s, t.L.mid);
  const float* st = t.stats + (static_cast<long long>(s) * t.L.heads + h) * 3 * cells;
  const float* ag = t.att_grad + static_cast<long long>(s) * cells;
  float4* s_q = smq;
  float2* s_kv = reinterpret_cast<float2*>(smq + cells);
  for (int i = threadIdx.x; i < cells; i += blockDim.x) {
    const float v = mv[i];
    s_kv[i] = make_float2(v * ks + kb, v * vs + vb);
    s_q[i] = make_float4(v * qs + qb, st[i], ag[i] * os * st[cells + i], st[2 * cells + i]);
  }
  __syncthreads();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  float gq_s = 0.f, gq_b = 0.f, gk_s = 0.f, gk_b = 0.f, gv_s = 0.f, gv_b = 0.f, go = 0.f;
  if (c < cells) {
    const float cv = mv[c];
    const float4 qc = s_q[c];
    const float2 kvc = s_kv[c];
    const float d_att_c = ag[c];
    float input_g = 0.0f;
    if (d_att_c != 0.0f) {
      float a0 = 0.0f, a1 = 0.0f;
      int j = 0;
      for (; j + 1 < cells; j += 2) {
        const float2 p0 = s_kv[j], p1 = s_kv[j + 1];
        a0 += __expf(qc.x * p0.x - qc.y) * (p0.y - qc.w) * p0.x;
        a1 += __expf(qc.x * p1.x - qc.y) * (p1.y - qc.w) * p1.x;
      }
      if (j < cells) {
        const float2 p0 = s_kv[j];
        a0 += __expf(qc.x * p0.x - qc.y) * (p0.y - qc.w) * p0.x;
      }
      const float d_query = qc.z * (a0 + a1);
      go = d_att_c * qc.w;
      gq_s = d_query * cv;
      gq_b = d_query;
      input_g += d_query * qs;
    }
    float sum_v = 0.0f, sum_k = 0.0f;
    for (int i = 0; i < cells; ++i) {
      const float4 y = s_q[i];
      if (y.z == 0.0f) continue;  // the same i in every lane: a uniform branch
      const float d = y.z * __expf(y.x * kvc.x - y.y);
      sum_v += d;
      sum_k += d * (kvc.y - y.w) * y.x;
    }
    gv_s = sum_v * cv;
    gv_b = sum_v;
    gk_s = sum_k * cv;
    gk_b = sum_k;
    input_g += sum_v * vs + sum_k * ks;
    t.igrad[(static_cast<long long>(s) * t.L.heads + h) * cells + c] = input_g;
  }
  float v7[7] = {gq_s, gq_b, gk_s, gk_b, gv_s, gv_b, go};
#pragma unroll
  for (int k = 0; k < 7; ++k)
    for (int o = 16; o > 0; o >>= 1) v7[k] += __shfl_xor_sync(0xffffffffu, v7[k], o);
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int k = 0; k < 7; ++k) s_red[threadIdx.x >> 5][k] = v7[k];
  __syncthreads();
  if (threadIdx.x < 7) {
    float r = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) r += s_red[i][threadIdx.x];
    hcta[(static_cast<long long>(s) * gridDim.x + blockIdx.x) * 8 + threadIdx.x] = r;
  }
}

// head-weight terms per sample (sum over the sample's CTAs in order) and the
// mid-state gradient (sum over heads in order)
__global__ void __launch_bounds__(256) sum_heads(Tr t, int h, const float* hcta, int ctas) {
  const int s = blockIdx.y;
  if (blockIdx.x == 0 && threadIdx.x < 7) {
    float r = 0.0f;
    for (int b = 0; b < ctas; ++b) r += hcta[(static_cast<long long>(s) * ctas + b) * 8 + threadIdx.x];
    t.hpart[(static_cast<long long>(s) * t.L.heads + h) * 8 + threadIdx.x] = r;
  }
  if (h != t.L.heads - 1) return;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= t.L.cells) return;
  float g = 0.0f;
  for (int k = 0; k < t.L.heads; ++k) g += t.igrad[(static_cast<long long>(s) * t.L.heads + k) * t.L.cells + cell];
  t.grad[hoff(t, s, t.L.mid) + cell] += g;
}

// expand backward (orbit_wars_cuda.cu:2307-2412): thread per (model, cell).
// The pair embedding of the cell is its own; the rest goes to cpart[m][cell]:
// [0] d_pre sum, [1..14] pair-feature terms.
__global__ void __launch_bounds__(256) bwd_expand(Tr t) {
  const int m = blockIdx.y;
  const int cell = blockIdx.x * blockDim.x + threadIdx.x;
  if (cell >= t.L.cells) return;
  const int s0 = t.mstart[m], s1 = t.mstart[m + 1];
  const int rows = t.L.rows;
  const int src = cell / rows, tgt = cell % rows;
  float acc[15];
#pragma unroll
  for (int i = 0; i < 15; ++i) acc[i] = 0.0f;
  for (int s = s0; s < s1; ++s) {
    const float mv = t.hist[hoff(t, s, 0) + cell];
    const float d_pre = t.grad[hoff(t, s, 0) + cell] * (1.0f - mv * mv);
    const float* xs = t.x + (static_cast<long long>(s) * rows + src) * 7;
    const float* xt = t.x + (static_cast<long long>(s) * rows + tgt) * 7;
    acc[0] += d_pre;
#pragma unroll
    for (int f = 0; f < 7; ++f) {
      acc[1 + f] += d_pre * xs[f];
      acc[8 + f] += d_pre * xt[f];
    }
  }
  float* cp = t.cpart + (static_cast<long long>(m) * t.L.cells + cell) * 16;
#pragma unroll
  for (int i = 0; i < 15; ++i) cp[i] = acc[i];
  if (s0 < s1) t.g[static_cast<long long>(m) * t.L.total + t.L.pair_emb + cell] += acc[0];
}

// ---------------------------------------------------------------- per-model reductions
// shared apply weights: g[attn + heads*7 + k] += sum over cells of cpart[m][cell][k]
__global__ void reduce_shared(Tr t) {
  const int m = blockIdx.x, k = threadIdx.x;
  if (k >= 6 || t.mstart[m] == t.mstart[m + 1]) return;
  float r = 0.0f;
  for (int c = 0; c < t.L.cells; ++c) r += t.cpart[(static_cast<long long>(m) * t.L.cells + c) * 16 + k];
  t.g[static_cast<long long>(m) * t.L.total + t.L.attn + t.L.heads * 7 + k] += r;
}

// head weights: g[attn + h*7 + k] += sum over the model's samples of hpart
__global__ void reduce_heads(Tr t) {
  const int m = blockIdx.x;
  const int h = threadIdx.x / 8, k = threadIdx.x % 8;
  if (h >= t.L.heads || k >= 7) return;
  float r = 0.0f;
  for (int s = t.mstart[m]; s < t.mstart[m + 1]; ++s) r += t.hpart[(static_cast<long long>(s) * t.L.heads + h) * 8 + k];
  t.g[static_cast<long long>(m) * t.L.total + t.L.attn + h * 7 + k] += r;
}

// expand weights from cpart: source/target row embeddings, bias, pair features.
// CTA per model, thread per entry.
__global__ void reduce_expand(Tr t) {
  const int m = blockIdx.x;
  if (t.mstart[m] == t.mstart[m + 1]) return;
  const int rows = t.L.rows;
  const float* cp = t.cpart + static_cast<long long>(m) * t.L.cells * 16;
  float* g = t.g + static_cast<long long>(m) * t.L.total;
  for (int e = threadIdx.x; e < 2 * rows + 1 + 14; e += blockDim.x) {
    float r = 0.0f;
    if (e < rows) {  // source row embedding: sum over target rows
      for (int tt = 0; tt < rows; ++tt) r += cp[(e * rows + tt) * 16];
      g[t.L.src_emb + e] += r;
    } else if (e < 2 * rows) {  // target row embedding: sum over source rows
      const int tt = e - rows;
      for (int ss = 0; ss < rows; ++ss) r += cp[(ss * rows + tt) * 16];
      g[t.L.tgt_emb + tt] += r;
    } else if (e == 2 * rows) {
      for (int c = 0; c < t.L.cells; ++c) r += cp[c * 16];
      g[t.L.bias] += r;
    } else {
      const int f = e - 2 * rows - 1;
      for (int c = 0; c < t.L.cells; ++c) r += cp[c * 16 + 1 + f];
      g[t.L.pair + f] += r;
    }
  }
}

// output weights (target biases, send biases, scalars): sum of the model's samples
__global__ void reduce_output(Tr t) {
  const int m = blockIdx.y;
  const int n_out = 2 * t.L.rows * 12 + 60;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_out) return;
  float r = 0.0f;
  for (int s = t.mstart[m]; s < t.mstart[m + 1]; ++s) r += t.opart[static_cast<long long>(s) * n_out + e];
  t.g[static_cast<long long>(m) * t.L.total + t.L.tbias + e] += r;
}

// w -= lr * g / count (orbit_wars_cuda.cu:2414-2433)
__global__ void apply_sgd(float* w, const float* g, const int* count, int models, long long total, float lr) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(models) * total) return;
  const int m = static_cast<int>(i / total);
  const int c = count[m];
  if (c == 0) return;
  w[i] -= lr * g[i] / static_cast<float>(c);
}

}  // namespace t2tr
