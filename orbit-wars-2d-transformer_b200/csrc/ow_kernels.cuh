// Non-GEMM kernels of the encoder-policy forward.
//
// Token layout in HBM: valid entities only, packed state after state
// ("varlen"): state b owns rows offsets[b] .. offsets[b+1]-1. Padded entity
// slots never enter the blocks; the head kernel writes their logits (0) and
// actions (-1) directly into the padded [B, N, ...] outputs.
#pragma once

#include "ow_common.cuh"

namespace ow {

// ------------------------------------------------------------------ offsets
// counts[B] -> offsets[B+1] (exclusive scan), one CTA of 1024 threads.
// A count outside [0, n_entities] records kErrBadCount and counts as 0.
__global__ void __launch_bounds__(1024) scan_counts_kernel(const int* counts, int batch, int n_entities,
                                                           int* offsets, int* err) {
  __shared__ int warp_tot[32];
  const int t = threadIdx.x;
  const int per = (batch + 1023) / 1024;
  const int b0 = t * per;
  int local = 0;
  for (int i = 0; i < per; ++i) {
    const int b = b0 + i;
    if (b < batch) {
      int c = counts[b];
      if (c < 0 || c > n_entities) {
        record_error(err, kErrBadCount);
        c = 0;
      }
      local += c;
    }
  }
  // inclusive scan of `local` over the block
  const int lane = t & 31, w = t >> 5;
  int v = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) warp_tot[w] = v;
  __syncthreads();
  if (w == 0) {
    int s = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += u;
    }
    warp_tot[lane] = s;
  }
  __syncthreads();
  int run = v - local + (w > 0 ? warp_tot[w - 1] : 0);  // exclusive prefix of this thread
  if (t == 0) offsets[0] = 0;
  for (int i = 0; i < per; ++i) {
    const int b = b0 + i;
    if (b < batch) {
      int c = counts[b];
      if (c < 0 || c > n_entities) c = 0;
      run += c;
      offsets[b + 1] = run;
    }
  }
}

// ------------------------------------------------------------------ embedding (+ first LayerNorm)
// One warp per entity slot (b, j); valid slots write packed row offsets[b]+j.
// Lane l owns columns l, l+32, ..., so weight reads are conflict-free.
// x = W_e.feat + b_e;  ln = LN(x; g, beta) -- the first block's pre-LN.
template <int DPL, int LN_MODE>  // x is f32; LN_MODE: 0 f32, 1 bf16, 2 e4m3+scale
__global__ void __launch_bounds__(256) embed_ln_kernel(const float* __restrict__ feats, const int* __restrict__ offsets,
                                                       int batch, int n_entities, int n_feat,
                                                       const float* __restrict__ w_e, const float* __restrict__ b_e,
                                                       const float* __restrict__ g, const float* __restrict__ beta,
                                                       float* __restrict__ x, void* __restrict__ ln_out,
                                                       float* __restrict__ ln_scale) {
  constexpr int D = DPL * 32;
  constexpr int PITCH = D + 1;    // odd pitch: the transposing fill is bank-conflict free
  extern __shared__ float s_w[];  // [F][PITCH] transposed embedding weights
  for (int i = threadIdx.x; i < n_feat * D; i += blockDim.x) {
    const int c = i / n_feat, f = i % n_feat;  // coalesced read of W_e[c, f]
    s_w[f * PITCH + c] = w_e[i];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const long long slots = static_cast<long long>(batch) * n_entities;
  float bias[DPL], gg[DPL], bb[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    bias[i] = b_e[i * 32 + lane];
    gg[i] = g[i * 32 + lane];
    bb[i] = beta[i * 32 + lane];
  }
  for (long long slot = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5); slot < slots;
       slot += static_cast<long long>(gridDim.x) * warps) {
    const int b = static_cast<int>(slot / n_entities);
    const int j = static_cast<int>(slot % n_entities);
    const int row0 = offsets[b];
    if (j >= offsets[b + 1] - row0) continue;
    const long long row = row0 + j;
    const float fv = lane < n_feat ? feats[slot * n_feat + lane] : 0.0f;
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = bias[i];
    for (int f = 0; f < n_feat; ++f) {
      const float xf = __shfl_sync(0xffffffffu, fv, f);
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = fmaf(xf, s_w[f * PITCH + i * 32 + lane], acc[i]);
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) s += acc[i];
    const float mean = warp_sum(s) * (1.0f / D);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const float dv = acc[i] - mean;
      q += dv * dv;
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + 1e-5f);
    float y[DPL];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      x[row * D + i * 32 + lane] = acc[i];
      y[i] = (acc[i] - mean) * rstd * gg[i] + bb[i];
      amax = fmaxf(amax, fabsf(y[i]));
    }
    if (LN_MODE == 0) {
#pragma unroll
      for (int i = 0; i < DPL; ++i) reinterpret_cast<float*>(ln_out)[row * D + i * 32 + lane] = y[i];
    } else if (LN_MODE == 1) {
#pragma unroll
      for (int i = 0; i < DPL; ++i)
        reinterpret_cast<__nv_bfloat16*>(ln_out)[row * D + i * 32 + lane] = __float2bfloat16_rn(y[i]);
    } else {
      amax = warp_max(amax);
      const float scale = amax > 0.0f ? amax * (1.0f / 448.0f) : 1.0f;
      const float inv = 1.0f / scale;
      if (lane == 0) ln_scale[row] = scale;
#pragma unroll
      for (int i = 0; i < DPL; ++i)
        reinterpret_cast<__nv_fp8_e4m3*>(ln_out)[row * D + i * 32 + lane] = __nv_fp8_e4m3(y[i] * inv);
    }
  }
}

// ------------------------------------------------------------------ fp32 path
// Row LayerNorm, fp32, warp per row (rows = packed valid tokens).
template <int DPL>
__global__ void __launch_bounds__(256) layernorm_f32_kernel(const float* __restrict__ x, const int* __restrict__ m_valid,
                                                            const float* __restrict__ g, const float* __restrict__ beta,
                                                            float* __restrict__ y) {
  constexpr int D = DPL * 32;
  const int lane = threadIdx.x & 31;
  const int rows = *m_valid;
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += gridDim.x * (blockDim.x >> 5)) {
    float v[DPL];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      v[i] = x[static_cast<size_t>(row) * D + i * 32 + lane];
      s += v[i];
    }
    const float mean = warp_sum(s) * (1.0f / D);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) q += (v[i] - mean) * (v[i] - mean);
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + 1e-5f);
#pragma unroll
    for (int i = 0; i < DPL; ++i)
      y[static_cast<size_t>(row) * D + i * 32 + lane] = (v[i] - mean) * rstd * g[i * 32 + lane] + beta[i * 32 + lane];
  }
}

enum F32Epi : int { kF32Bias = 0, kF32BiasGelu = 1, kF32BiasResid = 2 };

// C[m, n] = A[m, :] . W[n, :] + bias[n]  (+GELU | += into C), fp32 SIMT.
// 64x64 tile, 256 threads x (4x4), K step 16. Rows >= *m_valid are skipped.
template <int EPI>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, const float* __restrict__ W,
                                                       const float* __restrict__ bias, float* __restrict__ C,
                                                       const int* __restrict__ m_valid, int n, int k) {
  __shared__ float As[16][64 + 4];
  __shared__ float Ws[16][64 + 4];
  const int rows = *m_valid;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  if (m0 >= rows) return;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i / 16, kk = i % 16;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      As[kk][r] = (gm < rows && gk < k) ? A[static_cast<size_t>(gm) * k + gk] : 0.0f;
      Ws[kk][r] = (gn < n && gk < k) ? W[static_cast<size_t>(gn) * k + gk] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        w[i] = Ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= n) continue;
      float v = acc[i][j] + bias[gn];
      float* c = C + static_cast<size_t>(gm) * n + gn;
      if (EPI == kF32BiasGelu) v = gelu_erf(v);
      if (EPI == kF32BiasResid) v += *c;
      *c = v;
    }
  }
}

// Masked attention, fp32, one CTA per (state, head), head_dim 32.
// qkv: [rows, 3d]; out: [rows, d]. Scores of one state live in shared memory.
template <int NMAX>
__global__ void __launch_bounds__(128) attention_f32_kernel(const float* __restrict__ qkv, float* __restrict__ out,
                                                            const int* __restrict__ offsets, int d, float scale) {
  __shared__ float sk[NMAX][33];
  __shared__ float sv[NMAX][33];
  __shared__ float sp[4][NMAX];
  const int b = blockIdx.x, h = blockIdx.y;
  const int row0 = offsets[b];
  const int cnt = offsets[b + 1] - row0;
  if (cnt <= 0) return;
  const int ld = 3 * d;
  for (int i = threadIdx.x; i < cnt * 32; i += blockDim.x) {
    const int r = i / 32, c = i % 32;
    sk[r][c] = qkv[static_cast<size_t>(row0 + r) * ld + d + h * 32 + c];
    sv[r][c] = qkv[static_cast<size_t>(row0 + r) * ld + 2 * d + h * 32 + c];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int i = w; i < cnt; i += 4) {
    const float q = qkv[static_cast<size_t>(row0 + i) * ld + h * 32 + lane];
    float mx = -INFINITY;
    for (int j = 0; j < cnt; ++j) {
      const float s = warp_sum(q * sk[j][lane]) * scale;
      if (lane == 0) sp[w][j] = s;
      mx = fmaxf(mx, s);
    }
    __syncwarp();
    float den = 0.0f;
    for (int j = lane; j < cnt; j += 32) {
      const float e = expf(sp[w][j] - mx);
      sp[w][j] = e;
      den += e;
    }
    den = warp_sum(den);
    __syncwarp();
    float o = 0.0f;
    for (int j = 0; j < cnt; ++j) o = fmaf(sp[w][j], sv[j][lane], o);
    out[static_cast<size_t>(row0 + i) * d + h * 32 + lane] = o / den;
    __syncwarp();
  }
}

// ------------------------------------------------------------------ bf16 attention (mma.sync)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One CTA per (state, head); warp w owns query rows 16w..16w+15.
// S = Q K^T and P V on tensor cores, softmax in registers (fp32),
// keys j >= count masked. Q/K/V of the (state, head) staged in shared
// memory with an 80-byte row pitch (conflict-free ldmatrix).
template <int NMAX>
__global__ void __launch_bounds__(NMAX * 2) attention_bf16_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                   __nv_bfloat16* __restrict__ out,
                                                                   const int* __restrict__ offsets, int d,
                                                                   float scale_log2) {
  constexpr int PITCH = 40;  // bf16 elements per staged row
  constexpr int NT = NMAX / 8;
  __shared__ __align__(16) __nv_bfloat16 sq[NMAX * PITCH];
  __shared__ __align__(16) __nv_bfloat16 sk[NMAX * PITCH];
  __shared__ __align__(16) __nv_bfloat16 sv[NMAX * PITCH];
  const int b = blockIdx.x, h = blockIdx.y;
  const int row0 = offsets[b];
  const int cnt = offsets[b + 1] - row0;
  if (cnt <= 0) return;
  const int cnt16 = (cnt + 15) & ~15;
  const size_t ld = static_cast<size_t>(3) * d;
  for (int i = threadIdx.x; i < cnt16 * 12; i += blockDim.x) {
    const int r = i / 12, part = i % 12, mat = part >> 2, ch = part & 3;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < cnt)
      v = *reinterpret_cast<const uint4*>(qkv + static_cast<size_t>(row0 + r) * ld + mat * d + h * 32 + ch * 8);
    __nv_bfloat16* dst = (mat == 0 ? sq : (mat == 1 ? sk : sv)) + r * PITCH + ch * 8;
    *reinterpret_cast<uint4*>(dst) = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = warp * 16;
  if (q0 >= cnt) return;
  const int g = lane >> 2, t = lane & 3;

  // Q fragments for head-dim k-steps 0..15 and 16..31.
  uint32_t qa[2][4];
  {
    const int r = q0 + (lane & 15);
    const int c = (lane >> 4) * 8;
    ldsm_x4(smem_u32(sq + r * PITCH + c), qa[0][0], qa[0][1], qa[0][2], qa[0][3]);
    ldsm_x4(smem_u32(sq + r * PITCH + 16 + c), qa[1][0], qa[1][1], qa[1][2], qa[1][3]);
  }
  float s[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
    if (j * 8 < cnt16) {
      uint32_t k0, k1, k2, k3;
      ldsm_x4(smem_u32(sk + (j * 8 + (lane & 7)) * PITCH + (lane >> 3) * 8), k0, k1, k2, k3);
      mma_bf16_16816(s[j], qa[0][0], qa[0][1], qa[0][2], qa[0][3], k0, k1);
      mma_bf16_16816(s[j], qa[1][0], qa[1][1], qa[1][2], qa[1][3], k2, k3);
    }
  }
  // masked softmax over keys, rows g and g+8 of this warp's block
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int c0 = j * 8 + 2 * t;
    if (c0 >= cnt) s[j][0] = s[j][2] = -INFINITY;
    if (c0 + 1 >= cnt) s[j][1] = s[j][3] = -INFINITY;
    mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
    mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float off0 = mx0 * scale_log2, off1 = mx1 * scale_log2;
  float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    s[j][0] = exp2f(s[j][0] * scale_log2 - off0);
    s[j][1] = exp2f(s[j][1] * scale_log2 - off0);
    s[j][2] = exp2f(s[j][2] * scale_log2 - off1);
    s[j][3] = exp2f(s[j][3] * scale_log2 - off1);
    sum0 += s[j][0] + s[j][1];
    sum1 += s[j][2] + s[j][3];
  }
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
  sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
  sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);

  float o[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < NT / 2; ++kk) {
    if (kk * 16 < cnt16) {
      const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < 2; ++np) {  // pairs of 8-wide head-dim tiles
        uint32_t v0, v1, v2, v3;
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(smem_u32(sv + key * PITCH + col), v0, v1, v2, v3);
        mma_bf16_16816(o[2 * np], a0, a1, a2, a3, v0, v1);
        mma_bf16_16816(o[2 * np + 1], a0, a1, a2, a3, v2, v3);
      }
    }
  }
  const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
  const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int col = h * 32 + n * 8 + 2 * t;
    if (r0 < cnt)
      *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(row0 + r0) * d + col) =
          pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
    if (r1 < cnt)
      *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(row0 + r1) * d + col) =
          pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
  }
}

// ------------------------------------------------------------------ e4m3 quantiser (fp8 path)
// bf16 [rows, K] -> e4m3 [rows, K] with per-row scale absmax/448; warp per row.
__global__ void __launch_bounds__(256) quantize_rows_e4m3_kernel(const __nv_bfloat16* __restrict__ in,
                                                                 const int* __restrict__ m_valid, int k,
                                                                 uint8_t* __restrict__ out, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int rows = *m_valid;
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += gridDim.x * (blockDim.x >> 5)) {
    const __nv_bfloat16* src = in + static_cast<size_t>(row) * k;
    float amax = 0.0f;
    for (int c = lane * 8; c < k; c += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(src + c);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fmaxf(fabsf(bf16_lo(w[i])), fabsf(bf16_hi(w[i]))));
    }
    amax = warp_max(amax);
    const float s = amax > 0.0f ? amax * (1.0f / 448.0f) : 1.0f;
    const float inv = 1.0f / s;
    if (lane == 0) scale[row] = s;
    for (int c = lane * 8; c < k; c += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(src + c);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
      uint2 o;
      o.x = pack_e4m3x4(bf16_lo(w[0]) * inv, bf16_hi(w[0]) * inv, bf16_lo(w[1]) * inv, bf16_hi(w[1]) * inv);
      o.y = pack_e4m3x4(bf16_lo(w[2]) * inv, bf16_hi(w[2]) * inv, bf16_lo(w[3]) * inv, bf16_hi(w[3]) * inv);
      *reinterpret_cast<uint2*>(out + static_cast<size_t>(row) * k + c) = o;
    }
  }
}

// ------------------------------------------------------------------ heads
// Philox4x32-10 (Salmon et al., SC'11), from the paper's round function.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
  }
  return c;
}

// Heads. Persistent CTAs (4 warps) walk the states; W_p is staged in shared
// memory once per CTA. Lane l owns the float4 column groups l, l+32, ... so
// y loads are coalesced and W_p reads are conflict-free LDS.128. Each lane
// forms partial dots for all PP (= P rounded up to 8/16/32) actions, then a
// butterfly reduce-scatter leaves logit p in lanes p*32/PP .. +32/PP-1.
//   logits[b, j, :] = W_p.y_j + b_p (valid j), 0 (padded); actions = argmax
//   (+ Gumbel noise when sampling), -1 (padded); value[b] = W_v.mean_j(y_j) + b_v.
template <int DPL, int PP, bool LOGITS_BF16, bool VALUE_BF16>
__global__ void __launch_bounds__(128) heads_kernel(const float* __restrict__ y, const int* __restrict__ offsets,
                                                    int batch, int n_entities, int n_actions,
                                                    const float* __restrict__ w_p, const float* __restrict__ b_p,
                                                    const float* __restrict__ w_v, const float* __restrict__ b_v,
                                                    int sample, uint64_t seed, void* __restrict__ logits,
                                                    void* __restrict__ value, int* __restrict__ actions) {
  constexpr int D = DPL * 32;
  constexpr int G = DPL / 4;  // float4 groups per lane
  constexpr int LOG_PP = PP == 8 ? 3 : (PP == 16 ? 4 : 5);
  extern __shared__ float smem[];
  float* s_wp = smem;              // [PP][D], rows >= n_actions zero
  float* s_pool = smem + PP * D;   // [4][D]
  for (int i = threadIdx.x; i < PP * D; i += blockDim.x) s_wp[i] = (i / D) < n_actions ? w_p[i] : 0.0f;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int my_p = lane >> (5 - LOG_PP);
  const bool writer = (lane & ((32 / PP) - 1)) == 0 && my_p < n_actions;
  const float my_bias = my_p < n_actions ? b_p[my_p] : 0.0f;
  for (int b = blockIdx.x; b < batch; b += gridDim.x) {
    const int row0 = offsets[b];
    const int cnt = offsets[b + 1] - row0;
    float4 pool[G];
#pragma unroll
    for (int g = 0; g < G; ++g) pool[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = warp; j < n_entities; j += 4) {
      const size_t slot = static_cast<size_t>(b) * n_entities + j;
      if (j >= cnt) {
        if (writer) {
          if (LOGITS_BF16)
            reinterpret_cast<__nv_bfloat16*>(logits)[slot * n_actions + my_p] = __float2bfloat16_rn(0.0f);
          else
            reinterpret_cast<float*>(logits)[slot * n_actions + my_p] = 0.0f;
        }
        if (lane == 0) actions[slot] = -1;
        continue;
      }
      float4 yv[G];
      const float4* yr = reinterpret_cast<const float4*>(y + static_cast<size_t>(row0 + j) * D);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        yv[g] = yr[lane + 32 * g];
        pool[g].x += yv[g].x;
        pool[g].y += yv[g].y;
        pool[g].z += yv[g].z;
        pool[g].w += yv[g].w;
      }
      float v[PP];
#pragma unroll
      for (int p = 0; p < PP; ++p) {
        float a = 0.0f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 w = *reinterpret_cast<const float4*>(s_wp + p * D + 4 * (lane + 32 * g));
          a = fmaf(yv[g].x, w.x, fmaf(yv[g].y, w.y, fmaf(yv[g].z, w.z, fmaf(yv[g].w, w.w, a))));
        }
        v[p] = a;
      }
      // reduce-scatter: each level halves the values a lane keeps
#pragma unroll
      for (int lvl = 0; lvl < LOG_PP; ++lvl) {
        const int o = 16 >> lvl;
        const int half = PP >> (lvl + 1);
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < half; ++k) {
          const float send = upper ? v[k] : v[k + half];
          const float keep = upper ? v[k + half] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
#pragma unroll
      for (int o = (16 >> LOG_PP); o > 0; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
      float lg = v[0] + my_bias;
      if (LOGITS_BF16) lg = __bfloat162float(__float2bfloat16_rn(lg));
      if (writer) {
        if (LOGITS_BF16)
          reinterpret_cast<__nv_bfloat16*>(logits)[slot * n_actions + my_p] = __float2bfloat16_rn(lg);
        else
          reinterpret_cast<float*>(logits)[slot * n_actions + my_p] = lg;
      }
      float score = my_p < n_actions ? lg : -INFINITY;
      if (sample && my_p < n_actions) {
        const uint4 r = philox4x32_10(make_uint4(static_cast<uint32_t>(my_p) >> 2, static_cast<uint32_t>(j),
                                                 static_cast<uint32_t>(b), 0u),
                                      static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
        const int w4 = my_p & 3;
        const uint32_t word = w4 == 0 ? r.x : (w4 == 1 ? r.y : (w4 == 2 ? r.z : r.w));
        const float u = (static_cast<float>(word) + 0.5f) * 2.3283064365386963e-10f;
        score += -logf(-logf(u));
      }
      int idx = my_p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float os = __shfl_xor_sync(0xffffffffu, score, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (os > score || (os == score && oi < idx)) {
          score = os;
          idx = oi;
        }
      }
      if (lane == 0) actions[slot] = idx;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) *reinterpret_cast<float4*>(s_pool + warp * D + 4 * (lane + 32 * g)) = pool[g];
    __syncthreads();
    if (warp == 0) {
      float part = 0.0f;
      for (int c = lane; c < D; c += 32) {
        const float m = s_pool[c] + s_pool[D + c] + s_pool[2 * D + c] + s_pool[3 * D + c];
        part = fmaf(m, w_v[c], part);
      }
      part = warp_sum(part);
      if (lane == 0) {
        const float v = b_v[0] + (cnt > 0 ? part / static_cast<float>(cnt) : 0.0f);
        if (VALUE_BF16)
          reinterpret_cast<__nv_bfloat16*>(value)[b] = __float2bfloat16_rn(v);
        else
          reinterpret_cast<float*>(value)[b] = v;
      }
    }
    __syncthreads();  // s_pool reused by the next state
  }
}

}  // namespace ow
