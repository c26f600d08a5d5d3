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
  pdl_trigger();  // the next kernel on the stream may start launching
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
// TILE x TILE output tile (64: 4x4 per thread, K step 16; 32: 2x2 per thread,
// K step 64), 256 threads; the small tile gives small batches four times the
// CTAs and a quarter of the K steps (each a load and two barriers). Each output
// sums its K products in ascending order either way, so both tiles give the
// same bits. Rows >= *m_valid are skipped.
template <int EPI, int TILE = 64>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, const float* __restrict__ W,
                                                       const float* __restrict__ bias, float* __restrict__ C,
                                                       const int* __restrict__ m_valid, int n, int k) {
  constexpr int kPer = TILE / 16;           // outputs per thread along each axis
  constexpr int kStep = TILE == 32 ? 64 : 16;
  __shared__ float As[kStep][TILE + 4];
  __shared__ float Ws[kStep][TILE + 4];
  const int rows = *m_valid;
  const int m0 = blockIdx.y * TILE, n0 = blockIdx.x * TILE;
  if (m0 >= rows) return;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[kPer][kPer] = {};
  for (int k0 = 0; k0 < k; k0 += kStep) {
    for (int i = threadIdx.x; i < TILE * kStep; i += 256) {
      const int r = i / kStep, kk = i % kStep;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      As[kk][r] = (gm < rows && gk < k) ? A[static_cast<size_t>(gm) * k + gk] : 0.0f;
      Ws[kk][r] = (gn < n && gk < k) ? W[static_cast<size_t>(gn) * k + gk] : 0.0f;
    }
    __syncthreads();
#pragma unroll 16
    for (int kk = 0; kk < kStep; ++kk) {
      float a[kPer], w[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        a[i] = As[kk][ty * kPer + i];
        w[i] = Ws[kk][tx * kPer + i];
      }
#pragma unroll
      for (int i = 0; i < kPer; ++i)
#pragma unroll
        for (int j = 0; j < kPer; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int gm = m0 + ty * kPer + i;
    if (gm >= rows) continue;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int gn = n0 + tx * kPer + j;
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
// qkv: [rows, 3d]; out: [rows, d]. Keys and values of one state live in shared
// memory (row pitch 33: lanes reading different rows at one column hit
// different banks). A warp takes one query at a time: lane j forms score j as
// a 32-term dot product from shared memory (no shuffles), then a warp max and
// sum for the softmax, and lane c the output column c.
template <int NMAX>
__global__ void __launch_bounds__(128) attention_f32_kernel(const float* __restrict__ qkv, float* __restrict__ out,
                                                            const int* __restrict__ offsets, int d, float scale) {
  __shared__ float sk[NMAX][33];
  __shared__ float sv[NMAX][33];
  __shared__ float sq[4][32];
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
    sq[w][lane] = qkv[static_cast<size_t>(row0 + i) * ld + h * 32 + lane];
    __syncwarp();
    float mx = -INFINITY;
    for (int j = lane; j < cnt; j += 32) {
      float s = 0.0f;
#pragma unroll
      for (int c = 0; c < 32; ++c) s = fmaf(sq[w][c], sk[j][c], s);
      s *= scale;
      sp[w][j] = s;
      mx = fmaxf(mx, s);
    }
    mx = warp_max(mx);
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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Masked attention, bf16 tensor cores (mma.sync m16n8k16), one CTA per
// (state, group of HG heads), 8 warps. The group's Q, K and V columns of all
// the state's rows are copied into shared memory with cp.async (each row is
// three contiguous HG*64-byte runs); the row pitch HG*32+8 elements keeps the
// ldmatrix reads conflict-free. A (head, 16-query block) task: S = Q K^T on
// tensor cores, masked softmax over keys j < count in registers (fp32),
// O = P V on tensor cores, O / rowsum written as bf16.
// One (head, 16-query block) task with NKT 16-key blocks (the state's keys
// rounded up to 16): S = Q K^T, masked softmax, O = P V.
template <int NKT, int PITCH>
__device__ __forceinline__ void attention_task(const __nv_bfloat16* sq, const __nv_bfloat16* sk,
                                               const __nv_bfloat16* sv, int hc, int q0, int cnt, int lane,
                                               float scale_log2, __nv_bfloat16* __restrict__ out_row0, int d,
                                               int out_col) {
  constexpr int NT = 2 * NKT;
  const int g = lane >> 2, t = lane & 3;
  uint32_t qa[2][4];
  {
    const int r = q0 + (lane & 15);
    const int c = hc + (lane >> 4) * 8;
    ldsm_x4(smem_u32(sq + r * PITCH + c), qa[0][0], qa[0][1], qa[0][2], qa[0][3]);
    ldsm_x4(smem_u32(sq + r * PITCH + 16 + c), qa[1][0], qa[1][1], qa[1][2], qa[1][3]);
  }
  float s[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
    uint32_t k0, k1, k2, k3;
    ldsm_x4(smem_u32(sk + (j * 8 + (lane & 7)) * PITCH + hc + (lane >> 3) * 8), k0, k1, k2, k3);
    mma_bf16_16816(s[j], qa[0][0], qa[0][1], qa[0][2], qa[0][3], k0, k1);
    mma_bf16_16816(s[j], qa[1][0], qa[1][1], qa[1][2], qa[1][3], k2, k3);
  }
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
  // P is rounded to bf16 for the PV product: the single-instruction MUFU
  // exponential (relative error ~2^-22) is exact enough and saves the
  // range-handling instructions of exp2f (masked scores are -inf -> 0)
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    s[j][0] = ex2_approx_f(fmaf(s[j][0], scale_log2, -off0));
    s[j][1] = ex2_approx_f(fmaf(s[j][1], scale_log2, -off0));
    s[j][2] = ex2_approx_f(fmaf(s[j][2], scale_log2, -off1));
    s[j][3] = ex2_approx_f(fmaf(s[j][3], scale_log2, -off1));
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
  for (int kk = 0; kk < NKT; ++kk) {
    const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
    const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
    const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
    for (int np = 0; np < 2; ++np) {
      uint32_t v0, v1, v2, v3;
      const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int col = hc + np * 16 + (lane >> 4) * 8;
      ldsm_x4_t(smem_u32(sv + key * PITCH + col), v0, v1, v2, v3);
      mma_bf16_16816(o[2 * np], a0, a1, a2, a3, v0, v1);
      mma_bf16_16816(o[2 * np + 1], a0, a1, a2, a3, v2, v3);
    }
  }
  const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
  const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int col = out_col + n * 8 + 2 * t;
    if (r0 < cnt)
      *reinterpret_cast<uint32_t*>(out_row0 + static_cast<size_t>(r0) * d + col) = pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
    if (r1 < cnt)
      *reinterpret_cast<uint32_t*>(out_row0 + static_cast<size_t>(r1) * d + col) = pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
  }
}

// Masked attention, bf16 tensor cores (mma.sync m16n8k16), one CTA per
// (state, group of HG heads), 8 warps. The group's Q, K and V columns of the
// state's rows are copied into shared memory with cp.async (lanes along a
// row's 16-byte chunks, warps along rows); the row pitch HG*32+8 elements
// keeps ldmatrix conflict-free. Each (head, 16-query block) task runs exactly
// the state's ceil(count/16) key blocks.
template <int NMAX, int HG>
__global__ void __launch_bounds__(256, 4) attention_bf16_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                              __nv_bfloat16* __restrict__ out,
                                                              const int* __restrict__ offsets, int d,
                                                              float scale_log2) {
  constexpr int W = HG * 32;       // columns per matrix in the group
  constexpr int PITCH = W + 8;     // bf16 elements per staged row
  constexpr int CP = W / 8;        // 16-byte chunks per row per matrix
  constexpr int RPI = 32 / CP > 0 ? 32 / CP : 1;  // rows per warp iteration
  extern __shared__ __align__(16) __nv_bfloat16 s_qkv[];  // [3][NMAX][PITCH]
  __nv_bfloat16* sq = s_qkv;
  __nv_bfloat16* sk = s_qkv + NMAX * PITCH;
  __nv_bfloat16* sv = s_qkv + 2 * NMAX * PITCH;
  pdl_wait();  // q, k, v come from the projection launched before
  const int b = blockIdx.x, hg = blockIdx.y;
  const int row0 = offsets[b];
  const int cnt = offsets[b + 1] - row0;
  if (cnt <= 0) return;
  const int cnt16 = (cnt + 15) & ~15;
  const size_t ld = static_cast<size_t>(3) * d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const int ch = CP >= 32 ? lane : lane % CP;
    const int rsub = CP >= 32 ? 0 : lane / CP;
#pragma unroll
    for (int mat = 0; mat < 3; ++mat) {
      for (int r = warp * RPI + rsub; r < cnt16; r += 8 * RPI) {
        for (int c = ch; c < CP; c += 32) {
          __nv_bfloat16* dst = s_qkv + (mat * NMAX + r) * PITCH + c * 8;
          if (r < cnt)
            cp_async16(dst, qkv + static_cast<size_t>(row0 + r) * ld + mat * d + hg * W + c * 8);
          else
            *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
        }
      }
    }
  }
  cp_async_wait_all();
  __syncthreads();
  const int rblocks = cnt16 / 16;
  __nv_bfloat16* out_row0 = out + static_cast<size_t>(row0) * d;
  for (int task = warp; task < HG * rblocks; task += 8) {
    const int hh = task / rblocks, q0 = (task % rblocks) * 16;
    const int hc = hh * 32;
    const int oc = hg * W + hc;
    switch (rblocks) {
      case 1: attention_task<1, PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
      case 2: attention_task<2, PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
      case 3: attention_task<3, PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
      case 4: attention_task<4, PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
      case 5: if (NMAX >= 80) attention_task<(NMAX >= 80 ? 5 : 1), PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
      case 6: if (NMAX >= 96) attention_task<(NMAX >= 96 ? 6 : 1), PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
      case 7: if (NMAX >= 112) attention_task<(NMAX >= 112 ? 7 : 1), PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
      default: if (NMAX >= 128) attention_task<(NMAX >= 128 ? 8 : 1), PITCH>(sq, sk, sv, hc, q0, cnt, lane, scale_log2, out_row0, d, oc); break;
    }
  }
  pdl_trigger();  // the next kernel on the stream may start launching
}

// ------------------------------------------------------------------ embedding on tensor cores
// Both kernels are latency-bound: fewer registers per thread buy more resident
// warps. Measured at config 2: embed 41 -> 34 us with 64-column passes at 5 CTAs
// per SM, heads 38 -> 31 us at 6 CTAs per SM.
constexpr int kEmbedGroupCols = 64;  // output columns per MMA pass of embed_mma_kernel
constexpr int kEmbedMinBlocks = 5;   // register budget: CTAs of 128 threads per SM
constexpr int kHeadsMinBlocks = 6;

// Entity embedding + the first block's LayerNorm for the bf16 / fp8 paths.
// Packed row r is entity j = r - offsets[b] of state b (offsets[b] <= r <
// offsets[b+1], found by binary search). A warp takes 16 consecutive packed
// rows: features (f32 -> bf16) times W_e^T (K = 32 features) on m16n8k16
// tensor cores, kEmbedGroupCols output columns at a time. The MMA is
// recomputed per pass rather than held: pass 1 row statistics (each lane sums
// its columns shifted by its first value; the four lanes of a quad, which
// share a row, merge mean and M2 exactly, Chan et al.), [pass 2 e4m3 row
// absmax], last pass writes x (f32) and the LN output.
// XB: the residual stream x is stored as bf16 (else f32).
template <int D, int LN_MODE, bool XB>  // LN_MODE 1: bf16 out; 2: e4m3 out + per-row scale
__global__ void __launch_bounds__(128, kEmbedMinBlocks) embed_mma_kernel(const float* __restrict__ feats, const int* __restrict__ offsets,
                                                        int batch, int n_entities, int n_feat,
                                                        const __nv_bfloat16* __restrict__ w_e16,  // [D][32] bf16
                                                        const float* __restrict__ b_e,
                                                        const float* __restrict__ g, const float* __restrict__ beta,
                                                        void* __restrict__ x, void* __restrict__ ln_out,
                                                        float* __restrict__ ln_scale, int* __restrict__ row_slot) {
  constexpr int WP = 40;  // bf16 pitch of staged rows (32 features + pad: conflict-free ldmatrix)
  constexpr int kGW = kEmbedGroupCols;  // output columns per MMA pass (accumulators: kGW / 2 registers)
  constexpr int CG = D / kGW;
  extern __shared__ __align__(16) uint8_t smem_e[];
  __nv_bfloat16* s_w = reinterpret_cast<__nv_bfloat16*>(smem_e);         // [D][WP]
  __nv_bfloat16* s_f = s_w + D * WP;                                      // [4][16][WP]
  float* s_vec = reinterpret_cast<float*>(s_f + 4 * 16 * WP);            // bias, gamma, beta [3][D]
  {
    // batched 16-byte copies: issue every load of a batch before any store
    constexpr int kChunks = D * 4;  // 16-byte chunks of the [D][32] bf16 matrix
    constexpr int kPer = (kChunks + 127) / 128;
    uint4 v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + 128 * k;
      v[k] = i < kChunks ? reinterpret_cast<const uint4*>(w_e16)[i] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + 128 * k;
      if (i < kChunks) *reinterpret_cast<uint4*>(s_w + (i >> 2) * WP + (i & 3) * 8) = v[k];
    }
    constexpr int kVec = 3 * D / 4;  // float4s of bias, gamma, beta
    constexpr int kPerV = (kVec + 127) / 128;
    float4 u[kPerV];
#pragma unroll
    for (int k = 0; k < kPerV; ++k) {
      const int i = threadIdx.x + 128 * k;
      const int which = i / (D / 4), off = i % (D / 4);
      const float* src = which == 0 ? b_e : (which == 1 ? g : beta);
      u[k] = i < kVec ? reinterpret_cast<const float4*>(src)[off] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < kPerV; ++k) {
      const int i = threadIdx.x + 128 * k;
      if (i < kVec) reinterpret_cast<float4*>(s_vec)[i] = u[k];
    }
  }
  pdl_wait();  // weights above are constant; offsets and features come from earlier work
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, t = lane & 3;
  const int M = offsets[batch];
  __nv_bfloat16* sf = s_f + warp * 16 * WP;
  for (int blk = blockIdx.x * 4 + warp; blk * 16 < M; blk += gridDim.x * 4) {
    const int r0 = blk * 16;
    {  // stage 16 rows of features as bf16: lane -> (row lane & 15, features half*16 .. +15)
      const int rr = r0 + (lane & 15), half = lane >> 4;
      float fv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) fv[i] = 0.0f;
      if (rr < M) {
        int lo = 0, hi = batch;  // offsets[lo] <= rr < offsets[hi]
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (offsets[mid] <= rr) lo = mid;
          else hi = mid;
        }
        const size_t slot = static_cast<size_t>(lo) * n_entities + (rr - offsets[lo]);
        if (half == 0) row_slot[rr] = static_cast<int>(slot);
        const float* src = feats + slot * n_feat;
        if (n_feat == 32) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 v4 = reinterpret_cast<const float4*>(src + half * 16)[q];
            fv[4 * q] = v4.x;
            fv[4 * q + 1] = v4.y;
            fv[4 * q + 2] = v4.z;
            fv[4 * q + 3] = v4.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (half * 16 + i < n_feat) fv[i] = src[half * 16 + i];
        }
      }
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pk[i] = pack_bf16x2(fv[2 * i], fv[2 * i + 1]);
      uint4* dst = reinterpret_cast<uint4*>(sf + (lane & 15) * WP + half * 16);
      dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
    __syncwarp();
    uint32_t qa[2][4];
    {
      const int r = lane & 15, c = (lane >> 4) * 8;
      ldsm_x4(smem_u32(sf + r * WP + c), qa[0][0], qa[0][1], qa[0][2], qa[0][3]);
      ldsm_x4(smem_u32(sf + r * WP + 16 + c), qa[1][0], qa[1][1], qa[1][2], qa[1][3]);
    }
    __syncwarp();  // sf is rewritten by the next block of this warp
    const int ra = r0 + gq, rb = r0 + gq + 8;
    float mean0 = 0.f, mean1 = 0.f, rstd0 = 1.f, rstd1 = 1.f, inv0 = 1.f, inv1 = 1.f;
    float sh0 = 0.f, sh1 = 0.f, q0 = 0.f, q1 = 0.f;  // statistics pass: shifts, shifted sums of squares
    constexpr int kPasses = LN_MODE == 2 ? 3 : 2;
#pragma unroll 1
    for (int pass = 0; pass < kPasses; ++pass) {
      float a0 = 0.f, a1 = 0.f;  // per-pass reductions for rows ra, rb
#pragma unroll 1
      for (int cg = 0; cg < CG; ++cg) {
        float acc[kGW / 8][4];
#pragma unroll
        for (int nt = 0; nt < kGW / 8; ++nt) {
          acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(smem_u32(s_w + (cg * kGW + nt * 8 + (lane & 7)) * WP + (lane >> 3) * 8), b0, b1, b2, b3);
          mma_bf16_16816(acc[nt], qa[0][0], qa[0][1], qa[0][2], qa[0][3], b0, b1);
          mma_bf16_16816(acc[nt], qa[1][0], qa[1][1], qa[1][2], qa[1][3], b2, b3);
        }
#pragma unroll
        for (int nt = 0; nt < kGW / 8; ++nt) {
          const int col = cg * kGW + nt * 8 + 2 * t;
          const float bz0 = s_vec[col], bz1 = s_vec[col + 1];
          const float v00 = acc[nt][0] + bz0, v01 = acc[nt][1] + bz1;  // row ra
          const float v10 = acc[nt][2] + bz0, v11 = acc[nt][3] + bz1;  // row rb
          if (pass == 0) {
            if (cg == 0 && nt == 0) {
              sh0 = v00;
              sh1 = v10;
            }
            const float d00 = v00 - sh0, d01 = v01 - sh0, d10 = v10 - sh1, d11 = v11 - sh1;
            a0 += d00 + d01;
            a1 += d10 + d11;
            q0 = fmaf(d00, d00, fmaf(d01, d01, q0));
            q1 = fmaf(d10, d10, fmaf(d11, d11, q1));
          } else {
            const float g0 = s_vec[D + col], g1 = s_vec[D + col + 1];
            const float e0 = s_vec[2 * D + col], e1 = s_vec[2 * D + col + 1];
            const float y00 = (v00 - mean0) * rstd0 * g0 + e0, y01 = (v01 - mean0) * rstd0 * g1 + e1;
            const float y10 = (v10 - mean1) * rstd1 * g0 + e0, y11 = (v11 - mean1) * rstd1 * g1 + e1;
            if (LN_MODE == 2 && pass == 1) {
              a0 = fmaxf(a0, fmaxf(fabsf(y00), fabsf(y01)));
              a1 = fmaxf(a1, fmaxf(fabsf(y10), fabsf(y11)));
            } else {
              if (ra < M) {
                if (XB)
                  *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(x) + static_cast<size_t>(ra) * D + col) =
                      pack_bf16x2(v00, v01);
                else
                  *reinterpret_cast<float2*>(reinterpret_cast<float*>(x) + static_cast<size_t>(ra) * D + col) = make_float2(v00, v01);
                if (LN_MODE == 1)
                  *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(ln_out) + static_cast<size_t>(ra) * D + col) =
                      pack_bf16x2(y00, y01);
                else
                  *reinterpret_cast<__nv_fp8x2_storage_t*>(reinterpret_cast<uint8_t*>(ln_out) + static_cast<size_t>(ra) * D + col) =
                      __nv_cvt_float2_to_fp8x2(make_float2(y00 * inv0, y01 * inv0), __NV_SATFINITE, __NV_E4M3);
              }
              if (rb < M) {
                if (XB)
                  *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(x) + static_cast<size_t>(rb) * D + col) =
                      pack_bf16x2(v10, v11);
                else
                  *reinterpret_cast<float2*>(reinterpret_cast<float*>(x) + static_cast<size_t>(rb) * D + col) = make_float2(v10, v11);
                if (LN_MODE == 1)
                  *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(ln_out) + static_cast<size_t>(rb) * D + col) =
                      pack_bf16x2(y10, y11);
                else
                  *reinterpret_cast<__nv_fp8x2_storage_t*>(reinterpret_cast<uint8_t*>(ln_out) + static_cast<size_t>(rb) * D + col) =
                      __nv_cvt_float2_to_fp8x2(make_float2(y10 * inv1, y11 * inv1), __NV_SATFINITE, __NV_E4M3);
              }
            }
          }
        }
      }
      // reduce over the quad (the 4 lanes sharing rows ra, rb)
      if (LN_MODE == 2 && pass == 1) {
        a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
        a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
        const float sc0 = a0 > 0.f ? a0 * (1.0f / 448.0f) : 1.0f, sc1 = a1 > 0.f ? a1 * (1.0f / 448.0f) : 1.0f;
        inv0 = 1.0f / sc0;
        inv1 = 1.0f / sc1;
        if (t == 0 && ra < M) ln_scale[ra] = sc0;
        if (t == 0 && rb < M) ln_scale[rb] = sc1;
      } else if (pass == 0) {
        // per lane: mean and M2 over its D/4 columns; merged over the quad in two
        // steps of equal counts (the same operations in every lane of the quad)
        float cnt = static_cast<float>(D / 4);
        float m0 = sh0 + a0 / cnt, m1 = sh1 + a1 / cnt;
        float M0 = fmaxf(q0 - a0 * a0 / cnt, 0.0f), M1 = fmaxf(q1 - a1 * a1 / cnt, 0.0f);
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          const float om0 = __shfl_xor_sync(0xffffffffu, m0, o), oM0 = __shfl_xor_sync(0xffffffffu, M0, o);
          const float om1 = __shfl_xor_sync(0xffffffffu, m1, o), oM1 = __shfl_xor_sync(0xffffffffu, M1, o);
          const float e0 = om0 - m0, e1 = om1 - m1;
          M0 = (M0 + oM0) + e0 * e0 * (0.5f * cnt);
          M1 = (M1 + oM1) + e1 * e1 * (0.5f * cnt);
          m0 = 0.5f * (m0 + om0);
          m1 = 0.5f * (m1 + om1);
          cnt *= 2.0f;
        }
        mean0 = m0;
        mean1 = m1;
        rstd0 = rsqrtf(M0 * (1.0f / D) + 1e-5f);
        rstd1 = rsqrtf(M1 * (1.0f / D) + 1e-5f);
      }
    }
  }
  pdl_trigger();  // the next kernel on the stream may start launching
}

// ------------------------------------------------------------------ e4m3 quantiser (fp8 path)
// bf16 [rows, K] -> e4m3 [rows, K] with per-row scale absmax/448; warp per row.
__global__ void __launch_bounds__(256) quantize_rows_e4m3_kernel(const __nv_bfloat16* __restrict__ in,
                                                                 const int* __restrict__ m_valid, int k,
                                                                 uint8_t* __restrict__ out, float* __restrict__ scale) {
  pdl_wait();  // the rows come from the kernel launched before
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
  pdl_trigger();  // the next kernel on the stream may start launching
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
    constexpr int TOK = DPL <= 8 ? 4 : 2;  // tokens in flight per warp
    for (int j0 = warp * TOK; j0 < n_entities; j0 += 4 * TOK) {
      float4 yv[TOK][G];
      float v[TOK][PP];
#pragma unroll
      for (int u = 0; u < TOK; ++u) {
        const int j = j0 + u;
        const bool valid = j < cnt;
        const float4* yr = reinterpret_cast<const float4*>(y + static_cast<size_t>(row0 + (valid ? j : 0)) * D);
#pragma unroll
        for (int gg = 0; gg < G; ++gg) yv[u][gg] = valid ? yr[lane + 32 * gg] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < TOK; ++u) {
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
          pool[gg].x += yv[u][gg].x;
          pool[gg].y += yv[u][gg].y;
          pool[gg].z += yv[u][gg].z;
          pool[gg].w += yv[u][gg].w;
        }
#pragma unroll
        for (int p = 0; p < PP; ++p) {
          float a = 0.0f;
#pragma unroll
          for (int gg = 0; gg < G; ++gg) {
            const float4 w = *reinterpret_cast<const float4*>(s_wp + p * D + 4 * (lane + 32 * gg));
            a = fmaf(yv[u][gg].x, w.x, fmaf(yv[u][gg].y, w.y, fmaf(yv[u][gg].z, w.z, fmaf(yv[u][gg].w, w.w, a))));
          }
          v[u][p] = a;
        }
      }
      // reduce-scatter: each level halves the values a lane keeps (TOK chains interleaved)
#pragma unroll
      for (int lvl = 0; lvl < LOG_PP; ++lvl) {
        const int o = 16 >> lvl;
        const int half = PP >> (lvl + 1);
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < half; ++k) {
#pragma unroll
          for (int u = 0; u < TOK; ++u) {
            const float send = upper ? v[u][k] : v[u][k + half];
            const float keep = upper ? v[u][k + half] : v[u][k];
            v[u][k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
      }
#pragma unroll
      for (int o = (16 >> LOG_PP); o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < TOK; ++u) v[u][0] += __shfl_xor_sync(0xffffffffu, v[u][0], o);
#pragma unroll
      for (int u = 0; u < TOK; ++u) {
        const int j = j0 + u;
        if (j >= n_entities) continue;
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
        float lg = v[u][0] + my_bias;
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
          const float uu = (static_cast<float>(word) + 0.5f) * 2.3283064365386963e-10f;
          score += -logf(-logf(uu));
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

// Heads on tensor cores (tf32 mma.sync m16n8k8, f32 accumulate) for the
// bf16 / fp8 paths. A warp takes 16 packed rows of the final LayerNorm
// output y (f32). Output columns: P policy logits, then the value column
// W_v (mean_j(y_j).W_v == mean_j(y_j.W_v)), padded to 8-column tiles. The K
// index is permuted identically for A and B so that each thread's fragments
// are float4 loads: in a 16-column group, thread t owns columns 4t..4t+3,
// used as slots (t, t+4) of two consecutive k-steps.
// Per row: logits (rounded to the logits dtype) -> logits[slot], greedy or
// Gumbel-max action -> actions[slot], y.W_v -> sval[row]. Padded slots and
// the value are written by state_finalize_kernel.
__device__ __forceinline__ uint32_t to_tf32(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ void mma_tf32_1688(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int D, int NTILE, bool LOGITS_BF16>  // NTILE = 8-column tiles covering P logits + the value column
__global__ void __launch_bounds__(128, kHeadsMinBlocks) heads_mma_kernel(const float* __restrict__ y, const int* __restrict__ offsets,
                                                        int batch, int n_entities, int n_actions,
                                                        const int* __restrict__ row_slot,
                                                        const float* __restrict__ w_p, const float* __restrict__ b_p,
                                                        const float* __restrict__ w_v, int sample, uint64_t seed,
                                                        int state_base,
                                                        void* __restrict__ logits, int* __restrict__ actions,
                                                        float* __restrict__ sval) {
  constexpr int WPITCH = D + 16;  // f32 pitch: float4 fragment loads are conflict-free
  extern __shared__ __align__(16) float s_wh[];  // [NTILE*8][WPITCH]
  {
    // batched 16-byte copies, every load of the batch issued before any store
    // (a load-store loop here cost one L2 round trip per element per thread)
    constexpr int kQuads = NTILE * 8 * D / 4;
    constexpr int kPer = (kQuads + 127) / 128;
    float4 v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + 128 * k;
      const int n = (4 * i) / D, kk = (4 * i) % D;
      v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < kQuads) {
        if (n < n_actions) v[k] = *reinterpret_cast<const float4*>(w_p + n * D + kk);
        else if (n == n_actions) v[k] = *reinterpret_cast<const float4*>(w_v + kk);
      }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + 128 * k;
      if (i < kQuads) *reinterpret_cast<float4*>(s_wh + ((4 * i) / D) * WPITCH + (4 * i) % D) = v[k];
    }
  }
  pdl_wait();  // the head weights above are constant; y comes from the last block
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int M = offsets[batch];
  for (int blk = blockIdx.x * 4 + warp; blk * 16 < M; blk += gridDim.x * 4) {
    const int r0 = blk * 16;
    const int ra = r0 + g, rb = r0 + g + 8;
    const float* ya = y + static_cast<size_t>(ra < M ? ra : 0) * D;
    const float* yb = y + static_cast<size_t>(rb < M ? rb : 0) * D;
    float c[NTILE][4];
#pragma unroll
    for (int n = 0; n < NTILE; ++n) c[n][0] = c[n][1] = c[n][2] = c[n][3] = 0.0f;
#pragma unroll 4
    for (int gk = 0; gk < D / 16; ++gk) {
      const float4 va = *reinterpret_cast<const float4*>(ya + gk * 16 + 4 * t);
      const float4 vb = *reinterpret_cast<const float4*>(yb + gk * 16 + 4 * t);
      const uint32_t a0x = to_tf32(va.x), a0y = to_tf32(va.y), a0z = to_tf32(va.z), a0w = to_tf32(va.w);
      const uint32_t a1x = to_tf32(vb.x), a1y = to_tf32(vb.y), a1z = to_tf32(vb.z), a1w = to_tf32(vb.w);
#pragma unroll
      for (int n = 0; n < NTILE; ++n) {
        const float4 wv = *reinterpret_cast<const float4*>(s_wh + (n * 8 + g) * WPITCH + gk * 16 + 4 * t);
        // k-step A uses columns 4t, 4t+1 as slots t, t+4; k-step B columns 4t+2, 4t+3
        mma_tf32_1688(c[n], a0x, a1x, a0y, a1y, to_tf32(wv.x), to_tf32(wv.y));
        mma_tf32_1688(c[n], a0z, a1z, a0w, a1w, to_tf32(wv.z), to_tf32(wv.w));
      }
    }
    // c[n]: rows g (0,1) and g+8 (2,3), columns n*8 + 2t, +1
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? rb : ra;
      const bool live = r < M;
      int slot = 0, sb = 0, sj = 0;
      if (live) {
        slot = row_slot[r];
        sb = slot / n_entities;
        sj = slot - sb * n_entities;
      }
      float best = -INFINITY;
      int besti = 0x7fffffff;
#pragma unroll
      for (int n = 0; n < NTILE; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int p = n * 8 + 2 * t + e;
          float v = c[n][2 * half + e];
          if (p < n_actions) {
            v += b_p[p];
            if (LOGITS_BF16) v = __bfloat162float(__float2bfloat16_rn(v));
            float score = v;
            if (sample) {
              const uint4 rr = philox4x32_10(make_uint4(static_cast<uint32_t>(p) >> 2, static_cast<uint32_t>(sj),
                                                        static_cast<uint32_t>(sb + state_base), 0u),
                                             static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
              const int w4 = p & 3;
              const uint32_t word = w4 == 0 ? rr.x : (w4 == 1 ? rr.y : (w4 == 2 ? rr.z : rr.w));
              const float uu = (static_cast<float>(word) + 0.5f) * 2.3283064365386963e-10f;
              score += -logf(-logf(uu));
            }
            if (live) {
              if (LOGITS_BF16)
                reinterpret_cast<__nv_bfloat16*>(logits)[static_cast<size_t>(slot) * n_actions + p] = __float2bfloat16_rn(v);
              else
                reinterpret_cast<float*>(logits)[static_cast<size_t>(slot) * n_actions + p] = v;
            }
            if (score > best || (score == best && p < besti)) {
              best = score;
              besti = p;
            }
          } else if (p == n_actions && live) {
            sval[r] = v;
          }
        }
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ob > best || (ob == best && oi < besti)) {
          best = ob;
          besti = oi;
        }
      }
      if (t == 0 && live) actions[slot] = besti;
    }
  }
  pdl_trigger();  // the next kernel on the stream may start launching
}

// Per state: value = b_v + mean over its rows of sval; padded entity slots
// get logits 0 and action -1. One CTA of n_entities (rounded to 32) threads.
template <bool LOGITS_BF16, bool VALUE_BF16>
__global__ void state_finalize_kernel(const int* __restrict__ offsets, int n_entities, int n_actions,
                                      const float* __restrict__ sval, const float* __restrict__ b_v,
                                      void* __restrict__ logits, void* __restrict__ value,
                                      int* __restrict__ actions) {
  pdl_wait();  // sval comes from the heads kernel
  __shared__ float s_red[4];
  const int b = blockIdx.x, j = threadIdx.x;
  const int row0 = offsets[b];
  const int cnt = offsets[b + 1] - row0;
  float v = 0.0f;
  if (j < cnt) v = sval[row0 + j];
  if (j >= cnt && j < n_entities) {
    const size_t slot = static_cast<size_t>(b) * n_entities + j;
    for (int p = 0; p < n_actions; ++p) {
      if (LOGITS_BF16)
        reinterpret_cast<__nv_bfloat16*>(logits)[slot * n_actions + p] = __float2bfloat16_rn(0.0f);
      else
        reinterpret_cast<float*>(logits)[slot * n_actions + p] = 0.0f;
    }
    actions[slot] = -1;
  }
  v = warp_sum(v);
  if ((j & 31) == 0) s_red[j >> 5] = v;
  __syncthreads();
  if (j == 0) {
    float s = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += s_red[w];
    const float out = b_v[0] + (cnt > 0 ? s / static_cast<float>(cnt) : 0.0f);
    if (VALUE_BF16)
      reinterpret_cast<__nv_bfloat16*>(value)[b] = __float2bfloat16_rn(out);
    else
      reinterpret_cast<float*>(value)[b] = out;
  }
}

}  // namespace ow
