// Persistent tcgen05 GEMM for the encoder blocks: out[m, n] = A[m, :] . W[n, :] + epilogue.
//
//   A: activations, [rows, K] K-major (bf16 or e4m3), loaded by TMA with 128 B swizzle
//   W: weights, [N, K] K-major ([out, in] as stored), same loader
//   D: f32 accumulators in TMEM (128 lanes x BLOCK_N columns, double-buffered
//      when two tiles fit in the 512 columns so the epilogue of tile i
//      overlaps the MMAs of tile i+1)
//
// Roles: warp 0 lane 0 issues TMA, warp 1 lane 0 issues tcgen05.mma (and
// warp 1 owns the TMEM allocation), the epilogue warps drain TMEM. A warp may
// only read TMEM lanes 32*(warp%4)..+31, i.e. 32 rows of the tile; the
// bias/GELU epilogues run 8 warps (two per lane quadrant, each taking half of
// the columns), the LayerNorm epilogue 4 (one thread owns one whole row).
// Bias, LayerNorm gamma/beta and fp8 channel scales are staged in shared
// memory once per CTA and read as broadcast float4.
//
// The number of valid rows is read from device memory (the packed token
// count of the batch), so one launch shape serves every batch; tiles past the
// valid rows are never scheduled.
//
// Epilogues:
//   kEpiBias       out = bf16(acc*s + bias)                        (QKV projection)
//   kEpiBiasGelu   out = bf16(gelu(acc*s + bias))                  (FFN up-projection)
//   kEpiResidLn    x   = x + acc*s + bias in place (fp32 residual stream),
//                  and the LayerNorm of that row (BLOCK_N == d, the whole
//                  row is in this tile) -> ln_out as bf16 (next GEMM's A),
//                  e4m3 + per-row scale (fp8 path), or f32 (the final LN
//                  feeding the heads)                              (out-proj, FFN down-projection)
// where s = a_scale[m]*b_scale[n] for e4m3 operands and 1 otherwise.
#pragma once

#include "ow_common.cuh"

namespace ow {

enum EpiMode : int { kEpiBias = 0, kEpiBiasGelu = 1, kEpiResidLn = 2 };
enum LnMode : int { kLnBf16 = 0, kLnE4m3 = 1, kLnF32 = 2 };

struct TcGemmParams {
  const int* m_valid;  // device scalar: rows to compute
  int n;               // output columns (multiple of BLOCK_N)
  int k_blocks;        // K / (128 bytes of elements)
  const float* bias;   // [n]
  __nv_bfloat16* out;  // kEpiBias / kEpiBiasGelu: [rows, ld_out]
  int ld_out;
  float* resid;           // kEpiResidLn: x [rows, n] f32, updated in place
  const float* ln_g;      // [n]
  const float* ln_b;      // [n]
  void* ln_out;           // [rows, n]: bf16, e4m3 or f32 per ln_mode
  float* ln_scale;        // [rows] per-row dequant scale of ln_out (e4m3 only)
  int ln_mode;            // kLnBf16, kLnE4m3, kLnF32
  const float* a_scale;   // [rows] (e4m3 operands only)
  const float* b_scale;   // [n]    (e4m3 operands only)
  int* err;
};

constexpr int kParamFloats = 4096;  // staged epilogue vectors (bias + scales, or bias/g/b/scales)
constexpr int kSmemLimit = 232448;   // dynamic shared memory per CTA on sm_100

template <int EPI>
struct EpiWarps {
  static constexpr int kCount = EPI == kEpiResidLn ? 4 : 8;
  static constexpr int kThreads = 64 + 32 * kCount;
};

template <int BLOCK_N, int EPI>
struct TcGemmShape {
  static constexpr int kBlockM = 128;
  static constexpr int kRowBytes = 128;  // one swizzle atom row: 64 bf16 or 128 e4m3
  static constexpr int kATileBytes = kBlockM * kRowBytes;
  static constexpr int kBTileBytes = BLOCK_N * kRowBytes;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kInstN = BLOCK_N <= 256 ? BLOCK_N : BLOCK_N / 2;   // N of one tcgen05.mma
  static constexpr int kInstCount = BLOCK_N / kInstN;
  static constexpr int kBoxRows = BLOCK_N <= 256 ? BLOCK_N : BLOCK_N / 2;  // TMA box rows for W (<= 256)
  static constexpr int kBoxCount = BLOCK_N / kBoxRows;
  static constexpr int kAcc = (2 * BLOCK_N <= 512) ? 2 : 1;
  static constexpr int kTmemColsNeeded = BLOCK_N * kAcc;
  static constexpr int kTmemCols = kTmemColsNeeded <= 32 ? 32
                                   : kTmemColsNeeded <= 64 ? 64
                                   : kTmemColsNeeded <= 128 ? 128
                                   : kTmemColsNeeded <= 256 ? 256 : 512;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kParamBytes = kParamFloats * 4;
  static constexpr int kXposeBytes = EpiWarps<EPI>::kCount * 4096;  // per-warp 32 x 128 B transpose tile
  static constexpr int kFixedBytes = kBarrierBytes + kParamBytes + kXposeBytes + 1024;  // + align slack
  static constexpr int kStagesFit = (kSmemLimit - kFixedBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
  static constexpr int kSmemBytes = kStages * kStageBytes + kFixedBytes;
  static_assert(kStages >= 2, "at least double-buffered operand stages");
  static_assert(kInstN % 16 == 0 && kInstN <= 256, "M=128 UMMA needs N % 16 == 0, N <= 256");
  static_assert(kBoxRows <= 256, "TMA box rows <= 256");
  static_assert(kTmemColsNeeded <= 512, "TMEM has 512 columns");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory per CTA");
};

// Warp-cooperative transpose through a 32 x 128 B shared tile. 16-byte chunk
// j of row r lives at chunk slot j ^ (r & 7), so both the row-per-thread side
// (thread r touches row r) and the row-per-8-lanes side (8 lanes cover one
// 128 B row) are bank-conflict free.
__device__ __forceinline__ uint4* xpose_slot(uint8_t* tile, int row, int chunk) {
  return reinterpret_cast<uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4));
}
// rows [0, rows) of the tile -> global rows of `row_bytes` bytes (chunks_per_row 16 B chunks each)
__device__ __forceinline__ void xpose_store(uint8_t* tile, uint8_t* gbase, size_t gstride, int rows, int chunks_per_row,
                                            int lane) {
  const int rows_per_iter = 32 / chunks_per_row;
  const int j = lane % chunks_per_row;
  for (int r = lane / chunks_per_row; r < rows; r += rows_per_iter)
    *reinterpret_cast<uint4*>(gbase + r * gstride + j * 16) = *xpose_slot(tile, r, j);
}
__device__ __forceinline__ void xpose_load(uint8_t* tile, const uint8_t* gbase, size_t gstride, int rows,
                                           int chunks_per_row, int lane) {
  const int rows_per_iter = 32 / chunks_per_row;
  const int j = lane % chunks_per_row;
  for (int r = lane / chunks_per_row; r < rows; r += rows_per_iter)
    *xpose_slot(tile, r, j) = *reinterpret_cast<const uint4*>(gbase + r * gstride + j * 16);
}

template <int BLOCK_N, int EPI, bool FP8>
__global__ void __launch_bounds__(EpiWarps<EPI>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                   const TcGemmParams p) {
  using S = TcGemmShape<BLOCK_N, EPI>;
  constexpr int kEpiWarps = EpiWarps<EPI>::kCount;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + S::kStages * S::kATileBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* tfull = empty + S::kStages;
  uint64_t* tempty = tfull + S::kAcc;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + S::kAcc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_par = reinterpret_cast<float*>(smem + S::kStages * S::kStageBytes + S::kBarrierBytes);
  uint8_t* s_xpose = smem + S::kStages * S::kStageBytes + S::kBarrierBytes + S::kParamBytes;
  // staged vectors: s_bias[n], then (fp8) s_bscale[n], then (LN) s_g[n], s_b[n]
  float* s_bias = s_par;
  float* s_bscale = s_par + p.n;
  float* s_g = s_par + (FP8 ? 2 : 1) * p.n;
  float* s_b = s_g + p.n;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_valid = *p.m_valid;
  const int m_tiles = (m_valid + S::kBlockM - 1) / S::kBlockM;
  const int n_tiles = p.n / BLOCK_N;
  const int num_tiles = m_tiles * n_tiles;
  constexpr uint32_t kIdesc = FP8 ? idesc_e4m3(128, S::kInstN) : idesc_bf16(128, S::kInstN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < S::kAcc; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, S::kTmemCols);
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
    s_bias[i] = p.bias[i];
    if (FP8) s_bscale[i] = p.b_scale[i];
    if (EPI == kEpiResidLn) {
      s_g[i] = p.ln_g[i];
      s_b[i] = p.ln_b[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0 && num_tiles > 0) {
      tma_prefetch_desc(&map_a);
      tma_prefetch_desc(&map_w);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * S::kBlockM;
        const int n0 = (tile % n_tiles) * BLOCK_N;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          const int kx = kb * (FP8 ? 128 : 64);
          tma_load_2d(sa + stage * S::kATileBytes, &map_a, &full[stage], kx, m0);
#pragma unroll
          for (int c = 0; c < S::kBoxCount; ++c)
            tma_load_2d(sb + stage * S::kBTileBytes + c * S::kBoxRows * S::kRowBytes, &map_w, &full[stage], kx,
                        n0 + c * S::kBoxRows);
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && num_tiles > 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BLOCK_N);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sa + stage * S::kATileBytes);
          const uint32_t b_base = smem_u32(sb + stage * S::kBTileBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 4 x 32 bytes of K per 128-byte row
            const uint64_t adesc = sdesc_k_sw128(a_base + k * 32);
#pragma unroll
            for (int c = 0; c < S::kInstCount; ++c) {
              const uint64_t bdesc = sdesc_k_sw128(b_base + c * S::kInstN * S::kRowBytes + k * 32);
              const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
              if (FP8)
                umma_f8(d_tmem + c * S::kInstN, adesc, bdesc, kIdesc, accumulate);
              else
                umma_f16(d_tmem + c * S::kInstN, adesc, bdesc, kIdesc, accumulate);
            }
          }
          umma_commit(&empty[stage]);  // smem stage reusable once these MMAs retire
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);  // accumulator ready for the epilogue
        if (++acc == S::kAcc) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    // Epilogue warps 2 .. 2+kEpiWarps-1. Thread `lane` of a warp owns tile row
    // quad*32 + lane on the TMEM side; global traffic goes through the warp's
    // transpose tile so each warp instruction moves whole 128 B rows.
    const int quad = warp & 3;
    uint8_t* xt = s_xpose + (warp - 2) * 4096;
    constexpr int kCols = EPI == kEpiResidLn ? BLOCK_N : BLOCK_N * 4 / kEpiWarps;  // columns this warp drains
    const int col0 = EPI == kEpiResidLn ? 0 : ((warp - 2) / 4) * kCols;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err)) break;
      tc_fence_after();
      const int row_base = (tile / n_tiles) * S::kBlockM + quad * 32;  // first row of this warp's 32
      const int m = row_base + lane;
      const int rows = min(32, m_valid - row_base);                    // valid rows of the 32 (may be <= 0)
      const int n0 = (tile % n_tiles) * BLOCK_N;
      const bool live = m < m_valid;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BLOCK_N);
      const float a_s = (FP8 && live) ? p.a_scale[m] : 1.0f;

      if (EPI == kEpiBias || EPI == kEpiBiasGelu) {
        static_assert(kCols % 64 == 0, "64-column epilogue chunks");
#pragma unroll 1
        for (int c = col0; c < col0 + kCols; c += 64) {
          uint32_t r[64];
          tmem_ld32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld32(tbase + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          tmem_ld_wait();
          uint32_t packed[32];
#pragma unroll
          for (int i = 0; i < 64; i += 4) {
            const float4 bv = *reinterpret_cast<const float4*>(s_bias + n0 + c + i);
            float v0 = __uint_as_float(r[i]), v1 = __uint_as_float(r[i + 1]);
            float v2 = __uint_as_float(r[i + 2]), v3 = __uint_as_float(r[i + 3]);
            if (FP8) {
              const float4 sv = *reinterpret_cast<const float4*>(s_bscale + n0 + c + i);
              v0 *= a_s * sv.x;
              v1 *= a_s * sv.y;
              v2 *= a_s * sv.z;
              v3 *= a_s * sv.w;
            }
            v0 += bv.x;
            v1 += bv.y;
            v2 += bv.z;
            v3 += bv.w;
            if (EPI == kEpiBiasGelu) {
              v0 = gelu_erf(v0);
              v1 = gelu_erf(v1);
              v2 = gelu_erf(v2);
              v3 = gelu_erf(v3);
            }
            packed[i / 2] = pack_bf16x2(v0, v1);
            packed[i / 2 + 1] = pack_bf16x2(v2, v3);
          }
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *xpose_slot(xt, lane, q) = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          __syncwarp();
          if (rows > 0)
            xpose_store(xt, reinterpret_cast<uint8_t*>(p.out + static_cast<size_t>(row_base) * p.ld_out + n0 + c),
                        static_cast<size_t>(p.ld_out) * 2, rows, 8, lane);
          __syncwarp();
        }
      } else {
        // Residual add + LayerNorm over the full row (BLOCK_N == n == d): two
        // passes over TMEM. Pass 1 forms v = x + acc*s + bias, writes it back to
        // TMEM and accumulates shifted statistics (shift = the row's first v,
        // which keeps E[(v-k)^2] - E[v-k]^2 well conditioned); pass 2 writes x
        // and the normalised row.
        uint8_t* xg = reinterpret_cast<uint8_t*>(p.resid + static_cast<size_t>(row_base > 0 ? row_base : 0) * BLOCK_N);
        const size_t xstride = static_cast<size_t>(BLOCK_N) * 4;
        float shift = 0.0f, s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
        for (int c = 0; c < BLOCK_N; c += 32) {
          if (rows > 0) xpose_load(xt, xg + c * 4, xstride, rows, 8, lane);  // 32 rows x 32 f32 of x
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
          tmem_ld_wait();
          __syncwarp();
          float xv[32];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 t4 = live ? *reinterpret_cast<const float4*>(xpose_slot(xt, lane, q)) : make_float4(0.f, 0.f, 0.f, 0.f);
            xv[4 * q] = t4.x;
            xv[4 * q + 1] = t4.y;
            xv[4 * q + 2] = t4.z;
            xv[4 * q + 3] = t4.w;
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 bv = *reinterpret_cast<const float4*>(s_bias + c + i);
            float4 sv = make_float4(1.f, 1.f, 1.f, 1.f);
            if (FP8) sv = *reinterpret_cast<const float4*>(s_bscale + c + i);
            const float b4[4] = {bv.x, bv.y, bv.z, bv.w};
            const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float v = __uint_as_float(r[i + j]);
              if (FP8) v *= a_s * s4[j];
              v += b4[j] + xv[i + j];
              if (c == 0 && i + j == 0) shift = v;
              const float dv = v - shift;
              s1 += dv;
              s2 = fmaf(dv, dv, s2);
              r[i + j] = __float_as_uint(v);
            }
          }
          tmem_st32(tbase + c, r);
        }
        tmem_st_wait();
        const float md = s1 * (1.0f / BLOCK_N);
        const float var = fmaxf(s2 * (1.0f / BLOCK_N) - md * md, 0.0f);
        const float mean = shift + md;
        const float rstd = rsqrtf(var + 1e-5f);
        float inv_scale = 1.0f;
        if (p.ln_mode == kLnE4m3) {
          float amax = 0.0f;
#pragma unroll 1
          for (int c = 0; c < BLOCK_N; c += 32) {
            uint32_t r[32];
            tmem_ld32(tbase + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float y = (__uint_as_float(r[i]) - mean) * rstd * s_g[c + i] + s_b[c + i];
              amax = fmaxf(amax, fabsf(y));
            }
          }
          const float scale = amax > 0.0f ? amax * (1.0f / 448.0f) : 1.0f;
          inv_scale = 1.0f / scale;
          if (live) p.ln_scale[m] = scale;
        }
        const int ln_elt = p.ln_mode == kLnF32 ? 4 : (p.ln_mode == kLnE4m3 ? 1 : 2);
        uint8_t* lg = reinterpret_cast<uint8_t*>(p.ln_out) + static_cast<size_t>(row_base > 0 ? row_base : 0) * BLOCK_N * ln_elt;
        const size_t lstride = static_cast<size_t>(BLOCK_N) * ln_elt;
#pragma unroll 1
        for (int c = 0; c < BLOCK_N; c += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
          tmem_ld_wait();
          // x (f32): 32 columns = one 128 B row segment per thread
#pragma unroll
          for (int q = 0; q < 8; ++q) *xpose_slot(xt, lane, q) = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          __syncwarp();
          if (rows > 0) xpose_store(xt, xg + c * 4, xstride, rows, 8, lane);
          __syncwarp();
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 gv = *reinterpret_cast<const float4*>(s_g + c + i);
            const float4 bv = *reinterpret_cast<const float4*>(s_b + c + i);
            y[i] = (__uint_as_float(r[i]) - mean) * rstd * gv.x + bv.x;
            y[i + 1] = (__uint_as_float(r[i + 1]) - mean) * rstd * gv.y + bv.y;
            y[i + 2] = (__uint_as_float(r[i + 2]) - mean) * rstd * gv.z + bv.z;
            y[i + 3] = (__uint_as_float(r[i + 3]) - mean) * rstd * gv.w + bv.w;
          }
          int chunks;
          if (p.ln_mode == kLnE4m3) {
            uint32_t q8[8];
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              q8[i / 4] = pack_e4m3x4(y[i] * inv_scale, y[i + 1] * inv_scale, y[i + 2] * inv_scale,
                                      y[i + 3] * inv_scale);
            *xpose_slot(xt, lane, 0) = make_uint4(q8[0], q8[1], q8[2], q8[3]);
            *xpose_slot(xt, lane, 1) = make_uint4(q8[4], q8[5], q8[6], q8[7]);
            chunks = 2;
          } else if (p.ln_mode == kLnF32) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *xpose_slot(xt, lane, q) = make_uint4(__float_as_uint(y[4 * q]), __float_as_uint(y[4 * q + 1]),
                                                    __float_as_uint(y[4 * q + 2]), __float_as_uint(y[4 * q + 3]));
            chunks = 8;
          } else {
            uint32_t yo[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) yo[i / 2] = pack_bf16x2(y[i], y[i + 1]);
#pragma unroll
            for (int q = 0; q < 4; ++q) *xpose_slot(xt, lane, q) = make_uint4(yo[4 * q], yo[4 * q + 1], yo[4 * q + 2], yo[4 * q + 3]);
            chunks = 4;
          }
          __syncwarp();
          if (rows > 0) xpose_store(xt, lg + c * ln_elt, lstride, rows, chunks, lane);
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == S::kAcc) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace ow
