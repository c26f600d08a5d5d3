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
// Epilogue I/O is TMA-only: each epilogue warp owns 32 x 128 B staging tiles
// in the 128 B-swizzled layout (16 B chunk j of row r at slot j ^ (r & 7)),
// which the row-per-thread TMEM side writes without bank conflicts; outputs
// leave as asynchronous tiled TMA stores (bulk groups), and the LayerNorm
// epilogue's residual rows arrive as double-buffered TMA loads.
//
// The number of valid rows is read from device memory (the packed token
// count of the batch), so one launch shape serves every batch; tiles past the
// valid rows are never scheduled.
//
// Epilogues:
//   kEpiBias       out = bf16(acc*s + bias)                        (QKV projection)
//   kEpiBiasGelu   out = bf16(gelu(acc*s + bias))                  (FFN up-projection)
// map_o is the output map (bf16, box EpiWarps<EPI>::kChunkCols x 32 rows, in
// the swizzle of that row width) for the bias epilogues and the
// f32 residual map (box 32 x 32) for the LayerNorm epilogue; map_l is the
// LayerNorm output map (box 128 B x 32 rows of its dtype).
//   kEpiResidLn    x   = x + acc*s + bias in place (fp32 residual stream),
//                  and the LayerNorm of that row (BLOCK_N == d, the whole
//                  row is in this tile) -> ln_out as bf16 (next GEMM's A),
//                  e4m3 + per-row scale (fp8 path), or f32 (the final LN
//                  feeding the heads)                              (out-proj, FFN down-projection)
// where s = a_scale[m]*b_scale[n] for e4m3 operands and 1 otherwise.
#pragma once

#include "ow_common.cuh"

namespace ow {

enum EpiMode : int { kEpiBias = 0, kEpiBiasGelu = 1, kEpiResidLn = 2, kEpiResidLn16 = 3 };
enum LnMode : int { kLnBf16 = 0, kLnE4m3 = 1, kLnF32 = 2 };

struct TcGemmParams {
  const int* m_valid;  // device scalar: rows to compute
  int n;               // output columns (multiple of BLOCK_N)
  int k_blocks;        // K / (128 bytes of elements)
  const float* bias;   // [n]
  const float* bias2;  // fused FFN: b2 [d]
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
  int a_stream;           // A is read once and not again (the FFN hidden activations): load it evict_first
};

constexpr int kSmemLimit = 232448;  // dynamic shared memory per CTA on sm_100

#ifndef OW_BIAS_EPI_WARPS
#define OW_BIAS_EPI_WARPS 16
#endif
#ifndef OW_BIAS_CHUNK_COLS
#define OW_BIAS_CHUNK_COLS 32
#endif
#ifndef OW_GELU_EPI_WARPS
#define OW_GELU_EPI_WARPS 16
#endif
#ifndef OW_GELU_CHUNK_COLS
#define OW_GELU_CHUNK_COLS 32
#endif

// Epilogue warps per CTA and, for the bias / GELU epilogues, the columns of one
// output chunk (one TMA store box of 32 rows: 32 columns = 64 B rows, 64 = 128 B).
template <int EPI>
struct EpiWarps {
  static constexpr int kCount = EPI == kEpiResidLn ? 8
                                : EPI == kEpiResidLn16 ? 16
                                : (EPI == kEpiBias ? OW_BIAS_EPI_WARPS : OW_GELU_EPI_WARPS);
  static constexpr int kThreads = 64 + 32 * kCount;
  static constexpr int kChunkCols = EPI == kEpiBias ? OW_BIAS_CHUNK_COLS : OW_GELU_CHUNK_COLS;
  static_assert(kChunkCols == 32 || kChunkCols == 64, "output chunks of 64 B or 128 B rows");
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
  static constexpr int kBarrierBytes = 512;
  static constexpr int kParamFloats = EPI == kEpiResidLn ? 2048 : (EPI == kEpiResidLn16 ? 1024 : 4096);  // staged bias/scale/g/b vectors
  static constexpr int kParamBytes = kParamFloats * 4;
  // staging tiles (4 KB) per epilogue warp, used by the TMA loads of the
  // residual and the TMA stores of the outputs: 2, or 1 at d = 512 (budget)
  // (the bf16-residual LayerNorm epilogue keeps one tile per warp: its 32 rows x
  // 64 columns of the residual, rewritten in place by x and then the LN output)
  static constexpr int kTilesPerWarp = ((EPI == kEpiResidLn && BLOCK_N > 384) || EPI == kEpiResidLn16) ? 1 : 2;
  // bias/GELU epilogues stage 32 rows x kChunkCols bf16 columns; LayerNorm 32 x 128 B
  static constexpr int kTileBytes = (EPI == kEpiResidLn || EPI == kEpiResidLn16) ? 4096 : 32 * EpiWarps<EPI>::kChunkCols * 2;
  static constexpr int kXposeBytes = EpiWarps<EPI>::kCount * kTilesPerWarp * kTileBytes;
  // LayerNorm: per-row partial statistics exchanged between the two warps of a
  // lane quadrant: [2 parities][8 warps][32 lanes] x (mean, M2, amax, pad)
  // bf16-residual LayerNorm: (mean, M2) float2 and amax per [2 parities][16 warps][32 lanes]
  static constexpr int kStatsBytes = EPI == kEpiResidLn ? 2 * 8 * 32 * 16 : (EPI == kEpiResidLn16 ? 2 * 16 * 32 * 12 : 0);
  static constexpr int kWBytes = 0;  // resident weight slice (weight-stationary shape only)
  static constexpr int kFixedBytes = kBarrierBytes + kParamBytes + kXposeBytes + kStatsBytes + 1024;  // + align slack
  static constexpr int kStagesFit = (kSmemLimit - kFixedBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
  static constexpr int kSmemBytes = kStages * kStageBytes + kFixedBytes;
  static_assert(kStages >= 2, "at least double-buffered operand stages");
  static_assert(kInstN % 16 == 0 && kInstN <= 256, "M=128 UMMA needs N % 16 == 0, N <= 256");
  static_assert(kBoxRows <= 256, "TMA box rows <= 256");
  static_assert(kTmemColsNeeded <= 512, "TMEM has 512 columns");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory per CTA");
  static_assert(kStageBytes % 1024 == 0 && kXposeBytes % 1024 == 0, "swizzled tiles stay 1024 B aligned");
  static_assert(EPI != kEpiResidLn16 || BLOCK_N == 256, "bf16-residual LayerNorm epilogue: d = 256 (64 columns per warp)");
};

// Weight-stationary shape for the bias / GELU epilogues at BLOCK_N = 256 and
// K of at most 4 k-blocks (bf16 K <= 256, e4m3 K <= 512): the CTA's 256-row
// slice of W (up to 128 KB) is loaded once and stays in shared memory for all
// of the CTA's row tiles (the persistent grid is a multiple of the column
// tiles, so tile = blockIdx.x + k * gridDim.x keeps one slice per CTA); only
// A streams through the stages, 16 KB per k-block instead of 48 KB, so three
// stages cover three k-blocks of MMAs where the streaming shape fits three of
// 48 KB. One staging tile per epilogue warp.
template <int EPI>
struct TcGemmWsShape : TcGemmShape<256, EPI> {
  using Base = TcGemmShape<256, EPI>;
  static constexpr int kMaxKBlocks = 4;
  static constexpr int kStageBytes = Base::kATileBytes;
  static constexpr int kWBytes = kMaxKBlocks * Base::kBTileBytes;
  static constexpr int kTilesPerWarp = 1;
  static constexpr int kXposeBytes = EpiWarps<EPI>::kCount * kTilesPerWarp * Base::kTileBytes;
  static constexpr int kParamFloats = 2048;
  static constexpr int kParamBytes = kParamFloats * 4;
  static constexpr int kFixedBytes = Base::kBarrierBytes + kParamBytes + kXposeBytes + kWBytes + 1024;
  static constexpr int kStagesFit = (kSmemLimit - kFixedBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kSmemBytes = kStages * kStageBytes + kFixedBytes;
  static_assert(EPI == kEpiBias || EPI == kEpiBiasGelu, "weight-stationary shape: bias / GELU epilogues");
  static_assert(kStages >= 2, "at least double-buffered A stages");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory per CTA");
  static_assert(kWBytes % 1024 == 0 && kXposeBytes % 1024 == 0, "swizzled tiles stay 1024 B aligned");
};
template <int BLOCK_N, int EPI, bool WS>
struct GemmShapeSel {
  using T = TcGemmShape<BLOCK_N, EPI>;
};
template <int EPI>
struct GemmShapeSel<256, EPI, true> {
  using T = TcGemmWsShape<EPI>;
};

// 16 B chunk j of row r of a 32 x 128 B staging tile (128 B swizzle).
__device__ __forceinline__ uint4* xpose_slot(uint8_t* tile, int row, int chunk) {
  return reinterpret_cast<uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4));
}
// Same for 32 x 64 B boxes (64 B swizzle: chunk j of row r at j ^ ((r >> 1) & 3)).
__device__ __forceinline__ uint4* xpose_slot64(uint8_t* tile, int row, int chunk) {
  return reinterpret_cast<uint4*>(tile + row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
}
// Same for 32 x 32 B boxes (32 B swizzle: chunk j of row r at j ^ ((r >> 2) & 1)).
__device__ __forceinline__ uint4* xpose_slot32(uint8_t* tile, int row, int chunk) {
  return reinterpret_cast<uint4*>(tile + row * 32 + ((chunk ^ ((row >> 2) & 1)) << 4));
}

// Rendezvous of the two epilogue warps that share a lane quadrant: all 64
// threads arrive on the pair's mbarrier (count 64) and wait for the phase,
// bounded like every other wait (an expired wait raises the abort flag and the
// kernel runs out without further waiting).
__device__ __forceinline__ void pair_sync(uint64_t* bar, uint32_t& phase, volatile int* abort, int* err) {
  mbar_arrive(bar);
  mbar_wait(bar, phase, abort, err);
  phase ^= 1u;
}
__device__ __forceinline__ bool pair_sync_ok(uint64_t* bar, uint32_t& phase, volatile int* abort, int* err) {
  mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase, abort, err);
  phase ^= 1u;
  return ok;
}

// Residual add + LayerNorm over a full row (BLOCK_N == n == d) for one
// epilogue warp: TMEM lanes of quadrant `quad`, columns [half*BLOCK_N/2, +BLOCK_N/2)
// with half = ew / 4; the other half of each row is the epilogue warp ew ^ 4.
// The caller has issued the residual loads of this warp's first NT chunks
// (tile b <- columns cbase + b*32) on my_xbar[b]; bit b of xbits is that
// barrier's phase parity. Pass 1: v = x + acc*s + bias,
// written back to TMEM, shifted statistics per half; the halves' (mean, M2)
// are merged exactly (Chan et al.) through `st` and the pair's mbarrier
// (64 arrivals, bounded wait). Pass 2: x and the LN output leave by TMA
// stores from the warp's staging tiles.
// One 32-column chunk of LayerNorm output of this thread's row into a staging
// tile, in the box layout of its dtype (bf16: 64 B rows, e4m3: 32 B, f32: 128 B).
__device__ __forceinline__ void ln_to_staging(const float (&y)[32], uint8_t* lt, int lane, int ln_mode,
                                              float inv_scale) {
  if (ln_mode == kLnE4m3) {
    uint32_t q8[8];
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      q8[i / 4] = pack_e4m3x4(y[i] * inv_scale, y[i + 1] * inv_scale, y[i + 2] * inv_scale, y[i + 3] * inv_scale);
    *xpose_slot32(lt, lane, 0) = make_uint4(q8[0], q8[1], q8[2], q8[3]);
    *xpose_slot32(lt, lane, 1) = make_uint4(q8[4], q8[5], q8[6], q8[7]);
  } else if (ln_mode == kLnF32) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *xpose_slot(lt, lane, q) = make_uint4(__float_as_uint(y[4 * q]), __float_as_uint(y[4 * q + 1]),
                                            __float_as_uint(y[4 * q + 2]), __float_as_uint(y[4 * q + 3]));
  } else {
    uint32_t yo[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) yo[i / 2] = pack_bf16x2(y[i], y[i + 1]);
#pragma unroll
    for (int q = 0; q < 4; ++q) *xpose_slot64(lt, lane, q) = make_uint4(yo[4 * q], yo[4 * q + 1], yo[4 * q + 2], yo[4 * q + 3]);
  }
}

template <int BLOCK_N, bool FP8, int NT>
__device__ __forceinline__ void resid_ln_epilogue(uint32_t tbase, uint8_t* tiles, uint64_t* my_xbar, uint32_t& xbits,
                                                  float4* st, const float* s_bias, const float* s_bscale,
                                                  const float* s_g, const float* s_b, const CUtensorMap* map_o,
                                                  const CUtensorMap* map_l, const TcGemmParams& p,
                                                  volatile int* abort_flag, uint64_t* pair_bar, uint32_t& pair_phase,
                                                  int ew, int quad, int lane, int row_base, int m, bool live,
                                                  float a_s) {
  constexpr int HW = BLOCK_N / 2;
  constexpr int kChunks = HW / 32;
  const int half = ew >> 2;
  const int cbase = half * HW;
  // shifted sums in four interleaved partials (shorter dependency chains);
  // the next chunk's TMEM load is in flight while a chunk is processed
  float shift = 0.0f;
  float s1p[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s2p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  bool ok = true;
  uint32_t ra[32], rb[32];
  tmem_ld32(tbase + cbase, ra);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    uint32_t(&r)[32] = (c & 1) ? rb : ra;
    uint32_t(&rn)[32] = (c & 1) ? ra : rb;
    const int b = c % NT;
    if (!mbar_wait(&my_xbar[b], (xbits >> b) & 1u, abort_flag, p.err)) ok = false;
    xbits ^= 1u << b;
    tmem_ld_wait_dep(r);
    if (c + 1 < kChunks) tmem_ld32(tbase + cbase + (c + 1) * 32, rn);
    float xv[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 t4 = *reinterpret_cast<const float4*>(xpose_slot(tiles + b * 4096, lane, q));
      xv[4 * q] = t4.x;
      xv[4 * q + 1] = t4.y;
      xv[4 * q + 2] = t4.z;
      xv[4 * q + 3] = t4.w;
    }
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const int col = cbase + c * 32 + i;
      const float4 bv = *reinterpret_cast<const float4*>(s_bias + col);
      float4 sv = make_float4(1.f, 1.f, 1.f, 1.f);
      if (FP8) sv = *reinterpret_cast<const float4*>(s_bscale + col);
      const float b4[4] = {bv.x, bv.y, bv.z, bv.w};
      const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = __uint_as_float(r[i + j]);
        if (FP8) v *= a_s * s4[j];
        v += b4[j] + xv[i + j];
        if (c == 0 && i + j == 0) shift = v;
        const float dv = v - shift;
        s1p[j] += dv;
        s2p[j] = fmaf(dv, dv, s2p[j]);
        r[i + j] = __float_as_uint(v);
      }
    }
    tmem_st32(tbase + cbase + c * 32, r);
    // Refill staging tile b with chunk c + NT only now: the TMEM store consumes
    // every value read from the tile, so those shared-memory reads have
    // completed before the TMA write is issued (a write-after-read across
    // proxies; issued right after the reads, the TMA data could land first
    // while the tensor cores keep shared memory busy).
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && c + NT < kChunks && ok) {
      mbar_arrive_expect_tx(&my_xbar[b], 4096);
      tma_load_2d_hint(tiles + b * 4096, map_o, &my_xbar[b], cbase + (c + NT) * 32, row_base, l2_evict_last());
    }
  }
  const float s1 = (s1p[0] + s1p[1]) + (s1p[2] + s1p[3]);
  const float s2 = (s2p[0] + s2p[1]) + (s2p[2] + s2p[3]);
  tmem_st_wait();
  // merge the two halves' statistics (same operation order in both warps)
  const float mh = shift + s1 * (1.0f / HW);
  const float m2h = fmaxf(s2 - s1 * s1 * (1.0f / HW), 0.0f);
  st[ew * 32 + lane] = make_float4(mh, m2h, 0.0f, 0.0f);
  pair_sync(pair_bar, pair_phase, abort_flag, p.err);
  const float4 lo = st[(ew & 3) * 32 + lane];  // the pair: epilogue warps ew & 3 (half 0) and +4 (half 1)
  const float4 hi = st[((ew & 3) + 4) * 32 + lane];
  const float delta = hi.x - lo.x;
  const float mean = 0.5f * (lo.x + hi.x);
  const float var = (lo.y + hi.y + delta * delta * (0.25f * BLOCK_N)) * (1.0f / BLOCK_N);
  const float rstd = rsqrtf(var + 1e-5f);
  float inv_scale = 1.0f;
  if (p.ln_mode == kLnE4m3) {
    float amax = 0.0f;
#pragma unroll 1
    for (int c = 0; c < kChunks; ++c) {
      uint32_t r[32];
      tmem_ld32(tbase + cbase + c * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int col = cbase + c * 32 + i;
        const float y = (__uint_as_float(r[i]) - mean) * rstd * s_g[col] + s_b[col];
        amax = fmaxf(amax, fabsf(y));
      }
    }
    st[ew * 32 + lane].z = amax;
    pair_sync(pair_bar, pair_phase, abort_flag, p.err);
    amax = fmaxf(st[(ew & 3) * 32 + lane].z, st[((ew & 3) + 4) * 32 + lane].z);
    const float scale = amax > 0.0f ? amax * (1.0f / 448.0f) : 1.0f;
    inv_scale = 1.0f / scale;
    if (live && half == 0) p.ln_scale[m] = scale;
  }
  if constexpr (NT >= 2) {
    // x (staging tile 0) and the LN output (tile 1) of a chunk leave in one bulk
    // group behind one proxy fence; the next chunk waits for that group's reads
    uint8_t* xt = tiles;
    uint8_t* lt = tiles + 4096;
    uint32_t qa[32], qb[32];
    tmem_ld32(tbase + cbase, qa);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      uint32_t(&r)[32] = (c & 1) ? qb : qa;
      uint32_t(&rn)[32] = (c & 1) ? qa : qb;
      const int col0 = cbase + c * 32;
      if (lane == 0) bulk_wait_read<0>();
      tmem_ld_wait_dep(r);
      if (c + 1 < kChunks) tmem_ld32(tbase + cbase + (c + 1) * 32, rn);
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 8; ++q) *xpose_slot(xt, lane, q) = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
      float y[32];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 gv = *reinterpret_cast<const float4*>(s_g + col0 + i);
        const float4 bv = *reinterpret_cast<const float4*>(s_b + col0 + i);
        y[i] = (__uint_as_float(r[i]) - mean) * rstd * gv.x + bv.x;
        y[i + 1] = (__uint_as_float(r[i + 1]) - mean) * rstd * gv.y + bv.y;
        y[i + 2] = (__uint_as_float(r[i + 2]) - mean) * rstd * gv.z + bv.z;
        y[i + 3] = (__uint_as_float(r[i + 3]) - mean) * rstd * gv.w + bv.w;
      }
      ln_to_staging(y, lt, lane, p.ln_mode, inv_scale);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d_hint(map_o, xt, col0, row_base, l2_evict_last());
        tma_store_2d(map_l, lt, col0, row_base);
        bulk_commit();
      }
    }
  } else {
    // one staging tile (d = 512): x, then the LN output, each behind its own fence
    uint8_t* t = tiles;
#pragma unroll 1
    for (int c = 0; c < kChunks; ++c) {
      const int col0 = cbase + c * 32;
      uint32_t r[32];
      tmem_ld32(tbase + col0, r);
      if (lane == 0) bulk_wait_read<0>();
      tmem_ld_wait_dep(r);
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 8; ++q) *xpose_slot(t, lane, q) = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d_hint(map_o, t, col0, row_base, l2_evict_last());
        bulk_commit();
      }
      float y[32];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 gv = *reinterpret_cast<const float4*>(s_g + col0 + i);
        const float4 bv = *reinterpret_cast<const float4*>(s_b + col0 + i);
        y[i] = (__uint_as_float(r[i]) - mean) * rstd * gv.x + bv.x;
        y[i + 1] = (__uint_as_float(r[i + 1]) - mean) * rstd * gv.y + bv.y;
        y[i + 2] = (__uint_as_float(r[i + 2]) - mean) * rstd * gv.z + bv.z;
        y[i + 3] = (__uint_as_float(r[i + 3]) - mean) * rstd * gv.w + bv.w;
      }
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      ln_to_staging(y, t, lane, p.ln_mode, inv_scale);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map_l, t, col0, row_base);
        bulk_commit();
      }
    }
  }
}

// Residual add + LayerNorm with a bf16 residual stream, 16 epilogue warps
// (kEpiResidLn16, d = 256). Warp ew owns TMEM lane quadrant `quad` (32 rows,
// thread `lane` = row row_base + lane) and columns [64*(ew/4), +64) of them.
// Its staging tile receives those 32 rows x 64 bf16 columns of the residual
// (128 B rows, 128 B swizzle) by TMA when the tile starts, so they land while
// the MMAs run. Then
//   pass 1: v = x + acc*s + bias in packed f32x2 arithmetic, written back to
//           TMEM; shifted sums of the warp's 64 values per row;
//   merge:  the quadrant's four (mean, M2) partials meet in shared memory
//           (parity-double-buffered) at a 128-arrival mbarrier, and every warp
//           merges them in the same order (Chan et al., equal counts);
//   [fp8:   an absmax pass and a second rendezvous give the row's e4m3 scale;]
//   pass 2: x = bf16(v) into the staging tile in place of the residual (each
//           thread rewrites only its own row) and a TMA store; the LayerNorm
//           output is computed while that store reads the tile, then leaves
//           through the same tile (bf16: one 64-column box; e4m3: a 64 B-row
//           box; f32, the final LayerNorm: two 32-column boxes in turn).
// Row-per-thread global stores instead of the staging tile measured slower
// (each warp store touches 32 cache lines). The epilogue is issue-bound (the
// tensor cores run the next tile's MMAs on the other TMEM accumulator
// meanwhile), hence the packed arithmetic. The caller has issued the
// residual load on *xbar (phase parity xpar).
template <bool FP8>
__device__ __forceinline__ void resid_ln16_epilogue(uint32_t tbase, uint8_t* tile, uint64_t* xbar, uint32_t& xpar,
                                                    float2* st, float* st_amax, const float* s_bias,
                                                    const float* s_bscale, const float* s_g, const float* s_b,
                                                    const CUtensorMap* map_x, const CUtensorMap* map_l,
                                                    const TcGemmParams& p, volatile int* abort_flag,
                                                    uint64_t* quad_bar, uint32_t& quad_phase, int ew, int lane,
                                                    int row_base, int m, bool live, float a_s) {
  constexpr int kCols = 64;  // per warp
  constexpr int kChunks = kCols / 32;
  constexpr int kD = 256;
  const int cbase = (ew >> 2) * kCols;
  const int q0 = ew & 3;  // this quadrant's warps are q0, q0+4, q0+8, q0+12
  bool ok = mbar_wait(xbar, xpar, abort_flag, p.err);
  xpar ^= 1u;
  float2 shift = make_float2(0.0f, 0.0f);
  float2 s1 = make_float2(0.0f, 0.0f), s2 = make_float2(0.0f, 0.0f);
  uint32_t ra[32], rb[32];
  tmem_ld32(tbase + cbase, ra);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    uint32_t(&r)[32] = (c & 1) ? rb : ra;
    uint32_t(&rn)[32] = (c & 1) ? ra : rb;
    tmem_ld_wait_dep(r);
    if (c + 1 < kChunks) tmem_ld32(tbase + cbase + (c + 1) * 32, rn);
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // 16-byte chunk 4c+q of this thread's row: 8 bf16 residual values
      const uint4 u = *xpose_slot(tile, lane, 4 * c + q);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // 4 columns at a time
        const int i = 8 * q + 4 * h;
        const int col = cbase + c * 32 + i;
        const float4 bv = *reinterpret_cast<const float4*>(s_bias + col);
        float2 v0 = make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
        float2 v1 = make_float2(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
        if (FP8) {
          const float4 sv = *reinterpret_cast<const float4*>(s_bscale + col);
          v0 = mul_f2(v0, make_float2(a_s * sv.x, a_s * sv.y));
          v1 = mul_f2(v1, make_float2(a_s * sv.z, a_s * sv.w));
        }
        v0 = add_f2(add_f2(v0, make_float2(bv.x, bv.y)), bf16x2_to_f2(uw[2 * h]));
        v1 = add_f2(add_f2(v1, make_float2(bv.z, bv.w)), bf16x2_to_f2(uw[2 * h + 1]));
        if (c == 0 && i == 0) shift = make_float2(v0.x, v0.x);
        const float2 d0 = sub_f2(v0, shift), d1 = sub_f2(v1, shift);
        s1 = add_f2(s1, add_f2(d0, d1));
        s2 = fma_f2(d0, d0, fma_f2(d1, d1, s2));
        r[i] = __float_as_uint(v0.x);
        r[i + 1] = __float_as_uint(v0.y);
        r[i + 2] = __float_as_uint(v1.x);
        r[i + 3] = __float_as_uint(v1.y);
      }
    }
    tmem_st32(tbase + cbase + c * 32, r);
  }
  {
    const float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
    st[ew * 32 + lane] = make_float2(shift.x + t1 * (1.0f / kCols), fmaxf(t2 - t1 * t1 * (1.0f / kCols), 0.0f));
  }
  tmem_st_wait();
  if (!pair_sync_ok(quad_bar, quad_phase, abort_flag, p.err)) ok = false;
  // merge the four equal-count partials: (0,1), (2,3), then the two pairs
  const float2 w0 = st[(q0 + 0) * 32 + lane], w1 = st[(q0 + 4) * 32 + lane];
  const float2 w2 = st[(q0 + 8) * 32 + lane], w3 = st[(q0 + 12) * 32 + lane];
  const float d01 = w1.x - w0.x, d23 = w3.x - w2.x;
  const float m01 = 0.5f * (w0.x + w1.x), m23 = 0.5f * (w2.x + w3.x);
  const float M01 = w0.y + w1.y + d01 * d01 * (0.5f * kCols);
  const float M23 = w2.y + w3.y + d23 * d23 * (0.5f * kCols);
  const float dd = m23 - m01;
  const float mean = 0.5f * (m01 + m23);
  const float var = (M01 + M23 + dd * dd * kCols) * (1.0f / kD);
  const float rstd = rsqrtf(var + 1e-5f);
  const float2 mean2 = make_float2(mean, mean), rstd2 = make_float2(rstd, rstd);
  float inv_scale = 1.0f;
  if (p.ln_mode == kLnE4m3) {
    float amax = 0.0f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      uint32_t r[32];
      tmem_ld32(tbase + cbase + c * 32, r);
      tmem_ld_wait_dep(r);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const int col = cbase + c * 32 + i;
        const float2 y = fma_f2(mul_f2(sub_f2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), mean2), rstd2),
                                *reinterpret_cast<const float2*>(s_g + col), *reinterpret_cast<const float2*>(s_b + col));
        amax = fmaxf(amax, fmaxf(fabsf(y.x), fabsf(y.y)));
      }
    }
    st_amax[ew * 32 + lane] = amax;
    if (!pair_sync_ok(quad_bar, quad_phase, abort_flag, p.err)) ok = false;
    amax = fmaxf(fmaxf(st_amax[(q0 + 0) * 32 + lane], st_amax[(q0 + 4) * 32 + lane]),
                 fmaxf(st_amax[(q0 + 8) * 32 + lane], st_amax[(q0 + 12) * 32 + lane]));
    const float scale = amax > 0.0f ? amax * (1.0f / 448.0f) : 1.0f;
    inv_scale = 1.0f / scale;
    if (live && ew < 4) p.ln_scale[m] = scale;
  }
  // pass 2a: the new residual row, bf16, in place of the residual just read
  // (each thread rewrites only its own row), then one TMA store of the tile
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    uint32_t r[32];
    tmem_ld32(tbase + cbase + c * 32, r);
    tmem_ld_wait_dep(r);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *xpose_slot(tile, lane, 4 * c + q) =
          make_uint4(pack_bf16x2(__uint_as_float(r[8 * q]), __uint_as_float(r[8 * q + 1])),
                     pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                     pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                     pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && ok) {
    tma_store_2d_hint(map_x, tile, cbase, row_base, l2_evict_last());
    bulk_commit();
  }
  // pass 2b: the LayerNorm output through the same tile once that store has
  // read it (the first chunk is computed while it does); bf16: one 64-column
  // box, e4m3: one 64 B-row box, f32 (the final LayerNorm): one 32-column box
  // per chunk, in turn
  const bool f32_out = p.ln_mode == kLnF32;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    uint32_t r[32];
    tmem_ld32(tbase + cbase + c * 32, r);
    tmem_ld_wait_dep(r);
    float2 y[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const int col = cbase + c * 32 + i;
      y[i / 2] = fma_f2(mul_f2(sub_f2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), mean2), rstd2),
                        *reinterpret_cast<const float2*>(s_g + col), *reinterpret_cast<const float2*>(s_b + col));
    }
    if (c == 0 || f32_out) {
      if (lane == 0) bulk_wait_read<0>();  // the previous store has read the tile
      __syncwarp();
    }
    if (f32_out) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *xpose_slot(tile, lane, q) = make_uint4(__float_as_uint(y[2 * q].x), __float_as_uint(y[2 * q].y),
                                                __float_as_uint(y[2 * q + 1].x), __float_as_uint(y[2 * q + 1].y));
    } else if (p.ln_mode == kLnE4m3) {  // 32 rows x 64 B, 64 B swizzle: chunks 2c, 2c+1
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t q8[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 u = y[8 * h + 2 * i], v = y[8 * h + 2 * i + 1];
          q8[i] = pack_e4m3x4(u.x * inv_scale, u.y * inv_scale, v.x * inv_scale, v.y * inv_scale);
        }
        *xpose_slot64(tile, lane, 2 * c + h) = make_uint4(q8[0], q8[1], q8[2], q8[3]);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *xpose_slot(tile, lane, 4 * c + q) =
            make_uint4(pack_bf16x2(y[4 * q].x, y[4 * q].y), pack_bf16x2(y[4 * q + 1].x, y[4 * q + 1].y),
                       pack_bf16x2(y[4 * q + 2].x, y[4 * q + 2].y), pack_bf16x2(y[4 * q + 3].x, y[4 * q + 3].y));
    }
    if (f32_out || c + 1 == kChunks) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && ok) {
        tma_store_2d(map_l, tile, cbase + (f32_out ? 32 * c : 0), row_base);
        bulk_commit();
      }
    }
  }
}

template <int BLOCK_N, int EPI, bool FP8, bool WS = false>
__global__ void __launch_bounds__(EpiWarps<EPI>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                   const __grid_constant__ CUtensorMap map_o, const __grid_constant__ CUtensorMap map_l,
                   const TcGemmParams p) {
  using S = typename GemmShapeSel<BLOCK_N, EPI, WS>::T;
  static_assert(!WS || BLOCK_N == 256, "weight-stationary: BLOCK_N = 256");
  constexpr int kEpiWarps = EpiWarps<EPI>::kCount;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + S::kStages * S::kATileBytes;  // B stages, or (WS) the resident slice of W
  // layout: [operand stages][(WS) W slice][staging tiles (1024 B aligned: the
  // swizzle phase is taken from address bits)][barriers][epilogue vectors]
  uint8_t* s_xpose = smem + S::kStages * S::kStageBytes + S::kWBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_xpose + S::kXposeBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* tfull = empty + S::kStages;
  uint64_t* tempty = tfull + S::kAcc;
  uint64_t* xbar = tempty + S::kAcc;  // residual loads: one barrier per staging tile of each epilogue warp
  uint64_t* pair_bar = xbar + S::kTilesPerWarp * kEpiWarps;  // LayerNorm: one per lane quadrant (64 arrivals)
  uint64_t* w_full = pair_bar + 4;  // WS: the slice of W has landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(w_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_par = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + S::kBarrierBytes);
  float4* s_stats = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(s_par) + S::kParamBytes);
  // staged vectors: s_bias[n], then (fp8) s_bscale[n], then (LN) s_g[n], s_b[n]
  float* s_bias = s_par;
  float* s_bscale = s_par + p.n;
  float* s_g = s_par + (FP8 ? 2 : 1) * p.n;
  float* s_b = s_g + p.n;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles = p.n / BLOCK_N;
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
    for (int i = 0; i < S::kTilesPerWarp * kEpiWarps; ++i) mbar_init(&xbar[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], EPI == kEpiResidLn16 ? 128 : 64);
    mbar_init(w_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
    s_bias[i] = p.bias[i];
    if (FP8) s_bscale[i] = p.b_scale[i];
    if (EPI == kEpiResidLn || EPI == kEpiResidLn16) {
      s_g[i] = p.ln_g[i];
      s_b[i] = p.ln_b[i];
    }
  }
  // Everything above reads only weights; the operands, the residual and the
  // token count come from earlier kernels (programmatic dependent launch).
  pdl_wait();
  pdl_trigger();
  if (warp == 1) tmem_alloc(tmem_holder, S::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int m_valid = *p.m_valid;
  const int m_tiles = (m_valid + S::kBlockM - 1) / S::kBlockM;
  const int num_tiles = m_tiles * n_tiles;

  if (warp == 0) {
    if (lane == 0 && num_tiles > 0) {
      tma_prefetch_desc(&map_a);
      tma_prefetch_desc(&map_w);
      tma_prefetch_desc(&map_o);
      if (EPI == kEpiResidLn || EPI == kEpiResidLn16) tma_prefetch_desc(&map_l);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t a_policy = l2_evict_first();
      if (WS) {  // this CTA's slice of W, once (gridDim.x is a multiple of n_tiles)
        const int n0 = (static_cast<int>(blockIdx.x) % n_tiles) * BLOCK_N;
        mbar_arrive_expect_tx(w_full, p.k_blocks * S::kBTileBytes);
        for (int kb = 0; kb < p.k_blocks; ++kb)
          tma_load_2d(sb + kb * S::kBTileBytes, &map_w, w_full, kb * (FP8 ? 128 : 64), n0);
      }
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
          if (p.a_stream)
            tma_load_2d_hint(sa + stage * S::kATileBytes, &map_a, &full[stage], kx, m0, a_policy);
          else
            tma_load_2d(sa + stage * S::kATileBytes, &map_a, &full[stage], kx, m0);
#pragma unroll
          for (int c = 0; c < S::kBoxCount && !WS; ++c)
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
      bool ok = !WS || mbar_wait(w_full, 0, abort_flag, p.err);
      // Descriptors of stage 0 / k-step 0, built once: a stage or k-step
      // offset is an add to the start-address field (address >> 4, below 2^14
      // for any shared-memory address, so the field never carries).
      const uint64_t a_desc0 = sdesc_k_sw128(smem_u32(sa));
      const uint64_t b_desc0 = sdesc_k_sw128(smem_u32(sb));
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
          const uint64_t a_desc = a_desc0 + static_cast<uint64_t>((stage * S::kATileBytes) >> 4);
          const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(((WS ? kb : stage) * S::kBTileBytes) >> 4);
          const uint32_t acc_first = kb > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 4 x 32 bytes of K per 128-byte row
#pragma unroll
            for (int c = 0; c < S::kInstCount; ++c) {
              const uint64_t adesc = a_desc + static_cast<uint64_t>(k * 2);
              const uint64_t bdesc = b_desc + static_cast<uint64_t>((c * S::kInstN * S::kRowBytes + k * 32) >> 4);
              const uint32_t accumulate = k > 0 ? 1u : acc_first;
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
    // Epilogue warps 2 .. 2+kEpiWarps-1. Thread `lane` owns tile row
    // quad*32 + lane on the TMEM side; global traffic is TMA through the
    // warp's staging tiles.
    const int ew = warp - 2;
    const int quad = warp & 3;
    uint8_t* tiles = s_xpose + ew * S::kTilesPerWarp * S::kTileBytes;
    constexpr int kCols = EPI == kEpiResidLn ? BLOCK_N : BLOCK_N * 4 / kEpiWarps;  // columns this warp drains
    const int col0 = EPI == kEpiResidLn ? 0 : (ew / 4) * kCols;  // warps ew, ew+4, ... share a lane quadrant
    uint64_t* my_xbar = xbar + S::kTilesPerWarp * ew;
    uint32_t xbits = 0u;  // residual-load barrier parities, bit b = staging tile b
    uint32_t pair_phase = 0u;
    int stat_par = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int out_k = 0;  // output tiles used so far (alternates the double buffer)
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (EPI == kEpiResidLn) {
        // issue this tile's first residual chunks now: they land while the MMAs run
        const int rb = (tile / n_tiles) * S::kBlockM + quad * 32;
        if (lane == 0 && rb < m_valid) {
          bulk_wait_read<0>();  // staging tiles free: earlier stores have read them
#pragma unroll
          for (int b = 0; b < S::kTilesPerWarp; ++b) {
            mbar_arrive_expect_tx(&my_xbar[b], 4096);
            tma_load_2d_hint(tiles + b * 4096, &map_o, &my_xbar[b], (ew >> 2) * (BLOCK_N / 2) + b * 32, rb,
                             l2_evict_last());
          }
        }
        __syncwarp();
      } else if (EPI == kEpiResidLn16) {
        // this warp's 32 rows x 64 columns of the bf16 residual, landing while the MMAs run
        const int rb = (tile / n_tiles) * S::kBlockM + quad * 32;
        if (lane == 0 && rb < m_valid) {
          bulk_wait_read<0>();  // the staging tile is free: the previous tile's stores have read it
          mbar_arrive_expect_tx(&my_xbar[0], 4096);
          tma_load_2d_hint(tiles, &map_o, &my_xbar[0], (ew >> 2) * 64, rb, l2_evict_last());
        }
        __syncwarp();
      }
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err)) break;
      tc_fence_after();
      const int row_base = (tile / n_tiles) * S::kBlockM + quad * 32;  // first row of this warp's 32
      const int m = row_base + lane;
      const bool any = row_base < m_valid;
      const int n0 = (tile % n_tiles) * BLOCK_N;
      const bool live = m < m_valid;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BLOCK_N);
      const float a_s = (FP8 && live) ? p.a_scale[m] : 1.0f;

      if (EPI == kEpiBias || EPI == kEpiBiasGelu) {
        constexpr int CW = EpiWarps<EPI>::kChunkCols;
        static_assert(kCols % CW == 0, "whole epilogue chunks");
#pragma unroll 1
        for (int c = col0; c < col0 + kCols && any; c += CW) {
          uint32_t r[CW];
#pragma unroll
          for (int h = 0; h < CW / 32; ++h) tmem_ld32(tbase + c + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * h]));
          if (lane == 0) bulk_wait_read<S::kTilesPerWarp - 1>();  // the store that last used this tile has read it
          tmem_ld_wait();
          uint32_t packed[CW / 2];
#pragma unroll
          for (int i = 0; i < CW; i += 4) {
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
              v0 = gelu_bf16(v0);
              v1 = gelu_bf16(v1);
              v2 = gelu_bf16(v2);
              v3 = gelu_bf16(v3);
            }
            packed[i / 2] = pack_bf16x2(v0, v1);
            packed[i / 2 + 1] = pack_bf16x2(v2, v3);
          }
          uint8_t* ot = tiles + (out_k % S::kTilesPerWarp) * S::kTileBytes;
          __syncwarp();
#pragma unroll
          for (int q = 0; q < CW / 8; ++q) {
            const uint4 v = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
            if (CW == 64)
              *xpose_slot(ot, lane, q) = v;
            else
              *xpose_slot64(ot, lane, q) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (EPI == kEpiBiasGelu)
              tma_store_2d_hint(&map_o, ot, n0 + c, row_base, l2_evict_first());
            else
              tma_store_2d(&map_o, ot, n0 + c, row_base);
            bulk_commit();
          }
          ++out_k;
        }
      } else if (EPI == kEpiResidLn16) {
        if (any) {
          float2* st16 = reinterpret_cast<float2*>(s_stats);
          float* amax16 = reinterpret_cast<float*>(st16 + 2 * 16 * 32);
          resid_ln16_epilogue<FP8>(tbase, tiles, &my_xbar[0], xbits, st16 + stat_par * 16 * 32,
                                   amax16 + stat_par * 16 * 32, s_bias, s_bscale, s_g, s_b, &map_o, &map_l, p,
                                   abort_flag, &pair_bar[quad], pair_phase, ew, lane, row_base, m, live, a_s);
          stat_par ^= 1;
        }
      } else if (any) {
        resid_ln_epilogue<BLOCK_N, FP8, S::kTilesPerWarp>(tbase, tiles, my_xbar, xbits, s_stats + (stat_par * 8) * 32,
                                                          s_bias, s_bscale, s_g, s_b, &map_o, &map_l, p, abort_flag,
                                                          &pair_bar[quad], pair_phase, ew, quad, lane, row_base, m,
                                                          live, a_s);
        stat_par ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == S::kAcc) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();  // every TMA store of this warp has completed
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace ow
