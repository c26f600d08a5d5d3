// Masked multi-head attention on the 5th-generation tensor cores (tcgen05),
// head_dim 32, bf16 operands, f32 accumulation, over the packed token layout
// (state b owns rows offsets[b] .. offsets[b+1]-1; a row attends to the rows
// of its own state, which is the key-padding mask of the padded layout).
//
// Tiles of states. With BS = the block size (32, 64 or 128 rows, the smallest
// power of two >= N), a 128-row tile holds k = 128 / BS consecutive states,
// state j of the tile in block j (query and key positions j*BS .. j*BS+BS-1),
// each loaded by TMA from its own packed rows. A work unit is a tile and two
// heads; its Q, K and V arrive as one 128-byte (two-head) box per state and
// matrix, in the 128-byte swizzle, and each head's MMAs address its 64-byte
// half of the rows. Per head, with the tile's states sharing TMEM columns
// (each MMA writes only its state's lanes: the disable-output-lane mask):
//   S = Q K^T        per state j: tcgen05.mma, M = 128, N = BS, K = 32, into
//                    the warpgroup's score region (BS columns) at lanes
//                    j*BS .. j*BS+BS-1;
//   P = softmax(S)   one thread per query row reads its state's keys (at
//                    most BS / 32 chunks of 32 columns) from TMEM and writes P
//                    as bf16 into the same TMEM columns (two values per 32-bit
//                    column), 0 past the state's count;
//   O = P V          per state j: tcgen05.mma with A = P straight from TMEM
//                    and B = the state's V rows from shared memory
//                    (MN-major), into one of the warpgroup's two 32-column
//                    O buffers;
//   out = O / rowsum bf16, written by the same threads.
// A warpgroup thus holds a 64-column score region and two O buffers (at
// BS = 128 a 128-column region with O in its columns 64 .. 95). Every warp's 32 rows lie in one state, so the key range (and
// the mask of the last partial chunk) is the same for all its lanes. Key
// positions past a state's count hold whatever the stage held before (finite:
// stages start zeroed and TMA only brings finite rows), so their P of exactly
// 0 keeps O = P V exact.
//
// Roles: warp 0 issues the TMA loads; four warpgroups of four warps run the
// softmax and output, warpgroup w taking head w % 2 of every other unit; MMA warp g issues head g's products for the warpgroups of that
// head, polling each one's barriers and issuing whichever QK^T or PV is ready.
// A head takes twelve tcgen05.mma (QK^T: 2 per state, PV: BS / 16 per state),
// each of M = 128 and K = 16, issued every ~50 cycles at N = 64 from one
// thread with its descriptors precomputed, so the two issuers run in parallel
// and off the softmax path. A warpgroup's next scores go into its score region
// right behind the PV product that reads its P, so they are computed while the
// warpgroup writes the previous head's output.
#pragma once

#include "ow_common.cuh"

namespace ow {

struct TcAttnParams {
  const int* offsets;  // [batch + 1] packed row offsets
  __nv_bfloat16* out;  // [rows, d] attention output
  int* err;
  int batch;
  int d;      // heads * 32
  int heads;  // even
  float scale_log2;  // log2(e) / sqrt(32)
};

template <int BS>
struct TcAttnShape {
  static constexpr int kBS = BS;
  static constexpr int kStatesPerTile = 128 / BS;
  static constexpr int kChunks = BS / 32;           // key chunks of a block
  static constexpr int kGroup = 2;                  // heads per work unit
  static constexpr int kSCols = BS == 128 ? 128 : 64;  // TMEM columns of a score region (P over its first BS / 2)
  // softmax warpgroups: four (two TMEM buffers each) up to BS = 64; two at
  // BS = 128, where a head holds 128 columns and only four fit
  static constexpr int kWgs = 4;
  static constexpr int kWgPerHead = kWgs / kGroup;  // warpgroups taking alternate units' head h
  // a warpgroup's TMEM: one score region and two 32-column O buffers; at
  // BS = 128 (four 128-column regions fill TMEM) O goes into the region's
  // columns 64 .. 95, free once P (columns 0 .. 63) is written
  static constexpr bool kInRegionO = BS == 128;
  static constexpr int kWgCols = kInRegionO ? kSCols : kSCols + 64;
  static constexpr int kBoxBytes = BS * 128;       // one state's rows of one matrix, both heads (128 B per row)
  static constexpr int kTileBytes = 128 * 128;      // Q, K or V of a unit
  static constexpr int kStageBytes = 3 * kTileBytes;  // one unit
  static constexpr int kStages = 4;
  static constexpr int kThreads = 96 + 128 * kWgs;
  static constexpr int kBarrierBytes = 512;
  static constexpr int kOutBytes = 4 * kWgs * 32 * 64;  // per softmax warp: 32 rows x 64 B of output
  static constexpr int kTmemCols = 512;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kOutBytes + kBarrierBytes;
  // Registers per thread: an SM sub-partition holds every fourth warp (five of
  // nineteen, three of eleven) in its 16,384 registers.
  static constexpr int kMaxRegs = 96;
  static_assert(kStageBytes % 1024 == 0, "1024 B aligned stages");
  static_assert(kSmemBytes <= 232448, "227 KB of shared memory per CTA");
  static_assert(kWgs * kWgCols <= kTmemCols, "TMEM columns");
  static_assert(8 * (2 * kStages + 6 * kWgs) + 8 <= kBarrierBytes, "barrier area");
};

// MN-major operand in the 128-byte swizzle (V: rows = keys = K, 64 contiguous
// bf16 of two heads per 128 B row; a head's N = 32 starts at its 64-byte
// half): 8 key rows per 1024 B atom (SBO), LBO (the stride between 64-element
// column groups) never used, descriptor version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// D(tmem) (+)= A(tmem) * B(smem desc), bf16 inputs, f32 accumulate; A is
// K-major in TMEM (row = lane, two bf16 per 32-bit column).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same two forms with the disable-output-lane mask: bit i of word q set
// leaves TMEM lane 32 q + i of D unwritten.
__device__ __forceinline__ void umma_f16_lanes(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate, const uint32_t (&m)[4]) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(m[0]), "r"(m[1]), "r"(m[2]), "r"(m[3])
      : "memory");
}
__device__ __forceinline__ void umma_f16_ts_lanes(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t accumulate, const uint32_t (&m)[4]) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(m[0]), "r"(m[1]), "r"(m[2]), "r"(m[3])
      : "memory");
}
// Lanes of tile state j (rows j*BS .. j*BS+BS-1, BS >= 32) enabled, the rest disabled.
template <int BS>
__device__ __forceinline__ void state_lanes(int j, uint32_t (&m)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) m[q] = (32 * q >= j * BS && 32 * q < (j + 1) * BS) ? 0u : 0xFFFFFFFFu;
}

// 32 lanes x 16 columns of 32-bit TMEM <- 16 registers per thread.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}

// Non-blocking test of phase `parity` of `bar` (the MMA warps poll two barriers).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// One 32-key chunk of a row: e = 2^(s*scale + off) (off = -max*scale) for the
// first `valid` keys (all 32 when FULL) and 0 for the rest, summed in f32 and
// stored to TMEM as 16 bf16 pairs at p_addr.
template <bool FULL>
__device__ __forceinline__ void attn_exp_chunk(const uint32_t (&r)[32], int valid, float2 sc, float2 off,
                                               float2& sum2, uint32_t p_addr) {
  uint32_t pk[16];
  float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float2 v = fma_f2(make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), sc, off);
    float2 e = make_float2(ex2_approx_f(v.x), ex2_approx_f(v.y));
    if (!FULL) e = make_float2(2 * j < valid ? e.x : 0.0f, 2 * j + 1 < valid ? e.y : 0.0f);
    acc[j & 1] = add_f2(acc[j & 1], e);
    pk[j] = pack_bf16x2(e.x, e.y);
  }
  tmem_st16(p_addr, pk);
  sum2 = add_f2(sum2, add_f2(acc[0], acc[1]));
}
template <bool FULL>
__device__ __forceinline__ float attn_chunk_max(const uint32_t (&r)[32], int valid, float mx) {
  float m4[4] = {mx, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float a = FULL || j + 2 * h < valid ? __uint_as_float(r[j + 2 * h]) : -INFINITY;
      const float b = FULL || j + 2 * h + 1 < valid ? __uint_as_float(r[j + 2 * h + 1]) : -INFINITY;
      m4[h] = fmax3(m4[h], a, b);
    }
  }
  return fmax3(fmaxf(m4[0], m4[1]), m4[2], m4[3]);
}
// Chunk helpers on a runtime count of valid keys.
__device__ __forceinline__ float attn_max_any(const uint32_t (&r)[32], int valid, float mx) {
  return valid >= 32 ? attn_chunk_max<true>(r, 32, mx) : attn_chunk_max<false>(r, valid, mx);
}
__device__ __forceinline__ void attn_exp_any(const uint32_t (&r)[32], int valid, float2 sc, float2 off, float2& sum2,
                                             uint32_t p_addr) {
  if (valid >= 32) attn_exp_chunk<true>(r, 32, sc, off, sum2, p_addr);
  else attn_exp_chunk<false>(r, valid, sc, off, sum2, p_addr);
}

// Softmax of one warp's rows over their state's c keys, whose scores start at
// TMEM column tb + 32 * c0: writes P over the buffer's CHUNKS * 16 P columns
// (0 past the state's keys) and returns the pairwise f32 row sum.
template <int CHUNKS>
__device__ __forceinline__ float2 attn_softmax_rows(uint32_t tb, int c0, int c, float2 sc, float scale_log2) {
  const int nch = (c + 31) >> 5;
  float2 sum2 = make_float2(0.0f, 0.0f);
  if constexpr (CHUNKS <= 2) {
    // one TMEM round trip: both chunks in registers for the max and the
    // exponentials (the four-warpgroup kernel's 96 registers hold them; the
    // wider-state path below is compiled only for BS = 128)
    uint32_t r0[32], r1[32];
    tmem_ld32(tb + 32 * c0, r0);
    if (CHUNKS == 2 && nch == 2) tmem_ld32(tb + 32 * (c0 + 1), r1);
    tmem_ld_wait_dep(r0);
    if (CHUNKS == 2 && nch == 2) tmem_ld_wait_dep(r1);
    float mx = attn_max_any(r0, c, -INFINITY);
    if (CHUNKS == 2 && nch == 2) mx = attn_max_any(r1, c - 32, mx);
    const float2 off = make_float2(-mx * scale_log2, -mx * scale_log2);
    attn_exp_any(r0, c, sc, off, sum2, tb + 16 * c0);
    // P of chunk 0 goes to S chunk 0's columns, already read
    if (CHUNKS == 2 && nch == 2) attn_exp_any(r1, c - 32, sc, off, sum2, tb + 16 * (c0 + 1));
  } else {
    // wide states (BS = 128, 96 registers): the max with the next chunk's
    // load in flight, then each chunk read again for its exponentials (P
    // column 16 (c0 + k) lies in S chunk (c0 + k) / 2 <= c0 + k, already read)
    uint32_t ra[32], rb[32];
    float mx = -INFINITY;
    tmem_ld32(tb + 32 * c0, ra);
    for (int k = 0; k < nch; k += 2) {
      tmem_ld_wait_dep(ra);
      if (k + 1 < nch) tmem_ld32(tb + 32 * (c0 + k + 1), rb);
      mx = attn_max_any(ra, c - 32 * k, mx);
      if (k + 1 < nch) {
        tmem_ld_wait_dep(rb);
        if (k + 2 < nch) tmem_ld32(tb + 32 * (c0 + k + 2), ra);
        mx = attn_max_any(rb, c - 32 * (k + 1), mx);
      }
    }
    const float2 off = make_float2(-mx * scale_log2, -mx * scale_log2);
    for (int k = 0; k < nch; ++k) {
      tmem_ld32(tb + 32 * (c0 + k), ra);
      tmem_ld_wait_dep(ra);
      attn_exp_any(ra, c - 32 * k, sc, off, sum2, tb + 16 * (c0 + k));
    }
  }
  // P = 0 for the key chunks past the state's count (after the reads above)
  uint32_t z[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) z[j] = 0u;
#pragma unroll
  for (int k = 0; k < CHUNKS; ++k)
    if (k < c0 || k >= c0 + nch) tmem_st16(tb + 16 * k, z);
  return sum2;
}

template <int BS>
__global__ void __launch_bounds__(TcAttnShape<BS>::kThreads) __maxnreg__(TcAttnShape<BS>::kMaxRegs)
    tc_attention_kernel(const __grid_constant__ CUtensorMap map_qkv, const TcAttnParams p) {
  using S = TcAttnShape<BS>;
  constexpr int K = S::kStatesPerTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* out_stage = smem + S::kStages * S::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(out_stage + S::kOutBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* s_full = empty + S::kStages;    // [kWgs] scores of the warpgroup's head in its region
  uint64_t* p_full = s_full + S::kWgs;      // [kWgs] P written (the region's scores read)
  uint64_t* o_full = p_full + S::kWgs;      // [kWgs][2] O buffer written
  uint64_t* t_empty = o_full + 2 * S::kWgs; // [kWgs][2] O buffer read
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(t_empty + 2 * S::kWgs);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);  // both MMA warps' PV products have read the stage
    }
    for (int w = 0; w < S::kWgs; ++w) {
      mbar_init(&s_full[w], 1);
      mbar_init(&p_full[w], 4);
    }
    for (int b = 0; b < 2 * S::kWgs; ++b) {
      mbar_init(&o_full[b], 1);
      mbar_init(&t_empty[b], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // stages start zeroed: key positions a state does not fill stay finite
  for (int i = threadIdx.x; i < S::kStages * S::kStageBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(stages)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (warp == 0) tmem_alloc(tmem_holder, S::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // q, k, v and the offsets come from earlier kernels
  pdl_wait();
  pdl_trigger();
  const int hgs = p.heads / S::kGroup;
  const int n_tiles = (p.batch + K - 1) / K;
  const int n_units = n_tiles * hgs;
  const int my_units = n_units > static_cast<int>(blockIdx.x)
                           ? (n_units - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                 static_cast<int>(gridDim.x)
                           : 0;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA loads
    if (lane == 0 && my_units > 0) {
      tma_prefetch_desc(&map_qkv);
      // offsets of the states of the next two units (loaded ahead: the loads are L2 round trips)
      int nxt[2][K + 1];
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const int ua = static_cast<int>(blockIdx.x) + a * static_cast<int>(gridDim.x);
        const int s0 = (min(ua, n_units - 1) / hgs) * K;
#pragma unroll
        for (int j = 0; j <= K; ++j) nxt[a][j] = p.offsets[min(s0 + j, p.batch)];
      }
      int ui = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++ui) {
        const int col = (u % hgs) * S::kGroup * 32;
        int off[K + 1];
#pragma unroll
        for (int j = 0; j <= K; ++j) off[j] = nxt[ui & 1][j];
        {
          const int ua = u + 2 * static_cast<int>(gridDim.x);
          const int s0 = (min(ua, n_units - 1) / hgs) * K;
#pragma unroll
          for (int j = 0; j <= K; ++j) nxt[ui & 1][j] = p.offsets[min(s0 + j, p.batch)];
        }
        int live = 0;
#pragma unroll
        for (int j = 0; j < K; ++j) live += off[j + 1] > off[j] ? 1 : 0;
        const int s = ui % S::kStages;
        if (!mbar_wait(&empty[s], ((ui / S::kStages) & 1u) ^ 1u, abort_flag, p.err)) break;
        uint8_t* sq = stages + s * S::kStageBytes;
        mbar_arrive_expect_tx(&full[s], 3 * live * S::kBoxBytes);
#pragma unroll
        for (int j = 0; j < K; ++j) {
          if (off[j + 1] > off[j]) {
            uint8_t* dst = sq + j * S::kBoxBytes;
            tma_load_2d(dst, &map_qkv, &full[s], col, off[j]);
            tma_load_2d(dst + S::kTileBytes, &map_qkv, &full[s], p.d + col, off[j]);
            tma_load_2d(dst + 2 * S::kTileBytes, &map_qkv, &full[s], 2 * p.d + col, off[j]);
          }
        }
      }
    }
  } else if (warp <= 2) {
    // ---------------------------------------------------------------- MMA issue
    // MMA warp g issues head g of every unit. The CTA's unit i goes to
    // warpgroup w = g + 2 (i % kWgPerHead) as that warpgroup's k-th head,
    // k = i / kWgPerHead: stage i % kStages, the 64-byte half g of its rows.
    // PV(k) reads P from the warpgroup's score region and accumulates into its
    // O buffer k % 2 (free once the output of head k - 2 is read); QK(k + 1)
    // then goes straight into the same score region. tcgen05.mma operations
    // of one thread run in issue order, so it overwrites P only after PV(k)
    // has read it, and it runs while the warpgroup writes head k - 1's output.
    // The thread keeps one QK / PV position per warpgroup it serves, polls them
    // all and issues whatever is ready, so a slow warpgroup does not hold up
    // the other (a sleeping wait wakes too late here).
    if (lane == 0) {
      const int g = warp - 1;
      constexpr int H = S::kWgPerHead;
      constexpr uint32_t kIdescS = idesc_bf16(128, BS);
      constexpr uint32_t kIdescPV = idesc_bf16(128, 32) | (1u << 16);  // B (V) MN-major
      int nq[H], np[H], cnt[H];  // per served warpgroup: next QK / PV head, heads in all
#pragma unroll
      for (int h = 0; h < H; ++h) {
        nq[h] = 0;
        np[h] = 0;
        cnt[h] = my_units > h ? (my_units - h + H - 1) / H : 0;
      }
      // Descriptors of stage 0, built once: a stage, state or k-step offset is
      // an add to the start-address field (address >> 4, below 2^14 for any
      // shared-memory address, so the field never carries into the next one).
      const uint64_t q_desc0 = sdesc_k_sw128(smem_u32(stages) + g * 64);
      const uint64_t v_desc0 = sdesc_mn_sw128(smem_u32(stages) + 2 * S::kTileBytes + g * 64);
      unsigned long long t0 = 0;
      uint32_t idle = 0;
      int left = 0;
#pragma unroll
      for (int h = 0; h < H; ++h) left += cnt[h];
      while (left > 0) {
        bool progressed = false;
#pragma unroll
        for (int h = 0; h < H; ++h) {
          const int w = g + 2 * h;
          if (np[h] < nq[h]) {
            const int k = np[h], ob = 2 * w + (k & 1);
            if (mbar_test(&p_full[w], k & 1u) &&
                (S::kInRegionO || k < 2 || mbar_test(&t_empty[ob], ((k >> 1) - 1) & 1u))) {
              tc_fence_after();
              const int s = (h + H * k) % S::kStages;
              const uint32_t ta = tmem_base + static_cast<uint32_t>(w * S::kWgCols);
              const uint32_t to = ta + static_cast<uint32_t>(S::kInRegionO ? 64 : S::kSCols + 32 * (k & 1));
              const uint64_t vd = v_desc0 + static_cast<uint64_t>(s * (S::kStageBytes >> 4));
#pragma unroll
              for (int j = 0; j < K; ++j) {
                uint32_t m[4];
                state_lanes<BS>(j, m);
#pragma unroll
                for (int kk = 0; kk < BS / 16; ++kk)
                  umma_f16_ts_lanes(to, ta + 8 * kk, vd + static_cast<uint64_t>((j * BS + 16 * kk) * 8),
                                    kIdescPV, kk > 0 ? 1u : 0u, m);
              }
              umma_commit(&o_full[ob]);
              umma_commit(&empty[s]);
              ++np[h];
              --left;
              progressed = true;
            }
          }
          // QK(k) once PV(k - 1) is issued: the score region is the warpgroup's only one
          // (O in the region: also once the output of head k - 1 has left it)
          if (nq[h] < cnt[h] && nq[h] == np[h]) {
            const int k = nq[h], i = h + H * k;
            const int s = i % S::kStages;
            if (mbar_test(&full[s], (i / S::kStages) & 1u) &&
                (!S::kInRegionO || k == 0 || mbar_test(&t_empty[2 * w + ((k - 1) & 1)], ((k - 1) >> 1) & 1u))) {
              tc_fence_after();
              const uint32_t dt = tmem_base + static_cast<uint32_t>(w * S::kWgCols);
              const uint64_t qd = q_desc0 + static_cast<uint64_t>(s * (S::kStageBytes >> 4));
              const uint64_t kd = qd + static_cast<uint64_t>(S::kTileBytes >> 4);
#pragma unroll
              for (int j = 0; j < K; ++j) {
                uint32_t m[4];
                state_lanes<BS>(j, m);
                const uint64_t kdj = kd + static_cast<uint64_t>(j * BS * 8);  // key rows of state j
                umma_f16_lanes(dt, qd, kdj, kIdescS, 0u, m);
                umma_f16_lanes(dt, qd + 2u, kdj + 2u, kIdescS, 1u, m);  // + 32 bytes of K
              }
              umma_commit(&s_full[w]);
              ++nq[h];
              progressed = true;
            }
          }
        }
        if (progressed) {
          idle = 0;
        } else if ((++idle & 255u) == 0u) {
          if (*abort_flag) break;
          const unsigned long long now = global_ns();
          if (idle == 256u) {
            t0 = now;
          } else if (now - t0 > kWaitLimitNs) {
            record_error(p.err, kErrWaitTimeout);
            *abort_flag = 1;
            break;
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax + output
    // Warpgroup wg takes head wg % 2 of the CTA's units i with i % kWgPerHead
    // = wg / 2: its k-th head's scores and P in the warpgroup's score region,
    // its O in the warpgroup's O buffer k % 2.
    const int wg = (warp - 3) >> 2;
    const int par = wg >> 1;
    const int ustep = S::kWgPerHead * static_cast<int>(gridDim.x);
    const int quad = warp & 3;                    // TMEM lane quadrant: tile rows quad*32 .. +31
    const int blk = (quad * 32) / BS;             // the tile block (state) of this warp's rows
    const int rib = quad * 32 - blk * BS + lane;  // this thread's row within its block
    const float2 sc = make_float2(p.scale_log2, p.scale_log2);
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    bool ok = true;
    int prev_r = 0, prev_c = 0, prev_col = 0;  // the head whose output is pending
    float2 prev_sum = make_float2(0.0f, 0.0f);
    int nxt_r = 0, nxt_c = 0;  // this warp's state (first row, count) in the next unit
    if (my_units > par) {
      const int st = ((static_cast<int>(blockIdx.x) + par * static_cast<int>(gridDim.x)) / hgs) * K + blk;
      nxt_r = p.offsets[min(st, p.batch)];
      nxt_c = p.offsets[min(st + 1, p.batch)] - nxt_r;
    }
    // The output of head k: O / rowsum as bf16. Each thread puts its row's
    // 64 bytes into the warp's staging tile (16-byte chunks rotated by the row,
    // so a quarter-warp's stores hit distinct banks), then the warp writes 8
    // rows x 64 contiguous bytes per store instruction.
    uint8_t* ostage = out_stage + (warp - 3) * 32 * 64;
    auto output = [&](int k) -> bool {
      const int b = 2 * wg + (k & 1);
      if (!mbar_wait(&o_full[b], (k >> 1) & 1u, abort_flag, p.err)) return false;
      tc_fence_after();
      const int first = rib - lane;  // the warp's first row within its block
      if (first < prev_c) {          // the warp has rows of its state
        uint32_t r[32];
        tmem_ld32(tmem_base + lane_off +
                      static_cast<uint32_t>(wg * S::kWgCols + (S::kInRegionO ? 64 : S::kSCols + 32 * (k & 1))),
                  r);
        tmem_ld_wait_dep(r);
        const float inv = 1.0f / (prev_sum.x + prev_sum.y);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(ostage + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(pack_bf16x2(__uint_as_float(r[8 * q]) * inv, __uint_as_float(r[8 * q + 1]) * inv),
                         pack_bf16x2(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv),
                         pack_bf16x2(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv),
                         pack_bf16x2(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv));
        __syncwarp();
        const int cq = lane & 3;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = (lane >> 2) + 8 * i;  // staged row
          if (first + rr < prev_c) {
            const uint4 v = *reinterpret_cast<const uint4*>(ostage + rr * 64 + ((cq ^ ((rr >> 1) & 3)) << 4));
            *reinterpret_cast<uint4*>(p.out + static_cast<size_t>(prev_r + first + rr) * p.d + prev_col + cq * 8) = v;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[b]);
      return true;
    };
    // Iteration k: softmax(k), then the output of head k - 1 (whose PV ran
    // during this softmax), or at BS = 128 (O in the score region) the output
    // of head k itself, after which the region takes QK(k + 1).
    int k = 0;
    for (int u = blockIdx.x + par * static_cast<int>(gridDim.x); u < n_units; u += ustep, ++k) {
      const int col = ((u % hgs) * S::kGroup + (wg & 1)) * 32;
      const int r0 = nxt_r, c = nxt_c;
      if (u + ustep < n_units) {
        const int st = ((u + ustep) / hgs) * K + blk;
        nxt_r = p.offsets[min(st, p.batch)];
        nxt_c = p.offsets[min(st + 1, p.batch)] - nxt_r;
      }
      if (!mbar_wait(&s_full[wg], k & 1u, abort_flag, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float2 sum2 = make_float2(0.0f, 0.0f);
      if (rib - lane < c) {  // the warp has rows of its state
        sum2 = attn_softmax_rows<S::kChunks>(tmem_base + lane_off + static_cast<uint32_t>(wg * S::kWgCols), 0, c,
                                             sc, p.scale_log2);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[wg]);
      if constexpr (S::kInRegionO) {
        // O shares the score region: write this head's output now, which
        // frees the region for the next head's scores
        prev_r = r0;
        prev_c = c;
        prev_col = col;
        prev_sum = sum2;
        if (!output(k)) {
          ok = false;
          break;
        }
      } else {
        if (k > 0 && !output(k - 1)) {
          ok = false;
          break;
        }
        prev_r = r0;
        prev_c = c;
        prev_col = col;
        prev_sum = sum2;
      }
    }
    if (!S::kInRegionO && ok && k > 0) output(k - 1);
  }

  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace ow
