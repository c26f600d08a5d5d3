// Fused feed-forward block of the bf16 encoder, one persistent kernel:
//
//   x  += GELU(ln . W1^T + b1) . W2^T + b2      (f32 residual stream, in place)
//   ln' = LayerNorm(x)                           (the next block's LN1, or the final LN)
//
// per 128-row tile, without the f-wide hidden activations ever leaving the SM.
// For d = 256 the hidden layer is walked in chunks of 128 columns:
//
//   TMEM (512 columns): out accumulator [0, d), two hidden accumulators
//                       [d, d+128) and [d+128, d+256)
//   shared memory:      the tile's LN rows (A of the up-projection, 64 KB,
//                       loaded once per tile), two bf16 hidden-chunk buffers
//                       (A of the down-projection, 2 x 32 KB, 128 B swizzle),
//                       a ring of 16 KB weight boxes (128 rows x 64 bf16) that
//                       carries W1 and W2 in the order the MMAs consume them
//
//   chunk j:  H_j  = A . W1[j]^T            -> hidden accumulator j % 2
//             h_j  = bf16(GELU(H_j + b1))   -> hidden buffer j % 2 (epilogue warps)
//             O   += h_j . W2[:, j]^T       -> out accumulator
//
// The MMA warp issues the up-projection of chunk j+2 as soon as the epilogue
// has drained hidden accumulator j, ahead of the down-projection of chunk j,
// so the epilogue's GELU of one chunk overlaps the tensor cores' work. After the last chunk the same warps run the
// residual + LayerNorm epilogue on the out accumulator; its TMA staging tiles
// alias the hidden buffers (free once the last down-projection has retired),
// and the up-projections of the next tile already run meanwhile.
//
// Roles: warp 0 lane 0 issues TMA, warp 1 lane 0 issues tcgen05.mma and owns
// the TMEM allocation, warps 2..17 are the epilogue (warp w reads TMEM lanes
// 32*(w%4)..+31): for GELU the four warps of a lane quadrant take 32 of each
// chunk's 128 columns; the LayerNorm runs on the first eight, two per lane
// quadrant, half a row each. Every wait is an mbarrier wait bounded in time.
#pragma once

#include "ow_tc_gemm.cuh"

namespace ow {

template <int D>
struct TcFfnShape {
  static constexpr int kBlockM = 128;
  static constexpr int kChunk = 128;             // hidden columns per chunk
  static constexpr int kTile = 128 * 128;        // one 128-row x 128 B swizzled tile
  static constexpr int kDk = D / 64;             // K blocks of the up-projection
  static constexpr int kHk = kChunk / 64;        // K blocks of one chunk's down-projection
  static constexpr int kNh = D / 128;            // 128-row W2 boxes per K block
  static constexpr int kABytes = kDk * kTile;
  static constexpr int kHBytes = 2 * kHk * kTile;
  static constexpr int kEpiWarps = 16;            // GELU: 4 warps per TMEM lane quadrant, 32 columns each
  static constexpr int kLnWarps = 8;              // LayerNorm: the first 8 of them, half a row each
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kStageBytes = kTile;      // one weight box
  static constexpr int kBarrierBytes = 512;
  static constexpr int kParamFloats = 2048;      // b1[f], b2[d], gamma[d], beta[d]
  static constexpr int kStatsBytes = 2 * 8 * 32 * 16;
  static constexpr int kFixedBytes = kABytes + kHBytes + kBarrierBytes + kParamFloats * 4 + kStatsBytes + 1024;
  static constexpr int kStagesFit = (kSmemLimit - kFixedBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kSmemBytes = kFixedBytes + kStages * kStageBytes;
  static constexpr int kTmemCols = 512;
  static_assert(D == 256, "out accumulator + two 128-column hidden accumulators fill the 512 TMEM columns");
  static_assert(kHBytes == kLnWarps * 2 * 4096, "LayerNorm staging (2 x 4 KB per LayerNorm warp) aliases the hidden buffers");
  static_assert(kStages >= 4, "weight ring depth");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory per CTA");
};

// p.n = f (hidden width, multiple of 128, f + 3d <= kParamFloats), p.bias = b1,
// p.bias2 = b2, p.ln_g/ln_b/ln_mode as the LayerNorm epilogue (bf16 or f32 out).
template <int D>
__global__ void __launch_bounds__(TcFfnShape<D>::kThreads, 1)
    tc_ffn_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w1,
                  const __grid_constant__ CUtensorMap map_w2, const __grid_constant__ CUtensorMap map_x,
                  const __grid_constant__ CUtensorMap map_l, const TcGemmParams p) {
  using S = TcFfnShape<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sH = sA + S::kABytes;
  uint8_t* sW = sH + S::kHBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sW + S::kStages * S::kStageBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* a_full = empty + S::kStages;
  uint64_t* a_empty = a_full + 1;
  uint64_t* h_full = a_empty + 1;    // [2] hidden accumulator ready
  uint64_t* h_empty = h_full + 2;    // [2] hidden accumulator drained (every epilogue warp)
  uint64_t* hs_full = h_empty + 2;   // [2] hidden buffer written (every epilogue warp)
  uint64_t* hs_empty = hs_full + 2;  // [2] hidden buffer read by the down-projection
  uint64_t* o_full = hs_empty + 2;
  uint64_t* o_empty = o_full + 1;    // out accumulator drained (every epilogue warp)
  uint64_t* stg_free = o_empty + 1;  // LayerNorm stores have read the staging tiles (every epilogue thread)
  uint64_t* xbar = stg_free + 1;     // [LayerNorm warps x 2] residual loads
  uint64_t* pair_bar = xbar + 2 * S::kLnWarps;  // [4] LayerNorm pair rendezvous
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(pair_bar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_b1 = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + S::kBarrierBytes);
  float* s_b2 = s_b1 + p.n;
  float* s_g = s_b2 + D;
  float* s_be = s_g + D;
  float4* s_stats = reinterpret_cast<float4*>(s_b1 + S::kParamFloats);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_chunks = p.n / S::kChunk;
  // Each CTA walks the hidden chunks from its own starting chunk, so the CTAs
  // do not all stream the same weight boxes from the same L2 lines at once.
  const int rot = static_cast<int>(blockIdx.x % static_cast<unsigned>(n_chunks));
  auto chunk_id = [&](int j) { return (j + rot) % n_chunks; };
  constexpr uint32_t kIdesc = idesc_bf16(128, 128);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&h_full[b], 1);
      mbar_init(&h_empty[b], S::kEpiWarps);
      mbar_init(&hs_full[b], S::kEpiWarps);
      mbar_init(&hs_empty[b], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, S::kEpiWarps);
    mbar_init(stg_free, 32 * S::kEpiWarps);
    for (int i = 0; i < 2 * S::kLnWarps; ++i) mbar_init(&xbar[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) s_b1[i] = p.bias[i];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    s_b2[i] = p.bias2[i];
    s_g[i] = p.ln_g[i];
    s_be[i] = p.ln_b[i];
  }
  // weights only above; rows, residual and token count come from earlier kernels
  pdl_wait();
  pdl_trigger();
  if (warp == 1) tmem_alloc(tmem_holder, S::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int m_valid = *p.m_valid;
  const int m_tiles = (m_valid + S::kBlockM - 1) / S::kBlockM;

  if (warp == 0) {
    if (lane == 0 && m_tiles > blockIdx.x) {
      tma_prefetch_desc(&map_a);
      tma_prefetch_desc(&map_w1);
      tma_prefetch_desc(&map_w2);
      tma_prefetch_desc(&map_x);
      tma_prefetch_desc(&map_l);
      int stage = 0;
      uint32_t phase = 0, a_phase = 0;
      bool ok = true;
      // one weight box into the ring, in MMA consumption order
      auto push = [&](const CUtensorMap* map, int x, int y) {
        if (!ok || !mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
          ok = false;
          return;
        }
        mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
        tma_load_2d(sW + stage * S::kStageBytes, map, &full[stage], x, y);
        if (++stage == S::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int tile = blockIdx.x; tile < m_tiles && ok; tile += gridDim.x) {
        // the previous tile's up-projections have read the A rows
        if (!mbar_wait(a_empty, a_phase ^ 1u, abort_flag, p.err)) break;
        a_phase ^= 1u;
        mbar_arrive_expect_tx(a_full, S::kABytes);
#pragma unroll
        for (int kb = 0; kb < S::kDk; ++kb) tma_load_2d(sA + kb * S::kTile, &map_a, a_full, kb * 64, tile * S::kBlockM);
        // consumption order: up 0, up 1, then (up j+2, down j) for each chunk j
        for (int j = 0; j < 2 && j < n_chunks; ++j)
          for (int kb = 0; kb < S::kDk; ++kb) push(&map_w1, kb * 64, chunk_id(j) * S::kChunk);
        for (int j = 0; j < n_chunks && ok; ++j) {
          if (j + 2 < n_chunks)
            for (int kb = 0; kb < S::kDk; ++kb) push(&map_w1, kb * 64, chunk_id(j + 2) * S::kChunk);
          for (int kb = 0; kb < S::kHk; ++kb)
            for (int nh = 0; nh < S::kNh; ++nh) push(&map_w2, chunk_id(j) * S::kChunk + kb * 64, nh * 128);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && m_tiles > blockIdx.x) {
      int stage = 0;
      uint32_t phase = 0, a_phase = 0, o_uses = 0;
      // per-buffer phase parities as bits (bit b = buffer b), kept in registers
      uint32_t h_bits = 0u, hs_bits = 0u;
      bool ok = true;
      // Descriptors of the first weight box, the A tile and the first hidden
      // tile, built once: a box, k-block or k-step offset is an add to the
      // start-address field (address >> 4, below 2^14 for any shared-memory
      // address, so the field never carries into the next one).
      const uint64_t w_desc0 = sdesc_k_sw128(smem_u32(sW));
      const uint64_t a_desc0 = sdesc_k_sw128(smem_u32(sA));
      const uint64_t h_desc0 = sdesc_k_sw128(smem_u32(sH));
      // takes the next weight box of the ring: its descriptor (ok = false once a wait expired)
      auto take = [&]() -> uint64_t {
        if (!ok || !mbar_wait(&full[stage], phase, abort_flag, p.err)) {
          ok = false;
          return 0u;
        }
        tc_fence_after();
        return w_desc0 + static_cast<uint64_t>(stage * (S::kStageBytes >> 4));
      };
      auto release = [&]() {
        umma_commit(&empty[stage]);  // the box is reusable once these MMAs retire
        if (++stage == S::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int tile = blockIdx.x; tile < m_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(a_full, a_phase, abort_flag, p.err)) break;
        a_phase ^= 1u;
        tc_fence_after();
        // up-projection of chunk j into hidden accumulator j % 2
        auto up = [&](int j) {
          const int b = j & 1;
          if (!ok || !mbar_wait(&h_empty[b], ((h_bits >> b) & 1u) ^ 1u, abort_flag, p.err)) {
            ok = false;
            return;
          }
          h_bits ^= 1u << b;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(D + b * S::kChunk);
#pragma unroll
          for (int kb = 0; kb < S::kDk; ++kb) {
            const uint64_t wd = take();
            if (!ok) return;
            const uint64_t ad = a_desc0 + static_cast<uint64_t>(kb * (S::kTile >> 4));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(d_tmem, ad + static_cast<uint64_t>(2 * k), wd + static_cast<uint64_t>(2 * k), kIdesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
            release();
          }
          umma_commit(&h_full[b]);
          if (j == n_chunks - 1) umma_commit(a_empty);  // the tile's A rows are no longer read
        };
        // down-projection of chunk c from hidden buffer c % 2 into the out accumulator
        auto down = [&](int c) {
          const int b = c & 1;
          if (!ok || !mbar_wait(&hs_full[b], (hs_bits >> b) & 1u, abort_flag, p.err)) {
            ok = false;
            return;
          }
          hs_bits ^= 1u << b;
          // chunk 0: the previous tile's LayerNorm has drained the out accumulator
          if (c == 0 && !mbar_wait(o_empty, (o_uses & 1u) ^ 1u, abort_flag, p.err)) {
            ok = false;
            return;
          }
          tc_fence_after();
#pragma unroll
          for (int kb = 0; kb < S::kHk; ++kb) {
            const uint64_t hd = h_desc0 + static_cast<uint64_t>((b * S::kHk + kb) * (S::kTile >> 4));
#pragma unroll
            for (int nh = 0; nh < S::kNh; ++nh) {
              const uint64_t wd = take();
              if (!ok) return;
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f16(tmem_base + static_cast<uint32_t>(nh * 128), hd + static_cast<uint64_t>(2 * k),
                         wd + static_cast<uint64_t>(2 * k), kIdesc, (c > 0 || kb > 0 || k > 0) ? 1u : 0u);
              release();
            }
          }
          umma_commit(&hs_empty[b]);
        };
        // up j+2 is issued as soon as the epilogue has drained hidden accumulator j,
        // before down j waits for the epilogue to finish writing hidden chunk j
        for (int j = 0; j < 2 && j < n_chunks; ++j) up(j);
        for (int j = 0; j < n_chunks && ok; ++j) {
          if (j + 2 < n_chunks) up(j + 2);
          down(j);
        }
        if (!ok) break;
        umma_commit(o_full);
        ++o_uses;
      }
    }
  } else {
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int part = ew >> 2;              // GELU: columns part*32 .. +31 of each hidden chunk
    const int half = part;                 // LayerNorm (ew < 8): half of the row
    const bool ln_warp = ew < S::kLnWarps;
    uint8_t* stg = sH + ew * 8192;  // LayerNorm staging: 2 x 4 KB, inside the hidden buffers
    uint64_t* my_xbar = xbar + 2 * (ln_warp ? ew : 0);
    // mbarrier phase parities as bits (bit b = buffer / staging tile b), kept in registers
    uint32_t xbits = 0u, h_bits = 0u, hs_bits = 0u;
    uint32_t o_ph = 0u, stg_ph = 0u, pair_phase = 0u;
    int stat_par = 0;
    const uint32_t lanes = static_cast<uint32_t>(quad * 32) << 16;
    for (int tile = blockIdx.x; tile < m_tiles; tile += gridDim.x) {
      const int row_base = tile * S::kBlockM + quad * 32;
      const int m = row_base + lane;
      const bool any = row_base < m_valid;
      bool ok = true;
      for (int j = 0; j < n_chunks && ok; ++j) {
        const int b = j & 1;
        if (!mbar_wait(&h_full[b], (h_bits >> b) & 1u, abort_flag, p.err)) ok = false;
        h_bits ^= 1u << b;
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tmem_base + lanes + static_cast<uint32_t>(D + b * S::kChunk + part * 32), r);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_empty[b]);  // the next up-projection into this accumulator may start
        const float* bias = s_b1 + chunk_id(j) * S::kChunk + part * 32;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 bv = *reinterpret_cast<const float4*>(bias + i);
          const float v0 = gelu_bf16(__uint_as_float(r[i]) + bv.x);
          const float v1 = gelu_bf16(__uint_as_float(r[i + 1]) + bv.y);
          const float v2 = gelu_bf16(__uint_as_float(r[i + 2]) + bv.z);
          const float v3 = gelu_bf16(__uint_as_float(r[i + 3]) + bv.w);
          pk[i / 2] = pack_bf16x2(v0, v1);
          pk[i / 2 + 1] = pack_bf16x2(v2, v3);
        }
        // hidden buffer b: the down-projection of chunk j-2 has read it
        if (!mbar_wait(&hs_empty[b], ((hs_bits >> b) & 1u) ^ 1u, abort_flag, p.err)) ok = false;
        hs_bits ^= 1u << b;
        // 32 columns = half of one 128 B row of K block part / 2
        uint8_t* rows = sH + (b * S::kHk + (part >> 1)) * S::kTile + quad * 32 * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *xpose_slot(rows, lane, (part & 1) * 4 + q) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&hs_full[b]);
      }
      if (!mbar_wait(o_full, o_ph, abort_flag, p.err)) ok = false;
      o_ph ^= 1u;
      tc_fence_after();
      if (any && ln_warp) {
        // the hidden buffers are free (every down-projection retired): residual chunks into the staging tiles
        if (lane == 0) {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            mbar_arrive_expect_tx(&my_xbar[b], 4096);
            tma_load_2d(stg + b * 4096, &map_x, &my_xbar[b], half * (D / 2) + b * 32, row_base);
          }
        }
        __syncwarp();
        resid_ln_epilogue<D, false, 2>(tmem_base + lanes, stg, my_xbar, xbits, s_stats + (stat_par * 8) * 32, s_b2,
                                       nullptr, s_g, s_be, &map_x, &map_l, p, abort_flag, &pair_bar[quad], pair_phase,
                                       ew, quad, lane, row_base, m, m < m_valid, 1.0f);
        stat_par ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
      // the next tile's GELU writes the hidden buffers: every warp's stores must have read its staging tiles
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      mbar_arrive(stg_free);
      mbar_wait(stg_free, stg_ph, abort_flag, p.err);
      stg_ph ^= 1u;
      if (!ok || *abort_flag) break;
    }
    if (lane == 0) bulk_wait_all();
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
