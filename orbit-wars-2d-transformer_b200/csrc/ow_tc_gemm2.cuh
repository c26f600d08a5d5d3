// Persistent tcgen05 GEMM on CTA pairs (cta_group::2): the block GEMMs of the
// d = 256 tensor-core paths, out[m, n] = A[m, :] . W[n, :] + epilogue.
//
// A (2,1,1) cluster computes 256-row x BLOCK_N tiles. Each CTA loads its own
// 128 rows of A and its half (BLOCK_N/2 rows) of W into its own shared
// memory; the even CTA (the leader) issues one M = 256 MMA over both halves,
// and each CTA's TMEM receives D for its 128 rows and all BLOCK_N columns.
// Against the single-CTA kernel (tc_gemm_kernel) every CTA streams half the
// weight bytes per MMA, so a stage is 32 KB instead of 48 KB and four stages
// fit beside the epilogue's staging: the weight feed, which held the
// single-CTA mainloop at about half the tensor rate at K = 256..1024, halves.
//
// Protocol (all waits bounded, as in tc_gemm_kernel):
//   stage s:  both producers wait their own empty[s]; the leader's producer
//             expects both CTAs' bytes on its full[s]; both CTAs' TMA loads
//             complete on the leader's full[s] (cta_group::2 loads, the
//             barrier addressed through mapa); the leader's MMA waits full[s]
//             and its commits arrive on empty[s] in both CTAs.
//   tile:     the commits after a tile's last MMA arrive on tfull[acc] in
//             both CTAs; both CTAs' epilogue warps drain their TMEM and arrive
//             on the leader's tempty[acc] (2 x epilogue warps arrivals).
// TMEM is allocated by warp 1 of both CTAs with cta_group::2 (same columns),
// and a cluster barrier separates the barrier initialisation from the first
// remote arrival and the last MMA from the deallocation.
// Each CTA fetches its own boxes: no load here is shared between the CTAs.
#pragma once

#include "ow_tc_gemm.cuh"

namespace ow {

template <int BLOCK_N, int EPI>
struct TcGemm2Shape {
  using E = TcGemmShape<BLOCK_N, EPI>;  // epilogue staging, parameters, TMEM plan
  static constexpr int kBlockM = 128;   // this CTA's rows of a 256-row pair tile
  static constexpr int kRowBytes = 128;
  static constexpr int kATileBytes = kBlockM * kRowBytes;
  static constexpr int kBRows = BLOCK_N / 2;  // this CTA's rows of W per tile
  static constexpr int kBTileBytes = kBRows * kRowBytes;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kAcc = E::kAcc;
  static constexpr int kTmemCols = E::kTmemCols;
  static constexpr int kFixedBytes = E::kFixedBytes;
  static constexpr int kStagesFit = (kSmemLimit - kFixedBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kSmemBytes = kStages * kStageBytes + kFixedBytes;
  static_assert(BLOCK_N == 256, "pair tiles: 256 x 256 (M = 256, N = 256 MMA)");
  static_assert(kStages >= 3, "operand stages");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory per CTA");
  static_assert(kStageBytes % 1024 == 0, "swizzled tiles stay 1024 B aligned");
};

template <int BLOCK_N, int EPI, bool FP8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(EpiWarps<EPI>::kThreads, 1)
    tc_gemm2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                    const __grid_constant__ CUtensorMap map_o, const __grid_constant__ CUtensorMap map_l,
                    const TcGemmParams p) {
  using S = TcGemm2Shape<BLOCK_N, EPI>;
  using E = typename S::E;
  constexpr int kEpiWarps = EpiWarps<EPI>::kCount;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + S::kStages * S::kATileBytes;
  uint8_t* s_xpose = smem + S::kStages * S::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_xpose + E::kXposeBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* tfull = empty + S::kStages;
  uint64_t* tempty = tfull + S::kAcc;
  uint64_t* xbar = tempty + S::kAcc;
  uint64_t* pair_bar = xbar + E::kTilesPerWarp * kEpiWarps;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(pair_bar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_par = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + E::kBarrierBytes);
  float4* s_stats = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(s_par) + E::kParamBytes);
  float* s_bias = s_par;
  float* s_bscale = s_par + p.n;
  float* s_g = s_par + (FP8 ? 2 : 1) * p.n;
  float* s_b = s_g + p.n;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int n_tiles = p.n / BLOCK_N;
  constexpr uint32_t kIdesc = FP8 ? idesc_e4m3(256, BLOCK_N) : idesc_bf16(256, BLOCK_N);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < S::kAcc; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    for (int i = 0; i < E::kTilesPerWarp * kEpiWarps; ++i) mbar_init(&xbar[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], EPI == kEpiResidLn16 ? 128 : 64);
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
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
  if (warp == 1) tmem_alloc_pair(tmem_holder, S::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int m_valid = *p.m_valid;
  const int m_pairs = (m_valid + 2 * S::kBlockM - 1) / (2 * S::kBlockM);
  const int num_tiles = m_pairs * n_tiles;
  const int cid = static_cast<int>(blockIdx.x >> 1);
  const int n_clusters = static_cast<int>(gridDim.x >> 1);

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
      for (int tile = cid; tile < num_tiles && ok; tile += n_clusters) {
        const int m0 = (tile / n_tiles) * (2 * S::kBlockM) + static_cast<int>(rank) * S::kBlockM;
        const int n0 = (tile % n_tiles) * BLOCK_N + static_cast<int>(rank) * S::kBRows;

        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0u);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
          const int kx = kb * (FP8 ? 128 : 64);
          if (p.a_stream)
            tma_load_2d_pair_hint(sa + stage * S::kATileBytes, &map_a, full_leader, kx, m0, a_policy);
          else
            tma_load_2d_pair(sa + stage * S::kATileBytes, &map_a, full_leader, kx, m0);
          tma_load_2d_pair(sb + stage * S::kBTileBytes, &map_w, full_leader, kx, n0);
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0 && num_tiles > 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = cid; tile < num_tiles && ok; tile += n_clusters) {
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
            const uint64_t bdesc = sdesc_k_sw128(b_base + k * 32);
            const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
            if (FP8)
              umma_f8_pair(d_tmem, adesc, bdesc, kIdesc, accumulate);
            else
              umma_f16_pair(d_tmem, adesc, bdesc, kIdesc, accumulate);
          }
          umma_commit_pair(&empty[stage]);  // both CTAs' stage s reusable once these MMAs retire
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc]);  // both CTAs' accumulators ready for their epilogues
        if (++acc == S::kAcc) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    // Epilogue warps 2 .. 2+kEpiWarps-1 on this CTA's 128 rows; as in
    // tc_gemm_kernel, except that the accumulator is released on the leader.
    const int ew = warp - 2;
    const int quad = warp & 3;
    uint8_t* tiles = s_xpose + ew * E::kTilesPerWarp * E::kTileBytes;
    constexpr int kCols = EPI == kEpiResidLn ? BLOCK_N : BLOCK_N * 4 / kEpiWarps;
    const int col0 = EPI == kEpiResidLn ? 0 : (ew / 4) * kCols;
    uint64_t* my_xbar = xbar + E::kTilesPerWarp * ew;
    uint32_t xbits = 0u;
    uint32_t pair_phase = 0u;
    int stat_par = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int out_k = 0;
    for (int tile = cid; tile < num_tiles; tile += n_clusters) {
      const int row_base = (tile / n_tiles) * (2 * S::kBlockM) + static_cast<int>(rank) * S::kBlockM + quad * 32;
      if (EPI == kEpiResidLn) {
        if (lane == 0 && row_base < m_valid) {
          bulk_wait_read<0>();
#pragma unroll
          for (int b = 0; b < E::kTilesPerWarp; ++b) {
            mbar_arrive_expect_tx(&my_xbar[b], 4096);
            tma_load_2d_hint(tiles + b * 4096, &map_o, &my_xbar[b], (ew >> 2) * (BLOCK_N / 2) + b * 32, row_base,
                             l2_evict_last());
          }
        }
        __syncwarp();
      } else if (EPI == kEpiResidLn16) {
        if (lane == 0 && row_base < m_valid) {
          bulk_wait_read<0>();
          mbar_arrive_expect_tx(&my_xbar[0], 4096);
          tma_load_2d_hint(tiles, &map_o, &my_xbar[0], (ew >> 2) * 64, row_base, l2_evict_last());
        }
        __syncwarp();
      }
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err)) break;
      tc_fence_after();
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
          if (lane == 0) bulk_wait_read<1>();  // the store that last used this tile has read it
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
          uint8_t* ot = tiles + (out_k & 1) * E::kTileBytes;
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
        resid_ln_epilogue<BLOCK_N, FP8, E::kTilesPerWarp>(tbase, tiles, my_xbar, xbits, s_stats + (stat_par * 8) * 32,
                                                          s_bias, s_bscale, s_g, s_b, &map_o, &map_l, p, abort_flag,
                                                          &pair_bar[quad], pair_phase, ew, quad, lane, row_base, m,
                                                          live, a_s);
        stat_par ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0u));
      }
      if (++acc == S::kAcc) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  __syncthreads();
  // the leader's MMAs write the peer's TMEM and read its shared memory; the
  // peer's loads complete on the leader's barriers: both CTAs stay until all of it is done
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::kTmemCols);
  }
}

}  // namespace ow
