// Host side of the encoder-policy forward: handle lifetime, weight
// conversion/upload, TMA descriptors, the per-precision launch sequence and
// the extern "C" entry points declared in include/ow_policy.h.
//
// Error convention of the reference GPU ABI (native/cuda/orbit_wars_cuda.cu:
// 12-14 status codes, :274-279 status_from_cuda): arguments are validated
// before any launch (BAD_ARGUMENT), CUDA failures and device-side error flags
// become RUNTIME_ERROR with a static message. There is no CPU fallback: a
// missing device or a failed launch is an error.

#include "ow_policy.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "ow_common.cuh"
#include "ow_kernels.cuh"
#include "ow_tc_gemm.cuh"
#include "ow_tc_gemm2.cuh"
#include "ow_tc_ffn.cuh"
#include "ow_tc_attn.cuh"

namespace {

using namespace ow;

OwStatus st_ok() { return {OW_STATUS_OK, "ok"}; }
OwStatus st_bad(const char* m) { return {OW_STATUS_BAD_ARGUMENT, m}; }
OwStatus st_rt(const char* m) { return {OW_STATUS_RUNTIME_ERROR, m}; }
OwStatus st_cuda(cudaError_t e) { return e == cudaSuccess ? st_ok() : st_rt(cudaGetErrorString(e)); }

#define OW_TRY(expr)                         \
  do {                                       \
    const cudaError_t e_ = (expr);           \
    if (e_ != cudaSuccess) return st_cuda(e_); \
  } while (0)

const char* device_error_message(int code) {
  switch (code) {
    case kErrWaitTimeout: return "device wait timed out (kernel aborted)";
    case kErrBadCount: return "entity count outside [0, n_entities]";
    case kErrBadModelIndex: return "model index outside the population";
    default: return "device error";
  }
}

// ---------------------------------------------------------------- weight layout
struct BlobLayout {
  size_t we, be, lnf_g, lnf_b, wp, bp, wv, bv, total;
  struct Layer {
    size_t ln1g, ln1b, wqkv, bqkv, wo, bo, ln2g, ln2b, w1, b1, w2, b2;
  };
  std::vector<Layer> layer;
};

BlobLayout blob_layout(const OwPolicyConfig& c) {
  BlobLayout o;
  const size_t d = c.d_model, F = c.features, f = c.ffn, P = c.actions;
  size_t at = 0;
  auto take = [&at](size_t n) {
    const size_t r = at;
    at += n;
    return r;
  };
  o.we = take(d * F);
  o.be = take(d);
  o.layer.resize(c.layers);
  for (auto& L : o.layer) {
    L.ln1g = take(d);
    L.ln1b = take(d);
    L.wqkv = take(3 * d * d);
    L.bqkv = take(3 * d);
    L.wo = take(d * d);
    L.bo = take(d);
    L.ln2g = take(d);
    L.ln2b = take(d);
    L.w1 = take(f * d);
    L.b1 = take(f);
    L.w2 = take(d * f);
    L.b2 = take(d);
  }
  o.lnf_g = take(d);
  o.lnf_b = take(d);
  o.wp = take(P * d);
  o.bp = take(P);
  o.wv = take(d);
  o.bv = take(1);
  o.total = at;
  return o;
}

const char* validate_config(const OwPolicyConfig& c) {
  if (c.batch_capacity <= 0 || c.batch_capacity > (1 << 20)) return "batch_capacity out of range";
  if (c.n_entities <= 0 || c.n_entities > 128) return "n_entities must be in [1, 128]";
  if (c.features <= 0 || c.features > 32) return "features must be in [1, 32]";
  if (c.d_model % 32 != 0 || c.d_model < 128 || c.d_model > 512) return "d_model must be a multiple of 32 in [128, 512]";
  if (c.heads * 32 != c.d_model) return "heads must equal d_model / 32 (head_dim 32)";
  if (c.ffn <= 0 || c.ffn % 128 != 0 || c.ffn > 4096) return "ffn must be a multiple of 128 in [128, 4096]";
  if (c.layers <= 0 || c.layers > 64) return "layers must be in [1, 64]";
  if (c.actions <= 0 || c.actions > 32) return "actions must be in [1, 32]";
  if (c.precision < OW_PRECISION_F32 || c.precision > OW_PRECISION_FP8) return "unknown precision";
  if (c.sample_actions != 0 && c.sample_actions != 1) return "sample_actions must be 0 or 1";
  if ((c.logits_dtype != OW_DTYPE_F32 && c.logits_dtype != OW_DTYPE_BF16) ||
      (c.value_dtype != OW_DTYPE_F32 && c.value_dtype != OW_DTYPE_BF16))
    return "unknown output dtype";
  if (c.io != OW_IO_HOST && c.io != OW_IO_DEVICE) return "unknown io mode";
  if (c.precision != OW_PRECISION_F32) {
    // tensor-core path: QKV tiles of 256 or 128 columns, LN-fused tiles of d columns
    if ((3 * c.d_model) % 128 != 0) return "3*d_model must be a multiple of 128";
    if (c.d_model != 128 && c.d_model != 256 && c.d_model != 384 && c.d_model != 512)
      return "tensor-core path supports d_model 128, 256, 384, 512";
    if (c.ffn % 256 != 0) return "tensor-core path needs ffn % 256 == 0";
    if (c.precision == OW_PRECISION_FP8 && c.d_model != 256) return "fp8 path supports d_model 256";
  }
  return nullptr;
}

// ---------------------------------------------------------------- TMA descriptors
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major 2-D map over [rows, inner] elements of `elt` bytes with a box of
// box_bytes (128, 64 or 32 bytes of a row) x box_rows, in the swizzle of that
// width: the layout the UMMA operand descriptors (128 B) and the epilogue
// staging tiles (128/64/32 B) use.
enum MapType { kMapBf16, kMapU8, kMapF32 };
bool make_map_box(CUtensorMap* map, const void* base, MapType t, uint64_t inner, uint64_t rows, uint32_t box_bytes,
                  uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr || base == nullptr) return false;
  const uint32_t elt = t == kMapF32 ? 4 : (t == kMapBf16 ? 2 : 1);
  const CUtensorMapDataType dt = t == kMapF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : (t == kMapBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8);
  const CUtensorMapSwizzle sw = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : (box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * elt};
  cuuint32_t box[2] = {box_bytes / elt, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}
bool make_map_128b(CUtensorMap* map, const void* base, MapType t, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  return make_map_box(map, base, t, inner, rows, 128, box_rows);
}
// Epilogue output map: 32 columns x 32 rows in the element type's swizzle
// (f32 128 B, bf16 64 B, e4m3 32 B).
bool make_ln_map(CUtensorMap* map, const void* base, MapType t, uint64_t inner, uint64_t rows) {
  const uint32_t elt = t == kMapF32 ? 4 : (t == kMapBf16 ? 2 : 1);
  return make_map_box(map, base, t, inner, rows, 32 * elt, 32);
}
// Bias / GELU epilogue output map (bf16): chunk_cols columns x 32 rows.
bool make_out_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, int chunk_cols) {
  return make_map_box(map, base, kMapBf16, inner, rows, static_cast<uint32_t>(chunk_cols) * 2, 32);
}
// The tcgen05 attention's block: the smallest of 32, 64, 128 rows holding N entities.
uint32_t attn_block_rows(int n_entities) { return n_entities <= 32 ? 32u : (n_entities <= 64 ? 64u : 128u); }

// K-major GEMM operand map (bf16 or e4m3), box = 128 bytes x box_rows.
bool make_kmajor_map(CUtensorMap* map, const void* base, bool e4m3, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  return make_map_128b(map, base, e4m3 ? kMapU8 : kMapBf16, inner, rows, box_rows);
}

// ---------------------------------------------------------------- host conversions
uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return static_cast<uint16_t>((u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u));
  const uint32_t rounding = 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>((u + rounding) >> 16);
}

// Saturating round-to-nearest-even f32 -> e4m3, the same conversion the
// device kernels use (cuda_fp8.h, callable on the host).
uint8_t f32_to_e4m3_bits(float f) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3));
}

}  // namespace

// ---------------------------------------------------------------- handle
struct OwPolicy {
  OwPolicyConfig cfg{};
  BlobLayout lay;
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int num_sms = 148;
  size_t cap_rows = 0;
  int cap_states = 0;  // states the active lane's workspace holds

  // weights (device arena)
  uint8_t* warena = nullptr;
  size_t warena_bytes = 0;
  struct LayerW {
    float *ln1g, *ln1b, *bqkv, *bo, *ln2g, *ln2b, *b1, *b2;
    void *wqkv, *wo, *w1, *w2;      // f32 / bf16 / e4m3 [out, in]
    float *sqkv, *so, *s1, *s2;     // e4m3 per-output-channel scales
    CUtensorMap mqkv, mo, m1, m2;
    CUtensorMap m1f, m2f;           // fused FFN: W1 / W2 in 128-row boxes
    CUtensorMap mqkv2, mo2, m12, m22;  // CTA-pair GEMMs: each CTA's half of a 256-row box
  };
  std::vector<LayerW> lw;
  float *we = nullptr, *be = nullptr, *lnfg = nullptr, *lnfb = nullptr, *wp = nullptr, *bp = nullptr,
        *wv = nullptr, *bv = nullptr;
  __nv_bfloat16* we16 = nullptr;  // W_e as bf16 [d][32] (features zero-padded) for the tensor-core embedding

  // workspace
  uint8_t* ws = nullptr;
  int *counts = nullptr, *offsets = nullptr, *err = nullptr;
  float* feats = nullptr;
  void *logits = nullptr, *value = nullptr;
  int* actions = nullptr;
  int* row_slot = nullptr;  // packed row -> b*N + j
  float* sval = nullptr;    // packed row -> y.W_v (value head, before the per-state mean)
  void *x = nullptr, *ln = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *y = nullptr;
  uint8_t *ln8 = nullptr, *attn8 = nullptr, *h8 = nullptr;
  float *ln_scale = nullptr, *attn_scale = nullptr, *h_scale = nullptr;
  CUtensorMap m_ln, m_attn, m_h;       // GEMM A operands
  CUtensorMap e_qkv, e_h, e_x;         // epilogue outputs: qkv / h (bf16, 32-row boxes), x (f32)
  CUtensorMap e_ln, e_y;               // LayerNorm outputs: ln (bf16 or e4m3), y (f32, final LN)
  CUtensorMap a_qkv;                   // attention: qkv in 64-column (two heads) x block-row boxes, 128 B swizzle
  int qkv_block_n = 256;
  bool pdl = false;       // tensor-core path: programmatic dependent launches (ORBIT_WARS_PDL=0 turns them off)
  bool fuse_ffn = false;  // ORBIT_WARS_FFN_FUSED=1 at create selects the fused FFN kernel (d = 256, bf16, f32 x)
  // bf16 residual stream x (the spec's bf16 storage) with the 16-warp LayerNorm
  // epilogue: the tensor-core paths at d = 256 (ORBIT_WARS_X_F32=1 keeps f32)
  bool x16 = false;
  // block GEMMs on CTA pairs (tc_gemm2_kernel, cta_group::2) where x16 holds,
  // opt-in with ORBIT_WARS_PAIR=1: the pair mainloop is faster, but at config
  // 2 the epilogues bound the QKV, up-projection and out-projection GEMMs and
  // the pair couples the two CTAs' epilogues, so the forward measured slower
  // (1.41M -> 1.33M states/s); pair_clusters = the clusters of two that fit on
  // the device at once (the persistent grid)
  bool pair = false;
  int pair_clusters = 0;
  // masked attention on tcgen05 with S and P in TMEM (tc_attention_kernel);
  // ORBIT_WARS_ATTN_MMA=1 selects the mma.sync kernel with S and P in
  // registers (attention_bf16_kernel), measured faster at config 2 (30.8 us
  // against 33.5 us per layer): two softmax warpgroups per SM take the heads
  // one at a time, against the mma.sync kernel's many resident CTAs
  bool attn_tc = true;
  // bias / GELU GEMMs at BLOCK_N = 256 and K <= 4 k-blocks keep the CTA's slice
  // of W in shared memory (TcGemmWsShape); ORBIT_WARS_GEMM_WS=0 streams it
  bool gemm_ws = true;
  int launches = 0;
  // host-IO submissions (ow_policy_submit / ow_policy_wait): two slots, each
  // with its own device inputs, outputs and error word. Uploads run on
  // copy_in, the forward on `stream`, downloads on copy_out; events chain
  // them, so one slot's transfers overlap the other slot's forward.
  struct IoSlot {
    float* feats = nullptr;
    int* counts = nullptr;
    void* logits = nullptr;
    void* value = nullptr;
    int* actions = nullptr;
    int* err = nullptr;
    int* host_err = nullptr;  // pinned: the slot's device error word after the download
    cudaEvent_t in_done = nullptr, comp_done = nullptr, out_done = nullptr;
    int64_t ticket = -1;  // submission occupying the slot; -1 when free
  };
  static constexpr int kIoSlots = 2;
  IoSlot io[kIoSlots];
  // Compute lanes: a lane is a compute stream plus its own activation
  // workspace and tensor maps. The fields above (stream, ws, x, ln, ...,
  // m_ln, ..., e_y) are the active lane's; lanes[k] keeps each lane's copy.
  // Host-IO handles get a second lane when it fits in device memory, so the
  // forwards of the two IO slots can run at the same time.
  struct Lane {
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    uint8_t* ws = nullptr;
    size_t ws_bytes = 0;
    size_t cap_rows = 0;
    int cap_states = 0;
    int *counts = nullptr, *offsets = nullptr, *err = nullptr;
    float* feats = nullptr;
    void *logits = nullptr, *value = nullptr;
    int *actions = nullptr, *row_slot = nullptr;
    float* sval = nullptr;
    void *x = nullptr, *ln = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *y = nullptr;
    uint8_t *ln8 = nullptr, *attn8 = nullptr, *h8 = nullptr;
    float *ln_scale = nullptr, *attn_scale = nullptr, *h_scale = nullptr;
    CUtensorMap m_ln, m_attn, m_h, e_qkv, e_h, e_x, e_ln, e_y, a_qkv;
  };
  Lane lanes[2];
  int n_lanes = 1;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;  // device-IO split forward: lane 1 after lane 0's queue, and back
  bool split_lane = false;  // device IO: lane 1 holds half the capacity and takes the second half of a batch
  int state_base = 0;       // global index of the forward's first state (Gumbel keys) when a batch is split
  size_t ws_bytes = 0;  // the active lane's workspace size
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  int64_t next_ticket = 0;
  // profiling (ow_policy_profile_begin/_end)
  std::vector<cudaEvent_t> prof_events;
  std::vector<const char*> prof_names;
  size_t prof_used = 0;
  bool prof_on = false;
};

namespace {

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
    dev_ = dev;
  }
  ~DeviceGuard() {
    if (prev_ != dev_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0, dev_ = 0;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Launches `kernel` on P's stream. With P.pdl the launch is a programmatic
// dependent launch: the kernel may start (and run its weight-only prologue)
// while the previous kernel finishes; its pdl_wait() orders every read of
// earlier results. Only kernels that call pdl_wait() are launched this way.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(const OwPolicy& P, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = P.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = P.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int BN, int EPI, bool FP8>
cudaError_t set_gemm_attr() {
  return cudaFuncSetAttribute(tc_gemm_kernel<BN, EPI, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              TcGemmShape<BN, EPI>::kSmemBytes);
}
template <int EPI, bool FP8>
cudaError_t set_gemm_ws_attr() {
  return cudaFuncSetAttribute(tc_gemm_kernel<256, EPI, FP8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              TcGemmWsShape<EPI>::kSmemBytes);
}

template <int EPI, bool FP8>
cudaError_t set_gemm2_attr() {
  return cudaFuncSetAttribute(tc_gemm2_kernel<256, EPI, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              TcGemm2Shape<256, EPI>::kSmemBytes);
}

// Clusters of two CTAs of the pair GEMM that can be resident at once (the
// persistent grid is twice this, at most).
int pair_cluster_capacity(int num_sms) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms & ~1));
  cfg.blockDim = dim3(EpiWarps<kEpiResidLn16>::kThreads);
  cfg.dynamicSmemBytes = TcGemm2Shape<256, kEpiResidLn16>::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_gemm2_kernel<256, kEpiResidLn16, false>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// CTA-pair GEMM launch: a persistent grid of at most P.pair_clusters clusters.
template <int EPI, bool FP8>
cudaError_t launch_gemm2(const OwPolicy& P, const CUtensorMap& ma, const CUtensorMap& mw, const CUtensorMap& mo,
                         const CUtensorMap& ml, const TcGemmParams& prm) {
  using S = TcGemm2Shape<256, EPI>;
  const long long pair_tiles = static_cast<long long>((P.cap_rows + 255) / 256) * (prm.n / 256);
  const int clusters = static_cast<int>(std::max<long long>(1, std::min<long long>(P.pair_clusters, pair_tiles)));
  if (prm.n * ((FP8 ? 2 : 1) + (EPI == kEpiResidLn16 ? 2 : 0)) > S::E::kParamFloats) return cudaErrorInvalidValue;
  return launch_k(P, tc_gemm2_kernel<256, EPI, FP8>, 2 * clusters, EpiWarps<EPI>::kThreads, S::kSmemBytes, ma, mw, mo,
                  ml, prm);
}

template <int BN, int EPI, bool FP8>
cudaError_t launch_gemm(const OwPolicy& P, const CUtensorMap& ma, const CUtensorMap& mw, const CUtensorMap& mo,
                        const CUtensorMap& ml, const TcGemmParams& prm) {
  if constexpr (BN == 256 && (EPI == kEpiBias || EPI == kEpiBiasGelu)) {
    // weight-stationary: a multiple of the column tiles as the persistent grid,
    // so each CTA keeps one 256-row slice of W in shared memory
    using W = TcGemmWsShape<EPI>;
    const int n_tiles = prm.n / BN;
    if (P.gemm_ws && prm.k_blocks <= W::kMaxKBlocks && n_tiles <= P.num_sms &&
        prm.n * (FP8 ? 2 : 1) <= W::kParamFloats) {
      const long long m_tiles = static_cast<long long>((P.cap_rows + W::kBlockM - 1) / W::kBlockM);
      const int per = static_cast<int>(std::max<long long>(1, std::min<long long>(P.num_sms / n_tiles, m_tiles)));
      return launch_k(P, tc_gemm_kernel<BN, EPI, FP8, true>, per * n_tiles, EpiWarps<EPI>::kThreads, W::kSmemBytes,
                      ma, mw, mo, ml, prm);
    }
  }
  using S = TcGemmShape<BN, EPI>;
  const long long cap_tiles = static_cast<long long>((P.cap_rows + S::kBlockM - 1) / S::kBlockM) * (prm.n / BN);
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(P.num_sms, cap_tiles)));
  if (prm.n * ((FP8 ? 2 : 1) + ((EPI == kEpiResidLn || EPI == kEpiResidLn16) ? 2 : 0)) > S::kParamFloats)
    return cudaErrorInvalidValue;
  return launch_k(P, tc_gemm_kernel<BN, EPI, FP8>, grid, EpiWarps<EPI>::kThreads, S::kSmemBytes, ma, mw, mo, ml, prm);
}

// Dispatch on the d-wide LN-fused tile.
cudaError_t launch_gemm_resid_ln(const OwPolicy& P, const CUtensorMap& ma, const CUtensorMap& mw,
                                 const CUtensorMap& mx, const CUtensorMap& ml, const TcGemmParams& prm, bool fp8) {
  const int d = P.cfg.d_model;
  if (P.x16 && P.pair) {
    if (fp8) return launch_gemm2<kEpiResidLn16, true>(P, ma, mw, mx, ml, prm);
    return launch_gemm2<kEpiResidLn16, false>(P, ma, mw, mx, ml, prm);
  }
  if (P.x16) {
    if (fp8) return launch_gemm<256, kEpiResidLn16, true>(P, ma, mw, mx, ml, prm);
    return launch_gemm<256, kEpiResidLn16, false>(P, ma, mw, mx, ml, prm);
  }
  if (fp8) return launch_gemm<256, kEpiResidLn, true>(P, ma, mw, mx, ml, prm);
  switch (d) {
    case 128: return launch_gemm<128, kEpiResidLn, false>(P, ma, mw, mx, ml, prm);
    case 256: return launch_gemm<256, kEpiResidLn, false>(P, ma, mw, mx, ml, prm);
    case 384: return launch_gemm<384, kEpiResidLn, false>(P, ma, mw, mx, ml, prm);
    default: return launch_gemm<512, kEpiResidLn, false>(P, ma, mw, mx, ml, prm);
  }
}

// The fused FFN kernel serves the bf16 path at d = 256 (its TMEM plan), f a
// multiple of 128 with b1, b2, gamma and beta staged in shared memory.
bool ffn_fused(const OwPolicy& P) {
  const auto& c = P.cfg;
  return P.fuse_ffn && !P.x16 && c.precision == OW_PRECISION_BF16 && c.d_model == 256 && c.ffn % 128 == 0 &&
         c.ffn + 3 * c.d_model <= TcFfnShape<256>::kParamFloats;
}

cudaError_t launch_ffn(const OwPolicy& P, const CUtensorMap& ma, const CUtensorMap& m1, const CUtensorMap& m2,
                       const CUtensorMap& mx, const CUtensorMap& ml, const TcGemmParams& prm) {
  using S = TcFfnShape<256>;
  const long long cap_tiles = static_cast<long long>((P.cap_rows + S::kBlockM - 1) / S::kBlockM);
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(P.num_sms, cap_tiles)));
  return launch_k(P, tc_ffn_kernel<256>, grid, S::kThreads, S::kSmemBytes, ma, m1, m2, mx, ml, prm);
}

// Test hook support: packed row -> state * n + entity (the embedding kernel
// writes the same map in the forward).
__global__ void fill_row_slot_kernel(const int* offsets, int batch, int n, int* row_slot) {
  for (int b = blockIdx.x; b < batch; b += gridDim.x) {
    const int r0 = offsets[b], c = offsets[b + 1] - r0;
    for (int j = threadIdx.x; j < c; j += blockDim.x) row_slot[r0 + j] = b * n + j;
  }
}

cudaError_t set_all_gemm_attrs() {
  cudaError_t e = cudaSuccess;
  auto upd = [&e](cudaError_t r) {
    if (e == cudaSuccess) e = r;
  };
  upd(set_gemm_attr<128, kEpiBias, false>());
  upd(set_gemm_attr<256, kEpiBias, false>());
  upd(set_gemm_attr<256, kEpiBiasGelu, false>());
  upd(set_gemm_attr<128, kEpiResidLn, false>());
  upd(set_gemm_attr<256, kEpiResidLn, false>());
  upd(set_gemm_attr<384, kEpiResidLn, false>());
  upd(set_gemm_attr<512, kEpiResidLn, false>());
  upd(set_gemm_attr<256, kEpiBias, true>());
  upd(set_gemm_attr<256, kEpiBiasGelu, true>());
  upd(set_gemm_attr<256, kEpiResidLn, true>());
  upd(set_gemm_attr<256, kEpiResidLn16, false>());
  upd(set_gemm_attr<256, kEpiResidLn16, true>());
  upd(set_gemm_ws_attr<kEpiBias, false>());
  upd(set_gemm_ws_attr<kEpiBiasGelu, false>());
  upd(set_gemm_ws_attr<kEpiBias, true>());
  upd(set_gemm_ws_attr<kEpiBiasGelu, true>());
  upd(set_gemm2_attr<kEpiBias, false>());
  upd(set_gemm2_attr<kEpiBiasGelu, false>());
  upd(set_gemm2_attr<kEpiResidLn16, false>());
  upd(set_gemm2_attr<kEpiBias, true>());
  upd(set_gemm2_attr<kEpiBiasGelu, true>());
  upd(set_gemm2_attr<kEpiResidLn16, true>());
  upd(cudaFuncSetAttribute(tc_ffn_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TcFfnShape<256>::kSmemBytes));
  upd(cudaFuncSetAttribute(tc_attention_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TcAttnShape<32>::kSmemBytes));
  upd(cudaFuncSetAttribute(tc_attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TcAttnShape<64>::kSmemBytes));
  upd(cudaFuncSetAttribute(tc_attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TcAttnShape<128>::kSmemBytes));
  return e;
}

template <int DPL>
cudaError_t launch_embed(const OwPolicy& P, int batch) {
  const auto& c = P.cfg;
  const long long slots = static_cast<long long>(batch) * c.n_entities;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((slots + 7) / 8, P.num_sms * 6LL)));
  const size_t smem = static_cast<size_t>(c.features) * (DPL * 32 + 1) * sizeof(float);
  const float* g = P.lw[0].ln1g;
  const float* b = P.lw[0].ln1b;
  if (c.precision == OW_PRECISION_F32) {
    auto k = embed_ln_kernel<DPL, 0>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    k<<<grid, 256, smem, P.stream>>>(P.feats, P.offsets, batch, c.n_entities, c.features, P.we, P.be, g, b,
                                     static_cast<float*>(P.x), P.ln, nullptr);
  } else {
    constexpr int D = DPL * 32;
    const size_t esmem = static_cast<size_t>(D) * 40 * 2 + 4 * 16 * 40 * 2 + 3 * D * sizeof(float);
    // a warp takes 16 packed rows at a time; one wave of resident CTAs, each staging W_e once
    const int eg = static_cast<int>(std::max<size_t>(1, std::min<size_t>((P.cap_rows + 63) / 64,
                                                                          static_cast<size_t>(P.num_sms) * kEmbedMinBlocks)));
    if (c.precision == OW_PRECISION_BF16 && P.x16) {
      auto k = embed_mma_kernel<D, 1, true>;
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(esmem));
      return launch_k(P, k, eg, 128, esmem, static_cast<const float*>(P.feats), static_cast<const int*>(P.offsets),
                      batch, c.n_entities, c.features, static_cast<const __nv_bfloat16*>(P.we16),
                      static_cast<const float*>(P.be), g, b, P.x, static_cast<void*>(P.ln),
                      static_cast<float*>(nullptr), P.row_slot);
    } else if (c.precision == OW_PRECISION_BF16) {
      auto k = embed_mma_kernel<D, 1, false>;
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(esmem));
      return launch_k(P, k, eg, 128, esmem, static_cast<const float*>(P.feats), static_cast<const int*>(P.offsets),
                      batch, c.n_entities, c.features, static_cast<const __nv_bfloat16*>(P.we16),
                      static_cast<const float*>(P.be), g, b, P.x, static_cast<void*>(P.ln),
                      static_cast<float*>(nullptr), P.row_slot);
    } else if (P.x16) {
      auto k = embed_mma_kernel<D, 2, true>;
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(esmem));
      return launch_k(P, k, eg, 128, esmem, static_cast<const float*>(P.feats), static_cast<const int*>(P.offsets),
                      batch, c.n_entities, c.features, static_cast<const __nv_bfloat16*>(P.we16),
                      static_cast<const float*>(P.be), g, b, P.x, static_cast<void*>(P.ln8),
                      P.ln_scale, P.row_slot);
    } else {
      auto k = embed_mma_kernel<D, 2, false>;
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(esmem));
      return launch_k(P, k, eg, 128, esmem, static_cast<const float*>(P.feats), static_cast<const int*>(P.offsets),
                      batch, c.n_entities, c.features, static_cast<const __nv_bfloat16*>(P.we16),
                      static_cast<const float*>(P.be), g, b, P.x, static_cast<void*>(P.ln8),
                      P.ln_scale, P.row_slot);
    }
  }
  return cudaGetLastError();
}

template <int DPL, int PP, bool LB, bool VB>
void heads_launch(const OwPolicy& P, int batch, uint64_t seed, void* logits, void* value, int* actions) {
  const auto& c = P.cfg;
  const size_t smem = static_cast<size_t>(PP + 4) * DPL * 32 * sizeof(float);
  cudaFuncSetAttribute(heads_kernel<DPL, PP, LB, VB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  const int grid = std::max(1, std::min(batch, P.num_sms * 8));
  heads_kernel<DPL, PP, LB, VB><<<grid, 128, smem, P.stream>>>(static_cast<const float*>(P.y), P.offsets, batch,
                                                               c.n_entities, c.actions, P.wp, P.bp, P.wv, P.bv,
                                                               c.sample_actions, seed, logits, value, actions);
}

template <int DPL, int PP>
void heads_dtype(const OwPolicy& P, int batch, uint64_t seed, void* logits, void* value, int* actions) {
  const bool lb = P.cfg.logits_dtype == OW_DTYPE_BF16, vb = P.cfg.value_dtype == OW_DTYPE_BF16;
  if (lb && vb) heads_launch<DPL, PP, true, true>(P, batch, seed, logits, value, actions);
  else if (lb) heads_launch<DPL, PP, true, false>(P, batch, seed, logits, value, actions);
  else if (vb) heads_launch<DPL, PP, false, true>(P, batch, seed, logits, value, actions);
  else heads_launch<DPL, PP, false, false>(P, batch, seed, logits, value, actions);
}

template <int D, int NTILE, bool LB>
cudaError_t heads_mma_launch(const OwPolicy& P, int batch, uint64_t seed, void* logits, int* actions) {
  const auto& c = P.cfg;
  const size_t smem = static_cast<size_t>(NTILE) * 8 * (D + 16) * sizeof(float);
  cudaFuncSetAttribute(heads_mma_kernel<D, NTILE, LB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(smem));
  // a warp takes 16 packed rows at a time; one wave of resident CTAs, each staging the head weights once
  const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>((P.cap_rows + 63) / 64,
                                                                         static_cast<size_t>(P.num_sms) * kHeadsMinBlocks)));
  return launch_k(P, heads_mma_kernel<D, NTILE, LB>, grid, 128, smem, static_cast<const float*>(P.y),
           static_cast<const int*>(P.offsets), batch, c.n_entities, c.actions, static_cast<const int*>(P.row_slot),
           static_cast<const float*>(P.wp), static_cast<const float*>(P.bp), static_cast<const float*>(P.wv),
           c.sample_actions, seed, P.state_base, logits, actions, P.sval);
}

template <int D>
cudaError_t launch_heads_tc(const OwPolicy& P, int batch, uint64_t seed, void* logits, int* actions) {
  const int a = P.cfg.actions;
  const bool lb = P.cfg.logits_dtype == OW_DTYPE_BF16;
  // 8-column tiles covering the P logits plus the value column
  if (a < 8) return lb ? heads_mma_launch<D, 1, true>(P, batch, seed, logits, actions) : heads_mma_launch<D, 1, false>(P, batch, seed, logits, actions);
  if (a < 16) return lb ? heads_mma_launch<D, 2, true>(P, batch, seed, logits, actions) : heads_mma_launch<D, 2, false>(P, batch, seed, logits, actions);
  if (a < 24) return lb ? heads_mma_launch<D, 3, true>(P, batch, seed, logits, actions) : heads_mma_launch<D, 3, false>(P, batch, seed, logits, actions);
  if (a < 32) return lb ? heads_mma_launch<D, 4, true>(P, batch, seed, logits, actions) : heads_mma_launch<D, 4, false>(P, batch, seed, logits, actions);
  return lb ? heads_mma_launch<D, 5, true>(P, batch, seed, logits, actions) : heads_mma_launch<D, 5, false>(P, batch, seed, logits, actions);
}

cudaError_t launch_finalize(const OwPolicy& P, int batch, void* logits, void* value, int* actions) {
  const auto& c = P.cfg;
  const int threads = (c.n_entities + 31) / 32 * 32;
  const bool lb = c.logits_dtype == OW_DTYPE_BF16, vb = c.value_dtype == OW_DTYPE_BF16;
#define OW_FIN(LB, VB)                                                                                      \
  return launch_k(P, state_finalize_kernel<LB, VB>, batch, threads, 0, static_cast<const int*>(P.offsets),  \
                  c.n_entities, c.actions, static_cast<const float*>(P.sval), static_cast<const float*>(P.bv), \
                  logits, value, actions)
  if (lb && vb) OW_FIN(true, true);
  if (lb) OW_FIN(true, false);
  if (vb) OW_FIN(false, true);
  OW_FIN(false, false);
#undef OW_FIN
}

template <int DPL>
cudaError_t launch_heads(const OwPolicy& P, int batch, uint64_t seed, void* logits, void* value, int* actions) {
  // SIMT heads of the f32 path (f32 dot products for the 1e-4 tolerance)
  const int a = P.cfg.actions;
  if (a <= 8) heads_dtype<DPL, 8>(P, batch, seed, logits, value, actions);
  else if (a <= 16) heads_dtype<DPL, 16>(P, batch, seed, logits, value, actions);
  else heads_dtype<DPL, 32>(P, batch, seed, logits, value, actions);
  return cudaGetLastError();
}

template <int DPL>
cudaError_t launch_ln_f32(const OwPolicy& P, const int* m_valid, const float* g, const float* b) {
  const int grid = static_cast<int>(std::min<size_t>((P.cap_rows + 7) / 8, static_cast<size_t>(P.num_sms) * 8));
  layernorm_f32_kernel<DPL><<<grid, 256, 0, P.stream>>>(static_cast<const float*>(P.x), m_valid, g, b,
                                                        static_cast<float*>(P.ln));
  return cudaGetLastError();
}

cudaError_t dispatch_embed(const OwPolicy& P, int batch) {
  switch (P.cfg.d_model / 32) {
    case 4: return launch_embed<4>(P, batch);
    case 8: return launch_embed<8>(P, batch);
    case 12: return launch_embed<12>(P, batch);
    case 16: return launch_embed<16>(P, batch);
    default: return cudaErrorInvalidValue;
  }
}
cudaError_t dispatch_heads_tc(const OwPolicy& P, int batch, uint64_t seed, void* logits, int* actions) {
  switch (P.cfg.d_model) {
    case 128: return launch_heads_tc<128>(P, batch, seed, logits, actions);
    case 256: return launch_heads_tc<256>(P, batch, seed, logits, actions);
    case 384: return launch_heads_tc<384>(P, batch, seed, logits, actions);
    case 512: return launch_heads_tc<512>(P, batch, seed, logits, actions);
    default: return cudaErrorInvalidValue;
  }
}
cudaError_t dispatch_heads(const OwPolicy& P, int batch, uint64_t seed, void* logits, void* value, int* actions) {
  switch (P.cfg.d_model / 32) {
    case 4: return launch_heads<4>(P, batch, seed, logits, value, actions);
    case 8: return launch_heads<8>(P, batch, seed, logits, value, actions);
    case 12: return launch_heads<12>(P, batch, seed, logits, value, actions);
    case 16: return launch_heads<16>(P, batch, seed, logits, value, actions);
    default: return cudaErrorInvalidValue;
  }
}
cudaError_t dispatch_ln_f32(const OwPolicy& P, const int* m_valid, const float* g, const float* b) {
  switch (P.cfg.d_model / 32) {
    case 4: return launch_ln_f32<4>(P, m_valid, g, b);
    case 8: return launch_ln_f32<8>(P, m_valid, g, b);
    case 12: return launch_ln_f32<12>(P, m_valid, g, b);
    case 16: return launch_ln_f32<16>(P, m_valid, g, b);
    default: return cudaErrorInvalidValue;
  }
}

// tcgen05 attention: persistent, one CTA per SM; a work unit is a tile of
// 128 / BS states (BS = the power-of-two block >= N) and two heads.
template <int BS>
cudaError_t launch_attention_tc_bs(const OwPolicy& P, int batch, float scale_log2) {
  using S = TcAttnShape<BS>;
  const auto& c = P.cfg;
  TcAttnParams a{};
  a.offsets = P.offsets;
  a.out = static_cast<__nv_bfloat16*>(P.attn);
  a.err = P.err;
  a.batch = batch;
  a.d = c.d_model;
  a.heads = c.heads;
  a.scale_log2 = scale_log2;
  const long long units = static_cast<long long>((batch + S::kStatesPerTile - 1) / S::kStatesPerTile) *
                          (c.heads / S::kGroup);
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(P.num_sms, units)));
  return launch_k(P, tc_attention_kernel<BS>, grid, S::kThreads, S::kSmemBytes, P.a_qkv, a);
}

// The tcgen05 attention serves head_dim 32 with an even head count.
bool attention_tc(const OwPolicy& P) {
  const auto& c = P.cfg;
  return P.attn_tc && c.precision != OW_PRECISION_F32 && c.d_model == 32 * c.heads && c.heads % 2 == 0 &&
         c.n_entities <= 128;
}

cudaError_t launch_attention_tc(const OwPolicy& P, int batch, float scale_log2) {
  if (P.cfg.n_entities <= 32) return launch_attention_tc_bs<32>(P, batch, scale_log2);
  if (P.cfg.n_entities <= 64) return launch_attention_tc_bs<64>(P, batch, scale_log2);
  return launch_attention_tc_bs<128>(P, batch, scale_log2);
}

cudaError_t launch_attention(const OwPolicy& P, int batch) {
  const auto& c = P.cfg;
  const dim3 grid(batch, c.heads);
  const float scale = 1.0f / std::sqrt(32.0f);
  if (c.precision == OW_PRECISION_F32) {
    const float* q = static_cast<const float*>(P.qkv);
    float* o = static_cast<float*>(P.attn);
    if (c.n_entities <= 32) attention_f32_kernel<32><<<grid, 128, 0, P.stream>>>(q, o, P.offsets, c.d_model, scale);
    else if (c.n_entities <= 64) attention_f32_kernel<64><<<grid, 128, 0, P.stream>>>(q, o, P.offsets, c.d_model, scale);
    else attention_f32_kernel<128><<<grid, 128, 0, P.stream>>>(q, o, P.offsets, c.d_model, scale);
  } else if (attention_tc(P)) {
    return launch_attention_tc(P, batch, scale * 1.4426950408889634f);
  } else {
    const auto* q = static_cast<const __nv_bfloat16*>(P.qkv);
    auto* o = static_cast<__nv_bfloat16*>(P.attn);
    const float sl2 = scale * 1.4426950408889634f;
    const int nmax = c.n_entities <= 32 ? 32 : (c.n_entities <= 64 ? 64 : (c.n_entities <= 96 ? 96 : 128));
    // head group (4, 2, 1) dividing the head count whose staged Q/K/V fit ~110 KB: 4 heads per CTA
    // (52 KB at N = 64) let four CTAs share an SM, measured faster at config 2 than 8 (two per SM) or 2
    int hg = 4;
    while (hg > 1 && (c.heads % hg != 0 || 3 * nmax * (hg * 32 + 8) * 2 > 112 * 1024)) hg /= 2;
    const dim3 g2(batch, c.heads / hg);
    const size_t smem = static_cast<size_t>(3) * nmax * (hg * 32 + 8) * 2;
    cudaError_t e = cudaSuccess;
#define OW_ATTN(NM, HGV)                                                                                   \
  do {                                                                                                     \
    cudaFuncSetAttribute(attention_bf16_kernel<NM, HGV>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                         static_cast<int>(smem));                                                          \
    e = launch_k(P, attention_bf16_kernel<NM, HGV>, g2, 256, smem, q, o,                                 \
                 static_cast<const int*>(P.offsets), c.d_model, sl2);                                     \
  } while (0)
#define OW_ATTN_HG(NM)              \
  do {                              \
    if (hg == 8) OW_ATTN(NM, 8);    \
    else if (hg == 4) OW_ATTN(NM, 4); \
    else if (hg == 2) OW_ATTN(NM, 2); \
    else OW_ATTN(NM, 1);            \
  } while (0)
    if (nmax == 32) OW_ATTN_HG(32);
    else if (nmax == 64) OW_ATTN_HG(64);
    else if (nmax == 96) OW_ATTN_HG(96);
    else OW_ATTN_HG(128);
#undef OW_ATTN_HG
#undef OW_ATTN
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize(const OwPolicy& P, const int* m_valid, const void* in, int k, uint8_t* out,
                            float* scale) {
  const int grid = static_cast<int>(std::min<size_t>((P.cap_rows + 7) / 8, static_cast<size_t>(P.num_sms) * 8));
  return launch_k(P, quantize_rows_e4m3_kernel, grid, 256, 0, static_cast<const __nv_bfloat16*>(in), m_valid, k,
                  out, scale);
}

// m_valid lives at offsets[batch]: the kernels read it from there.
cudaError_t run_blocks(OwPolicy& P, int batch, uint64_t seed, void* logits, void* value, int* actions) {
  const auto& c = P.cfg;
  const int* m_valid = P.offsets + batch;
  int launches = 0;
  cudaError_t e;
#define OW_STEP(name, expr)                                         \
  do {                                                              \
    if (P.prof_on && P.prof_used + 1 < P.prof_events.size()) {      \
      cudaEventRecord(P.prof_events[P.prof_used], P.stream);         \
      P.prof_names[P.prof_used++] = (name);                          \
    }                                                               \
    e = (expr);                                                     \
    if (e != cudaSuccess) return e;                                 \
    ++launches;                                                     \
  } while (0)
  OW_STEP("scan_counts", (scan_counts_kernel<<<1, 1024, 0, P.stream>>>(P.counts, batch, c.n_entities, P.offsets, P.err),
           cudaGetLastError()));
  OW_STEP("embed_ln", dispatch_embed(P, batch));
  const int d = c.d_model, f = c.ffn;
  if (c.precision == OW_PRECISION_F32) {
    const dim3 blk(256);
    // 32 x 32 tiles when 64 x 64 ones would not give every SM two CTAs (small batches)
    const bool small = static_cast<long long>((P.cap_rows + 63) / 64) * ((d + 63) / 64) < 2LL * P.num_sms;
    auto grid_for = [&](int n) {
      const int t = small ? 32 : 64;
      return dim3((n + t - 1) / t, static_cast<unsigned>((P.cap_rows + t - 1) / t));
    };
    float* x = static_cast<float*>(P.x);
    float* ln = static_cast<float*>(P.ln);
    float* qkv = static_cast<float*>(P.qkv);
    float* attn = static_cast<float*>(P.attn);
    float* h = static_cast<float*>(P.h);
    for (int l = 0; l < c.layers; ++l) {
      const auto& W = P.lw[l];
      OW_STEP("gemm_f32_qkv", ((small ? gemm_f32_kernel<kF32Bias, 32> : gemm_f32_kernel<kF32Bias, 64>)<<<grid_for(3 * d), blk, 0, P.stream>>>(
                   ln, static_cast<const float*>(W.wqkv), W.bqkv, qkv, m_valid, 3 * d, d),
               cudaGetLastError()));
      OW_STEP("attention", launch_attention(P, batch));
      OW_STEP("gemm_f32_out_resid", ((small ? gemm_f32_kernel<kF32BiasResid, 32> : gemm_f32_kernel<kF32BiasResid, 64>)<<<grid_for(d), blk, 0, P.stream>>>(
                   attn, static_cast<const float*>(W.wo), W.bo, x, m_valid, d, d),
               cudaGetLastError()));
      OW_STEP("layernorm_f32", dispatch_ln_f32(P, m_valid, W.ln2g, W.ln2b));
      OW_STEP("gemm_f32_ffn_up", ((small ? gemm_f32_kernel<kF32BiasGelu, 32> : gemm_f32_kernel<kF32BiasGelu, 64>)<<<grid_for(f), blk, 0, P.stream>>>(
                   ln, static_cast<const float*>(W.w1), W.b1, h, m_valid, f, d),
               cudaGetLastError()));
      OW_STEP("gemm_f32_ffn_down_resid", ((small ? gemm_f32_kernel<kF32BiasResid, 32> : gemm_f32_kernel<kF32BiasResid, 64>)<<<grid_for(d), blk, 0, P.stream>>>(
                   h, static_cast<const float*>(W.w2), W.b2, x, m_valid, d, f),
               cudaGetLastError()));
      const bool last = l + 1 == c.layers;
      OW_STEP("layernorm_f32", dispatch_ln_f32(P, m_valid, last ? P.lnfg : P.lw[l + 1].ln1g, last ? P.lnfb : P.lw[l + 1].ln1b));
    }
  } else {
    const bool fp8 = c.precision == OW_PRECISION_FP8;
    for (int l = 0; l < c.layers; ++l) {
      const auto& W = P.lw[l];
      const bool last = l + 1 == c.layers;
      TcGemmParams q{};
      q.m_valid = m_valid;
      q.err = P.err;
      // QKV projection
      q.n = 3 * d;
      q.k_blocks = fp8 ? d / 128 : d / 64;
      q.bias = W.bqkv;
      q.out = static_cast<__nv_bfloat16*>(P.qkv);
      q.ld_out = 3 * d;
      q.a_scale = P.ln_scale;
      q.b_scale = W.sqkv;
      if (P.pair && fp8) OW_STEP("gemm_qkv", (launch_gemm2<kEpiBias, true>(P, P.m_ln, W.mqkv2, P.e_qkv, P.e_qkv, q)));
      else if (P.pair) OW_STEP("gemm_qkv", (launch_gemm2<kEpiBias, false>(P, P.m_ln, W.mqkv2, P.e_qkv, P.e_qkv, q)));
      else if (fp8) OW_STEP("gemm_qkv", (launch_gemm<256, kEpiBias, true>(P, P.m_ln, W.mqkv, P.e_qkv, P.e_qkv, q)));
      else if (P.qkv_block_n == 256)
        OW_STEP("gemm_qkv", (launch_gemm<256, kEpiBias, false>(P, P.m_ln, W.mqkv, P.e_qkv, P.e_qkv, q)));
      else OW_STEP("gemm_qkv", (launch_gemm<128, kEpiBias, false>(P, P.m_ln, W.mqkv, P.e_qkv, P.e_qkv, q)));
      // attention
      OW_STEP("attention", launch_attention(P, batch));
      if (fp8) OW_STEP("quantize_e4m3", launch_quantize(P, m_valid, P.attn, d, P.attn8, P.attn_scale));
      // out-projection + residual + LN2
      TcGemmParams o{};
      o.m_valid = m_valid;
      o.err = P.err;
      o.n = d;
      o.k_blocks = fp8 ? d / 128 : d / 64;
      o.bias = W.bo;
      o.resid = static_cast<float*>(P.x);
      o.ln_g = W.ln2g;
      o.ln_b = W.ln2b;
      o.ln_mode = fp8 ? kLnE4m3 : kLnBf16;
      o.ln_out = fp8 ? static_cast<void*>(P.ln8) : P.ln;
      o.ln_scale = P.ln_scale;
      o.a_scale = P.attn_scale;
      o.b_scale = W.so;
      OW_STEP("gemm_out_resid_ln", launch_gemm_resid_ln(P, P.m_attn, P.pair ? W.mo2 : W.mo, P.e_x, P.e_ln, o, fp8));
      if (ffn_fused(P)) {
        // FFN up + GELU + down + residual + next LN in one kernel
        TcGemmParams w{};
        w.m_valid = m_valid;
        w.err = P.err;
        w.n = f;
        w.bias = W.b1;
        w.bias2 = W.b2;
        w.resid = static_cast<float*>(P.x);
        w.ln_g = last ? P.lnfg : P.lw[l + 1].ln1g;
        w.ln_b = last ? P.lnfb : P.lw[l + 1].ln1b;
        w.ln_mode = last ? kLnF32 : kLnBf16;
        w.ln_out = last ? P.y : P.ln;
        OW_STEP("ffn_fused", launch_ffn(P, P.m_ln, W.m1f, W.m2f, P.e_x, last ? P.e_y : P.e_ln, w));
        continue;
      }
      // FFN up + GELU
      TcGemmParams u{};
      u.m_valid = m_valid;
      u.err = P.err;
      u.n = f;
      u.k_blocks = fp8 ? d / 128 : d / 64;
      u.bias = W.b1;
      u.out = static_cast<__nv_bfloat16*>(P.h);
      u.ld_out = f;
      u.a_scale = P.ln_scale;
      u.b_scale = W.s1;
      if (P.pair && fp8) OW_STEP("gemm_ffn_up_gelu", (launch_gemm2<kEpiBiasGelu, true>(P, P.m_ln, W.m12, P.e_h, P.e_h, u)));
      else if (P.pair) OW_STEP("gemm_ffn_up_gelu", (launch_gemm2<kEpiBiasGelu, false>(P, P.m_ln, W.m12, P.e_h, P.e_h, u)));
      else if (fp8) OW_STEP("gemm_ffn_up_gelu", (launch_gemm<256, kEpiBiasGelu, true>(P, P.m_ln, W.m1, P.e_h, P.e_h, u)));
      else OW_STEP("gemm_ffn_up_gelu", (launch_gemm<256, kEpiBiasGelu, false>(P, P.m_ln, W.m1, P.e_h, P.e_h, u)));
      if (fp8) OW_STEP("quantize_e4m3", launch_quantize(P, m_valid, P.h, f, P.h8, P.h_scale));
      // FFN down + residual + next LN (LN1 of the next block, or the final LN)
      TcGemmParams w{};
      w.m_valid = m_valid;
      w.err = P.err;
      w.n = d;
      w.k_blocks = fp8 ? f / 128 : f / 64;
      w.bias = W.b2;
      w.resid = static_cast<float*>(P.x);
      w.ln_g = last ? P.lnfg : P.lw[l + 1].ln1g;
      w.ln_b = last ? P.lnfb : P.lw[l + 1].ln1b;
      w.ln_mode = last ? kLnF32 : (fp8 ? kLnE4m3 : kLnBf16);
      w.ln_out = last ? P.y : (fp8 ? static_cast<void*>(P.ln8) : P.ln);
      w.ln_scale = P.ln_scale;
      w.a_scale = P.h_scale;
      w.b_scale = W.s2;
      w.a_stream = 1;  // h is read once here
      OW_STEP("gemm_ffn_down_resid_ln",
              launch_gemm_resid_ln(P, P.m_h, P.pair ? W.m22 : W.m2, P.e_x, last ? P.e_y : P.e_ln, w, fp8));
    }
  }
  if (c.precision == OW_PRECISION_F32) {
    OW_STEP("heads", dispatch_heads(P, batch, seed, logits, value, actions));
  } else {
    OW_STEP("heads", dispatch_heads_tc(P, batch, seed, logits, actions));
    OW_STEP("state_finalize", launch_finalize(P, batch, logits, value, actions));
  }
  if (P.prof_on && P.prof_used < P.prof_events.size()) {
    cudaEventRecord(P.prof_events[P.prof_used], P.stream);
    P.prof_names[P.prof_used++] = nullptr;  // end of this forward
  }
#undef OW_STEP
  P.launches = launches;
  return cudaSuccess;
}

size_t elem_bytes_for(int precision) { return precision == OW_PRECISION_F32 ? 4 : (precision == OW_PRECISION_BF16 ? 2 : 1); }

// Builds the device weight-arena image on the host and uploads it.
OwStatus upload_weights(OwPolicy& P, const float* w) {
  const auto& c = P.cfg;
  const auto& L = P.lay;
  const int prec = c.precision;
  const size_t eb = elem_bytes_for(prec);
  const size_t d = c.d_model, f = c.ffn;
  // arena plan
  std::vector<uint8_t> img;
  auto reserve = [&img](size_t bytes) {
    const size_t at = align_up(img.size(), 256);
    img.resize(at + bytes);
    return at;
  };
  auto put_f32 = [&](size_t src, size_t n) {
    const size_t at = reserve(n * 4);
    std::memcpy(img.data() + at, w + src, n * 4);
    return at;
  };
  struct Mat {
    size_t at, scale_at;
  };
  auto put_mat = [&](size_t src, size_t rows, size_t cols) {
    Mat m{};
    m.at = reserve(rows * cols * eb);
    m.scale_at = 0;
    if (prec == OW_PRECISION_F32) {
      std::memcpy(img.data() + m.at, w + src, rows * cols * 4);
    } else if (prec == OW_PRECISION_BF16) {
      uint16_t* dst = reinterpret_cast<uint16_t*>(img.data() + m.at);
      for (size_t i = 0; i < rows * cols; ++i) dst[i] = f32_to_bf16_bits(w[src + i]);
    } else {
      std::vector<float> scales(rows);
      for (size_t r = 0; r < rows; ++r) {
        float amax = 0.0f;
        for (size_t k = 0; k < cols; ++k) amax = std::max(amax, std::fabs(w[src + r * cols + k]));
        scales[r] = amax > 0.0f ? amax / 448.0f : 1.0f;
      }
      uint8_t* dst = img.data() + m.at;
      for (size_t r = 0; r < rows; ++r)
        for (size_t k = 0; k < cols; ++k) dst[r * cols + k] = f32_to_e4m3_bits(w[src + r * cols + k] / scales[r]);
      m.scale_at = reserve(rows * 4);
      std::memcpy(img.data() + m.scale_at, scales.data(), rows * 4);
    }
    return m;
  };
  const size_t we = put_f32(L.we, d * c.features), be = put_f32(L.be, d);
  const size_t we16 = reserve(d * 32 * 2);
  {
    uint16_t* dst = reinterpret_cast<uint16_t*>(img.data() + we16);
    for (size_t r = 0; r < d; ++r)
      for (size_t f = 0; f < 32; ++f)
        dst[r * 32 + f] = f < static_cast<size_t>(c.features) ? f32_to_bf16_bits(w[L.we + r * c.features + f]) : 0;
  }
  struct LayerAt {
    size_t ln1g, ln1b, bqkv, bo, ln2g, ln2b, b1, b2;
    Mat qkv, o, w1, w2;
  };
  std::vector<LayerAt> la(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const auto& s = L.layer[l];
    la[l].ln1g = put_f32(s.ln1g, d);
    la[l].ln1b = put_f32(s.ln1b, d);
    la[l].qkv = put_mat(s.wqkv, 3 * d, d);
    la[l].bqkv = put_f32(s.bqkv, 3 * d);
    la[l].o = put_mat(s.wo, d, d);
    la[l].bo = put_f32(s.bo, d);
    la[l].ln2g = put_f32(s.ln2g, d);
    la[l].ln2b = put_f32(s.ln2b, d);
    la[l].w1 = put_mat(s.w1, f, d);
    la[l].b1 = put_f32(s.b1, f);
    la[l].w2 = put_mat(s.w2, d, f);
    la[l].b2 = put_f32(s.b2, d);
  }
  const size_t lnfg = put_f32(L.lnf_g, d), lnfb = put_f32(L.lnf_b, d);
  const size_t wp = put_f32(L.wp, c.actions * d), bp = put_f32(L.bp, c.actions);
  const size_t wv = put_f32(L.wv, d), bv = put_f32(L.bv, 1);
  img.resize(align_up(img.size(), 256));

  if (P.warena == nullptr || P.warena_bytes != img.size()) {
    if (P.warena != nullptr) cudaFree(P.warena);
    P.warena = nullptr;
    OW_TRY(cudaMalloc(&P.warena, img.size()));
    P.warena_bytes = img.size();
  }
  OW_TRY(cudaMemcpyAsync(P.warena, img.data(), img.size(), cudaMemcpyHostToDevice, P.stream));
  OW_TRY(cudaStreamSynchronize(P.stream));

  uint8_t* base = P.warena;
  auto F = [base](size_t at) { return reinterpret_cast<float*>(base + at); };
  P.we = F(we);
  P.be = F(be);
  P.we16 = reinterpret_cast<__nv_bfloat16*>(base + we16);
  P.lnfg = F(lnfg);
  P.lnfb = F(lnfb);
  P.wp = F(wp);
  P.bp = F(bp);
  P.wv = F(wv);
  P.bv = F(bv);
  P.lw.resize(c.layers);
  const bool tc = prec != OW_PRECISION_F32;
  const bool e4 = prec == OW_PRECISION_FP8;
  const uint32_t qkv_rows = static_cast<uint32_t>(P.qkv_block_n);
  const uint32_t d_rows = d <= 256 ? static_cast<uint32_t>(d) : static_cast<uint32_t>(d / 2);
  for (int l = 0; l < c.layers; ++l) {
    auto& W = P.lw[l];
    W.ln1g = F(la[l].ln1g);
    W.ln1b = F(la[l].ln1b);
    W.bqkv = F(la[l].bqkv);
    W.bo = F(la[l].bo);
    W.ln2g = F(la[l].ln2g);
    W.ln2b = F(la[l].ln2b);
    W.b1 = F(la[l].b1);
    W.b2 = F(la[l].b2);
    W.wqkv = base + la[l].qkv.at;
    W.wo = base + la[l].o.at;
    W.w1 = base + la[l].w1.at;
    W.w2 = base + la[l].w2.at;
    W.sqkv = e4 ? F(la[l].qkv.scale_at) : nullptr;
    W.so = e4 ? F(la[l].o.scale_at) : nullptr;
    W.s1 = e4 ? F(la[l].w1.scale_at) : nullptr;
    W.s2 = e4 ? F(la[l].w2.scale_at) : nullptr;
    if (tc) {
      if (!make_kmajor_map(&W.mqkv, W.wqkv, e4, d, 3 * d, e4 ? 256u : qkv_rows) ||
          !make_kmajor_map(&W.mo, W.wo, e4, d, d, d_rows) || !make_kmajor_map(&W.m1, W.w1, e4, d, f, 256u) ||
          !make_kmajor_map(&W.m2, W.w2, e4, f, d, d_rows))
        return st_rt("cuTensorMapEncodeTiled failed for a weight matrix");
      if (P.pair && (!make_kmajor_map(&W.mqkv2, W.wqkv, e4, d, 3 * d, 128u) ||
                     !make_kmajor_map(&W.mo2, W.wo, e4, d, d, 128u) || !make_kmajor_map(&W.m12, W.w1, e4, d, f, 128u) ||
                     !make_kmajor_map(&W.m22, W.w2, e4, f, d, 128u)))
        return st_rt("cuTensorMapEncodeTiled failed for a CTA-pair weight map");
      if (ffn_fused(P) && (!make_kmajor_map(&W.m1f, W.w1, false, d, f, 128u) ||
                           !make_kmajor_map(&W.m2f, W.w2, false, f, d, 128u)))
        return st_rt("cuTensorMapEncodeTiled failed for an FFN weight matrix");
    }
  }
  return st_ok();
}

// Activation workspace (and tensor maps) for `cap_states` states on P's stream.
OwStatus alloc_workspace(OwPolicy& P, int cap_states) {
  const auto& c = P.cfg;
  const size_t B = cap_states, N = c.n_entities, rows = B * N;
  P.cap_rows = rows;
  P.cap_states = cap_states;
  const size_t act = c.precision == OW_PRECISION_F32 ? 4 : 2;
  const size_t d = c.d_model, f = c.ffn;
  size_t at = 0;
  auto take = [&at](size_t bytes) {
    const size_t r = align_up(at, 256);
    at = r + bytes;
    return r;
  };
  const size_t o_counts = take(B * 4), o_offsets = take((B + 1) * 4), o_err = take(16);
  const size_t o_feats = take(rows * c.features * 4);
  const size_t o_logits = take(rows * c.actions * 4), o_value = take(B * 4), o_actions = take(rows * 4);
  // the second host-IO slot's inputs, outputs and error word (the first slot uses the ones above)
  const bool host_io = c.io == OW_IO_HOST;
  const size_t o2_counts = host_io ? take(B * 4) : 0, o2_err = host_io ? take(16) : 0;
  const size_t o2_feats = host_io ? take(rows * c.features * 4) : 0;
  const size_t o2_logits = host_io ? take(rows * c.actions * 4) : 0, o2_value = host_io ? take(B * 4) : 0;
  const size_t o2_actions = host_io ? take(rows * 4) : 0;
  const size_t o_slot = take(rows * 4), o_sval = take(rows * 4);
  const size_t o_x = take(rows * d * 4), o_ln = take(rows * d * act), o_qkv = take(rows * 3 * d * act);
  const size_t o_y = c.precision == OW_PRECISION_F32 ? o_ln : take(rows * d * 4);
  const size_t o_attn = take(rows * d * act), o_h = take(rows * f * act);
  const bool e4 = c.precision == OW_PRECISION_FP8;
  size_t o_ln8 = 0, o_attn8 = 0, o_h8 = 0, o_ls = 0, o_as = 0, o_hs = 0;
  if (e4) {
    o_ln8 = take(rows * d);
    o_attn8 = take(rows * d);
    o_h8 = take(rows * f);
    o_ls = take(rows * 4);
    o_as = take(rows * 4);
    o_hs = take(rows * 4);
  }
  const size_t total = align_up(at, 256);
  P.ws_bytes = total;
  OW_TRY(cudaMalloc(&P.ws, total));
  OW_TRY(cudaMemsetAsync(P.ws, 0, total, P.stream));
  uint8_t* b = P.ws;
  P.counts = reinterpret_cast<int*>(b + o_counts);
  P.offsets = reinterpret_cast<int*>(b + o_offsets);
  P.err = reinterpret_cast<int*>(b + o_err);
  P.feats = reinterpret_cast<float*>(b + o_feats);
  P.logits = b + o_logits;
  P.value = b + o_value;
  P.actions = reinterpret_cast<int*>(b + o_actions);
  if (host_io && P.copy_in == nullptr) {  // the IO slots and copy streams, once per handle
    P.io[0].feats = P.feats;
    P.io[0].counts = P.counts;
    P.io[0].logits = P.logits;
    P.io[0].value = P.value;
    P.io[0].actions = P.actions;
    P.io[0].err = P.err;
    P.io[1].feats = reinterpret_cast<float*>(b + o2_feats);
    P.io[1].counts = reinterpret_cast<int*>(b + o2_counts);
    P.io[1].logits = b + o2_logits;
    P.io[1].value = b + o2_value;
    P.io[1].actions = reinterpret_cast<int*>(b + o2_actions);
    P.io[1].err = reinterpret_cast<int*>(b + o2_err);
    OW_TRY(cudaStreamCreateWithFlags(&P.copy_in, cudaStreamNonBlocking));
    OW_TRY(cudaStreamCreateWithFlags(&P.copy_out, cudaStreamNonBlocking));
    for (auto& sl : P.io) {
      OW_TRY(cudaMallocHost(&sl.host_err, sizeof(int)));
      *sl.host_err = 0;
      OW_TRY(cudaEventCreateWithFlags(&sl.in_done, cudaEventDisableTiming));
      OW_TRY(cudaEventCreateWithFlags(&sl.comp_done, cudaEventDisableTiming));
      OW_TRY(cudaEventCreateWithFlags(&sl.out_done, cudaEventDisableTiming));
    }
  }
  P.row_slot = reinterpret_cast<int*>(b + o_slot);
  P.sval = reinterpret_cast<float*>(b + o_sval);
  P.x = b + o_x;
  P.ln = b + o_ln;
  P.y = b + o_y;
  P.qkv = b + o_qkv;
  P.attn = b + o_attn;
  P.h = b + o_h;
  if (e4) {
    P.ln8 = b + o_ln8;
    P.attn8 = b + o_attn8;
    P.h8 = b + o_h8;
    P.ln_scale = reinterpret_cast<float*>(b + o_ls);
    P.attn_scale = reinterpret_cast<float*>(b + o_as);
    P.h_scale = reinterpret_cast<float*>(b + o_hs);
  }
  if (c.precision != OW_PRECISION_F32) {
    bool ok;
    if (e4)
      ok = make_kmajor_map(&P.m_ln, P.ln8, true, d, rows, 128) && make_kmajor_map(&P.m_attn, P.attn8, true, d, rows, 128) &&
           make_kmajor_map(&P.m_h, P.h8, true, f, rows, 128);
    else
      ok = make_kmajor_map(&P.m_ln, P.ln, false, d, rows, 128) && make_kmajor_map(&P.m_attn, P.attn, false, d, rows, 128) &&
           make_kmajor_map(&P.m_h, P.h, false, f, rows, 128);
    ok = ok && make_out_map(&P.e_qkv, P.qkv, 3 * d, rows, ow::EpiWarps<ow::kEpiBias>::kChunkCols) &&
         make_out_map(&P.e_h, P.h, f, rows, ow::EpiWarps<ow::kEpiBiasGelu>::kChunkCols) &&
         make_ln_map(&P.e_y, P.y, kMapF32, d, rows) && make_map_box(&P.a_qkv, P.qkv, kMapBf16, 3 * d, rows, 128, attn_block_rows(c.n_entities));
    if (P.x16)  // 64-column boxes: x (bf16, 128 B rows), LN out (bf16 128 B rows or e4m3 64 B rows)
      ok = ok && make_map_128b(&P.e_x, P.x, kMapBf16, d, rows, 32) &&
           (e4 ? make_map_box(&P.e_ln, P.ln8, kMapU8, d, rows, 64, 32) : make_map_128b(&P.e_ln, P.ln, kMapBf16, d, rows, 32));
    else
      ok = ok && make_map_128b(&P.e_x, P.x, kMapF32, d, rows, 32) &&
           (e4 ? make_ln_map(&P.e_ln, P.ln8, kMapU8, d, rows) : make_ln_map(&P.e_ln, P.ln, kMapBf16, d, rows));
    if (!ok) return st_rt("cuTensorMapEncodeTiled failed for an activation buffer");
  }
  OW_TRY(cudaStreamSynchronize(P.stream));
  return st_ok();
}

void save_lane(const OwPolicy& P, OwPolicy::Lane& L) {
  L.stream = P.stream;
  L.own_stream = P.own_stream;
  L.ws = P.ws;
  L.ws_bytes = P.ws_bytes;
  L.cap_rows = P.cap_rows;
  L.cap_states = P.cap_states;
  L.counts = P.counts; L.offsets = P.offsets; L.err = P.err; L.feats = P.feats;
  L.logits = P.logits; L.value = P.value; L.actions = P.actions; L.row_slot = P.row_slot; L.sval = P.sval;
  L.x = P.x; L.ln = P.ln; L.qkv = P.qkv; L.attn = P.attn; L.h = P.h; L.y = P.y;
  L.ln8 = P.ln8; L.attn8 = P.attn8; L.h8 = P.h8;
  L.ln_scale = P.ln_scale; L.attn_scale = P.attn_scale; L.h_scale = P.h_scale;
  L.m_ln = P.m_ln; L.m_attn = P.m_attn; L.m_h = P.m_h;
  L.e_qkv = P.e_qkv; L.e_h = P.e_h; L.e_x = P.e_x; L.e_ln = P.e_ln; L.e_y = P.e_y; L.a_qkv = P.a_qkv;
}

void load_lane(OwPolicy& P, const OwPolicy::Lane& L) {
  P.stream = L.stream;
  P.own_stream = L.own_stream;
  P.ws = L.ws;
  P.ws_bytes = L.ws_bytes;
  P.cap_rows = L.cap_rows;
  P.cap_states = L.cap_states;
  P.counts = L.counts; P.offsets = L.offsets; P.err = L.err; P.feats = L.feats;
  P.logits = L.logits; P.value = L.value; P.actions = L.actions; P.row_slot = L.row_slot; P.sval = L.sval;
  P.x = L.x; P.ln = L.ln; P.qkv = L.qkv; P.attn = L.attn; P.h = L.h; P.y = L.y;
  P.ln8 = L.ln8; P.attn8 = L.attn8; P.h8 = L.h8;
  P.ln_scale = L.ln_scale; P.attn_scale = L.attn_scale; P.h_scale = L.h_scale;
  P.m_ln = L.m_ln; P.m_attn = L.m_attn; P.m_h = L.m_h;
  P.e_qkv = L.e_qkv; P.e_h = L.e_h; P.e_x = L.e_x; P.e_ln = L.e_ln; P.e_y = L.e_y; P.a_qkv = L.a_qkv;
}

// Lane 0 is the handle's stream and workspace. On the tensor-core path a
// second lane (own stream, own workspace) is added unless ORBIT_WARS_LANES=1:
// host-IO handles get a full-capacity lane when it takes at most half of the
// free device memory (the two IO slots' forwards then run at the same time);
// device-IO handles get a lane for half the capacity, which takes the second
// half of each large batch while lane 0 runs the first.
OwStatus add_second_lane(OwPolicy& P) {
  save_lane(P, P.lanes[0]);
  P.n_lanes = 1;
  const char* e = std::getenv("ORBIT_WARS_LANES");
  if (P.cfg.precision == OW_PRECISION_F32 || (e != nullptr && e[0] == '1')) return st_ok();
  const bool host = P.cfg.io == OW_IO_HOST;
  const int cap = host ? P.cfg.batch_capacity : (P.cfg.batch_capacity + 1) / 2;
  const size_t need = host ? P.ws_bytes : P.ws_bytes / 2;
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess || need > free_b / 2) return st_ok();
  cudaStream_t s2 = nullptr;
  OW_TRY(cudaStreamCreateWithFlags(&s2, cudaStreamNonBlocking));
  P.stream = s2;
  P.own_stream = true;
  P.ws = nullptr;
  const OwStatus st = alloc_workspace(P, cap);
  save_lane(P, P.lanes[1]);
  load_lane(P, P.lanes[0]);
  if (st.code != OW_STATUS_OK) {
    if (P.lanes[1].ws) cudaFree(P.lanes[1].ws);
    cudaStreamDestroy(s2);
    P.lanes[1] = OwPolicy::Lane{};
    return st;
  }
  P.n_lanes = 2;
  P.split_lane = !host;
  return st_ok();
}

void release(OwPolicy* P) {
  if (P == nullptr) return;
  DeviceGuard g(P->device);
  if (P->stream) cudaStreamSynchronize(P->stream);
  if (P->copy_in) cudaStreamSynchronize(P->copy_in);
  if (P->copy_out) cudaStreamSynchronize(P->copy_out);
  for (auto& sl : P->io) {
    if (sl.in_done) cudaEventDestroy(sl.in_done);
    if (sl.comp_done) cudaEventDestroy(sl.comp_done);
    if (sl.out_done) cudaEventDestroy(sl.out_done);
    if (sl.host_err) cudaFreeHost(sl.host_err);
  }
  if (P->copy_in) cudaStreamDestroy(P->copy_in);
  if (P->copy_out) cudaStreamDestroy(P->copy_out);
  for (auto ev : P->prof_events) cudaEventDestroy(ev);
  if (P->fork_ev) cudaEventDestroy(P->fork_ev);
  if (P->join_ev) cudaEventDestroy(P->join_ev);
  for (int k = 1; k < P->n_lanes; ++k) {
    auto& L = P->lanes[k];
    if (L.stream) cudaStreamSynchronize(L.stream);
    if (L.ws) cudaFree(L.ws);
    if (L.own_stream && L.stream) cudaStreamDestroy(L.stream);
  }
  if (P->n_lanes > 1) {  // the active fields may show another lane: free lane 0 through its record
    P->ws = P->lanes[0].ws;
    P->stream = P->lanes[0].stream;
  }
  if (P->ws) cudaFree(P->ws);
  if (P->warena) cudaFree(P->warena);
  if (P->own_stream && P->stream) cudaStreamDestroy(P->stream);
  delete P;
}

}  // namespace

extern "C" {

OwStatus ow_policy_preset(int preset, OwPolicyConfig* config) {
  if (config == nullptr) return st_bad("null config");
  OwPolicyConfig c{};
  c.features = 32;
  c.actions = 16;
  c.io = OW_IO_HOST;
  c.logits_dtype = OW_DTYPE_BF16;
  c.value_dtype = OW_DTYPE_F32;
  switch (preset) {
    case 1:
      c.batch_capacity = 64; c.n_entities = 32; c.features = 16; c.d_model = 128; c.heads = 4; c.ffn = 512;
      c.layers = 2; c.actions = 8; c.precision = OW_PRECISION_F32; c.logits_dtype = OW_DTYPE_F32;
      break;
    case 2:
      c.batch_capacity = 1024; c.n_entities = 64; c.d_model = 256; c.heads = 8; c.ffn = 1024; c.layers = 4;
      c.precision = OW_PRECISION_BF16;
      break;
    case 3:
      c.batch_capacity = 4096; c.n_entities = 64; c.d_model = 256; c.heads = 8; c.ffn = 1024; c.layers = 4;
      c.precision = OW_PRECISION_FP8; c.value_dtype = OW_DTYPE_BF16;
      break;
    case 4:
      c.batch_capacity = 8192; c.n_entities = 96; c.d_model = 384; c.heads = 12; c.ffn = 1536; c.layers = 6;
      c.precision = OW_PRECISION_BF16; c.sample_actions = 1;
      break;
    case 5:
      c.batch_capacity = 65536; c.n_entities = 128; c.d_model = 512; c.heads = 16; c.ffn = 2048; c.layers = 8;
      c.precision = OW_PRECISION_BF16;
      break;
    default:
      return st_bad("preset must be 1..5");
  }
  *config = c;
  return st_ok();
}

OwStatus ow_policy_weight_count(const OwPolicyConfig* config, size_t* count) {
  if (config == nullptr || count == nullptr) return st_bad("null argument");
  if (const char* m = validate_config(*config)) return st_bad(m);
  *count = blob_layout(*config).total;
  return st_ok();
}

OwStatus ow_policy_create(const OwPolicyConfig* config, const float* weights, size_t weight_count, int device,
                          void* stream, OwPolicy** out) {
  if (config == nullptr || out == nullptr) return st_bad("null argument");
  *out = nullptr;
  if (const char* m = validate_config(*config)) return st_bad(m);
  const BlobLayout lay = blob_layout(*config);
  if (weight_count != lay.total) return st_bad("weight_count does not match the config");
  // weights == NULL: zero weights, to be filled by a broadcast from another rank
  std::vector<float> zeros;
  if (weights == nullptr) {
    zeros.assign(lay.total, 0.0f);
    weights = zeros.data();
  }
  for (size_t i = 0; i < weight_count; ++i)
    if (!std::isfinite(weights[i])) return st_bad("non-finite weight");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return st_rt("no cuda devices");
  if (device < 0 || device >= ndev) return st_bad("device index out of range");
  DeviceGuard g(device);
  cudaDeviceProp prop{};
  OW_TRY(cudaGetDeviceProperties(&prop, device));
  if (config->precision != OW_PRECISION_F32 && prop.major != 10)
    return st_rt("tensor-core path needs an sm_100 (B200) device");
  auto* P = new OwPolicy();
  P->cfg = *config;
  P->lay = lay;
  P->device = device;
  P->num_sms = prop.multiProcessorCount;
  P->qkv_block_n = (3 * config->d_model) % 256 == 0 ? 256 : 128;
  {
    const char* e = std::getenv("ORBIT_WARS_FFN_FUSED");
    P->fuse_ffn = e != nullptr && e[0] == '1';
    const char* q = std::getenv("ORBIT_WARS_PDL");
    P->pdl = config->precision != OW_PRECISION_F32 && !(q != nullptr && q[0] == '0');
    const char* xf = std::getenv("ORBIT_WARS_X_F32");
    P->x16 = config->precision != OW_PRECISION_F32 && config->d_model == 256 && !(xf != nullptr && xf[0] == '1');
    const char* pr = std::getenv("ORBIT_WARS_PAIR");
    P->pair = P->x16 && pr != nullptr && pr[0] == '1';
    const char* am = std::getenv("ORBIT_WARS_ATTN_MMA");
    P->attn_tc = !(am != nullptr && am[0] == '1');
    const char* ws = std::getenv("ORBIT_WARS_GEMM_WS");
    P->gemm_ws = !(ws != nullptr && ws[0] == '0');
  }
  if (stream != nullptr) {
    P->stream = static_cast<cudaStream_t>(stream);
  } else {
    if (cudaStreamCreateWithFlags(&P->stream, cudaStreamNonBlocking) != cudaSuccess) {
      delete P;
      return st_rt("stream creation failed");
    }
    P->own_stream = true;
  }
  OwStatus s = st_cuda(set_all_gemm_attrs());
  if (s.code == OW_STATUS_OK && P->pair) {
    P->pair_clusters = pair_cluster_capacity(P->num_sms);
    if (P->pair_clusters <= 0) P->pair = false;
  }
  if (s.code == OW_STATUS_OK) s = alloc_workspace(*P, config->batch_capacity);
  if (s.code == OW_STATUS_OK) s = add_second_lane(*P);
  if (s.code == OW_STATUS_OK) s = upload_weights(*P, weights);
  if (s.code != OW_STATUS_OK) {
    release(P);
    return s;
  }
  *out = P;
  return st_ok();
}

OwStatus ow_policy_set_weights(OwPolicy* policy, const float* weights, size_t weight_count) {
  if (policy == nullptr || weights == nullptr) return st_bad("null argument");
  if (weight_count != policy->lay.total) return st_bad("weight_count does not match the config");
  for (size_t i = 0; i < weight_count; ++i)
    if (!std::isfinite(weights[i])) return st_bad("non-finite weight");
  DeviceGuard g(policy->device);
  // every lane's forwards read the weight arena: let them finish first
  for (int k = 0; k < policy->n_lanes; ++k) OW_TRY(cudaStreamSynchronize(policy->lanes[k].stream));
  OW_TRY(cudaStreamSynchronize(policy->stream));
  return upload_weights(*policy, weights);
}

OwStatus ow_policy_submit(OwPolicy* policy, const float* features, const int32_t* counts, int32_t batch,
                          void* logits, void* value, int32_t* actions, uint64_t seed, int64_t* ticket) {
  if (policy == nullptr || ticket == nullptr) return st_bad("null argument");
  auto& P = *policy;
  const auto& c = P.cfg;
  if (c.io != OW_IO_HOST) return st_bad("submit / wait need a host-IO handle");
  if (batch <= 0 || batch > c.batch_capacity) return st_bad("batch outside [1, batch_capacity]");
  if (features == nullptr || counts == nullptr) return st_bad("null features or counts");
  for (int32_t b = 0; b < batch; ++b)
    if (counts[b] < 0 || counts[b] > c.n_entities) return st_bad("entity count outside [0, n_entities]");
  auto& sl = P.io[P.next_ticket % OwPolicy::kIoSlots];
  if (sl.ticket >= 0) return st_bad("two submissions in flight: wait for the older one first");
  DeviceGuard g(P.device);
  const size_t B = batch, N = c.n_entities;
  const size_t lbytes = B * N * c.actions * (c.logits_dtype == OW_DTYPE_BF16 ? 2 : 4);
  const size_t vbytes = B * (c.value_dtype == OW_DTYPE_BF16 ? 2 : 4);
  // upload (the slot's previous forward has completed: its submission was waited for)
  OW_TRY(cudaMemsetAsync(sl.err, 0, sizeof(int), P.copy_in));
  OW_TRY(cudaMemcpyAsync(sl.feats, features, B * N * c.features * sizeof(float), cudaMemcpyHostToDevice, P.copy_in));
  OW_TRY(cudaMemcpyAsync(sl.counts, counts, B * sizeof(int), cudaMemcpyHostToDevice, P.copy_in));
  OW_TRY(cudaEventRecord(sl.in_done, P.copy_in));
  // forward on the slot's lane (its own stream and workspace when the handle
  // has two lanes), reading and writing the slot's buffers
  const int lane = static_cast<int>(P.next_ticket % P.n_lanes);
  load_lane(P, P.lanes[lane]);
  P.feats = sl.feats;
  P.counts = sl.counts;
  P.err = sl.err;
  cudaError_t e = cudaStreamWaitEvent(P.stream, sl.in_done, 0);
  if (e == cudaSuccess) e = run_blocks(P, batch, seed, sl.logits, sl.value, sl.actions);
  if (e == cudaSuccess) e = cudaEventRecord(sl.comp_done, P.stream);
  load_lane(P, P.lanes[0]);
  OW_TRY(e);
  // download
  OW_TRY(cudaStreamWaitEvent(P.copy_out, sl.comp_done, 0));
  if (logits) OW_TRY(cudaMemcpyAsync(logits, sl.logits, lbytes, cudaMemcpyDeviceToHost, P.copy_out));
  if (value) OW_TRY(cudaMemcpyAsync(value, sl.value, vbytes, cudaMemcpyDeviceToHost, P.copy_out));
  if (actions) OW_TRY(cudaMemcpyAsync(actions, sl.actions, B * N * sizeof(int), cudaMemcpyDeviceToHost, P.copy_out));
  OW_TRY(cudaMemcpyAsync(sl.host_err, sl.err, sizeof(int), cudaMemcpyDeviceToHost, P.copy_out));
  OW_TRY(cudaEventRecord(sl.out_done, P.copy_out));
  sl.ticket = P.next_ticket;
  *ticket = P.next_ticket++;
  return st_ok();
}

OwStatus ow_policy_wait(OwPolicy* policy, int64_t ticket) {
  if (policy == nullptr) return st_bad("null policy");
  auto& P = *policy;
  if (P.cfg.io != OW_IO_HOST) return st_bad("submit / wait need a host-IO handle");
  if (ticket < 0) return st_bad("unknown ticket");
  auto& sl = P.io[ticket % OwPolicy::kIoSlots];
  if (sl.ticket != ticket) return st_bad("unknown ticket");
  DeviceGuard g(P.device);
  const cudaError_t e = cudaEventSynchronize(sl.out_done);
  sl.ticket = -1;
  OW_TRY(e);
  if (*sl.host_err != 0) return st_rt(device_error_message(*sl.host_err));
  return st_ok();
}

OwStatus ow_policy_forward(OwPolicy* policy, const float* features, const int32_t* counts, int32_t batch,
                           void* logits, void* value, int32_t* actions, uint64_t seed) {
  if (policy == nullptr) return st_bad("null policy");
  auto& P = *policy;
  const auto& c = P.cfg;
  if (batch <= 0 || batch > c.batch_capacity) return st_bad("batch outside [1, batch_capacity]");
  if (features == nullptr || counts == nullptr) return st_bad("null features or counts");
  DeviceGuard g(P.device);
  if (c.io == OW_IO_HOST) {
    int64_t t = 0;
    const OwStatus s = ow_policy_submit(policy, features, counts, batch, logits, value, actions, seed, &t);
    if (s.code != OW_STATUS_OK) return s;
    return ow_policy_wait(policy, t);
  }
  // Device IO: features / counts / outputs are device pointers; the pipeline
  // reads the features and counts in place and writes the outputs directly.
  // With a half-capacity second lane, a batch of 64 states or more is split:
  // lane 1 runs the second half on its own stream and workspace while lane 0
  // runs the first, and each fills SMs the other leaves idle (between kernels
  // and in the last round of row tiles). Rows and states are independent and
  // the Gumbel keys use the global state index, so the outputs are those of
  // one unsplit forward. Profiled forwards are not split.
  const size_t N = c.n_entities;
  void* lo = logits ? logits : P.logits;
  void* vo = value ? value : P.value;
  int32_t* ao = actions ? actions : P.actions;
  float* saved_feats = P.feats;
  int* saved_counts = P.counts;
  int32_t per_fwd = 0;
  ow_policy_launches_per_forward(&P, &per_fwd);
  // profiling records this forward only while event capacity remains (profile_begin's max_forwards)
  const bool profiling = P.prof_on && P.prof_used + static_cast<size_t>(per_fwd) + 1 < P.prof_events.size();
  const bool split = P.n_lanes == 2 && P.split_lane && !profiling && batch >= 64 &&
                     batch - (batch + 1) / 2 <= P.lanes[1].cap_states && (batch + 1) / 2 <= P.lanes[0].cap_states;
  if (!split) {
    P.feats = const_cast<float*>(features);
    P.counts = const_cast<int*>(counts);
    P.state_base = 0;
    const cudaError_t e = run_blocks(P, batch, seed, lo, vo, ao);
    P.feats = saved_feats;
    P.counts = saved_counts;
    return st_cuda(e);
  }
  const int n0 = (batch + 1) / 2, n1 = batch - n0;
  const size_t lb = c.logits_dtype == OW_DTYPE_BF16 ? 2 : 4, vb = c.value_dtype == OW_DTYPE_BF16 ? 2 : 4;
  if (P.fork_ev == nullptr) {
    OW_TRY(cudaEventCreateWithFlags(&P.fork_ev, cudaEventDisableTiming));
    OW_TRY(cudaEventCreateWithFlags(&P.join_ev, cudaEventDisableTiming));
  }
  // fork: lane 1 starts after everything already queued on the handle's stream,
  // together with lane 0 (starting lane 1 some kernels later measured slower)
  OW_TRY(cudaEventRecord(P.fork_ev, P.stream));
  OW_TRY(cudaStreamWaitEvent(P.lanes[1].stream, P.fork_ev, 0));
  P.feats = const_cast<float*>(features);
  P.counts = const_cast<int*>(counts);
  P.state_base = 0;
  cudaError_t e = run_blocks(P, n0, seed, lo, vo, ao);
  P.feats = saved_feats;
  P.counts = saved_counts;
  OW_TRY(e);
  load_lane(P, P.lanes[1]);
  P.feats = const_cast<float*>(features) + static_cast<size_t>(n0) * N * c.features;
  P.counts = const_cast<int*>(counts) + n0;
  P.state_base = n0;
  e = run_blocks(P, n1, seed, static_cast<uint8_t*>(lo) + static_cast<size_t>(n0) * N * c.actions * lb,
                 static_cast<uint8_t*>(vo) + static_cast<size_t>(n0) * vb, ao + static_cast<size_t>(n0) * N);
  if (e == cudaSuccess) e = cudaEventRecord(P.join_ev, P.stream);
  load_lane(P, P.lanes[0]);
  P.state_base = 0;
  OW_TRY(e);
  // join: work queued after this forward on the handle's stream sees both halves
  return st_cuda(cudaStreamWaitEvent(P.stream, P.join_ev, 0));
}

OwStatus ow_policy_synchronize(OwPolicy* policy) {
  if (policy == nullptr) return st_bad("null policy");
  DeviceGuard g(policy->device);
  for (int k = 1; k < policy->n_lanes; ++k) OW_TRY(cudaStreamSynchronize(policy->lanes[k].stream));
  if (policy->copy_in != nullptr) OW_TRY(cudaStreamSynchronize(policy->copy_in));
  if (policy->copy_out != nullptr) OW_TRY(cudaStreamSynchronize(policy->copy_out));
  int herr[2] = {0, 0};
  OW_TRY(cudaMemcpyAsync(&herr[0], policy->err, sizeof(int), cudaMemcpyDeviceToHost, policy->stream));
  if (policy->split_lane)  // the second half of split forwards records its errors in lane 1's word
    OW_TRY(cudaMemcpyAsync(&herr[1], policy->lanes[1].err, sizeof(int), cudaMemcpyDeviceToHost, policy->stream));
  OW_TRY(cudaStreamSynchronize(policy->stream));
  const int code = herr[0] != 0 ? herr[0] : herr[1];
  if (code != 0) {
    cudaMemsetAsync(policy->err, 0, sizeof(int), policy->stream);
    if (policy->split_lane) cudaMemsetAsync(policy->lanes[1].err, 0, sizeof(int), policy->stream);
    cudaStreamSynchronize(policy->stream);
    return st_rt(device_error_message(code));
  }
  return st_ok();
}

OwStatus ow_policy_device_weights(OwPolicy* policy, void** ptr, size_t* bytes) {
  if (policy == nullptr || ptr == nullptr || bytes == nullptr) return st_bad("null argument");
  *ptr = policy->warena;
  *bytes = policy->warena_bytes;
  return st_ok();
}

OwStatus ow_policy_profile_begin(OwPolicy* policy, int32_t max_forwards) {
  if (policy == nullptr || max_forwards <= 0 || max_forwards > 100000) return st_bad("bad profile arguments");
  DeviceGuard g(policy->device);
  int32_t per = 0;
  ow_policy_launches_per_forward(policy, &per);
  const size_t need = static_cast<size_t>(max_forwards) * (per + 1) + 1;
  while (policy->prof_events.size() < need) {
    cudaEvent_t ev;
    OW_TRY(cudaEventCreate(&ev));
    policy->prof_events.push_back(ev);
  }
  policy->prof_names.assign(policy->prof_events.size(), nullptr);
  policy->prof_used = 0;
  policy->prof_on = true;
  return st_ok();
}

OwStatus ow_policy_profile_end(OwPolicy* policy, OwKernelTiming* out, int32_t capacity, int32_t* count) {
  if (policy == nullptr || count == nullptr) return st_bad("null argument");
  DeviceGuard g(policy->device);
  policy->prof_on = false;
  OW_TRY(cudaStreamSynchronize(policy->stream));
  int32_t n = 0;
  for (size_t i = 0; i + 1 < policy->prof_used; ++i) {
    const char* name = policy->prof_names[i];
    if (name == nullptr) continue;
    float ms = 0.0f;
    OW_TRY(cudaEventElapsedTime(&ms, policy->prof_events[i], policy->prof_events[i + 1]));
    int32_t k = 0;
    while (k < n && std::strcmp(out[k].name, name) != 0) ++k;
    if (k == n) {
      if (out == nullptr || n >= capacity) continue;
      out[n].name = name;
      out[n].launches = 0;
      out[n].total_ms = 0.0f;
      ++n;
    }
    out[k].launches += 1;
    out[k].total_ms += ms;
  }
  *count = n;
  policy->prof_used = 0;
  return st_ok();
}

OwStatus ow_selftest_gemm(int precision, int epilogue, int m, int n, int k, const void* a, const void* w,
                          const float* bias, void* out, float* resid, const float* ln_g, const float* ln_b,
                          void* ln_out, int ln_mode, float* ln_scale, const float* a_scale, const float* b_scale,
                          void* stream) {
  const bool fp8 = precision == OW_PRECISION_FP8;
  const bool pair = (epilogue & 16) != 0;  // the CTA-pair kernel (n a multiple of 256; bias, GELU or epilogue 3)
  epilogue &= 15;
  if (pair && (n % 256 != 0 || !(epilogue == kEpiBias || epilogue == kEpiBiasGelu || epilogue == kEpiResidLn16)))
    return st_bad("the CTA-pair GEMM takes n a multiple of 256 and epilogue 0, 1 or 3");
  if (precision != OW_PRECISION_BF16 && !fp8) return st_bad("selftest precision must be bf16 or fp8");
  if (m <= 0 || n <= 0 || k <= 0 || a == nullptr || w == nullptr || bias == nullptr) return st_bad("bad selftest args");
  if (k % (fp8 ? 128 : 64) != 0) return st_bad("k must be a multiple of 128 bytes");
  int bn = 0;
  if (epilogue == kEpiResidLn16) {  // bf16 residual stream (resid points at bf16 values)
    if (resid == nullptr || ln_g == nullptr || ln_b == nullptr || ln_out == nullptr) return st_bad("bad ln args");
    if (n != 256) return st_bad("the bf16-residual LayerNorm epilogue needs n = 256");
    bn = n;
  } else if (epilogue == kEpiResidLn) {
    if (resid == nullptr || ln_g == nullptr || ln_b == nullptr || ln_out == nullptr) return st_bad("bad ln args");
    if (!(n == 128 || n == 256 || n == 384 || n == 512) || (fp8 && n != 256)) return st_bad("unsupported ln width");
    bn = n;
  } else if (epilogue == kEpiBias || epilogue == kEpiBiasGelu) {
    if (out == nullptr) return st_bad("null out");
    bn = n % 256 == 0 ? 256 : (n % 128 == 0 ? 128 : 0);
    if (bn == 0 || (fp8 && bn != 256) || (epilogue == kEpiBiasGelu && bn != 256)) return st_bad("unsupported n");
  } else {
    return st_bad("unknown epilogue");
  }
  if (fp8 && (a_scale == nullptr || b_scale == nullptr)) return st_bad("fp8 needs scales");
  int dev = 0;
  OW_TRY(cudaGetDevice(&dev));
  OwPolicy P;
  P.device = dev;
  {
    const char* ws = std::getenv("ORBIT_WARS_GEMM_WS");
    P.gemm_ws = !(ws != nullptr && ws[0] == '0');
  }
  P.stream = static_cast<cudaStream_t>(stream);
  P.cap_rows = static_cast<size_t>(m);
  cudaDeviceProp prop{};
  OW_TRY(cudaGetDeviceProperties(&prop, dev));
  P.num_sms = prop.multiProcessorCount;
  OW_TRY(set_all_gemm_attrs());
  uint32_t box_rows = bn <= 256 ? static_cast<uint32_t>(bn) : static_cast<uint32_t>(bn / 2);
  if (pair) {
    box_rows = 128;
    P.pair = true;
    P.pair_clusters = pair_cluster_capacity(P.num_sms);
    if (P.pair_clusters <= 0) return st_rt("no CTA-pair cluster fits on this device");
  }
  CUtensorMap ma, mw, mo, ml;
  if (!make_kmajor_map(&ma, a, fp8, k, m, 128) || !make_kmajor_map(&mw, w, fp8, k, n, box_rows))
    return st_rt("cuTensorMapEncodeTiled failed");
  bool mok;
  if (epilogue == kEpiResidLn16) {
    mok = make_map_128b(&mo, resid, kMapBf16, n, m, 32) &&
          (ln_mode == kLnF32 ? make_ln_map(&ml, ln_out, kMapF32, n, m)
                             : (ln_mode == kLnE4m3 ? make_map_box(&ml, ln_out, kMapU8, n, m, 64, 32)
                                                   : make_map_128b(&ml, ln_out, kMapBf16, n, m, 32)));
  } else if (epilogue == kEpiResidLn) {
    const MapType lt = ln_mode == kLnF32 ? kMapF32 : (ln_mode == kLnE4m3 ? kMapU8 : kMapBf16);
    mok = make_map_128b(&mo, resid, kMapF32, n, m, 32) && make_ln_map(&ml, ln_out, lt, n, m);
  } else {
    mok = make_out_map(&mo, out, n, m, epilogue == kEpiBias ? ow::EpiWarps<ow::kEpiBias>::kChunkCols
                                                             : ow::EpiWarps<ow::kEpiBiasGelu>::kChunkCols);
    ml = mo;
  }
  if (!mok) return st_rt("cuTensorMapEncodeTiled failed for an epilogue buffer");
  int* d_m = nullptr;
  int* d_err = nullptr;
  OW_TRY(cudaMalloc(&d_m, 2 * sizeof(int)));
  d_err = d_m + 1;
  const int host_m[2] = {m, 0};
  cudaError_t e = cudaMemcpyAsync(d_m, host_m, sizeof(host_m), cudaMemcpyHostToDevice, P.stream);
  TcGemmParams q{};
  q.m_valid = d_m;
  q.err = d_err;
  q.n = n;
  q.k_blocks = fp8 ? k / 128 : k / 64;
  q.bias = bias;
  q.out = static_cast<__nv_bfloat16*>(out);
  q.ld_out = n;
  q.resid = resid;
  q.ln_g = ln_g;
  q.ln_b = ln_b;
  q.ln_out = ln_out;
  q.ln_mode = ln_mode;
  q.ln_scale = ln_scale;
  q.a_scale = a_scale;
  q.b_scale = b_scale;
  if (e == cudaSuccess) {
    if (epilogue == kEpiResidLn16) {
      P.cfg.d_model = n;
      P.x16 = true;
      e = launch_gemm_resid_ln(P, ma, mw, mo, ml, q, fp8);
    } else if (epilogue == kEpiResidLn) {
      P.cfg.d_model = n;
      e = launch_gemm_resid_ln(P, ma, mw, mo, ml, q, fp8);
    } else if (pair) {
      if (epilogue == kEpiBias) e = fp8 ? launch_gemm2<kEpiBias, true>(P, ma, mw, mo, ml, q)
                                        : launch_gemm2<kEpiBias, false>(P, ma, mw, mo, ml, q);
      else e = fp8 ? launch_gemm2<kEpiBiasGelu, true>(P, ma, mw, mo, ml, q)
                   : launch_gemm2<kEpiBiasGelu, false>(P, ma, mw, mo, ml, q);
    } else if (epilogue == kEpiBias) {
      if (fp8) e = launch_gemm<256, kEpiBias, true>(P, ma, mw, mo, ml, q);
      else if (bn == 256) e = launch_gemm<256, kEpiBias, false>(P, ma, mw, mo, ml, q);
      else e = launch_gemm<128, kEpiBias, false>(P, ma, mw, mo, ml, q);
    } else {
      if (fp8) e = launch_gemm<256, kEpiBiasGelu, true>(P, ma, mw, mo, ml, q);
      else e = launch_gemm<256, kEpiBiasGelu, false>(P, ma, mw, mo, ml, q);
    }
  }
  int herr = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, d_err, sizeof(int), cudaMemcpyDeviceToHost, P.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(P.stream);
  cudaFree(d_m);
  if (e != cudaSuccess) return st_cuda(e);
  if (herr != 0) return st_rt(device_error_message(herr));
  return st_ok();
}

OwStatus ow_selftest_ffn(int m, int d, int f, const void* ln, const void* w1, const float* b1, const void* w2,
                         const float* b2, float* x, const float* ln_g, const float* ln_b, void* ln_out, int ln_mode,
                         void* stream) {
  if (m <= 0 || d != 256 || f <= 0 || f % 128 != 0 || f + 3 * d > TcFfnShape<256>::kParamFloats)
    return st_bad("fused FFN selftest needs d = 256 and f a multiple of 128 (f <= 1280)");
  if (ln == nullptr || w1 == nullptr || b1 == nullptr || w2 == nullptr || b2 == nullptr || x == nullptr ||
      ln_g == nullptr || ln_b == nullptr || ln_out == nullptr || (ln_mode != kLnBf16 && ln_mode != kLnF32))
    return st_bad("bad fused FFN selftest args");
  int dev = 0;
  OW_TRY(cudaGetDevice(&dev));
  OwPolicy P;
  P.device = dev;
  P.stream = static_cast<cudaStream_t>(stream);
  P.cap_rows = static_cast<size_t>(m);
  cudaDeviceProp prop{};
  OW_TRY(cudaGetDeviceProperties(&prop, dev));
  P.num_sms = prop.multiProcessorCount;
  OW_TRY(set_all_gemm_attrs());
  CUtensorMap ma, m1, m2, mx, ml;
  if (!make_kmajor_map(&ma, ln, false, d, m, 128) || !make_kmajor_map(&m1, w1, false, d, f, 128) ||
      !make_kmajor_map(&m2, w2, false, f, d, 128) || !make_map_128b(&mx, x, kMapF32, d, m, 32) ||
      !make_ln_map(&ml, ln_out, ln_mode == kLnF32 ? kMapF32 : kMapBf16, d, m))
    return st_rt("cuTensorMapEncodeTiled failed");
  int* d_m = nullptr;
  OW_TRY(cudaMalloc(&d_m, 2 * sizeof(int)));
  int* d_err = d_m + 1;
  const int host_m[2] = {m, 0};
  cudaError_t e = cudaMemcpyAsync(d_m, host_m, sizeof(host_m), cudaMemcpyHostToDevice, P.stream);
  TcGemmParams q{};
  q.m_valid = d_m;
  q.err = d_err;
  q.n = f;
  q.bias = b1;
  q.bias2 = b2;
  q.resid = x;
  q.ln_g = ln_g;
  q.ln_b = ln_b;
  q.ln_out = ln_out;
  q.ln_mode = ln_mode;
  if (e == cudaSuccess) e = launch_ffn(P, ma, m1, m2, mx, ml, q);
  int herr = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, d_err, sizeof(int), cudaMemcpyDeviceToHost, P.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(P.stream);
  cudaFree(d_m);
  if (e != cudaSuccess) return st_cuda(e);
  if (herr != 0) return st_rt(device_error_message(herr));
  return st_ok();
}

OwStatus ow_selftest_attention(int kernel, int batch, int n_entities, int heads, const int32_t* counts,
                               const void* qkv, void* out, void* stream) {
  if ((kernel != 0 && kernel != 1) || batch <= 0 || n_entities <= 0 || n_entities > 128 || heads <= 0 ||
      heads > 16 || counts == nullptr || qkv == nullptr || out == nullptr)
    return st_bad("bad attention selftest args");
  int dev = 0;
  OW_TRY(cudaGetDevice(&dev));
  OwPolicy P;
  P.device = dev;
  P.stream = static_cast<cudaStream_t>(stream);
  P.cap_rows = static_cast<size_t>(batch) * n_entities;
  cudaDeviceProp prop{};
  OW_TRY(cudaGetDeviceProperties(&prop, dev));
  P.num_sms = prop.multiProcessorCount;
  P.cfg.precision = OW_PRECISION_BF16;
  P.cfg.n_entities = n_entities;
  P.cfg.heads = heads;
  P.cfg.d_model = 32 * heads;
  P.attn_tc = kernel == 0;
  OW_TRY(set_all_gemm_attrs());
  if (kernel == 0 && heads % 2 != 0) return st_bad("the tcgen05 attention needs an even head count");
  if (!make_map_box(&P.a_qkv, qkv, kMapBf16, 3 * P.cfg.d_model, P.cap_rows, 128, attn_block_rows(n_entities)))
    return st_rt("cuTensorMapEncodeTiled failed");
  // device scratch: error word, offsets, row -> slot map
  int* buf = nullptr;
  OW_TRY(cudaMalloc(&buf, (static_cast<size_t>(batch) + 2 + P.cap_rows) * sizeof(int)));
  P.err = buf;
  P.offsets = buf + 1;
  P.row_slot = buf + 2 + batch;
  P.qkv = const_cast<void*>(qkv);
  P.attn = out;
  cudaError_t e = cudaMemsetAsync(P.err, 0, sizeof(int), P.stream);
  if (e == cudaSuccess) {
    scan_counts_kernel<<<1, 1024, 0, P.stream>>>(counts, batch, n_entities, P.offsets, P.err);
    fill_row_slot_kernel<<<std::min(batch, 4 * P.num_sms), 128, 0, P.stream>>>(P.offsets, batch, n_entities,
                                                                                P.row_slot);
    e = cudaGetLastError();
  }

  if (e == cudaSuccess) e = launch_attention(P, batch);
  int herr = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, P.err, sizeof(int), cudaMemcpyDeviceToHost, P.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(P.stream);
  cudaFree(buf);
  if (e != cudaSuccess) return st_cuda(e);
  if (herr != 0) return st_rt(device_error_message(herr));
  return st_ok();
}

OwStatus ow_policy_launches_per_forward(const OwPolicy* policy, int32_t* launches) {
  if (policy == nullptr || launches == nullptr) return st_bad("null argument");
  const auto& c = policy->cfg;
  int per_layer = c.precision == OW_PRECISION_F32 ? 7 : (c.precision == OW_PRECISION_FP8 ? 7 : 5);
  if (ffn_fused(*policy)) per_layer = 4;  // qkv, attention, out-proj, fused FFN
  *launches = 3 + per_layer * c.layers + (c.precision == OW_PRECISION_F32 ? 0 : 1);  // scan, embed, blocks, heads(+finalize)
  return st_ok();
}

void ow_policy_destroy(OwPolicy* policy) { release(policy); }

}  // extern "C"
