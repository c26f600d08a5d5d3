// Device encoder: encode_state (crates/orbit-wars-core/src/encoder.rs:37-208)
// for a batch of requests over a batch of game states.
//
// One warp per request. Per request the warp
//   1. finds the home planet, the first current planet owned by the player
//      (encoder.rs:46-49; none -> MissingHomePlanet);
//   2. ranks the initial planets other than the home (:65-74) by squared
//      distance to the home, compared with f32::total_cmp, ties by input
//      position (the stable sort): rank k < initial_slots - 1 goes to row 1 + k;
//   3. ranks the current planets whose id is in the comet list (:93-107) by
//      (first position in the comet list, total_cmp distance, input position):
//      rank k < comet_slots goes to row initial_slots + k;
//   4. fills every row (fill_row, :134-165): the first current planet with the
//      row's id gives owner class (:179-208), ship_log_percent
//      (crates/orbit-wars-core/src/scaler.rs:3-12), position / board size,
//      clamp(production / 5, 0, 1), clamp(velocity / fleet_speed_max, -1, 1);
//      a row whose id is on no current planet is absent_on_map, a row with no id
//      is empty (types.rs:48-72).
// Ranks replace the sorts: every key is unique (the input position is part of
// it), so rank = the number of smaller keys, computed by each lane for its
// elements against the warp's keys in shared memory.
//
// Errors follow the reference's order: the first row, in fill order, whose
// owner class is invalid gives InvalidOwnerClass; a row past max_rows gives
// RowOverflow (unreachable under a validated config, kept for parity).
//
// Arithmetic is the reference's f32 arithmetic, operation for operation: the
// products and sums use the _rn intrinsics so that nothing contracts into an
// FMA. ln is computed in double and rounded to f32 (correctly rounded but for
// double-rounding ties), so ship_log_percent can differ from a platform logf
// in the last bit.
#pragma once

#include <cstdint>

namespace enc {

constexpr int kMaxRows = 64;  // config.rs MAX_ROWS: EncodedState holds 64 rows
constexpr int kFeatures = 7;
constexpr int kWarps = 4;     // requests per CTA at most (fewer for games whose shared memory needs more)
constexpr uint64_t kNoKey = ~0ull;

constexpr int kOk = 0, kInvalidConfig = 1, kInvalidOwnerClass = 2, kMissingHome = 3, kRowOverflow = 4;
constexpr uint8_t kRowOwned = 1, kRowAbsent = 2;

// The AgentConfig values the kernel reads, as kernel parameter.
struct Cfg {
  int max_rows, init_slots, comet_slots, max_players;
  float pivot, cap;
  float own, enemy1, enemy2, enemy3, neutral, empty, absent;
  float board, speed;
};

// Planet as the engine lays it out (types.rs:6-16), 36 bytes.
struct Planet {
  int32_t id, owner;
  float x, y, radius, ships, production, vx, vy;
};
static_assert(sizeof(Planet) == 36, "planet layout");

struct Batch {
  const Planet* planets;
  const unsigned long long* p_off;
  const Planet* initial;
  const unsigned long long* i_off;
  const int32_t* comets;            // nullptr: no comet lists
  const unsigned long long* c_off;
  const uint32_t* req_game;
  const int32_t* req_player;
};

struct Out {
  float* rows;       // [n][max_rows][7]
  int32_t* ids;      // [n][max_rows]
  uint8_t* flags;    // [n][max_rows]
  float* ships;      // [n][max_rows] or nullptr
  int32_t* errors;   // [n]
};

// Shared memory per warp for games of up to max_p current and max_i initial planets.
__host__ __device__ inline size_t warp_smem_bytes(int max_p, int max_i) {
  auto up16 = [](size_t b) { return (b + 15) & ~size_t(15); };
  return up16(size_t(max_i) * 8) + up16(size_t(max_p) * 8) + up16(size_t(max_p) * 4) + up16(kMaxRows * 4) +
         up16(kMaxRows * kFeatures * 4);
}

// f32::total_cmp as an unsigned key: the IEEE-754 totalOrder predicate
// (-NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN).
__device__ __forceinline__ uint32_t total_order_key(float v) {
  const int32_t b = __float_as_int(v);
  const int32_t k = b ^ static_cast<int32_t>(static_cast<uint32_t>(b >> 31) >> 1);
  return static_cast<uint32_t>(k) ^ 0x80000000u;
}

// The NaN an x86-64 SSE operation a (op) b returns, which decides where
// f32::total_cmp puts a NaN distance in the reference's sorts: a NaN operand
// propagates, quieted, the first operand first; an invalid operation on
// numbers gives the default NaN 0xFFC00000, whose sign bit sorts it before
// every number. (The GPU's own NaN is 0x7FFFFFFF whatever the operands.)
__device__ __forceinline__ float x86_nan(float a, float b, float r) {
  if (isnan(a)) return __int_as_float(__float_as_int(a) | 0x00400000);
  if (isnan(b)) return __int_as_float(__float_as_int(b) | 0x00400000);
  if (isnan(r)) return __int_as_float(static_cast<int>(0xFFC00000u));
  return r;
}

// Planet::distance_squared_to (types.rs:19-23), unfused, with x86 NaNs.
__device__ __forceinline__ float dist2(float ax, float ay, float bx, float by) {
  const float dx = x86_nan(ax, bx, __fsub_rn(ax, bx)), dy = x86_nan(ay, by, __fsub_rn(ay, by));
  const float xx = x86_nan(dx, dx, __fmul_rn(dx, dx)), yy = x86_nan(dy, dy, __fmul_rn(dy, dy));
  return x86_nan(xx, yy, __fadd_rn(xx, yy));
}

__device__ __forceinline__ float ln(float v) { return static_cast<float>(log(static_cast<double>(v))); }

// f32::clamp: NaN passes through.
__device__ __forceinline__ float clamp_f(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// scaler.rs:3-12
__device__ __forceinline__ float ship_log_percent(float ships, const Cfg& c) {
  const float s = fmaxf(ships, 0.0f);  // f32::max: NaN -> 0
  if (s <= c.pivot) return __fdiv_rn(__fmul_rn(0.9f, ln(__fadd_rn(1.0f, s))), ln(__fadd_rn(1.0f, c.pivot)));
  const float upper = __fdiv_rn(ln(__fdiv_rn(s, c.pivot)), ln(__fdiv_rn(c.cap, c.pivot)));
  return __fadd_rn(0.9f, __fmul_rn(0.1f, clamp_f(upper, 0.0f, 1.0f)));
}

// encoder.rs:179-208; false = InvalidOwnerClass.
__device__ __forceinline__ bool owner_class(int owner, int player, const Cfg& c, float* cls) {
  if (owner < 0) { *cls = c.neutral; return true; }
  if (owner == player) { *cls = c.own; return true; }
  if (player < 0 || owner >= c.max_players || player >= c.max_players) return false;
  const int slot = owner < player ? owner : owner - 1;  // position among 0..max_players without the player
  if (slot > 2) return false;
  *cls = slot == 0 ? c.enemy1 : (slot == 1 ? c.enemy2 : c.enemy3);
  return true;
}

// CTA of `warps` warps (blockDim.x = 32 * warps), one request per warp.
__global__ void __launch_bounds__(kWarps * 32) encode_kernel(Batch b, Cfg c, int n, int max_p, int max_i, int warps,
                                                             Out o) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * warps + warp;
  if (r >= n) return;  // whole warps leave together
  unsigned char* w = smem + warp * warp_smem_bytes(max_p, max_i);
  auto up16 = [](size_t v) { return (v + 15) & ~size_t(15); };
  uint64_t* ikey = reinterpret_cast<uint64_t*>(w);
  uint64_t* ckey = reinterpret_cast<uint64_t*>(w + up16(size_t(max_i) * 8));
  int32_t* pid = reinterpret_cast<int32_t*>(w + up16(size_t(max_i) * 8) + up16(size_t(max_p) * 8));
  int32_t* row_id = pid + up16(size_t(max_p) * 4) / 4;
  float* stage = reinterpret_cast<float*>(row_id + kMaxRows);

  const uint32_t g = b.req_game[r];
  const int player = b.req_player[r];
  const long long p0 = static_cast<long long>(b.p_off[g]);
  const int np = static_cast<int>(b.p_off[g + 1] - b.p_off[g]);
  const long long i0 = static_cast<long long>(b.i_off[g]);
  const int ni = static_cast<int>(b.i_off[g + 1] - b.i_off[g]);
  long long c0 = 0;
  int nc = 0;
  if (b.comets != nullptr) {
    c0 = static_cast<long long>(b.c_off[g]);
    nc = static_cast<int>(b.c_off[g + 1] - b.c_off[g]);
  }
  const Planet* P = b.planets + p0;
  const Planet* I = b.initial + i0;

  for (int i = lane; i < np; i += 32) pid[i] = P[i].id;
  row_id[lane] = -1;
  row_id[lane + 32] = -1;

  // 1. home planet
  int home = -1;
  for (int base = 0; base < np && home < 0; base += 32) {
    const int i = base + lane;
    const unsigned m = __ballot_sync(0xffffffffu, i < np && P[i].owner == player);
    if (m != 0u) home = base + __ffs(m) - 1;
  }
  int err = kOk;
  if (home < 0) {
    err = kMissingHome;
  } else {
    const int hid = P[home].id;
    const float hx = P[home].x, hy = P[home].y;
    // 2./3. keys
    for (int j = lane; j < ni; j += 32)
      ikey[j] = I[j].id == hid ? kNoKey
                               : (static_cast<uint64_t>(total_order_key(dist2(I[j].x, I[j].y, hx, hy))) << 32) |
                                     static_cast<uint64_t>(j);
    for (int i = lane; i < np; i += 32) {
      int order = -1;
      for (int k = 0; k < nc; ++k)
        if (b.comets[c0 + k] == pid[i]) { order = k; break; }
      ckey[i] = order < 0 ? kNoKey
                          : (static_cast<uint64_t>(order) << 48) |
                                (static_cast<uint64_t>(total_order_key(dist2(P[i].x, P[i].y, hx, hy))) << 16) |
                                static_cast<uint64_t>(i);
    }
    __syncwarp();
    if (lane == 0) row_id[0] = hid;
    bool overflow = false;
    for (int j = lane; j < ni; j += 32) {
      const uint64_t key = ikey[j];
      if (key == kNoKey) continue;
      int rank = 0;
      for (int k = 0; k < ni; ++k) rank += ikey[k] < key;
      if (rank < c.init_slots - 1) {
        const int row = 1 + rank;
        if (row < c.max_rows) row_id[row] = I[j].id; else overflow = true;
      }
    }
    for (int i = lane; i < np; i += 32) {
      const uint64_t key = ckey[i];
      if (key == kNoKey) continue;
      int rank = 0;
      for (int k = 0; k < np; ++k) rank += ckey[k] < key;
      if (rank < c.comet_slots) {
        const int row = c.init_slots + rank;
        if (row < c.max_rows) row_id[row] = pid[i]; else overflow = true;
      }
    }
    __syncwarp();
    // 4. fill rows lane and lane + 32
    int bad_row = kMaxRows;
    for (int row = lane; row < c.max_rows; row += 32) {
      const int q = row_id[row];
      float f[kFeatures] = {c.empty, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint8_t flag = 0;
      float ships = 0.0f;
      if (q != -1) {
        int at = -1;
        for (int i = 0; i < np; ++i)
          if (pid[i] == q) { at = i; break; }
        if (at < 0) {
          f[0] = c.absent;
          flag = kRowAbsent;
        } else {
          const Planet& p = P[at];
          if (!owner_class(p.owner, player, c, &f[0])) bad_row = min(bad_row, row);
          f[1] = ship_log_percent(p.ships, c);
          f[2] = __fdiv_rn(p.x, c.board);
          f[3] = __fdiv_rn(p.y, c.board);
          f[4] = clamp_f(__fdiv_rn(p.production, 5.0f), 0.0f, 1.0f);
          f[5] = clamp_f(__fdiv_rn(p.vx, c.speed), -1.0f, 1.0f);
          f[6] = clamp_f(__fdiv_rn(p.vy, c.speed), -1.0f, 1.0f);
          flag = p.owner == player ? kRowOwned : 0;
          ships = p.ships;
        }
      }
#pragma unroll
      for (int k = 0; k < kFeatures; ++k) stage[row * kFeatures + k] = f[k];
      const long long o_row = static_cast<long long>(r) * c.max_rows + row;
      o.flags[o_row] = flag;
      if (o.ships != nullptr) o.ships[o_row] = ships;
    }
    for (int off = 16; off > 0; off >>= 1) bad_row = min(bad_row, __shfl_xor_sync(0xffffffffu, bad_row, off));
    if (bad_row < kMaxRows) err = kInvalidOwnerClass;
    else if (__any_sync(0xffffffffu, overflow)) err = kRowOverflow;
  }
  // a failed request gets empty rows
  if (err != kOk) {
    for (int row = lane; row < c.max_rows; row += 32) {
      row_id[row] = -1;
      stage[row * kFeatures] = c.empty;
      for (int k = 1; k < kFeatures; ++k) stage[row * kFeatures + k] = 0.0f;
      const long long o_row = static_cast<long long>(r) * c.max_rows + row;
      o.flags[o_row] = 0;
      if (o.ships != nullptr) o.ships[o_row] = 0.0f;
    }
  }
  __syncwarp();
  float* rows = o.rows + static_cast<long long>(r) * c.max_rows * kFeatures;
  for (int k = lane; k < c.max_rows * kFeatures; k += 32) rows[k] = stage[k];
  for (int row = lane; row < c.max_rows; row += 32) o.ids[static_cast<long long>(r) * c.max_rows + row] = row_id[row];
  if (lane == 0) o.errors[r] = err;
}

}  // namespace enc
