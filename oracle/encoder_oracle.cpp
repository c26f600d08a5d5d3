// CPU oracle for the engine's state encoder.
//
// TEST INFRASTRUCTURE ONLY: called by tests and the bench's CPU-baseline leg
// as the checker; the product library never uses it.
//
// Restates, step for step and in the reference's f32 arithmetic:
//   encode_state            crates/orbit-wars-core/src/encoder.rs:37-125
//   comet_order / fill_row  encoder.rs:127-165
//   position / production / velocity normalisation  encoder.rs:167-177
//   owner_class_for_planet  encoder.rs:179-208
//   ship_log_percent        crates/orbit-wars-core/src/scaler.rs:3-12
//   Planet::distance_squared_to  crates/orbit-wars-core/src/types.rs:19-23
//   RowFeature::empty / absent_on_map  types.rs:48-72
//   AgentConfig::validate (the fields read here)  config.rs:335-377
// The sorts are the reference's stable sorts under f32::total_cmp. Pinned by
// the reference's own encoder and scaler tests (encoder.rs:210-324,
// scaler.rs:14-37), restated in tests/test_encoder.py.
//
// Besides the rows it writes, per row, the planet id (-1 for none), flags
// (1 = the current planet belongs to the player, 2 = the id is on no current
// planet) and the current planet's ships, as the device encoder does. A request
// that fails gets empty rows and its EncodeError code (1..4 in declaration
// order, encoder.rs:29-35).

// Rust evaluates a * b + c as two rounded operations; keep GCC from fusing them.
#pragma GCC optimize("fp-contract=off")

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr size_t kMaxRows = 64;  // config.rs MAX_ROWS
constexpr size_t kFeatures = 7;
constexpr int kOk = 0, kInvalidConfig = 1, kInvalidOwnerClass = 2, kMissingHome = 3, kRowOverflow = 4;

}  // namespace

extern "C" {

// types.rs:6-16
struct OwoPlanet {
  int32_t id;
  int32_t owner;
  float x, y, radius, ships, production, velocity_x, velocity_y;
};

// The AgentConfig fields the encoder reads, in the device ABI's layout.
struct OwoEncoderConfig {
  size_t max_rows, initial_planet_slots, comet_slots, padding_slots;
  float ship_log_pivot, ship_log_cap;
  size_t max_players;
  float owner_class_own, owner_class_enemy_1, owner_class_enemy_2, owner_class_enemy_3;
  float owner_class_neutral, owner_class_empty, owner_class_absent_on_map;
  float board_size, fleet_speed_max;
};

}  // extern "C"

namespace {

using Cfg = OwoEncoderConfig;

bool validate(const Cfg& c) {
  if (c.max_rows != c.initial_planet_slots + c.comet_slots + c.padding_slots) return false;
  if (c.max_rows == 0 || c.initial_planet_slots == 0 || c.max_rows > kMaxRows) return false;
  if (!(c.ship_log_pivot > 0.0f && c.ship_log_cap > c.ship_log_pivot)) return false;
  if (c.max_players != 4) return false;
  const float cls[7] = {c.owner_class_own,     c.owner_class_enemy_1, c.owner_class_enemy_2, c.owner_class_enemy_3,
                        c.owner_class_neutral, c.owner_class_empty,   c.owner_class_absent_on_map};
  for (int i = 0; i < 7; ++i) {
    if (!std::isfinite(cls[i])) return false;
    for (int j = i + 1; j < 7; ++j)
      if (cls[i] == cls[j]) return false;
  }
  if (!(std::isfinite(c.board_size) && c.board_size > 0.0f)) return false;
  return c.fleet_speed_max >= 1.0f;
}

float dist2(const OwoPlanet& a, const OwoPlanet& b) {
  const float dx = a.x - b.x;
  const float dy = a.y - b.y;
  return dx * dx + dy * dy;
}

// f32::total_cmp(a, b) == Less
bool total_less(float a, float b) {
  int32_t x, y;
  std::memcpy(&x, &a, 4);
  std::memcpy(&y, &b, 4);
  x ^= static_cast<int32_t>(static_cast<uint32_t>(x >> 31) >> 1);
  y ^= static_cast<int32_t>(static_cast<uint32_t>(y >> 31) >> 1);
  return x < y;
}

float clamp_f(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }  // f32::clamp

float ship_log_percent(float ships, const Cfg& c) {
  const float s = std::fmax(ships, 0.0f);  // f32::max: NaN -> 0
  if (s <= c.ship_log_pivot) return 0.9f * std::log(1.0f + s) / std::log(1.0f + c.ship_log_pivot);
  const float upper = std::log(s / c.ship_log_pivot) / std::log(c.ship_log_cap / c.ship_log_pivot);
  return 0.9f + 0.1f * clamp_f(upper, 0.0f, 1.0f);
}

bool owner_class(int32_t owner, int32_t player, const Cfg& c, float* out) {
  if (owner < 0) { *out = c.owner_class_neutral; return true; }
  if (owner == player) { *out = c.owner_class_own; return true; }
  if (player < 0 || static_cast<size_t>(owner) >= c.max_players || static_cast<size_t>(player) >= c.max_players)
    return false;
  int slot = -1, pos = 0;
  for (int32_t cand = 0; cand < static_cast<int32_t>(c.max_players); ++cand) {
    if (cand == player) continue;
    if (cand == owner) { slot = pos; break; }
    ++pos;
  }
  const float classes[3] = {c.owner_class_enemy_1, c.owner_class_enemy_2, c.owner_class_enemy_3};
  if (slot < 0 || slot > 2) return false;
  *out = classes[slot];
  return true;
}

struct Rows {
  float* rows;
  int32_t* ids;
  uint8_t* flags;
  float* ships;
};

int fill_row(Rows& o, size_t& next_row, int32_t planet_id, const OwoPlanet* planets, size_t np, int32_t player,
             const Cfg& c) {
  if (next_row >= c.max_rows) return kRowOverflow;
  o.ids[next_row] = planet_id;
  float* f = o.rows + next_row * kFeatures;
  const OwoPlanet* cur = nullptr;
  for (size_t i = 0; i < np; ++i)
    if (planets[i].id == planet_id) { cur = &planets[i]; break; }
  if (cur != nullptr) {
    if (!owner_class(cur->owner, player, c, &f[0])) return kInvalidOwnerClass;
    f[1] = ship_log_percent(cur->ships, c);
    f[2] = cur->x / c.board_size;
    f[3] = cur->y / c.board_size;
    f[4] = clamp_f(cur->production / 5.0f, 0.0f, 1.0f);
    f[5] = clamp_f(cur->velocity_x / c.fleet_speed_max, -1.0f, 1.0f);
    f[6] = clamp_f(cur->velocity_y / c.fleet_speed_max, -1.0f, 1.0f);
    o.flags[next_row] = cur->owner == player ? 1 : 0;
    o.ships[next_row] = cur->ships;
  } else {
    f[0] = c.owner_class_absent_on_map;
    for (size_t k = 1; k < kFeatures; ++k) f[k] = 0.0f;
    o.flags[next_row] = 2;
    o.ships[next_row] = 0.0f;
  }
  ++next_row;
  return kOk;
}

void empty_rows(Rows& o, const Cfg& c, size_t rows) {
  for (size_t r = 0; r < rows; ++r) {
    o.rows[r * kFeatures] = c.owner_class_empty;
    for (size_t k = 1; k < kFeatures; ++k) o.rows[r * kFeatures + k] = 0.0f;
    o.ids[r] = -1;
    o.flags[r] = 0;
    o.ships[r] = 0.0f;
  }
}

int encode(const OwoPlanet* planets, size_t np, const OwoPlanet* initial, size_t ni, const int32_t* comets, size_t nc,
           int32_t player, const Cfg& c, Rows o) {
  const size_t rows = std::min(c.max_rows, kMaxRows);
  empty_rows(o, c, rows);
  if (!validate(c)) return kInvalidConfig;
  const OwoPlanet* home = nullptr;
  for (size_t i = 0; i < np; ++i)
    if (planets[i].owner == player) { home = &planets[i]; break; }
  if (home == nullptr) return kMissingHome;
  size_t next_row = 0;
  int e = fill_row(o, next_row, home->id, planets, np, player, c);
  if (e != kOk) return e;

  std::vector<OwoPlanet> ordered_initial;
  for (size_t j = 0; j < ni; ++j)
    if (initial[j].id != home->id) ordered_initial.push_back(initial[j]);
  std::stable_sort(ordered_initial.begin(), ordered_initial.end(), [&](const OwoPlanet& a, const OwoPlanet& b) {
    return total_less(dist2(a, *home), dist2(b, *home));
  });
  const size_t take = c.initial_planet_slots > 0 ? c.initial_planet_slots - 1 : 0;
  for (size_t k = 0; k < ordered_initial.size() && k < take; ++k)
    if ((e = fill_row(o, next_row, ordered_initial[k].id, planets, np, player, c)) != kOk) return e;

  next_row = c.initial_planet_slots;
  auto comet_order = [&](int32_t id) {
    for (size_t k = 0; k < nc; ++k)
      if (comets[k] == id) return k;
    return nc;
  };
  std::vector<OwoPlanet> ordered_comets;
  for (size_t i = 0; i < np; ++i)
    if (comet_order(planets[i].id) < nc) ordered_comets.push_back(planets[i]);
  std::stable_sort(ordered_comets.begin(), ordered_comets.end(), [&](const OwoPlanet& a, const OwoPlanet& b) {
    const size_t oa = comet_order(a.id), ob = comet_order(b.id);
    if (oa != ob) return oa < ob;
    return total_less(dist2(a, *home), dist2(b, *home));
  });
  for (size_t k = 0; k < ordered_comets.size() && k < c.comet_slots; ++k)
    if ((e = fill_row(o, next_row, ordered_comets[k].id, planets, np, player, c)) != kOk) return e;
  return kOk;
}

}  // namespace

extern "C" {

// One request: rows [max_rows][7], ids / flags / ships [max_rows]; returns the
// EncodeError code (0 = encoded).
int owo_encode_state(const OwoPlanet* planets, size_t np, const OwoPlanet* initial, size_t ni, const int32_t* comets,
                     size_t nc, int32_t player, const OwoEncoderConfig* c, float* rows, int32_t* ids, uint8_t* flags,
                     float* ships) {
  Rows o{rows, ids, flags, ships};
  const int r = encode(planets, np, initial, ni, comets, nc, player, *c, o);
  if (r != kOk) empty_rows(o, *c, std::min(c->max_rows, kMaxRows));
  return r;
}

// A batch in the device ABI's CSR form (comets / comet_offsets may be NULL),
// requests spread over `threads` OpenMP threads (0 = all).
void owo_encode_batch(const OwoPlanet* planets, const size_t* p_off, const OwoPlanet* initial, const size_t* i_off,
                      const int32_t* comets, const size_t* c_off, const uint32_t* req_game,
                      const int32_t* req_player, size_t n, const OwoEncoderConfig* c, float* rows, int32_t* ids,
                      uint8_t* flags, float* ships, int32_t* errors, int threads) {
  const size_t R = c->max_rows <= kMaxRows ? c->max_rows : kMaxRows;
#ifdef _OPENMP
  const int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 16) num_threads(nt)
#endif
  for (long long r = 0; r < static_cast<long long>(n); ++r) {
    const uint32_t g = req_game[r];
    Rows o{rows + r * R * kFeatures, ids + r * R, flags + r * R, ships + r * R};
    const size_t nc = comets != nullptr ? c_off[g + 1] - c_off[g] : 0;
    int e = encode(planets + p_off[g], p_off[g + 1] - p_off[g], initial + i_off[g], i_off[g + 1] - i_off[g],
                   comets != nullptr ? comets + c_off[g] : nullptr, nc, req_player[r], *c, o);
    if (e != kOk) empty_rows(o, *c, R);
    errors[r] = e;
  }
  (void)threads;
}

}  // extern "C"
