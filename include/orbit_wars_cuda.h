/* Drop-in replacement for the reference engine's GPU ABI.
 *
 * Same symbols, struct layouts, argument meaning and status convention as
 * native/cuda/orbit_wars_cuda.h:9-92 of TryDotAtwo/Orbit-Wars-2D-Transformer,
 * so the engine's dlopen binding (crates/orbit-wars-trainer/src/cuda_true2d.rs:
 * 360-451, RTLD_NOW, five symbols) loads this library unchanged through
 * ORBIT_WARS_CUDA_LIB_PATH. Implementation: sm_100a kernels in
 * orbit-wars-2d-transformer_b200/csrc/orbit_wars_true2d.cu.
 *
 * Status: code 0 OK, 1 BAD_ARGUMENT, 2 RUNTIME_ERROR; message is a static
 * string the caller does not free. All buffers are host buffers unless noted;
 * calls are synchronous and use device 0, like the reference.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* orbit_wars_cuda.h:9-12 */
typedef struct OrbitWarsCudaStatus {
  int code;
  const char* message;
} OrbitWarsCudaStatus;

/* orbit_wars_cuda.h:14-19: legacy TrainableTransformer shape */
typedef struct OrbitWarsCudaTransformerShape {
  size_t layer_count;
  size_t d_model;
  size_t head_count;
  size_t row_count;
} OrbitWarsCudaTransformerShape;

/* orbit_wars_cuda.h:21-25: True2D shape */
typedef struct OrbitWarsCudaTrue2DShape {
  size_t layer_count;
  size_t row_count;
  size_t head_count;
} OrbitWarsCudaTrue2DShape;

/* orbit_wars_cuda.h:27-35 */
typedef struct OrbitWarsCudaTrue2DTrainingConfig {
  size_t batch_sample_count;
  float learning_rate;
  float reward_normalizer;
  float send_threshold;
  float owner_class_own;
  float owner_class_empty;
  float owner_class_absent_on_map;
} OrbitWarsCudaTrue2DTrainingConfig;

/* orbit_wars_cuda.h:37; .cu:2438-2448 -- OK when a CUDA device is visible. */
OrbitWarsCudaStatus orbit_wars_cuda_status(void);

/* orbit_wars_cuda.h:39-44; .cu:2450-2466 -- device-pointer copy of
 * games x rows x features floats. */
OrbitWarsCudaStatus orbit_wars_cuda_encode_identity_batch(
    const float* input_rows,
    float* output_rows,
    size_t game_count,
    size_t row_count,
    size_t feature_count);

/* orbit_wars_cuda.h:46-51; .cu:2468-2582 -- legacy TrainableTransformer
 * (crates/orbit-wars-core/src/model.rs:210-301). Input games x rows x 2,
 * output games x rows x 2 (target, send). The reference copied back 24
 * floats per row into a 2-per-row buffer; this one writes exactly 2. */
OrbitWarsCudaStatus orbit_wars_cuda_trainable_forward(
    const float* input_rows,
    const float* weights,
    float* output_rows,
    size_t game_count,
    OrbitWarsCudaTransformerShape shape);

/* orbit_wars_cuda.h:53-58; .cu:3332-3483 -- one True2D model
 * (true2d_model.rs:197-283). Input games x rows x 7, output games x rows x 24. */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward(
    const float* input_rows,
    const float* weights,
    float* output_rows,
    size_t game_count,
    OrbitWarsCudaTrue2DShape shape);

/* orbit_wars_cuda.h:60-67; .cu:2738-2770 -- request r uses model
 * model_indices[r] of all_weights (models back to back). Leaves the
 * population resident for ..._forward_many_resident. */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward_many(
    const float* input_rows,
    const size_t* model_indices,
    const float* all_weights,
    float* output_rows,
    size_t request_count,
    size_t model_count,
    OrbitWarsCudaTrue2DShape shape);

/* orbit_wars_cuda.h:69-73; .cu:2772-2800 -- uploads a population into the
 * persistent device workspace sized for request_capacity requests. */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_upload_population(
    const float* all_weights,
    size_t model_count,
    size_t request_capacity,
    OrbitWarsCudaTrue2DShape shape);

/* orbit_wars_cuda.h:75-80; .cu:2802-2821 -- forward on the resident
 * population (errors when none is loaded, the shape differs or the request
 * count exceeds the uploaded capacity). */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward_many_resident(
    const float* input_rows,
    const size_t* model_indices,
    float* output_rows,
    size_t request_count,
    OrbitWarsCudaTrue2DShape shape);

/* orbit_wars_cuda.h:82-92; .cu:2823-3330 -- one full-batch SGD step per
 * model: all_weights (model_count x weight count, host buffer) is updated in
 * place with w -= learning_rate * (sum over the model's samples of the loss
 * gradient) / (the model's sample count). Per sample: input rows (rows x 7),
 * the outputs it produced (rows x 24), an int reward and rows x 12 target
 * action rewards. Samples are processed in chunks of at most
 * batch_sample_count; the result does not depend on the chunking beyond f32
 * rounding. BAD_ARGUMENT "invalid true2d training batch" or "true2d training
 * model index out of range" as the reference. */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_train_full_attention(
    const float* input_rows,
    const float* output_rows,
    const int* rewards,
    const float* target_action_rewards,
    const size_t* model_indices,
    float* all_weights,
    size_t sample_count,
    size_t model_count,
    OrbitWarsCudaTrue2DShape shape,
    OrbitWarsCudaTrue2DTrainingConfig training_config);

/* Allocation-free forward -- no counterpart in the reference ABI.
 * For callers that cannot allocate device memory: an engine whose device
 * memory is all reserved by its own pool or budget (a cudaMalloc would fail or
 * fragment it), or a self-play loop that must not pay the implicit device-wide
 * synchronisation of cudaMalloc/cudaFree between turns. Same math as
 * orbit_wars_cuda_true2d_forward for one model, but input_rows
 * (games x rows x 7), weights (the reference layout) and output_rows
 * (games x rows x 24) are DEVICE pointers, the call is enqueued on `stream`
 * (NULL: the legacy default stream) and returns without waiting.
 * Scratch is a fixed 1 MiB device array inside the library, held by every GPU
 * that loads it until exit: game_count * (row_count^2 + 1) must be <= 262,080
 * (63 requests at 64 rows), else BAD_ARGUMENT. Every call looks the array's
 * device address up again (so a device reset leaves nothing stale); the first
 * call on a device also loads the library's device code, so make that first
 * call before any stream capture. The three kernels of this path raise no
 * device-side error (with one model there is no model index to check), so
 * the returned status, which carries launch errors, is the whole result; a
 * fault during execution surfaces at the caller's next synchronisation.
 * All calls share the array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller. */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_forward_noalloc(
    const float* input_rows,
    const float* weights,
    float* output_rows,
    size_t game_count,
    OrbitWarsCudaTrue2DShape shape,
    void* stream);

/* Row flags written by the device encoder and read by the device decode, one
 * byte per (request, row). */
#define ORBIT_WARS_ROW_OWNED 1u  /* the row's planet belongs to the player */
#define ORBIT_WARS_ROW_ABSENT 2u /* the row names a planet no longer on the map */

/* Forward + decode on the device -- no counterpart in the reference ABI.
 * Runs ..._forward_many_resident on the resident population, then the part of
 * the engine's decoder that needs no geometry (crates/orbit-wars-core/src/
 * decoder.rs:85-124, target_row_from_fraction :457-461) before anything is
 * copied back. Per request r and row s (request_count x row_count each):
 * row_planet_ids[r][s] (-1 = no planet, the encoder's NO_PLANET_ID),
 * row_flags[r][s] (ORBIT_WARS_ROW_OWNED when the row's planet belongs to the
 * player; ORBIT_WARS_ROW_ABSENT when it is not on the map -- the decoder's
 * planet_by_id misses, decoder.rs:93 and :112), source_ships[r][s] (its ships).
 * A source row is decoded when it is active, owned and not absent. Per
 * (r, s, target slot a), 12 slots: target_rows = the target row (-1 when the
 * decoder skips the pair: the source row itself, an absent target, send <= 0,
 * or fewer than one ship) and ship_counts = floor(ships * clamp(send_fraction,
 * 0, 1)) (0 when skipped). The engine then runs only its geometry (intercept
 * angles) for the pairs with target_rows >= 0. output_rows (request_count x
 * row_count x 24, the raw outputs) may be NULL. A non-finite output of a
 * decoded source returns RUNTIME_ERROR "non-finite model output", as the
 * decoder's NonFiniteModelOutput. */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_decode_many_resident(
    const float* input_rows,
    const size_t* model_indices,
    const int32_t* row_planet_ids,
    const uint8_t* row_flags,
    const float* source_ships,
    int32_t* target_rows,
    int32_t* ship_counts,
    float* output_rows,
    size_t request_count,
    OrbitWarsCudaTrue2DShape shape);

/* The same decode on outputs the caller already has (host buffers:
 * output_rows request_count x row_count x 24, the rest as above). */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_decode_outputs(
    const float* output_rows,
    const int32_t* row_planet_ids,
    const uint8_t* row_flags,
    const float* source_ships,
    int32_t* target_rows,
    int32_t* ship_counts,
    size_t request_count,
    size_t row_count);

/* ---- device encoder -- no counterpart in the reference ABI ----------------
 * crates/orbit-wars-core/src/encoder.rs:37-208 (encode_state) on the device,
 * for a batch of requests over a batch of game states. */

/* crates/orbit-wars-core/src/types.rs:6-16, field for field (a #[repr(C)]
 * Planet on the engine side has this layout: 36 bytes). */
typedef struct OrbitWarsPlanet {
  int32_t id;
  int32_t owner;
  float x;
  float y;
  float radius;
  float ships;
  float production;
  float velocity_x;
  float velocity_y;
} OrbitWarsPlanet;

/* The AgentConfig fields encode_state reads (crates/orbit-wars-core/src/
 * config.rs:115-140); orbit_wars_encoder_config_default fills the defaults
 * of config.rs:1-19. Checked as AgentConfig::validate checks them
 * (config.rs:335-377): max_rows = initial + comet + padding slots, max_rows
 * and initial slots positive, 0 < pivot < cap, max_players = 4, the seven
 * owner classes finite and distinct, board size finite and positive,
 * fleet_speed_max >= 1; and here also max_rows <= 64 (the model's rows). */
typedef struct OrbitWarsEncoderConfig {
  size_t max_rows;
  size_t initial_planet_slots;
  size_t comet_slots;
  size_t padding_slots;
  float ship_log_pivot;
  float ship_log_cap;
  size_t max_players;
  float owner_class_own;
  float owner_class_enemy_1;
  float owner_class_enemy_2;
  float owner_class_enemy_3;
  float owner_class_neutral;
  float owner_class_empty;
  float owner_class_absent_on_map;
  float board_size;
  float fleet_speed_max;
} OrbitWarsEncoderConfig;

void orbit_wars_encoder_config_default(OrbitWarsEncoderConfig* out);

/* Game states in CSR form (host buffers): game g's current planets are
 * planets[planet_offsets[g] .. planet_offsets[g + 1]), its initial planets
 * initial_planets[initial_offsets[g] ..), its comet planet ids
 * comet_planet_ids[comet_offsets[g] ..); each offsets array has game_count + 1
 * entries starting at 0. comet_planet_ids and comet_offsets may both be NULL
 * (no comets, as the trainer encodes: crates/orbit-wars-trainer/src/
 * main.rs:3633-3639). */
typedef struct OrbitWarsGameBatch {
  const OrbitWarsPlanet* planets;
  const size_t* planet_offsets;
  const OrbitWarsPlanet* initial_planets;
  const size_t* initial_offsets;
  const int32_t* comet_planet_ids;
  const size_t* comet_offsets;
  size_t game_count;
} OrbitWarsGameBatch;

/* encode_errors values: 0 = encoded; then EncodeError (encoder.rs:29-35) in
 * declaration order. */
#define ORBIT_WARS_ENCODE_OK 0
#define ORBIT_WARS_ENCODE_INVALID_CONFIG 1
#define ORBIT_WARS_ENCODE_INVALID_OWNER_CLASS 2
#define ORBIT_WARS_ENCODE_MISSING_HOME_PLANET 3
#define ORBIT_WARS_ENCODE_ROW_OVERFLOW 4

/* Encodes request r = encode_state(game request_games[r]'s planets, initial
 * planets and comet ids, request_players[r], config) for every request.
 * Outputs (host buffers, request_count x max_rows each): input_rows x 7 floats
 * in the order pack_rows_into writes them (crates/orbit-wars-trainer/src/
 * cuda_true2d.rs:469-487), ready for ..._forward_many_resident;
 * row_planet_ids; row_flags (ORBIT_WARS_ROW_*); row_ships (the row planet's
 * current ships, 0 for empty and absent rows; may be NULL); encode_errors
 * (one per request; may be NULL). A request that fails gets empty rows. When
 * any request fails the call returns BAD_ARGUMENT naming the first failing
 * request's error, after filling every output. A bad config returns
 * BAD_ARGUMENT "invalid encoder config" (EncodeError::InvalidConfig). */
OrbitWarsCudaStatus orbit_wars_cuda_encode_states(
    const OrbitWarsGameBatch* games,
    const uint32_t* request_games,
    const int32_t* request_players,
    size_t request_count,
    const OrbitWarsEncoderConfig* config,
    float* input_rows,
    int32_t* row_planet_ids,
    uint8_t* row_flags,
    float* row_ships,
    int32_t* encode_errors);

/* One policy turn on the device: encode (as ..._encode_states), forward on the
 * resident population (model_indices per request, as ..._forward_many_resident)
 * and decode (as ..._decode_many_resident), with only the game states going up
 * and row_planet_ids (request_count x row_count) plus target_rows / ship_counts
 * (request_count x row_count x 12) coming back. input_rows (request_count x
 * row_count x 7) and output_rows (x 24) may be NULL; when given they receive
 * the encoded rows and the raw outputs. config.max_rows must equal
 * shape.row_count. Errors as the three calls it fuses. */
OrbitWarsCudaStatus orbit_wars_cuda_true2d_play_many_resident(
    const OrbitWarsGameBatch* games,
    const uint32_t* request_games,
    const int32_t* request_players,
    const size_t* model_indices,
    size_t request_count,
    const OrbitWarsEncoderConfig* config,
    int32_t* row_planet_ids,
    int32_t* target_rows,
    int32_t* ship_counts,
    int32_t* encode_errors,
    float* input_rows,
    float* output_rows,
    OrbitWarsCudaTrue2DShape shape);

/* Measured rate of the GPU's special-function (MUFU) pipe -- no counterpart in
 * the reference ABI; the roofline of the True2D matrix layers, whose tanh and
 * sigmoid are one ex2.approx and one rcp.approx each. op 0 = ex2.approx,
 * 1 = rcp.approx. One CTA of 1024 threads per SM runs 8 independent chains
 * per thread; *ops_per_second is event-timed, *ops_per_clock_per_sm comes
 * from each CTA's clock64 span, *sm_clock_mhz is their ratio. Allocates and
 * frees its small buffers (a measurement call, not for a hot loop). */
OrbitWarsCudaStatus orbit_wars_cuda_mufu_rate(int32_t op, double* ops_per_second, double* ops_per_clock_per_sm,
                                              double* sm_clock_mhz);

/* Device timing of the True2D forwards -- no counterpart in the reference ABI;
 * for benchmarks. profile_begin arms CUDA events around each kernel of the next
 * `max_calls` calls of ..._true2d_forward / _forward_many / _forward_many_resident /
 * _decode_many_resident / _play_many_resident (encoder, forward kernels and
 * decode; events only, no extra synchronisation). profile_end waits for the library's
 * stream and returns, per kernel name, the launches and the summed
 * event-to-event milliseconds; names are static strings. */
typedef struct OrbitWarsCudaKernelTiming {
  const char* name;
  int32_t launches;
  float total_ms;
} OrbitWarsCudaKernelTiming;

OrbitWarsCudaStatus orbit_wars_cuda_true2d_profile_begin(int32_t max_calls);

OrbitWarsCudaStatus orbit_wars_cuda_true2d_profile_end(
    OrbitWarsCudaKernelTiming* out,
    int32_t capacity,
    int32_t* count);

#ifdef __cplusplus
}
#endif
