/* Orbit Wars entity-encoder policy forward on NVIDIA B200 (sm_100a): C ABI.
 *
 * A batch of game states, each a padded set of N entity tokens of F
 * features plus a per-state valid count, runs through an entity embedding,
 * L pre-LN encoder blocks (masked multi-head attention + GELU FFN), per-entity
 * policy logits, a mean-pooled value head and greedy or Gumbel-max actions.
 * The math and the weight-blob layout are fixed; ow_policy_weight_count gives the blob size.
 *
 * Conventions follow the reference engine's GPU ABI
 * (native/cuda/orbit_wars_cuda.h:9-12, native/cuda/orbit_wars_cuda.cu:12-14):
 * every call returns {code, message}; code 0 = OK, 1 = BAD_ARGUMENT,
 * 2 = RUNTIME_ERROR; message is a static string the caller does not free.
 * Buffers are contiguous row-major, request x rows x features, like the
 * packed f32 batches of crates/orbit-wars-trainer/src/cuda_true2d.rs:469-487.
 *
 * The reference has no encoder policy: these symbols are new, added beside
 * the reference's orbit_wars_cuda_* symbols (orbit_wars_cuda.h) in the same
 * library. A handle is bound to one device and one stream; separate handles
 * may be used from separate threads.
 */
#ifndef OW_POLICY_H_
#define OW_POLICY_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct OwStatus {
  int code;
  const char* message;
} OwStatus;

enum { OW_STATUS_OK = 0, OW_STATUS_BAD_ARGUMENT = 1, OW_STATUS_RUNTIME_ERROR = 2 };
enum { OW_PRECISION_F32 = 0, OW_PRECISION_BF16 = 1, OW_PRECISION_FP8 = 2 };
enum { OW_DTYPE_F32 = 0, OW_DTYPE_BF16 = 1 };
enum { OW_IO_HOST = 0, OW_IO_DEVICE = 1 };

typedef struct OwPolicyConfig {
  int32_t batch_capacity; /* max states per forward call */
  int32_t n_entities;     /* N, padded entity slots per state, 1..128 */
  int32_t features;       /* F, 1..32 */
  int32_t d_model;        /* d, multiple of 32 (head_dim 32), 128..512 */
  int32_t heads;          /* d / 32 */
  int32_t ffn;            /* f, multiple of 128 */
  int32_t layers;         /* L >= 1 */
  int32_t actions;        /* P, 1..32 */
  int32_t precision;      /* OW_PRECISION_* */
  int32_t sample_actions; /* 0 greedy argmax, 1 Gumbel-max (Philox4x32-10) */
  int32_t logits_dtype;   /* OW_DTYPE_* */
  int32_t value_dtype;    /* OW_DTYPE_* */
  int32_t io;             /* OW_IO_HOST: host buffers, synchronous; OW_IO_DEVICE: device buffers, async on the stream */
} OwPolicyConfig;

typedef struct OwPolicy OwPolicy;

/* Fills *config with preset 1..5 (the five documented workloads). */
OwStatus ow_policy_preset(int preset, OwPolicyConfig* config);

/* Number of f32 weights the blob for this config holds. */
OwStatus ow_policy_weight_count(const OwPolicyConfig* config, size_t* count);

/* Creates a handle on `device`: validates the config, converts and uploads
 * the f32 weight blob (to bf16 / e4m3 + per-channel scales as the precision
 * asks), allocates the batch_capacity workspace. `stream` may be NULL (a
 * handle-owned stream is created). `weights` may be NULL (weight_count still
 * the config's count): the handle then holds zero weights, for a receiver of
 * ow_policy_broadcast_weights*. */
OwStatus ow_policy_create(const OwPolicyConfig* config, const float* weights, size_t weight_count, int device,
                          void* stream, OwPolicy** out);

/* Replaces the weights of an existing handle (same config). */
OwStatus ow_policy_set_weights(OwPolicy* policy, const float* weights, size_t weight_count);

/* One forward of `batch` states (batch <= batch_capacity).
 *   features f32 [batch, N, F]; counts int32 [batch], each in [0, N]
 *   logits [batch, N, P] (logits_dtype), value [batch] (value_dtype),
 *   actions int32 [batch, N]; any output pointer may be NULL to skip it.
 * OW_IO_HOST: host pointers; returns after the outputs are on the host.
 * OW_IO_DEVICE: device pointers; enqueued on the handle's stream, returns
 * at once (call ow_policy_synchronize to collect device-side errors). */
OwStatus ow_policy_forward(OwPolicy* policy, const float* features, const int32_t* counts, int32_t batch,
                           void* logits, void* value, int32_t* actions, uint64_t seed);

/* Pipelined host IO (host-IO handles). ow_policy_submit validates the counts,
 * enqueues the upload of `features` / `counts`, the forward and the download
 * of the outputs, and returns at once with a ticket; ow_policy_wait(ticket)
 * blocks until that submission's outputs are in the host buffers and returns
 * its status (a device-side error of that forward included). Two submissions
 * may be in flight: the uploads and downloads of one overlap the forward of
 * the other when the host buffers are pinned. The host buffers must stay
 * valid until the wait; a third submit before the older one is waited for
 * returns BAD_ARGUMENT. Not thread-safe per handle. ow_policy_forward on a
 * host-IO handle is submit + wait. A host-IO handle on the tensor-core path
 * keeps a second activation workspace and compute stream when that takes at
 * most half of the free device memory (ORBIT_WARS_LANES=1 at create turns it
 * off), so the forwards of two in-flight submissions also run at the same
 * time, filling each other's idle SMs. */
OwStatus ow_policy_submit(OwPolicy* policy, const float* features, const int32_t* counts, int32_t batch,
                          void* logits, void* value, int32_t* actions, uint64_t seed, int64_t* ticket);
OwStatus ow_policy_wait(OwPolicy* policy, int64_t ticket);

/* Waits for the handle's stream and reports any device-side error
 * (a bad count, a bounded wait that expired). */
OwStatus ow_policy_synchronize(OwPolicy* policy);

/* Device pointer and byte size of the handle's packed device weights (the
 * tensor a weight broadcast moves), for callers that run their own NCCL. */
OwStatus ow_policy_device_weights(OwPolicy* policy, void** ptr, size_t* bytes);

/* ---- Weight broadcast over NCCL (NVLink / NVSwitch).
 * A data-parallel run shards states across GPUs with no exchange on the data
 * path; the one exchange is the model. These calls move a handle's packed
 * device weight arena (the bf16 / e4m3 matrices with their scales and the f32
 * vectors the kernels read, ow_policy_device_weights) from the root rank's
 * handle into every other rank's, as one ncclBroadcast: no host round trip and
 * no re-conversion on the receivers. All ranks' handles must have the same
 * config (the arena layout is a function of the config). A receiver can be
 * created with weights == NULL (ow_policy_create): it holds zero weights
 * until the broadcast fills them. Reference counterpart: none in the ABI; the
 * nearest operation is the population upload (native/cuda/orbit_wars_cuda.cu:
 * 2772-2800), which copies weights from host memory on one device.
 * NCCL is loaded at run time: the libnccl.so.2 already in the process, else
 * $ORBIT_WARS_NCCL_LIB, else libnccl.so.2 from the loader path; without it
 * these calls return RUNTIME_ERROR. Every wait is bounded by
 * $ORBIT_WARS_COMM_TIMEOUT_S (default 120 s): a rank that does not join makes
 * the others return RUNTIME_ERROR with their communicator aborted. */
typedef struct OwComm OwComm;

/* One process per GPU: one rank calls ow_comm_unique_id (128 bytes into
 * `id`), the caller shares those bytes over its own channel, then every rank
 * calls ow_comm_init_rank with them, its rank and its device. */
OwStatus ow_comm_unique_id(void* id, size_t id_bytes);
OwStatus ow_comm_init_rank(const void* id, size_t id_bytes, int nranks, int rank, int device, OwComm** out);
/* One process driving n GPUs (distinct devices): comms[i] is rank i on devices[i]. */
OwStatus ow_comm_init_all(const int* devices, int n, OwComm** comms);
OwStatus ow_comm_info(const OwComm* comm, int* rank, int* nranks, int* device);
void ow_comm_destroy(OwComm* comm);

/* Every rank calls this with its own handle (on the communicator's device):
 * the root's weights replace the others'. Waits for the handle's forwards in
 * flight first and returns after the copy completed; *elapsed_ms (may be
 * NULL) is the broadcast's device time on this rank. */
OwStatus ow_policy_broadcast_weights_comm(OwPolicy* policy, OwComm* comm, int root, float* elapsed_ms);

/* One process, handles[i] on distinct devices: handles[0]'s weights go to
 * every other handle (a communicator over those devices is created for the
 * call and released after it). */
OwStatus ow_policy_broadcast_weights(OwPolicy** handles, int n_gpus);

/* NCCL version code of the loaded library (e.g. 22809 for 2.28.9). */
OwStatus ow_nccl_version(int* version);

/* Per-kernel device timing. ow_policy_profile_begin arms CUDA events around
 * every launch of the next `max_forwards` forwards (events only, no host
 * synchronisation); ow_policy_profile_end synchronises and returns, per
 * kernel name, the launches and the summed event-to-event milliseconds. */
typedef struct OwKernelTiming {
  const char* name;
  int32_t launches;
  float total_ms;
} OwKernelTiming;

OwStatus ow_policy_profile_begin(OwPolicy* policy, int32_t max_forwards);
OwStatus ow_policy_profile_end(OwPolicy* policy, OwKernelTiming* out, int32_t capacity, int32_t* count);

/* Kernel launches one forward issues (for launch accounting). */
OwStatus ow_policy_launches_per_forward(const OwPolicy* policy, int32_t* launches);

void ow_policy_destroy(OwPolicy* policy);

/* Test hook, not part of the forward: one tensor-core GEMM launch on device
 * buffers, out[m, n] = a[m, :] . w[n, :] + epilogue, exactly as the forward
 * issues it. precision OW_PRECISION_BF16 or _FP8 (then a_scale[m], b_scale[n]
 * dequantise); epilogue 0 bias -> bf16 out, 1 bias + GELU -> bf16 out,
 * 2 residual (f32 resid, in place) + LayerNorm -> ln_out (ln_mode 0 bf16,
 * 1 e4m3 + ln_scale, 2 f32); 3 the same with a bf16 residual (resid points at
 * bf16 values; n = 256). epilogue + 16 runs the CTA-pair kernel (cta_group::2,
 * 256-row tiles; n a multiple of 256; epilogue 0, 1 or 3). Synchronous on
 * `stream`. */
OwStatus ow_selftest_gemm(int precision, int epilogue, int m, int n, int k, const void* a, const void* w,
                          const float* bias, void* out, float* resid, const float* ln_g, const float* ln_b,
                          void* ln_out, int ln_mode, float* ln_scale, const float* a_scale, const float* b_scale,
                          void* stream);

/* Test hook, not part of the forward: one launch of the fused feed-forward
 * kernel on device buffers, as the bf16 forward issues it at d = 256:
 * x[m, d] += GELU(ln . w1^T + b1) . w2^T + b2 (f32, in place), then
 * ln_out = LayerNorm(x) * ln_g + ln_b (ln_mode 0 bf16, 2 f32). ln, w1 [f, d]
 * and w2 [d, f] are bf16; f a multiple of 128, at most 1280. Synchronous on
 * `stream`. */
OwStatus ow_selftest_ffn(int m, int d, int f, const void* ln, const void* w1, const float* b1, const void* w2,
                         const float* b2, float* x, const float* ln_g, const float* ln_b, void* ln_out, int ln_mode,
                         void* stream);

/* Test hook, not part of the forward: one launch of the bf16 masked attention
 * on device buffers, as the forward issues it. counts[batch] (device) are the
 * valid entities per state (<= n_entities); qkv is [Σcounts rows, 3 * 32 *
 * heads] bf16 in the packed layout (rows of state b after those of states < b;
 * the buffer holds batch * n_entities rows); out [rows, 32 * heads] bf16.
 * kernel 0 runs the tcgen05 kernel (S and P in tensor memory), 1 the
 * mma.sync kernel. Synchronous on `stream`. */
OwStatus ow_selftest_attention(int kernel, int batch, int n_entities, int heads, const int32_t* counts,
                               const void* qkv, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OW_POLICY_H_ */
