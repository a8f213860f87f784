/*
 * klearu_gpu.h -- C ABI of the B200 (sm_100a) SLIDE sparse-layer engine.
 *
 * This is the drop-in boundary for klearu-core's SLIDE hot path.  Every entry
 * point below replaces one method of the Rust reference API and cites it as
 * `crates/<crate>/src/<file>:<line>`.  A Rust FFI crate binds these symbols 1:1
 * (`extern "C"` block + `#[repr(C)]` mirrors of the structs below).
 *
 * Conventions
 *  - Every pointer argument is a caller-owned DEVICE buffer unless its name ends
 *    in `_host`, in which case it is host memory.  Configuration structs and the
 *    explicit hash/weight parameter arrays passed at creation time are host memory.
 *  - Every call returns a kl_status.  No C++ exception crosses this boundary.
 *    On failure, kl_last_error(ctx) returns a message for the failing call.
 *  - A context is bound to one CUDA device and one CUDA stream.  Calls are
 *    asynchronous on that stream unless they return host data (`*_host`
 *    outputs), which synchronise the stream before returning.
 *  - Handles are not thread-safe: one host thread at a time per handle
 *    (mirrors `&mut self` in the reference).  Distinct handles are independent.
 *  - Query outputs are sets sorted by neuron id.  The reference returns them in
 *    HashMap iteration order (crates/klearu-core/src/lsh/index.rs:219-249); the
 *    set (and each id's count) is identical, only the order is normalised.
 *  - Kernels never trap: device-side bound violations are recorded in a
 *    per-context error word and reported as KL_EBOUNDS by the next
 *    synchronising call or kl_ctx_check().
 */
#ifndef KLEARU_GPU_H
#define KLEARU_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KLEARU_GPU_ABI_VERSION 2

#if defined(__GNUC__)
#define KL_API __attribute__((visibility("default")))
#else
#define KL_API
#endif

/* ------------------------------------------------------------------------ */
/* Status codes.  The reference panics (assert!) where these are returned;   */
/* e.g. FifoBucket::new capacity>0 (crates/klearu-core/src/bucket/fifo.rs:18) */
/* ------------------------------------------------------------------------ */
typedef enum {
  KL_OK = 0,
  KL_EINVAL = 1,       /* bad argument / configuration                       */
  KL_ENOMEM = 2,       /* device allocation failed                           */
  KL_ECUDA = 3,        /* CUDA runtime error                                 */
  KL_ENCCL = 4,        /* NCCL error (sharded networks)                      */
  KL_ETIMEOUT = 5,     /* bounded device wait gave up                        */
  KL_EBOUNDS = 6,      /* device kernel saw an out-of-range id/index         */
  KL_ECAPACITY = 7,    /* an output did not fit its capacity (truncated)     */
  KL_EUNSUPPORTED = 8  /* valid in the reference but not supported here      */
} kl_status;

/* Enumerations mirror crates/klearu-core/src/config.rs:3-38 (same order). */
typedef enum {
  KL_HASH_SIMHASH = 0,
  KL_HASH_WTA = 1,
  KL_HASH_DWTA = 2,
  KL_HASH_MINHASH = 3,
  KL_HASH_SRP = 4
} kl_hash_kind;

typedef enum { KL_BUCKET_FIFO = 0, KL_BUCKET_RESERVOIR = 1 } kl_bucket_type;

typedef enum {
  KL_SAMPLING_VANILLA = 0,
  KL_SAMPLING_TOPK = 1,
  KL_SAMPLING_THRESHOLD = 2
} kl_sampling;

typedef enum {
  KL_ACT_RELU = 0,
  KL_ACT_SIGMOID = 1,
  KL_ACT_TANH = 2,
  KL_ACT_SOFTMAX = 3,
  KL_ACT_IDENTITY = 4
} kl_activation;

typedef enum { KL_OPT_SGD = 0, KL_OPT_ADAM = 1 } kl_optimizer;

/* Weight storage.  F32 is the reference's storage (Vec<f32> per neuron,
 * crates/klearu-core/src/network/neuron.rs:6-12).  BF16 is klearu-accel's
 * Mode 2: bf16 storage, f32 arithmetic, round-to-nearest-even store
 * (crates/klearu-accel/src/bf16/mod.rs:22-107).  Adam/SGD state is f32. */
typedef enum { KL_DTYPE_F32 = 0, KL_DTYPE_BF16 = 1 } kl_dtype;

typedef enum { KL_QUERY_COUNTS = 0, KL_QUERY_UNION = 1 } kl_query_mode;

/* EXACT_SEQUENTIAL = Network::train_step semantics: per example forward,
 * backward and immediate optimizer update (crates/klearu-core/src/network/net.rs:81-119).
 * BATCHED = every example of the batch is forwarded against the step-start
 * weights, per-row gradients are summed over the batch (in sample order) and
 * one optimizer update is applied to every touched row. */
typedef enum { KL_MODE_EXACT_SEQUENTIAL = 0, KL_MODE_BATCHED = 1 } kl_train_mode;

typedef struct kl_ctx_s* kl_ctx_t;
typedef struct kl_hash_s* kl_hash_t;
typedef struct kl_index_s* kl_index_t;
typedef struct kl_net_s* kl_net_t;
typedef struct kl_dataset_s* kl_dataset_t;
typedef struct kl_batch_iter_s* kl_batch_iter_t;

/* ------------------------------------------------------------------------ */
/* Context                                                                  */
/* ------------------------------------------------------------------------ */

/* Create a context on `device` issuing work on `stream` (a cudaStream_t; NULL
 * selects the legacy default stream).  No reference counterpart: the Rust
 * reference is single-process CPU code with no device state. */
KL_API kl_status kl_ctx_create(int device, void* stream, kl_ctx_t* out);
KL_API kl_status kl_ctx_destroy(kl_ctx_t ctx);
KL_API kl_status kl_ctx_set_stream(kl_ctx_t ctx, void* stream);
/* Wait for all work issued on the context's stream; reports device errors. */
KL_API kl_status kl_ctx_sync(kl_ctx_t ctx);
/* Synchronise and report (then clear) the device-side error word. */
KL_API kl_status kl_ctx_check(kl_ctx_t ctx);
/* Message of the context's last failed call.  With ctx NULL: the message of
 * the last failed call made on this host thread (the dataset calls below take
 * no context). */
KL_API const char* kl_last_error(kl_ctx_t ctx);
KL_API int kl_abi_version(void);

/* ------------------------------------------------------------------------ */
/* Hash families -- replaces trait HashFamily                               */
/* (crates/klearu-core/src/hash/mod.rs:24-39)                               */
/* ------------------------------------------------------------------------ */

/* Explicit hash parameters (host memory).  Only the member(s) of the chosen
 * kind are read.
 *  SIMHASH : planes [L][K][d] int8 in {-1,0,1}    (SimHash::hyperplanes, simhash.rs:21-27)
 *  WTA/DWTA: windows [L][K][window] uint32 dims    (DwtaHash::windows, dwta.rs:19-29; wta.rs:22-32)
 *  MINHASH : perms [L][d] uint32, perms[t][dim] = permuted index (minhash.rs:18-28)
 *  SRP     : per (table*K + bit) sorted sparse rows: rowptr [L*K+1], idx, coef in {-1,+1}
 *            (SparseRandomProjection::projections, srp.rs:22-31) */
typedef struct {
  const int8_t* planes;
  const uint32_t* windows;
  const uint32_t* perms;
  const uint32_t* srp_rowptr;
  const uint32_t* srp_idx;
  const int8_t* srp_coef;
} kl_hash_params;

/* Replaces SimHash::new / WtaHash::new / DwtaHash::new / MinHash::new /
 * SparseRandomProjection::new (simhash.rs:37-58, wta.rs:42-84, dwta.rs:39-84,
 * minhash.rs:38-60, srp.rs:43-80) with explicit parameters.  `window_size` is
 * read for WTA/DWTA only. */
KL_API kl_status kl_hash_create(kl_ctx_t ctx, int kind, int input_dim, int k, int num_tables,
                         int window_size, const kl_hash_params* params_host, kl_hash_t* out);
/* Seeded construction following the reference distributions (ternary
 * 1/6-2/3-1/6 planes, first-w-of-a-shuffle windows, full shuffles for MinHash,
 * SRP density `srp_sparsity`).  The random stream is this library's SplitMix64,
 * not rand 0.8.5's ChaCha12, so seeds do not reproduce the Rust parameters. */
KL_API kl_status kl_hash_create_seeded(kl_ctx_t ctx, int kind, int input_dim, int k, int num_tables,
                                int window_size, float srp_sparsity, uint64_t seed,
                                kl_hash_t* out);
KL_API kl_status kl_hash_destroy(kl_hash_t h);
/* HashFamily::k / input_dim / num_tables (hash/mod.rs:32-38). */
KL_API kl_status kl_hash_info(kl_hash_t h, int* kind_host, int* input_dim_host, int* k_host,
                       int* num_tables_host);
/* Arithmetic of the SimHash / SRP projection of dense rows (no reference
 * counterpart; the reference has one scalar path, simhash.rs:75-126).
 *  KL_PROJ_AUTO (0, default): batches of >= 4096 bf16 rows (table rebuilds)
 *    on the tensor cores (exact bf16 products, f32 accumulation in the tensor
 *    core's order), everything else on the sequential path;
 *  KL_PROJ_SEQUENTIAL (1): always the reference's sequential f32 sums, so
 *    every code equals the reference's bit for bit;
 *  KL_PROJ_TENSOR (2): the tensor cores for every bf16 row batch.
 * On the tensor cores a projection within a few f32 ulps of zero (|p| far
 * below 1e-6 for unit-scale rows) may take the other sign; min_abs_proj
 * outputs identify such rows. */
#define KL_PROJ_AUTO 0
#define KL_PROJ_SEQUENTIAL 1
#define KL_PROJ_TENSOR 2
KL_API kl_status kl_hash_set_projection(kl_hash_t h, int mode);
/* The same setting on an index's hash family (for a network layer's index,
 * from kl_net_layer_index). */
KL_API kl_status kl_index_set_projection(kl_index_t ix, int mode);
/* Batched HashFamily::hash_dense (hash/mod.rs:26): codes[i*L + t] =
 * hash_dense(X[i*ldx ..], t) for all rows i < n and tables t < L.  For
 * SIMHASH/SRP, `min_abs_proj` (nullable, [n][L]) receives min over the K bits
 * of |projection|, so callers can log near-zero projections whose sign is
 * summation-order sensitive. */
KL_API kl_status kl_hash_dense_batch(kl_hash_t h, const float* X, int n, int ldx, uint64_t* codes,
                              float* min_abs_proj);
/* kl_hash_dense_batch over rows of either storage type: rows [n][ld] of
 * `dtype` (KL_DTYPE_F32 / KL_DTYPE_BF16), as the index rebuild hashes them. */
KL_API kl_status kl_hash_dense_batch_rows(kl_hash_t h, const void* rows, int n, int ld, int dtype, uint64_t* codes,
                                          float* min_abs_proj);
/* Batched HashFamily::hash_sparse (hash/mod.rs:29) over a CSR batch with
 * sorted, unique column indices per row. */
KL_API kl_status kl_hash_sparse_batch(kl_hash_t h, const int32_t* rowptr, const uint32_t* idx,
                               const float* val, int n, uint64_t* codes, float* min_abs_proj);

/* ------------------------------------------------------------------------ */
/* LSH index -- replaces trait LshIndexTrait (lsh/index.rs:21-67) and       */
/* create_lsh_index (lsh/index.rs:339-374)                                  */
/* ------------------------------------------------------------------------ */

/* LshIndex::new (index.rs:193-205): L tables x 2^K buckets of `capacity` ids.
 * The index keeps its own reference to `h` (h may be destroyed afterwards). */
KL_API kl_status kl_index_create(kl_ctx_t ctx, kl_hash_t h, int bucket_type, int capacity,
                          kl_index_t* out);
KL_API kl_status kl_index_destroy(kl_index_t ix);
KL_API kl_status kl_index_info(kl_index_t ix, int* num_tables_host, int* num_buckets_host,
                        int* capacity_host, int* bucket_type_host);
/* n sequential LshIndexTrait::insert calls (index.rs:257-262), in array order.
 * rows: [n][ld] elements of `dtype` (KL_DTYPE_F32 / KL_DTYPE_BF16). */
KL_API kl_status kl_index_insert_batch(kl_index_t ix, const uint32_t* ids, const void* rows, int n,
                                int ld, int dtype);
/* n sequential LshIndexTrait::insert_sparse calls (index.rs:264-269). */
KL_API kl_status kl_index_insert_sparse_batch(kl_index_t ix, const uint32_t* ids,
                                       const int32_t* rowptr, const uint32_t* idx,
                                       const float* val, int n);
/* n sequential LshIndexTrait::remove calls (index.rs:278-280). */
KL_API kl_status kl_index_remove(kl_index_t ix, const uint32_t* ids, int n);
/* n sequential LshIndexTrait::remove_with_weights calls (index.rs:271-276). */
KL_API kl_status kl_index_remove_with_weights(kl_index_t ix, const uint32_t* ids, const void* rows,
                                       int n, int ld, int dtype);
/* LshIndexTrait::rebuild (index.rs:302-307): clear, then insert (ids[i], rows[i])
 * in order.  ids == NULL means ids 0..n-1 (Layer::rebuild_index, layer.rs:228-233). */
KL_API kl_status kl_index_rebuild(kl_index_t ix, const uint32_t* ids, const void* rows, int n, int ld,
                           int dtype);
/* LshIndexTrait::clear (index.rs:313-315). */
KL_API kl_status kl_index_clear(kl_index_t ix);
/* Batched LshIndexTrait::query / query_with_counts / query_union
 * (index.rs:282-292).  Results for query i are out_ids[out_offsets[i] ..
 * out_offsets[i+1]) sorted by id; out_counts (COUNTS mode; nullable) holds the
 * number of tables each id was found in.  out_offsets has n+1 entries.  If the
 * total exceeds `capacity`, results are truncated, *overflow (device, nullable)
 * is set to 1 and KL_ECAPACITY is reported by the next synchronising call. */
KL_API kl_status kl_index_query_batch(kl_index_t ix, const float* X, int n, int ldx, int mode,
                               uint32_t* out_ids, uint32_t* out_counts, int32_t* out_offsets,
                               int32_t capacity, int32_t* overflow);
/* Allocation-free variant of kl_index_query_batch, for callers that cannot
 * call cudaMalloc: a host runtime that owns all device memory, or a memory
 * budget fixed at start-up.  No counterpart in the reference (its queries
 * are CPU calls).  Same arguments, results and errors as
 * kl_index_query_batch, but the call allocates nothing: its scratch is a
 * fixed KL_NOALLOC_SCRATCH_BYTES array inside this library's device image,
 * held by every GPU that loads the library until the process exits.
 *  - n queries need about n * L * capacity * 8 bytes of it (plus L*n*2 and
 *    n*4); a larger batch is refused with KL_ECAPACITY: split it.
 *  - The first call on a device looks up the array's device address (no
 *    allocation); make that first call before any stream capture.
 *  - All calls on a device share the array; calls whose GPU work overlaps
 *    (other streams, other contexts on the same device) race on it. */
#define KL_NOALLOC_SCRATCH_BYTES (16u << 20)
KL_API kl_status kl_index_query_batch_noalloc(kl_index_t ix, const float* X, int n, int ldx, int mode,
                                              uint32_t* out_ids, uint32_t* out_counts,
                                              int32_t* out_offsets, int32_t capacity,
                                              int32_t* overflow);
/* Batched query_sparse_union / query_sparse_with_counts (index.rs:290-300). */
KL_API kl_status kl_index_query_sparse_batch(kl_index_t ix, const int32_t* rowptr,
                                      const uint32_t* idx, const float* val, int n, int mode,
                                      uint32_t* out_ids, uint32_t* out_counts,
                                      int32_t* out_offsets, int32_t capacity,
                                      int32_t* overflow);
/* Copy the bucket arrays out (checkpointing / parity): ids [L][2^K][cap] in
 * bucket order (Bucket::contents, bucket/mod.rs:11-31), lens [L][2^K],
 * insertion counts [L][2^K] (ReservoirBucket::total_insertions; nullable). */
/* BOLT SparseInferenceEngine::infer / infer_linear
 * (crates/klearu-bolt/src/sparse_inference.rs:32-106) for n inputs X [n][ldx]
 * (device f32): the index's candidates ordered by table count descending
 * (ties by id ascending, where the reference's follow HashMap order), the
 * first effective_k = (int)((float)base_top_k * sparsity_multiplier) kept,
 * and for each kept id < num_neurons the activation
 * sum_j X[j] * weights[id][j] (sequential f32, the reference's order)
 * + bias[id] (bias nullable = 0), clamped at 0 when `relu` (infer) or not
 * (infer_linear).  weights: [num_neurons][ld] of `dtype`, device.  Output per
 * input i: out_ids / out_act [i*stride .. i*stride + out_n[i]) in that order;
 * more than `stride` results are truncated and reported as KL_ECAPACITY by
 * the next synchronising call. */
KL_API kl_status kl_bolt_infer_batch(kl_index_t ix, const void* weights, int dtype, int ld, const float* bias,
                                     int num_neurons, const float* X, int n, int ldx, float sparsity_multiplier,
                                     int base_top_k, int relu, uint32_t* out_ids, float* out_act, int32_t* out_n,
                                     int stride);
KL_API kl_status kl_index_export(kl_index_t ix, uint32_t* ids, uint32_t* lens, uint64_t* counts);
/* Inverse of kl_index_export. */
KL_API kl_status kl_index_import(kl_index_t ix, const uint32_t* ids, const uint32_t* lens,
                          const uint64_t* counts);

/* ------------------------------------------------------------------------ */
/* Adaptive rebuild scheduling -- replaces klearu_mongoose::AdaptiveScheduler */
/* (crates/klearu-mongoose/src/scheduler.rs:44-213)                          */
/* ------------------------------------------------------------------------ */
typedef struct kl_adaptive_s* kl_adaptive_t;
/* AdaptiveScheduler::new (scheduler.rs:53-87); EMA alpha 0.3. */
KL_API kl_status kl_adaptive_create(kl_ctx_t ctx, uint64_t min_interval, uint64_t max_interval,
                             float sample_fraction, float drift_threshold, kl_adaptive_t* out);
KL_API kl_status kl_adaptive_destroy(kl_adaptive_t a);
/* record_baseline (scheduler.rs:96-129): hash the sampled rows of `rows`
 * ([n][ld] of `dtype`, device) with `h` and keep their codes.  Sampled row
 * indices are explicit (`sampled_host`, n_sampled) or, when NULL, the first
 * ceil(n * sample_fraction) of a shuffle seeded by `seed` (this library's
 * SplitMix64 stream: rand 0.8.5's StdRng is not reproduced).  Synchronises. */
KL_API kl_status kl_adaptive_record_baseline(kl_adaptive_t a, kl_hash_t h, const void* rows, int n, int ld,
                                      int dtype, const uint32_t* sampled_host, int n_sampled,
                                      uint64_t seed);
/* should_rebuild (scheduler.rs:133-159) on the current rows; a drift check
 * (every min_interval steps) hashes the sampled rows on the GPU and
 * synchronises to read the changed count. */
KL_API kl_status kl_adaptive_should_rebuild(kl_adaptive_t a, const void* rows, int n, int ld, int dtype,
                                     int* rebuild_host);
/* notify_rebuild / drift_estimate / steps_since_rebuild (scheduler.rs:198-211);
 * n_sampled_host: number of rows in the baseline (baseline_codes.len()). */
KL_API kl_status kl_adaptive_notify_rebuild(kl_adaptive_t a);
KL_API kl_status kl_adaptive_state(kl_adaptive_t a, float* drift_ema_host, uint64_t* steps_since_rebuild_host,
                            int* n_sampled_host);

/* ------------------------------------------------------------------------ */
/* Network -- replaces klearu_core::network::Network (network/net.rs:10-173) */
/* ------------------------------------------------------------------------ */

/* LshConfig (config.rs:40-65).  range_pow is carried but unused, as in the
 * reference (the index uses 2^num_hashes buckets, index.rs:194). */
typedef struct {
  int32_t hash_function;        /* kl_hash_kind */
  int32_t bucket_type;          /* kl_bucket_type */
  int32_t num_tables;           /* L */
  int32_t range_pow;
  int32_t num_hashes;           /* K */
  int32_t bucket_capacity;
  int32_t rebuild_interval_base;
  double rebuild_decay;
} kl_lsh_config;

/* LayerConfig (config.rs:67-106). */
typedef struct {
  int32_t input_dim;
  int32_t num_neurons;
  int32_t activation;           /* kl_activation */
  kl_lsh_config lsh;
  int32_t sampling;             /* kl_sampling */
  int32_t sampling_threshold;
  int32_t top_k;
  int32_t is_output;
} kl_layer_config;

/* SlideConfig + NetworkConfig (config.rs:108-143) plus device-side knobs. */
typedef struct {
  int32_t num_layers;
  const kl_layer_config* layers; /* host array [num_layers] */
  int32_t optimizer;             /* kl_optimizer */
  double learning_rate;          /* carried; train_step takes lr explicitly, as in net.rs:81 */
  int32_t batch_size;
  int32_t num_threads;
  uint64_t seed;
  int32_t weight_dtype;          /* kl_dtype */
  int32_t max_batch;             /* capacity of per-step buffers (examples per call) */
  /* Largest sample-major gradient matrix (bytes) the output-layer update may
   * use (the dense-collision path); a layer whose matrix would be larger takes
   * the segmented path.  0 = 2 GiB; < 0 = always the segmented path.  No
   * reference counterpart (a memory/speed choice of this engine). */
  int64_t dense_update_max_bytes;
} kl_net_config;

/* Explicit initial parameters of one layer (host memory).  weights/bias are
 * the reference's per-neuron Vec<f32> rows [num_neurons][input_dim] and biases
 * (Neuron, neuron.rs:6-12).  NULL weights => seeded N(0, sqrt(2/d)) rows from
 * this library's generator; NULL bias => 0 (neuron.rs:23-43). */
typedef struct {
  const float* weights;
  const float* bias;
  kl_hash_params hash;
} kl_layer_init;

/* A batch of examples (device memory): CSR features with sorted unique
 * indices per row (Example / SparseVector, data/dataset.rs:5-16,
 * tensor/sparse.rs:14-20) and CSR label lists. */
typedef struct {
  int32_t batch;
  const int32_t* rowptr;    /* [batch+1] */
  const uint32_t* idx;      /* [rowptr[batch]] */
  const float* val;         /* [rowptr[batch]] */
  const int32_t* label_ptr; /* [batch+1] */
  const uint32_t* labels;   /* [label_ptr[batch]] */
  int32_t nnz;              /* host-side copy of rowptr[batch] (sizes scratch) */
  int32_t nlabels;          /* host-side copy of label_ptr[batch] */
} kl_batch;

/* Network::new (net.rs:19-57): layers, initial table build (layer.rs:40-44),
 * optimizer state, RebuildScheduler from layer 0's LSH config.  `init` is
 * NULL (all seeded) or an array of num_layers entries. */
KL_API kl_status kl_net_create(kl_ctx_t ctx, const kl_net_config* cfg_host,
                        const kl_layer_init* init_host, kl_net_t* out);
KL_API kl_status kl_net_destroy(kl_net_t net);
/* Network::train_step (net.rs:81-119), returning the mean loss: into
 * `loss` (device, nullable) and/or `loss_host` (host, nullable; synchronises).
 * Increments step once and runs the rebuild check, as the reference does. */
KL_API kl_status kl_net_train_step(kl_net_t net, const kl_batch* batch_host, double lr, int mode,
                            float* loss, float* loss_host);
/* Network::train_step (net.rs:81-119) on a batch in HOST memory (every
 * pointer of `batch_host` is host memory; nnz / nlabels are taken from
 * rowptr[batch] / label_ptr[batch]).  The arrays are copied into an internal
 * pinned buffer and uploaded with one copy on a separate stream, so the call
 * returns without waiting for the GPU and the next batch's upload overlaps
 * this step.  The mean loss is copied to `loss_host` (nullable) in stream
 * order: it is valid after kl_ctx_sync, and the copy only stays
 * asynchronous when `loss_host` is pinned memory. */
KL_API kl_status kl_net_train_step_host(kl_net_t net, const kl_batch* batch_host, double lr, int mode,
                                        float* loss_host);
/* Network::forward (net.rs:62-78) for every example of the batch, without any
 * update.  Per-layer results are read with kl_net_layer_output. */
KL_API kl_status kl_net_forward(kl_net_t net, const kl_batch* batch_host);
/* LayerOutput (layer.rs:19-26) of the last forward / train_step, compact:
 * for example i, active ids (sorted by id) are ids[i*stride ..
 * i*stride+counts[i]) with their pre-activations and activations at the same
 * positions; stride is kl_net_layer_info's max_active.  Any output may be NULL. */
KL_API kl_status kl_net_layer_output(kl_net_t net, int layer, uint32_t* ids, int32_t* counts,
                              float* pre, float* act);
KL_API kl_status kl_net_layer_info(kl_net_t net, int layer, int* input_dim_host,
                            int* num_neurons_host, int* max_active_host);
/* Network::predict_top_k (net.rs:159-173): per example the k highest final
 * activations over all N neurons (inactive ones score 0), ties by lower id. */
KL_API kl_status kl_net_predict_topk(kl_net_t net, const kl_batch* batch_host, int k,
                              uint32_t* top_ids, float* top_scores);
/* Read / write one layer's parameters as reference-layout f32 rows (host
 * memory): weights [N][d], bias [N], optimizer state m/v [N][d] and mb/vb [N]
 * (Adam m_w, v_w, m_b, v_b; SGD momentum in m/mb).  Any pointer may be NULL. */
/* kl_bolt_infer_batch over layer `layer` (>= 1) of a network: its LSH index,
 * weights and bias; X [n][ldx] is the layer's input (the previous layer's
 * activations), device f32. */
KL_API kl_status kl_net_bolt_infer(kl_net_t net, int layer, const float* X, int n, int ldx,
                                   float sparsity_multiplier, int base_top_k, int relu, uint32_t* out_ids,
                                   float* out_act, int32_t* out_n, int stride);
KL_API kl_status kl_net_get_layer(kl_net_t net, int layer, float* weights_host, float* bias_host,
                           float* m_host, float* v_host, float* mb_host, float* vb_host);
KL_API kl_status kl_net_set_layer(kl_net_t net, int layer, const float* weights_host,
                           const float* bias_host, const float* m_host, const float* v_host,
                           const float* mb_host, const float* vb_host);
/* Layer::rebuild_index (layer.rs:228-233) on every layer. */
KL_API kl_status kl_net_rebuild(kl_net_t net);
/* Borrow a layer's LSH index (Layer::lsh_index, layer.rs:12).  Owned by net. */
KL_API kl_status kl_net_layer_index(kl_net_t net, int layer, kl_index_t* out);
/* Network::step and RebuildScheduler state (net.rs:13-14, maintenance.rs:20-26). */
KL_API kl_status kl_net_get_step(kl_net_t net, uint64_t* step_host, uint64_t* next_rebuild_host,
                          uint64_t* rebuild_count_host);
KL_API kl_status kl_net_set_step(kl_net_t net, uint64_t step, uint64_t next_rebuild,
                          uint64_t rebuild_count);

/* Rebuild policy of a network's LSH tables (no reference counterpart as a
 * network setting: the reference's Network always uses RebuildScheduler,
 * net.rs:109-116, and klearu-mongoose's AdaptiveScheduler is a standalone
 * component, crates/klearu-mongoose/src/scheduler.rs:44-213).
 *  KL_REBUILD_SCHEDULE (default): RebuildScheduler, every layer at once.
 *  KL_REBUILD_ADAPTIVE: one AdaptiveScheduler per layer with the given
 *    intervals, sample fraction and drift threshold; a layer is rebuilt when
 *    the EMA of the fraction of its sampled neurons whose hash codes changed
 *    reaches the threshold (or at max_interval), and its baseline is then
 *    re-recorded from a sample drawn with `seed`.  Setting the policy records
 *    the first baselines.  A drift check (every min_interval steps) reads a
 *    count back from the device, so it waits for the step to finish. */
#define KL_REBUILD_SCHEDULE 0
#define KL_REBUILD_ADAPTIVE 1
typedef struct {
  int32_t kind;
  uint64_t min_interval;
  uint64_t max_interval;
  float sample_fraction;
  float drift_threshold;
  uint64_t seed;
} kl_rebuild_policy;
KL_API kl_status kl_net_set_rebuild_policy(kl_net_t net, const kl_rebuild_policy* policy_host);
/* A layer's rebuild state: its AdaptiveScheduler's drift EMA and steps since
 * its last rebuild (0 under KL_REBUILD_SCHEDULE), and its rebuild count. */
KL_API kl_status kl_net_rebuild_state(kl_net_t net, int layer, float* drift_ema_host,
                                      uint64_t* steps_since_rebuild_host, uint64_t* rebuilds_host);

/* Checkpoint (no reference counterpart: the reference has no resume).  One
 * file holds everything a train step reads or writes: every layer's weights
 * (storage type), bias, Adam moments, LSH tables (ids, lengths, reservoir
 * counts), the step, the RebuildScheduler and the AdaptiveScheduler states.
 * kl_net_load restores into a network created with the same configuration
 * (and, for a sharded network, the same rank and rank count: each rank saves
 * and loads its own file); KL_EINVAL on a mismatch or a corrupt file
 * (FNV-1a checksum).  Both synchronise the context stream. */
KL_API kl_status kl_net_save(kl_net_t net, const char* path);
KL_API kl_status kl_net_load(kl_net_t net, const char* path);

/* Per-step work counters accumulated on the device since the last reset
 * (used for the HBM roofline): sum of active set sizes, distinct rows touched
 * by the optimizer, input nnz, examples, steps, rebuilds; per layer. */
typedef struct {
  uint64_t active_sum;      /* sum over examples of |active set| */
  uint64_t touched_rows;    /* rows (neurons) updated by the optimizer */
  uint64_t input_nnz;       /* layer 0 only: sum of input nnz */
  uint64_t examples;
  uint64_t steps;
  uint64_t rebuilds;
} kl_layer_stats;
KL_API kl_status kl_net_stats(kl_net_t net, int layer, kl_layer_stats* stats_host, int reset);

/* Phase timing for roofline accounting (no reference counterpart; the
 * reference has no profiler hooks).  When enabled, CUDA events bracket each
 * phase of each layer on the context stream. */
typedef enum {
  KL_PHASE_HASH = 0,     /* hash the layer input against the L tables         */
  KL_PHASE_PROBE = 1,    /* bucket probe, union/counts, sampling              */
  KL_PHASE_FORWARD = 2,  /* active-row gather-dot (+ fused loss grad and dX)  */
  KL_PHASE_BACKWARD = 3, /* local gradients, input gradients                  */
  KL_PHASE_UPDATE = 4,   /* segmented gradient reduction + optimizer          */
  KL_PHASE_REBUILD = 5,  /* table rebuild                                     */
  KL_PHASE_STREAM = 6,   /* layer 0 only: the streaming Adam pass over all     */
                         /* feature rows (inside KL_PHASE_UPDATE)              */
  KL_NPHASES = 7
} kl_phase;
KL_API kl_status kl_net_profile(kl_net_t net, int enable);
/* Accumulated milliseconds and call counts per phase of `layer` since the last
 * reset (synchronises).  ms_host / calls_host have KL_NPHASES entries. */
KL_API kl_status kl_net_profile_read(kl_net_t net, int layer, double* ms_host, uint64_t* calls_host,
                                     int reset);
/* Kernels launched by this library in this process so far. */
KL_API kl_status kl_launch_count(uint64_t* count_host);
/* Device (cudaMalloc) and pinned host (cudaHostAlloc) allocations made by this
 * library in this process so far.  No reference counterpart (diagnostic). */
KL_API kl_status kl_alloc_count(uint64_t* count_host);

/* ------------------------------------------------------------------------ */
/* Neuron sharding of the output layer over NCCL (no reference counterpart: */
/* the reference's only parallelism is HOGWILD threads, optim/hogwild.rs).  */
/* ------------------------------------------------------------------------ */

/* Size in bytes of the opaque communicator id (ncclUniqueId). */
KL_API int kl_dist_unique_id_size(void);
/* Rank 0 creates the id; it is shared with all ranks out of band. */
KL_API kl_status kl_dist_get_unique_id(void* id_host);
/* Like kl_net_create, but for one rank of an `nranks`-process job (one GPU
 * each).  No reference counterpart: the reference's only parallelism is
 * HOGWILD threads (crates/klearu-core/src/optim/hogwild.rs:65-95).
 *  - The output (last) layer's neurons are split into contiguous slices
 *    [r*N/P, (r+1)*N/P); this rank owns slice `rank`: its rows, optimizer
 *    state and LSH tables, whose buckets hold bucket_capacity / nranks ids so
 *    that an example's candidates over all shards stay num_tables *
 *    bucket_capacity, as in the unsharded network.
 *  - The sparse-input hidden layer is data parallel: in kl_net_train_step
 *    each rank passes exactly `max_batch` examples; the step trains on the
 *    global batch of all ranks' examples in rank order (KL_MODE_BATCHED only).
 *    Its weights and bias are replicated; its Adam moments are split by
 *    feature: rank r updates feature rows [r*R, (r+1)*R), R = ceil(d/nranks)
 *    (kl_net_owned_features), and the updated rows are all-gathered.
 *  - Collectives per step (NCCL): all-gather of the batches and of the hidden
 *    activations, all-reduce of per-example selection counts (overlapping the
 *    output forward), all-reduce of the label probabilities with a
 *    reduce-scatter of the output layer's input gradient, all-gather of the
 *    hidden local gradients and touched masks, and all-gather of the updated
 *    hidden weight rows.  The output layer's update runs on a second stream
 *    beside the collectives after its forward.
 *  - Output selection is decided over all shards, as in the unsharded layer.
 *    Vanilla, and TopK with top_k >= num_tables * bucket_capacity, take every
 *    candidate; TopK below that (count descending, id ascending) and
 *    Threshold (count >= threshold, else the single best) sum per-example
 *    histograms of the local candidates' table counts over the ranks
 *    (all-reduce), cut there, and all-gather each rank's number of
 *    candidates at the cut so the lowest ids are taken first.  An example
 *    that selects nothing on any rank takes every neuron (layer.rs:82-84).
 *  - A rank's batch that cannot be exchanged (another example count, or more
 *    than 512 nnz / 32 labels per example on average) does not make that rank
 *    leave the collective sequence: it is sent empty with a fault flag, every
 *    rank applies the step with a zero learning rate and reports KL_EBOUNDS
 *    (example count) or KL_ECAPACITY at its next synchronising call.
 *  - Supported shapes: two layers, non-softmax output.  Per example at most
 *    512 input nnz and 32 labels.
 *  - kl_net_forward and kl_net_predict_topk take exactly `max_batch`
 *    examples per rank, like the train step (labels may be absent).  After
 *    kl_net_forward, kl_net_layer_output(1) holds the global batch's
 *    (nranks * max_batch examples, rank order) active sets on this rank's
 *    slice; kl_net_predict_topk returns the top k over all N neurons of this
 *    rank's own examples (k <= N / nranks; local top-k lists all-gathered and
 *    merged).  KL_MODE_EXACT_SEQUENTIAL returns KL_EUNSUPPORTED.
 *    kl_net_get_layer / set_layer / layer_output address the rank's slice of
 *    the output layer with local row ids (see kl_net_shard_info); layer
 *    outputs hold nranks * max_batch rows.
 * `init` holds the FULL parameters (every rank passes the same);
 * `unique_id_host` is kl_dist_get_unique_id's output from rank 0. */
KL_API kl_status kl_net_create_sharded(kl_ctx_t ctx, const kl_net_config* cfg_host,
                                const kl_layer_init* init_host, const void* unique_id_host,
                                int rank, int nranks, kl_net_t* out);
/* This rank's place in a sharded network: rank, number of ranks, global id of
 * its first output neuron and its number of output neurons (1, 0, N for an
 * unsharded network). */
KL_API kl_status kl_net_shard_info(kl_net_t net, int* rank_host, int* nranks_host, uint32_t* id_base_host,
                            int* num_local_host);
/* Failure detection of a sharded network.  The reference has no counterpart:
 * its Network runs in one process (net.rs:10-173) and reports failures by
 * panicking (error.rs:3-33 is never returned by it).
 *
 * kl_net_set_comm_timeout: 0 (the default) keeps plain blocking waits.  With a
 * timeout, every wait of this net that depends on other ranks (kl_net_sync,
 * a train step's host loss read, a sharded forward or predict_top_k, destroy)
 * polls the net's streams and the communicator's asynchronous error.  A
 * communicator error returns KL_ENCCL, and no progress within timeout_ms
 * returns KL_ETIMEOUT; both abort the communicator (the waiting collectives
 * then return).  Every later call that needs the communicator returns
 * KL_ENCCL; recreate the network (from a checkpoint) to continue.  Choose a
 * timeout well above the longest step, including a table rebuild.
 *
 * kl_net_sync: waits for this net's work (bounded as above) and reports
 * device-side faults, like kl_ctx_sync.  After an abort it still waits for
 * the drained queue (KL_ETIMEOUT if the abort left work pending), so the
 * net's state can be read back.
 *
 * kl_net_comm_abort: aborts the communicator now, for a caller whose own
 * health check (a heartbeat over the process group's store) found a rank
 * missing between steps.  A no-op on an unsharded network. */
KL_API kl_status kl_net_set_comm_timeout(kl_net_t net, int timeout_ms);
KL_API kl_status kl_net_sync(kl_net_t net);
KL_API kl_status kl_net_comm_abort(kl_net_t net);
/* The hidden layer's feature rows [first, first + count) whose Adam moments
 * this rank updates (every feature of an unsharded network).  In
 * kl_net_get_layer(0)'s [neuron][feature] layout these are columns; the
 * moments of the other columns are another rank's. */
KL_API kl_status kl_net_owned_features(kl_net_t net, uint32_t* first_host, uint32_t* count_host);

/* ---------------------------------------------------------------------------
 * Deja Vu sparse FFN.
 * --------------------------------------------------------------------------- */
typedef struct kl_predictor_s* kl_predictor_t;
typedef struct kl_sparse_mlp_s* kl_sparse_mlp_t;

/* SparsityPredictor::from_weights (klearu-dejavu predictor/mlp_predictor.rs:65-84):
 * w1 [hidden_dim][input_dim], w2 [output_dim][hidden_dim] row-major f32 (host),
 * stored as bf16 (round to nearest even); b1 / b2 f32 (NULL = zeros). */
KL_API kl_status kl_predictor_create(kl_ctx_t ctx, int input_dim, int hidden_dim, int output_dim,
                                     const float* w1_host, const float* b1_host, const float* w2_host,
                                     const float* b2_host, kl_predictor_t* out);
KL_API kl_status kl_predictor_destroy(kl_predictor_t p);
KL_API kl_status kl_predictor_info(kl_predictor_t p, int* input_dim_host, int* hidden_dim_host,
                                   int* output_dim_host);
/* SparsityPredictor::predict (mlp_predictor.rs:102-123) for n_tokens inputs:
 * x [n_tokens][input_dim] -> scores [n_tokens][output_dim] (device, f32). */
KL_API kl_status kl_predictor_predict(kl_predictor_t p, const float* x, int n_tokens, float* scores);
/* SparsityPredictor::select_top_k (mlp_predictor.rs:126-132): per token the
 * min(k, output_dim) indices of the largest scores, in descending score order
 * with ties in ascending index order (the reference's stable sort).
 * idx [n_tokens][min(k, output_dim)] (device); scores (device, nullable)
 * receives the predict() output.  Scores must be finite. */
KL_API kl_status kl_predictor_select_topk(kl_predictor_t p, const float* x, int n_tokens, int k, uint32_t* idx,
                                          float* scores);

/* SwiGLU MLP weights (klearu-llm model/mlp.rs): gate / up [intermediate][hidden],
 * down [hidden][intermediate] row-major f32 (host), stored bf16; down_bias
 * (nullable, klearu-dejavu mlp.rs:50-53) f32 [hidden]. */
KL_API kl_status kl_sparse_mlp_create(kl_ctx_t ctx, int hidden, int intermediate, const float* gate_host,
                                      const float* up_host, const float* down_host, const float* down_bias_host,
                                      kl_sparse_mlp_t* out);
KL_API kl_status kl_sparse_mlp_destroy(kl_sparse_mlp_t m);
/* sparse_mlp::forward_sparse (klearu-llm sparse/sparse_mlp.rs:4-37) for each
 * token: out[t] = down[:, sel[t]] . (silu(gate[sel[t]] . x[t]) * (up[sel[t]] . x[t]))
 * (+ bias).  x [n_tokens][hidden], sel [n_tokens][k] (uint32 neuron ids),
 * out [n_tokens][hidden]; all device. */
KL_API kl_status kl_sparse_mlp_forward(kl_sparse_mlp_t m, const float* x, int n_tokens, const uint32_t* sel, int k,
                                       float* out);

/* The MLP half of SparseModel::forward_decode_sparse
 * (crates/klearu-llm/src/sparse/mod.rs:112-141) over n_layers layers: for
 * each layer l, norm = RMSNorm_l(hidden) (model/rms_norm.rs: x / sqrt(mean(x^2)
 * + eps) * w, or * (1 + w) with one_plus_weight), idx = predictors[l]'s
 * select_top_k(norm, k) with k = ceil(intermediate * neuron_sparsity)
 * (mod.rs:121-125), hidden += sparse_mlp_l(norm, idx).  Attention, embedding,
 * the final norm and the LM head are outside this engine: `hidden` is the
 * residual stream the caller's attention writes.  The predictor and MLP
 * handles are borrowed (they must outlive the stack and share its context);
 * norm_weights_host is [n_layers][hidden] f32. */
typedef struct kl_ffn_stack_s* kl_ffn_stack_t;
KL_API kl_status kl_ffn_stack_create(kl_ctx_t ctx, int n_layers, const kl_predictor_t* predictors_host,
                                     const kl_sparse_mlp_t* mlps_host, const float* norm_weights_host, float eps,
                                     int one_plus_weight, kl_ffn_stack_t* out);
KL_API kl_status kl_ffn_stack_destroy(kl_ffn_stack_t s);
/* hidden [n_tokens][hidden] (device f32), updated in place.  The second call
 * with the same (hidden pointer, n_tokens, k) captures the per-layer launches
 * in a CUDA graph, later calls replay it. */
KL_API kl_status kl_ffn_stack_decode(kl_ffn_stack_t s, float* hidden, int n_tokens, float neuron_sparsity);

/* ------------------------------------------------------------------------ */
/* Datasets: LibSVM / XML files and shuffled CSR batches (host memory).      */
/* These calls take no context; on failure kl_last_error(NULL) returns the   */
/* message (parse errors name the 1-based line, as the reference does).      */
/* ------------------------------------------------------------------------ */
/* LibSvmDataset::load (crates/klearu-core/src/data/libsvm.rs:31-36): parse a
 * file of "l1,l2,... idx:val idx:val ..." lines on `threads` host threads
 * (<= 0: all).  1-based indices are detected over the whole file (minimum
 * index 1, no index 0) and shifted; indices >= feature_dim are clamped to
 * feature_dim - 1; each row is sorted by index with duplicates summed
 * (SparseVector::from_pairs, tensor/sparse.rs:36-57).  KL_EINVAL on a
 * malformed line, with the reference's messages (libsvm.rs:127-185). */
KL_API kl_status kl_libsvm_load(const char* path, int64_t feature_dim, int64_t num_labels, int threads,
                                kl_dataset_t* out);
/* LibSvmDataset::load_from_reader (libsvm.rs:39-111) over an in-memory text. */
KL_API kl_status kl_libsvm_parse(const char* text_host, size_t len, int64_t feature_dim, int64_t num_labels,
                                 int threads, kl_dataset_t* out);
/* LibSvmDataset::from_examples (libsvm.rs:114-124): a dataset over CSR arrays
 * (rows already sorted and unique), copied. */
KL_API kl_status kl_dataset_from_csr(const int64_t* rowptr_host, const uint32_t* idx_host, const float* val_host,
                                     const int64_t* label_ptr_host, const uint32_t* labels_host, int64_t n,
                                     int64_t feature_dim, int64_t num_labels, kl_dataset_t* out);
KL_API kl_status kl_dataset_destroy(kl_dataset_t ds);
/* Dataset::len / feature_dim / num_labels (data/dataset.rs:19-35), plus the
 * total feature and label counts. */
KL_API kl_status kl_dataset_info(kl_dataset_t ds, int64_t* len_host, int64_t* feature_dim_host,
                                 int64_t* num_labels_host, int64_t* nnz_host, int64_t* nlabels_host);
/* Dataset::get (dataset.rs:29) for every example at once: the store's CSR
 * arrays (rowptr / label_ptr [len+1]), valid while the dataset lives. */
KL_API kl_status kl_dataset_csr(kl_dataset_t ds, const int64_t** rowptr, const uint32_t** idx, const float** val,
                                const int64_t** label_ptr, const uint32_t** labels);
/* BatchIterator::new (dataset.rs:48-56): the example order is the SplitMix64
 * Fisher-Yates shuffle of the reference (dataset.rs:60-87) for `seed`.  With
 * `prefetch` a worker thread assembles the next batch while the caller trains
 * on the current one.  The dataset must outlive the iterator. */
KL_API kl_status kl_batch_iter_create(kl_dataset_t ds, int batch_size, uint64_t seed, int prefetch,
                                      kl_batch_iter_t* out);
/* BatchIterator::reset (dataset.rs:58-68): reshuffle from the identity order. */
KL_API kl_status kl_batch_iter_reset(kl_batch_iter_t it, uint64_t seed);
/* Iterator::next (dataset.rs:94-111): the next batch_size examples in
 * shuffled order (the last batch short) as a kl_batch of HOST arrays in
 * page-locked memory, ready for kl_net_train_step_host; nnz / nlabels are
 * filled.  The arrays stay valid until the next call on the iterator.  At the
 * end of the epoch it returns KL_OK with batch_host->batch == 0. */
KL_API kl_status kl_batch_iter_next(kl_batch_iter_t it, kl_batch* batch_host);
KL_API kl_status kl_batch_iter_destroy(kl_batch_iter_t it);

#ifdef __cplusplus
}
#endif
#endif /* KLEARU_GPU_H */
