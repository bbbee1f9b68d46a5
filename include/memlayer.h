/*
 * memlayer.h -- C ABI of the B200 (sm_100a) product-key memory layer.
 *
 * Drop-in boundary for the memory layer of KumarDev7/model:
 *   - memlayer_pool_forward   replaces MemoryPool.__call__
 *                             (memory_pool_model/memory.py:119-227);
 *   - memlayer_layer_forward  replaces the memory-layer block of
 *                             MemoryPoolLM.__call__ (memory_pool_model/model.py:108-120):
 *                             router Dense -> MemoryPool -> silu(Dense) gate -> Dense.
 * A jax.ffi handler (or any other host) binds these symbols directly.
 *
 * Conventions
 *   - Every pointer in the argument structs is a device pointer unless its
 *     comment says otherwise.  All float tensors are float32, row-major,
 *     contiguous and 16-byte aligned; the value table may be float32,
 *     float16 or bfloat16.
 *   - The library allocates nothing on these paths: the caller passes a
 *     device workspace of at least memlayer_*_workspace_size() bytes, 256-byte
 *     aligned.  The workspace's contents need not be initialised.
 *   - Calls are stream-ordered on the given cudaStream_t (passed as void*),
 *     return as soon as the work is enqueued and never synchronise the device.
 *     A large call may run part of its work on a stream the library keeps per
 *     device (ordered by events); the given stream waits for that work before
 *     the call's last launch, so ordering on the given stream is unchanged.
 *   - No C++ exception crosses this boundary; errors are memlayer_status codes.
 *     Argument errors are detected on the host before anything is enqueued.
 *   - Thread safety: calls on different streams may run concurrently from
 *     different host threads as long as they use different workspaces and
 *     output buffers.
 */
#ifndef MEMLAYER_H_
#define MEMLAYER_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MEMLAYER_ABI_VERSION 1

typedef enum {
  MEMLAYER_OK = 0,
  MEMLAYER_ERR_BAD_SHAPE = 1,     /* a dimension is out of range or inconsistent */
  MEMLAYER_ERR_BAD_POINTER = 2,   /* a required pointer is NULL or misaligned */
  MEMLAYER_ERR_UNSUPPORTED = 3,   /* a valid reference setting this build does not implement */
  MEMLAYER_ERR_WORKSPACE = 4,     /* workspace missing or smaller than required */
  MEMLAYER_ERR_CUDA = 5,          /* a CUDA launch or runtime call failed */
  MEMLAYER_ERR_PEER_TIMEOUT = 6   /* a bounded wait on another GPU gave up */
} memlayer_status;

typedef enum {
  MEMLAYER_F32 = 0,
  MEMLAYER_F16 = 1,
  MEMLAYER_BF16 = 2
} memlayer_dtype;

/* The MemoryPool fields (memory.py:72-97, config.py:35-59) plus the call's
 * leading size.  d_model is used only by memlayer_layer_forward. */
typedef struct {
  int64_t tokens;                /* M: product of the queries' leading dims */
  int32_t heads;                 /* pool_heads (H) */
  int32_t n_sub_keys;            /* n; the pool has n*n slots */
  int32_t d_key;                 /* even; each half has d_key/2 dims */
  int32_t d_value;               /* d */
  int32_t top_k;                 /* k, 1 <= k <= min(n, 32) */
  int32_t d_model;               /* hidden size for the layer entry */
  int32_t values_dtype;          /* memlayer_dtype of the value table */
  float routing_noise;           /* scale of the Gumbel selection noise */
  float min_temperature;         /* clamp of exp(log_temperature) */
  float max_temperature;
  int32_t query_scale;           /* scale scores by |q_half| / sqrt(d_key/2) */
  int32_t balance_temperature_grad; /* P uses the full scores (with q_len) */
} memlayer_config;

/* Optional stage timestamps for profiling: cudaEvent_t handles (as void*)
 * that the call records on its stream at fixed stage boundaries.  NULL
 * entries are skipped.  Boundaries:
 *   0 start                       3 after score GEMM + per-half top-k
 *   1 after router / gate GEMMs   4 after k*k combine + softmax + gather
 *   2 after key / query prep      5 end (stats, output projection done)   */
#define MEMLAYER_STAGE_EVENTS 6
typedef struct {
  void* events[MEMLAYER_STAGE_EVENTS];
} memlayer_stage_events;

/* Per-call inputs/outputs of MemoryPool.__call__. */
typedef struct {
  /* inputs */
  const float* queries;          /* [M, H, d_key] router queries */
  const float* sub_keys;         /* [H, 2, n, d_key/2] (normalised inside, as memory.py:139) */
  const float* log_temperature;  /* [1] */
  const void* values;            /* [n*n, d] of values_dtype; 16-byte aligned */
  const float* gumbel;           /* [M, H, 2, n] standard Gumbel sample, or NULL */
  float noise_scale;             /* multiplies routing_noise (memory.py:158) */
  int32_t train;                 /* selection noise is applied only when train != 0 */
  int32_t shuffle_reads;         /* read (slot + N/2 + 1) % N (memory.py:179) */
  /* outputs */
  float* out;                    /* [M, d] */
  int32_t* slots;                /* [M, H, k] */
  float* weights;                /* [M, H, k] */
  /* optional aux outputs (NULL = not computed) */
  float* queries_unit;           /* [M, H, 2, d_key/2] aux["queries"] */
  float* subkey_counts;          /* [H, 2, n] */
  float* slot_counts;            /* [n*n] */
  float* balance_loss;           /* [1] */
  float* top1_weight;            /* [1] */
  float* temperature;            /* [1] */
  const memlayer_stage_events* stage_events;  /* optional profiling hook, or NULL */
} memlayer_pool_args;

/* Per-call inputs/outputs of the memory-layer block (model.py:108-120):
 *   q   = h @ w_router + b_router                      (router_i)
 *   mem = MemoryPool(q)                                (pool)
 *   y   = (mem * silu(h @ w_gate + b_gate)) @ w_out + b_out   (mem_gate_i, mem_out_i)
 * y is the term the reference adds into the residual-stream update. */
typedef struct {
  const float* h;                /* [M, d_model] layer-normalised hidden state */
  const float* w_router;         /* [d_model, H*d_key] */
  const float* b_router;         /* [H*d_key] or NULL (zero bias) */
  const float* w_gate;           /* [d_model, d] */
  const float* b_gate;           /* [d] or NULL */
  const float* w_out;            /* [d, d_model] */
  const float* b_out;            /* [d_model] or NULL */
  float* y;                      /* [M, d_model] output */
  float* mem;                    /* [M, d] pool output before the gate, or NULL */
  memlayer_pool_args pool;       /* pool.queries is ignored (computed from h);
                                    pool.out may be NULL */
} memlayer_layer_args;

/* ABI version of the loaded library (MEMLAYER_ABI_VERSION at build time). */
int32_t memlayer_abi_version(void);

/* Human-readable name of a status code (static storage). */
const char* memlayer_status_string(int32_t status);

/* Diagnostics: number of kernels this library has launched in this process
 * (all devices, all threads).  Has no counterpart in the reference. */
int64_t memlayer_kernel_launch_count(void);

/* Bytes of device workspace memlayer_pool_forward needs for cfg. */
int32_t memlayer_pool_workspace_size(const memlayer_config* cfg, size_t* bytes);

/* MemoryPool.__call__ (memory.py:119-227).  Reference interface replaced:
 * memory_pool_model/memory.py:119 `MemoryPool.__call__(queries, *, train,
 * sparse_grad, noise_scale, shuffle_reads) -> (out, aux)`; sparse_grad only
 * affects differentiation and has no forward effect. */
int32_t memlayer_pool_forward(const memlayer_config* cfg, const memlayer_pool_args* args,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of device workspace memlayer_layer_forward needs for cfg. */
int32_t memlayer_layer_workspace_size(const memlayer_config* cfg, size_t* bytes);

/* Memory-layer block of MemoryPoolLM.__call__ (model.py:108-120).
 * Reference interface replaced: model.py:110-119 (router_i Dense, pool call,
 * mem_gate_i / mem_out_i Dense) inside each layer in cfg.memory_layers. */
int32_t memlayer_layer_forward(const memlayer_config* cfg, const memlayer_layer_args* args,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Most chunks memlayer_layer_forward_host splits a call into. */
#define MEMLAYER_HOST_MAX_CHUNKS 16

/* Bytes of device workspace memlayer_layer_forward_host needs. */
int32_t memlayer_layer_host_workspace_size(const memlayer_config* cfg, int32_t chunks, size_t* bytes);

/* memlayer_layer_forward with the hidden state and the output in HOST
 * memory (args->h, args->y; pinned memory lets the copies overlap).  The
 * tokens are split into `chunks` (at most MEMLAYER_HOST_MAX_CHUNKS, fewer
 * when a chunk would hold under 256 tokens); the copy of chunk c+1 in, the
 * layer on chunk c and the copy of chunk c-1 out run concurrently on two
 * copy streams the library keeps per device and on `stream`, which covers
 * the whole call when it returns (synchronise it before reading y).  The
 * other pointers are device pointers as in memlayer_layer_forward;
 * subkey_counts, slot_counts, balance_loss and top1_weight must be NULL.
 * Same reference interface as memlayer_layer_forward (model.py:110-119),
 * for callers whose activations live on the host. */
int32_t memlayer_layer_forward_host(const memlayer_config* cfg, const memlayer_layer_args* args, int32_t chunks,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Device-side status of the last call that used this workspace: 0, or a
 * code recorded by a kernel (a bounded wait that gave up, an out-of-range
 * sub-key id).  Copies one word to the host and synchronises `stream`.
 * Has no counterpart in the reference (its errors are Python exceptions). */
int32_t memlayer_workspace_status(const memlayer_config* cfg, const void* workspace, int32_t* code, void* stream);

/* memlayer_layer_forward for a call whose sub-key normalisation and
 * Dense-kernel preparation already ran on this workspace: the previous call
 * on `workspace` was memlayer_layer_forward (or this function) with the
 * same cfg, sub_keys, log_temperature, Dense kernels and biases, unchanged
 * since.  Only the hidden state and what follows from it are recomputed;
 * results equal memlayer_layer_forward's.  For decode loops (one call per
 * generated token on fixed weights; no counterpart in the reference, whose
 * jitted step recomputes everything).  Single GPU.  Returns
 * MEMLAYER_ERR_WORKSPACE, before launching anything, when the last
 * successful memlayer_layer_forward on `workspace` had another cfg or other
 * sub-key, temperature or Dense-kernel pointers (in-place changes of those
 * buffers are the caller's to track). */
int32_t memlayer_layer_forward_prepared(const memlayer_config* cfg, const memlayer_layer_args* args, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* ---- Row-sharded value table over the GPUs of one node -------------------
 * No counterpart in the reference, which replicates every parameter,
 * the value table included, on each device of its data-parallel mesh
 * (memory_pool_model/train.py:229-236,267); these calls serve tables larger
 * than one GPU.  One process per GPU; slot s lives on rank s % world as its
 * local row s / world (memlayer_shard_rows gives each rank's row count).
 * Sub-keys and the Dense kernels are replicated.  Each rank routes its own
 * tokens; a forward is three phases per rank:
 *   ROUTE   routing + stage 2; (local row, weight) entries are stored into
 *           the owner ranks' inboxes over NVLink;
 *   GATHER  each owner gathers its rows for every rank's tokens and stores
 *           one float32 partial row per (token, owner) into the token
 *           owner's buffer;
 *   REDUCE  the token owner adds the partials in rank order (deterministic),
 *           then gate and output projection (layer entry).
 * A call with MEMLAYER_PHASE_ALL runs all three.  Ranks hand over through
 * flags in each other's buffers, with bounded waits (about 2 s): a wait that
 * gives up records code 31/32 in the workspace status word and skips its
 * work.  Calling the phases separately lets one process drive several
 * communicators on one GPU (all ranks' ROUTE, then all GATHER, then all
 * REDUCE, on one stream), where waits never depend on later launches. */
#define MEMLAYER_MAX_SHARDS 8
#define MEMLAYER_IPC_HANDLE_BYTES 64

typedef struct memlayer_shard_comm memlayer_shard_comm;

typedef enum {
  MEMLAYER_PHASE_ROUTE = 1,
  MEMLAYER_PHASE_GATHER = 2,
  MEMLAYER_PHASE_REDUCE = 4,
  MEMLAYER_PHASE_ALL = 7,
  /* Exchange in two token halves.  With all three phases in one call, the
   * second half's push runs while the first half is gathered (on a stream
   * the library keeps per device, ordered by events) and the first half's
   * reduce while the second is gathered; `stream` covers the whole call.
   * Every rank must pass the same flag in the same call. */
  MEMLAYER_PHASE_SPLIT = 8
} memlayer_shard_phase;

/* Value rows held by `rank`: the slots s < pool_size with s % world == rank. */
int64_t memlayer_shard_rows(int64_t pool_size, int32_t rank, int32_t world);

/* Create this rank's communicator on the current device, sized for cfg
 * (cfg->tokens = the most tokens any rank passes in one call).  Every rank
 * must pass the same cfg: ranks address each other's buffers with their own
 * offsets.  Allocates
 * and zeroes one device buffer (inboxes, partial rows, flags); this is the
 * only allocation of the sharded path and happens here, not per call. */
int32_t memlayer_shard_comm_create(const memlayer_config* cfg, int32_t rank, int32_t world,
                                   memlayer_shard_comm** comm);

/* The communicator's rank, world size, CUDA device ordinal and buffer
 * bytes (any pointer may be NULL). */
int32_t memlayer_shard_comm_info(const memlayer_shard_comm* comm, int32_t* rank, int32_t* world, int32_t* device,
                                 size_t* bytes);

/* CUDA IPC handle (MEMLAYER_IPC_HANDLE_BYTES bytes, host memory) of this
 * rank's buffer, to be all-gathered by the caller (for instance with
 * torch.distributed.all_gather_object). */
int32_t memlayer_shard_comm_ipc_handle(const memlayer_shard_comm* comm, void* handle);

/* Map every other rank's buffer: handles = world consecutive handles in
 * rank order (host memory; this rank's own entry is ignored). */
int32_t memlayer_shard_comm_open_peers(memlayer_shard_comm* comm, const void* handles);

/* Use another communicator of this process (same device, or a device with
 * peer access enabled) as rank `peer` instead of an IPC mapping. */
int32_t memlayer_shard_comm_set_peer(memlayer_shard_comm* comm, int32_t peer, const memlayer_shard_comm* other);

/* Budget of every wait on another rank in this communicator's calls, in
 * nanoseconds of the GPU's global timer (default 2 s; 1 us .. 60 s).  A wait
 * that runs out records its code (31-36) in the workspace status word and
 * makes the call's later waits give up at once, so a rank that never
 * arrives leaves its peers with an error status, not a hang.  No counterpart
 * in the reference. */
int32_t memlayer_shard_comm_set_wait_budget(memlayer_shard_comm* comm, int64_t nanoseconds);

/* Unmap the peers and free the buffer (after all calls have completed). */
int32_t memlayer_shard_comm_destroy(memlayer_shard_comm* comm);

/* Workspace bytes of the sharded forward (layer != 0: layer entry). */
int32_t memlayer_shard_workspace_size(const memlayer_config* cfg, int32_t world, int32_t layer, size_t* bytes);

/* Sharded MemoryPool.__call__ / memory-layer block: same arguments as
 * memlayer_pool_forward / memlayer_layer_forward, with `values` = this
 * rank's local rows [memlayer_shard_rows(n*n, rank, world), d] (16-byte
 * aligned, d a multiple of 4).  cfg must match the communicator's shapes,
 * with cfg->tokens no larger than its capacity.  slot_counts /
 * subkey_counts / balance_loss / top1_weight cover this rank's tokens.
 * Pass the same workspace to every phase of one call. */
int32_t memlayer_pool_forward_sharded(const memlayer_config* cfg, const memlayer_pool_args* args,
                                      memlayer_shard_comm* comm, int32_t phases, void* workspace,
                                      size_t workspace_bytes, void* stream);
int32_t memlayer_layer_forward_sharded(const memlayer_config* cfg, const memlayer_layer_args* args,
                                       memlayer_shard_comm* comm, int32_t phases, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* ---- Row-sharded forward with a staged exchange ---------------------------
 * The same row-sharded layer with the exchange left to the caller's
 * collective library (NCCL's all-gather and reduce-scatter, for instance),
 * run on the same stream between the phases; no communicator, no peer
 * memory.  The data-parallel step it stands beside is the reference's
 * all-gather of replicated tables (memory_pool_model/train.py:196-197); the
 * row-sharded table itself has no counterpart in the reference.
 *   ROUTE   projections and routing of this rank's M tokens: slots and
 *           weights into args->pool.slots / weights [M, H, k]; the gate
 *           stays in the workspace;
 *   (caller: all-gather every rank's slots and weights, rank-major, into
 *    all_slots / all_weights [world, M, H, k])
 *   GATHER  for every token of every rank, the sum of w * V[row] over the
 *           entries this rank owns (slot % world == rank; read slots under
 *           shuffle_reads) -> partials [world, M, d], zero rows included;
 *   (caller: reduce-scatter (sum) partials into mem [M, d])
 *   REDUCE  gate and output projection from mem -> y (and mem into
 *           args->mem / pool.out when given).
 * Every rank passes the same cfg (cfg->tokens = M on every rank) and the
 * same workspace to every phase of one call (memlayer_layer_workspace_size
 * bytes).  values = this rank's local rows, as for the sharded forward.
 * Partial rows are bit-identical to the peer-store exchange's; the sum over
 * owners follows the collective's order. */
typedef struct {
  const int32_t* all_slots;      /* [world][M, H, k] every rank's slots, rank-major */
  const float* all_weights;      /* [world][M, H, k] */
  int64_t route_stride;          /* elements from one rank's block of all_slots / all_weights to the
                                    next (0: M*H*k); lets one all-gather move slots and weights
                                    packed as [world][2][M*H*k] */
  float* partials;               /* [world, M, d] output of GATHER, 16-byte aligned */
  const float* mem;              /* [M, d] input of REDUCE: the reduce-scattered partials */
  int32_t rank, world;
} memlayer_staged_args;

int32_t memlayer_layer_forward_staged(const memlayer_config* cfg, const memlayer_layer_args* args,
                                      const memlayer_staged_args* staged, int32_t phases, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* ---- Fetched-row gradients and row-wise Adagrad (training) ---------------
 * With sparse_grad the value table gets no dense gradient; the trainer
 * reads dL/d(read output) from zero "probes" added to each read
 * (model.py:114-115) and turns it into per-row gradients of the fetched
 * rows only.  One read = one memory layer's call on the shared pool. */
#define MEMLAYER_MAX_READS 8

typedef struct {
  const int32_t* slots;          /* [tokens, H, k] the read's aux["slots"] */
  const float* weights;          /* [tokens, H, k] the read's aux["weights"] */
  const float* grad;             /* [tokens, d] dL/d(read output), 16-byte aligned */
  int64_t tokens;
} memlayer_read;

/* Workspace bytes for `fetches` = sum over the reads of tokens * H * k. */
int32_t memlayer_rowgrad_workspace_size(const memlayer_config* cfg, int64_t fetches, size_t* bytes);

/* fetched_row_grads + _merge_rows (memory_pool_model/train.py:146-172):
 * uniq [cap] = the distinct fetched slots in ascending order, padded with
 * n*n; rows [cap, d] = for each, the sum over its fetches of w * grad[token]
 * (zero rows for the padding); cap = min(fetches, n*n).  Fetches of every
 * slot are summed in fetch order (reads in argument order, then token,
 * head, rank), so results are deterministic.  rows, n_unique [1] and
 * sq_norm [1] (sum of rows^2, for the global-norm clip) may be NULL.
 * cfg supplies heads, top_k, n_sub_keys and d_value (tokens is ignored). */
int32_t memlayer_fetched_row_grads(const memlayer_config* cfg, const memlayer_read* reads, int32_t n_reads,
                                   int32_t* uniq, float* rows, int32_t* n_unique, float* sq_norm,
                                   void* workspace, size_t workspace_bytes, void* stream);

typedef struct {
  float* values;                 /* [n*n, d] float32 value table, updated in place */
  float* accum;                  /* [n*n] Adagrad accumulator (the trainer's pool_v), updated in place */
  float lr;                      /* schedule(step) * pool_lr_mult */
  float grad_clip;               /* global-norm clip threshold (train.py grad_clip) */
  const float* rest_sq_norm;     /* [1] squared norm of all other gradients, or NULL for 0 */
  float* clip_scale;             /* [1] optional output: min(1, clip / (norm + 1e-6)) */
  int32_t* n_unique;             /* [1] optional output: touched rows */
} memlayer_adagrad_args;

/* Row-wise Adagrad on the fetched rows (train.py:378-383 clip by the
 * global norm of both parts, :396-399 update): with g = scale * row grad,
 * accum[s] += mean(g^2); values[s] -= lr / (sqrt(accum[s]) + 1e-8) * g,
 * for every touched slot s only.  Float32 tables only. */
int32_t memlayer_row_adagrad(const memlayer_config* cfg, const memlayer_read* reads, int32_t n_reads,
                             const memlayer_adagrad_args* args, void* workspace, size_t workspace_bytes,
                             void* stream);

/* ---- Value table in page-locked host memory (the host tier) -------------
 * memory.py:180-183 with host_pool.fetch (host_pool.py:206-220): the value
 * table lives off the GPU (a pool larger than HBM) and only the fetched rows
 * come in.  args->values points to page-locked host memory the device can
 * read (cudaHostAlloc / cudaMallocHost, or cudaHostRegister with
 * cudaHostRegisterMapped; device memory also works).  The GPU routes the
 * tokens, removes duplicate read slots, copies each distinct row once from
 * host memory into the workspace and mixes from there: outputs, slots,
 * weights and statistics are those of memlayer_pool_forward on the same
 * table, bit for bit.  Same arguments as memlayer_pool_forward; the
 * workspace holds a staging copy of up to min(tokens * H * k, n*n) rows. */
int32_t memlayer_host_table_workspace_size(const memlayer_config* cfg, size_t* bytes);
int32_t memlayer_pool_forward_host_table(const memlayer_config* cfg, const memlayer_pool_args* args, void* workspace,
                                         size_t workspace_bytes, void* stream);

/* ---- Sub-key maintenance (training) -------------------------------------
 * cfg supplies heads, n_sub_keys and d_key (tokens and d_value are
 * checked but unused).  sub_keys is [H, 2, n, d_key/2] float32. */

/* Workspace bytes of memlayer_key_diversity. */
int32_t memlayer_key_diversity_workspace_size(const memlayer_config* cfg, size_t* bytes);

/* key_diversity_loss (memory_pool_model/memory.py:230-240): loss [1] = mean
 * over codebooks and ordered pairs i != j of the squared cosine of the
 * l2-normalised sub-keys; grad [H, 2, n, d_key/2] = grad_scale * d loss /
 * d sub_keys (the trainer adds key_diversity_coef * loss, train.py:327-329,
 * so grad_scale = key_diversity_coef gives its gradient).  Either output
 * may be NULL, not both.  n = 1 gives NaN, as the reference's 0/0. */
int32_t memlayer_key_diversity(const memlayer_config* cfg, const float* sub_keys, float* loss, float* grad,
                               float grad_scale, void* workspace, size_t workspace_bytes, void* stream);

typedef struct {
  float* sub_keys;               /* [H, 2, n, d_key/2], updated in place */
  float* usage;                  /* [H, 2, n] EMA usage (rows sum to 1), updated in place */
  const float* queries;          /* [query_tokens, H, 2, d_key/2] unit query halves (aux["queries"]) */
  int64_t query_tokens;          /* >= 1 */
  const int32_t* pick;           /* [H, 2, n] token drawn for each key (randint(0, query_tokens)) */
  const float* noise;            /* [H, 2, n, d_key/2] standard normal draws */
  float threshold;               /* dead when usage < threshold / n (train.py revive_threshold) */
  float noise_scale;             /* the reference's `noise` argument (default 0.05) */
  int32_t* dead;                 /* [H, 2, n] optional output: 1 where revived */
  float* moment0;                /* optional [H, 2, n, d_key/2] optimiser moments of sub_keys, */
  float* moment1;                /*   zeroed on revived rows (train.py:497-509), or NULL */
} memlayer_revive_args;

/* revive_dead_keys (memory_pool_model/memory.py:243-281) with the random
 * draws passed in (the reference draws pick and noise from its rng inside
 * the call): a dead key becomes l2_normalize(queries[pick, h, c] +
 * noise_scale * noise), its usage 1/n, and each [h, c] usage row is divided
 * by its sum.  A pick outside [0, query_tokens) is wrapped once if negative
 * and then clamped, as the reference's gather does. */
int32_t memlayer_revive_dead_keys(const memlayer_config* cfg, const memlayer_revive_args* args, void* stream);

/* ---- Layer backward (training) --------------------------------------------
 * Gradients of sum(dy * y) + balance_coef * balance_loss through one memory
 * layer (model.py:110-119 with memory.py:133-214), as the reference trainer's
 * jax.value_and_grad computes them with sparse_grad: the value table gets no
 * gradient; its rows' gradient is the read-output gradient `probe`
 * (model.py:114-115), the input of memlayer_fetched_row_grads.  Routing
 * (the forward's slots, weights and clean top-k counts) carries no gradient;
 * the temperature clamp is straight-through.  Outputs may be NULL. */
typedef struct {
  const float* dy;               /* [M, d_model] d loss / d y (model.py:119's term) */
  float balance_coef;            /* the trainer's balance_coef (train.py:328); 0: no balance term */
  int32_t route_through_pool;    /* the gate reads stop_gradient(h) (model.py:116-117) */
  const void* forward_workspace; /* the forward call's workspace, unchanged since (its clean top-k
                                    counts feed the balance term); needed when balance_coef != 0 */
  float* dh;                     /* [M, d_model] */
  float* dw_router;              /* [d_model, H*d_key] */
  float* db_router;              /* [H*d_key] */
  float* dsub_keys;              /* [H, 2, n, d_key/2] */
  float* dlog_temperature;       /* [1] */
  float* dw_gate;                /* [d_model, d] */
  float* db_gate;                /* [d] */
  float* dw_out;                 /* [d, d_model] */
  float* db_out;                 /* [d_model] */
  float* probe;                  /* [M, d] d loss / d read output */
} memlayer_layer_grads;

/* Workspace bytes of memlayer_layer_backward (balance != 0: with the balance term). */
int32_t memlayer_layer_backward_workspace_size(const memlayer_config* cfg, int32_t balance, size_t* bytes);

/* `args` = the forward's layer arguments (h, Dense kernels and biases,
 * sub_keys, log_temperature, values, its slots / weights outputs, and
 * balance_loss non-NULL when balance_coef != 0); args->mem, when non-NULL,
 * still holds the forward's read output, which the routing backward then
 * reads instead of re-gathering it.  d_key/2 must be a multiple of 4 and at
 * most 128.  Every GEMM runs on this library's tensor-core kernels inside
 * the caller's workspace: backward calls on one device may overlap. */
int32_t memlayer_layer_backward(const memlayer_config* cfg, const memlayer_layer_args* args,
                                const memlayer_layer_grads* grads, void* workspace, size_t workspace_bytes,
                                void* stream);

/* The same backward on a row-sharded table (model.py:110-119 with
 * memory.py:133-214 under the reference trainer's data parallelism,
 * train.py:229-236, with the table split over the ranks as in
 * memlayer_layer_forward_sharded): call it after that forward on `comm`, once
 * per forward, with the forward's `args` (`mem`, else `pool.out`, holding its
 * read output).  Each rank publishes its probe rows; each owner returns
 * probe . row for every read of its rows (the forward's inbox entries: no
 * value row crosses NVLink); the rest is local.  Phases as the forward's:
 * ROUTE = projections, probe published; GATHER = this owner's dots; REDUCE =
 * routing backward from the owners' dots, then the Dense, sub-key and
 * temperature gradients of this rank's tokens, which the caller sums over
 * the ranks as data-parallel training does.  Every rank runs every phase;
 * waits are bounded (status 35: probe rows, 36: dots).  One workspace of
 * memlayer_layer_backward_workspace_size bytes serves every phase of a call. */
int32_t memlayer_layer_backward_sharded(const memlayer_config* cfg, const memlayer_layer_args* args,
                                        const memlayer_layer_grads* grads, memlayer_shard_comm* comm,
                                        int32_t phases, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Owner-sharded row update (row-sharded table, training) -------------
 * Replaces fetched_row_grads_sharded + the replicated update
 * (memory_pool_model/train.py:175-206, 378-399): with the table row-sharded
 * as in memlayer_layer_forward_sharded (slot s on rank s % world, local row
 * s / world), each rank merges its own fetches, pushes every merged row to
 * its owner over NVLink, the owner merges the rows of all ranks in rank
 * order, and the global-norm clip (sum over every owner's rows, identical on
 * all ranks) and row-wise Adagrad update the owner's rows only.  Phases
 * (memlayer_shard_phase): ROUTE = local merge + push, GATHER = owner merge +
 * publish of its squared norm, REDUCE = clip + Adagrad; waits are bounded
 * (status 33: inbox, 34: norm partials).  Float32 tables only. */

/* Communicator for the row update: cfg->tokens = the most tokens of one read
 * on any rank, n_reads = memory layers sharing the pool.  Wire the peers as
 * for memlayer_shard_comm_create (ipc_handle / open_peers or set_peer,
 * destroy); forward calls reject it. */
int32_t memlayer_shard_comm_create_rowgrad(const memlayer_config* cfg, int32_t n_reads, int32_t rank, int32_t world,
                                           memlayer_shard_comm** comm);

/* Workspace bytes of memlayer_row_adagrad_sharded for `fetches` = sum over
 * this rank's reads of tokens * H * k. */
int32_t memlayer_shard_rowgrad_workspace_size(const memlayer_shard_comm* comm, int64_t fetches, size_t* bytes);

/* One row-update step on this rank: reads = this rank's reads (tokens of
 * this rank); args->values / args->accum = this rank's rows
 * [memlayer_shard_rows(n*n, rank, world), d] / [rows]; clip_scale = the
 * global scale (same on every rank); n_unique = local rows this rank
 * updated.  rest_sq_norm must be the same on every rank.  Every rank calls
 * every step with the same phases; pass the same reads and workspace to
 * every phase of one step. */
int32_t memlayer_row_adagrad_sharded(const memlayer_config* cfg, const memlayer_read* reads, int32_t n_reads,
                                     const memlayer_adagrad_args* args, memlayer_shard_comm* comm, int32_t phases,
                                     void* workspace, size_t workspace_bytes, void* stream);

/* ---- The language model around the memory layer -------------------------
 * MemoryPoolLM (memory_pool_model/model.py:15-127) in inference form and its
 * decode step with a key / value cache (generate.py:23-65): token and
 * position embeddings; per layer LayerNorm -> causal multi-head attention ->
 * residual, LayerNorm -> feed-forward (Dense, GELU, Dense) or, in the memory
 * layers, the memory-layer block (memlayer_layer_forward on the shared pool;
 * both when memory_ffn) -> residual; final LayerNorm and tied logits.
 * Dropout is the identity (inference).  LayerNorm is flax's (epsilon 1e-6,
 * variance E[x^2] - E[x]^2), GELU its tanh form, attention scales the query
 * by 1/sqrt(head_dim).  head_dim = d_model / n_heads must be 32 or 64;
 * d_model one of 32, 64, 128, 256, 512, 1024.  The status of a model call (token ids out of range: 26,
 * and the memory layers' codes) is read with memlayer_workspace_status(&cfg->pool,
 * workspace, ...). */
#define MEMLAYER_MAX_LAYERS 32

typedef struct {
  int32_t vocab_size, max_len, d_model, n_layers, n_heads, ffn_mult;
  uint32_t memory_layers;        /* bit i set: layer i reads the pool (config.py:31) */
  int32_t memory_ffn;            /* memory layers keep their feed-forward (config.py:36) */
  memlayer_config pool;          /* the shared pool's fields; tokens is ignored, d_model must match */
} memlayer_model_config;

/* One layer's parameters, float32, row-major; Dense kernels as [in, out].
 * The flax attention parameters map as: w_qkv = [query | key | value]
 * kernels [d_model, H, head_dim] reshaped to [d_model, d_model] and
 * concatenated along the columns (b_qkv likewise); w_attn_out = the out
 * kernel [H, head_dim, d_model] reshaped to [d_model, d_model]. */
typedef struct {
  const float *ln_attn_scale, *ln_attn_bias;    /* [d_model] ln_attn_i */
  const float *w_qkv, *b_qkv;                   /* [d_model, 3*d_model], [3*d_model] attn_i */
  const float *w_attn_out, *b_attn_out;         /* [d_model, d_model], [d_model] */
  const float *ln_ffn_scale, *ln_ffn_bias;      /* [d_model] ln_ffn_i */
  const float *w_ffn_in, *b_ffn_in;             /* [d_model, F], [F]; F = d_model*ffn_mult (when used) */
  const float *w_ffn_out, *b_ffn_out;           /* [F, d_model], [d_model] */
  const float *w_router, *b_router;             /* memory layers: router_i, mem_gate_i, mem_out_i */
  const float *w_gate, *b_gate;
  const float *w_out, *b_out;
} memlayer_block_params;

typedef struct {
  const float* embedding;        /* [vocab_size, d_model] embed (also the tied output projection) */
  const float* pos_embed;        /* [max_len, d_model] */
  const memlayer_block_params* layers;   /* host array of n_layers entries */
  const float *ln_final_scale, *ln_final_bias;
  const float* sub_keys;         /* the shared pool: [H, 2, n, d_key/2] */
  const float* log_temperature;  /* [1] */
  const void* values;            /* [n*n, d] of pool.values_dtype */
} memlayer_model_params;

/* Workspace of memlayer_model_forward / memlayer_model_decode_step for
 * `tokens` rows (batch * seq for a forward, batch for a decode step). */
int32_t memlayer_model_workspace_size(const memlayer_model_config* cfg, int64_t tokens, size_t* bytes);

/* logits [batch, seq, vocab] of tokens [batch, seq] (int32, device), seq <= max_len. */
int32_t memlayer_model_forward(const memlayer_model_config* cfg, const memlayer_model_params* params,
                               const int32_t* tokens, int64_t batch, int64_t seq, float* logits, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Bytes of the key / value cache of `batch` rows: [n_layers][2][batch][max_len][d_model] float32. */
int32_t memlayer_model_cache_size(const memlayer_model_config* cfg, int64_t batch, size_t* bytes);

/* One decode step: tokens [batch] (device) at position *pos (device int32,
 * read on the GPU, so a captured CUDA graph can be replayed for every
 * position) -> logits [batch, vocab]; the step's keys and values are written
 * into `cache` at *pos, and the step attends to cache positions 0..*pos.  A
 * fresh cache need not be cleared: positions beyond *pos are never read. */
int32_t memlayer_model_decode_step(const memlayer_model_config* cfg, const memlayer_model_params* params,
                                   const int32_t* tokens, int64_t batch, const int32_t* pos, void* cache,
                                   float* logits, void* workspace, size_t workspace_bytes, void* stream);

/* Size of the library's built-in scratch array used by
 * memlayer_pool_forward_noalloc (64 MiB).  A device holds it from the moment
 * the library's code is loaded there -- with CUDA's default lazy module
 * loading, at the first memlayer_pool_forward_noalloc call on that device;
 * with eager loading (CUDA_MODULE_LOADING=EAGER), when the library is
 * loaded -- until the process exits. */
#define MEMLAYER_NOALLOC_SCRATCH_BYTES (64u << 20)

/* MemoryPool.__call__ for callers that cannot allocate or pass a device
 * workspace (for example a runtime whose custom-call operands are fixed at
 * compile time, or a per-token serving loop that must not enter the CUDA
 * allocator).  No counterpart in the reference.  Same arguments and results
 * as memlayer_pool_forward, but the workspace is the library's own fixed
 * array; the library allocates nothing.  Returns MEMLAYER_ERR_WORKSPACE when
 * memlayer_pool_workspace_size(cfg) exceeds MEMLAYER_NOALLOC_SCRATCH_BYTES.
 * The first call on a device (with it current) resolves the array's device
 * address; make it before any stream capture.  All calls share the array:
 * calls that can run concurrently on the GPU (unordered streams) race. */
int32_t memlayer_pool_forward_noalloc(const memlayer_config* cfg, const memlayer_pool_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MEMLAYER_H_ */
