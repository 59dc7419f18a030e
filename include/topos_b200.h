/*
 * topos_b200.h -- C ABI of the B200 execution backend for topos compiled plans.
 *
 * topos (crate `topos`, repository shergin/poorgrad) compiles a recorded graph
 * into a `Plan` (engine/plan.rs:97-283) and runs it node by node on the CPU
 * (`Plan::forward`, engine/plan.rs:514-640).  Acceleration enters through its
 * backend seam: a `Backend` variant with a `Manifest` (backend/manifest.rs:16-37)
 * whose `status()` reports `BackendUnavailable` (backend/backend.rs:168-204),
 * and per-task offers (`Elementary::gemm` / `map`, payload/elementary.rs:74-95)
 * that answer "declined" (`None`) or a result.
 *
 * This library is a new implementer behind that seam.  A whole compiled plan
 * (its node columns and the wanted/readable/required columns of `Plan::new`)
 * is handed over once; the library lowers it into a device program (fused
 * elementwise/broadcast/reduce kernels emitted per fusion group, row kernels,
 * gather/scatter, tcgen05 GEMMs), lays every materialized value out in one
 * liveness-planned device arena, and replays the program as a CUDA graph.
 *
 * Conventions (the reference's, kept):
 *  - Every call returns TB_OK (0) or an error code; the thread-local message of
 *    the last failure is `tb_last_error()`.
 *  - TB_DECLINED means "this backend does not serve the request"; the caller
 *    computes on its own path, exactly like a backend offer answering `None`.
 *  - A runtime failure poisons the library (backend/cuda/kernels/mod.rs:94-105):
 *    `tb_status` then answers TB_POISONED and every later call declines.
 *  - The caller owns host buffers; the library owns device memory and handles.
 *  - There is no CPU fallback inside the library: a missing device answers
 *    TB_PLATFORM_UNSUPPORTED from `tb_status` and an error from every call.
 */
#ifndef TOPOS_B200_H
#define TOPOS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes; 1..4 mirror `BackendUnavailable` (backend/backend.rs:168-204) */
enum {
  TB_OK = 0,
  TB_NOT_COMPILED = 1,          /* BackendUnavailable::NotCompiled */
  TB_PLATFORM_UNSUPPORTED = 2,  /* BackendUnavailable::PlatformUnsupported */
  TB_INITIALIZATION = 3,        /* BackendUnavailable::Initialization(msg) */
  TB_POISONED = 4,              /* BackendUnavailable::Poisoned(msg) */
  TB_DECLINED = 5,              /* the offer answers `None` */
  TB_INVALID = 6,               /* a malformed request (the reference panics) */
  TB_RUNTIME = 7                /* a CUDA / NCCL failure during a call */
};

/* ---- opcodes: `Function` variant order (function/function.rs:26-59) */
enum {
  TB_OP_LEAF = 0, TB_OP_PARAMETER, TB_OP_INPUT, TB_OP_ADD, TB_OP_SUB, TB_OP_MUL,
  TB_OP_DIV, TB_OP_NEG, TB_OP_TANH, TB_OP_EXP, TB_OP_LN, TB_OP_MATMUL,
  TB_OP_TRANSPOSE, TB_OP_SUM, TB_OP_SUM_ALONG, TB_OP_BROADCAST,
  TB_OP_BROADCAST_ALONG, TB_OP_RESHAPE, TB_OP_PERMUTE, TB_OP_NARROW, TB_OP_PAD,
  TB_OP_UNFOLD, TB_OP_FOLD, TB_OP_GATHER, TB_OP_SCATTER, TB_OP_LOG_SOFTMAX,
  TB_OP_LOG_SUM_EXP, TB_OP_SQRT, TB_OP_POWF, TB_OP_MAXIMUM, TB_OP_RELU,
  TB_OP_STEP, TB_OP_COUNT
};

/* ---- payload kinds: the storage representations (payload/storage.rs:36-51) */
enum { TB_PAYLOAD_NONE = 0, TB_PAYLOAD_DENSE = 1, TB_PAYLOAD_CONSTANT = 2, TB_PAYLOAD_SELECTION = 3 };

/* ---- numerics posture (backend/numerics.rs:25-43) */
enum { TB_NUMERICS_FAST = 0, TB_NUMERICS_EXACT = 1 };
/* Payload element types (`Tensor<f32>`, `Tensor<Bf16>`: payload/bf16.rs).  A bf16 network
 * rounds every payload operation's f32 result once to the nearest bf16 (ties to even,
 * bf16.rs:39-50) and accumulates products, sums, folds and scatters in f32 before one
 * rounding (tensor.rs:1015-1022, 1055-1093, 1431-1451, 1605-1616; gemm.rs:149-161).  Values
 * cross this ABI in f32 containers holding bf16 values: every generated kernel rounds its
 * results and loads, parameter uploads and reads round on the host, and the optimizer steps
 * in bf16 with bf16 hyperparameters (note that 0.999 rounds to 1 in bf16).  The gradient
 * exchange (tb_plan_attach_comm) answers TB_DECLINED for bf16 plans. */
enum { TB_ELEMENT_F32 = 0, TB_ELEMENT_BF16 = 1 };

#define TB_MAX_RANK 8

/* One recorded node: a row of the tape's structure columns
 * (graph/structure.rs:23-61) plus the plan's per-node columns. */
typedef struct tb_node {
  int32_t op;                   /* TB_OP_* */
  int32_t rank;                 /* rank of the node's shape */
  int64_t shape[TB_MAX_RANK];   /* the recorded shape */
  int32_t operands[2];          /* operand node indices, -1 when absent */
  int64_t attrs[TB_MAX_RANK];   /* axis/start/len/full_extent/size/step/dilation/extent/rows,
                                   or the permute order; see each op's record site */
  int32_t slot;                 /* Parameter / Input slot, else -1 */
  int32_t payload;              /* TB_PAYLOAD_* of a Leaf, or of an Input's fed kind */
  float constant;               /* CONSTANT value; SELECTION `one` */
  int32_t vocab;                /* SELECTION vocabulary (= shape[1]) */
  const float* dense;           /* DENSE leaf elements, row-major, host memory */
  const int32_t* indices;       /* SELECTION leaf indices (shape[0] entries), host memory */
  uint8_t wanted;               /* Plan::new closure (engine/plan.rs:154-172) */
  uint8_t readable;             /* a root or observed value */
  uint8_t required;             /* read by a derivative rule of a training plan (201-225) */
  uint8_t reserved;
} tb_node;

/* A compiled request over a network (`Network::compile`, engine/plan.rs:655-663). */
typedef struct tb_plan_desc {
  int64_t node_count;
  const tb_node* nodes;
  int32_t backward;             /* Request::backward (engine/request.rs:70) */
  int32_t numerics;             /* TB_NUMERICS_* (engine/request.rs:84) */
  int32_t element;              /* TB_ELEMENT_*: the network's payload element type */
} tb_plan_desc;

/* One fed input (`Plan::forward` feeds, engine/plan.rs:534-564). */
typedef struct tb_feed {
  int32_t slot;                 /* input slot */
  int32_t on_device;            /* 1: pointers are device memory; 0: host memory */
  const float* dense;           /* DENSE input: volume elements */
  const int32_t* indices;       /* SELECTION input: shape[0] indices */
} tb_feed;

typedef struct tb_plan tb_plan;
typedef struct tb_params tb_params;
typedef struct tb_optimizer tb_optimizer;
typedef struct tb_comm tb_comm;
typedef struct tb_run tb_run;

typedef struct tb_plan_stats {
  int64_t kernels;              /* launches in one run of the device program */
  int64_t arena_bytes;          /* liveness-planned arena size */
  int64_t unplanned_bytes;      /* sum of all buffer sizes without reuse */
  int64_t fused_nodes;          /* wanted nodes that were never materialized */
  int32_t bit_identical;        /* 1 when every kernel reproduces the interpreter bitwise */
  int32_t gemms;                /* GEMM launches per run */
} tb_plan_stats;

/* ---- backend status (`Manifest::status`, backend/manifest.rs:16-37) */
/* Replaces: the cuda backend's lazy `context()` + POISON check
 * (backend/cuda/kernels/mod.rs:36-58). Forces lazy set-up; returns TB_* code. */
int tb_status(char* message, size_t capacity);
/* Thread-local message of the last failed call on this thread. */
const char* tb_last_error(void);

/* ---- compiled plans */
/* Replaces: the node loop of `Plan::forward` (engine/plan.rs:566-622) for one
 * compiled request.  Lowers the plan to a device program.  Answers TB_DECLINED
 * for an EXACT-posture plan that holds a kernel that is not bit-identical
 * (`Fidelity::meets`, backend/coverage.rs:26-32). */
int tb_plan_compile(const tb_plan_desc* desc, tb_plan** plan);
void tb_plan_destroy(tb_plan* plan);
int tb_plan_stats_get(const tb_plan* plan, tb_plan_stats* stats);
/* Human-readable kernel list of the device program (cf. `Plan::describe`,
 * engine/plan.rs:408-490); returns the needed length. */
int64_t tb_plan_describe(const tb_plan* plan, char* buffer, size_t capacity);

/* ---- device-resident `Parameters` (graph/parameters.rs:27) */
/* Creates zeroed device storage for every parameter slot of the plan's network. */
int tb_params_create(const tb_plan* plan, tb_params** params);
void tb_params_destroy(tb_params* params);
int tb_params_upload(tb_params* params, int32_t slot, const float* host, int64_t count);
int tb_params_download(const tb_params* params, int32_t slot, float* host, int64_t count);

/* ---- running (`Plan::forward` -> `Run`, engine/plan.rs:514-640; `Run::of`, run.rs:139) */
/* Enqueues one run on the plan's main instance: feeds are copied into its
 * input buffers, then the device program (and an attached gradient exchange
 * and optimizer step) is launched as one CUDA graph.  Asynchronous with
 * respect to the host.  One thread at a time; concurrent runs of one plan use
 * `tb_run_begin`. */
int tb_plan_run(tb_plan* plan, tb_params* params, int32_t feed_count, const tb_feed* feeds);
/* Replaces: `Run::backward(output)` then `Gradients::of(parameter)` (engine/run.rs:229-318)
 * for a plan compiled with `backward` set: the reverse scan of every scalar readable root
 * runs inside each `tb_plan_run`, and this answers the node whose value (read with
 * `tb_plan_read`) is d root / d parameter. */
int tb_plan_gradient_node(const tb_plan* plan, int64_t root, int64_t parameter, int64_t* node);
/* Waits for the plan's stream. */
int tb_plan_synchronize(tb_plan* plan);
/* Copies a readable value (row-major, volume elements) to host memory (waits). */
int tb_plan_read(tb_plan* plan, int64_t node, float* host, int64_t count);
/* Replaces: `Run::of(value)` (engine/run.rs:139) read without waiting: enqueues the copy of a
 * readable value to host memory on the plan's stream (tb_plan_stream) and returns, so that a
 * training loop can launch the next step before it looks at this step's loss.  The values are
 * in `host` once the stream passes the copy (tb_plan_synchronize, or an event recorded on
 * tb_plan_stream after this call); `host` should be page-locked, or the copy does not overlap.
 * A later tb_plan_run overwrites the value on the device, not the copy already enqueued.
 * bf16 plans answer TB_INVALID (their reads round on the host): use tb_plan_read. */
int tb_plan_read_async(tb_plan* plan, int64_t node, float* host, int64_t count);
/* Device address of a readable value's contiguous buffer (valid until the next run). */
int tb_plan_device_pointer(tb_plan* plan, int64_t node, const float** device);
/* The CUDA stream (cudaStream_t) the plan runs on. */
void* tb_plan_stream(tb_plan* plan);

/* ---- concurrent runs of one plan (`Plan` and `Run` are Send + Sync and run from
 *      many threads: engine/plan.rs:20, run.rs:14, examples/makemore/mlp_parallel.rs:136-165) */
/* Replaces: `Plan::forward(parameters, feeds) -> Run` from any thread.  Draws an
 * instance (its own stream, arena and input buffers) from the plan's pool,
 * creating one when all are in use, copies the feeds and launches the device
 * program on it.  Runs drawn this way carry no optimizer or gradient
 * exchange.  Thread-safe; asynchronous with respect to the host. */
int tb_run_begin(tb_plan* plan, tb_params* params, int32_t feed_count, const tb_feed* feeds,
                 tb_run** run);
/* Waits for the run's stream. */
int tb_run_synchronize(tb_run* run);
/* Replaces `Run::of(node)` (run.rs:139): copies a readable value of this run to host memory (waits). */
int tb_run_read(tb_run* run, int64_t node, float* host, int64_t count);
/* Device address of a readable value of this run (valid until the run is released). */
int tb_run_device_pointer(tb_run* run, int64_t node, const float** device);
/* The CUDA stream (cudaStream_t) the run executes on. */
void* tb_run_stream(tb_run* run);
/* Replaces dropping the `Run`: returns its instance to the plan's pool. */
void tb_run_release(tb_run* run);

/* ---- optimizer step (graph/parameters.rs:90-146; neural/optimizer.rs:40-51; neural/adam.rs:19-171) */
enum { TB_OPTIMIZER_SGD = 0, TB_OPTIMIZER_ADAM = 1, TB_OPTIMIZER_ADAMW = 2 };
typedef struct tb_optimizer_desc {
  int32_t kind;                 /* TB_OPTIMIZER_* */
  float learning_rate;
  float beta1, beta2, epsilon;  /* Adam / AdamW (adam.rs:33-45) */
  float decay;                  /* AdamW (adam.rs:118-126), applied to rank >= 2 (adam.rs:167-169) */
  float gradient_scale;         /* multiplies each gradient first (1/shards, mlp_parallel.rs:170-171); 1 = off */
} tb_optimizer_desc;
/* Binds gradient nodes of a plan (readable values) to parameter slots. */
int tb_optimizer_create(tb_plan* plan, tb_params* params, const tb_optimizer_desc* desc,
                        int32_t count, const int32_t* slots, const int64_t* gradient_nodes,
                        tb_optimizer** optimizer);
void tb_optimizer_destroy(tb_optimizer* optimizer);
int tb_optimizer_set_learning_rate(tb_optimizer* optimizer, float learning_rate);
/* Runs the step inside every later `tb_plan_run` of its plan (one graph launch per step). */
int tb_plan_attach_optimizer(tb_plan* plan, tb_optimizer* optimizer);
/* Replaces: `Parameters::step(&gradients, &mut optimizer)` (graph/parameters.rs:90-146) called by
 * the caller: one update of the bound parameters now, on `stream` (a cudaStream_t; NULL = the
 * plan's).  `gradients` NULL steps with the bound gradient values of the plan's last
 * `tb_plan_run`; otherwise it holds one device pointer per bound slot, in binding order (for
 * example gradients summed over several `tb_run_begin` runs).  Updates the same moments and
 * beta powers as the in-graph step. */
int tb_optimizer_step(tb_optimizer* optimizer, const float* const* gradients, void* stream);
/* Downloads Adam moments of a slot (first, second); count elements each. */
int tb_optimizer_state(const tb_optimizer* optimizer, int32_t slot, float* first, float* second, int64_t count);
/* Checkpoints of the optimizer state (the `first`/`second` fields and beta powers that
 * neural/adam.rs:19-31 keeps between steps; the reference's checkpoint.rs snapshots
 * parameters only, and a resumed run needs both).  tb_optimizer_powers reads beta1^t and
 * beta2^t; tb_optimizer_restore writes a slot's moments; tb_optimizer_restore_powers writes
 * the powers, so the next step continues the saved trajectory bitwise.  Adam and AdamW only
 * (TB_INVALID for SGD); each waits for the device first. */
int tb_optimizer_powers(const tb_optimizer* optimizer, float powers[2]);
int tb_optimizer_restore(tb_optimizer* optimizer, int32_t slot, const float* first,
                         const float* second, int64_t count);
int tb_optimizer_restore_powers(tb_optimizer* optimizer, const float powers[2]);

/* ---- data parallel gradient exchange (new: the reference has no communication backend;
 *      replaces the host `tree_sum` of examples/makemore/mlp_parallel.rs:59-71) */
int tb_comm_unique_id(uint8_t id[128]);
int tb_comm_init(int32_t rank, int32_t world, const uint8_t id[128], tb_comm** comm);
void tb_comm_destroy(tb_comm* comm);
/* Sum-allreduces the plan's gradient outputs bound by its optimizer, bucket by
 * bucket as the program finishes them, before the optimizer step. */
int tb_plan_attach_comm(tb_plan* plan, tb_comm* comm, int64_t bucket_bytes);
/* How the attached communicator sums gradients:
 *  TB_REDUCTION_NCCL  ncclAllReduce (NCCL's own order; the default);
 *  TB_REDUCTION_TREE  all-gather of the shard gradients, then the pairwise tree of `tree_sum`
 *                     (examples/makemore/mlp_parallel.rs:59-71) over ranks in order, on every
 *                     rank -- bit-identical to the reference's host sum of the same shard
 *                     gradients, at the cost of N x the bucket bytes moved. */
enum { TB_REDUCTION_NCCL = 0, TB_REDUCTION_TREE = 1 };
int tb_plan_set_reduction(tb_plan* plan, int32_t reduction);
int tb_comm_allreduce(tb_comm* comm, float* device, int64_t count, void* stream);

/* ---- per-task faces (`Elementary::gemm` / `map`, payload/elementary.rs:74-95) */
/* Replaces: `executed_f32` of the cuda backend (backend/cuda/kernels/gemm.rs:54-163).
 * out[m, n] = a[m, k] . b[k, n] with element (i, j) of a at a[i*a_strides[0] + j*a_strides[1]]
 * (`GemmTask`, payload/gemm.rs:40-125); host buffers.  TB_DECLINED below the size
 * threshold or for unsupported strides.  The device workspace is kept per device and grown on
 * demand; calls on one device are serialized.  A CUDA failure answers TB_RUNTIME and poisons
 * the library (backend/cuda/kernels/mod.rs:94-105), as it does for tb_map_f32 and
 * tb_batch_norm_f32. */
int tb_gemm_f32(const float* a, int64_t a_len, const int64_t a_strides[2],
                const float* b, int64_t b_len, const int64_t b_strides[2],
                int64_t m, int64_t k, int64_t n, float* out);
/* Replaces: `MapTask` offers (payload/elementary.rs:89-95): op is TB_OP_EXP,
 * TB_OP_LN, TB_OP_SQRT or TB_OP_TANH; host buffers. */
int tb_map_f32(int32_t op, const float* in, int64_t count, float* out);
/* Replaces: `Elementary::batch_norm` offers (payload/elementary.rs:107-113, `BatchNormTask`,
 * payload/normalized.rs:18-98): training-mode batch normalization of the row-major
 * [batch, features] input over the batch axis, with the operation order of the recorded
 * formula (payload/tensorial.rs:240-258) -- bit-identical to it.  Writes the output and the
 * per-feature mean and biased variance (`Normalized`); host buffers.  TB_DECLINED below
 * 2^17 elements. */
int tb_batch_norm_f32(const float* input, const float* scale, const float* shift, float epsilon,
                      int64_t batch, int64_t features, float* output, float* mean,
                      float* variance);

/* ---- allocation-free GEMM (no counterpart in the reference: topos's cuda backend always
 *      allocates device buffers from its pool for each product).
 * For callers that cannot let the library call cudaMalloc -- a host framework whose own pool
 * owns and accounts for every device allocation, or code that must not allocate after start-up.
 * out[m, n] = a[m, k] . b[k, n], all DEVICE pointers, strides in elements as in tb_gemm_f32;
 * enqueued on `stream` (a cudaStream_t; 0 = the legacy default stream), asynchronous.
 * The only scratch is a fixed 16 MiB device array inside the library: requests needing more
 * than 2*(m+n)*roundup(k,32) <= 4,194,304 floats answer TB_INVALID (tb_last_error says so).
 * Every call resolves the array's address with the calling device current.  The array is
 * committed when the library's device code loads on a device (under CUDA's lazy loading, at the
 * first call that needs it), so make the first call on each device before any stream capture.
 * Calls that overlap on the GPU share the array and race; the caller serializes them.
 * TB_OK means the work was enqueued; a launch failure answers TB_RUNTIME and poisons the
 * library.  A tensor-core wait that expires on the device (a hung copy, 4 s) leaves the output
 * unwritten and is reported by the next tb_plan_synchronize / tb_run_synchronize, or at once by
 * the internal hook tbx_gemm_error() read after the caller synchronizes the stream. */
int tb_gemm_f32_noalloc(const float* a, const int64_t a_strides[2], const float* b,
                        const int64_t b_strides[2], int64_t m, int64_t k, int64_t n, float* out,
                        void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TOPOS_B200_H */
