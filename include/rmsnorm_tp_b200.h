/*
 * rmsnorm_tp_b200 -- C ABI of the B200-native fused tensor-parallel RMSNorm.
 *
 * Drop-in native boundary for the reference's pybind11 module `rmsnorm_tp_cpp`
 * (haowen-han/RmsnormTP, csrc/bindings.cpp:150-197). Plain pointers, sizes and
 * integer status codes only: no torch or C++ types cross this boundary, and no
 * C++ exception escapes it. Every function returns RMSNORM_TP_OK (0) or an
 * rmsnorm_tp_error code; rmsnorm_tp_last_error() gives the message of the last
 * failure on the calling thread.
 *
 * Threading: one host thread drives one communicator. rmsnorm_tp_forward is a
 * collective: every rank of the TP group calls it the same number of times, in
 * the same order, with the same number of rows (the reference's implicit
 * contract, rmsnorm_tp/__init__.py:87-131).
 *
 * Data layout: x and out are [rows, local_hidden] row-major, weight is
 * [local_hidden], all of one dtype, on the communicator's device. The fast
 * kernels need 16-byte aligned x/out/weight and local_hidden * sizeof(dtype)
 * a multiple of 16; other shapes run a slower generic kernel (still on the GPU).
 */
#ifndef RMSNORM_TP_B200_H_
#define RMSNORM_TP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RMSNORM_TP_MAX_TP 8          /* reference csrc/common.hpp:9 (MAX_TP_SIZE) */
#define RMSNORM_TP_HANDLE_BYTES 128  /* reference csrc/common.hpp:10 (HANDLE_SIZE) */

/* Element types of x, weight and out. */
enum rmsnorm_tp_dtype {
  RMSNORM_TP_F32 = 0,   /* the only type the reference supports (__init__.py:96-97) */
  RMSNORM_TP_BF16 = 1,
  RMSNORM_TP_F16 = 2
};

/* Host-side status codes returned by every function. */
enum rmsnorm_tp_error {
  RMSNORM_TP_OK = 0,
  RMSNORM_TP_ERR_INVALID = 1,  /* bad argument (null pointer, size, dtype, rank) */
  RMSNORM_TP_ERR_CUDA = 2,     /* a CUDA runtime call failed */
  RMSNORM_TP_ERR_STATE = 3,    /* call out of order (not finalized, peer missing) */
  RMSNORM_TP_ERR_ROWS = 4,     /* rows > num_max_rows (reference __init__.py:109 assert) */
  RMSNORM_TP_ERR_DEVICE = 5,   /* an earlier launch recorded a device-side failure
                                  (a peer's partial sum never arrived); call
                                  rmsnorm_tp_reset on every rank */
  RMSNORM_TP_ERR_HANDLE = 6    /* peer handle bytes malformed or from another group */
};

/* Device-side failure codes (rmsnorm_tp_status_info.code). */
enum rmsnorm_tp_device_status {
  RMSNORM_TP_STATUS_OK = 0,
  RMSNORM_TP_STATUS_TIMEOUT = 1,  /* a wait for a peer's partial sum ran out */
  RMSNORM_TP_STATUS_ABORTED = 2,  /* gave up because another CTA timed out */
  RMSNORM_TP_STATUS_LOAD_TIMEOUT = 3  /* a bulk copy into shared memory never completed */
};

typedef struct rmsnorm_tp_comm rmsnorm_tp_comm;

typedef struct rmsnorm_tp_status_info {
  uint32_t code;          /* rmsnorm_tp_device_status */
  uint32_t src_rank;      /* rank whose partial sum did not arrive */
  int64_t row;            /* row that timed out */
  uint32_t expected_tag;  /* tag that was awaited */
  uint32_t seen_tag;      /* tag found in the slot when the wait ended */
  uint64_t generation;    /* call number of the failing launch */
  uint64_t next_generation; /* device generation counter now */
} rmsnorm_tp_status_info;

typedef struct rmsnorm_tp_plan_info {
  int32_t variant;        /* -1 = generic kernel */
  int32_t vec_per_lane;
  int32_t team_warps;
  int32_t rows_per_tile;
  int32_t block_threads;
  int32_t teams_per_cta;
  int64_t tiles;
  int32_t grid;
  int32_t depth;          /* tiles in flight per team: register kernels 3 with an exchange
                             (TP > 1), 3/4/6 without (TP = 1); bulk kernels: stages; generic 1 */
} rmsnorm_tp_plan_info;

/* ---- communicator lifecycle -------------------------------------------- */

/* Allocate this rank's mailbox (zeroed) and device state on `device`.
 * Replaces CommBuffer(rank, tp_size, num_max_rows) + allocate()
 * (reference csrc/bindings.cpp:20-53, rmsnorm_tp/__init__.py:67-68). */
int rmsnorm_tp_create(int rank, int tp_size, int64_t num_max_rows, int device,
                      rmsnorm_tp_comm** out);

/* Serialise this rank's mailbox handle into RMSNORM_TP_HANDLE_BYTES bytes.
 * Replaces get_ipc_handle() + IpcHandle.to_bytes()
 * (reference csrc/bindings.cpp:55-61, :154-156). */
int rmsnorm_tp_export_handle(const rmsnorm_tp_comm* comm, void* out, size_t cap,
                             size_t* len);

/* Map peer `peer`'s mailbox from its exported handle bytes (validated).
 * Replaces IpcHandle.from_bytes() + open_remote_handle()
 * (reference csrc/bindings.cpp:157-162, :63-77). */
int rmsnorm_tp_open_peer(rmsnorm_tp_comm* comm, int peer, const void* bytes,
                         size_t len);

/* Use an already-mapped device pointer as peer `peer`'s mailbox (memory that
 * the caller mapped itself, or a stand-in that no rank serves, for the
 * bounded-wait test). No counterpart in the reference. */
int rmsnorm_tp_attach_peer(rmsnorm_tp_comm* comm, int peer, void* mailbox);

/* This rank's mailbox base and size in bytes. Analogue of the pointer-table
 * getters sums_ptrs_gpu()/gen_ptrs_gpu() (reference csrc/bindings.cpp:171-176). */
int rmsnorm_tp_mailbox(const rmsnorm_tp_comm* comm, void** ptr, size_t* bytes);

/* Check that every peer is mapped and wait for set-up work on the device.
 * Replaces finalize_setup() (reference csrc/bindings.cpp:79-82). */
int rmsnorm_tp_finalize(rmsnorm_tp_comm* comm);

/* Close peer mappings and free. Call only after every rank has stopped
 * launching (the Python layer puts a barrier first; the reference has none,
 * csrc/bindings.cpp:84-99). Accepts NULL. */
int rmsnorm_tp_destroy(rmsnorm_tp_comm* comm);

/* ---- hot path ------------------------------------------------------------ */

/* out = x * rsqrt(S / hidden + eps) * weight, S = sum over the TP group of the
 * fp32 sum of squares of the row. One kernel: load, reduce, push the partial to
 * every peer's mailbox, poll the local mailbox, normalise. Stream-ordered on
 * `stream` (a cudaStream_t; NULL = legacy default). The generation is
 * device-resident, so the launch can be captured in a CUDA graph.
 * Replaces launch_fused_rmsnorm (reference csrc/rmsnorm_tp.cu:184-207,
 * csrc/bindings.cpp:182-196), whose `generation` argument is dropped. */
int rmsnorm_tp_forward(rmsnorm_tp_comm* comm, void* out, const void* x,
                       const void* weight, int64_t rows, int64_t local_hidden,
                       int64_t hidden, int dtype, float eps, void* stream);

/* TP = 1: local RMSNorm, no communicator. Replaces the eager torch path of
 * FusedTPRMSNorm.forward at tp_size == 1 (reference rmsnorm_tp/__init__.py:103-107). */
int rmsnorm_local_forward(void* out, const void* x, const void* weight,
                          int64_t rows, int64_t hidden, int dtype, float eps,
                          void* stream);

/* Fused residual add + TP RMSNorm, in the same launch:
 *   z = x + residual   (fp32 add, rounded once to the dtype; written back to residual)
 *   out = z * rsqrt(S / hidden + eps) * weight, S = sum over the TP group of sum(z^2)
 * residual is [rows, local_hidden] in x's dtype, read and overwritten; it must
 * not overlap out. x may be out (in place). On a failed exchange the residual
 * still holds z and out is NaN, as for rmsnorm_tp_forward. No counterpart in
 * the reference (its forward has no residual); the norm is the same as
 * rmsnorm_tp_forward's applied to z, i.e. the reference's AllReduce path
 * (bench_rmsnorm_tp.py:16-22) on (x + residual).to(dtype). */
int rmsnorm_tp_forward_residual(rmsnorm_tp_comm* comm, void* out, void* residual,
                                const void* x, const void* weight, int64_t rows,
                                int64_t local_hidden, int64_t hidden, int dtype, float eps,
                                void* stream);
int rmsnorm_local_forward_residual(void* out, void* residual, const void* x,
                                   const void* weight, int64_t rows, int64_t hidden,
                                   int dtype, float eps, void* stream);

/* ---- fused row-parallel linear -> reduce-scatter -> TP RMSNorm ------------
 * No counterpart in the reference, which leaves the step before its norm to
 * torch: the partial output of a row-parallel linear goes through an NCCL
 * all-reduce / reduce-scatter, then its AllReduce TP RMSNorm normalises
 * (bench_rmsnorm_tp.py:16-22). Here one kernel per call does all of it.
 *
 * Rank r holds a [rows, k_local] (its slice of the linear's input) and
 * linear_weight [hidden, k_local] (nn.Linear layout, its slice of the input
 * features); its partial product a @ linear_weight^T [rows, hidden] is computed
 * on the tensor cores and each 128-column block goes straight into the
 * receive buffer of the rank that owns those columns (rank o owns columns
 * [o * hidden / tp, (o + 1) * hidden / tp)). Rank o sums the tp partials of its
 * columns in rank order (fp32) and rounds to the dtype (x), adds the residual
 * when one is given (z = x + residual, written back into residual), and
 * normalises: out = z * rsqrt(S / hidden + eps) * norm_weight, S = sum over the
 * group of sum(z^2). out and residual are [rows, hidden / tp]; norm_weight is
 * [hidden / tp]. bf16 or fp16; k_local a multiple of 64; hidden a multiple of
 * 128 * tp; every pointer 16-byte aligned; out and residual must not overlap a,
 * linear_weight or norm_weight. A collective like rmsnorm_tp_forward
 * (one generation per call), on a communicator made by rmsnorm_tp_create_linear,
 * whose mailbox allocation also holds the receive buffer
 * (num_max_rows * hidden * 2 bytes) and its flags; the same export / open /
 * finalize / destroy calls set it up. */
int rmsnorm_tp_create_linear(int rank, int tp_size, int64_t num_max_rows, int64_t hidden,
                             int device, rmsnorm_tp_comm** out);
int rmsnorm_tp_linear_forward(rmsnorm_tp_comm* comm, void* out, void* residual, const void* a,
                              const void* linear_weight, const void* norm_weight, int64_t rows,
                              int64_t k_local, int dtype, float eps, void* stream);
/* Every rank of the group in one cooperative launch on one GPU (comms[r] are
 * rank r of a group attached to each other's mailboxes); residuals may be NULL. */
int rmsnorm_tp_linear_forward_emulated(rmsnorm_tp_comm* const* comms, int tp, void* const* outs,
                                       void* const* residuals, const void* const* as,
                                       const void* const* linear_weights,
                                       const void* const* norm_weights, int64_t rows,
                                       int64_t k_local, int dtype, float eps, void* stream);

/* ---- backward (no reference counterpart: the reference is forward-only) --- */

/* Gradients of out = x * rsqrt(S / hidden + eps) * weight (S over the TP group):
 *   D  = sum over the group of sum(dy * weight * x)       (per row, exchanged)
 *   dx = inv * dy * weight - x * inv^3 * D / hidden,  inv = rsqrt(S / hidden + eps)
 *   dw = sum over rows of dy * x * inv                     (this rank's columns)
 * S and D are exchanged through the mailbox in two consecutive generations, so
 * a backward call counts as two calls of the collective's generation. dx is
 * [rows, local_hidden], dw [local_hidden], both in x's dtype; dx must not
 * overlap x or dy. `workspace` is device memory of at least
 * rmsnorm_tp_backward_workspace_bytes(rows, local_hidden) bytes (per-CTA fp32
 * partials of dw, summed in a fixed order: deterministic). local_hidden may be
 * at most 53248. Stream-ordered, graph-capturable like rmsnorm_tp_forward. */
size_t rmsnorm_tp_backward_workspace_bytes(int64_t rows, int64_t local_hidden);
int rmsnorm_tp_backward(rmsnorm_tp_comm* comm, void* dx, void* dw, const void* dy,
                        const void* x, const void* weight, int64_t rows, int64_t local_hidden,
                        int64_t hidden, int dtype, float eps, void* workspace,
                        size_t workspace_bytes, void* stream);
/* TP = 1, no communicator. */
int rmsnorm_local_backward(void* dx, void* dw, const void* dy, const void* x, const void* weight,
                           int64_t rows, int64_t hidden, int dtype, float eps, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ---- failure detection and recovery (no reference counterpart) ---------- */

/* Limit on each wait for a peer's partial sum, in nanoseconds (default
 * 10 s, or RMSNORM_TP_TIMEOUT_MS from the environment at create time). */
int rmsnorm_tp_set_timeout(rmsnorm_tp_comm* comm, uint64_t timeout_ns);

/* Optional in-kernel counters for later launches of this communicator (NULL
 * turns them off): dev_counters points to 20 uint64 in device memory that the
 * kernels add to (times in ns of the GPU global timer) -- [0] ns spent waiting
 * for peers' partial sums (summed over waiting lanes), [1] waits that found the
 * slot not yet written, [2] waits satisfied by the first poll, [3] earliest CTA
 * start and [4] latest CTA end; per CTA: [5] sum of start -> partials pushed and
 * [6] of partials pushed -> end, [7] CTAs that report the pushed mark (resident
 * kernel only), [8] sum of start -> end, [9] CTAs; per launch: [10] sum of
 * first CTA start -> last CTA end, [11] launches, [12] sum of the gaps between
 * one launch's last CTA end and the next launch's first CTA start, [13] gaps
 * counted; [14]..[16] scratch; [17] sum over the CTAs of every launch but the
 * first of (CTA start - the previous launch's end), [18] those CTAs; [19]
 * unused. Initialise [3] and [14] to UINT64_MAX, the rest to 0. */
int rmsnorm_tp_set_profile(rmsnorm_tp_comm* comm, uint64_t* dev_counters);

/* Non-blocking: nonzero in *code once a launch has recorded a device failure
 * (reads host-mapped memory the kernel writes; no CUDA call). */
int rmsnorm_tp_poll_error(const rmsnorm_tp_comm* comm, uint32_t* code);

/* Blocking: synchronise the device and read the full failure record. */
int rmsnorm_tp_status(rmsnorm_tp_comm* comm, rmsnorm_tp_status_info* out);

/* Blocking: wait for the device, zero the mailbox, clear the failure record
 * and set the generation counter to `generation` (at most 2^44 - 1). Every
 * rank must call it between two group barriers, with the same generation. */
int rmsnorm_tp_reset(rmsnorm_tp_comm* comm, uint64_t generation);

/* Blocking: read the device generation counter (launches completed). */
int rmsnorm_tp_get_generation(rmsnorm_tp_comm* comm, uint64_t* out);

/* ---- test and measurement helpers (no reference counterpart) ----------- */

/* Run all `tp` ranks of a group on ONE GPU in one cooperative launch
 * (grid.y = rank), so the push/poll protocol can be checked without several
 * GPUs. comms[r] must be rank r of a group whose peers were attached with
 * rmsnorm_tp_attach_peer to each other's mailboxes. */
int rmsnorm_tp_forward_emulated(rmsnorm_tp_comm* const* comms, int tp,
                                void* const* outs, const void* const* xs,
                                const void* const* weights, int64_t rows,
                                int64_t local_hidden, int dtype, float eps,
                                void* stream);
/* The backward (rmsnorm_tp_backward) of every rank in one cooperative launch;
 * workspaces[r] of workspace_bytes each. */
int rmsnorm_tp_backward_emulated(rmsnorm_tp_comm* const* comms, int tp, void* const* dxs,
                                 void* const* dws, const void* const* dys, const void* const* xs,
                                 const void* const* weights, int64_t rows, int64_t local_hidden,
                                 int dtype, float eps, void* const* workspaces,
                                 size_t workspace_bytes, void* stream);
/* The same with a fused residual add (rmsnorm_tp_forward_residual) per rank. */
int rmsnorm_tp_forward_emulated_residual(rmsnorm_tp_comm* const* comms, int tp,
                                         void* const* outs, void* const* residuals,
                                         const void* const* xs, const void* const* weights,
                                         int64_t rows, int64_t local_hidden, int dtype,
                                         float eps, void* stream);

/* No counterpart in the reference. The fused TP RMSNorm of a whole TP group
 * whose `tp` slices all sit on the current GPU (outs/xs/weights[r] = rank r's
 * tensors, same shapes as rmsnorm_tp_forward_emulated), without allocating
 * any device memory: for callers that may not call cudaMalloc, such as serving
 * runtimes that fix their memory pool at start-up and plugin hosts that hand a
 * kernel only its inputs and outputs. The mailboxes and per-rank state live in
 * a static device array of RMSNORM_TP_STATIC_SCRATCH_BYTES that every GPU
 * loading the library holds until exit; calls needing more than
 * 16 * tp^2 * rows + 256 * tp bytes of it are rejected (RMSNORM_TP_ERR_ROWS).
 * Each call clears the part it uses on `stream` before its launch; calls that
 * overlap on the GPU share the array and race, so serialise them. The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * A wait that runs out on the device is not returned by the call (it has
 * returned by then): the affected rows are written as NaN and the failure stays
 * in the array until the next call clears it; read it with
 * rmsnorm_tp_forward_group_static_status before that next call. */
#define RMSNORM_TP_STATIC_SCRATCH_BYTES (4u << 20)
int rmsnorm_tp_forward_group_static(int tp, void* const* outs, const void* const* xs,
                                    const void* const* weights, int64_t rows,
                                    int64_t local_hidden, int dtype, float eps, void* stream);
/* No counterpart in the reference. Blocking: waits for the current device, then
 * reads the failure record the last rmsnorm_tp_forward_group_static call on this
 * device left in the static array (out->code 0: no failure; otherwise the first
 * failing rank's record, as rmsnorm_tp_status gives it). Allocates nothing.
 * RMSNORM_TP_ERR_STATE if no call was made on this device yet. */
int rmsnorm_tp_forward_group_static_status(rmsnorm_tp_status_info* out);

/* One-hop NVLink latency probe between this rank and `peer`: `iters` round
 * trips of a store into the peer's mailbox and a poll of the local one. Both
 * ranks call it at the same time; the lower rank starts. Writes the average
 * round-trip time in ns to *dev_out_ns (device memory). Bounded waits. */
int rmsnorm_tp_probe_roundtrip(rmsnorm_tp_comm* comm, int peer, int iters,
                               void* stream, int64_t* dev_out_ns);

/* Kernel family used by every later launch of this process:
 * 0 = automatic (with an exchange: the batch kernels for aligned rows of
 * <= 16 KB; at TP = 1: the local register kernels, bulk-copy kernels from
 * 256 MiB of x), 1 = register kernels only, 2 = bulk-copy kernels wherever
 * eligible (aligned rows of <= 16 KB), 3 = batch kernels wherever eligible
 * (aligned rows of <= 16 KB, TP = 1 included). Family 2 also makes the backward
 * use its one-CTA-per-row kernel instead of the register kernel. For tests and
 * benchmarks that compare the implementations. */
int rmsnorm_tp_set_kernel_family(int family);
int rmsnorm_tp_get_kernel_family(void);

/* Encoding of the exchange for every later launch of this process:
 * 0 = {tag, fp32 partial} in one 64-bit system-scope store per slot (default);
 * 1 = the partial, then the tag with a separate release store, read with an
 * acquire of the tag -- the reference's value + flag scheme
 * (csrc/rmsnorm_tp.cu:102-115, :121-138), kept for measured comparison.
 * Every rank of a group must use the same encoding. */
int rmsnorm_tp_set_push_mode(int mode);
int rmsnorm_tp_get_push_mode(void);

/* Programmatic dependent launch for every later forward launch of this process
 * (1 = on, the default; 0 = off). When on, a forward kernel is launched with
 * CUDA's programmatic stream serialization: it may be scheduled while the
 * previous kernel of the stream is still finishing, and waits (griddepcontrol)
 * for that kernel's completion and memory before it reads anything; it also
 * lets the next kernel of the stream be scheduled early. Results are identical
 * either way; the overlap hides launch latency between back-to-back calls,
 * eagerly or in a CUDA graph. The emulated group launch (cooperative) never
 * uses it. No counterpart in the reference, which launches with <<<>>>
 * (csrc/rmsnorm_tp.cu:199-207). */
int rmsnorm_tp_set_dependent_launch(int enable);
int rmsnorm_tp_get_dependent_launch(void);

/* The launch plan the forward call would use (pure host arithmetic; no GPU).
 * variant: -1 generic, 0..6 register kernels (TP > 1), 100..111 bulk-copy
 * kernels (vec_per_lane then = stages per warp, rows_per_tile = rows per
 * stage), 200..213 register kernels without an exchange (TP = 1), 500..501
 * batch kernels (vec_per_lane = depth = ring slots, rows_per_tile = rows per
 * batch, team_warps = warps per CTA). */
int rmsnorm_tp_plan(int64_t rows, int64_t local_hidden, int dtype, int aligned, int tp,
                    int resident_ctas, rmsnorm_tp_plan_info* out);

/* Count, for every row, how many teams of `plan` visit it (coverage check of
 * the row -> team mapping the kernels use; host only). counts has `rows` slots. */
int rmsnorm_tp_plan_coverage(const rmsnorm_tp_plan_info* plan, int64_t rows,
                             int32_t* counts);

/* Generation arithmetic the kernels use (host copies, for tests). */
uint32_t rmsnorm_tp_tag_of(uint64_t generation);
uint32_t rmsnorm_tp_buffer_of(uint64_t generation);

/* Message of the last failure on this thread ("" if none). */
const char* rmsnorm_tp_last_error(void);

/* ABI version (major * 100 + minor). 1.01 added the residual, backward and
 * dependent-launch entry points and named the plan's last field `depth`; 1.02
 * added rmsnorm_tp_forward_group_static_status, the batch kernel family
 * (rmsnorm_tp_set_kernel_family(3)), the push encodings and the fused
 * row-parallel linear entry points; 1.03 widened the profile counters of
 * rmsnorm_tp_set_profile from 5 to 20. */
int rmsnorm_tp_abi_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* RMSNORM_TP_B200_H_ */
