// Internal interface between the C-ABI host code (comm.cpp) and the kernels
// (kernels.cu). Not installed; the public interface is include/rmsnorm_tp_b200.h.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "rtp_common.h"

namespace rtp {

// Pointers of one rank's call.
struct RankPtrs {
  void* out;
  const void* x;
  const void* w;
  DeviceState* state;        // null at TP = 1
  unsigned int* host_flag;   // device alias of the host-mapped failure flag (may be null)
  void* res;                 // residual stream [rows, hl], read and rewritten (fused add); or null
};

// Kernel parameters (passed by value, read through __grid_constant__).
struct KArgs {
  RankPtrs rp[kMaxTP];                 // [0] for a normal launch, [blockIdx.y] when emulated
  unsigned long long* mbox[kMaxTP];    // mailbox base of every rank, as this process maps it
  int64_t rows;
  int64_t hl;                          // local hidden width (elements)
  int64_t nmax;                        // num_max_rows: stride between source blocks of the mailbox
  float hidden_f;                      // global hidden width (divisor of the sum of squares)
  float eps;
  int rank;                            // this rank (normal launch)
  int tp;
  int emulated;                        // 1: every rank in one launch, rank = blockIdx.y
  int tile_rows;                       // bulk kernels: rows per shared-memory stage
  unsigned int stage_bytes;            // bulk kernels: bytes per stage (multiple of 128)
  int lag;                             // bulk kernels: tiles reduced before the oldest is finished
  int schedule;                        // bulk kernels, tiles of several rows: bit 0 = reduce
                                       // the rows one after another (else interleaved), bit 1 =
                                       // normalise them one after another (else interleaved)
  unsigned long long timeout_ns;
  unsigned long long* prof;            // optional wait/timing counters (20 x u64), or null
  int push_mode;                       // kPushPacked (default) or kPushRelease
  int depth;                           // batch kernels: shared-memory ring slots
};

// Push encodings of the exchange (process-wide, rmsnorm_tp_set_push_mode):
// kPushPacked: {tag, fp32 partial} in one 64-bit relaxed system-scope store;
// kPushRelease: the value, then the tag with a release store, read back with an
// acquire of the tag (the reference's scheme), for measured comparison.
enum PushMode { kPushPacked = 0, kPushRelease = 1 };
void set_push_mode(int mode);
int get_push_mode();

enum Dtype { kF32 = 0, kBF16 = 1, kF16 = 2 };

// Kernel family selection (process-wide): automatic, or one family forced.
enum Family { kFamilyAuto = 0, kFamilyRegister = 1, kFamilyBulk = 2, kFamilyBatch = 3 };
void set_family(int family);
int get_family();

// Programmatic dependent launch of single-GPU launches (process-wide, default on).
void set_dependent_launch(bool enable);
bool get_dependent_launch();

// Shape of a kernel variant (template parameters of the vectorised kernel).
struct VariantDesc {
  int id;              // -1 = generic, 0..kNumShapes-1 register kernels, >= kBulkBase bulk kernels
  int vec_per_lane;    // register kernels: 16-byte vectors per lane; bulk: stages per warp
  int team_warps;      // warps sharing one row (bulk: 1)
  int rows_per_tile;
  int block_threads;
  unsigned int stage_bytes;   // bulk kernels only
  unsigned int smem_bytes;    // dynamic shared memory of the launch
  int lag;                    // bulk kernels: exchange lag in tiles
  int schedule;               // bulk kernels: KArgs::schedule
  int depth;                  // tiles in flight per team (Plan::depth)
};

constexpr int kBulkBase = 100;
constexpr int kLocalBase = 200;   // TP = 1 register kernels: base + shape * depths + depth index
// fused residual add: TP = 1 register kernels (base + shape), bulk kernels
// (base + row bound), generic kernel
constexpr int kLocalResBase = 300;
constexpr int kBulkResBase = 400;
constexpr int kGenericRes = -2;
constexpr int kBatchBase = 500;   // batch kernels: base + index of the warp count
// resident register kernels (TP > 1, at most kResidentDepth tiles per team):
// base + register shape
constexpr int kResidentBase = 600;
constexpr int kResidentDepth = 4;
constexpr int64_t kResidentMaxRows = 256;   // the resident kernel serves calls of at most this many rows
// The register plan `v` (TP > 1) becomes the resident register kernel when every
// team of a grid of `resident_ctas` CTAs holds at most kResidentDepth tiles.
VariantDesc finalize_variant(const VariantDesc& v, int tp, int64_t rows, int resident_ctas);

int elem_bytes(int dtype);

// Records `msg` as the calling thread's last error (rmsnorm_tp_last_error) and
// returns `code`.
int record_error(int code, const char* msg);
// `sms`: SM count of the device (sizes the batch kernels' batches).
VariantDesc choose_variant(int64_t hl, int dtype, bool aligned, int tp = 1, int64_t rows = 0,
                           int family = kFamilyAuto, bool residual = false, int sms = 148);
Plan plan_for(const VariantDesc& v, int64_t rows, int resident_ctas);

// Launch the forward kernel. grid_y > 1 only for the emulated (all ranks on one
// GPU, cooperative) launch. Returns a CUDA error; *plan_out (optional) gets the plan.
cudaError_t launch_forward(const KArgs& a, int dtype, int device, int grid_y,
                           cudaStream_t stream, Plan* plan_out);

// Backward launch: the forward's KArgs (rp[r].x = x, rp[r].w = weight,
// rp[r].out = dx, the exchange fields) plus, per rank, dy and the fp32
// workspace of per-CTA dw partials ([grid][hl]).
struct BArgs {
  KArgs k;
  const void* dy[kMaxTP];
  float* ws[kMaxTP];
};
// Upper bound of the backward grid (rows of the dw workspace).
constexpr int kBackwardMaxGrid = 296;
// Largest local width the backward kernel takes (its fp32 dw partial lives in
// shared memory).
constexpr int64_t kBackwardMaxHidden = 53248;
// Launch the backward kernel (cooperative when grid_y > 1, emulated ranks);
// *grid_out receives the grid (the dw partials per rank to reduce).
cudaError_t launch_backward(const BArgs& b, int dtype, int device, int grid_y, cudaStream_t stream,
                            int* grid_out);
// dw[j] = sum over parts c of ws[c][j], rounded to the dtype (fixed order).
cudaError_t launch_dw_reduce(const float* ws, int parts, int64_t hl, void* dw, int dtype,
                             cudaStream_t stream);

// ---------------------------------------------------------------------------
// Fused row-parallel linear -> reduce-scatter -> TP RMSNorm (linear.cu).
//
// Rank r holds A_r [rows, k_local] and the linear weight W_r [hidden, k_local]
// (nn.Linear layout: out x in, K contiguous). Its partial product
// P_r = A_r W_r^T [rows, hidden] is scattered by column block: the columns
// [o * hl, (o + 1) * hl) (hl = hidden / tp) go to rank o's receive buffer,
// slot [src = r]; rank o sums the tp slots in rank order (fp32), rounds to the
// dtype (x), optionally adds the residual, and normalises its hl columns with
// the one-scalar-per-row exchange of the forward kernels.
//
// Receive region of a rank (inside its IPC-mapped mailbox allocation, after
// the slots and the probe area): flags u32 [2 buffers][tp src][mblocks][nblocks]
// (a tile of 128 rows x the call's tile width from src has landed when its flag
// equals the call's tag; nblocks counts the narrowest, 64-column tiles), then
// partials T [tp src][num_max_rows][hl].
// ---------------------------------------------------------------------------
constexpr int kLinTileM = 128;
constexpr int kLinTileN = 128;      // hidden / tp must be a multiple of this
constexpr int kLinTileNMin = 64;    // the narrowest tile width of a call
constexpr int kLinTileK = 64;

struct LinearLayout {
  int64_t flags_off;    // bytes from the region base
  int64_t recv_off;
  int64_t mblocks;      // ceil(num_max_rows / 128)
  int64_t nblocks;      // hl / 128
  int64_t bytes;        // end of the receive region
};
// Layout of the receive region for (tp, num_max_rows, hidden) after `base` bytes
// (the slots and probe area); 2-byte elements.
LinearLayout linear_layout(int tp, int64_t nmax, int64_t hidden, int64_t base);

struct LinRank {
  void* out;                 // y [rows, hl]
  void* res;                 // residual [rows, hl] (read, rewritten with z) or null
  const void* gamma;         // norm weight [hl]
  DeviceState* state;
  unsigned int* host_flag;
};

struct alignas(64) LArgs {
  unsigned char tmaps[2 * kMaxTP][128];   // CUtensorMap of A_r then W_r per rank, 64-aligned
  LinRank rk[kMaxTP];                     // [0] normal launch, [blockIdx.y] when emulated
  unsigned char* region[kMaxTP];          // every rank's mailbox region as this process maps it
  int64_t rows;
  int64_t k;                              // k_local
  int64_t hidden;
  int64_t hl;
  int64_t nmax;
  int64_t flags_off, recv_off, mblocks, nblocks;
  float eps;
  int rank;
  int tp;
  int emulated;
  int push_mode;
  unsigned long long timeout_ns;
};

// Encodes the tensor maps and launches the fused kernel (cooperative when
// grid_y > 1: emulated ranks on one GPU). `as`/`ws`: per rank A_r and W_r.
cudaError_t launch_linear(LArgs& a, const void* const* as, const void* const* ws, int dtype,
                          int device, int grid_y, cudaStream_t stream);
// Tile width (64, 128 or 256 columns) launch_linear picks for a call.
int linear_tile_width(int64_t rows, int64_t hidden, int64_t hl, int sms);

cudaError_t launch_probe(unsigned long long* remote_slot, unsigned long long* local_slot,
                         unsigned long long seq, int iters, int initiator,
                         unsigned long long timeout_ns, long long* out_ns,
                         unsigned int* err_flag, cudaStream_t stream);

}  // namespace rtp
