// C-ABI host side of the fused TP RMSNorm: communicator (mailbox + peer
// mappings), launch entry points, failure record, recovery.
//
// Replaces the reference's pybind11 CommBuffer / IpcHandle / launch binding
// (csrc/bindings.cpp:18-197, csrc/common.hpp:1-18). Differences that matter:
//   * the mailbox is u64 slot[2][tp][num_max_rows] (partial sum and tag in one
//     word, two generation buffers, rows strided by num_max_rows);
//   * the generation lives on the device and is advanced by the kernel itself;
//   * peer pointers travel as kernel parameters (constant bank), not as a
//     device pointer table that the kernel must load first;
//   * handle bytes carry a magic, version, group shape and device UUID, checked
//     on open;
//   * errors come back as status codes plus a thread-local message, never as
//     exceptions, and launch errors are checked (the reference does not check,
//     csrc/rmsnorm_tp.cu:203-206).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>

#include "../../include/rmsnorm_tp_b200.h"
#include "internal.h"
#include "rtp_common.h"

using rtp::DeviceState;
using rtp::KArgs;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

}  // namespace

int rtp::record_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

namespace {

int cuda_fail(cudaError_t e, const char* what) {
  return fail(RMSNORM_TP_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int cuda_fail(cudaError_t e, const char* who, const char* what) {
  return fail(RMSNORM_TP_ERR_CUDA, "%s: %s: %s (%s)", who, what, cudaGetErrorString(e),
              cudaGetErrorName(e));
}

#define RTP_CUDA(call, what)                 \
  do {                                       \
    cudaError_t e_ = (call);                 \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// Makes `device` current for the scope, restoring the caller's device after.
struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  cudaError_t err = cudaSuccess;
  explicit DeviceGuard(int device) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) {
      err = cudaSetDevice(device);
      switched = (err == cudaSuccess);
    }
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(prev);
  }
};

// Serialised mailbox handle: same size as the reference's IpcHandle bytes
// (common.hpp:13-16, bindings.cpp:154-162), with metadata checked on open.
struct HandleBytes {
  cudaIpcMemHandle_t ipc;       // 64 bytes
  uint32_t magic;
  uint32_t version;
  int32_t rank;
  int32_t tp;
  int64_t nmax;
  uint64_t mailbox_bytes;
  unsigned char uuid[16];
  int64_t linear_hidden;        // hidden width of the fused linear's receive region (0: none)
  unsigned char reserved[8];
};
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "cudaIpcMemHandle_t is 64 bytes");
static_assert(sizeof(HandleBytes) == rtp::kHandleBytes, "handle is 128 bytes");

constexpr size_t kProbeBytes = 256;   // after the slots: one probe word per source rank
constexpr unsigned long long kDefaultTimeoutNs = 10ull * 1000ull * 1000ull * 1000ull;

size_t slots_bytes(int tp, int64_t nmax) {
  size_t b = (size_t)rtp::mailbox_slots(tp, nmax) * sizeof(unsigned long long);
  return (b + 255) & ~(size_t)255;
}

bool valid_dtype(int dtype) { return dtype >= RMSNORM_TP_F32 && dtype <= RMSNORM_TP_F16; }

}  // namespace

struct rmsnorm_tp_comm {
  int rank = 0;
  int tp = 1;
  int device = 0;
  int64_t nmax = 0;
  unsigned long long* mailbox = nullptr;   // local, cudaMalloc'd (IPC-exportable)
  size_t mailbox_bytes = 0;
  unsigned long long* peers[rtp::kMaxTP] = {};
  bool opened[rtp::kMaxTP] = {};           // mapped with cudaIpcOpenMemHandle (must be closed)
  DeviceState* state = nullptr;            // local device memory
  unsigned int* host_flag = nullptr;       // pinned host memory, mapped
  unsigned int* host_flag_dev = nullptr;   // its device alias
  unsigned long long timeout_ns = kDefaultTimeoutNs;
  bool finalized = false;
  unsigned long long probe_seq = 0;
  unsigned char uuid[16] = {};
  unsigned long long* prof = nullptr;      // optional device counters (20 x u64)
  int64_t linear_hidden = 0;               // fused linear: hidden width of the receive region
  rtp::LinearLayout lin{};                 // fused linear: layout of the receive region
};

static void release(rmsnorm_tp_comm* c) {
  for (int q = 0; q < rtp::kMaxTP; ++q) {
    if (c->opened[q] && c->peers[q]) cudaIpcCloseMemHandle(c->peers[q]);
    c->opened[q] = false;
    c->peers[q] = nullptr;
  }
  if (c->mailbox) cudaFree(c->mailbox);
  if (c->state) cudaFree(c->state);
  if (c->host_flag) cudaFreeHost(c->host_flag);
  c->mailbox = nullptr;
  c->state = nullptr;
  c->host_flag = nullptr;
  c->host_flag_dev = nullptr;
}

extern "C" {

const char* rmsnorm_tp_last_error(void) { return g_last_error.c_str(); }

int rmsnorm_tp_abi_version(void) { return 103; }

uint32_t rmsnorm_tp_tag_of(uint64_t generation) { return rtp::tag_of(generation); }
uint32_t rmsnorm_tp_buffer_of(uint64_t generation) { return rtp::buffer_of(generation); }

static int create_impl(int rank, int tp_size, int64_t num_max_rows, int64_t linear_hidden,
                       int device, rmsnorm_tp_comm** out) {
  if (!out) return fail(RMSNORM_TP_ERR_INVALID, "create: out is NULL");
  *out = nullptr;
  if (tp_size < 1 || tp_size > rtp::kMaxTP)
    return fail(RMSNORM_TP_ERR_INVALID, "create: tp_size %d outside [1, %d]", tp_size, rtp::kMaxTP);
  if (rank < 0 || rank >= tp_size)
    return fail(RMSNORM_TP_ERR_INVALID, "create: rank %d outside [0, %d)", rank, tp_size);
  if (num_max_rows < 1 || num_max_rows > (int64_t(1) << 31))
    return fail(RMSNORM_TP_ERR_INVALID, "create: num_max_rows %lld outside [1, 2^31]",
                (long long)num_max_rows);
  int ndev = 0;
  RTP_CUDA(cudaGetDeviceCount(&ndev), "create: cudaGetDeviceCount");
  if (device < 0 || device >= ndev)
    return fail(RMSNORM_TP_ERR_INVALID, "create: device %d outside [0, %d)", device, ndev);

  DeviceGuard guard(device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "create: cudaSetDevice");

  rmsnorm_tp_comm* c = new (std::nothrow) rmsnorm_tp_comm();
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "create: out of host memory");
  c->rank = rank;
  c->tp = tp_size;
  c->device = device;
  c->nmax = num_max_rows;
  c->mailbox_bytes = slots_bytes(tp_size, num_max_rows) + kProbeBytes;
  if (linear_hidden > 0) {
    c->linear_hidden = linear_hidden;
    c->lin = rtp::linear_layout(tp_size, num_max_rows, linear_hidden, (int64_t)c->mailbox_bytes);
    c->mailbox_bytes = (size_t)c->lin.bytes;
  }
  if (const char* env = std::getenv("RMSNORM_TP_TIMEOUT_MS")) {
    const long long ms = std::atoll(env);
    if (ms > 0) c->timeout_ns = (unsigned long long)ms * 1000000ull;
  }

  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&c->mailbox), c->mailbox_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->mailbox, 0, c->mailbox_bytes);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->state), sizeof(DeviceState));
  if (e == cudaSuccess) e = cudaMemset(c->state, 0, sizeof(DeviceState));
  if (e == cudaSuccess)
    e = cudaHostAlloc(reinterpret_cast<void**>(&c->host_flag), 256,
                      cudaHostAllocMapped | cudaHostAllocPortable);
  if (e == cudaSuccess) {
    std::memset(c->host_flag, 0, 256);
    e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->host_flag_dev), c->host_flag, 0);
  }
  cudaDeviceProp prop;
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, device);
  if (e == cudaSuccess) std::memcpy(c->uuid, prop.uuid.bytes, 16);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();   // zeroed before any peer can map it
  if (e != cudaSuccess) {
    int rc = cuda_fail(e, "create: allocation");
    release(c);
    delete c;
    return rc;
  }
  c->peers[rank] = c->mailbox;
  *out = c;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_create(int rank, int tp_size, int64_t num_max_rows, int device,
                      rmsnorm_tp_comm** out) {
  return create_impl(rank, tp_size, num_max_rows, 0, device, out);
}

int rmsnorm_tp_create_linear(int rank, int tp_size, int64_t num_max_rows, int64_t hidden,
                             int device, rmsnorm_tp_comm** out) {
  if (out) *out = nullptr;
  if (tp_size < 1 || tp_size > rtp::kMaxTP)
    return fail(RMSNORM_TP_ERR_INVALID, "create_linear: tp_size %d outside [1, %d]", tp_size,
                rtp::kMaxTP);
  if (hidden < 1 || hidden % ((int64_t)tp_size * rtp::kLinTileN) != 0 || hidden > (int64_t(1) << 20))
    return fail(RMSNORM_TP_ERR_INVALID,
                "create_linear: hidden %lld must be a positive multiple of tp * %d (<= 2^20)",
                (long long)hidden, rtp::kLinTileN);
  return create_impl(rank, tp_size, num_max_rows, hidden, device, out);
}

int rmsnorm_tp_export_handle(const rmsnorm_tp_comm* c, void* out, size_t cap, size_t* len) {
  if (!c || !out) return fail(RMSNORM_TP_ERR_INVALID, "export_handle: NULL argument");
  if (cap < sizeof(HandleBytes))
    return fail(RMSNORM_TP_ERR_INVALID, "export_handle: buffer of %zu bytes < %zu", cap,
                sizeof(HandleBytes));
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "export_handle: cudaSetDevice");
  HandleBytes h;
  std::memset(&h, 0, sizeof(h));
  RTP_CUDA(cudaIpcGetMemHandle(&h.ipc, c->mailbox), "export_handle: cudaIpcGetMemHandle");
  h.magic = rtp::kHandleMagic;
  h.version = rtp::kHandleVersion;
  h.rank = c->rank;
  h.tp = c->tp;
  h.nmax = c->nmax;
  h.mailbox_bytes = c->mailbox_bytes;
  h.linear_hidden = c->linear_hidden;
  std::memcpy(h.uuid, c->uuid, 16);
  std::memcpy(out, &h, sizeof(h));
  if (len) *len = sizeof(h);
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_open_peer(rmsnorm_tp_comm* c, int peer, const void* bytes, size_t len) {
  if (!c || !bytes) return fail(RMSNORM_TP_ERR_INVALID, "open_peer: NULL argument");
  if (peer < 0 || peer >= c->tp || peer == c->rank)
    return fail(RMSNORM_TP_ERR_INVALID, "open_peer: peer %d invalid for rank %d of %d", peer,
                c->rank, c->tp);
  if (len != sizeof(HandleBytes))
    return fail(RMSNORM_TP_ERR_HANDLE, "open_peer: handle is %zu bytes, expected %zu", len,
                sizeof(HandleBytes));
  if (c->peers[peer])
    return fail(RMSNORM_TP_ERR_STATE, "open_peer: peer %d already mapped", peer);
  HandleBytes h;
  std::memcpy(&h, bytes, sizeof(h));
  if (h.magic != rtp::kHandleMagic || h.version != rtp::kHandleVersion)
    return fail(RMSNORM_TP_ERR_HANDLE, "open_peer: not a mailbox handle (magic %08x version %u)",
                h.magic, h.version);
  if (h.rank != peer || h.tp != c->tp || h.nmax != c->nmax || h.mailbox_bytes != c->mailbox_bytes ||
      h.linear_hidden != c->linear_hidden)
    return fail(RMSNORM_TP_ERR_HANDLE,
                "open_peer: handle of rank %d (tp %d, num_max_rows %lld, linear hidden %lld) does "
                "not match peer %d (tp %d, num_max_rows %lld, linear hidden %lld)",
                h.rank, h.tp, (long long)h.nmax, (long long)h.linear_hidden, peer, c->tp,
                (long long)c->nmax, (long long)c->linear_hidden);
  if (std::memcmp(h.uuid, c->uuid, 16) == 0)
    return fail(RMSNORM_TP_ERR_HANDLE,
                "open_peer: peer %d is on this rank's GPU; one GPU per rank is required", peer);
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "open_peer: cudaSetDevice");
  void* p = nullptr;
  RTP_CUDA(cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess),
           "open_peer: cudaIpcOpenMemHandle");
  c->peers[peer] = reinterpret_cast<unsigned long long*>(p);
  c->opened[peer] = true;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_attach_peer(rmsnorm_tp_comm* c, int peer, void* mailbox) {
  if (!c || !mailbox) return fail(RMSNORM_TP_ERR_INVALID, "attach_peer: NULL argument");
  if (peer < 0 || peer >= c->tp || peer == c->rank)
    return fail(RMSNORM_TP_ERR_INVALID, "attach_peer: peer %d invalid for rank %d of %d", peer,
                c->rank, c->tp);
  if (reinterpret_cast<uintptr_t>(mailbox) & 7u)
    return fail(RMSNORM_TP_ERR_INVALID, "attach_peer: mailbox not 8-byte aligned");
  if (c->peers[peer])
    return fail(RMSNORM_TP_ERR_STATE, "attach_peer: peer %d already mapped", peer);
  c->peers[peer] = reinterpret_cast<unsigned long long*>(mailbox);
  c->opened[peer] = false;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_mailbox(const rmsnorm_tp_comm* c, void** ptr, size_t* bytes) {
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "mailbox: NULL communicator");
  if (ptr) *ptr = c->mailbox;
  if (bytes) *bytes = c->mailbox_bytes;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_finalize(rmsnorm_tp_comm* c) {
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "finalize: NULL communicator");
  for (int q = 0; q < c->tp; ++q)
    if (!c->peers[q]) return fail(RMSNORM_TP_ERR_STATE, "finalize: peer %d not mapped", q);
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "finalize: cudaSetDevice");
  RTP_CUDA(cudaDeviceSynchronize(), "finalize: cudaDeviceSynchronize");
  c->finalized = true;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_destroy(rmsnorm_tp_comm* c) {
  if (!c) return RMSNORM_TP_OK;
  int rc = RMSNORM_TP_OK;
  {
    DeviceGuard guard(c->device);
    if (guard.err == cudaSuccess) {
      cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) rc = cuda_fail(e, "destroy: cudaDeviceSynchronize");
    }
    release(c);
  }
  delete c;
  return rc;
}

int rmsnorm_tp_set_timeout(rmsnorm_tp_comm* c, uint64_t timeout_ns) {
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "set_timeout: NULL communicator");
  if (timeout_ns == 0) return fail(RMSNORM_TP_ERR_INVALID, "set_timeout: timeout must be > 0");
  c->timeout_ns = timeout_ns;
  return RMSNORM_TP_OK;
}

static int check_shape(const char* who, int64_t rows, int64_t hl, int64_t hidden, int dtype,
                       const void* out, const void* x, const void* w) {
  if (!valid_dtype(dtype)) return fail(RMSNORM_TP_ERR_INVALID, "%s: unknown dtype %d", who, dtype);
  if (rows < 0) return fail(RMSNORM_TP_ERR_INVALID, "%s: rows %lld < 0", who, (long long)rows);
  if (hl < 1 || hl > (int64_t(1) << 31))
    return fail(RMSNORM_TP_ERR_INVALID, "%s: local_hidden %lld outside [1, 2^31]", who,
                (long long)hl);
  if (hidden < hl)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: hidden %lld < local_hidden %lld", who,
                (long long)hidden, (long long)hl);
  if (rows > 0 && (!out || !x || !w))
    return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL tensor pointer", who);
  return RMSNORM_TP_OK;
}

// The residual of a fused residual add must not overlap the output (the kernel
// writes both); any other overlap follows element-wise semantics.
static int check_residual(const char* who, int64_t rows, int64_t hl, int dtype, const void* res,
                          const void* out) {
  if (rows > 0 && !res) return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL residual", who);
  const uintptr_t n = (uintptr_t)rows * (uintptr_t)hl * (uintptr_t)rtp::elem_bytes(dtype);
  const uintptr_t r0 = reinterpret_cast<uintptr_t>(res), o0 = reinterpret_cast<uintptr_t>(out);
  if (rows > 0 && r0 < o0 + n && o0 < r0 + n)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: residual overlaps the output", who);
  return RMSNORM_TP_OK;
}

static int forward_impl(const char* who, rmsnorm_tp_comm* c, void* out, void* res, const void* x,
                        const void* w, int64_t rows, int64_t hl, int64_t hidden, int dtype,
                        float eps, void* stream) {
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL communicator", who);
  if (!c->finalized) return fail(RMSNORM_TP_ERR_STATE, "%s: communicator not finalized", who);
  int rc = check_shape(who, rows, hl, hidden, dtype, out, x, w);
  if (rc != RMSNORM_TP_OK) return rc;
  if (rows > c->nmax)
    return fail(RMSNORM_TP_ERR_ROWS, "%s: rows %lld > num_max_rows %lld", who, (long long)rows,
                (long long)c->nmax);
  const unsigned flag = *reinterpret_cast<volatile unsigned*>(c->host_flag);
  if (flag != 0u)
    return fail(RMSNORM_TP_ERR_DEVICE,
                "%s: an earlier launch recorded device failure %u (a peer's partial sum "
                "never arrived); reset the communicator on every rank",
                who, flag);
  if (rows == 0) return RMSNORM_TP_OK;
  KArgs a;
  std::memset(&a, 0, sizeof(a));
  a.rp[0] = rtp::RankPtrs{out, x, w, c->state, c->host_flag_dev, res};
  for (int q = 0; q < c->tp; ++q) a.mbox[q] = c->peers[q];
  a.rows = rows;
  a.hl = hl;
  a.nmax = c->nmax;
  a.hidden_f = (float)hidden;
  a.eps = eps;
  a.rank = c->rank;
  a.tp = c->tp;
  a.emulated = 0;
  a.timeout_ns = c->timeout_ns;
  a.prof = c->prof;
  int cur = -1;
  cudaGetDevice(&cur);
  cudaError_t e;
  if (cur == c->device) {
    e = rtp::launch_forward(a, dtype, c->device, 1, reinterpret_cast<cudaStream_t>(stream), nullptr);
  } else {
    DeviceGuard guard(c->device);
    e = rtp::launch_forward(a, dtype, c->device, 1, reinterpret_cast<cudaStream_t>(stream), nullptr);
  }
  if (e != cudaSuccess) return cuda_fail(e, who, "kernel launch");
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_forward(rmsnorm_tp_comm* c, void* out, const void* x, const void* w, int64_t rows,
                       int64_t hl, int64_t hidden, int dtype, float eps, void* stream) {
  return forward_impl("forward", c, out, nullptr, x, w, rows, hl, hidden, dtype, eps, stream);
}

int rmsnorm_tp_forward_residual(rmsnorm_tp_comm* c, void* out, void* residual, const void* x,
                                const void* w, int64_t rows, int64_t hl, int64_t hidden,
                                int dtype, float eps, void* stream) {
  if (valid_dtype(dtype) && rows >= 0 && hl >= 1) {
    const int rc = check_residual("forward_residual", rows, hl, dtype, residual, out);
    if (rc != RMSNORM_TP_OK) return rc;
  }
  return forward_impl("forward_residual", c, out, residual, x, w, rows, hl, hidden, dtype, eps,
                      stream);
}

static int local_forward_impl(const char* who, bool with_res, void* out, void* res, const void* x,
                              const void* w, int64_t rows, int64_t hidden, int dtype, float eps,
                              void* stream) {
  int rc = check_shape(who, rows, hidden, hidden, dtype, out, x, w);
  if (rc != RMSNORM_TP_OK) return rc;
  if (with_res) {
    rc = check_residual(who, rows, hidden, dtype, res, out);
    if (rc != RMSNORM_TP_OK) return rc;
  }
  if (rows == 0) return RMSNORM_TP_OK;
  KArgs a;
  std::memset(&a, 0, sizeof(a));
  a.rp[0] = rtp::RankPtrs{out, x, w, nullptr, nullptr, res};
  a.rows = rows;
  a.hl = hidden;
  a.nmax = rows;
  a.hidden_f = (float)hidden;
  a.eps = eps;
  a.rank = 0;
  a.tp = 1;
  int dev = 0;
  RTP_CUDA(cudaGetDevice(&dev), "local_forward: cudaGetDevice");
  cudaError_t e =
      rtp::launch_forward(a, dtype, dev, 1, reinterpret_cast<cudaStream_t>(stream), nullptr);
  if (e != cudaSuccess) return cuda_fail(e, who, "kernel launch");
  return RMSNORM_TP_OK;
}

int rmsnorm_local_forward(void* out, const void* x, const void* w, int64_t rows, int64_t hidden,
                          int dtype, float eps, void* stream) {
  return local_forward_impl("local_forward", false, out, nullptr, x, w, rows, hidden, dtype, eps,
                            stream);
}

int rmsnorm_local_forward_residual(void* out, void* residual, const void* x, const void* w,
                                   int64_t rows, int64_t hidden, int dtype, float eps,
                                   void* stream) {
  return local_forward_impl("local_forward_residual", true, out, residual, x, w, rows, hidden, dtype,
                            eps, stream);
}

static int forward_emulated_impl(const char* who, rmsnorm_tp_comm* const* comms, int tp,
                                 void* const* outs, void* const* residuals, const void* const* xs,
                                 const void* const* ws, int64_t rows, int64_t hl, int dtype,
                                 float eps, void* stream) {
  if (!comms || !outs || !xs || !ws)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL argument", who);
  if (tp < 2 || tp > rtp::kMaxTP)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: tp %d outside [2, %d]", who, tp, rtp::kMaxTP);
  for (int r = 0; r < tp; ++r) {
    const rmsnorm_tp_comm* c = comms[r];
    if (!c) return fail(RMSNORM_TP_ERR_INVALID, "%s: comms[%d] is NULL", who, r);
    if (c->rank != r || c->tp != tp || c->device != comms[0]->device || c->nmax != comms[0]->nmax)
      return fail(RMSNORM_TP_ERR_INVALID,
                  "%s: comms[%d] is rank %d of %d on device %d; expected rank %d of "
                  "%d on device %d",
                  who, r, c->rank, c->tp, c->device, r, tp, comms[0]->device);
    if (!c->finalized)
      return fail(RMSNORM_TP_ERR_STATE, "%s: comms[%d] not finalized", who, r);
    int rc = check_shape(who, rows, hl, hl * tp, dtype, outs[r], xs[r], ws[r]);
    if (rc != RMSNORM_TP_OK) return rc;
    if (residuals != nullptr) {
      rc = check_residual(who, rows, hl, dtype, residuals[r], outs[r]);
      if (rc != RMSNORM_TP_OK) return rc;
    }
    if (*reinterpret_cast<volatile unsigned*>(c->host_flag) != 0u)
      return fail(RMSNORM_TP_ERR_DEVICE, "%s: rank %d recorded a device failure", who, r);
  }
  if (rows > comms[0]->nmax)
    return fail(RMSNORM_TP_ERR_ROWS, "%s: rows %lld > num_max_rows %lld",
                who, (long long)rows, (long long)comms[0]->nmax);
  if (rows == 0) return RMSNORM_TP_OK;
  KArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int r = 0; r < tp; ++r) {
    a.rp[r] = rtp::RankPtrs{outs[r], xs[r], ws[r], comms[r]->state, comms[r]->host_flag_dev,
                            residuals != nullptr ? residuals[r] : nullptr};
    a.mbox[r] = comms[r]->mailbox;
  }
  a.rows = rows;
  a.hl = hl;
  a.nmax = comms[0]->nmax;
  a.hidden_f = (float)(hl * tp);
  a.eps = eps;
  a.rank = 0;
  a.tp = tp;
  a.emulated = 1;
  a.timeout_ns = comms[0]->timeout_ns;
  a.prof = comms[0]->prof;
  DeviceGuard guard(comms[0]->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, who, "cudaSetDevice");
  cudaError_t e = rtp::launch_forward(a, dtype, comms[0]->device, tp,
                                      reinterpret_cast<cudaStream_t>(stream), nullptr);
  if (e != cudaSuccess) return cuda_fail(e, who, "cooperative launch");
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_forward_emulated(rmsnorm_tp_comm* const* comms, int tp, void* const* outs,
                                const void* const* xs, const void* const* ws, int64_t rows,
                                int64_t hl, int dtype, float eps, void* stream) {
  return forward_emulated_impl("forward_emulated", comms, tp, outs, nullptr, xs, ws, rows, hl, dtype,
                               eps, stream);
}

int rmsnorm_tp_forward_emulated_residual(rmsnorm_tp_comm* const* comms, int tp, void* const* outs,
                                         void* const* residuals, const void* const* xs,
                                         const void* const* ws, int64_t rows, int64_t hl,
                                         int dtype, float eps, void* stream) {
  if (!residuals) return fail(RMSNORM_TP_ERR_INVALID, "forward_emulated_residual: NULL residuals");
  return forward_emulated_impl("forward_emulated_residual", comms, tp, outs, residuals, xs, ws, rows,
                               hl, dtype, eps, stream);
}

// ---- fused row-parallel linear -> reduce-scatter -> TP RMSNorm ---------------

static int check_linear(const char* who, const rmsnorm_tp_comm* c, int64_t rows, int64_t k,
                        int dtype, const void* out, const void* res, const void* a, const void* w,
                        const void* gamma) {
  if (!c->finalized) return fail(RMSNORM_TP_ERR_STATE, "%s: communicator not finalized", who);
  if (c->linear_hidden == 0)
    return fail(RMSNORM_TP_ERR_STATE, "%s: communicator made without a linear receive region "
                "(use rmsnorm_tp_create_linear)", who);
  if (dtype != RMSNORM_TP_BF16 && dtype != RMSNORM_TP_F16)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: dtype %d; the tensor-core path takes bf16 or fp16",
                who, dtype);
  if (rows < 0 || rows > c->nmax)
    return fail(rows < 0 ? RMSNORM_TP_ERR_INVALID : RMSNORM_TP_ERR_ROWS,
                "%s: rows %lld outside [0, num_max_rows %lld]", who, (long long)rows,
                (long long)c->nmax);
  if (k < rtp::kLinTileK || k % rtp::kLinTileK != 0 || k > (int64_t(1) << 20))
    return fail(RMSNORM_TP_ERR_INVALID, "%s: k_local %lld must be a positive multiple of %d",
                who, (long long)k, rtp::kLinTileK);
  if (rows > 0 && (!out || !a || !w || !gamma))
    return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL tensor pointer", who);
  const uintptr_t bits = reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(res) |
                         reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) |
                         reinterpret_cast<uintptr_t>(gamma);
  if (bits & 15u)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: every tensor must be 16-byte aligned", who);
  if (res != nullptr) {
    const int rc = check_residual(who, rows, c->linear_hidden / c->tp, dtype, res, out);
    if (rc != RMSNORM_TP_OK) return rc;
  }
  // out and the residual are written while other CTAs may still read a and the
  // weights (the GEMM phase of the kernel): neither may overlap an input
  const uintptr_t out_n = (uintptr_t)rows * (uintptr_t)(c->linear_hidden / c->tp) * 2u;
  const uintptr_t in_p[3] = {reinterpret_cast<uintptr_t>(a), reinterpret_cast<uintptr_t>(w),
                             reinterpret_cast<uintptr_t>(gamma)};
  const uintptr_t in_n[3] = {(uintptr_t)rows * (uintptr_t)k * 2u,
                             (uintptr_t)c->linear_hidden * (uintptr_t)k * 2u,
                             (uintptr_t)(c->linear_hidden / c->tp) * 2u};
  const uintptr_t dst[2] = {reinterpret_cast<uintptr_t>(out), reinterpret_cast<uintptr_t>(res)};
  for (int d = 0; d < 2 && rows > 0; ++d) {
    if (dst[d] == 0) continue;
    for (int i = 0; i < 3; ++i)
      if (dst[d] < in_p[i] + in_n[i] && in_p[i] < dst[d] + out_n)
        return fail(RMSNORM_TP_ERR_INVALID, "%s: %s overlaps an input", who,
                    d == 0 ? "out" : "residual");
  }
  if (*reinterpret_cast<volatile unsigned*>(c->host_flag) != 0u)
    return fail(RMSNORM_TP_ERR_DEVICE,
                "%s: an earlier launch recorded a device failure; reset the communicator on "
                "every rank", who);
  return RMSNORM_TP_OK;
}

static void fill_linear(rtp::LArgs& L, const rmsnorm_tp_comm* c, int64_t rows, int64_t k,
                        float eps) {
  L.rows = rows;
  L.k = k;
  L.hidden = c->linear_hidden;
  L.hl = c->linear_hidden / c->tp;
  L.nmax = c->nmax;
  L.flags_off = c->lin.flags_off;
  L.recv_off = c->lin.recv_off;
  L.mblocks = c->lin.mblocks;
  L.nblocks = c->lin.nblocks;
  L.eps = eps;
  L.tp = c->tp;
  L.timeout_ns = c->timeout_ns;
}

int rmsnorm_tp_linear_forward(rmsnorm_tp_comm* c, void* out, void* residual, const void* a,
                              const void* linear_weight, const void* norm_weight, int64_t rows,
                              int64_t k_local, int dtype, float eps, void* stream) {
  const char* who = "linear_forward";
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL communicator", who);
  int rc = check_linear(who, c, rows, k_local, dtype, out, residual, a, linear_weight, norm_weight);
  if (rc != RMSNORM_TP_OK) return rc;
  if (rows == 0) return RMSNORM_TP_OK;
  rtp::LArgs* L = new (std::nothrow) rtp::LArgs();
  if (!L) return fail(RMSNORM_TP_ERR_INVALID, "%s: out of host memory", who);
  fill_linear(*L, c, rows, k_local, eps);
  L->rk[0] = rtp::LinRank{out, residual, norm_weight, c->state, c->host_flag_dev};
  for (int q = 0; q < c->tp; ++q) L->region[q] = reinterpret_cast<unsigned char*>(c->peers[q]);
  L->rank = c->rank;
  L->emulated = 0;
  const void* as[1] = {a};
  const void* ws[1] = {linear_weight};
  DeviceGuard guard(c->device);
  cudaError_t e = guard.err;
  if (e == cudaSuccess)
    e = rtp::launch_linear(*L, as, ws, dtype, c->device, 1, reinterpret_cast<cudaStream_t>(stream));
  delete L;
  if (e != cudaSuccess) return cuda_fail(e, who, "kernel launch");
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_linear_forward_emulated(rmsnorm_tp_comm* const* comms, int tp, void* const* outs,
                                       void* const* residuals, const void* const* as,
                                       const void* const* linear_weights,
                                       const void* const* norm_weights, int64_t rows,
                                       int64_t k_local, int dtype, float eps, void* stream) {
  const char* who = "linear_forward_emulated";
  if (!comms || !outs || !as || !linear_weights || !norm_weights)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL argument", who);
  if (tp < 2 || tp > rtp::kMaxTP)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: tp %d outside [2, %d]", who, tp, rtp::kMaxTP);
  for (int r = 0; r < tp; ++r) {
    const rmsnorm_tp_comm* c = comms[r];
    if (!c) return fail(RMSNORM_TP_ERR_INVALID, "%s: comms[%d] is NULL", who, r);
    if (c->rank != r || c->tp != tp || c->device != comms[0]->device ||
        c->nmax != comms[0]->nmax || c->linear_hidden != comms[0]->linear_hidden)
      return fail(RMSNORM_TP_ERR_INVALID, "%s: comms[%d] is not rank %d of one group", who, r, r);
    const int rc = check_linear(who, c, rows, k_local, dtype, outs[r],
                                residuals ? residuals[r] : nullptr, as[r], linear_weights[r],
                                norm_weights[r]);
    if (rc != RMSNORM_TP_OK) return rc;
  }
  if (rows == 0) return RMSNORM_TP_OK;
  rtp::LArgs* L = new (std::nothrow) rtp::LArgs();
  if (!L) return fail(RMSNORM_TP_ERR_INVALID, "%s: out of host memory", who);
  fill_linear(*L, comms[0], rows, k_local, eps);
  for (int r = 0; r < tp; ++r) {
    L->rk[r] = rtp::LinRank{outs[r], residuals ? residuals[r] : nullptr, norm_weights[r],
                            comms[r]->state, comms[r]->host_flag_dev};
    L->region[r] = reinterpret_cast<unsigned char*>(comms[r]->mailbox);
  }
  L->rank = 0;
  L->emulated = 1;
  DeviceGuard guard(comms[0]->device);
  cudaError_t e = guard.err;
  if (e == cudaSuccess)
    e = rtp::launch_linear(*L, as, linear_weights, dtype, comms[0]->device, tp,
                           reinterpret_cast<cudaStream_t>(stream));
  delete L;
  if (e != cudaSuccess) return cuda_fail(e, who, "cooperative launch");
  return RMSNORM_TP_OK;
}

// ---- backward ---------------------------------------------------------------

size_t rmsnorm_tp_backward_workspace_bytes(int64_t rows, int64_t hl) {
  if (rows <= 0 || hl < 1) return 0;
  const int64_t parts = rows < rtp::kBackwardMaxGrid ? rows : rtp::kBackwardMaxGrid;
  return (size_t)parts * (size_t)hl * sizeof(float);
}

static bool overlaps(const void* a, const void* b, uintptr_t n) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return n > 0 && a0 < b0 + n && b0 < a0 + n;
}

static int check_backward(const char* who, int64_t rows, int64_t hl, int64_t hidden, int dtype,
                          const void* dx, const void* dw, const void* dy, const void* x,
                          const void* w, const void* workspace, size_t workspace_bytes) {
  int rc = check_shape(who, rows, hl, hidden, dtype, dx, x, w);
  if (rc != RMSNORM_TP_OK) return rc;
  if (hl > rtp::kBackwardMaxHidden)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: local_hidden %lld > %lld", who, (long long)hl,
                (long long)rtp::kBackwardMaxHidden);
  if (!dw || (rows > 0 && (!dy || !workspace)))
    return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL dw, dy or workspace", who);
  if (workspace_bytes < rmsnorm_tp_backward_workspace_bytes(rows, hl))
    return fail(RMSNORM_TP_ERR_INVALID, "%s: workspace of %zu bytes < %zu", who, workspace_bytes,
                rmsnorm_tp_backward_workspace_bytes(rows, hl));
  const uintptr_t n = (uintptr_t)rows * (uintptr_t)hl * (uintptr_t)rtp::elem_bytes(dtype);
  if (overlaps(dx, x, n) || overlaps(dx, dy, n))
    return fail(RMSNORM_TP_ERR_INVALID, "%s: dx overlaps x or dy", who);
  return RMSNORM_TP_OK;
}

// Launch the backward of `nranks` ranks (cooperative when emulated), then one
// dw reduction per rank. rows == 0: only dw = 0.
static int run_backward(const char* who, const rtp::BArgs& b, int dtype, int device, int nranks,
                        void* const* dws, void* stream) {
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int parts = 0;
  if (b.k.rows > 0) {
    const cudaError_t e = rtp::launch_backward(b, dtype, device, b.k.emulated ? nranks : 1, st,
                                               &parts);
    if (e != cudaSuccess) return cuda_fail(e, who, "backward launch");
  }
  for (int r = 0; r < nranks; ++r) {
    const cudaError_t e = rtp::launch_dw_reduce(b.ws[r], parts, b.k.hl, dws[r], dtype, st);
    if (e != cudaSuccess) return cuda_fail(e, who, "dw reduction launch");
  }
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_backward(rmsnorm_tp_comm* c, void* dx, void* dw, const void* dy, const void* x,
                        const void* w, int64_t rows, int64_t hl, int64_t hidden, int dtype,
                        float eps, void* workspace, size_t workspace_bytes, void* stream) {
  const char* who = "backward";
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL communicator", who);
  if (!c->finalized) return fail(RMSNORM_TP_ERR_STATE, "%s: communicator not finalized", who);
  int rc = check_backward(who, rows, hl, hidden, dtype, dx, dw, dy, x, w, workspace,
                          workspace_bytes);
  if (rc != RMSNORM_TP_OK) return rc;
  if (rows > c->nmax)
    return fail(RMSNORM_TP_ERR_ROWS, "%s: rows %lld > num_max_rows %lld", who, (long long)rows,
                (long long)c->nmax);
  const unsigned flag = *reinterpret_cast<volatile unsigned*>(c->host_flag);
  if (flag != 0u)
    return fail(RMSNORM_TP_ERR_DEVICE,
                "%s: an earlier launch recorded device failure %u; reset the communicator on "
                "every rank",
                who, flag);
  rtp::BArgs b;
  std::memset(&b, 0, sizeof(b));
  b.k.rp[0] = rtp::RankPtrs{dx, x, w, c->state, c->host_flag_dev, nullptr};
  for (int q = 0; q < c->tp; ++q) b.k.mbox[q] = c->peers[q];
  b.k.rows = rows;
  b.k.hl = hl;
  b.k.nmax = c->nmax;
  b.k.hidden_f = (float)hidden;
  b.k.eps = eps;
  b.k.rank = c->rank;
  b.k.tp = c->tp;
  b.k.timeout_ns = c->timeout_ns;
  b.k.prof = c->prof;
  b.dy[0] = dy;
  b.ws[0] = static_cast<float*>(workspace);
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, who, "cudaSetDevice");
  void* dws[1] = {dw};
  return run_backward(who, b, dtype, c->device, 1, dws, stream);
}

int rmsnorm_local_backward(void* dx, void* dw, const void* dy, const void* x, const void* w,
                           int64_t rows, int64_t hidden, int dtype, float eps, void* workspace,
                           size_t workspace_bytes, void* stream) {
  const char* who = "local_backward";
  int rc = check_backward(who, rows, hidden, hidden, dtype, dx, dw, dy, x, w, workspace,
                          workspace_bytes);
  if (rc != RMSNORM_TP_OK) return rc;
  rtp::BArgs b;
  std::memset(&b, 0, sizeof(b));
  b.k.rp[0] = rtp::RankPtrs{dx, x, w, nullptr, nullptr, nullptr};
  b.k.rows = rows;
  b.k.hl = hidden;
  b.k.nmax = rows;
  b.k.hidden_f = (float)hidden;
  b.k.eps = eps;
  b.k.tp = 1;
  b.dy[0] = dy;
  b.ws[0] = static_cast<float*>(workspace);
  int dev = 0;
  RTP_CUDA(cudaGetDevice(&dev), "local_backward: cudaGetDevice");
  void* dws[1] = {dw};
  return run_backward(who, b, dtype, dev, 1, dws, stream);
}

int rmsnorm_tp_backward_emulated(rmsnorm_tp_comm* const* comms, int tp, void* const* dxs,
                                 void* const* dws, const void* const* dys, const void* const* xs,
                                 const void* const* ws, int64_t rows, int64_t hl, int dtype,
                                 float eps, void* const* workspaces, size_t workspace_bytes,
                                 void* stream) {
  const char* who = "backward_emulated";
  if (!comms || !dxs || !dws || !dys || !xs || !ws || !workspaces)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: NULL argument", who);
  if (tp < 2 || tp > rtp::kMaxTP)
    return fail(RMSNORM_TP_ERR_INVALID, "%s: tp %d outside [2, %d]", who, tp, rtp::kMaxTP);
  for (int r = 0; r < tp; ++r) {
    const rmsnorm_tp_comm* c = comms[r];
    if (!c) return fail(RMSNORM_TP_ERR_INVALID, "%s: comms[%d] is NULL", who, r);
    if (c->rank != r || c->tp != tp || c->device != comms[0]->device || c->nmax != comms[0]->nmax)
      return fail(RMSNORM_TP_ERR_INVALID, "%s: comms[%d] is not rank %d of one group", who, r, r);
    if (!c->finalized) return fail(RMSNORM_TP_ERR_STATE, "%s: comms[%d] not finalized", who, r);
    int rc = check_backward(who, rows, hl, hl * tp, dtype, dxs[r], dws[r], dys[r], xs[r], ws[r],
                            workspaces[r], workspace_bytes);
    if (rc != RMSNORM_TP_OK) return rc;
    if (*reinterpret_cast<volatile unsigned*>(c->host_flag) != 0u)
      return fail(RMSNORM_TP_ERR_DEVICE, "%s: rank %d recorded a device failure", who, r);
  }
  if (rows > comms[0]->nmax)
    return fail(RMSNORM_TP_ERR_ROWS, "%s: rows %lld > num_max_rows %lld", who, (long long)rows,
                (long long)comms[0]->nmax);
  rtp::BArgs b;
  std::memset(&b, 0, sizeof(b));
  for (int r = 0; r < tp; ++r) {
    b.k.rp[r] = rtp::RankPtrs{dxs[r], xs[r], ws[r], comms[r]->state, comms[r]->host_flag_dev,
                              nullptr};
    b.k.mbox[r] = comms[r]->mailbox;
    b.dy[r] = dys[r];
    b.ws[r] = static_cast<float*>(workspaces[r]);
  }
  b.k.rows = rows;
  b.k.hl = hl;
  b.k.nmax = comms[0]->nmax;
  b.k.hidden_f = (float)(hl * tp);
  b.k.eps = eps;
  b.k.tp = tp;
  b.k.emulated = 1;
  b.k.timeout_ns = comms[0]->timeout_ns;
  b.k.prof = comms[0]->prof;
  DeviceGuard guard(comms[0]->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, who, "cudaSetDevice");
  return run_backward(who, b, dtype, comms[0]->device, tp, dws, stream);
}

int rmsnorm_tp_set_profile(rmsnorm_tp_comm* c, uint64_t* dev_counters) {
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "set_profile: NULL communicator");
  if (reinterpret_cast<uintptr_t>(dev_counters) & 7u)
    return fail(RMSNORM_TP_ERR_INVALID, "set_profile: counters not 8-byte aligned");
  c->prof = reinterpret_cast<unsigned long long*>(dev_counters);
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_poll_error(const rmsnorm_tp_comm* c, uint32_t* code) {
  if (!c || !code) return fail(RMSNORM_TP_ERR_INVALID, "poll_error: NULL argument");
  *code = *reinterpret_cast<volatile unsigned*>(c->host_flag);
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_status(rmsnorm_tp_comm* c, rmsnorm_tp_status_info* out) {
  if (!c || !out) return fail(RMSNORM_TP_ERR_INVALID, "status: NULL argument");
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "status: cudaSetDevice");
  RTP_CUDA(cudaDeviceSynchronize(), "status: cudaDeviceSynchronize");
  DeviceState st;
  RTP_CUDA(cudaMemcpy(&st, c->state, sizeof(st), cudaMemcpyDeviceToHost), "status: copy state");
  std::memset(out, 0, sizeof(*out));
  out->code = st.err_code;
  out->src_rank = st.err_src;
  out->row = st.err_row;
  out->expected_tag = st.err_expected;
  out->seen_tag = st.err_seen;
  out->generation = st.err_call;
  out->next_generation = st.call >> rtp::kGenShift;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_reset(rmsnorm_tp_comm* c, uint64_t generation) {
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "reset: NULL communicator");
  if (generation > rtp::kGenMax)
    return fail(RMSNORM_TP_ERR_INVALID, "reset: generation %llu above the counter's %llu",
                (unsigned long long)generation, (unsigned long long)rtp::kGenMax);
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "reset: cudaSetDevice");
  RTP_CUDA(cudaDeviceSynchronize(), "reset: cudaDeviceSynchronize");
  RTP_CUDA(cudaMemset(c->mailbox, 0, c->mailbox_bytes), "reset: zero mailbox");
  DeviceState st;
  std::memset(&st, 0, sizeof(st));
  st.call = generation << rtp::kGenShift;
  RTP_CUDA(cudaMemcpy(c->state, &st, sizeof(st), cudaMemcpyHostToDevice), "reset: write state");
  RTP_CUDA(cudaDeviceSynchronize(), "reset: cudaDeviceSynchronize");
  *reinterpret_cast<volatile unsigned*>(c->host_flag) = 0u;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_get_generation(rmsnorm_tp_comm* c, uint64_t* out) {
  if (!c || !out) return fail(RMSNORM_TP_ERR_INVALID, "get_generation: NULL argument");
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "get_generation: cudaSetDevice");
  RTP_CUDA(cudaDeviceSynchronize(), "get_generation: cudaDeviceSynchronize");
  unsigned long long g = 0;
  RTP_CUDA(cudaMemcpy(&g, &c->state->call, sizeof(g), cudaMemcpyDeviceToHost),
           "get_generation: copy");
  *out = g >> rtp::kGenShift;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_probe_roundtrip(rmsnorm_tp_comm* c, int peer, int iters, void* stream,
                               int64_t* dev_out_ns) {
  if (!c) return fail(RMSNORM_TP_ERR_INVALID, "probe_roundtrip: NULL communicator");
  if (!c->finalized) return fail(RMSNORM_TP_ERR_STATE, "probe_roundtrip: not finalized");
  if (peer < 0 || peer >= c->tp || peer == c->rank)
    return fail(RMSNORM_TP_ERR_INVALID, "probe_roundtrip: peer %d invalid", peer);
  if (iters < 1 || iters > (1 << 30))
    return fail(RMSNORM_TP_ERR_INVALID, "probe_roundtrip: iters %d outside [1, 2^30]", iters);
  const size_t probe_off = slots_bytes(c->tp, c->nmax) / sizeof(unsigned long long);
  unsigned long long* remote = c->peers[peer] + probe_off + c->rank;
  unsigned long long* local = c->mailbox + probe_off + peer;
  c->probe_seq += 1;
  DeviceGuard guard(c->device);
  if (guard.err != cudaSuccess) return cuda_fail(guard.err, "probe_roundtrip: cudaSetDevice");
  cudaError_t e = rtp::launch_probe(remote, local, c->probe_seq, iters, c->rank < peer ? 1 : 0,
                                    c->timeout_ns, reinterpret_cast<long long*>(dev_out_ns),
                                    nullptr, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "probe_roundtrip: launch");
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_set_kernel_family(int family) {
  if (family < rtp::kFamilyAuto || family > rtp::kFamilyBatch)
    return fail(RMSNORM_TP_ERR_INVALID, "set_kernel_family: unknown family %d", family);
  rtp::set_family(family);
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_get_kernel_family(void) { return rtp::get_family(); }

int rmsnorm_tp_set_push_mode(int mode) {
  if (mode != rtp::kPushPacked && mode != rtp::kPushRelease)
    return fail(RMSNORM_TP_ERR_INVALID, "set_push_mode: expected 0 or 1, got %d", mode);
  rtp::set_push_mode(mode);
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_get_push_mode(void) { return rtp::get_push_mode(); }

int rmsnorm_tp_set_dependent_launch(int enable) {
  if (enable != 0 && enable != 1)
    return fail(RMSNORM_TP_ERR_INVALID, "set_dependent_launch: expected 0 or 1, got %d", enable);
  rtp::set_dependent_launch(enable == 1);
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_get_dependent_launch(void) { return rtp::get_dependent_launch() ? 1 : 0; }

int rmsnorm_tp_plan(int64_t rows, int64_t hl, int dtype, int aligned, int tp, int resident_ctas,
                    rmsnorm_tp_plan_info* out) {
  if (!out) return fail(RMSNORM_TP_ERR_INVALID, "plan: NULL out");
  if (!valid_dtype(dtype)) return fail(RMSNORM_TP_ERR_INVALID, "plan: unknown dtype %d", dtype);
  if (rows < 0 || hl < 1 || resident_ctas < 1 || tp < 1 || tp > rtp::kMaxTP)
    return fail(RMSNORM_TP_ERR_INVALID, "plan: rows %lld, local_hidden %lld, tp %d, resident %d",
                (long long)rows, (long long)hl, tp, resident_ctas);
  const rtp::VariantDesc v = rtp::finalize_variant(
      rtp::choose_variant(hl, dtype, aligned != 0, tp, rows), tp, rows, resident_ctas);
  const rtp::Plan p = rtp::plan_for(v, rows, resident_ctas);
  out->variant = p.variant;
  out->vec_per_lane = p.vec_per_lane;
  out->team_warps = p.team_warps;
  out->rows_per_tile = p.rows_per_tile;
  out->block_threads = p.block_threads;
  out->teams_per_cta = p.teams_per_cta;
  out->tiles = p.tiles;
  out->grid = p.grid;
  out->depth = p.depth;
  return RMSNORM_TP_OK;
}

int rmsnorm_tp_plan_coverage(const rmsnorm_tp_plan_info* p, int64_t rows, int32_t* counts) {
  if (!p || (!counts && rows > 0)) return fail(RMSNORM_TP_ERR_INVALID, "plan_coverage: NULL");
  if (p->grid < 1 || p->teams_per_cta < 1 || p->rows_per_tile < 1)
    return fail(RMSNORM_TP_ERR_INVALID, "plan_coverage: malformed plan");
  for (int64_t i = 0; i < rows; ++i) counts[i] = 0;
  if (p->variant >= rtp::kBatchBase && p->variant < rtp::kResidentBase) {
    // Batch kernels: CTA c owns batches [B c / G, B (c + 1) / G) of rows_per_tile rows.
    const int64_t B = (rows + p->rows_per_tile - 1) / p->rows_per_tile;
    const int64_t G = p->grid;
    for (int64_t c = 0; c < G; ++c)
      for (int64_t b = B * c / G; b < B * (c + 1) / G; ++b)
        for (int r = 0; r < p->rows_per_tile; ++r) {
          const int64_t row = b * p->rows_per_tile + r;
          if (row < rows) counts[row] += 1;
        }
    return RMSNORM_TP_OK;
  }
  // Same walk as the kernels: team g visits tiles g, g + T, g + 2T, ... (T = all teams).
  const int64_t teams_total = (int64_t)p->grid * p->teams_per_cta;
  const int64_t tiles = (rows + p->rows_per_tile - 1) / p->rows_per_tile;
  for (int64_t g = 0; g < teams_total; ++g) {
    for (int64_t it = 0;; ++it) {
      const int64_t t = rtp::tile_of(g, it, teams_total);
      if (t >= tiles) break;
      for (int r = 0; r < p->rows_per_tile; ++r) {
        const int64_t row = t * p->rows_per_tile + r;
        if (row < rows) counts[row] += 1;
      }
    }
  }
  return RMSNORM_TP_OK;
}

}  // extern "C"
