// rmsnorm_tp_forward_group_static: the fused TP RMSNorm of a whole TP group
// held on one GPU, for callers that cannot allocate device memory.
//
// Some callers may not call cudaMalloc at all: serving runtimes that size
// their device memory pool once at start-up and treat any later allocation as
// an out-of-budget failure, and plugin hosts that hand a kernel its input and
// output buffers and nothing else. The regular path allocates a mailbox and a
// device state per rank (rmsnorm_tp_create); this entry point instead keeps
// them in the file-scope array below, which every GPU that loads the library
// holds (4 MiB) until the process exits.
//
// The array's name is only a host-side stand-in in host code: its device
// address is looked up once per device with cudaGetSymbolAddress (with that
// device current) and that address is what the kernel receives.
//
// A wait that runs out inside the kernel cannot be returned by the call that
// launched it (the call has returned by then): it writes NaN rows and records
// the failure in the rank's state in the array, where
// rmsnorm_tp_forward_group_static_status reads it until the next call clears it.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/rmsnorm_tp_b200.h"
#include "internal.h"
#include "rtp_common.h"

namespace {

constexpr size_t kScratchBytes = RMSNORM_TP_STATIC_SCRATCH_BYTES;
constexpr size_t kStateStride = 256;                // one DeviceState per rank, padded
constexpr unsigned long long kStaticTimeoutNs = 10ull * 1000ull * 1000ull * 1000ull;
static_assert(sizeof(rtp::DeviceState) <= kStateStride, "state fits its stride");

static __device__ __align__(256) unsigned char g_group_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<unsigned char*> g_scratch_ptr[kMaxDevices];
std::atomic<int> g_last_tp[kMaxDevices];   // group size of the last call per device (0: none)
std::mutex g_setup_mutex;

int fail_static(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail_static(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return rtp::record_error(code, buf);   // reported by rmsnorm_tp_last_error()
}

// Device address of g_group_scratch on `device` (the current device), looked up
// on the first call for that device.
int scratch_of(int device, unsigned char** out) {
  unsigned char* p = g_scratch_ptr[device].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_ptr[device].load(std::memory_order_acquire);
    if (p == nullptr) {
      void* addr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&addr, g_group_scratch);
      if (e != cudaSuccess)
        return fail_static(RMSNORM_TP_ERR_CUDA, "forward_group_static: cudaGetSymbolAddress: %s",
                           cudaGetErrorString(e));
      p = static_cast<unsigned char*>(addr);
      g_scratch_ptr[device].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return RMSNORM_TP_OK;
}

}  // namespace

extern "C" int rmsnorm_tp_forward_group_static(int tp, void* const* outs, const void* const* xs,
                                               const void* const* weights, int64_t rows,
                                               int64_t local_hidden, int dtype, float eps,
                                               void* stream) {
  if (tp < 2 || tp > rtp::kMaxTP)
    return fail_static(RMSNORM_TP_ERR_INVALID, "forward_group_static: tp %d outside [2, %d]", tp,
                       rtp::kMaxTP);
  if (!outs || !xs || !weights)
    return fail_static(RMSNORM_TP_ERR_INVALID, "forward_group_static: NULL pointer array");
  if (dtype < RMSNORM_TP_F32 || dtype > RMSNORM_TP_F16)
    return fail_static(RMSNORM_TP_ERR_INVALID, "forward_group_static: unknown dtype %d", dtype);
  if (rows < 0 || local_hidden < 1 || local_hidden > (int64_t(1) << 31))
    return fail_static(RMSNORM_TP_ERR_INVALID,
                       "forward_group_static: rows %lld, local_hidden %lld out of range",
                       (long long)rows, (long long)local_hidden);
  for (int r = 0; r < tp; ++r)
    if (rows > 0 && (!outs[r] || !xs[r] || !weights[r]))
      return fail_static(RMSNORM_TP_ERR_INVALID, "forward_group_static: NULL tensor of rank %d", r);
  if (rows == 0) return RMSNORM_TP_OK;
  // per rank: one state + a mailbox u64 slot[2][tp][rows]. The row limit is
  // checked before any product is formed, so a huge `rows` cannot wrap the
  // byte count around to a small number.
  const int64_t max_rows =
      (int64_t)((kScratchBytes - (size_t)tp * kStateStride) / (16ull * (size_t)tp * (size_t)tp));
  if (rows > max_rows)
    return fail_static(RMSNORM_TP_ERR_ROWS,
                       "forward_group_static: %d ranks x %lld rows do not fit; the static scratch "
                       "holds %zu bytes (16 * tp^2 * rows + 256 * tp bytes must fit: at most "
                       "%lld rows at tp %d)",
                       tp, (long long)rows, kScratchBytes, (long long)max_rows, tp);
  const size_t mailbox_bytes = (size_t)rtp::mailbox_slots(tp, rows) * sizeof(unsigned long long);
  const size_t need = (size_t)tp * kStateStride + (size_t)tp * mailbox_bytes;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= kMaxDevices)
    return fail_static(RMSNORM_TP_ERR_CUDA, "forward_group_static: cudaGetDevice: %s",
                       cudaGetErrorString(e));
  unsigned char* scratch = nullptr;
  const int rc = scratch_of(device, &scratch);
  if (rc != RMSNORM_TP_OK) return rc;

  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The array keeps the last call's contents: start from zeroed states
  // (generation 0) and zeroed mailboxes. Stream-ordered before the launch.
  e = cudaMemsetAsync(scratch, 0, need, s);
  if (e != cudaSuccess)
    return fail_static(RMSNORM_TP_ERR_CUDA, "forward_group_static: clearing scratch: %s",
                       cudaGetErrorString(e));
  rtp::KArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int r = 0; r < tp; ++r) {
    auto* st = reinterpret_cast<rtp::DeviceState*>(scratch + (size_t)r * kStateStride);
    a.rp[r] = rtp::RankPtrs{outs[r], xs[r], weights[r], st, nullptr};
    a.mbox[r] = reinterpret_cast<unsigned long long*>(scratch + (size_t)tp * kStateStride +
                                                      (size_t)r * mailbox_bytes);
  }
  a.rows = rows;
  a.hl = local_hidden;
  a.nmax = rows;
  a.hidden_f = (float)(local_hidden * tp);
  a.eps = eps;
  a.rank = 0;
  a.tp = tp;
  a.emulated = 1;
  a.timeout_ns = kStaticTimeoutNs;
  a.prof = nullptr;
  e = rtp::launch_forward(a, dtype, device, tp, s, nullptr);
  if (e != cudaSuccess)
    return fail_static(RMSNORM_TP_ERR_CUDA, "forward_group_static: cooperative launch: %s",
                       cudaGetErrorString(e));
  g_last_tp[device].store(tp, std::memory_order_release);
  return RMSNORM_TP_OK;
}

extern "C" int rmsnorm_tp_forward_group_static_status(rmsnorm_tp_status_info* out) {
  if (!out) return fail_static(RMSNORM_TP_ERR_INVALID, "forward_group_static_status: NULL out");
  std::memset(out, 0, sizeof(*out));
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= kMaxDevices)
    return fail_static(RMSNORM_TP_ERR_CUDA, "forward_group_static_status: cudaGetDevice: %s",
                       cudaGetErrorString(e));
  const int tp = g_last_tp[device].load(std::memory_order_acquire);
  if (tp == 0)
    return fail_static(RMSNORM_TP_ERR_STATE,
                       "forward_group_static_status: no call on device %d yet", device);
  unsigned char* scratch = nullptr;
  const int rc = scratch_of(device, &scratch);
  if (rc != RMSNORM_TP_OK) return rc;
  // the last call's kernel must have finished before its states are read
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess)
    return fail_static(RMSNORM_TP_ERR_CUDA, "forward_group_static_status: synchronize: %s",
                       cudaGetErrorString(e));
  for (int r = 0; r < tp; ++r) {
    rtp::DeviceState st;
    e = cudaMemcpy(&st, scratch + (size_t)r * kStateStride, sizeof(st), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess)
      return fail_static(RMSNORM_TP_ERR_CUDA, "forward_group_static_status: reading state: %s",
                         cudaGetErrorString(e));
    if (r == 0) out->next_generation = st.call >> rtp::kGenShift;
    if (st.err_code != rtp::kStatusOk && out->code == rtp::kStatusOk) {
      out->code = st.err_code;
      out->src_rank = st.err_src;
      out->row = st.err_row;
      out->expected_tag = st.err_expected;
      out->seen_tag = st.err_seen;
      out->generation = st.err_call;
    }
  }
  return RMSNORM_TP_OK;
}
