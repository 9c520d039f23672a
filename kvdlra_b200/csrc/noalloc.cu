// kvd_bug_step_noalloc: the batched BUG step for callers that cannot allocate.
//
// Some callers of this library run where they may not allocate device memory
// at all: a host runtime that reserves its whole memory pool up front and owns
// every allocation, a plugin loaded into such a runtime, or code that must not
// synchronise the device (cudaMalloc/cudaFree can).  kvd_bug_step needs a
// caller-provided workspace; this entry point instead uses a fixed scratch
// area that lives in the library itself, so the caller passes only its inputs
// and outputs.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (16 MiB).  Every GPU that loads the library holds it until the process
// exits.  Its device address is looked up once per device, with that device
// current, by the first call on that device -- so make that first call before
// any stream capture.  A call uses the scratch of the device that is current
// on the calling thread, so the stream it is given must belong to that device
// (as every entry point of this library assumes).  All calls share the one
// array and it keeps the last call's contents; nothing in it has to start at
// zero (the step writes every scratch value before reading it).  Two calls whose executions overlap on the
// GPU (different streams, or concurrent host threads) race on the scratch and
// must be serialised by the caller.
#include <mutex>

#include "kernels.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
using kvd::kMaxDevices;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device (set up once per
// device).  In host code the symbol name is only a host-side handle, never a
// device address, so it is never passed to a kernel directly.
int scratch_for_current_device(unsigned char** out) {
  static std::mutex mu;
  static unsigned char* addr[kMaxDevices] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    kvd_host::set_error("kvd_bug_step_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return KVD_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    kvd_host::set_error("kvd_bug_step_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
    return KVD_ERR_ARG;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      kvd_host::set_error("kvd_bug_step_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return KVD_ERR_CUDA;
    }
    addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = addr[dev];
  return KVD_OK;
}

inline long a16(long x) { return (x + 15) & ~15L; }

}  // namespace

extern "C" size_t kvd_bug_step_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

extern "C" int kvd_bug_step_noalloc(int32_t n_batch, int32_t n, int32_t b, int32_t rank_cap,
                                    int32_t ld_u, const float* u, float* u_out, float* sigma,
                                    int32_t* r, const float* block, float* rot_out,
                                    int32_t* m_out, float* coords_out, int32_t has_theta,
                                    float theta, int32_t* status, kvd_stream_t stream) {
  using namespace kvd_host;
  if (n_batch <= 0 || n <= 0 || b <= 0 || rank_cap < 1 || rank_cap > ld_u) {
    set_error("kvd_bug_step_noalloc: bad sizes (n_batch=%d n=%d b=%d rank_cap=%d ld=%d)", n_batch,
              n, b, rank_cap, ld_u);
    return KVD_ERR_ARG;
  }
  const long per = bug_step_ws_per_problem(n, b, ld_u);
  const long dims_bytes = a16(16L * n_batch);
  const size_t need = (size_t)dims_bytes + (size_t)n_batch * (size_t)per;
  if (need > kNoAllocScratchBytes) {
    set_error("kvd_bug_step_noalloc: %d problems of n=%d, b=%d, rank width %d need %zu bytes of "
              "scratch, more than the fixed %zu; use kvd_bug_step with a workspace",
              n_batch, n, b, ld_u, need, kNoAllocScratchBytes);
    return KVD_ERR_WORKSPACE;
  }
  if (u == u_out) {
    set_error("kvd_bug_step_noalloc: u_out must not alias u");
    return KVD_ERR_ARG;
  }
  unsigned char* base = nullptr;
  if (int rc = scratch_for_current_device(&base)) return rc;
  int* dims = reinterpret_cast<int*>(base);
  char* ws = reinterpret_cast<char*>(base + dims_bytes);
  kvd::BugStepBatch batch;
  kvd::BugStepArgs& a = batch.s[0];
  a.n = n; a.b = b; a.rank_cap = rank_cap; a.ld = ld_u;
  a.u = u; a.u_out = u_out; a.u_sp = (long)n * ld_u;
  a.sigma = sigma; a.sig_sp = ld_u; a.r = r;
  a.x = block; a.x_sp = (long)b * n;
  a.rot = rot_out; a.rot_sp = (long)ld_u * ld_u;
  a.dims = dims;
  a.coords = coords_out; a.coords_sp = (long)b * ld_u; a.coords_ld = ld_u;
  a.has_theta = has_theta; a.theta = theta; a.status = status;
  a.ws = ws; a.ws_sp = per;
  batch.s[1] = a;
  int rc = launch_bug_step(batch, n_batch, 1, (cudaStream_t)stream);
  if (rc) return rc;
  if (m_out) {
    const cudaError_t e = cudaMemcpy2DAsync(m_out, sizeof(int32_t), dims + 2, 4 * sizeof(int),
                                            sizeof(int32_t), n_batch, cudaMemcpyDeviceToDevice,
                                            (cudaStream_t)stream);
    if (e != cudaSuccess) {
      set_error("kvd_bug_step_noalloc: copying m: %s", cudaGetErrorString(e));
      return KVD_ERR_CUDA;
    }
  }
  return check_launch("kvd_bug_step_noalloc");
}
