// mep_dest_ranks_noalloc: the replica round-robin destination scan for callers
// that cannot allocate device memory.
//
// Who needs it: a serving process that hands all free HBM to its own pool at
// start-up (a later cudaMalloc fails or fragments that pool), and host code on
// a latency-critical path, where cudaMalloc/cudaFree would synchronise the
// device and stall the streams in flight. Such callers cannot create a
// mep_ctx, which allocates its buffers. This entry point takes the placement
// table on the host, the round-robin state and the ids on the device, and
// keeps its intermediate buffers in one fixed, file-scope device array
// instead of allocating any.
//
// Limits and sharing rules:
//   * at most kNoAllocMaxIds expert ids per call, at most 128 experts and
//     8 ranks; larger calls are rejected with MEP_ERR_INVALID;
//   * the array below (about 650 KiB) is reserved on every GPU that loads
//     this library, until the process exits;
//   * every call uses the same array: calls whose kernels may overlap on a
//     GPU (other streams, other host threads) race and must be serialised
//     by the caller. Each call writes every scratch word it later reads, so
//     nothing has to be cleared between calls;
//   * every call copies the placement from pageable host (stack) memory with
//     cudaMemcpyAsync, and the first call on each device looks up the
//     array's device address (cudaGetSymbolAddress): no call may be made
//     while its stream is being captured;
//   * an id outside [0, E) gets destination -1 and is left out of the
//     round-robin advance, as in mep_dest_ranks, but there is no context
//     error word to report it in: callers validate ids that can be invalid.
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "miniep_b200.h"
#include "mep_internal.h"

namespace mep {
void set_global_error(const std::string& msg);  // mep_api.cu: read by mep_last_error(NULL)
}

using namespace mep;

namespace {

constexpr int64_t kNoAllocMaxIds = 65536;
constexpr int64_t kNoAllocChunks = kNoAllocMaxIds / kRouteChunkTokens;
// byte offsets inside the scratch array
constexpr size_t kOffHist = 0;
constexpr size_t kOffDest = kOffHist + kNoAllocChunks * kMaxExperts * sizeof(int32_t);
constexpr size_t kOffGrp = kOffDest + kNoAllocMaxIds * sizeof(int32_t);
constexpr size_t kOffOwners = kOffGrp + kNoAllocMaxIds * sizeof(int32_t);
constexpr size_t kOffNrep = kOffOwners + kMaxExperts * kMaxWorld * sizeof(int32_t);
constexpr size_t kScratchBytes = kOffNrep + kMaxExperts * sizeof(int32_t);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

int invalid(const std::string& msg) {
  set_global_error("mep_dest_ranks_noalloc: " + msg);
  return MEP_ERR_INVALID;
}

int cuda_error(cudaError_t e, const char* what) {
  set_global_error(std::string("mep_dest_ranks_noalloc: ") + what + ": " + cudaGetErrorString(e));
  return MEP_ERR_CUDA;
}

// Device address of the scratch array on the current device (looked up once
// per device; the host-side name g_noalloc_scratch is not a device address).
int scratch_on_current_device(unsigned char** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return invalid("device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress");
    g_scratch_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
  return MEP_OK;
}

}  // namespace

extern "C" int mep_dest_ranks_noalloc(int num_experts, int world, const int64_t* table,
                                      const int64_t* n_rep, int rmax, int64_t* rr,
                                      const int64_t* expert_ids, int64_t m, int64_t* dest_out,
                                      void* stream) {
  if (num_experts < 1 || num_experts > kMaxExperts) return invalid("num_experts must be 1..128");
  if (world < 1 || world > kMaxWorld) return invalid("world must be 1..8");
  if (rmax < 1 || rmax > kMaxWorld) return invalid("rmax must be 1..8");
  if (m < 0 || m > kNoAllocMaxIds)
    return invalid("m = " + std::to_string(m) + " exceeds the fixed scratch (at most " +
                   std::to_string(kNoAllocMaxIds) + " ids per call)");
  if (!table || !n_rep || !rr) return invalid("table, n_rep and rr are required");
  if (m > 0 && (!expert_ids || !dest_out)) return invalid("expert_ids and dest_out are required");

  // placement in the kernels' layout, validated on the host (stack arrays only)
  int32_t own[kMaxExperts * kMaxWorld];
  int32_t nr[kMaxExperts];
  for (int e = 0; e < num_experts; ++e) {
    const int64_t n = n_rep[e];
    if (n < 1 || n > rmax || n > world) return invalid("n_rep out of range");
    for (int j = 0; j < n; ++j) {
      const int64_t r = table[(int64_t)e * rmax + j];
      if (r < 0 || r >= world) return invalid("owner rank out of range");
      for (int i = 0; i < j; ++i)
        if (own[e * kMaxWorld + i] == r) return invalid("duplicate owner");
      own[e * kMaxWorld + j] = (int32_t)r;
    }
    for (int j = (int)n; j < kMaxWorld; ++j) own[e * kMaxWorld + j] = own[e * kMaxWorld];
    nr[e] = (int32_t)n;
  }

  unsigned char* s = nullptr;
  if (int rc = scratch_on_current_device(&s)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(s + kOffOwners, own, (size_t)num_experts * kMaxWorld * 4,
                                  cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync(table)");
  e = cudaMemcpyAsync(s + kOffNrep, nr, (size_t)num_experts * 4, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync(n_rep)");

  launch_dest_only(m, num_experts, expert_ids, reinterpret_cast<const int32_t*>(s + kOffOwners),
                   reinterpret_cast<const int32_t*>(s + kOffNrep), rr,
                   reinterpret_cast<int32_t*>(s + kOffHist), reinterpret_cast<int32_t*>(s + kOffDest),
                   reinterpret_cast<int32_t*>(s + kOffGrp), dest_out, WaitCfg{nullptr, 0}, st);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "kernel launch");
  return MEP_OK;
}
