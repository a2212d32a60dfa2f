// mla_decode_fwd_noalloc: the decode call for callers that cannot allocate
// device memory.
//
// Some callers of a decode kernel are not allowed to call cudaMalloc (or any
// allocating library routine) at the point where they decode: code that runs
// while a CUDA graph is being captured, inference servers that reserve all
// device memory up front and forbid allocation on the serving path, and
// plugin hosts whose memory is owned by another runtime.  They still pass
// their own inputs and outputs, but cannot hand us a workspace.  This entry
// point takes its split-KV scratch (per-split partial outputs and
// log-sum-exps) from a fixed file-scope __device__ array instead.
//
// Limits and rules:
//  * The array holds kNoAllocScratchBytes (8 MiB).  A shape/config whose
//    workspace (mla_workspace_bytes) is larger is rejected with
//    MLA_ERR_WORKSPACE and a message; nothing is launched.
//  * Every GPU that loads this library holds the 8 MiB until the process
//    exits.
//  * The first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (once per device, with that device current).  Make
//    that first call before any stream capture begins.
//  * All calls share the one array, which keeps the last call's contents.
//    The bytes the kernels need zeroed on entry (the tensor-core kernel's status
//    word and piece counters, mla_describe_plan out4[3]) are cleared with a
//    cudaMemsetAsync on the caller's stream before each launch; everything else
//    is overwritten before it is read.  Two calls whose kernels overlap on the
//    GPU (different streams without ordering between them) race on the array
//    and both results are undefined.  Serialise such calls on one stream.
//  * Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>

#include "mla_common.cuh"

namespace mla {
namespace {

constexpr size_t kNoAllocScratchBytes = MLA_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code `g_noalloc_scratch` is only a host-side
// stand-in for the symbol, never a device address: the device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    set_error("mla_decode_fwd_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("mla_decode_fwd_noalloc: device ordinal %d out of range", dev);
    return MLA_ERR_ARG;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr) {
      set_error("mla_decode_fwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(err));
      return MLA_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MLA_OK;
}

}  // namespace
}  // namespace mla

extern "C" {

int32_t mla_decode_fwd_noalloc(const void* q, const void* q_pe, const void* kv, const void* k_pe,
                               void* out, float* lse, int32_t batch, int32_t heads,
                               int32_t seqlen_kv, int32_t dtype, const MlaCfg* cfg, void* stream) {
  mla::set_error("%s", "");   // so a 0 below is told apart from a rejected shape
  const size_t need = mla_workspace_bytes(batch, heads, seqlen_kv, dtype, cfg);
  if (need == 0 && mla_last_error()[0] != '\0') return MLA_ERR_ARG;   // bad shape/config
  if (need > mla::kNoAllocScratchBytes) {
    mla::set_error(
        "mla_decode_fwd_noalloc: this shape needs %zu bytes of scratch but the static array "
        "holds %zu; use mla_decode_fwd with a caller workspace, or fewer splits",
        need, mla::kNoAllocScratchBytes);
    return MLA_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  int rc = mla::scratch_address(&scratch);
  if (rc != MLA_OK) return rc;
  // The array keeps whatever the previous call left; the part the kernels need
  // zeroed on entry (tensor-core status word and piece counters) is cleared here.
  int64_t info[4];
  rc = mla_describe_plan(batch, heads, seqlen_kv, dtype, cfg, info);
  if (rc != MLA_OK) return rc;
  if (info[3] > 0) {
    const cudaError_t err =
        cudaMemsetAsync(scratch, 0, (size_t)info[3], static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) {
      mla::set_error("mla_decode_fwd_noalloc: clearing the scratch header failed: %s",
                     cudaGetErrorString(err));
      return MLA_ERR_CUDA;
    }
  }
  return mla_decode_fwd(q, q_pe, kv, k_pe, out, lse, scratch, mla::kNoAllocScratchBytes, batch,
                        heads, seqlen_kv, dtype, cfg, stream);
}

}  // extern "C"
