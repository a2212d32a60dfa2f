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
//  * The array's device address is looked up with cudaGetSymbolAddress, once
//    per device, with that device current: by mla_noalloc_init(), or else by
//    the first decode call on the device.  Make one of them before any stream
//    capture begins.
//  * All calls share the one array, which keeps the last call's contents.
//    The bytes the kernels need zeroed on entry (the tensor-core kernel's status
//    word and piece counters, mla_describe_plan out4[3]) are cleared with a
//    cudaMemsetAsync on the caller's stream before each launch; everything else
//    is overwritten before it is read.  Two calls whose kernels overlap on the
//    GPU (different streams without ordering between them) race on the array
//    and both results are undefined.  Serialise such calls on one stream.
//  * A call that is rejected (bad shape, pointer, alignment or config, or too
//    much scratch) enqueues nothing, so it cannot disturb a call in flight.
//  * The array starts with a status block: the tensor-core kernel's own (its
//    workspace begins with it), or, for a CUDA-core call, 256 bytes kept in
//    front of that kernel's scratch.  Every call clears the status word; the
//    tensor-core kernel records there a bounded wait that gave up.
//    mla_noalloc_status copies the word out (on the stream, after the call it
//    concerns and before the next one).
//  * Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>

#include "mla_common.cuh"

namespace mla {
namespace {

constexpr size_t kNoAllocScratchBytes = MLA_NOALLOC_SCRATCH_BYTES;
constexpr size_t kStatusBlock = 256;   // status block in front of a CUDA-core call's scratch
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
    set_error("mla noalloc scratch: cudaGetDevice failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("mla noalloc scratch: device ordinal %d out of range", dev);
    return MLA_ERR_ARG;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr) {
      set_error("mla noalloc scratch: cudaGetSymbolAddress failed on device %d: %s", dev,
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

int32_t mla_noalloc_init(void) {
  mla::set_error("%s", "");
  void* scratch = nullptr;
  return mla::scratch_address(&scratch);
}

int32_t mla_noalloc_status(uint32_t* status_out, void* stream) {
  if (status_out == nullptr) {
    mla::set_error("mla_noalloc_status: null output");
    return MLA_ERR_ARG;
  }
  void* scratch = nullptr;
  const int rc = mla::scratch_address(&scratch);
  if (rc != MLA_OK) return rc;
  // the status word is the first 4 bytes of the array (the tensor-core kernel's
  // workspace header); cudaMemcpyDefault: status_out may be device or host memory
  const cudaError_t err = cudaMemcpyAsync(status_out, scratch, sizeof(uint32_t), cudaMemcpyDefault,
                                          static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    mla::set_error("mla_noalloc_status: copy failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

int32_t mla_decode_fwd_noalloc(const void* q, const void* q_pe, const void* kv, const void* k_pe,
                               void* out, float* lse, int32_t batch, int32_t heads,
                               int32_t seqlen_kv, int32_t dtype, const MlaCfg* cfg, void* stream) {
  const char* fn = "mla_decode_fwd_noalloc";
  mla::set_error("%s", "");
  // Everything mla_decode_fwd would reject is rejected here first: nothing may be
  // enqueued on the shared array for a call that then fails its checks.
  int rc = mla::check_decode_call(fn, q, q_pe, kv, k_pe, out, batch, heads, seqlen_kv, dtype, cfg);
  if (rc != MLA_OK) return rc;
  int64_t info[4];
  rc = mla_describe_plan(batch, heads, seqlen_kv, dtype, cfg, info);
  if (rc != MLA_OK) return rc;
  // The tensor-core kernel's workspace starts with its status block; the CUDA-core
  // kernel's has none, so its scratch starts kStatusBlock bytes in and the block
  // in front of it only carries a zero status word: mla_noalloc_status then means
  // the same after either kernel.
  const bool tc = info[3] > 0;
  const size_t front = tc ? 0 : mla::kStatusBlock;
  const size_t need = mla_workspace_bytes(batch, heads, seqlen_kv, dtype, cfg);
  if (need + front > mla::kNoAllocScratchBytes) {
    mla::set_error(
        "%s: this shape needs %zu bytes of scratch but the static array holds %zu; use "
        "mla_decode_fwd with a caller workspace, or fewer splits",
        fn, need + front, mla::kNoAllocScratchBytes);
    return MLA_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  rc = mla::scratch_address(&scratch);
  if (rc != MLA_OK) return rc;
  // The array keeps whatever the previous call left; the part the kernels need
  // zeroed on entry (tensor-core status word and piece counters), or the status
  // word alone, is cleared here.
  const cudaError_t err = cudaMemsetAsync(scratch, 0, tc ? (size_t)info[3] : sizeof(uint32_t),
                                          static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    mla::set_error("%s: clearing the scratch header failed: %s", fn, cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return mla_decode_fwd(q, q_pe, kv, k_pe, out, lse, static_cast<char*>(scratch) + front,
                        mla::kNoAllocScratchBytes - front, batch, heads, seqlen_kv, dtype, cfg, stream);
}

}  // extern "C"
