// The sequence split's exchange over NVLink peer memory, without a collective library.
//
// Every rank (one GPU each, all on one node) decodes its part of every sequence's KV
// rows to a float32 (O, LSE) block (mla_decode_partial) in its own gather buffer;
// the merge needs every rank's block.  Instead of an all-gather, each rank pushes its
// block straight into every peer's gather buffer (plain 16-byte stores to peer
// memory through the CUDA IPC mapping of that buffer), and one flag per (call
// parity, source rank) in the receiving buffer says the block is complete.  The
// same launch then waits, with a time limit, until every peer's block has arrived
// in its own buffer; the LSE combine (mla_combine_strided) merges the blocks where
// they landed.  Blocks and flags are double-buffered by the call's parity: a rank
// can only start pushing call k + 1 after its own call k merged, which waited for
// every peer's call-k push, which each peer issued after its own call k - 1 merge;
// so call k + 1 never overwrites a block a peer still reads.
//
// The buffer layout (every rank's is the same) is in mla_common.cuh; this file
// uses its blocks, block flags, push counter and status word.  The same buffers
// serve mla_seqsplit_decode / mla_seqsplit_merge (one launch that exchanges and
// merges row by row, in mla_sm100.cu), which use the row flags.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include <mutex>

#include "mla_common.cuh"

namespace mla {
namespace {

constexpr int kMaxWorld = kSeqMaxWorld;
constexpr int kPushThreads = 256;
constexpr int kPushBlocks = 32;

struct Xchg {
  float* bufs[kMaxWorld];   // every rank's buffer as mapped in this process
  size_t chunk;             // floats per block
  size_t header;            // byte offset of the header in a buffer
  int world, rank, par;
  uint32_t epoch;
};

__device__ __forceinline__ uint32_t* header_of(const Xchg& x, int r) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(x.bufs[r]) + x.header);
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kPushThreads) mla_seqsplit_push_kernel(Xchg x) {
  // this rank's block of this call's parity, the same place in every buffer
  const size_t off = ((size_t)x.par * x.world + x.rank) * x.chunk;
  const float4* src = reinterpret_cast<const float4*>(x.bufs[x.rank] + off);
  const size_t n4 = x.chunk / 4;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = src[i];
#pragma unroll 1
    for (int p = 0; p < x.world; ++p)
      if (p != x.rank) reinterpret_cast<float4*>(x.bufs[p] + off)[i] = v;
  }
  // every thread's peer stores are visible system-wide before its CTA counts itself
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t* mine = header_of(x, x.rank);
  if (atomicAdd(mine + 16, 1u) + 1u != gridDim.x) return;
  // the last CTA: every CTA's stores are fenced; reset the counter, raise this
  // rank's flag in every peer's buffer, then wait for every peer's flag here
  mine[16] = 0u;
  __threadfence_system();
  for (int p = 0; p < x.world; ++p)
    if (p != x.rank) st_release_sys(header_of(x, p) + x.par * kMaxWorld + x.rank, x.epoch);
  const unsigned long long t0 = now_ns();
  for (int q = 0; q < x.world; ++q) {
    if (q == x.rank) continue;
    const uint32_t* f = mine + x.par * kMaxWorld + q;
    while ((int)(ld_acquire_sys(f) - x.epoch) < 0) {
      if (now_ns() - t0 > kSeqWaitNs) {
        atomicCAS(mine + 17, 0u, kErrExchange);   // a peer never delivered: the merge is invalid
        return;
      }
      __nanosleep(64);
    }
  }
}

// cuMemGetAddressRange through the runtime's driver entry point (the library links
// only the CUDA runtime)
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(f);
  });
  return fn;
}

}  // namespace
}  // namespace mla

using namespace mla;

extern "C" {

size_t mla_seqsplit_buffer_bytes(int32_t world, int32_t batch, int32_t heads) {
  if (world < 1 || world > kMaxWorld || batch < 1 || heads < 1) {
    set_error("mla_seqsplit_buffer_bytes: world must be 1..%d and batch, heads >= 1", kMaxWorld);
    return 0;
  }
  return seq_buffer_bytes(world, batch, heads);
}

int32_t mla_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr) {
    set_error("mla_ipc_export: null pointer");
    return MLA_ERR_ARG;
  }
  // the handle names the whole allocation: find its base
  CUdeviceptr base = 0;
  size_t size = 0;
  cudaPointerAttributes attr{};
  cudaError_t err = cudaPointerGetAttributes(&attr, ptr);
  if (err != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
    set_error("mla_ipc_export: not device memory (%s)", cudaGetErrorString(err));
    return MLA_ERR_ARG;
  }
  const AddressRangeFn range = address_range_fn();
  if (range == nullptr || range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("mla_ipc_export: cuMemGetAddressRange failed");
    return MLA_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) {
    set_error("mla_ipc_export: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return MLA_OK;
}

int32_t mla_ipc_import(const void* handle, uint64_t offset, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) {
    set_error("mla_ipc_import: null pointer");
    return MLA_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) {
    set_error("mla_ipc_import: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  *ptr_out = static_cast<char*>(base) + offset;
  return MLA_OK;
}

int32_t mla_ipc_close(void* ptr, uint64_t offset) {
  if (ptr == nullptr) return MLA_OK;
  const cudaError_t err = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (err != cudaSuccess) {
    set_error("mla_ipc_close: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

int32_t mla_seqsplit_exchange(void* const* bufs, int32_t world, int32_t rank, uint32_t epoch, int32_t batch,
                              int32_t heads, void* stream) {
  if (bufs == nullptr || world < 2 || world > kMaxWorld || rank < 0 || rank >= world || batch < 1 || heads < 1 ||
      epoch == 0) {
    set_error("mla_seqsplit_exchange: bad argument (world %d, rank %d, epoch %u)", world, rank, epoch);
    return MLA_ERR_ARG;
  }
  Xchg x{};
  for (int r = 0; r < world; ++r) {
    if (bufs[r] == nullptr || (reinterpret_cast<uintptr_t>(bufs[r]) & 255u) != 0) {
      set_error("mla_seqsplit_exchange: buffer %d is null or not 256-byte aligned", r);
      return MLA_ERR_ARG;
    }
    x.bufs[r] = static_cast<float*>(bufs[r]);
  }
  x.chunk = seq_chunk_floats(batch, heads);
  x.header = seq_header_offset(world, batch, heads);
  x.world = world;
  x.rank = rank;
  x.par = (int)(epoch & 1u);
  x.epoch = epoch;
  mla_seqsplit_push_kernel<<<kPushBlocks, kPushThreads, 0, static_cast<cudaStream_t>(stream)>>>(x);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error("mla_seqsplit_exchange: launch failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

}  // extern "C"
