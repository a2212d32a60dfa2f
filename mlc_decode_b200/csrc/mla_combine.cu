// LSE combine of split-KV partial results.
//
// Restates the reference's combine kernel (mla_decode.py:194-246): the global
// log-sum-exp of a (batch, head) row is LSE = m + log(sum_k exp(lse_k - m)),
// m = max_k lse_k, and out = sum_k exp(lse_k - LSE) * o_k.  The reference
// pads its LSE vector to a multiple of 64 with -inf and tree-reduces; here a
// CTA of 128 threads owns one row: the max and sum are block reductions over
// the splits (strided, any count), the weights go to shared memory, and each
// thread accumulates 4 consecutive latent columns with 16-byte loads, four
// splits in flight per iteration.  All LSEs are natural-log.
#include <math.h>

#include "mla_common.cuh"

namespace mla {
namespace {

constexpr int kThreads = 128;   // 128 threads x 4 columns = 512
constexpr int kMaxSplits = 8192;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <typename T>
__device__ __forceinline__ void store4(T* dst, float4 v);
template <>
__device__ __forceinline__ void store4<__half>(__half* dst, float4 v) {
  uint2 w;
  w.x = Elt<__half>::pack2(v.x, v.y);
  w.y = Elt<__half>::pack2(v.z, v.w);
  *reinterpret_cast<uint2*>(dst) = w;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float4 v) {
  uint2 w;
  w.x = Elt<__nv_bfloat16>::pack2(v.x, v.y);
  w.y = Elt<__nv_bfloat16>::pack2(v.z, v.w);
  *reinterpret_cast<uint2*>(dst) = w;
}

template <>
__device__ __forceinline__ void store4<float>(float* dst, float4 v) {
  *reinterpret_cast<float4*>(dst) = v;
}

// Split k's LSE of row r is part_lse[k * lse_stride + r], its O row starts at
// part_o + k * o_stride + r * 512 (strides in floats; o_stride a multiple of 4).
template <typename T>
__global__ void __launch_bounds__(kThreads)
mla_combine_kernel(const float* __restrict__ part_lse, const float* __restrict__ part_o,
                   int ns, int rows, size_t lse_stride, size_t o_stride, T* __restrict__ out,
                   float* __restrict__ lse_out) {
  extern __shared__ float s_w[];        // [ns] weights
  __shared__ float s_red[kThreads / 32];
  __shared__ float s_bcast;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  float mx = -INFINITY;
  for (int k = tid; k < ns; k += kThreads) mx = fmaxf(mx, part_lse[(size_t)k * lse_stride + row]);
  mx = warp_max(mx);
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float v = s_red[0];
    for (int w = 1; w < kThreads / 32; ++w) v = fmaxf(v, s_red[w]);
    s_bcast = v;
  }
  __syncthreads();
  mx = s_bcast;
  const bool all_empty = !(mx > -INFINITY);
  const float msafe = all_empty ? 0.f : mx;

  float sum = 0.f;
  for (int k = tid; k < ns; k += kThreads)
    sum += exp2f((part_lse[(size_t)k * lse_stride + row] - msafe) * kLog2e);
  sum = warp_sum(sum);
  __syncthreads();
  if (lane == 0) s_red[warp] = sum;
  __syncthreads();
  if (tid == 0) {
    float v = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) v += s_red[w];
    s_bcast = v;
  }
  __syncthreads();
  const float lse = all_empty ? -INFINITY : msafe + logf(s_bcast);
  for (int k = tid; k < ns; k += kThreads)
    s_w[k] = all_empty ? 0.f : exp2f((part_lse[(size_t)k * lse_stride + row] - lse) * kLog2e);
  __syncthreads();

  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* po = reinterpret_cast<const float4*>(part_o) + (size_t)row * (kDim / 4) + tid;
  const size_t split_stride = o_stride / 4;
  // eight partial rows in flight per thread and round (the tail rides in the last
  // round): one L2 round trip per eight splits instead of one per split
  for (int k = 0; k < ns; k += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      v[u] = k + u < ns ? __ldg(po + (size_t)(k + u) * split_stride) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (k + u >= ns) break;
      const float w = s_w[k + u];
      acc.x = fmaf(w, v[u].x, acc.x);
      acc.y = fmaf(w, v[u].y, acc.y);
      acc.z = fmaf(w, v[u].z, acc.z);
      acc.w = fmaf(w, v[u].w, acc.w);
    }
  }
  store4<T>(out + (size_t)row * kDim + 4 * tid, acc);
  if (lse_out != nullptr && tid == 0) lse_out[row] = lse;
}

}  // namespace

cudaError_t launch_combine_strided(const float* part_lse, size_t lse_stride, const float* part_o,
                                   size_t o_stride, int ns, int batch, int heads, void* out, float* lse,
                                   int dtype, cudaStream_t stream) {
  if (ns < 1 || ns > kMaxSplits || o_stride % 4 != 0) return cudaErrorInvalidValue;
  const int rows = batch * heads;
  const size_t smem = sizeof(float) * (size_t)ns;
  if (dtype == MLA_DTYPE_F16) {
    mla_combine_kernel<__half><<<rows, kThreads, smem, stream>>>(
        part_lse, part_o, ns, rows, lse_stride, o_stride, static_cast<__half*>(out), lse);
  } else if (dtype == MLA_DTYPE_F32) {
    mla_combine_kernel<float><<<rows, kThreads, smem, stream>>>(
        part_lse, part_o, ns, rows, lse_stride, o_stride, static_cast<float*>(out), lse);
  } else {
    mla_combine_kernel<__nv_bfloat16><<<rows, kThreads, smem, stream>>>(
        part_lse, part_o, ns, rows, lse_stride, o_stride, static_cast<__nv_bfloat16*>(out), lse);
  }
  return cudaGetLastError();
}

cudaError_t launch_combine(const float* part_lse, const float* part_o, int ns, int batch,
                           int heads, void* out, float* lse, int dtype, cudaStream_t stream) {
  const size_t rows = (size_t)batch * heads;
  return launch_combine_strided(part_lse, rows, part_o, rows * kDim, ns, batch, heads, out, lse, dtype,
                                stream);
}

}  // namespace mla
