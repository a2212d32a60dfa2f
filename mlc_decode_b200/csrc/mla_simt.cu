// CUDA-core split-KV MLA decode kernel.
//
// The general-shape path: any head count, any seqlen_kv >= 1, fp16/bf16.  It
// computes the same per-split quantities as the reference main kernel
// (mla_decode.py:78-192): for one (split, 16-head group, batch) it walks its
// KV tiles with an online softmax (running max, exp2 with the log2e-folded
// scale, running sum, rescaled accumulator) and writes the split's normalised
// partial output and log-sum-exp.  When the plan has a single split it writes
// the final output directly and the combine kernel is skipped.
//
// Work decomposition: grid (ns, ceil(heads/16), batch), 256 threads.  Thread
// t owns head row t/16 of the group; for QK^T it computes two of the tile's
// 32 scores, for P.V it owns 32 latent columns {2*(t%16) + 32k + e}.
#include <math.h>
#include <stdio.h>

#include "mla_common.cuh"

namespace mla {
namespace {

constexpr int kHeadsPerCta = 16;
constexpr int kTileN = 32;              // KV rows per tile
constexpr int kThreads = 256;
constexpr int kQStride = kQkDim + 1;    // floats per Q row in smem (bank spread)
constexpr int kKStride = kQkDim + 2;    // elements per KV row in smem (odd word stride)
constexpr int kPStride = kTileN + 1;

constexpr size_t kSmemBytes = sizeof(float) * kHeadsPerCta * kQStride +
                              sizeof(uint16_t) * kTileN * kKStride +
                              sizeof(float) * kHeadsPerCta * kPStride;

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
mla_simt_splitkv_kernel(const T* __restrict__ q, const T* __restrict__ q_pe,
                        const T* __restrict__ kv, const T* __restrict__ k_pe,
                        void* __restrict__ out, float* __restrict__ lse_out,
                        float* __restrict__ part_o, float* __restrict__ part_lse,
                        int batch, int heads, int seqlen_kv, int ns, int bpc, int extra,
                        int block_n, float scale_log2, bool out_f32) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sQ = reinterpret_cast<float*>(smem_raw);
  uint16_t* sK = reinterpret_cast<uint16_t*>(sQ + kHeadsPerCta * kQStride);
  float* sP = reinterpret_cast<float*>(sK + kTileN * kKStride);

  const int z = blockIdx.x;
  const int h0 = blockIdx.y * kHeadsPerCta;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int nh = min(kHeadsPerCta, heads - h0);
  const int hr = tid >> 4;         // head row inside the group
  const int l16 = tid & 15;

  int t0, t1;
  split_range(z, bpc, extra, block_n, seqlen_kv, &t0, &t1);

  // Q (and Q_pe) of the head group, as float.
  for (int i = tid; i < kHeadsPerCta * kQkDim; i += kThreads) {
    const int r = i / kQkDim, c = i - r * kQkDim;
    float v = 0.f;
    if (r < nh) {
      const size_t row = (size_t)b * heads + h0 + r;
      v = c < kDim ? Elt<T>::to1(q[row * kDim + c]) : Elt<T>::to1(q_pe[row * kPeDim + (c - kDim)]);
    }
    sQ[r * kQStride + c] = v;
  }

  float m = -INFINITY;   // running max of raw scores
  float l = 0.f;         // running sum of exp2((s - m) * scale_log2)
  float o[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i] = 0.f;

  const uint32_t* kv32 = reinterpret_cast<const uint32_t*>(kv);
  const uint32_t* kpe32 = reinterpret_cast<const uint32_t*>(k_pe);

  for (int tt = t0; tt < t1; tt += kTileN) {
    const int nrow = min(kTileN, t1 - tt);
    __syncthreads();   // previous tile fully consumed (and Q staged on entry)
    for (int i = tid; i < kTileN * (kQkDim / 2); i += kThreads) {
      const int r = i / (kQkDim / 2), c2 = i - r * (kQkDim / 2);
      uint32_t w = 0;
      if (r < nrow) {
        const size_t tok = (size_t)b * seqlen_kv + tt + r;
        w = c2 < kDim / 2 ? __ldg(kv32 + tok * (kDim / 2) + c2)
                          : __ldg(kpe32 + tok * (kPeDim / 2) + (c2 - kDim / 2));
      }
      *reinterpret_cast<uint32_t*>(sK + r * kKStride + 2 * c2) = w;
    }
    __syncthreads();

    // scores of tokens l16 and l16 + 16 against head row hr
    float s0 = 0.f, s1 = 0.f;
    {
      const float* qr = sQ + hr * kQStride;
      const uint16_t* k0 = sK + l16 * kKStride;
      const uint16_t* k1 = sK + (l16 + 16) * kKStride;
#pragma unroll 8
      for (int c = 0; c < kQkDim; c += 2) {
        const float2 a = Elt<T>::to2(*reinterpret_cast<const uint32_t*>(k0 + c));
        const float2 bb = Elt<T>::to2(*reinterpret_cast<const uint32_t*>(k1 + c));
        const float qa = qr[c], qb = qr[c + 1];
        s0 = fmaf(qa, a.x, fmaf(qb, a.y, s0));
        s1 = fmaf(qa, bb.x, fmaf(qb, bb.y, s1));
      }
    }
    if (l16 >= nrow) s0 = -INFINITY;
    if (l16 + 16 >= nrow) s1 = -INFINITY;

    float mx = fmaxf(s0, s1);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m, mx);            // finite: row 0 of a tile is always valid
    const float alpha = exp2f((m - m_new) * scale_log2);
    const float p0 = exp2f((s0 - m_new) * scale_log2);
    const float p1 = exp2f((s1 - m_new) * scale_log2);
    float ps = p0 + p1;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    l = l * alpha + ps;
    m = m_new;
    sP[hr * kPStride + l16] = p0;
    sP[hr * kPStride + l16 + 16] = p1;
    __syncwarp();   // the 16 threads of a head row share one warp

#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] *= alpha;
    for (int j = 0; j < nrow; ++j) {
      const float p = sP[hr * kPStride + j];
      const uint16_t* vr = sK + j * kKStride + 2 * l16;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float2 v = Elt<T>::to2(*reinterpret_cast<const uint32_t*>(vr + 32 * k));
        o[2 * k] = fmaf(p, v.x, o[2 * k]);
        o[2 * k + 1] = fmaf(p, v.y, o[2 * k + 1]);
      }
    }
    __syncwarp();
  }

  if (hr >= nh) return;
  const size_t row = (size_t)b * heads + h0 + hr;
  const bool empty = !(t1 > t0);
  const float inv = empty ? 0.f : 1.f / l;
  const float lse_nat = empty ? -INFINITY : (m * scale_log2 + log2f(l)) * kLn2;
  if (ns == 1) {
    if (out_f32) {
      float2* orow = reinterpret_cast<float2*>(static_cast<float*>(out) + row * kDim);
#pragma unroll
      for (int k = 0; k < 16; ++k) orow[l16 + 16 * k] = make_float2(o[2 * k] * inv, o[2 * k + 1] * inv);
    } else {
      uint32_t* orow = reinterpret_cast<uint32_t*>(static_cast<T*>(out) + row * kDim);
#pragma unroll
      for (int k = 0; k < 16; ++k)
        orow[l16 + 16 * k] = Elt<T>::pack2(o[2 * k] * inv, o[2 * k + 1] * inv);
    }
    if (lse_out != nullptr && l16 == 0) lse_out[row] = lse_nat;
  } else {
    const size_t prow = (size_t)z * batch * heads + row;
    float2* orow = reinterpret_cast<float2*>(part_o + prow * kDim);
#pragma unroll
    for (int k = 0; k < 16; ++k) orow[l16 + 16 * k] = make_float2(o[2 * k] * inv, o[2 * k + 1] * inv);
    if (l16 == 0) part_lse[prow] = lse_nat;
  }
}

template <typename T>
cudaError_t launch_typed(const DecodeArgs& a) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 64 && !attr_done[dev]) {
    err = cudaFuncSetAttribute(mla_simt_splitkv_kernel<T>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (err != cudaSuccess) return err;
    attr_done[dev] = true;
  }
  const dim3 grid(a.plan.ns, (a.heads + kHeadsPerCta - 1) / kHeadsPerCta, a.batch);
  const float scale_log2 = a.softmax_scale * kLog2e;
  mla_simt_splitkv_kernel<T><<<grid, kThreads, kSmemBytes, a.stream>>>(
      static_cast<const T*>(a.q), static_cast<const T*>(a.q_pe), static_cast<const T*>(a.kv),
      static_cast<const T*>(a.k_pe), a.out, a.lse, a.part_o, a.part_lse,
      a.batch, a.heads, a.seqlen_kv, a.plan.ns, a.plan.bpc, a.plan.extra, a.plan.block_n,
      scale_log2, a.out_dtype == MLA_DTYPE_F32);
  return cudaGetLastError();
}

}  // namespace

int simt_block_n() { return kTileN; }
int simt_ctas_per_sm() { return 2; }

cudaError_t launch_simt_decode(const DecodeArgs& a) {
  if (a.plan.block_n % kTileN != 0) return cudaErrorInvalidValue;
  return a.dtype == MLA_DTYPE_F16 ? launch_typed<__half>(a) : launch_typed<__nv_bfloat16>(a);
}

}  // namespace mla
