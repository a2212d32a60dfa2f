// Shared definitions of the sm_100a MLA decode library: constants, element
// conversions, the KV split planner and the launcher prototypes that the C ABI
// (mla_capi.cu) dispatches to.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/mla_decode_b200.h"

namespace mla {

constexpr int kDim = 512;      // latent width (keys and values)
constexpr int kPeDim = 64;     // rope width (keys only)
constexpr int kQkDim = kDim + kPeDim;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// element conversions
// ---------------------------------------------------------------------------
template <typename T> struct Elt;
template <> struct Elt<__half> {
  static __device__ __forceinline__ float2 to2(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  static __device__ __forceinline__ float to1(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to2(uint32_t w) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w);
    return __bfloat1622float2(h);
  }
  static __device__ __forceinline__ float to1(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// ---------------------------------------------------------------------------
// split planner: _split_plan (mla_decode.py:9-30)
// ---------------------------------------------------------------------------
struct SplitPlan {
  int ns;            // number of splits actually used (partial slots)
  int bpc;           // KV tiles per split (tensor-core plan: CTA pairs)
  int extra;         // the first `extra` splits take one more tile (tensor-core plan: slots per pair)
  int block_n;       // KV rows per tile
  long long part_rows;   // partial rows in the workspace (0: derive from ns x batch x heads)
  bool needs_combine;    // a second (combine) launch is needed
};

inline SplitPlan split_plan(int seqlen_kv, int num_split, int block_n, bool spread) {
  SplitPlan p{};
  p.block_n = block_n;
  const int nb = (seqlen_kv + block_n - 1) / block_n;
  if (num_split < 1) num_split = 1;
  if (!spread) {
    const int chunk = (seqlen_kv + num_split - 1) / num_split;
    p.bpc = (chunk + block_n - 1) / block_n;
    if (p.bpc < 1) p.bpc = 1;
    p.ns = (nb + p.bpc - 1) / p.bpc;
    if (p.ns < 1) p.ns = 1;
    p.extra = 0;
  } else {
    p.ns = num_split < nb ? num_split : nb;
    if (p.ns < 1) p.ns = 1;
    p.bpc = nb / p.ns;
    p.extra = nb % p.ns;
  }
  p.part_rows = 0;
  p.needs_combine = p.ns > 1;
  return p;
}

// Token range [t0, t1) of split z under plan p (mla_decode.py:113-120; rows past
// seqlen_kv are masked in the reference, i.e. the range is clipped).
__host__ __device__ __forceinline__ void split_range(int z, int bpc, int extra, int block_n,
                                                     int seqlen_kv, int* t0, int* t1) {
  const int first = z * bpc + (z < extra ? z : extra);
  const int ntiles = bpc + (z < extra ? 1 : 0);
  long long a = (long long)first * block_n;
  long long e = a + (long long)ntiles * block_n;
  if (a > seqlen_kv) a = seqlen_kv;
  if (e > seqlen_kv) e = seqlen_kv;
  *t0 = (int)a;
  *t1 = (int)e;
}

// ---------------------------------------------------------------------------
// host-side error text (thread local, read through mla_last_error)
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

// Checks a decode call's shape, dtype, tensor pointers (non-null, 16-byte
// aligned) and config exactly as mla_decode_fwd does before it launches
// anything; MLA_OK or the status mla_decode_fwd would return (error text set).
int check_decode_call(const char* fn, const void* q, const void* q_pe, const void* kv, const void* k_pe,
                      const void* out, int batch, int heads, int seqlen_kv, int dtype, const MlaCfg* cfg);

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
struct DecodeArgs {
  const void* q;
  const void* q_pe;
  const void* kv;
  const void* k_pe;
  void* out;          // final output (used when ns == 1)
  int out_dtype;      // MlaDtype of `out`: dtype, or MLA_DTYPE_F32 (mla_decode_partial)
  float* lse;         // optional final lse (natural log)
  float* part_o;      // [ns, batch, heads, 512]
  float* part_lse;    // [ns, batch, heads]
  uint32_t* status;   // workspace status word (tensor-core kernel), nullable
  uint32_t* counters; // per-(sequence, CTA rank) piece counters (tensor-core kernel)
  // ragged calls (mla_decode_paged): per-sequence lengths, optional page table
  const int* seqlens;      // [batch] or nullptr
  const int* block_table;  // [batch][max_pages] or nullptr (contiguous [batch, seqlen_kv] rows)
  int page_size, num_pages, max_pages;
  uint32_t* cu_tiles;      // workspace: flattened-tile prefix sums (batch x head groups + 1)
  int batch, heads, seqlen_kv, dtype;
  // query positions per sequence (causal within the step) and KV heads (query
  // heads [i*h/kv_heads, (i+1)*h/kv_heads) read KV head i); 0 means 1.
  // Tensor-core kernel only.
  int q_len, kv_heads;
  // kv holds e4m3 latent rows (one byte per dim) to be multiplied by kv_scale
  // (tensor-core kernel only); k_pe stays in `dtype`
  int kv_fp8;
  float kv_scale;
  float softmax_scale;  // multiplies raw scores
  SplitPlan plan;
  cudaStream_t stream;
};

// Query side of a call as the tensor-core kernel sees it: qb = batch x q_len x
// kv_heads query sequences of g = heads / kv_heads rows, hg groups of up to 128
// rows each, vb = qb x hg virtual sequences.
struct QShape {
  int q_len, kv_heads, qb, g, hg, vb;
};

// ---------------------------------------------------------------------------
// The sequence split's gather buffer (one per rank, the same layout everywhere;
// mla_seqsplit_buffer_bytes):
//   float blocks [2][world][chunk]: rank q's float32 (O, LSE) block for calls of
//     parity p at (p * world + q) * chunk; chunk = b*h*512 O floats, then the b*h
//     LSEs, padded to a multiple of 64 floats;
//   a 256-byte header at round_up(2 * world * chunk * 4, 256): uint32 block flags
//     [2][8] at byte 0, the push counter at byte 64, the status word at byte 68
//     (0, or kErrExchange once a wait for a peer gave up);
//   row words uint2 [2][world][rows_pad][512] after the header, then LSE words
//     uint2 [2][world][rows_pad] (rows_pad = round_up(b*h, 64)): rank q's rows of
//     parity p as (value bits, call number) pairs, each pair written by one 8-byte
//     part of a 16-byte store, so a reader that sees this call's number in a pair
//     has that pair's value (no fence or separate flag between writer and reader).
// ---------------------------------------------------------------------------
constexpr int kSeqMaxWorld = 8;
constexpr uint32_t kErrExchange = 0x201;
constexpr unsigned long long kSeqWaitNs = 2000000000ull;   // 2 s
__host__ __device__ inline size_t seq_rows_pad(int batch, int heads) {
  return ((size_t)batch * heads + 63) / 64 * 64;
}
__host__ __device__ inline size_t seq_chunk_floats(int batch, int heads) {
  return (size_t)batch * heads * kDim + seq_rows_pad(batch, heads);
}
__host__ __device__ inline size_t seq_header_offset(int world, int batch, int heads) {
  return (2 * (size_t)world * seq_chunk_floats(batch, heads) * 4 + 255) / 256 * 256;
}
__host__ __device__ inline size_t seq_ll_rows_offset(int world, int batch, int heads) {
  return seq_header_offset(world, batch, heads) + 256;
}
__host__ __device__ inline size_t seq_ll_lse_offset(int world, int batch, int heads) {
  return seq_ll_rows_offset(world, batch, heads) + 2 * (size_t)world * seq_rows_pad(batch, heads) * kDim * 8;
}
inline size_t seq_buffer_bytes(int world, int batch, int heads) {
  return seq_ll_lse_offset(world, batch, heads) + 2 * (size_t)world * seq_rows_pad(batch, heads) * 8;
}

// Every rank's gather buffer as mapped in this process, and this call's place.
struct PeerRows {
  float* bufs[kSeqMaxWorld];
  size_t chunk;     // floats per block
  size_t header;    // byte offset of the header in a buffer
  size_t ll_rows;   // byte offset of the row words
  size_t ll_lse;    // byte offset of the LSE words
  size_t rows_pad;
  int world, rank, par;
  uint32_t epoch;   // call number, from 1
};

// The sequence split's merge and exchange (mla_sm100.cu): `pieces` merges this
// rank's rows from the tensor-core kernel's pieces in the workspace where it left
// them (plan variant 1), else takes the rows this rank's block holds; the world
// ranks' rows are then exchanged and merged into out (dtype) / lse.
cudaError_t launch_seqsplit_combine(const DecodeArgs& a, bool pieces, const PeerRows& x, void* out, float* lse,
                                    int dtype);

// CUDA-core split-KV kernel (mla_simt.cu).  Returns a cudaError_t.
cudaError_t launch_simt_decode(const DecodeArgs& a);
int simt_block_n();                       // KV rows per tile of the SIMT kernel
int simt_ctas_per_sm();                   // resident CTAs per SM (occupancy target)

// LSE combine (mla_combine.cu): split-major partials, or split k's LSE rows at
// part_lse + k * lse_stride and O rows at part_o + k * o_stride (floats).
cudaError_t launch_combine(const float* part_lse, const float* part_o, int ns, int batch,
                           int heads, void* out, float* lse, int dtype, cudaStream_t stream);
cudaError_t launch_combine_strided(const float* part_lse, size_t lse_stride, const float* part_o,
                                   size_t o_stride, int ns, int batch, int heads, void* out, float* lse,
                                   int dtype, cudaStream_t stream);

}  // namespace mla
