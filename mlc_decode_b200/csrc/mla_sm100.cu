// tcgen05 / TMA / TMEM split-KV MLA decode kernel for sm_100a (B200).
//
// Computes the same per-range quantities as the reference's split-KV main
// kernel (mla_decode.py:78-192): for a run of 128-row KV tiles of one sequence,
// S = [q|q_pe].[kv|k_pe]^T on the tensor cores, an online softmax with the
// log2e-folded scale, and O = P.kv on the tensor cores, then O/l and the
// log-sum-exp.  The B200 design:
//
//  * A CTA pair (cluster of 2) owns all 128 heads of one sequence; CTA r holds
//    heads [64r, 64r+64).  Both GEMMs are pair-wide UMMAs (tcgen05.mma
//    .cta_group::2, M = 128): A (Q or P) is split by rows between the CTAs,
//    B (K or V) by columns, so each 128-row KV tile is loaded once for QK^T.
//  * TMEM (per CTA, 2x2 data-path layout of the pair MMA: lanes 0-63 hold
//    columns [0, N/2), lanes 64-127 columns [N/2, N) of the CTA's 64 rows):
//    S double buffer in columns [0, 64) and [64, 128); O (64 x 512 fp32) in
//    columns [128, 384).
//  * Two TMA producer threads per CTA feed two mbarrier rings of 16 KB stages
//    (SWIZZLE_128B boxes of 64 rows x 128 B): the K ring (per tile four latent
//    units of 128 columns and one rope unit, each CTA its own 64 rows) and the
//    V ring (per tile four units; for P.V each CTA supplies 128 latent columns
//    of all 128 rows, bytes that come a second time, from L2, because the two
//    GEMMs need the tile in different per-CTA arrangements).
//  * Two MMA issuer threads in the even CTA: one issues QK^T into the S double
//    buffer as soon as K data and a free S buffer exist; the other issues P.V
//    as soon as P and V exist.  Neither blocks the other.
//  * Four softmax warps per CTA (one TMEM lane quarter each) read S with
//    tcgen05.ld, exchange the row max between the two lane halves of a row,
//    and write P to shared memory once the previous P.V has completed (one P
//    buffer).  For bf16 inputs P is written as a bf16 hi/lo pair and P.V runs
//    twice (P_hi.V + P_lo.V): bf16 P alone costs ~1.5e-3 relative L2 error in
//    the output, the hi/lo pair keeps it near fp32 accuracy.  O is rescaled
//    only when a row max grows by more than 2^8 (exact: the final
//    normalisation uses the same stale max), so the accumulator stays in TMEM.
//  * Work: pair p takes the flattened tile range [p*T/P, (p+1)*T/P) over all
//    sequences (T = batch x tiles per sequence).  A range that covers a whole
//    sequence writes `out` directly; partial ranges write float32 partials to
//    slot p*maxp + k, merged by mla_pair_combine_kernel.
//  * Every wait is bounded (about 2 s of %globaltimer); on timeout the CTA
//    pair raises an abort flag, records a status code in the workspace and
//    winds down (no trap, no hang).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>
#include <type_traits>

#include "mla_sm100.cuh"
#include "mla_sm100_ptx.cuh"

namespace mla {
namespace sm100 {

constexpr int kHeads = 128;           // heads per CTA pair
constexpr int kTile = 128;            // KV rows per tile
constexpr uint32_t kStageBytes = 16384;
constexpr uint32_t kChunkBytes = 8192;       // one 64 x 128 B swizzled box
constexpr uint32_t kQBytes = 9 * kChunkBytes;
constexpr uint32_t kPBytes = 2 * kChunkBytes;   // one P operand: 64 rows x 128 tokens
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 128;
constexpr int kThreads = 256;
constexpr float kRescaleLog2 = 8.0f;
constexpr uint64_t kTimeoutNs = 2000000000ull;

// status codes written to the workspace status word on a timeout
constexpr uint32_t kErrKLoad = 0x101, kErrVLoad = 0x102, kErrQK = 0x103, kErrPV = 0x104,
                   kErrSoftmax = 0x105, kErrDrain = 0x106;

// Compile-time configuration per input type.  bf16 needs the hi/lo P pair
// (two P operands); fp16 P is exact enough and gives the space to the rings.
template <typename T>
struct Cfg;
template <>
struct Cfg<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  static constexpr int kPParts = 2;
  static constexpr int kKStages = 4;
  static constexpr int kVStages = 3;
};
template <>
struct Cfg<__half> {
  static constexpr uint32_t kFmt = 0;
  static constexpr int kPParts = 1;
  static constexpr int kKStages = 5;
  static constexpr int kVStages = 3;
};

struct Barriers {
  uint64_t kfull[8], kempty[8];
  uint64_t vfull[8], vempty[8];
  uint64_t q_full, q_empty;
  uint64_t s_full[2], s_free[2];
  uint64_t p_full;
  uint64_t xchg[2];
  uint64_t o_done, o_free, lx;
  uint64_t drain_qk, drain_pv;
};
static_assert(sizeof(Barriers) <= 512, "barrier block");

// shared memory map (offsets from the 1024-byte aligned base)
template <typename T>
struct Smem {
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kP = kQ + kQBytes;
  static constexpr uint32_t kKRing = kP + Cfg<T>::kPParts * kPBytes;
  static constexpr uint32_t kVRing = kKRing + Cfg<T>::kKStages * kStageBytes;
  static constexpr uint32_t kBar = kVRing + Cfg<T>::kVStages * kStageBytes;
  static constexpr uint32_t kXmax = kBar + 512;
  static constexpr uint32_t kXl = kXmax + 2 * 128 * 4;
  static constexpr uint32_t kMisc = kXl + 128 * 4;
  static constexpr uint32_t kBytes = kMisc + 64 + 1024;   // + alignment slack
  static_assert(kBytes <= 232448, "shared memory");
};

struct Params {
  CUtensorMap tm_kv;    // [b*s, 512], box 64 x 64
  CUtensorMap tm_kpe;   // [b*s, 64]
  CUtensorMap tm_q;     // [b*128, 512]
  CUtensorMap tm_qpe;   // [b*128, 64]
  void* out;
  float* lse_out;
  float* part_o;
  float* part_lse;
  uint32_t* status;
  long long total_tiles;
  int batch, seqlen, nt, pairs, maxp;
  float sl2;            // softmax scale * log2(e)
};

struct Ctx {
  uint32_t* abort_local;
  uint32_t abort_peer;   // shared::cluster address of the peer's abort flag
  uint32_t* status;
};

__device__ __forceinline__ void raise_abort(const Ctx& c, uint32_t code) {
  *reinterpret_cast<volatile uint32_t*>(c.abort_local) = 1u;
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(c.abort_peer), "r"(1u) : "memory");
  if (c.status != nullptr) atomicCAS(c.status, 0u, code);
}

// Bounded wait for the phase of `parity` on a local barrier.
__device__ __noinline__ bool wait_bar(const Ctx& c, uint32_t bar, uint32_t parity, uint32_t code) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile uint32_t*>(c.abort_local) != 0u) return false;
    if (ptx::globaltimer() - t0 > kTimeoutNs) {
      raise_abort(c, code);
      return false;
    }
  }
}

__device__ __forceinline__ bool aborted(const Ctx& c) {
  return *reinterpret_cast<volatile uint32_t*>(c.abort_local) != 0u;
}

// One contiguous run of tiles of one sequence inside a pair's range.
struct Piece {
  int bb;        // sequence
  int first;     // first tile (within the sequence)
  int end;       // one past the last tile
  bool full;     // the run is the whole sequence
};

// Iterates the pieces of pair `pair`'s tile range [pair*T/P, (pair+1)*T/P).
struct PieceIter {
  long long t, t1;
  int nt;
  __device__ PieceIter(const Params& p, int pair) : nt(p.nt) {
    t = (long long)pair * p.total_tiles / p.pairs;
    t1 = (long long)(pair + 1) * p.total_tiles / p.pairs;
  }
  __device__ bool next(Piece* pc) {
    if (t >= t1) return false;
    pc->bb = (int)(t / nt);
    const long long bstart = (long long)pc->bb * nt;
    const long long e = t1 < bstart + nt ? t1 : bstart + nt;
    pc->first = (int)(t - bstart);
    pc->end = (int)(e - bstart);
    pc->full = pc->first == 0 && pc->end == nt;
    t = e;
    return true;
  }
};

// Position in a ring of `kStages` shared-memory stages.
template <int kStages>
struct Ring {
  uint32_t stage = 0, phase = 0;
  __device__ __forceinline__ void advance() {
    if (++stage == kStages) {
      stage = 0;
      phase ^= 1u;
    }
  }
};

// ---------------------------------------------------------------------------
// K producer: Q once per piece, then per tile 4 latent units + 1 rope unit.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void k_producer(const Params& p, const Ctx& c, uint32_t rank, int pair,
                                           uint32_t sbase, Barriers* bars) {
  using S = Smem<T>;
  constexpr int KS = Cfg<T>::kKStages;
  const bool leader = rank == 0;
  const uint32_t kfull0 = ptx::smem_u32(&bars->kfull[0]);
  const uint32_t kfull0_leader = ptx::mapa(kfull0, 0);
  const uint32_t kempty0 = ptx::smem_u32(&bars->kempty[0]);
  const uint32_t q_full = ptx::smem_u32(&bars->q_full);
  const uint32_t q_full_leader = ptx::mapa(q_full, 0);
  const uint32_t q_empty = ptx::smem_u32(&bars->q_empty);
  Ring<KS> ring;
  PieceIter it(p, pair);
  Piece pc;
  int piece = 0;
  while (it.next(&pc)) {
    if (piece > 0 && !wait_bar(c, q_empty, (uint32_t)(piece - 1) & 1u, kErrKLoad)) return;
    if (leader) ptx::mbar_arrive_expect_tx(q_full, 2 * kQBytes);
    const int qrow = pc.bb * kHeads + 64 * (int)rank;
#pragma unroll 1
    for (int ch = 0; ch < 8; ++ch)
      ptx::tma_load_2d_pair(sbase + S::kQ + ch * kChunkBytes, &p.tm_q, q_full_leader, 64 * ch, qrow);
    ptx::tma_load_2d_pair(sbase + S::kQ + 8 * kChunkBytes, &p.tm_qpe, q_full_leader, 0, qrow);
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j) {
      const int y = pc.bb * p.seqlen + j * kTile + 64 * (int)rank;
#pragma unroll 1
      for (int u = 0; u < 5; ++u) {
        if (!wait_bar(c, kempty0 + 8 * ring.stage, ring.phase ^ 1u, kErrKLoad)) return;
        if (leader)
          ptx::mbar_arrive_expect_tx(kfull0 + 8 * ring.stage, u < 4 ? 2 * kStageBytes : 2 * kChunkBytes);
        const uint32_t dst = sbase + S::kKRing + ring.stage * kStageBytes;
        const uint32_t bar = kfull0_leader + 8 * ring.stage;
        if (u < 4) {
          ptx::tma_load_2d_pair(dst, &p.tm_kv, bar, 128 * u, y);
          ptx::tma_load_2d_pair(dst + kChunkBytes, &p.tm_kv, bar, 128 * u + 64, y);
        } else {
          ptx::tma_load_2d_pair(dst, &p.tm_kpe, bar, 0, y);
        }
        ring.advance();
      }
    }
    ++piece;
  }
}

// ---------------------------------------------------------------------------
// V producer: per tile 4 units u = (N half nh, token half th): this CTA's 128
// latent columns [256 nh + 128 rank, +128) of the tile's tokens [64 th, +64).
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void v_producer(const Params& p, const Ctx& c, uint32_t rank, int pair,
                                           uint32_t sbase, Barriers* bars) {
  using S = Smem<T>;
  constexpr int VS = Cfg<T>::kVStages;
  const bool leader = rank == 0;
  const uint32_t vfull0 = ptx::smem_u32(&bars->vfull[0]);
  const uint32_t vfull0_leader = ptx::mapa(vfull0, 0);
  const uint32_t vempty0 = ptx::smem_u32(&bars->vempty[0]);
  Ring<VS> ring;
  PieceIter it(p, pair);
  Piece pc;
  while (it.next(&pc)) {
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j) {
      const int y0 = pc.bb * p.seqlen + j * kTile;
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        const int nh = u >> 1, th = u & 1;
        if (!wait_bar(c, vempty0 + 8 * ring.stage, ring.phase ^ 1u, kErrVLoad)) return;
        if (leader) ptx::mbar_arrive_expect_tx(vfull0 + 8 * ring.stage, 2 * kStageBytes);
        const uint32_t dst = sbase + S::kVRing + ring.stage * kStageBytes;
        const uint32_t bar = vfull0_leader + 8 * ring.stage;
        const int x = 256 * nh + 128 * (int)rank;
        ptx::tma_load_2d_pair(dst, &p.tm_kv, bar, x, y0 + 64 * th);
        ptx::tma_load_2d_pair(dst + kChunkBytes, &p.tm_kv, bar, x + 64, y0 + 64 * th);
        ring.advance();
      }
    }
  }
}

// ---------------------------------------------------------------------------
// QK^T issuer (one thread of the even CTA): S[gi % 2] = Q . K_tile^T
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void qk_issuer(const Params& p, const Ctx& c, int pair, uint32_t sbase,
                                          uint32_t tmem, Barriers* bars) {
  using S = Smem<T>;
  constexpr int KS = Cfg<T>::kKStages;
  constexpr uint32_t kIdesc = ptx::idesc_f16(Cfg<T>::kFmt, 128, 128, 0);
  const uint32_t kfull0 = ptx::smem_u32(&bars->kfull[0]);
  const uint32_t kempty0 = ptx::smem_u32(&bars->kempty[0]);
  const uint32_t q_full = ptx::smem_u32(&bars->q_full);
  const uint32_t q_empty = ptx::smem_u32(&bars->q_empty);
  const uint32_t s_full0 = ptx::smem_u32(&bars->s_full[0]);
  const uint32_t s_free0 = ptx::smem_u32(&bars->s_free[0]);
  const uint32_t qbase = sbase + S::kQ;
  Ring<KS> ring;
  uint32_t gi = 0;
  PieceIter it(p, pair);
  Piece pc;
  int piece = 0;
  while (it.next(&pc)) {
    if (!wait_bar(c, q_full, (uint32_t)piece & 1u, kErrQK)) return;
    ptx::tc_fence_after();
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j, ++gi) {
      const uint32_t b = gi & 1u;
      // the softmax warps must have read S[b] of tile gi - 2
      if (gi >= 2 && !wait_bar(c, s_free0 + 8 * b, ((gi - 2) >> 1) & 1u, kErrQK)) return;
      ptx::tc_fence_after();
      const uint32_t s_tmem = tmem + 64 * b;
#pragma unroll 1
      for (int u = 0; u < 5; ++u) {
        if (!wait_bar(c, kfull0 + 8 * ring.stage, ring.phase, kErrQK)) return;
        ptx::tc_fence_after();
        const uint32_t kb = sbase + S::kKRing + ring.stage * kStageBytes;
        const int nk = u < 4 ? 8 : 4;
#pragma unroll 1
        for (int kk = 0; kk < nk; ++kk) {
          const int qc = u < 4 ? 2 * u + (kk >> 2) : 8;
          const uint64_t a = ptx::sw128_desc(qbase + qc * kChunkBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = ptx::sw128_desc(kb + (kk >> 2) * kChunkBytes + (kk & 3) * 32, 16, 1024);
          ptx::mma_pair_f16(s_tmem, a, bd, kIdesc, (u == 0 && kk == 0) ? 0u : 1u);
        }
        ptx::mma_commit_pair_mc(kempty0 + 8 * ring.stage, 0x3);
        ring.advance();
      }
      ptx::mma_commit_pair_mc(s_full0 + 8 * b, 0x3);
      if (j == pc.end - 1) ptx::mma_commit_pair_mc(q_empty, 0x3);
    }
    ++piece;
  }
}

// ---------------------------------------------------------------------------
// P.V issuer (one thread of the even CTA): O += P . V_tile (P_hi and P_lo for bf16)
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void pv_issuer(const Params& p, const Ctx& c, int pair, uint32_t sbase,
                                          uint32_t tmem, Barriers* bars) {
  using S = Smem<T>;
  constexpr int VS = Cfg<T>::kVStages;
  constexpr uint32_t kIdesc = ptx::idesc_f16(Cfg<T>::kFmt, 128, 256, 1);
  const uint32_t vfull0 = ptx::smem_u32(&bars->vfull[0]);
  const uint32_t vempty0 = ptx::smem_u32(&bars->vempty[0]);
  const uint32_t p_full = ptx::smem_u32(&bars->p_full);
  const uint32_t o_done = ptx::smem_u32(&bars->o_done);
  const uint32_t o_free = ptx::smem_u32(&bars->o_free);
  Ring<VS> ring;
  uint32_t gi = 0;
  PieceIter it(p, pair);
  Piece pc;
  int piece = 0;
  while (it.next(&pc)) {
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j, ++gi) {
      const bool first = j == pc.first;
      if (!wait_bar(c, p_full, gi & 1u, kErrPV)) return;
      // a new piece restarts O: the previous piece's epilogue must have read it
      if (first && piece > 0 && !wait_bar(c, o_free, (uint32_t)(piece - 1) & 1u, kErrPV)) return;
      ptx::tc_fence_after();
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        const int nh = u >> 1, th = u & 1;
        if (!wait_bar(c, vfull0 + 8 * ring.stage, ring.phase, kErrPV)) return;
        ptx::tc_fence_after();
        const uint32_t vb = sbase + S::kVRing + ring.stage * kStageBytes;
#pragma unroll
        for (int part = 0; part < Cfg<T>::kPParts; ++part) {
          const uint32_t pb = sbase + S::kP + part * kPBytes + th * kChunkBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a = ptx::sw128_desc(pb + kk * 32, 16, 1024);
            const uint64_t bd = ptx::sw128_desc(vb + kk * 2048, kChunkBytes, 1024);
            ptx::mma_pair_f16(tmem + kColO + 128 * nh, a, bd, kIdesc,
                              (first && th == 0 && kk == 0 && part == 0) ? 0u : 1u);
          }
        }
        ptx::mma_commit_pair_mc(vempty0 + 8 * ring.stage, 0x3);
        ring.advance();
      }
      ptx::mma_commit_pair_mc(o_done, 0x3);
    }
    ++piece;
  }
}

// ---------------------------------------------------------------------------
// softmax + epilogue: warps 4..7 of each CTA; thread <-> TMEM lane L
// (row m = L % 64 of this CTA's heads, tokens [64*(L/64), +64) of each tile)
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return Elt<T>::pack2(a, b);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void softmax_epilogue(const Params& p, const Ctx& c, uint32_t rank, int pair,
                                                 uint8_t* smem, uint32_t tmem, Barriers* bars, int wq,
                                                 int lane) {
  using S = Smem<T>;
  const int L = wq * 32 + lane;
  const int m = L & 63;
  const int hf = L >> 6;
  const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
  float* xmax = reinterpret_cast<float*>(smem + S::kXmax);
  float* xl = reinterpret_cast<float*>(smem + S::kXl);
  const uint32_t s_full0 = ptx::smem_u32(&bars->s_full[0]);
  const uint32_t xchg0 = ptx::smem_u32(&bars->xchg[0]);
  const uint32_t o_done = ptx::smem_u32(&bars->o_done);
  const uint32_t lx = ptx::smem_u32(&bars->lx);
  const uint32_t s_free0_leader = ptx::mapa(ptx::smem_u32(&bars->s_free[0]), 0);
  const uint32_t p_full_leader = ptx::mapa(ptx::smem_u32(&bars->p_full), 0);
  const uint32_t o_free_leader = ptx::mapa(ptx::smem_u32(&bars->o_free), 0);
  const float sl2 = p.sl2;
  uint32_t gi = 0;

  PieceIter it(p, pair);
  Piece pc;
  int piece = 0;
  while (it.next(&pc)) {
    float m_run = -INFINITY, l = 0.f;
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j, ++gi) {
      const uint32_t b = gi & 1u;
      if (!wait_bar(c, s_full0 + 8 * b, (gi >> 1) & 1u, kErrSoftmax)) return;
      ptx::tc_fence_after();
      uint32_t r0[32], r1[32];
      ptx::tmem_ld32(tmem + lane_off + 64 * b, r0);
      ptx::tmem_ld32(tmem + lane_off + 64 * b + 32, r1);
      ptx::tmem_wait_ld();
      // S[b] is in registers: hand the buffer back to the QK^T issuer
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(s_free0_leader + 8 * b);
      float v[64];
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        v[k] = __uint_as_float(r0[k]);
        v[32 + k] = __uint_as_float(r1[k]);
      }
      const int nvalid = p.seqlen - (j * kTile + 64 * hf);
      if (nvalid < 64) {
#pragma unroll
        for (int k = 0; k < 64; ++k)
          if (k >= nvalid) v[k] = -INFINITY;
      }
      float mx = v[0];
#pragma unroll
      for (int k = 1; k < 64; ++k) mx = fmaxf(mx, v[k]);
      // the two lane halves of a row hold its two 64-token halves: exchange maxima
      xmax[b * 128 + L] = mx;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa(xchg0 + 8 * b, rank));
      if (!wait_bar(c, xchg0 + 8 * b, (gi >> 1) & 1u, kErrSoftmax)) return;
      mx = fmaxf(mx, xmax[b * 128 + (L ^ 64)]);
      const float m_new = fmaxf(m_run, mx);
      const bool rescale = (m_new - m_run) * sl2 > kRescaleLog2;
      float alpha = 1.f;
      if (rescale) {
        alpha = exp2f((m_run - m_new) * sl2);
        l *= alpha;
        m_run = m_new;
      }
      const float ms = m_run * sl2;
      uint32_t phi[32], plo[32];
      float ls = 0.f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float a = ex2(fmaf(v[2 * k], sl2, -ms));
        const float b2 = ex2(fmaf(v[2 * k + 1], sl2, -ms));
        ls += a + b2;
        phi[k] = pack2<T>(a, b2);
        if constexpr (Cfg<T>::kPParts == 2) {
          const float ah = __uint_as_float(phi[k] << 16);
          const float bh = __uint_as_float(phi[k] & 0xffff0000u);
          plo[k] = pack2<T>(a - ah, b2 - bh);
        }
      }
      l += ls;
      if (j > pc.first) {
        // P.V of the previous tile must be complete before O is touched or P rewritten
        if (!wait_bar(c, o_done, (gi - 1) & 1u, kErrSoftmax)) return;
        ptx::tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int cc = 0; cc < 8; ++cc) {
            uint32_t o[32];
            ptx::tmem_ld32(tmem + lane_off + kColO + 32 * cc, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
            ptx::tmem_st32(tmem + lane_off + kColO + 32 * cc, o);
          }
          ptx::tmem_wait_st();
        }
      }
      // P row m of token half hf, SWIZZLE_128B: 16-byte granule g at g ^ (m & 7)
      uint8_t* prow = smem + S::kP + hf * kChunkBytes + m * 128;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const uint32_t off = (uint32_t)((g ^ (m & 7)) << 4);
        *reinterpret_cast<uint4*>(prow + off) =
            make_uint4(phi[4 * g], phi[4 * g + 1], phi[4 * g + 2], phi[4 * g + 3]);
        if constexpr (Cfg<T>::kPParts == 2)
          *reinterpret_cast<uint4*>(prow + kPBytes + off) =
              make_uint4(plo[4 * g], plo[4 * g + 1], plo[4 * g + 2], plo[4 * g + 3]);
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(p_full_leader);
    }

    // ---- epilogue of this piece
    if (!wait_bar(c, o_done, (gi - 1) & 1u, kErrSoftmax)) return;
    ptx::tc_fence_after();
    xl[L] = l;
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa(lx, rank));
    if (!wait_bar(c, lx, (uint32_t)piece & 1u, kErrSoftmax)) return;
    const float ltot = l + xl[L ^ 64];
    const float inv = 1.f / ltot;
    const float lse = (m_run * sl2 + log2f(ltot)) * kLn2;
    const int head = 64 * (int)rank + m;
    const int slot = pair * p.maxp + piece;
#pragma unroll 1
    for (int nh = 0; nh < 2; ++nh) {
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t o[32];
        ptx::tmem_ld32(tmem + lane_off + kColO + 128 * nh + 32 * cc, o);
        ptx::tmem_wait_ld();
        const int d0 = 256 * nh + 128 * hf + 32 * cc;
        if (pc.full) {
          T* dst = static_cast<T*>(p.out) + ((size_t)pc.bb * kHeads + head) * kDim + d0;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 w;
            w.x = pack2<T>(__uint_as_float(o[8 * g + 0]) * inv, __uint_as_float(o[8 * g + 1]) * inv);
            w.y = pack2<T>(__uint_as_float(o[8 * g + 2]) * inv, __uint_as_float(o[8 * g + 3]) * inv);
            w.z = pack2<T>(__uint_as_float(o[8 * g + 4]) * inv, __uint_as_float(o[8 * g + 5]) * inv);
            w.w = pack2<T>(__uint_as_float(o[8 * g + 6]) * inv, __uint_as_float(o[8 * g + 7]) * inv);
            reinterpret_cast<uint4*>(dst)[g] = w;
          }
        } else {
          float* dst = p.part_o + ((size_t)slot * kHeads + head) * kDim + d0;
#pragma unroll
          for (int g = 0; g < 8; ++g)
            reinterpret_cast<float4*>(dst)[g] =
                make_float4(__uint_as_float(o[4 * g]) * inv, __uint_as_float(o[4 * g + 1]) * inv,
                            __uint_as_float(o[4 * g + 2]) * inv, __uint_as_float(o[4 * g + 3]) * inv);
        }
      }
    }
    if (hf == 0) {
      if (pc.full) {
        if (p.lse_out != nullptr) p.lse_out[(size_t)pc.bb * kHeads + head] = lse;
      } else {
        p.part_lse[(size_t)slot * kHeads + head] = lse;
      }
    }
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive_cluster(o_free_leader);
    ++piece;
  }
}

// ---------------------------------------------------------------------------
// the kernel: warp 0 K producer, warp 1 TMEM owner + QK^T issuer, warp 2 V
// producer, warp 3 P.V issuer, warps 4..7 softmax/epilogue
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
mla_sm100_decode_kernel(const __grid_constant__ Params p) {
  using S = Smem<T>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  Barriers* bars = reinterpret_cast<Barriers*>(smem + S::kBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kMisc);
  uint32_t* abort_flag = reinterpret_cast<uint32_t*>(smem + S::kMisc + 4);
  const uint32_t rank = ptx::cluster_ctarank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 8; ++s) {
      ptx::mbar_init(ptx::smem_u32(&bars->kfull[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->kempty[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->vfull[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->vempty[s]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(&bars->q_full), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->q_empty), 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(ptx::smem_u32(&bars->s_full[b]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->s_free[b]), 8);
      ptx::mbar_init(ptx::smem_u32(&bars->xchg[b]), 4);
    }
    ptx::mbar_init(ptx::smem_u32(&bars->p_full), 8);
    ptx::mbar_init(ptx::smem_u32(&bars->o_done), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->o_free), 8);
    ptx::mbar_init(ptx::smem_u32(&bars->lx), 4);
    ptx::mbar_init(ptx::smem_u32(&bars->drain_qk), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->drain_pv), 1);
    *abort_flag = 0u;
    ptx::fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&p.tm_kv);
    ptx::prefetch_tensormap(&p.tm_kpe);
    ptx::prefetch_tensormap(&p.tm_q);
    ptx::prefetch_tensormap(&p.tm_qpe);
  }
  if (warp == 1) ptx::tmem_alloc_pair(ptx::smem_u32(tmem_slot), kTmemCols);
  ptx::tc_fence_before();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  Ctx c;
  c.abort_local = abort_flag;
  c.abort_peer = ptx::mapa(ptx::smem_u32(abort_flag), rank ^ 1u);
  c.status = p.status;

  if (warp == 0) {
    if (lane == 0) k_producer<T>(p, c, rank, pair, sbase, bars);
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      qk_issuer<T>(p, c, pair, sbase, tmem, bars);
      // every tcgen05 op this thread issued has completed once this commit lands
      ptx::mma_commit_pair_mc(ptx::smem_u32(&bars->drain_qk), 0x1);
      wait_bar(c, ptx::smem_u32(&bars->drain_qk), 0u, kErrDrain);
    }
  } else if (warp == 2) {
    if (lane == 0) v_producer<T>(p, c, rank, pair, sbase, bars);
  } else if (warp == 3) {
    if (rank == 0 && lane == 0) {
      pv_issuer<T>(p, c, pair, sbase, tmem, bars);
      ptx::mma_commit_pair_mc(ptx::smem_u32(&bars->drain_pv), 0x1);
      wait_bar(c, ptx::smem_u32(&bars->drain_pv), 0u, kErrDrain);
    }
  } else {
    softmax_epilogue<T>(p, c, rank, pair, smem, tmem, bars, warp & 3, lane);
  }
  __syncwarp();
  if (aborted(c)) {
    // let copies already in flight land before the CTA's shared memory goes away
    const uint64_t t0 = ptx::globaltimer();
    while (ptx::globaltimer() - t0 < 2000000ull) __nanosleep(1000);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, kTmemCols);
    ptx::tmem_relinquish_pair();
  }
}

// ---------------------------------------------------------------------------
// combine for the pair schedule: one 128-thread CTA per (head, sequence);
// sequences that one pair covered whole were written directly and are skipped.
// Same LSE algebra as mla_combine.cu (mla_decode.py:212-246).
// ---------------------------------------------------------------------------
constexpr int kMaxPairs = 256;

template <typename T>
__global__ void __launch_bounds__(128)
mla_pair_combine_kernel(const float* __restrict__ part_lse, const float* __restrict__ part_o,
                        T* __restrict__ out, float* __restrict__ lse_out, long long total_tiles,
                        int nt, int pairs, int maxp) {
  __shared__ float s_w[kMaxPairs];
  __shared__ int s_slot[kMaxPairs];
  __shared__ float s_lse;
  const int head = blockIdx.x, bb = blockIdx.y, tid = threadIdx.x;
  const long long x0 = (long long)bb * nt;
  // first/last pair whose range [p*T/P, (p+1)*T/P) meets this sequence's tiles
  const int pf = (int)(((x0 + 1) * pairs + total_tiles - 1) / total_tiles) - 1;
  const int pl = (int)(((x0 + nt) * pairs + total_tiles - 1) / total_tiles) - 1;
  if (pf == pl) return;
  const int n = pl - pf + 1;
  if (tid == 0) {
    float mx = -INFINITY;
    for (int k = 0; k < n; ++k) {
      const int pp = pf + k;
      const long long t0 = (long long)pp * total_tiles / pairs;
      const int slot = pp * maxp + (bb - (int)(t0 / nt));
      s_slot[k] = slot;
      s_w[k] = part_lse[(size_t)slot * kHeads + head];
      mx = fmaxf(mx, s_w[k]);
    }
    float sum = 0.f;
    for (int k = 0; k < n; ++k) sum += exp2f((s_w[k] - mx) * kLog2e);
    const float lse = mx + logf(sum);
    for (int k = 0; k < n; ++k) s_w[k] = exp2f((s_w[k] - lse) * kLog2e);
    s_lse = lse;
  }
  __syncthreads();
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
  for (int k = 0; k < n; ++k) {
    const float4 v = __ldg(
        reinterpret_cast<const float4*>(part_o + ((size_t)s_slot[k] * kHeads + head) * kDim) + tid);
    const float w = s_w[k];
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
  }
  uint2 o;
  o.x = pack2<T>(acc.x, acc.y);
  o.y = pack2<T>(acc.z, acc.w);
  reinterpret_cast<uint2*>(out + ((size_t)bb * kHeads + head) * kDim)[tid] = o;
  if (lse_out != nullptr && tid == 0) lse_out[(size_t)bb * kHeads + head] = s_lse;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2D row-major [rows, cols] tensor, 64 x 64 boxes, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, CUtensorMapDataType dt) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per-device launch facts: attributes set, how many clusters of 2 fit at once.
struct DeviceInfo {
  bool ready = false;
  int max_pairs = 0;
};
DeviceInfo g_dev[64];
std::mutex g_dev_mutex;

template <typename T>
cudaError_t set_attrs_and_count(int* pairs) {
  cudaError_t err = cudaFuncSetAttribute(mla_sm100_decode_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Smem<T>::kBytes);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * 74, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Smem<T>::kBytes;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaOccupancyMaxActiveClusters(pairs, mla_sm100_decode_kernel<T>, &cfg);
}

cudaError_t device_info(int dev, DeviceInfo* out) {
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int nb = 0, nh = 0;
    cudaError_t err = set_attrs_and_count<__nv_bfloat16>(&nb);
    if (err != cudaSuccess) return err;
    err = set_attrs_and_count<__half>(&nh);
    if (err != cudaSuccess) return err;
    d.max_pairs = nb < nh ? nb : nh;
    d.ready = true;
  }
  *out = d;
  return cudaSuccess;
}

int current_max_pairs() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  DeviceInfo d;
  if (device_info(dev, &d) != cudaSuccess) {
    cudaGetLastError();   // clear a sticky-free error from the query
    return 0;
  }
  return d.max_pairs;
}

}  // namespace sm100

bool sm100_supports(int heads, int seqlen_kv) { return heads == sm100::kHeads && seqlen_kv >= 1; }

SplitPlan sm100_plan(int batch, int heads, int seqlen_kv, const MlaCfg& cfg, int* variant) {
  (void)heads;
  SplitPlan pl{};
  *variant = 0;
  pl.block_n = sm100::kTile;
  const int nt = (seqlen_kv + sm100::kTile - 1) / sm100::kTile;
  const long long total = (long long)batch * nt;
  int pairs = cfg.num_split > 0 ? cfg.num_split : 0;
  int cap = sm100::current_max_pairs();
  if (cap <= 0) cap = 74;   // planning on a host without a usable GPU
  if (pairs == 0 || pairs > cap) pairs = cap;
  if (pairs > sm100::kMaxPairs) pairs = sm100::kMaxPairs;
  if ((long long)pairs > total) pairs = (int)total;
  const long long per = (total + pairs - 1) / pairs;
  const int maxp = (int)((per + nt - 1) / nt) + 1;
  pl.ns = pairs * maxp;          // partial slots
  pl.bpc = pairs;                // CTA pairs
  pl.extra = maxp;               // slots per pair
  pl.part_rows = (long long)pairs * maxp * sm100::kHeads;
  // no combine launch when every pair's range starts on a sequence boundary
  pl.needs_combine = false;
  for (int pp = 1; pp < pairs; ++pp)
    if (((long long)pp * total / pairs) % nt != 0) pl.needs_combine = true;
  return pl;
}

cudaError_t launch_sm100_decode(const DecodeArgs& a, int) {
  using namespace sm100;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  DeviceInfo info;
  err = device_info(dev, &info);
  if (err != cudaSuccess) return err;
  const int pairs = a.plan.bpc;
  if (pairs < 1 || pairs > info.max_pairs) return cudaErrorInvalidConfiguration;
  Params p{};
  const CUtensorMapDataType dt =
      a.dtype == MLA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t kv_rows = (uint64_t)a.batch * a.seqlen_kv;
  const uint64_t q_rows = (uint64_t)a.batch * kHeads;
  if (!make_map(&p.tm_kv, a.kv, kDim, kv_rows, dt) || !make_map(&p.tm_kpe, a.k_pe, kPeDim, kv_rows, dt) ||
      !make_map(&p.tm_q, a.q, kDim, q_rows, dt) || !make_map(&p.tm_qpe, a.q_pe, kPeDim, q_rows, dt))
    return cudaErrorInvalidValue;
  p.out = a.out;
  p.lse_out = a.lse;
  p.part_o = a.part_o;
  p.part_lse = a.part_lse;
  p.status = a.status;
  p.batch = a.batch;
  p.seqlen = a.seqlen_kv;
  p.nt = (a.seqlen_kv + kTile - 1) / kTile;
  p.total_tiles = (long long)a.batch * p.nt;
  p.pairs = pairs;
  p.maxp = a.plan.extra;
  p.sl2 = a.softmax_scale * kLog2e;
  if (a.dtype == MLA_DTYPE_BF16)
    mla_sm100_decode_kernel<__nv_bfloat16>
        <<<2 * pairs, kThreads, Smem<__nv_bfloat16>::kBytes, a.stream>>>(p);
  else
    mla_sm100_decode_kernel<__half><<<2 * pairs, kThreads, Smem<__half>::kBytes, a.stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_sm100_combine(const DecodeArgs& a) {
  using namespace sm100;
  const int nt = (a.seqlen_kv + kTile - 1) / kTile;
  const long long total = (long long)a.batch * nt;
  const dim3 grid(kHeads, a.batch);
  if (a.dtype == MLA_DTYPE_BF16)
    mla_pair_combine_kernel<__nv_bfloat16><<<grid, 128, 0, a.stream>>>(
        a.part_lse, a.part_o, static_cast<__nv_bfloat16*>(a.out), a.lse, total, nt, a.plan.bpc,
        a.plan.extra);
  else
    mla_pair_combine_kernel<__half><<<grid, 128, 0, a.stream>>>(
        a.part_lse, a.part_o, static_cast<__half*>(a.out), a.lse, total, nt, a.plan.bpc, a.plan.extra);
  return cudaGetLastError();
}

}  // namespace mla
