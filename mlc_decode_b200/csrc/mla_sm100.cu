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
//  * FP8 KV cache (Kv8<T>): the latent cache is e4m3 with one per-tensor scale
//    s (true value = s x code); the rope cache stays T.  QK^T runs as
//    kind::f8f6f4 UMMAs straight from the e4m3 K tiles (8 KB stages): q is
//    multiplied by a per-row power of two a and quantised to an e4m3 hi/lo
//    pair (hi in TMEM, lo in shared memory), and the rope part of q carries
//    a/s as a T hi/lo pair, so every score comes out scaled by a/s and the
//    softmax folds s/a into its log2 scale.  For P.V the e4m3 V tiles are
//    loaded locally and widened to fp16 by eight converter warps (warps
//    8..15) into the fp16 operand ring; P is fp16 and the output is scaled
//    by s in the epilogue.
#include <cuda.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <string.h>

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
// Q rows in shared memory: latent dims [256, 512) (4 boxes) and the rope dims (1 box);
// latent dims [0, 256) live in TMEM as the A operand of the first 16 QK^T k-steps.
constexpr int kQTDims = 256;
constexpr uint32_t kQBytes = 5 * kChunkBytes;
constexpr uint32_t kPBytes = 2 * kChunkBytes;   // one P operand: 64 rows x 128 tokens
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 128;
constexpr uint32_t kColQT = 384;      // Q dims [0, 256) as bf16/fp16 pairs: 128 columns
// Registers per thread after the split: launch budget 384 x 168 (512 x 128 for
// the FP8 variant's 4 warpgroups); producers, issuers, the Q loader and the
// converters need few, the softmax warps many.
constexpr uint32_t kRegsLow = 88, kRegsSoftmax = 232;
static_assert(2 * 128 * kRegsLow + 128 * kRegsSoftmax <= 384 * 168, "register split");
static_assert(3 * 128 * kRegsLow + 128 * kRegsSoftmax <= 512 * 128, "register split (FP8 variant)");
constexpr float kRescaleLog2 = 8.0f;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr int kMaxPairs = 256;        // CTA pairs per launch (schedule bound)
constexpr int kFuseMaxPieces = 3;     // most pieces of one sequence merged in-kernel
// bf16 calls run the Cv variant (each V stage converted to fp16 in place by the
// converter warps: one P.V pass, fp16 P); fp16 calls the plain variant (V is
// already fp16; only tail units are rewritten)
constexpr bool kConvV = true;
constexpr double kWholeSlack = 10.0;  // tiles per pair a whole-sequence assignment may add
// The cooperative merge stages up to 128 KB + 16 bytes a piece from offset 0 and
// keeps its tables at this offset (all below the barrier block of every variant).
constexpr uint32_t kMergeTab = 136 * 1024;
// A merge stages another pair's 64 partial rows (fp32, 2 KB each) in shared memory
// at this row pitch (16 bytes of padding: threads reading one column of 32 rows
// hit distinct banks).
constexpr uint32_t kMergePitch = kDim * 4 + 16;

// The workspace status block (256 bytes): word 0 the status word; 64-bit words
// kProbeWord.. accumulate the clock probe over calls (SM cycles, ns, calls).
constexpr int kProbeWord = 1;
// status codes written to the workspace status word on a timeout
constexpr uint32_t kErrKLoad = 0x101, kErrVLoad = 0x102, kErrQK = 0x103, kErrPV = 0x104,
                   kErrSoftmax = 0x105, kErrDrain = 0x106, kErrMerge = 0x107;

// Compile-time configuration per input type.  bf16 needs the hi/lo P pair
// (two P operands); fp16 P is exact enough and gives the space to the rings.
template <typename T>
struct Cfg;
template <>
struct Cfg<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  static constexpr uint32_t kPvFmt = 1;   // operand type of P.V (P and V)
  static constexpr uint32_t kRopeFmt = 1;
  static constexpr int kPParts = 2;
  static constexpr int kKStages = 4;
  static constexpr uint32_t kKStageBytes = kStageBytes;
  static constexpr int kVStages = 3;
  static constexpr int kV8Stages = 0;
  using PT = __nv_bfloat16;   // P operand type
};
template <>
struct Cfg<__half> {
  static constexpr uint32_t kFmt = 0;
  static constexpr uint32_t kPvFmt = 0;
  static constexpr uint32_t kRopeFmt = 0;
  static constexpr int kPParts = 1;
  static constexpr int kKStages = 6;
  static constexpr uint32_t kKStageBytes = kStageBytes;
  static constexpr int kVStages = 3;
  static constexpr int kV8Stages = 0;
  using PT = __half;
};

// The FP8 variant: latent KV rows in e4m3 (one byte per dim).  QK^T runs on the
// e4m3 tiles as loaded (kind::f8f6f4) against Q split into two e4m3 parts,
// hi = e4m3(q a) and lo = e4m3(q a - hi), a a per-row power of two that puts the
// row's largest |q a| near 224 (hi from TMEM, lo from shared memory): 8
// significant bits, exact for bf16 q.  The rope dims run in T against
// q_pe a / s as a T hi/lo pair (s the cache's scale), so the scores come out as
// (a / s) x the true ones and the softmax multiplies by s / a.  V is dequantized
// to fp16 in shared memory by converter warps (exact) and P.V runs in fp16 with
// fp16 P (no hi/lo pair); s is folded into the output normalisation.  T is the
// type of q, q_pe, k_pe and out.
template <typename T>
struct Kv8 {};
// The converter variant of a bf16 or fp16 call: each CTA's V producer loads V by
// TMA into its own stage of the V ring (a local barrier), and four converter
// warps (warps 12..15) rewrite the landed stage in place before the P.V issuer
// may read it: rows past the sequence's length become zeros (P.V then never
// multiplies a zero weight by a non-finite value the cache may hold there:
// uninitialised or recycled pages, another sequence's rows) and, with kF16 (bf16
// inputs), every value is converted to fp16 (exact within fp16's range), so P is
// fp16 and P.V runs once instead of as the bf16 hi/lo pair.
template <typename T, bool kF16>
struct Cv {};
template <typename K>
struct Io {
  using Out = K;
  static constexpr bool kKv8 = false;
  static constexpr bool kConv = false;   // V through the converter warps
};
template <typename T>
struct Io<Kv8<T>> {
  using Out = T;
  static constexpr bool kKv8 = true;
  static constexpr bool kConv = false;
};
template <typename T, bool kF16>
struct Io<Cv<T, kF16>> {
  using Out = T;
  static constexpr bool kKv8 = false;
  static constexpr bool kConv = true;
};
template <typename T>
struct Cfg<Kv8<T>> {
  static constexpr uint32_t kFmt = 0;
  static constexpr uint32_t kPvFmt = 0;
  static constexpr uint32_t kRopeFmt = Cfg<T>::kFmt;
  static constexpr int kPParts = 1;
  static constexpr int kKStages = 8;                 // e4m3 latent or rope units as loaded
  static constexpr uint32_t kKStageBytes = kChunkBytes;
  static constexpr int kVStages = 3;                 // fp16 V operand stages (16 KB)
  static constexpr int kV8Stages = 3;                // e4m3 V units as loaded (8 KB)
  using PT = __half;
  static_assert(kV8Stages <= 8, "barrier arrays");
};
template <typename T, bool kF16>
struct Cfg<Cv<T, kF16>> {
  // converting bf16 V to fp16: fp16 P, one P.V pass, the P space goes to the V ring
  static constexpr bool kToF16 = kF16 && std::is_same<T, __nv_bfloat16>::value;
  static constexpr uint32_t kFmt = Cfg<T>::kFmt;       // QK^T on the loaded K tiles
  static constexpr uint32_t kPvFmt = kToF16 ? 0u : Cfg<T>::kPvFmt;
  static constexpr uint32_t kRopeFmt = Cfg<T>::kFmt;
  static constexpr int kPParts = kToF16 ? 1 : Cfg<T>::kPParts;
  static constexpr int kKStages = kToF16 ? 5 : Cfg<T>::kKStages;
  static constexpr uint32_t kKStageBytes = kStageBytes;
  static constexpr int kVStages = kToF16 ? 4 : Cfg<T>::kVStages;
  static constexpr int kV8Stages = 0;
  using PT = typename std::conditional<kToF16, __half, typename Cfg<T>::PT>::type;
};
template <typename K>
constexpr int threads_of() { return (Io<K>::kKv8 || Io<K>::kConv) ? 512 : 384; }

struct Barriers {
  uint64_t kfull[8], kempty[8];
  uint64_t vfull[8], vempty[8];
  uint64_t v8full[8], v8empty[8];   // FP8 variant: e4m3 V units as loaded (plain and Cv: local V landing)
  uint64_t vfix[8];                 // plain variants: a tail unit rewritten in both CTAs
  uint64_t q_full, q_empty, qt_full;
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2];
  uint64_t xchg[2];
  uint64_t o_done[2], o_free, lx, stg, stg2, mload, mdone;
  uint64_t qts, qtr;     // Q dims [0, 256) staged in shared memory / copied to TMEM
  uint64_t q_go;         // the first piece's Q loads are issued: K and V loads may start
  uint64_t drain_qk, drain_pv;
};
static_assert(sizeof(Barriers) <= 1024, "barrier block");

// shared memory map (offsets from the 1024-byte aligned base)
template <typename T>
struct Smem {
  static constexpr uint32_t kQ = 0;
  // Q region: 4 latent boxes (fp16/bf16 dims [256, 512), or the FP8 variant's e4m3 lo
  // of all 512 dims) and the rope box (FP8: the rope hi and lo boxes)
  static constexpr uint32_t kP = kQ + (Io<T>::kKv8 ? 6 * kChunkBytes : kQBytes);
  static constexpr uint32_t kPBuf = Cfg<T>::kPParts * kPBytes;     // one P buffer (hi [, lo])
  static constexpr uint32_t kKRing = kP + 2 * kPBuf;
  static constexpr uint32_t kVRing = kKRing + Cfg<T>::kKStages * Cfg<T>::kKStageBytes;
  static constexpr uint32_t kV8Ring = kVRing + Cfg<T>::kVStages * kStageBytes;
  static constexpr uint32_t kBar = kV8Ring + Cfg<T>::kV8Stages * kChunkBytes;
  static constexpr uint32_t kXmax = kBar + 1024;
  static constexpr uint32_t kXl = kXmax + 2 * 128 * 4;
  static constexpr uint32_t kMisc = kXl + 128 * 4;
  static constexpr uint32_t kBytes = kMisc + 64 + 1024;   // + alignment slack
  static_assert(kBytes <= 232448, "shared memory");
  static_assert(kBar >= kMergeTab + 6 * 1024, "cooperative merge staging");
};

struct Params {
  CUtensorMap tm_kv;    // [b*s][kv_heads][512], box 64 x 1 x 64 rows (e4m3: 128 x 1 x 64)
  CUtensorMap tm_kpe;   // [b*s][kv_heads][64]
  CUtensorMap tm_q;     // [qb][h][512], box 64 x 64 x 1 (rows past h read as zero)
  CUtensorMap tm_qpe;   // [qb][h][64]
  CUtensorMap tm_out;   // [qb][h][512] output rows, box 64 x 64 x 1 (stores; rows past h not written)
  CUtensorMap tm_part;  // [slots*128, 512] float32 partial rows, box 32 x 64 (stores)
  const uint8_t* kv;    // raw latent rows (converter warps)
  const uint8_t* q;     // raw Q rows, for L2 prefetch
  const uint8_t* qpe;
  void* out;
  float* lse_out;
  float* part_o;
  float* part_lse;
  uint32_t* status;
  uint32_t* counters;   // [batch][4] per sequence: pieces published per CTA rank, then (cooperative
                        // merges) CTAs done merging per rank; zero between calls
  float kv_scale;       // FP8 variant: dequantisation scale of the e4m3 latent rows
  // Work units are "virtual sequences".  The query side is qb = b x q_len x
  // kv_heads query sequences qs = (s * q_len + t) * kv_heads + kvh (query
  // position t of sequence s, the query heads of KV head kvh: rows of q/out
  // that are contiguous in memory), each of `heads` rows; head group g (rows
  // [128 g, 128 g + 128)) of query sequence qs is v = qs * hgroups + g, and
  // batch counts them.  The KV side of v is sequence s, KV head kvh, and its
  // first len(s) - (q_len - 1 - t) rows (causal within the decode step).
  uint32_t total_tiles;  // batch x tiles per sequence; total_tiles * (pairs + 1) < 2^32
  int batch, seqlen, nt, pairs, maxp;
  int heads, hgroups;   // query rows per query sequence (h / kv_heads); groups of 128 of them
  int q_len, kv_heads;  // query positions per sequence, KV heads
  int out_f32;          // `out` is float32 (tm_out then has 32 x 64 float boxes)
  int fuse_max;         // sequences split into at most this many pieces are merged here
  int coop;             // cooperative launch: wider splits are merged here too (every pair waits)
  // Ragged calls (per-sequence lengths, optionally paged KV): cu_tiles[v] is the
  // first tile of virtual sequence v in the flattened list (batch + 1 entries,
  // written by the plan kernel); nullptr for fixed-length calls.
  const uint32_t* cu_tiles;
  const int* seqlens;      // [real batch] KV rows per sequence, or nullptr (all seqlen)
  const int* block_table;  // [real batch][max_pages] page ids, or nullptr (contiguous rows)
  int page_size, max_pages;
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

// Slow path of wait_bar: poll with a time limit.  (Inlined: a call out of a
// setmaxnreg region would have to follow the kernel-wide register budget.)
__device__ __forceinline__ bool wait_bar_slow(const Ctx& c, uint32_t bar, uint32_t parity, uint32_t code,
                                              uint64_t limit_ns = kTimeoutNs) {
  const uint64_t t0 = ptx::globaltimer();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile uint32_t*>(c.abort_local) != 0u) return false;
    if (ptx::globaltimer() - t0 > limit_ns) {
      raise_abort(c, code);
      return false;
    }
  }
}

// Bounded wait for the phase of `parity` on a local barrier.
__device__ __forceinline__ bool wait_bar(const Ctx& c, uint32_t bar, uint32_t parity, uint32_t code) {
  return ptx::mbar_try_wait(bar, parity) || wait_bar_slow(c, bar, parity, code);
}

__device__ __forceinline__ bool aborted(const Ctx& c) {
  return *reinterpret_cast<volatile uint32_t*>(c.abort_local) != 0u;
}

// Query sequence and first head row (within it) of virtual sequence v.
__device__ __forceinline__ int vseq_seq(const Params& p, int v) { return p.hgroups == 1 ? v : v / p.hgroups; }
__device__ __forceinline__ int vseq_head0(const Params& p, int v) {
  return p.hgroups == 1 ? 0 : (v % p.hgroups) * kHeads;
}
// KV sequence and KV head of virtual sequence v.
__device__ __forceinline__ int vseq_kvseq(const Params& p, int v) {
  const int qs = vseq_seq(p, v), per = p.q_len * p.kv_heads;
  return per == 1 ? qs : qs / per;
}
__device__ __forceinline__ int vseq_kvh(const Params& p, int v) {
  return p.kv_heads == 1 ? 0 : vseq_seq(p, v) % p.kv_heads;
}
// KV rows of query sequence qs: its sequence's length (nullptr: all max_len),
// clamped to [0, max_len], less the rows the causal mask hides from position t.
__device__ __forceinline__ int qseq_len(const int* seqlens, int qs, int q_len, int kv_heads, int max_len) {
  int len = max_len;
  if (seqlens != nullptr) {
    len = __ldg(seqlens + qs / (q_len * kv_heads));
    len = len < 0 ? 0 : (len > max_len ? max_len : len);
  }
  len -= q_len - 1 - (qs / kv_heads) % q_len;
  return len < 0 ? 0 : len;
}

// One contiguous run of tiles of one (virtual) sequence inside a pair's range.
struct Piece {
  int bb;        // sequence
  int first;     // first tile (within the sequence)
  int end;       // one past the last tile
  bool full;     // the run is the whole sequence
};

// The flattened tile list: virtual sequence v owns tiles [first(v), first(v+1)).
// Fixed-length calls: first(v) = v * nt; ragged calls: the prefix sums cu_tiles.
// Pair pp owns [pp*T/P, (pp+1)*T/P) (32-bit arithmetic: the host keeps
// T * (P + 1) below 2^32).
struct TileMap {
  const uint32_t* cu;
  uint32_t nt, total, pairs;
  int batch;
  __device__ __forceinline__ uint32_t first(int v) const {
    return cu != nullptr ? __ldg(cu + v) : (uint32_t)v * nt;
  }
  __device__ __forceinline__ uint32_t range_start(int pp) const { return (uint32_t)pp * total / pairs; }
  // pair whose range holds tile x
  __device__ __forceinline__ int pair_of(uint32_t x) const {
    return (int)(((x + 1) * pairs + total - 1) / total) - 1;
  }
  // sequence holding tile x (x < total): the last v with first(v) <= x
  __device__ int seq_of(uint32_t x) const {
    if (cu == nullptr) return (int)(x / nt);
    int lo = 0, hi = batch - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (first(mid) <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
};

// Pairs that own tiles: a ragged call may launch more pairs than it has tiles;
// the extra pairs own empty ranges past the end, never one inside a sequence.
__device__ __forceinline__ uint32_t effective_pairs(uint32_t launched, uint32_t total) {
  const uint32_t pp = launched < total ? launched : total;
  return pp > 0 ? pp : 1u;
}

__device__ __forceinline__ TileMap tile_map(const Params& p) {
  TileMap m;
  m.cu = p.cu_tiles;
  m.nt = (uint32_t)p.nt;
  m.batch = p.batch;
  m.total = p.cu_tiles != nullptr ? __ldg(p.cu_tiles + p.batch) : p.total_tiles;
  m.pairs = effective_pairs((uint32_t)p.pairs, m.total);
  return m;
}

// Iterates the pieces of pair `pair`'s tile range; empty sequences are skipped.
struct PieceIter {
  TileMap m;
  uint32_t t, t1;
  int v;
  __device__ PieceIter(const Params& p, int pair) : m(tile_map(p)) {
    if ((uint32_t)pair < m.pairs) {
      t = m.range_start(pair);
      t1 = m.range_start(pair + 1);
    } else {
      t = t1 = m.total;   // a pair past the ones that own tiles
    }
    v = t < t1 ? m.seq_of(t) : 0;
  }
  __device__ bool next(Piece* pc) {
    if (t >= t1) return false;
    while (m.first(v + 1) <= t) ++v;
    const uint32_t bstart = m.first(v), bend = m.first(v + 1);
    const uint32_t e = t1 < bend ? t1 : bend;
    pc->bb = v;
    pc->first = (int)(t - bstart);
    pc->end = (int)(e - bstart);
    pc->full = t == bstart && e == bend;
    t = e;
    return true;
  }
};

// KV rows of virtual sequence v, and the row in the KV tensor map of row `row`
// of sequence `seq` (contiguous [b, seqlen] rows, or a page of block_table).
// Longest sequence a call can hold: max_seqlen_kv, and for a paged call the rows
// its block table covers.
__device__ __forceinline__ int max_len(const Params& p) {
  if (p.block_table == nullptr) return p.seqlen;
  const long long cover = (long long)p.max_pages * p.page_size;
  return cover < p.seqlen ? (int)cover : p.seqlen;
}
__device__ __forceinline__ int seq_len(const Params& p, int v) {
  if (p.seqlens == nullptr && p.q_len == 1) return p.seqlen;
  // the plan kernel counts tiles with the same lengths
  return qseq_len(p.seqlens, vseq_seq(p, v), p.q_len, p.kv_heads, max_len(p));
}
__device__ __forceinline__ int kv_row(const Params& p, int seq, int row, int len) {
  if (p.block_table == nullptr) return seq * p.seqlen + row;
  // rows past the sequence's end are masked: read page 0 rather than a table entry
  // the caller may not have filled
  const int pg = row < len ? __ldg(p.block_table + (size_t)seq * p.max_pages + row / p.page_size) : 0;
  return pg * p.page_size + row % p.page_size;
}

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
  Ring<KS> ring;
  PieceIter it(p, pair);
  // the first Q rows are requested before any K or V traffic
  if (!wait_bar(c, ptx::smem_u32(&bars->q_go), 0u, kErrKLoad)) return;
  // Latent rows are read twice (K now, V one tile later): keep them in L2;
  // rope rows are read once.  (No bulk L2 prefetch ahead of the ring: on B200
  // it measured ~6 % slower at the bench shape.)
  const uint64_t keep = ptx::l2_policy_evict_last();
  const uint64_t once = ptx::l2_policy_evict_first();
  Piece pc;
  if constexpr (Io<T>::kKv8) {
    // FP8: per tile 4 e4m3 latent units (64 rows x 128 dims, one 8 KB box) and the
    // rope unit, straight into the K ring for the kind::f8f6f4 QK^T
    while (it.next(&pc)) {
      const int kseq = vseq_kvseq(p, pc.bb), kvh = vseq_kvh(p, pc.bb), klen = seq_len(p, pc.bb);
#pragma unroll 1
      for (int j = pc.first; j < pc.end; ++j) {
        const int y = kv_row(p, kseq, j * kTile + 64 * (int)rank, klen);
#pragma unroll 1
        for (int u = 0; u < 5; ++u) {
          if (!wait_bar(c, kempty0 + 8 * ring.stage, ring.phase ^ 1u, kErrKLoad)) return;
          if (leader) ptx::mbar_arrive_expect_tx(kfull0 + 8 * ring.stage, 2 * kChunkBytes);
          const uint32_t dst = sbase + S::kKRing + ring.stage * kChunkBytes;
          const uint32_t bar = kfull0_leader + 8 * ring.stage;
          if (u < 4)
            ptx::tma_load_3d_pair_hint(dst, &p.tm_kv, bar, 128 * u, kvh, y, keep);
          else
            ptx::tma_load_3d_pair_hint(dst, &p.tm_kpe, bar, 0, kvh, y, once);
          ring.advance();
        }
      }
    }
  } else {
  // K units stream straight across piece boundaries: Q has its own loader thread
  while (it.next(&pc)) {
    const int kseq = vseq_kvseq(p, pc.bb), kvh = vseq_kvh(p, pc.bb), klen = seq_len(p, pc.bb);
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j) {
      const int y = kv_row(p, kseq, j * kTile + 64 * (int)rank, klen);
#pragma unroll 1
      for (int u = 0; u < 5; ++u) {
        if (!wait_bar(c, kempty0 + 8 * ring.stage, ring.phase ^ 1u, kErrKLoad)) return;
        if (leader)
          ptx::mbar_arrive_expect_tx(kfull0 + 8 * ring.stage, u < 4 ? 2 * kStageBytes : 2 * kChunkBytes);
        const uint32_t dst = sbase + S::kKRing + ring.stage * kStageBytes;
        const uint32_t bar = kfull0_leader + 8 * ring.stage;
        if (u < 4) {
          ptx::tma_load_3d_pair_hint(dst, &p.tm_kv, bar, 128 * u, kvh, y, keep);
          ptx::tma_load_3d_pair_hint(dst + kChunkBytes, &p.tm_kv, bar, 128 * u + 64, kvh, y, keep);
        } else {
          ptx::tma_load_3d_pair_hint(dst, &p.tm_kpe, bar, 0, kvh, y, once);
        }
        ring.advance();
      }
    }
  }
  }
}

// Pull this CTA's (up to) 64 Q rows of virtual sequence `v` into L2.
__device__ __forceinline__ void prefetch_q(const Params& p, int v, uint32_t rank) {
  const int h0 = vseq_head0(p, v) + 64 * (int)rank;
  const int rows = p.heads - h0 < 64 ? p.heads - h0 : 64;
  if (rows <= 0) return;
  const long long row0 = (long long)vseq_seq(p, v) * p.heads + h0;
  ptx::prefetch_l2(p.q + row0 * (kDim * 2), (uint32_t)rows * (kDim * 2));
  ptx::prefetch_l2(p.qpe + row0 * (kPeDim * 2), (uint32_t)rows * (kPeDim * 2));
}

// ---------------------------------------------------------------------------
// Q loader, per piece, once the previous piece's QK^T no longer reads the Q
// region: first Q dims [0, 256) of this CTA's rows (staged for the softmax
// warps, which copy them into TMEM), then, once copied, Q dims [256, 512) and
// the rope dims for the shared-memory operand.  The next piece's rows are
// pulled into L2 ahead of time.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void q_loader(const Params& p, const Ctx& c, uint32_t rank, int pair,
                                         uint32_t sbase, Barriers* bars) {
  using S = Smem<T>;
  const bool leader = rank == 0;
  const uint32_t q_full = ptx::smem_u32(&bars->q_full);
  const uint32_t q_full_leader = ptx::mapa(q_full, 0);
  const uint32_t q_empty = ptx::smem_u32(&bars->q_empty);
  const uint32_t qts = ptx::smem_u32(&bars->qts);
  const uint32_t qtr = ptx::smem_u32(&bars->qtr);
  const uint32_t q_go = ptx::smem_u32(&bars->q_go);
  PieceIter it(p, pair);
  if constexpr (Io<T>::kKv8) {
    // FP8: the softmax warps read each piece's Q rows from global memory (they
    // quantize them); this thread only pulls the rows into L2 ahead of time
    Piece pq;
    bool first = true;
    while (it.next(&pq)) {
      prefetch_q(p, pq.bb, rank);
      if (first) ptx::mbar_arrive_local(q_go);
      first = false;
    }
    return;
  }
  {
    PieceIter first = it;
    Piece p0;
    if (first.next(&p0)) prefetch_q(p, p0.bb, rank);
  }
  Piece pc;
  int piece = 0;
  while (it.next(&pc)) {
    PieceIter peek = it;
    Piece nxt;
    if (peek.next(&nxt)) prefetch_q(p, nxt.bb, rank);
    if (piece > 0 && !wait_bar(c, q_empty, (uint32_t)(piece - 1) & 1u, kErrKLoad)) return;
    const int qseq = vseq_seq(p, pc.bb);
    const int qrow = vseq_head0(p, pc.bb) + 64 * (int)rank;   // head row within the sequence
    // the first piece stages dims [0, 256) in the (still unused) P buffers and loads
    // everything at once; later pieces reuse the Q region once the TMEM copy is made
    const uint32_t qt_dst = sbase + (piece == 0 ? S::kP : S::kQ);
    ptx::mbar_arrive_expect_tx(qts, 4 * kChunkBytes);
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch)
      ptx::tma_load_3d_local(qt_dst + ch * kChunkBytes, &p.tm_q, qts, 64 * ch, qrow, qseq);
    if (piece > 0 && !wait_bar(c, qtr, (uint32_t)piece & 1u, kErrKLoad)) return;
    if (leader) ptx::mbar_arrive_expect_tx(q_full, 2 * kQBytes);
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch)
      ptx::tma_load_3d_pair(sbase + S::kQ + ch * kChunkBytes, &p.tm_q, q_full_leader, kQTDims + 64 * ch,
                            qrow, qseq);
    ptx::tma_load_3d_pair(sbase + S::kQ + 4 * kChunkBytes, &p.tm_qpe, q_full_leader, 0, qrow, qseq);
    if (piece == 0) ptx::mbar_arrive_local(q_go);
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
  const uint64_t once = ptx::l2_policy_evict_first();
  const uint32_t vfull0 = ptx::smem_u32(&bars->vfull[0]);
  const uint32_t vfull0_leader = ptx::mapa(vfull0, 0);
  const uint32_t vempty0 = ptx::smem_u32(&bars->vempty[0]);
  Ring<VS> ring;
  PieceIter it(p, pair);
  if (!wait_bar(c, ptx::smem_u32(&bars->q_go), 0u, kErrVLoad)) return;
  Piece pc;
  if constexpr (Io<T>::kKv8) {
    // FP8: unit u = (nh, th) is this CTA's 128 latent dims [256 nh + 128 rank, +128)
    // of tokens [64 th, +64) in e4m3 (one 8 KB box), on a local barrier
    const uint32_t v8full0 = ptx::smem_u32(&bars->v8full[0]);
    const uint32_t v8empty0 = ptx::smem_u32(&bars->v8empty[0]);
    Ring<Cfg<T>::kV8Stages> r8;
    while (it.next(&pc)) {
      const int vseq = vseq_kvseq(p, pc.bb), kvh = vseq_kvh(p, pc.bb), vlen = seq_len(p, pc.bb);
#pragma unroll 1
      for (int j = pc.first; j < pc.end; ++j) {
        const int yv0 = kv_row(p, vseq, j * kTile, vlen), yv1 = kv_row(p, vseq, j * kTile + 64, vlen);
#pragma unroll 1
        for (int u = 0; u < 4; ++u) {
          const int nh = u >> 1, th = u & 1;
          if (!wait_bar(c, v8empty0 + 8 * r8.stage, r8.phase ^ 1u, kErrVLoad)) return;
          const uint32_t bar = v8full0 + 8 * r8.stage;
          ptx::mbar_arrive_expect_tx(bar, kChunkBytes);
          ptx::tma_load_3d_local_hint(sbase + S::kV8Ring + r8.stage * kChunkBytes, &p.tm_kv, bar,
                                      256 * nh + 128 * (int)rank, kvh, th == 0 ? yv0 : yv1, once);
          r8.advance();
        }
      }
    }
  } else if constexpr (Io<T>::kConv) {
    // Cv: this CTA's 128 latent columns of the tile's 64-token halves into its own
    // stage, landing on a local barrier: the converter warps rewrite the stage
    // before the P.V issuer is told it is full
    const uint32_t land0 = ptx::smem_u32(&bars->v8full[0]);
    while (it.next(&pc)) {
      const int vseq = vseq_kvseq(p, pc.bb), kvh = vseq_kvh(p, pc.bb), vlen = seq_len(p, pc.bb);
#pragma unroll 1
      for (int j = pc.first; j < pc.end; ++j) {
        const int yv0 = kv_row(p, vseq, j * kTile, vlen), yv1 = kv_row(p, vseq, j * kTile + 64, vlen);
#pragma unroll 1
        for (int u = 0; u < 4; ++u) {
          const int nh = u >> 1, th = u & 1;
          if (!wait_bar(c, vempty0 + 8 * ring.stage, ring.phase ^ 1u, kErrVLoad)) return;
          const uint32_t bar = land0 + 8 * ring.stage;
          ptx::mbar_arrive_expect_tx(bar, kStageBytes);
          const uint32_t dst = sbase + S::kVRing + ring.stage * kStageBytes;
          const int x = 256 * nh + 128 * (int)rank;
          const int yv = th == 0 ? yv0 : yv1;
          ptx::tma_load_3d_local_hint(dst, &p.tm_kv, bar, x, kvh, yv, once);
          ptx::tma_load_3d_local_hint(dst + kChunkBytes, &p.tm_kv, bar, x + 64, kvh, yv, once);
          ring.advance();
        }
      }
    }
  } else {
  const uint32_t land0 = ptx::smem_u32(&bars->v8full[0]);
  while (it.next(&pc)) {
    const int vseq = vseq_kvseq(p, pc.bb), kvh = vseq_kvh(p, pc.bb), vlen = seq_len(p, pc.bb);
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j) {
      // both token halves' rows, looked up before the ring waits (page-table loads)
      const int yv0 = kv_row(p, vseq, j * kTile, vlen), yv1 = kv_row(p, vseq, j * kTile + 64, vlen);
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        const int nh = u >> 1, th = u & 1;
        if (!wait_bar(c, vempty0 + 8 * ring.stage, ring.phase ^ 1u, kErrVLoad)) return;
        const uint32_t dst = sbase + S::kVRing + ring.stage * kStageBytes;
        const int x = 256 * nh + 128 * (int)rank;
        // the latent rows' last read
        const int yv = th == 0 ? yv0 : yv1;
        if (vlen - (j * kTile + 64 * th) < 64) {
          // a tail unit: into this CTA's stage on a local barrier; the tail fixer zeroes
          // the rows past the length before the stage is reported full
          const uint32_t bar = land0 + 8 * ring.stage;
          ptx::mbar_arrive_expect_tx(bar, kStageBytes);
          ptx::tma_load_3d_local_hint(dst, &p.tm_kv, bar, x, kvh, yv, once);
          ptx::tma_load_3d_local_hint(dst + kChunkBytes, &p.tm_kv, bar, x + 64, kvh, yv, once);
        } else {
          if (leader) ptx::mbar_arrive_expect_tx(vfull0 + 8 * ring.stage, 2 * kStageBytes);
          const uint32_t bar = vfull0_leader + 8 * ring.stage;
          ptx::tma_load_3d_pair_hint(dst, &p.tm_kv, bar, x, kvh, yv, once);
          ptx::tma_load_3d_pair_hint(dst + kChunkBytes, &p.tm_kv, bar, x + 64, kvh, yv, once);
        }
        ring.advance();
      }
    }
  }
  }
}

// ---------------------------------------------------------------------------
// FP8 variant: V converter warps (warps 8..15).  All eight take every e4m3 V unit
// (64 tokens x 128 dims, one SW128 box), each an eighth of its 16-byte granules,
// and write the fp16 operand stage P.V reads (the same rows as two SW128 boxes of
// 64 dims); then each releases the e4m3 stage (local, count 8) and signals the
// operand stage to the even CTA's P.V issuer (count 8 warps x 2 CTAs).  e4m3 ->
// fp16 is exact.
// ---------------------------------------------------------------------------
constexpr int kConvWarps = 8;

__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v & 0xffffu), __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

template <typename T>
__device__ __forceinline__ void v_converter(const Params& p, const Ctx& c, int pair, uint8_t* smem,
                                            Barriers* bars, int ct, int lane) {
  using S = Smem<T>;
  constexpr int kPer = 512 / (32 * kConvWarps);   // granules per thread and unit
  const uint32_t full8 = ptx::smem_u32(&bars->v8full[0]);
  const uint32_t empty8 = ptx::smem_u32(&bars->v8empty[0]);
  const uint32_t op_empty = ptx::smem_u32(&bars->vempty[0]);
  const uint32_t op_full_leader = ptx::mapa(ptx::smem_u32(&bars->vfull[0]), 0);
  const uint8_t* ring8 = smem + S::kV8Ring;
  uint8_t* ring_op = smem + S::kVRing;
  Ring<Cfg<T>::kV8Stages> r8;
  Ring<Cfg<T>::kVStages> rop;
  PieceIter it(p, pair);
  Piece pc;
  while (it.next(&pc)) {
    const int klen = seq_len(p, pc.bb);
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j) {
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        if (!wait_bar(c, full8 + 8 * r8.stage, r8.phase, kErrVLoad)) return;
        if (!wait_bar(c, op_empty + 8 * rop.stage, rop.phase ^ 1u, kErrVLoad)) return;
        const uint8_t* src = ring8 + r8.stage * kChunkBytes;
        uint8_t* dst = ring_op + rop.stage * kStageBytes;
        // rows past the sequence's length become zeros (whatever codes the cache holds there)
        const int nvalid = klen - (j * kTile + 64 * (u & 1));
        // all of this thread's granules in flight before any conversion
        uint4 x[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          // logical 16-byte granule g of row r (elements [16 g, 16 g + 16)) sits at g ^ (r & 7)
          const int i = ct + 32 * kConvWarps * k, r = i >> 3, g = i & 7;
          x[k] = r < nvalid ? *reinterpret_cast<const uint4*>(src + r * 128 + ((g ^ (r & 7)) << 4))
                            : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int i = ct + 32 * kConvWarps * k, r = i >> 3, g = i & 7;
          uint8_t* row = dst + (g >> 2) * kChunkBytes + r * 128;
          const int g1 = 2 * (g & 3);
          *reinterpret_cast<uint4*>(row + ((g1 ^ (r & 7)) << 4)) =
              make_uint4(e4m3x2_to_h2(x[k].x), e4m3x2_to_h2(x[k].x >> 16), e4m3x2_to_h2(x[k].y),
                         e4m3x2_to_h2(x[k].y >> 16));
          *reinterpret_cast<uint4*>(row + (((g1 + 1) ^ (r & 7)) << 4)) =
              make_uint4(e4m3x2_to_h2(x[k].z), e4m3x2_to_h2(x[k].z >> 16), e4m3x2_to_h2(x[k].w),
                         e4m3x2_to_h2(x[k].w >> 16));
        }
        // the tensor core reads the stage through the async proxy
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::mbar_arrive_local(empty8 + 8 * r8.stage);
          ptx::mbar_arrive_cluster(op_full_leader + 8 * rop.stage);
        }
        r8.advance();
        rop.advance();
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Tail fixer of the plain variants (warp 9 of each CTA).  A V unit whose 64 token
// rows run past the sequence's length (the last tile of a sequence) is loaded by
// the V producer into this CTA's stage on a local barrier instead of the pair
// barrier; this warp zeroes the rows past the length (so that P = 0 never meets a
// non-finite value the cache holds there: uninitialised or recycled pages,
// another sequence's rows), signals the even CTA's fixer, which reports the stage
// full to the P.V issuer once both halves are done.  Full units are not touched.
// Tail units are rare, so each stage's local barriers keep their own phase bit.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void v_tailfix(const Params& p, const Ctx& c, uint32_t rank, int pair, uint8_t* smem,
                                          Barriers* bars, int lane) {
  using S = Smem<T>;
  constexpr int VS = Cfg<T>::kVStages;
  const uint32_t land0 = ptx::smem_u32(&bars->v8full[0]);
  const uint32_t fix0 = ptx::smem_u32(&bars->vfix[0]);
  const uint32_t fix0_leader = ptx::mapa(fix0, 0);
  const uint32_t vfull0 = ptx::smem_u32(&bars->vfull[0]);
  uint8_t* ring = smem + S::kVRing;
  uint32_t par = 0;   // per stage: phase of its next tail use
  Ring<VS> rg;
  PieceIter it(p, pair);
  Piece pc;
  while (it.next(&pc)) {
    const int vlen = seq_len(p, pc.bb);
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j) {
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        const int nvalid = vlen - (j * kTile + 64 * (u & 1));
        if (nvalid < 64) {
          const uint32_t ph = (par >> rg.stage) & 1u;
          if (!wait_bar(c, land0 + 8 * rg.stage, ph, kErrVLoad)) return;
          uint4* st = reinterpret_cast<uint4*>(ring + rg.stage * kStageBytes);
          // 1024 16-byte granules; granule i is in row (i / 8) % 64 whatever the swizzle
#pragma unroll 4
          for (int i = lane; i < 1024; i += 32)
            if (((i >> 3) & 63) >= nvalid) st[i] = make_uint4(0u, 0u, 0u, 0u);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::mbar_arrive_cluster(fix0_leader + 8 * rg.stage);
            if (rank == 0) {
              // both CTAs' halves are rewritten: the stage is full for the P.V issuer
              if (!wait_bar(c, fix0 + 8 * rg.stage, ph, kErrVLoad)) return;
              ptx::mbar_arrive_local(vfull0 + 8 * rg.stage);
            }
          }
          __syncwarp();
          par ^= 1u << rg.stage;
        }
        rg.advance();
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Converter warps of the Cv variant (warps 12..15): every V unit of the ring, as
// the V producer's local TMA lands it (this CTA's 128 latent dims of 64 tokens,
// two SW128 boxes), is rewritten in place: rows past the sequence's length as
// zeros, and (kToF16) bf16 values as fp16.  The conversion is elementwise, so the
// swizzle does not matter: thread ct takes 16-byte granules ct + 128 k of the
// 16 KB stage (row = (granule / 8) % 64).  Then each warp signals the stage to
// the even CTA's P.V issuer (count 4 warps x 2 CTAs).
// ---------------------------------------------------------------------------
constexpr int kFixWarps = 4;

// two bf16 (low half first) -> two fp16, round to nearest (exact in fp16's range)
__device__ __forceinline__ uint32_t bf16x2_to_h2(uint32_t w) {
  return Elt<__half>::pack2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

template <typename KT>
__device__ __forceinline__ void v_fix(const Params& p, const Ctx& c, int pair, uint8_t* smem, Barriers* bars,
                                      int ct, int lane) {
  using S = Smem<KT>;
  constexpr int VS = Cfg<KT>::kVStages;
  constexpr bool kToF16 = Cfg<KT>::kToF16;
  constexpr int kPer = (int)kStageBytes / 16 / (32 * kFixWarps);   // granules per thread and unit
  const uint32_t land0 = ptx::smem_u32(&bars->v8full[0]);
  const uint32_t full0_leader = ptx::mapa(ptx::smem_u32(&bars->vfull[0]), 0);
  uint8_t* ring = smem + S::kVRing;
  Ring<VS> rg;
  PieceIter it(p, pair);
  Piece pc;
  while (it.next(&pc)) {
    const int klen = seq_len(p, pc.bb);
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j) {
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        if (!wait_bar(c, land0 + 8 * rg.stage, rg.phase, kErrVLoad)) return;
        uint4* st = reinterpret_cast<uint4*>(ring + rg.stage * kStageBytes);
        const int nvalid = klen - (j * kTile + 64 * (u & 1));
        if constexpr (kToF16) {
          uint4 x[kPer];
#pragma unroll
          for (int k = 0; k < kPer; ++k) x[k] = st[ct + 128 * k];
#pragma unroll
          for (int k = 0; k < kPer; ++k) {
            const int i = ct + 128 * k, r = (i >> 3) & 63;
            st[i] = r < nvalid ? make_uint4(bf16x2_to_h2(x[k].x), bf16x2_to_h2(x[k].y), bf16x2_to_h2(x[k].z),
                                            bf16x2_to_h2(x[k].w))
                               : make_uint4(0u, 0u, 0u, 0u);
          }
          ptx::fence_proxy_async_smem();
        } else if (nvalid < 64) {
#pragma unroll
          for (int k = 0; k < kPer; ++k) {
            const int i = ct + 128 * k, r = (i >> 3) & 63;
            if (r >= nvalid) st[i] = make_uint4(0u, 0u, 0u, 0u);
          }
          ptx::fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(full0_leader + 8 * rg.stage);
        rg.advance();
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
  constexpr uint32_t kIdescRope = ptx::idesc_f16(Cfg<T>::kRopeFmt, 128, 128, 0);
  const uint32_t kfull0 = ptx::smem_u32(&bars->kfull[0]);
  const uint32_t kempty0 = ptx::smem_u32(&bars->kempty[0]);
  const uint32_t q_full = ptx::smem_u32(&bars->q_full);
  const uint32_t q_empty = ptx::smem_u32(&bars->q_empty);
  const uint32_t qt_full = ptx::smem_u32(&bars->qt_full);
  const uint32_t s_full0 = ptx::smem_u32(&bars->s_full[0]);
  const uint32_t s_free0 = ptx::smem_u32(&bars->s_free[0]);
  const uint32_t qlo = ptx::sw128_desc_lo(sbase + S::kQ, 16);
  constexpr uint32_t kHiK = ptx::sw128_desc_hi(1024);
  Ring<KS> ring;
  uint32_t gi = 0;
  PieceIter it(p, pair);
  Piece pc;
  int piece = 0;
  while (it.next(&pc)) {
    // (FP8: qt_full covers the whole quantized Q, written by the softmax warps)
    if (!Io<T>::kKv8 && !wait_bar(c, q_full, (uint32_t)piece & 1u, kErrQK)) return;
    if (!wait_bar(c, qt_full, (uint32_t)piece & 1u, kErrQK)) return;
    ptx::tc_fence_after();
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j, ++gi) {
      const uint32_t b = gi & 1u;
      // the softmax warps must have read S[b] of tile gi - 2
      if (gi >= 2 && !wait_bar(c, s_free0 + 8 * b, ((gi - 2) >> 1) & 1u, kErrQK)) return;
      ptx::tc_fence_after();
      const uint32_t s_tmem = tmem + 64 * b;
#pragma unroll
      for (int u = 0; u < 5; ++u) {
        if (!wait_bar(c, kfull0 + 8 * ring.stage, ring.phase, kErrQK)) return;
        ptx::tc_fence_after();
        // descriptor low words; +512 = next 8 KB box, +2 = next 32-byte k-step
        const uint32_t kb = ptx::sw128_desc_lo(sbase + S::kKRing + ring.stage * Cfg<T>::kKStageBytes, 16);
        if (Io<T>::kKv8 && u < 4) {
          // FP8: latent dims [128 u, +128) in e4m3, 32 per k-step: Q hi from TMEM (4
          // elements per column), Q lo from box u of the Q region
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bd = ptx::make_desc(kb + kk * 2, kHiK);
            ptx::mma_pair_f8_ts(s_tmem, tmem + kColQT + 8 * (4 * u + kk), bd, kIdesc,
                                (u == 0 && kk == 0) ? 0u : 1u);
            ptx::mma_pair_f8(s_tmem, ptx::make_desc(qlo + u * 512 + kk * 2, kHiK), bd, kIdesc, 1u);
          }
        } else if (!Io<T>::kKv8 && u < 2) {
          // latent dims [0, 256): Q from TMEM, 8 columns (16 elements) per k-step
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            ptx::mma_pair_f16_ts(s_tmem, tmem + kColQT + 8 * (8 * u + kk),
                                 ptx::make_desc(kb + (kk >> 2) * 512 + (kk & 3) * 2, kHiK), kIdesc,
                                 (u == 0 && kk == 0) ? 0u : 1u);
        } else {
          const uint32_t qa = qlo + (u < 4 ? 2 * (u - 2) : 4) * 512;
          const int nk = u < 4 ? 8 : 4;
#pragma unroll
          for (int kk = 0; kk < nk; ++kk)
            ptx::mma_pair_f16(s_tmem, ptx::make_desc(qa + (kk >> 2) * 512 + (kk & 3) * 2, kHiK),
                              ptx::make_desc(kb + (kk >> 2) * 512 + (kk & 3) * 2, kHiK),
                              u < 4 ? kIdesc : kIdescRope, 1u);
          if (Io<T>::kKv8) {
            // FP8: the rope's lo part (box 5 of the Q region)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              ptx::mma_pair_f16(s_tmem, ptx::make_desc(qlo + 5 * 512 + kk * 2, kHiK), ptx::make_desc(kb + kk * 2, kHiK),
                                kIdescRope, 1u);
          }
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
  constexpr uint32_t kIdesc = ptx::idesc_f16(Cfg<T>::kPvFmt, 128, 256, 1);
  const uint32_t vfull0 = ptx::smem_u32(&bars->vfull[0]);
  const uint32_t vempty0 = ptx::smem_u32(&bars->vempty[0]);
  const uint32_t p_full0 = ptx::smem_u32(&bars->p_full[0]);
  const uint32_t o_done0 = ptx::smem_u32(&bars->o_done[0]);
  const uint32_t o_free = ptx::smem_u32(&bars->o_free);
  const uint32_t plo = ptx::sw128_desc_lo(sbase + S::kP, 16);
  constexpr uint32_t kHi = ptx::sw128_desc_hi(1024);
  Ring<VS> ring;
  uint32_t gi = 0;
  PieceIter it(p, pair);
  Piece pc;
  int piece = 0;
  while (it.next(&pc)) {
#pragma unroll 1
    for (int j = pc.first; j < pc.end; ++j, ++gi) {
      const bool first = j == pc.first;
      const uint32_t b = gi & 1u;
      if (!wait_bar(c, p_full0 + 8 * b, (gi >> 1) & 1u, kErrPV)) return;
      // a new piece restarts O: the previous piece's epilogue must have read it
      if (first && piece > 0 && !wait_bar(c, o_free, (uint32_t)(piece - 1) & 1u, kErrPV)) return;
      ptx::tc_fence_after();
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        const int nh = u >> 1, th = u & 1;
        if (!wait_bar(c, vfull0 + 8 * ring.stage, ring.phase, kErrPV)) return;
        ptx::tc_fence_after();
        // descriptor low words: V is MN-major (+128 = next 16 rows), P K-major (+2 = next k-step)
        const uint32_t vb = ptx::sw128_desc_lo(sbase + S::kVRing + ring.stage * kStageBytes, kChunkBytes);
#pragma unroll
        for (int part = 0; part < Cfg<T>::kPParts; ++part) {
          const uint32_t pa = plo + b * (S::kPBuf >> 4) + part * (kPBytes >> 4) + th * 512;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            ptx::mma_pair_f16(tmem + kColO + 128 * nh, ptx::make_desc(pa + kk * 2, kHi),
                              ptx::make_desc(vb + kk * 128, kHi), kIdesc,
                              (first && th == 0 && kk == 0 && part == 0) ? 0u : 1u);
        }
        ptx::mma_commit_pair_mc(vempty0 + 8 * ring.stage, 0x3);
        ring.advance();
      }
      ptx::mma_commit_pair_mc(o_done0 + 8 * b, 0x3);
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

// Workspace slot of sequence bb's piece inside pair pp's range: two per pair,
// 0 for the piece the range starts in, 1 for the piece it ends in (only a
// range's first and last pieces can be parts of a split sequence).
__device__ __forceinline__ size_t pair_slot(const TileMap& m, int pp, int bb) {
  return (size_t)pp * 2 + (m.first(bb) <= m.range_start(pp) ? 0 : 1);
}

// First and last pair whose tile range meets (non-empty) sequence bb.
__device__ __forceinline__ void pairs_of_sequence(const TileMap& m, int bb, int* pf, int* pl) {
  *pf = m.pair_of(m.first(bb));
  *pl = m.pair_of(m.first(bb + 1) - 1);
}

// Copy this CTA's staged Q rows, latent dims [0, 256) (four SW128 boxes at
// `src`: the P buffers for the first piece, else the start of the Q region), into
// TMEM as the A operand of the first 16 QK^T k-steps: lane L <- row L % 64, so both
// lane halves hold the rows (the duplicated layout of a pair MMA's A operand in
// TMEM).
__device__ __forceinline__ void copy_qt(const uint8_t* src, int m, uint32_t tmem, uint32_t lane_off) {
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const uint8_t* row = src + ch * kChunkBytes + m * 128;
    uint32_t w[32];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const uint4 x = *reinterpret_cast<const uint4*>(row + ((g ^ (m & 7)) << 4));
      w[4 * g] = x.x;
      w[4 * g + 1] = x.y;
      w[4 * g + 2] = x.z;
      w[4 * g + 3] = x.w;
    }
    ptx::tmem_st32(tmem + lane_off + kColQT + 32 * ch, w);
  }
  ptx::tmem_wait_st();
}

// Row m (128 bytes) of an SW128 staging box: 16-byte granule g at g ^ (m & 7).
__device__ __forceinline__ void st_box_row(uint8_t* box, int m, const uint32_t (&w)[32]) {
#pragma unroll
  for (int g = 0; g < 8; ++g)
    *reinterpret_cast<uint4*>(box + m * 128 + ((g ^ (m & 7)) << 4)) =
        make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
}

// FP8 variant: this thread's Q row for the kind::f8f6f4 QK^T (see Kv8).  Row m of
// CTA `rank`'s 64 heads of virtual sequence v, read from global memory (rows past
// the head count are zero); a = a power of two with max |q a| <= 224 (and
// |q_pe a / s| <= 16384, s the cache's scale).  Writes hi = e4m3(q a) for all 512
// dims to this lane's TMEM columns [kColQT, +128) (4 dims per column; both lane
// halves hold the row), lo = e4m3(q a - hi) for this thread's half of the dims
// (hf) to boxes 2 hf, 2 hf + 1 of the Q region (128 dims = 128 bytes a row,
// SW128), and its half of q_pe a / s as a T hi/lo pair to boxes 4 and 5.
// Returns s / a, the factor that takes the row's scores to their true values.
__device__ __forceinline__ uint32_t f2_to_e4m3x2(float a, float b) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float2 e4m3x2_to_f2(uint32_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v & 0xffffu), __NV_E4M3);
  __half2 hh;
  hh.x = __ushort_as_half(h.x);
  hh.y = __ushort_as_half(h.y);
  return __half22float2(hh);
}

template <typename Out>
__device__ __forceinline__ float quantize_q(const Params& p, int v, uint32_t rank, int m, int hf, uint8_t* qreg,
                                            uint32_t tmem, uint32_t lane_off) {
  const int h = vseq_head0(p, v) + 64 * (int)rank + m;
  const bool real = h < p.heads;
  const size_t row = (size_t)vseq_seq(p, v) * p.heads + (real ? h : 0);
  const uint4* qg = reinterpret_cast<const uint4*>(p.q) + row * (kDim / 8);      // 8 elements a granule
  const uint4* rg = reinterpret_cast<const uint4*>(p.qpe) + row * (kPeDim / 8);
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  float amax = 0.f, rmax = 0.f;
  // eight 16-byte loads of the row in flight at a time (one at a time, the scan
  // took ~64 L2 round trips before the piece's first QK^T could start)
#pragma unroll 1
  for (int g0 = 0; g0 < kDim / 8; g0 += 8) {
    uint4 xs[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) xs[k] = real ? __ldg(qg + g0 + k) : zero;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t w[4] = {xs[k].x, xs[k].y, xs[k].z, xs[k].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Elt<Out>::to2(w[e]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
#pragma unroll
  for (int g = 0; g < kPeDim / 8; ++g) {
    const uint4 x = real ? __ldg(rg + g) : zero;
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Elt<Out>::to2(w[e]);
      rmax = fmaxf(rmax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  const float s = p.kv_scale;
  float a = amax > 0.f ? exp2f(floorf(log2f(224.f / amax))) : 1.f;
  if (rmax * a > 16384.f * s) a = exp2f(floorf(log2f(16384.f * s / rmax)));
  const float qs = a;
#pragma unroll 1
  for (int cb = 0; cb < 4; ++cb) {   // 128 dims: 32 TMEM columns, one lo box
    uint32_t w[32];
    uint8_t* lrow = qreg + cb * kChunkBytes + m * 128;
    const bool mine = (cb >> 1) == hf;
#pragma unroll
    for (int g = 0; g < 16; ++g) {
      const uint4 x = real ? __ldg(qg + cb * 16 + g) : zero;
      const uint32_t in[4] = {x.x, x.y, x.z, x.w};
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Elt<Out>::to2(in[e]);
        const float2 v2 = make_float2(f.x * qs, f.y * qs);
        hi[e] = f2_to_e4m3x2(v2.x, v2.y);
        const float2 hb = e4m3x2_to_f2(hi[e]);
        lo[e] = f2_to_e4m3x2(v2.x - hb.x, v2.y - hb.y);
      }
      w[2 * g] = hi[0] | (hi[1] << 16);
      w[2 * g + 1] = hi[2] | (hi[3] << 16);
      if (mine)   // 8 bytes: half of 16-byte granule g / 2 (at (g / 2) ^ (m & 7))
        *reinterpret_cast<uint2*>(lrow + (((g >> 1) ^ (m & 7)) << 4) + (g & 1) * 8) =
            make_uint2(lo[0] | (lo[1] << 16), lo[2] | (lo[3] << 16));
    }
    ptx::tmem_st32(tmem + lane_off + kColQT + 32 * cb, w);
  }
  ptx::tmem_wait_st();
  uint8_t* rrow = qreg + 4 * kChunkBytes + m * 128;
  const float ra = a / s;
#pragma unroll
  for (int g = 4 * hf; g < 4 * hf + 4; ++g) {
    const uint4 x = real ? __ldg(rg + g) : zero;
    const uint32_t in[4] = {x.x, x.y, x.z, x.w};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Elt<Out>::to2(in[e]);
      const float2 v2 = make_float2(f.x * ra, f.y * ra);
      hi[e] = Elt<Out>::pack2(v2.x, v2.y);
      const float2 hb = Elt<Out>::to2(hi[e]);
      lo[e] = Elt<Out>::pack2(v2.x - hb.x, v2.y - hb.y);
    }
    const uint32_t off = (uint32_t)((g ^ (m & 7)) << 4);
    *reinterpret_cast<uint4*>(rrow + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(rrow + kChunkBytes + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
  return s / a;
}

// ---------------------------------------------------------------------------
// Cooperative merge of one sequence split between more than fuse_max pairs
// (p.coop: every pair of the launch is resident).  The LSE combine of
// mla_decode.py:212-246 over all of the sequence's pieces, spread over every CTA
// of this rank that holds one: CTA k of n waits (bounded) until all n pieces of
// its rank are published, then merges its contiguous share [o0, o1) of the rank's
// 64 x 128 output quads (4 latent columns of one head): that share of every piece
// is staged in the (idle) shared memory by one bulk copy per piece, all in flight
// at once, while the weights of its heads are computed from the pieces' LSEs;
// then each thread sums its quads over the pieces from shared memory.  Run by the
// 4 softmax warps (L is the thread's index among them); `bar` / `ph` is their
// 4-warp barrier, `mbar` / `mph` the staging barrier.
// ---------------------------------------------------------------------------
template <typename Out>
__device__ __noinline__ bool coop_merge(const Params& p, const Ctx& c, const TileMap& tm, uint32_t rank, int pair,
                                        uint8_t* smem, uint32_t bar, uint32_t& ph, uint32_t mbar, uint32_t& mph,
                                        volatile uint32_t* flag, int L, int lane, int bb, int pf, int pl) {
  auto sync4 = [&]() -> bool {
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive_local(bar);
    const bool ok = wait_bar(c, bar, ph & 1u, kErrSoftmax);
    ++ph;
    return ok;
  };
  const int n = pl - pf + 1, k = pair - pf;
  uint32_t* arrive = p.counters + 4 * bb + rank;
  uint32_t* done = p.counters + 4 * bb + 2 + rank;
  constexpr int kQuads = 64 * (kDim / 4);            // this rank's output quads
  const int o0 = (int)((long long)k * kQuads / n), o1 = (int)((long long)(k + 1) * kQuads / n);
  const int h_lo = o0 / (kDim / 4), nh = (o1 - 1) / (kDim / 4) - h_lo + 1;
  const uint32_t chunk = (uint32_t)(o1 - o0) * 16u;   // bytes of this CTA's share of one piece
  // the idle shared memory: every piece's share staged from offset 0 (at most
  // 128 KB + 16 n bytes), the tables at kMergeTab
  uint32_t* s_slot = reinterpret_cast<uint32_t*>(smem + kMergeTab);   // [n]
  float* s_w = reinterpret_cast<float*>(s_slot + kMaxPairs);          // [n][nh], n * nh <= 64 + 2n
  float* s_big = s_w + 64 + 2 * kMaxPairs;                             // [nh]
  const float4* stage = reinterpret_cast<const float4*>(smem);
  for (int q = L; q < n; q += 128) s_slot[q] = (uint32_t)pair_slot(tm, pf + q, bb);
  if (L == 0) {
    const uint64_t t0 = ptx::globaltimer();
    uint32_t ok = 1u;
    while (ptx::ld_acquire_gpu(arrive) < (uint32_t)n) {
      if (aborted(c)) {
        ok = 0u;
        break;
      }
      if (ptx::globaltimer() - t0 > kTimeoutNs) {
        raise_abort(c, kErrMerge);
        ok = 0u;
        break;
      }
      __nanosleep(32);
    }
    *flag = ok;
  }
  if (!sync4()) return false;
  if (*flag == 0u) return false;
  if (L == 0) {
    // every piece's share in flight at once (bulk copies, one per piece)
    ptx::fence_proxy_async_all();
    ptx::mbar_arrive_expect_tx(mbar, (uint32_t)n * chunk);
    const uint32_t dst = ptx::smem_u32(smem);
    for (int q = 0; q < n; ++q)
      ptx::bulk_load(dst + (uint32_t)q * chunk,
                     p.part_o + ((size_t)s_slot[q] * kHeads + 64 * rank) * kDim + (size_t)o0 * 4, chunk, mbar);
  }
  // meanwhile: LSEs of this CTA's heads, then per head (one warp each, lanes over the
  // pieces) the merged LSE and the pieces' weights, in place
  for (int i = L; i < n * nh; i += 128) {
    const int q = i / nh, hi = i - q * nh;
    s_w[i] = __ldcg(p.part_lse + (size_t)s_slot[q] * kHeads + 64 * rank + h_lo + hi);
  }
  if (!sync4()) return false;
  for (int hi = L >> 5; hi < nh; hi += 4) {
    float mx = -INFINITY;
    for (int q = lane; q < n; q += 32) mx = fmaxf(mx, s_w[q * nh + hi]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.f;
    for (int q = lane; q < n; q += 32) sum += exp2f((s_w[q * nh + hi] - mx) * kLog2e);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float big = mx + logf(sum);
    for (int q = lane; q < n; q += 32) s_w[q * nh + hi] = exp2f((s_w[q * nh + hi] - big) * kLog2e);
    if (lane == 0) s_big[hi] = big;
  }
  if (!sync4()) return false;
  if (!wait_bar(c, mbar, mph & 1u, kErrMerge)) return false;
  ++mph;
  const int oseq = vseq_seq(p, bb), h0 = vseq_head0(p, bb);
  const int per = (int)(chunk / 16u);
  for (int i = L; i < o1 - o0; i += 128) {
    const int o = o0 + i, hr = o / (kDim / 4), col = 4 * (o % (kDim / 4));
    const float* wq = s_w + (hr - h_lo);
    // four independent sums over the pieces (no chain of dependent adds)
    float4 a[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) a[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    int q = 0;
    for (; q + 4 <= n; q += 4) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float w = wq[(q + r) * nh];
        const float4 v = stage[(q + r) * per + i];
        a[r].x = fmaf(w, v.x, a[r].x);
        a[r].y = fmaf(w, v.y, a[r].y);
        a[r].z = fmaf(w, v.z, a[r].z);
        a[r].w = fmaf(w, v.w, a[r].w);
      }
    }
    for (; q < n; ++q) {
      const float w = wq[q * nh];
      const float4 v = stage[q * per + i];
      a[0].x = fmaf(w, v.x, a[0].x);
      a[0].y = fmaf(w, v.y, a[0].y);
      a[0].z = fmaf(w, v.z, a[0].z);
      a[0].w = fmaf(w, v.w, a[0].w);
    }
    const float4 acc = make_float4((a[0].x + a[1].x) + (a[2].x + a[3].x), (a[0].y + a[1].y) + (a[2].y + a[3].y),
                                   (a[0].z + a[1].z) + (a[2].z + a[3].z), (a[0].w + a[1].w) + (a[2].w + a[3].w));
    const int hglob = h0 + 64 * (int)rank + hr;
    if (hglob < p.heads) {
      const size_t orow = (size_t)oseq * p.heads + hglob;
      if (p.out_f32)
        *reinterpret_cast<float4*>(static_cast<float*>(p.out) + orow * kDim + col) = acc;
      else
        *reinterpret_cast<uint2*>(static_cast<Out*>(p.out) + orow * kDim + col) =
            make_uint2(pack2<Out>(acc.x, acc.y), pack2<Out>(acc.z, acc.w));
      if (col == 0 && p.lse_out != nullptr) p.lse_out[orow] = s_big[hr - h_lo];
    }
  }
  // every CTA of the rank counts itself done; the last one resets both counters for
  // the next call (all others are past their waits by then)
  if (!sync4()) return false;
  if (L == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) + 1u == (uint32_t)n) {
      atomicExch(arrive, 0u);
      atomicExch(done, 0u);
    }
  }
  return true;
}

template <typename T>
__device__ __forceinline__ void softmax_epilogue(const Params& p, const Ctx& c, uint32_t rank, int pair,
                                                 uint8_t* smem, uint32_t tmem, Barriers* bars, int wq,
                                                 int lane) {
  using S = Smem<T>;
  using Out = typename Io<T>::Out;   // type of out (and of q)
  using PT = typename Cfg<T>::PT;    // type of the P operand
  constexpr bool kK8 = Io<T>::kKv8;
  const int L = wq * 32 + lane;
  const int m = L & 63;
  const int hf = L >> 6;
  const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
  float* xmax = reinterpret_cast<float*>(smem + S::kXmax);
  float* xl = reinterpret_cast<float*>(smem + S::kXl);
  volatile uint32_t* merge_flag = reinterpret_cast<volatile uint32_t*>(smem + S::kMisc + 8);
  // epilogue staging: the P buffers, idle between pieces; kSB boxes of 8 KB per
  // round, kHB of them from each lane half
  uint8_t* stage = smem + S::kP;
  constexpr int kSB = 2 * S::kPBuf / kChunkBytes;
  constexpr int kHB = kSB / 2;
  const uint32_t stage_u32 = ptx::smem_u32(stage);
  const uint32_t s_full0 = ptx::smem_u32(&bars->s_full[0]);
  const uint32_t xchg0 = ptx::smem_u32(&bars->xchg[0]);
  const uint32_t o_done0 = ptx::smem_u32(&bars->o_done[0]);
  const uint32_t lx = ptx::smem_u32(&bars->lx);
  const uint32_t stg = ptx::smem_u32(&bars->stg);
  const uint32_t stg2 = ptx::smem_u32(&bars->stg2);
  const uint32_t qts = ptx::smem_u32(&bars->qts);
  const uint32_t qtr = ptx::smem_u32(&bars->qtr);
  const uint32_t mload = ptx::smem_u32(&bars->mload);
  const uint32_t mdone = ptx::smem_u32(&bars->mdone);
  const uint32_t qt_full_leader = ptx::mapa(ptx::smem_u32(&bars->qt_full), 0);
  const uint32_t s_free0_leader = ptx::mapa(ptx::smem_u32(&bars->s_free[0]), 0);
  const uint32_t p_full0_leader = ptx::mapa(ptx::smem_u32(&bars->p_full[0]), 0);
  const uint32_t o_free_leader = ptx::mapa(ptx::smem_u32(&bars->o_free), 0);
  float sl2 = p.sl2;       // FP8: per piece, times this row's s / a
  float qinv_next = 1.f;   // FP8: s / a of the piece whose Q was quantized last
  uint32_t gi = 0;
  uint32_t n_lx = 0, n_stg = 0, n_stg2 = 0, n_stage = 0, n_done = 0;   // barrier phases

  // all four softmax warps meet at `bar` (count 4)
  auto sync4 = [&](uint32_t bar, uint32_t& ph) -> bool {
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive_local(bar);
    const bool ok = wait_bar(c, bar, ph & 1u, kErrSoftmax);
    ++ph;
    return ok;
  };
  // thread L == 0 has done something the others must wait for (stg2, count 1)
  auto wait_leader = [&]() -> bool {
    if (L == 0) ptx::mbar_arrive_local(stg2);
    const bool ok = wait_bar(c, stg2, n_stg2 & 1u, kErrSoftmax);
    ++n_stg2;
    return ok;
  };
  // Q dims [0, 256) of piece `k` (virtual sequence bb), staged by the Q loader,
  // into TMEM.  FP8: the whole quantized Q of the piece, from global memory.
  auto take_qt = [&](int k, int bb) -> bool {
    if constexpr (kK8) {
      qinv_next = quantize_q<Out>(p, bb, rank, m, hf, smem + S::kQ, tmem, lane_off);
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(qt_full_leader);
      return true;
    }
    if (!wait_bar(c, qts, (uint32_t)k & 1u, kErrSoftmax)) return false;
    copy_qt(smem + (k == 0 ? S::kP : S::kQ), m, tmem, lane_off);
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      ptx::mbar_arrive_local(qtr);
      ptx::mbar_arrive_cluster(qt_full_leader);
    }
    return true;
  };
  // stage O (TMEM) x scale as the output rows of this CTA's heads and store them
  // with TMA; output chunk co = (nh, bx) of a thread is dims 256 nh + 128 hf + 64 bx
  // stage O (TMEM) x scale as float32 rows and store them with TMA to rows
  // [y, y + 64) of `map`; fp32 chunk ci = (nh, k) of a thread is dims
  // 256 nh + 128 hf + 32 k
  auto store_rows_f32 = [&](const CUtensorMap* map, int y, int z, float scale) -> bool {
#pragma unroll 1
    for (int r = 0; r < 8 / kHB; ++r) {
#pragma unroll 1
      for (int i = 0; i < kHB; ++i) {
        const int ci = r * kHB + i;
        uint32_t o[32];
        ptx::tmem_ld32(tmem + lane_off + kColO + 32 * ci, o);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * scale);
        st_box_row(stage + (hf * kHB + i) * kChunkBytes, m, o);
      }
      ptx::fence_proxy_async_smem();
      if (!sync4(stg, n_stg)) return false;
      if (L == 0) {
        for (int sb = 0; sb < kSB; ++sb) {
          const int ci = r * kHB + sb % kHB;
          const int x = 256 * (ci >> 2) + 128 * (sb / kHB) + 32 * (ci & 3);
          if (z < 0)
            ptx::tma_store_2d(map, stage_u32 + sb * kChunkBytes, x, y);
          else
            ptx::tma_store_3d(map, stage_u32 + sb * kChunkBytes, x, y, z);
        }
        ptx::bulk_commit();
        ptx::bulk_wait_read();
      }
      if (!wait_leader()) return false;
    }
    return true;
  };
  auto write_out = [&](int bb, float scale) -> bool {
    const int oseq = vseq_seq(p, bb), orow = vseq_head0(p, bb) + 64 * (int)rank;
    if (p.out_f32) return store_rows_f32(&p.tm_out, orow, oseq, scale);
#pragma unroll 1
    for (int r = 0; r < 4 / kHB; ++r) {
#pragma unroll 1
      for (int i = 0; i < kHB; ++i) {
        const int co = r * kHB + i;
        uint32_t a[32], b2[32], w[32];
        ptx::tmem_ld32(tmem + lane_off + kColO + 64 * co, a);
        ptx::tmem_ld32(tmem + lane_off + kColO + 64 * co + 32, b2);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          w[k] = pack2<Out>(__uint_as_float(a[2 * k]) * scale, __uint_as_float(a[2 * k + 1]) * scale);
          w[16 + k] = pack2<Out>(__uint_as_float(b2[2 * k]) * scale, __uint_as_float(b2[2 * k + 1]) * scale);
        }
        st_box_row(stage + (hf * kHB + i) * kChunkBytes, m, w);
      }
      ptx::fence_proxy_async_smem();
      if (!sync4(stg, n_stg)) return false;
      if (L == 0) {
        for (int sb = 0; sb < kSB; ++sb) {
          const int co = r * kHB + sb % kHB;
          const int x = 256 * (co >> 1) + 128 * (sb / kHB) + 64 * (co & 1);
          ptx::tma_store_3d(&p.tm_out, stage_u32 + sb * kChunkBytes, x, orow, oseq);
        }
        ptx::bulk_commit();
        ptx::bulk_wait_read();
      }
      if (!wait_leader()) return false;
    }
    return true;
  };

  PieceIter it(p, pair);
  const TileMap& tm = it.m;
  Piece pc;
  int piece = 0;
  // sequences split between more than fuse_max pairs that this pair has a piece of
  // (at most its first and its last piece), merged at the end in a cooperative launch
  int n_wide = 0, wide_bb[2] = {0, 0}, wide_pf[2] = {0, 0}, wide_pl[2] = {0, 0};
  bool have = it.next(&pc);
  if (have && !take_qt(0, pc.bb)) return;
  while (have) {
    PieceIter peek = it;
    Piece nxt;
    const bool has_next = peek.next(&nxt);
    const int slen = seq_len(p, pc.bb);
    if constexpr (kK8) sl2 = p.sl2 * qinv_next;   // this piece's scores are (a / s) x true
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
      const int nvalid = slen - (j * kTile + 64 * hf);
      if (nvalid < 64) {
#pragma unroll
        for (int k = 0; k < 64; ++k)
          if (k >= nvalid) v[k] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = v[k];
#pragma unroll
      for (int k = 8; k < 64; ++k) mx8[k & 7] = fmaxf(mx8[k & 7], v[k]);
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // the two lane halves of a row hold its two 64-token halves: exchange maxima
      xmax[b * 128 + L] = mx;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_local(xchg0 + 8 * b);
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
        phi[k] = pack2<PT>(a, b2);
        if constexpr (Cfg<T>::kPParts == 2) {
          const float ah = __uint_as_float(phi[k] << 16);
          const float bh = __uint_as_float(phi[k] & 0xffff0000u);
          plo[k] = pack2<PT>(a - ah, b2 - bh);
        }
      }
      l += ls;
      // P buffer b was last read by P.V of tile gi - 2
      if (gi >= 2 && !wait_bar(c, o_done0 + 8 * b, ((gi - 2) >> 1) & 1u, kErrSoftmax)) return;
      if (j > pc.first && __any_sync(0xffffffffu, rescale)) {
        // rare: O must be rescaled, after P.V of the previous tile has landed in it
        if (!wait_bar(c, o_done0 + 8 * (b ^ 1u), ((gi - 1) >> 1) & 1u, kErrSoftmax)) return;
        ptx::tc_fence_after();
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
      // P row m of token half hf, SWIZZLE_128B: 16-byte granule g at g ^ (m & 7)
      uint8_t* prow = smem + S::kP + b * S::kPBuf + hf * kChunkBytes + m * 128;
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
      if (lane == 0) ptx::mbar_arrive_cluster(p_full0_leader + 8 * b);
      // this piece's QK^T is complete (its last S was read): the next piece's Q goes to TMEM
      if (j == pc.end - 1 && has_next && !take_qt(piece + 1, nxt.bb)) return;
    }

    // ---- epilogue of this piece: wait for P.V of its last tile
    if (!wait_bar(c, o_done0 + 8 * ((gi - 1) & 1u), ((gi - 1) >> 1) & 1u, kErrSoftmax)) return;
    ptx::tc_fence_after();
    int pf = 0, pl = 0;
    if (!pc.full) pairs_of_sequence(tm, pc.bb, &pf, &pl);
    uint32_t* cnt = p.counters + 4 * pc.bb + rank;
    const uint32_t npieces = (uint32_t)(pl - pf + 1);
    // sequences split between more pairs are left to the combine launch
    const bool fuse = npieces <= (uint32_t)p.fuse_max;
    xl[L] = l;
    // a split sequence whose other pieces are all counted already is completed by this CTA
    if (!pc.full && fuse && L == 0)
      *merge_flag = (ptx::ld_acquire_gpu(cnt) + 1u == npieces) ? 1u : 0u;
    if (!sync4(lx, n_lx)) return;
    const float ltot = l + xl[L ^ 64];
    const float inv = (kK8 ? p.kv_scale : 1.f) / ltot;   // FP8: V's scale, folded here
    const float lse = (m_run * sl2 + log2f(ltot)) * kLn2;
    const int head = 64 * (int)rank + m;                   // row within the head group
    const int hglob = vseq_head0(p, pc.bb) + head;         // head within the sequence
    const size_t orow_g = (size_t)vseq_seq(p, pc.bb) * p.heads + hglob;
    const bool real = hglob < p.heads;
    bool merge = false;
    if (!pc.full) {
      merge = fuse && *merge_flag != 0u;
      if (!merge) {
        // Publish this piece (normalised O in fp32 and its LSE) for the CTA that
        // completes the sequence: the LSE combine of mla_decode.py:212-246, fused
        // into this kernel (no second launch; nobody waits on another CTA).
        const int slot = 2 * pair + (piece == 0 ? 0 : 1);
        if (hf == 0) p.part_lse[(size_t)slot * kHeads + head] = lse;
        if (!store_rows_f32(&p.tm_part, slot * kHeads + 64 * (int)rank, -1, inv)) return;
        if (fuse) {
          // the LSE stores of every thread are ordered before the count below
          __threadfence();
          if (!sync4(stg, n_stg)) return;
          if (L == 0) {
            ptx::bulk_wait();
            ptx::fence_proxy_async_all();
            __threadfence();
            const uint32_t done = atomicAdd(cnt, 1u) + 1u;
            const bool last = done == npieces;
            if (last) atomicExch(cnt, 0u);   // ready for the next call
            *merge_flag = last ? 1u : 0u;
          }
          if (!wait_leader()) return;
          merge = *merge_flag != 0u;
        } else if (p.coop) {
          // split between many pairs: counted here, merged by all of them together
          // once every piece is published (after each pair's last piece, below)
          __threadfence();
          if (!sync4(stg, n_stg)) return;
          if (L == 0) {
            ptx::bulk_wait();
            ptx::fence_proxy_async_all();
            __threadfence();
            atomicAdd(cnt, 1u);
          }
          if (n_wide < 2) {
            wide_bb[n_wide] = pc.bb;
            wide_pf[n_wide] = pf;
            wide_pl[n_wide] = pl;
            ++n_wide;
          }
        }
        // else: a combine launch after this kernel merges the sequence
      } else if (L == 0) {
        atomicExch(cnt, 0u);   // every other piece was counted: reset for the next call
      }
    }
    if (!merge) {
      if (pc.full) {
        if (!write_out(pc.bb, inv)) return;
        if (hf == 0 && real && p.lse_out != nullptr) p.lse_out[orow_g] = lse;
      }
    } else {
      // this CTA completes a split sequence: merge every piece into `out`
      __threadfence();
      const int own = pair;
      float mx = lse;
      for (int pp = pf; pp <= pl; ++pp)
        if (pp != own)
          mx = fmaxf(mx, __ldcg(p.part_lse + pair_slot(tm, pp, pc.bb) *
                                                kHeads + head));
      float sum = exp2f((lse - mx) * kLog2e);
      for (int pp = pf; pp <= pl; ++pp)
        if (pp != own)
          sum += exp2f((__ldcg(p.part_lse + pair_slot(tm, pp, pc.bb) *
                                               kHeads + head) - mx) * kLog2e);
      const float big = mx + logf(sum);
      if (!has_next) {
        // Last piece of this pair: the rings and the Q/P buffers are idle.  O of
        // this piece is still in TMEM: scale it by its merge weight, then add each
        // other piece, staged row by row in shared memory (padded rows: threads
        // reading one column of 32 rows hit distinct banks).
        const float w_own = exp2f((lse - big) * kLog2e) * inv;
#pragma unroll 1
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t o[32];
          ptx::tmem_ld32(tmem + lane_off + kColO + 32 * cc, o);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * w_own);
          ptx::tmem_st32(tmem + lane_off + kColO + 32 * cc, o);
        }
        ptx::tmem_wait_st();
        const uint32_t mstage = ptx::smem_u32(smem);
        for (int pp = pf; pp <= pl; ++pp) {
          if (pp == own) continue;
          const size_t sl = pair_slot(tm, pp, pc.bb);
          const float w = exp2f((__ldcg(p.part_lse + sl * kHeads + head) - big) * kLog2e);
          if (L == 0) {
            ptx::fence_proxy_async_all();
            ptx::mbar_arrive_expect_tx(mload, 64 * kDim * 4);
            const float* src = p.part_o + (sl * kHeads + 64 * rank) * kDim;
            for (int r = 0; r < 64; ++r)
              ptx::bulk_load(mstage + r * kMergePitch, src + (size_t)r * kDim, kDim * 4, mload);
          }
          if (!wait_bar(c, mload, n_stage & 1u, kErrSoftmax)) return;
          ++n_stage;
          const float* srow = reinterpret_cast<const float*>(smem + m * kMergePitch);
#pragma unroll 1
          for (int cc = 0; cc < 8; ++cc) {
            const int d0 = 256 * (cc >> 2) + 128 * hf + 32 * (cc & 3);
            uint32_t o[32];
            ptx::tmem_ld32(tmem + lane_off + kColO + 32 * cc, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              const float4 x = *reinterpret_cast<const float4*>(srow + d0 + 4 * g);
              o[4 * g] = __float_as_uint(fmaf(w, x.x, __uint_as_float(o[4 * g])));
              o[4 * g + 1] = __float_as_uint(fmaf(w, x.y, __uint_as_float(o[4 * g + 1])));
              o[4 * g + 2] = __float_as_uint(fmaf(w, x.z, __uint_as_float(o[4 * g + 2])));
              o[4 * g + 3] = __float_as_uint(fmaf(w, x.w, __uint_as_float(o[4 * g + 3])));
            }
            ptx::tmem_st32(tmem + lane_off + kColO + 32 * cc, o);
          }
          ptx::tmem_wait_st();
          // everyone is done reading the stage before it is refilled or reused
          if (!sync4(mdone, n_done)) return;
        }
        if (!write_out(pc.bb, 1.f)) return;
      } else {
        // rare (the pair's range goes on: the shared memory is busy): merge from
        // global memory, row by row in registers
        const size_t orow = orow_g * kDim;
#pragma unroll 1
        for (int cc = 0; cc < 8; ++cc) {
          const int d0 = 256 * (cc >> 2) + 128 * hf + 32 * (cc & 3);
          uint32_t o[32];
          ptx::tmem_ld32(tmem + lane_off + kColO + 32 * cc, o);
          ptx::tmem_wait_ld();
          const float w_own = exp2f((lse - big) * kLog2e) * inv;
          float acc[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) acc[k] = __uint_as_float(o[k]) * w_own;
          for (int pp = pf; pp <= pl; ++pp) {
            if (pp == own) continue;
            const size_t sl = pair_slot(tm, pp, pc.bb);
            const float w = exp2f((__ldcg(p.part_lse + sl * kHeads + head) - big) * kLog2e);
            const float4* src = reinterpret_cast<const float4*>(p.part_o + (sl * kHeads + head) * kDim + d0);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              const float4 x = __ldcg(src + g);
              acc[4 * g] = fmaf(w, x.x, acc[4 * g]);
              acc[4 * g + 1] = fmaf(w, x.y, acc[4 * g + 1]);
              acc[4 * g + 2] = fmaf(w, x.z, acc[4 * g + 2]);
              acc[4 * g + 3] = fmaf(w, x.w, acc[4 * g + 3]);
            }
          }
          if (!real) {
            // a head past h in the last head group: computed, not stored
          } else if (p.out_f32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + orow + d0);
#pragma unroll
            for (int g = 0; g < 8; ++g)
              dst[g] = make_float4(acc[4 * g], acc[4 * g + 1], acc[4 * g + 2], acc[4 * g + 3]);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<Out*>(p.out) + orow + d0);
#pragma unroll
            for (int g = 0; g < 4; ++g)
              dst[g] = make_uint4(pack2<Out>(acc[8 * g], acc[8 * g + 1]), pack2<Out>(acc[8 * g + 2], acc[8 * g + 3]),
                                  pack2<Out>(acc[8 * g + 4], acc[8 * g + 5]),
                                  pack2<Out>(acc[8 * g + 6], acc[8 * g + 7]));
          }
        }
      }
      if (hf == 0 && real && p.lse_out != nullptr) p.lse_out[orow_g] = big;
    }
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive_cluster(o_free_leader);
    ++piece;
    it = peek;
    pc = nxt;
    have = has_next;
  }

  // ---- cooperative merge of the sequences split between many pairs (p.coop only):
  // out of line, so that its load streams do not weigh on the registers of the
  // per-tile loop above
  for (int w = 0; w < n_wide; ++w)
    if (!coop_merge<Out>(p, c, tm, rank, pair, smem, lx, n_lx, mload, n_stage, merge_flag, L, lane, wide_bb[w],
                         wide_pf[w], wide_pl[w]))
      return;
}

// ---------------------------------------------------------------------------
// the kernel: warp 0 K producer, warp 1 TMEM owner + QK^T issuer, warp 2 V
// producer, warp 3 P.V issuer, warps 4..7 softmax/epilogue, warp 8 Q loader
// (warps 9..11 complete the third warpgroup).  For an FP8 cache the block has
// 16 warps: warp 2 also prefetches Q, and warps 8..15 convert V to fp16.  The
// Cv variant has 16 warps too: warps 12..15 rewrite each landed V stage (tail
// rows zeroed, bf16 -> fp16 with kF16); warps 9..11 are idle.  In the plain
// variants warp 9 zeroes the tail rows of a sequence's last V units.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_of<T>(), 1)
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
    // V operand stages: one expect-tx arrival (TMA), or FP8: kConvWarps converter warps x 2 CTAs
    const uint32_t n_vfull = Io<T>::kKv8 ? 2u * kConvWarps : (Io<T>::kConv ? 2u * kFixWarps : 1u);
    for (int s = 0; s < 8; ++s) {
      ptx::mbar_init(ptx::smem_u32(&bars->kfull[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->kempty[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->vfull[s]), n_vfull);
      ptx::mbar_init(ptx::smem_u32(&bars->vempty[s]), 1);
    }
    for (int s = 0; s < 8; ++s) {
      ptx::mbar_init(ptx::smem_u32(&bars->v8full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->v8empty[s]), kConvWarps);
      ptx::mbar_init(ptx::smem_u32(&bars->vfix[s]), 2);
    }
    ptx::mbar_init(ptx::smem_u32(&bars->q_full), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->q_empty), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->qt_full), 8);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(ptx::smem_u32(&bars->s_full[b]), 1);
      ptx::mbar_init(ptx::smem_u32(&bars->s_free[b]), 8);
      ptx::mbar_init(ptx::smem_u32(&bars->xchg[b]), 4);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(ptx::smem_u32(&bars->p_full[b]), 8);
      ptx::mbar_init(ptx::smem_u32(&bars->o_done[b]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(&bars->o_free), 8);
    ptx::mbar_init(ptx::smem_u32(&bars->lx), 4);
    ptx::mbar_init(ptx::smem_u32(&bars->stg), 4);
    ptx::mbar_init(ptx::smem_u32(&bars->stg2), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->qts), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->qtr), 4);
    ptx::mbar_init(ptx::smem_u32(&bars->q_go), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->mload), 1);
    ptx::mbar_init(ptx::smem_u32(&bars->mdone), 4);
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
    ptx::prefetch_tensormap(&p.tm_out);
    if (p.part_o != nullptr) ptx::prefetch_tensormap(&p.tm_part);
  }
  if (warp == 1) ptx::tmem_alloc_pair(ptx::smem_u32(tmem_slot), kTmemCols);
  ptx::tc_fence_before();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // a combine launch queued behind this grid may be set up now (it waits for this
  // grid's completion before it reads anything)
  if (threadIdx.x == 0) ptx::grid_dep_launch();
  // clock probe: SM cycles and %globaltimer ns of this CTA's run (thread 0 of CTA 0)
  const bool probe = blockIdx.x == 0 && threadIdx.x == 0 && p.status != nullptr;
  const uint64_t probe_c0 = probe ? (uint64_t)clock64() : 0ull;
  const uint64_t probe_t0 = probe ? ptx::globaltimer() : 0ull;

  Ctx c;
  c.abort_local = abort_flag;
  c.abort_peer = ptx::mapa(ptx::smem_u32(abort_flag), rank ^ 1u);
  c.status = p.status;

  // One role per warp: a lane blocked in mbarrier.try_wait holds back every
  // other lane of its warp.  Warpgroup 1 (warps 4..7) runs the softmax.
  if ((warp >> 2) == 1) {
    ptx::setmaxnreg_inc<kRegsSoftmax>();
    softmax_epilogue<T>(p, c, rank, pair, smem, tmem, bars, warp & 3, lane);
    ptx::setmaxnreg_dec<kRegsLow>();   // same budget as the other warps from here on
  } else {
    ptx::setmaxnreg_dec<kRegsLow>();
  if (warp == 0) {
    if (lane == 0) k_producer<T>(p, c, rank, pair, sbase, bars);
  } else if (warp == 8 && !Io<T>::kKv8) {
    if (lane == 0) q_loader<T>(p, c, rank, pair, sbase, bars);
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      qk_issuer<T>(p, c, pair, sbase, tmem, bars);
      // every tcgen05 op this thread issued has completed once this commit lands
      ptx::mma_commit_pair_mc(ptx::smem_u32(&bars->drain_qk), 0x1);
      wait_bar(c, ptx::smem_u32(&bars->drain_qk), 0u, kErrDrain);
    }
  } else if (warp == 2) {
    // (FP8: the Q loader only prefetches and never waits; it runs here first)
    if (Io<T>::kKv8 && lane == 0) q_loader<T>(p, c, rank, pair, sbase, bars);
    if (lane == 0) v_producer<T>(p, c, rank, pair, sbase, bars);
  } else if (warp == 3) {
    if (rank == 0 && lane == 0) {
      pv_issuer<T>(p, c, pair, sbase, tmem, bars);
      ptx::mma_commit_pair_mc(ptx::smem_u32(&bars->drain_pv), 0x1);
      wait_bar(c, ptx::smem_u32(&bars->drain_pv), 0u, kErrDrain);
    }
  } else if (Io<T>::kKv8 && warp >= 8) {
    // FP8: warps 8..15 dequantize the V units
    v_converter<T>(p, c, pair, smem, bars, (warp - 8) * 32 + lane, lane);
  } else if (warp == 9 && !Io<T>::kKv8 && !Io<T>::kConv) {
    v_tailfix<T>(p, c, rank, pair, smem, bars, lane);
  } else if (warp >= 12) {
    if constexpr (Io<T>::kConv) v_fix<T>(p, c, pair, smem, bars, (warp - 12) * 32 + lane, lane);
  }
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
  if (probe) {
    // accumulated over calls in the workspace's status block (words 1..3 after the
    // status word): cycles / ns is the SM clock the kernel actually ran at
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(p.status) + kProbeWord;
    atomicAdd(acc, (unsigned long long)((uint64_t)clock64() - probe_c0));
    atomicAdd(acc + 1, (unsigned long long)(ptx::globaltimer() - probe_t0));
    atomicAdd(acc + 2, 1ull);
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, kTmemCols);
    ptx::tmem_relinquish_pair();
  }
}

// ---------------------------------------------------------------------------
// Self-test of the timeout path (faults nothing, hangs nothing): in one CTA pair
// each CTA's thread 0 waits, through wait_bar_slow, on an mbarrier of its own that
// nothing ever arrives on.  CTA 0 gives up after limit_ns and takes the path every
// role of the decode kernel takes on a timeout: abort flags raised in both CTAs,
// `code` recorded in the status word.  CTA 1 waits with 100 x the limit and must
// leave early through the abort flag its peer raised.  result[2 r] = 1 when CTA
// r's wait returned false, result[2 r + 1] = how long it waited (ns).
// ---------------------------------------------------------------------------
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(32, 1)
mla_wait_selftest_kernel(uint32_t* status, unsigned long long* result, uint64_t limit_ns, uint32_t code) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t abort_flag;
  const uint32_t rank = ptx::cluster_ctarank();
  const uint32_t bar_addr = ptx::smem_u32(&bar);
  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_addr, 1);
    abort_flag = 0u;
    ptx::fence_mbarrier_init();
  }
  ptx::cluster_sync();
  Ctx c;
  c.abort_local = &abort_flag;
  c.abort_peer = ptx::mapa(ptx::smem_u32(&abort_flag), rank ^ 1u);
  c.status = status;
  if (threadIdx.x == 0) {
    const uint64_t t0 = ptx::globaltimer();
    const bool ok = wait_bar_slow(c, bar_addr, 0u, code, rank == 0 ? limit_ns : 100 * limit_ns);
    result[2 * rank] = ok ? 0ull : 1ull;
    result[2 * rank + 1] = (unsigned long long)(ptx::globaltimer() - t0);
  }
  // the peer's abort flag is written through the cluster window: both CTAs stay
  // resident until both have finished
  ptx::cluster_sync();
}

// ---------------------------------------------------------------------------
// combine launch for sequences split between more pairs than the kernel above
// merges itself (fuse_max): one CTA per (head, sequence) of kCombineGroups groups of
// 128 threads; group g takes every kCombineGroups-th piece and thread t columns
// [4t, 4t + 4).  Latency, not bandwidth, bounds it (a few MB, just written, in L2):
// every thread issues the loads of all its pieces (up to kCombinePer) at once,
// before it needs the LSEs, so that one round trip covers the whole merge; the
// groups' sums meet in shared memory.  Launched as a programmatic dependent of the
// decode kernel: the grid is set up while the decode kernel runs, and waits for its
// completion before the first load.  Sequences the decode kernel wrote itself are
// skipped.  Same LSE algebra as mla_combine.cu (mla_decode.py:212-246).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store4_out(float* dst, float4 v) { *reinterpret_cast<float4*>(dst) = v; }
template <typename T>
__device__ __forceinline__ void store4_out(T* dst, float4 v) {
  *reinterpret_cast<uint2*>(dst) = make_uint2(pack2<T>(v.x, v.y), pack2<T>(v.z, v.w));
}

constexpr int kCombineGroups = 4;
constexpr int kCombinePer = 20;   // pieces per thread and round: 80 per round (B200: at most 74)

template <typename OutT>
__global__ void __launch_bounds__(128 * kCombineGroups)
mla_pair_combine_kernel(const float* __restrict__ part_lse, const float* __restrict__ part_o,
                        OutT* __restrict__ out, float* __restrict__ lse_out, const uint32_t* cu,
                        uint32_t total_fixed, int nt, int pairs, int vbatch, int heads, int hgroups,
                        int fuse_max) {
  constexpr int G = kCombineGroups;
  __shared__ float s_lse[kMaxPairs];
  __shared__ float4 s_acc[G - 1][128];
  const int head = blockIdx.x, bb = blockIdx.y;
  const int grp = threadIdx.x >> 7, tid = threadIdx.x & 127;   // piece group, column quad
  ptx::grid_dep_wait();   // the decode kernel's partials are complete and visible
  TileMap m;
  m.cu = cu;
  m.nt = (uint32_t)nt;
  m.batch = vbatch;
  m.total = cu != nullptr ? __ldg(cu + vbatch) : total_fixed;
  m.pairs = effective_pairs((uint32_t)pairs, m.total);
  if (m.first(bb) == m.first(bb + 1)) return;   // empty sequence (written by the plan kernel)
  int pf, pl;
  pairs_of_sequence(m, bb, &pf, &pl);
  const int n = pl - pf + 1;
  if (n <= fuse_max) return;   // whole, or merged by the decode kernel
  // piece k's slot (pair_slot without a division per piece): every pair after the
  // first starts its range inside the sequence, so the piece is that pair's first
  const size_t slot0 = pair_slot(m, pf, bb);
  auto slot = [&](int k) -> size_t { return k == 0 ? slot0 : (size_t)(pf + k) * 2; };
  const float4* po = reinterpret_cast<const float4*>(part_o) + (size_t)head * (kDim / 4) + tid;
  constexpr size_t kSlotQuads = (size_t)kHeads * kDim / 4;   // float4 per slot
  // first round of O loads in flight before anything waits
  float4 v[kCombinePer];
#pragma unroll
  for (int u = 0; u < kCombinePer; ++u) {
    const int k = grp + G * u;
    v[u] = k < n ? __ldcg(po + slot(k) * kSlotQuads) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int k = threadIdx.x; k < n; k += 128 * G) s_lse[k] = __ldcg(part_lse + slot(k) * kHeads + head);
  __syncthreads();
  // the sequence's LSE: every warp reduces the n piece LSEs itself (lanes over pieces)
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
  for (int k = lane; k < n; k += 32) mx = fmaxf(mx, s_lse[k]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  if (mx != -INFINITY)
    for (int k = lane; k < n; k += 32) sum += exp2f((s_lse[k] - mx) * kLog2e);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float lse = mx != -INFINITY ? mx + logf(sum) : -INFINITY;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k0 = 0;; k0 += G * kCombinePer) {
#pragma unroll
    for (int u = 0; u < kCombinePer; ++u) {
      const int k = k0 + grp + G * u;
      if (k >= n) break;
      const float w = lse != -INFINITY ? exp2f((s_lse[k] - lse) * kLog2e) : 0.f;
      acc.x = fmaf(w, v[u].x, acc.x);
      acc.y = fmaf(w, v[u].y, acc.y);
      acc.z = fmaf(w, v[u].z, acc.z);
      acc.w = fmaf(w, v[u].w, acc.w);
    }
    const int k1 = k0 + G * kCombinePer;
    if (k1 >= n) break;
    // more pieces than one round holds (more pairs than a B200 has)
#pragma unroll
    for (int u = 0; u < kCombinePer; ++u) {
      const int k = k1 + grp + G * u;
      v[u] = k < n ? __ldcg(po + slot(k) * kSlotQuads) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (grp > 0) s_acc[grp - 1][tid] = acc;
  __syncthreads();
  if (grp > 0) return;
#pragma unroll
  for (int g2 = 0; g2 < G - 1; ++g2) {
    const float4 o = s_acc[g2][tid];
    acc.x += o.x;
    acc.y += o.y;
    acc.z += o.z;
    acc.w += o.w;
  }
  const int hglob = (bb % hgroups) * kHeads + head;
  if (hglob >= heads) return;   // a head past h in the last head group
  const size_t orow = (size_t)(bb / hgroups) * heads + hglob;
  store4_out(out + orow * kDim + 4 * tid, acc);
  if (lse_out != nullptr && tid == 0) lse_out[orow] = lse;
}

// ---------------------------------------------------------------------------
// The sequence split's merge and exchange in one launch.  Every rank holds the
// float32 (O, LSE) of its own KV rows for every output row; the output is their
// LSE merge over the world ranks.  CTA i takes the rows i, i + G, ... (G CTAs, at
// most one per SM) in two passes.  Pass 1, per row: its local value (pieces mode:
// merged from the decode kernel's pieces as the combine launch above does when
// the sequence was split between more than fuse_max pairs; else the row the
// decode kernel or an earlier launch wrote to this rank's block) goes to this
// rank's block and, over NVLink, to this rank's row words in every peer's buffer:
// each 16-byte store carries two (value bits, call number) pairs, and a reader
// takes a pair as this call's value once it carries this call's number, so the
// writer needs no fence and no flag (the low-latency scheme NCCL's LL protocol
// uses).  Pass 2, per row: every thread polls its own words of each peer's row,
// with a time limit, until they carry this call's number, then merges the world
// rows into out / lse.  Pass 1 never waits, so no rank's stores depend on another
// rank's progress.  Row words alternate by call parity: a rank writes call k + 1
// only after its call k read every peer's call-k words, which each peer wrote
// after its own call k - 1 had read the words of parity k + 1.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_pairs(uint32_t* p, float a, float b, uint32_t tag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(__float_as_uint(a)), "r"(tag),
               "r"(__float_as_uint(b)), "r"(tag)
               : "memory");
}
__device__ __forceinline__ uint4 ld_pairs(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_pair(uint32_t* p, float a, uint32_t tag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(a)), "r"(tag) : "memory");
}
__device__ __forceinline__ uint2 ld_pair(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

template <typename OutT>
__global__ void __launch_bounds__(128 * kCombineGroups)
mla_seqsplit_combine_kernel(const float* __restrict__ part_lse, const float* __restrict__ part_o,
                            const uint32_t* cu, uint32_t total_fixed, int nt, int pairs, int vbatch, int heads,
                            int hgroups, int fuse_max, const __grid_constant__ PeerRows x, OutT* __restrict__ out,
                            float* __restrict__ lse_out) {
  constexpr int G = kCombineGroups;
  __shared__ float s_lse[kMaxPairs];
  __shared__ float4 s_acc[G - 1][128];
  const int grp = threadIdx.x >> 7, tid = threadIdx.x & 127, lane = threadIdx.x & 31;
  const bool pieces = fuse_max >= 0;
  ptx::grid_dep_wait();   // the decode kernel's pieces / rows are complete and visible
  TileMap m;
  m.cu = cu;
  m.nt = (uint32_t)nt;
  m.batch = vbatch;
  m.total = !pieces ? 0u : (cu != nullptr ? __ldg(cu + vbatch) : total_fixed);
  m.pairs = effective_pairs((uint32_t)pairs, m.total);
  const int rows = vbatch * kHeads;
  const size_t bh = (size_t)(vbatch / hgroups) * heads;   // output rows
  float* own = x.bufs[x.rank] + ((size_t)x.par * x.world + x.rank) * x.chunk;
  // rank q's row words and LSE words of this parity in buffer `buf`
  auto row_words = [&](float* buf, int q, size_t orow) -> uint32_t* {
    return reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(buf) + x.ll_rows) +
           (((size_t)x.par * x.world + q) * x.rows_pad + orow) * (2 * kDim);
  };
  auto lse_word = [&](float* buf, int q, size_t orow) -> uint32_t* {
    return reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(buf) + x.ll_lse) +
           (((size_t)x.par * x.world + q) * x.rows_pad + orow) * 2;
  };
  // ---- pass 1: this rank's value of each row, to its block and every peer's words
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int head = r % kHeads, bb = r / kHeads;
    const int hglob = (bb % hgroups) * kHeads + head;
    if (hglob >= heads) continue;   // a head past h in the last head group: no row
    const size_t orow = (size_t)(bb / hgroups) * heads + hglob;
    int n = 0, pf = 0, pl = -1;
    if (pieces && m.first(bb) != m.first(bb + 1)) {
      pairs_of_sequence(m, bb, &pf, &pl);
      n = pl - pf + 1;
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float lse = -INFINITY;
    if (pieces && n > fuse_max) {
      const size_t slot0 = pair_slot(m, pf, bb);
      auto slot = [&](int k) -> size_t { return k == 0 ? slot0 : (size_t)(pf + k) * 2; };
      const float4* po = reinterpret_cast<const float4*>(part_o) + (size_t)head * (kDim / 4) + tid;
      constexpr size_t kSlotQuads = (size_t)kHeads * kDim / 4;
      float4 v[kCombinePer];
#pragma unroll
      for (int u = 0; u < kCombinePer; ++u) {
        const int k = grp + G * u;
        v[u] = k < n ? __ldcg(po + slot(k) * kSlotQuads) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      for (int k = threadIdx.x; k < n; k += 128 * G) s_lse[k] = __ldcg(part_lse + slot(k) * kHeads + head);
      __syncthreads();
      float mx = -INFINITY;
      for (int k = lane; k < n; k += 32) mx = fmaxf(mx, s_lse[k]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sum = 0.f;
      if (mx != -INFINITY)
        for (int k = lane; k < n; k += 32) sum += exp2f((s_lse[k] - mx) * kLog2e);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      lse = mx != -INFINITY ? mx + logf(sum) : -INFINITY;
      for (int k0 = 0;; k0 += G * kCombinePer) {
#pragma unroll
        for (int u = 0; u < kCombinePer; ++u) {
          const int k = k0 + grp + G * u;
          if (k >= n) break;
          const float w = lse != -INFINITY ? exp2f((s_lse[k] - lse) * kLog2e) : 0.f;
          acc.x = fmaf(w, v[u].x, acc.x);
          acc.y = fmaf(w, v[u].y, acc.y);
          acc.z = fmaf(w, v[u].z, acc.z);
          acc.w = fmaf(w, v[u].w, acc.w);
        }
        const int k1 = k0 + G * kCombinePer;
        if (k1 >= n) break;
#pragma unroll
        for (int u = 0; u < kCombinePer; ++u) {
          const int k = k1 + grp + G * u;
          v[u] = k < n ? __ldcg(po + slot(k) * kSlotQuads) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      if (grp > 0) s_acc[grp - 1][tid] = acc;
      __syncthreads();
      if (grp == 0) {
#pragma unroll
        for (int g2 = 0; g2 < G - 1; ++g2) {
          const float4 o = s_acc[g2][tid];
          acc.x += o.x;
          acc.y += o.y;
          acc.z += o.z;
          acc.w += o.w;
        }
        reinterpret_cast<float4*>(own + orow * kDim)[tid] = acc;
        if (tid == 0) own[bh * kDim + orow] = lse;
      }
    } else if (grp == 0) {
      acc = __ldcg(reinterpret_cast<const float4*>(own + orow * kDim) + tid);
      lse = __ldcg(own + bh * kDim + orow);
    }
    if (grp == 0) {
      for (int q = 0; q < x.world; ++q) {
        if (q == x.rank) continue;
        uint32_t* w = row_words(x.bufs[q], x.rank, orow) + 8 * tid;
        st_pairs(w, acc.x, acc.y, x.epoch);
        st_pairs(w + 4, acc.z, acc.w, x.epoch);
        if (tid == 0) st_pair(lse_word(x.bufs[q], x.rank, orow), lse, x.epoch);
      }
    }
    __syncthreads();   // s_lse and s_acc are free for the next row
  }
  // ---- pass 2: every peer's value of each row (polled), then the merge
  if (grp != 0) return;
  uint32_t* status = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(x.bufs[x.rank]) + x.header) + 17;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int head = r % kHeads, bb = r / kHeads;
    const int hglob = (bb % hgroups) * kHeads + head;
    if (hglob >= heads) continue;
    const size_t orow = (size_t)(bb / hgroups) * heads + hglob;
    float lq[kSeqMaxWorld];
    float4 vq[kSeqMaxWorld];
    bool ok = true;
#pragma unroll
    for (int q = 0; q < kSeqMaxWorld; ++q) {
      lq[q] = -INFINITY;
      vq[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q >= x.world || !ok) continue;
      if (q == x.rank) {
        vq[q] = __ldcg(reinterpret_cast<const float4*>(own + orow * kDim) + tid);
        lq[q] = __ldcg(own + bh * kDim + orow);
        continue;
      }
      const uint32_t* w = row_words(x.bufs[x.rank], q, orow) + 8 * tid;
      const uint32_t* lw = lse_word(x.bufs[x.rank], q, orow);
      uint4 a = ld_pairs(w), b2 = ld_pairs(w + 4);
      uint2 l2 = ld_pair(lw);
      if (a.y != x.epoch || a.w != x.epoch || b2.y != x.epoch || b2.w != x.epoch || l2.y != x.epoch) {
        const uint64_t t0 = ptx::globaltimer();
        for (;;) {
          a = ld_pairs(w);
          b2 = ld_pairs(w + 4);
          l2 = ld_pair(lw);
          if (a.y == x.epoch && a.w == x.epoch && b2.y == x.epoch && b2.w == x.epoch && l2.y == x.epoch) break;
          // give up at the time limit, or at once when another thread already has
          if (*reinterpret_cast<volatile uint32_t*>(status) != 0u || ptx::globaltimer() - t0 > kSeqWaitNs) {
            atomicCAS(status, 0u, kErrExchange);   // a peer never delivered: the merge is invalid
            ok = false;
            break;
          }
          __nanosleep(32);
        }
      }
      vq[q] = make_float4(__uint_as_float(a.x), __uint_as_float(a.z), __uint_as_float(b2.x), __uint_as_float(b2.z));
      lq[q] = __uint_as_float(l2.x);
    }
    if (!ok) return;
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < kSeqMaxWorld; ++q) mx = fmaxf(mx, lq[q]);
    float sum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (mx != -INFINITY) {
#pragma unroll
      for (int q = 0; q < kSeqMaxWorld; ++q) {
        const float w = exp2f((lq[q] - mx) * kLog2e);   // 0 for the unused slots (lq = -inf)
        sum += w;
        acc.x = fmaf(w, vq[q].x, acc.x);
        acc.y = fmaf(w, vq[q].y, acc.y);
        acc.z = fmaf(w, vq[q].z, acc.z);
        acc.w = fmaf(w, vq[q].w, acc.w);
      }
      const float inv = 1.f / sum;
      acc.x *= inv;
      acc.y *= inv;
      acc.z *= inv;
      acc.w *= inv;
    }
    const float lse = mx != -INFINITY ? mx + logf(sum) : -INFINITY;
    store4_out(out + orow * kDim + 4 * tid, acc);
    if (lse_out != nullptr && tid == 0) lse_out[orow] = lse;
  }
}

// ---------------------------------------------------------------------------
// Plan of a ragged call (per-sequence KV lengths), one CTA: cu[v] = first tile of
// virtual sequence v (qb x head groups + 1 entries, qb query sequences of `heads`
// rows) over the lengths qseq_len gives (seqlens nullptr: max_len for all); query
// sequences with no KV rows get out = 0 and lse = -inf here (the decode kernel
// never visits them).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
mla_ragged_plan_kernel(const int* __restrict__ seqlens, int qb, int heads, int hgroups, int q_len, int kv_heads,
                       int max_len, uint32_t* __restrict__ cu, void* __restrict__ out, float* __restrict__ lse,
                       int out_elem_bytes) {
  __shared__ uint32_t s_part[1024];
  const int tid = threadIdx.x;
  const int vb = qb * hgroups;
  auto tiles = [&](int v) -> uint32_t {
    const int len = qseq_len(seqlens, v / hgroups, q_len, kv_heads, max_len);
    return (uint32_t)((len + kTile - 1) / kTile);
  };
  const int per = (vb + 1023) / 1024;
  const int v0 = tid * per, v1 = v0 + per < vb ? v0 + per : vb;
  uint32_t sum = 0;
  for (int v = v0; v < v1; ++v) sum += tiles(v);
  s_part[tid] = sum;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {   // inclusive scan of the chunk sums
    const uint32_t x = tid >= off ? s_part[tid - off] : 0u;
    __syncthreads();
    s_part[tid] += x;
    __syncthreads();
  }
  uint32_t run = tid > 0 ? s_part[tid - 1] : 0u;
  for (int v = v0; v < v1; ++v) {
    cu[v] = run;
    run += tiles(v);
  }
  if (tid == 1023) cu[vb] = s_part[1023];
  for (int row = tid; row < qb * heads; row += 1024) {
    if (qseq_len(seqlens, row / heads, q_len, kv_heads, max_len) > 0) continue;
    uint4* o = reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + (size_t)row * kDim * out_elem_bytes);
    for (int i = 0; i < kDim * out_elem_bytes / 16; ++i) o[i] = make_uint4(0u, 0u, 0u, 0u);
    if (lse != nullptr) lse[row] = -INFINITY;
  }
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

// 2D row-major [rows, cols] tensor, boxes of 64 rows x 128 bytes, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, CUtensorMapDataType dt,
              uint32_t elem_bytes = 2) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * elem_bytes};
  const cuuint32_t box[2] = {128 / elem_bytes, 64};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3D row-major [depth, rows, cols] tensor (batch, heads, dims), boxes of 64 rows x
// 128 bytes x 1, 128-byte swizzle.
bool make_map3(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t depth,
               CUtensorMapDataType dt, uint32_t elem_bytes = 2) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {cols, rows, depth};
  const cuuint64_t strides[2] = {cols * elem_bytes, rows * cols * elem_bytes};
  const cuuint32_t box[3] = {128 / elem_bytes, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// KV rows [rows][kv_heads][cols] (row-major), boxes of 64 rows x 1 KV head x 128
// bytes, 128-byte swizzle: the smem tile of one KV head is the 2D 64 x 128-byte box.
bool make_map_kv(CUtensorMap* m, const void* base, uint64_t cols, uint64_t kv_heads, uint64_t rows,
                 CUtensorMapDataType dt, uint32_t elem_bytes = 2) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {cols, kv_heads, rows};
  const cuuint64_t strides[2] = {cols * elem_bytes, kv_heads * cols * elem_bytes};
  const cuuint32_t box[3] = {128 / elem_bytes, 1, 64};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per-device launch facts: attributes set, how many clusters of 2 fit at once.
struct DeviceInfo {
  bool ready = false;
  int max_pairs = 0;
  bool coop = false;   // cooperative launches available (in-kernel merge of wide splits)
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
  cfg.blockDim = dim3(threads_of<T>(), 1, 1);
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
    int n[5] = {0, 0, 0, 0, 0};
    cudaError_t err = set_attrs_and_count<__nv_bfloat16>(&n[0]);
    if (err == cudaSuccess) err = set_attrs_and_count<__half>(&n[1]);
    if (err == cudaSuccess) err = set_attrs_and_count<Kv8<__nv_bfloat16>>(&n[2]);
    if (err == cudaSuccess) err = set_attrs_and_count<Kv8<__half>>(&n[3]);
    if (err == cudaSuccess) err = set_attrs_and_count<Cv<__nv_bfloat16, true>>(&n[4]);
    if (err != cudaSuccess) return err;
    d.max_pairs = n[0];
    for (int i = 1; i < 5; ++i) d.max_pairs = n[i] < d.max_pairs ? n[i] : d.max_pairs;
    int coop = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess) {
      cudaGetLastError();
      coop = 0;
    }
    d.coop = coop != 0;
    d.ready = true;
  }
  *out = d;
  return cudaSuccess;
}

int current_max_pairs(bool* coop = nullptr) {
  if (coop != nullptr) *coop = false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  DeviceInfo d;
  if (device_info(dev, &d) != cudaSuccess) {
    cudaGetLastError();   // clear a sticky-free error from the query
    return 0;
  }
  if (coop != nullptr) *coop = d.coop;
  return d.max_pairs;
}

}  // namespace sm100

int head_groups(int heads) { return (heads + sm100::kHeads - 1) / sm100::kHeads; }

QShape qshape(const DecodeArgs& a) {
  QShape s;
  s.q_len = a.q_len > 0 ? a.q_len : 1;
  s.kv_heads = a.kv_heads > 0 ? a.kv_heads : 1;
  s.qb = a.batch * s.q_len * s.kv_heads;
  s.g = a.heads / s.kv_heads;
  s.hg = head_groups(s.g);
  s.vb = s.qb * s.hg;
  return s;
}

bool sm100_supports_ext(int batch, int q_len, int heads, int kv_heads, int seqlen_kv) {
  // 32-bit tile arithmetic in the kernel and int32 TMA row coordinates
  if (heads < 1 || seqlen_kv < 1 || batch < 1 || q_len < 1 || kv_heads < 1 || heads % kv_heads != 0)
    return false;
  const long long nt = (seqlen_kv + sm100::kTile - 1) / sm100::kTile;
  const long long qb = (long long)batch * q_len * kv_heads;
  const long long vb = qb * head_groups(heads / kv_heads);
  return vb * nt * (sm100::kMaxPairs + 1) < (1ll << 32) && qb * heads < (1ll << 31) &&
         (long long)batch * seqlen_kv < (1ll << 31) - sm100::kTile;
}

bool sm100_supports(int batch, int heads, int seqlen_kv) { return sm100_supports_ext(batch, 1, heads, 1, seqlen_kv); }

SplitPlan sm100_plan(int batch, int heads, int seqlen_kv, const MlaCfg& cfg, int* variant) {
  batch *= head_groups(heads);   // virtual sequences: one per (sequence, group of 128 heads)
  SplitPlan pl{};
  *variant = 0;
  pl.block_n = sm100::kTile;
  const int nt = (seqlen_kv + sm100::kTile - 1) / sm100::kTile;
  const long long total = (long long)batch * nt;
  int pairs = cfg.num_split > 0 ? cfg.num_split : 0;
  bool coop = false;
  int cap = sm100::current_max_pairs(&coop);
  if (cap <= 0) {
    cap = 74;     // planning on a host without a usable GPU: a B200's plan
    coop = true;
  }
  if (pairs == 0 || pairs > cap) pairs = cap;
  if (pairs > sm100::kMaxPairs) pairs = sm100::kMaxPairs;
  if (cfg.num_split <= 0) {
    // Whole sequences per pair (no split, no merge, no partial traffic) when that
    // costs at most kWholeSlack more tiles per pair than spreading the tiles over
    // every pair (measured 4.6 % faster at 64 sequences x 64 tiles on 74 pairs),
    // as long as it keeps at least 80 % of the pairs busy.
    const long long k = ((long long)batch + pairs - 1) / pairs;   // sequences per pair
    const long long whole = ((long long)batch + k - 1) / k;
    if ((double)k * nt - (double)total / pairs <= sm100::kWholeSlack && whole * 5 >= (long long)pairs * 4)
      pairs = (int)whole;
  }
  if ((long long)pairs > total) pairs = (int)total;
  const int maxp = 2;            // partial slots per pair: its first and its last piece
  pl.ns = pairs * maxp;          // partial slots
  pl.bpc = pairs;                // CTA pairs
  pl.extra = maxp;               // slots per pair
  pl.part_rows = (long long)pairs * maxp * sm100::kHeads;
  // partials exist unless every pair's range starts on a sequence boundary
  pl.needs_combine = false;
  for (int pp = 1; pp < pairs; ++pp)
    if (((long long)pp * total / pairs) % nt != 0) pl.needs_combine = true;
  // Sequences split between a few pairs are merged inside the kernel by the last
  // pair to finish; one split between many (long contexts, small batches) goes to
  // a combine launch, which merges all heads in parallel instead of one pair
  // reading every partial.
  int most = 1;
  for (int bb = 0; bb < batch && pl.needs_combine; ++bb) {
    const long long x0 = (long long)bb * nt;
    const long long pf = ((x0 + 1) * pairs + total - 1) / total - 1;
    const long long pz = ((x0 + nt) * pairs + total - 1) / total - 1;
    if (pz - pf + 1 > most) most = (int)(pz - pf + 1);
  }
  // sequences split between many pairs: merged by the combine launch (variant 1;
  // measured faster on B200: b1 s131072 77.6 against 94.1 us per call, b16 s8192
  // 95 against 124 us), or, when the config asks for it (combine_groups < 0), by
  // all of their pairs inside the decode launch (variant 2, cooperative launch)
  const bool in_kernel = cfg.combine_groups < 0;
  *variant = most > sm100::kFuseMaxPieces ? ((coop && in_kernel) ? 2 : 1) : 0;
  return pl;
}

bool sm100_coop_available() {
  bool coop = false;
  if (sm100::current_max_pairs(&coop) <= 0) return true;   // host without a GPU: a B200's plan
  return coop;
}

// One launch of the decode kernel variant K: cooperative (every CTA resident at
// once, which the in-kernel merge of wide splits waits on) when p.coop is set.
template <typename K>
cudaError_t launch_variant(const sm100::Params& p, int pairs, cudaStream_t stream) {
  using namespace sm100;
  if (!p.coop) {
    mla_sm100_decode_kernel<K><<<2 * pairs, threads_of<K>(), Smem<K>::kBytes, stream>>>(p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(threads_of<K>(), 1, 1);
  cfg.dynamicSmemBytes = Smem<K>::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeCooperative;
  attr.val.cooperative = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mla_sm100_decode_kernel<K>, p);
}

cudaError_t launch_sm100_combine(const DecodeArgs& a);

cudaError_t launch_sm100_decode_plain_then_combine(const DecodeArgs& a, const sm100::Params& p) {
  using namespace sm100;
  const int pairs = a.plan.bpc;
  cudaError_t err;
  if (a.kv_fp8)
    err = a.dtype == MLA_DTYPE_BF16 ? launch_variant<Kv8<__nv_bfloat16>>(p, pairs, a.stream)
                                    : launch_variant<Kv8<__half>>(p, pairs, a.stream);
  else if (a.dtype == MLA_DTYPE_BF16)
    err = kConvV ? launch_variant<Cv<__nv_bfloat16, true>>(p, pairs, a.stream)
                 : launch_variant<__nv_bfloat16>(p, pairs, a.stream);
  else
    err = launch_variant<__half>(p, pairs, a.stream);
  return err == cudaSuccess ? launch_sm100_combine(a) : err;
}

namespace sm100 {

// The six tensor maps of a call, encoded by the driver (cuTensorMapEncodeTiled, a
// few microseconds of host time for all of them) or taken from a small per-thread
// cache of the last calls' maps: a decode loop calls again and again with the same
// tensors, and a map depends only on the key below.
struct MapKey {
  const void *q, *q_pe, *kv, *k_pe, *out, *part_o;
  long long part_rows, kv_rows;
  int g, qb, kv_heads, dtype, out_f32, kv_fp8;
  bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapEntry {
  MapKey key;
  CUtensorMap kv, kpe, q, qpe, out, part;
};

bool tensor_maps(const DecodeArgs& a, const QShape& qs, Params* p) {
  MapKey key;
  memset(&key, 0, sizeof(key));   // padding included: keys compare bytewise
  key.q = a.q;
  key.q_pe = a.q_pe;
  key.kv = a.kv;
  key.k_pe = a.k_pe;
  key.out = a.out;
  key.part_o = a.part_o;
  key.part_rows = a.part_o != nullptr ? a.plan.part_rows : 0;
  key.kv_rows = a.block_table != nullptr ? (long long)a.num_pages * a.page_size : (long long)a.batch * a.seqlen_kv;
  key.g = qs.g;
  key.qb = qs.qb;
  key.kv_heads = qs.kv_heads;
  key.dtype = a.dtype;
  key.out_f32 = p->out_f32;
  key.kv_fp8 = a.kv_fp8;
  constexpr int kSlots = 8;
  thread_local MapEntry cache[kSlots];
  thread_local int filled = 0, next = 0;
  for (int i = 0; i < filled; ++i) {
    if (cache[i].key == key) {
      p->tm_kv = cache[i].kv;
      p->tm_kpe = cache[i].kpe;
      p->tm_q = cache[i].q;
      p->tm_qpe = cache[i].qpe;
      p->tm_out = cache[i].out;
      p->tm_part = cache[i].part;
      return true;
    }
  }
  const CUtensorMapDataType dt =
      a.dtype == MLA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t kv_rows = (uint64_t)key.kv_rows;
  const bool ok_kv = a.kv_fp8 ? make_map_kv(&p->tm_kv, a.kv, kDim, qs.kv_heads, kv_rows,
                                            CU_TENSOR_MAP_DATA_TYPE_UINT8, 1)
                               : make_map_kv(&p->tm_kv, a.kv, kDim, qs.kv_heads, kv_rows, dt);
  if (!ok_kv || !make_map_kv(&p->tm_kpe, a.k_pe, kPeDim, qs.kv_heads, kv_rows, dt) ||
      !make_map3(&p->tm_q, a.q, kDim, qs.g, qs.qb, dt) || !make_map3(&p->tm_qpe, a.q_pe, kPeDim, qs.g, qs.qb, dt))
    return false;
  if (!(p->out_f32 ? make_map3(&p->tm_out, a.out, kDim, qs.g, qs.qb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4)
                   : make_map3(&p->tm_out, a.out, kDim, qs.g, qs.qb, dt)))
    return false;
  if (a.part_o != nullptr &&
      !make_map(&p->tm_part, a.part_o, kDim, (uint64_t)a.plan.part_rows, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4))
    return false;
  MapEntry& e = cache[next];
  e.key = key;
  e.kv = p->tm_kv;
  e.kpe = p->tm_kpe;
  e.q = p->tm_q;
  e.qpe = p->tm_qpe;
  e.out = p->tm_out;
  e.part = p->tm_part;
  next = (next + 1) % kSlots;
  if (filled < kSlots) ++filled;
  return true;
}

}  // namespace sm100

cudaError_t launch_sm100_decode(const DecodeArgs& a, int variant) {
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
  const QShape qs = qshape(a);
  p.out_f32 = a.out_dtype == MLA_DTYPE_F32 ? 1 : 0;
  // variant 1: the combine launch takes what the kernel does not merge; variant 2:
  // a cooperative launch merges every split sequence in the kernel
  p.fuse_max = kFuseMaxPieces;
  p.coop = (variant == 2 && info.coop) ? 1 : 0;
  if (!tensor_maps(a, qs, &p)) return cudaErrorInvalidValue;
  p.kv = static_cast<const uint8_t*>(a.kv);
  p.q = static_cast<const uint8_t*>(a.q);
  p.qpe = static_cast<const uint8_t*>(a.q_pe);
  p.out = a.out;
  p.lse_out = a.lse;
  p.part_o = a.part_o;
  p.part_lse = a.part_lse;
  p.status = a.status;
  p.counters = a.counters;
  p.heads = qs.g;
  p.hgroups = qs.hg;
  p.batch = qs.vb;
  p.q_len = qs.q_len;
  p.kv_heads = qs.kv_heads;
  p.seqlen = a.seqlen_kv;
  p.nt = (a.seqlen_kv + kTile - 1) / kTile;
  p.total_tiles = (uint32_t)p.batch * (uint32_t)p.nt;
  p.pairs = pairs;
  p.maxp = a.plan.extra;
  p.sl2 = a.softmax_scale * kLog2e;
  p.cu_tiles = a.cu_tiles;
  p.seqlens = a.seqlens;
  p.block_table = a.block_table;
  p.page_size = a.page_size;
  p.max_pages = a.max_pages;
  p.kv_scale = a.kv_fp8 ? a.kv_scale : 1.f;
  cudaError_t lerr;
  if (a.kv_fp8) {
    lerr = a.dtype == MLA_DTYPE_BF16 ? launch_variant<Kv8<__nv_bfloat16>>(p, pairs, a.stream)
                                     : launch_variant<Kv8<__half>>(p, pairs, a.stream);
  } else if (a.dtype == MLA_DTYPE_BF16) {
    lerr = kConvV ? launch_variant<Cv<__nv_bfloat16, true>>(p, pairs, a.stream)
                  : launch_variant<__nv_bfloat16>(p, pairs, a.stream);
  } else {
    lerr = launch_variant<__half>(p, pairs, a.stream);
  }
  if (lerr != cudaSuccess && p.coop) {
    // the cooperative launch was refused: the plain launch, and the combine launch
    // merges what the kernel then leaves
    cudaGetLastError();
    p.coop = 0;
    return launch_sm100_decode_plain_then_combine(a, p);
  }
  return lerr;
}

cudaError_t launch_wait_selftest(uint32_t* status, unsigned long long* result, uint64_t limit_ns,
                                 uint32_t code, cudaStream_t stream) {
  sm100::mla_wait_selftest_kernel<<<2, 32, 0, stream>>>(status, result, limit_ns, code);
  return cudaGetLastError();
}

cudaError_t launch_sm100_combine(const DecodeArgs& a) {
  using namespace sm100;
  const int nt = (a.seqlen_kv + kTile - 1) / kTile;
  const QShape qs = qshape(a);
  const int hg = qs.hg, vb = qs.vb;
  const uint32_t total = (uint32_t)vb * (uint32_t)nt;
  // a programmatic dependent of the decode kernel before it in the stream
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(kHeads, vb, 1);
  cfg.blockDim = dim3(128 * kCombineGroups, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const float* pl = a.part_lse;
  const float* po = a.part_o;
  const uint32_t* cu = a.cu_tiles;
  const int pairs = a.plan.bpc, g = qs.g, fm = kFuseMaxPieces;
  if (a.out_dtype == MLA_DTYPE_F32)
    return cudaLaunchKernelEx(&cfg, mla_pair_combine_kernel<float>, pl, po, static_cast<float*>(a.out), a.lse, cu,
                              total, nt, pairs, vb, g, hg, fm);
  if (a.dtype == MLA_DTYPE_BF16)
    return cudaLaunchKernelEx(&cfg, mla_pair_combine_kernel<__nv_bfloat16>, pl, po,
                              static_cast<__nv_bfloat16*>(a.out), a.lse, cu, total, nt, pairs, vb, g, hg, fm);
  return cudaLaunchKernelEx(&cfg, mla_pair_combine_kernel<__half>, pl, po, static_cast<__half*>(a.out), a.lse, cu,
                            total, nt, pairs, vb, g, hg, fm);
}

cudaError_t launch_seqsplit_combine(const DecodeArgs& a, bool pieces, const PeerRows& x, void* out, float* lse,
                                    int dtype) {
  using namespace sm100;
  const int nt = (a.seqlen_kv + kTile - 1) / kTile;
  const QShape qs = qshape(a);
  const int hg = qs.hg, vb = qs.vb;
  const uint32_t total = (uint32_t)vb * (uint32_t)nt;
  // at most one CTA per SM: pass 1 of every CTA runs without waiting on anything
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n > 0 ? n : 1;
  }
  const int rows = vb * kHeads;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(rows < sms[dev] ? rows : sms[dev], 1, 1);
  cfg.blockDim = dim3(128 * kCombineGroups, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const float* pl = a.part_lse;
  const float* po = a.part_o;
  const uint32_t* cu = a.cu_tiles;
  const int pairs = a.plan.bpc, g = qs.g, fm = pieces ? kFuseMaxPieces : -1;
  if (dtype == MLA_DTYPE_BF16)
    return cudaLaunchKernelEx(&cfg, mla_seqsplit_combine_kernel<__nv_bfloat16>, pl, po, cu, total, nt, pairs, vb, g, hg,
                              fm, x, static_cast<__nv_bfloat16*>(out), lse);
  if (dtype == MLA_DTYPE_F16)
    return cudaLaunchKernelEx(&cfg, mla_seqsplit_combine_kernel<__half>, pl, po, cu, total, nt, pairs, vb, g, hg, fm,
                              x, static_cast<__half*>(out), lse);
  return cudaLaunchKernelEx(&cfg, mla_seqsplit_combine_kernel<float>, pl, po, cu, total, nt, pairs, vb, g, hg, fm, x,
                            static_cast<float*>(out), lse);
}

}  // namespace mla

namespace mla {

SplitPlan sm100_plan_ragged(int batch, int heads, int max_seqlen_kv, const MlaCfg& cfg) {
  SplitPlan pl{};
  pl.block_n = sm100::kTile;
  const int nt = (max_seqlen_kv + sm100::kTile - 1) / sm100::kTile;
  const long long total_max = (long long)batch * head_groups(heads) * nt;
  int pairs = cfg.num_split > 0 ? cfg.num_split : 0;
  int cap = sm100::current_max_pairs();
  if (cap <= 0) cap = 74;
  if (pairs == 0 || pairs > cap) pairs = cap;
  if (pairs > sm100::kMaxPairs) pairs = sm100::kMaxPairs;
  if ((long long)pairs > total_max) pairs = (int)(total_max > 0 ? total_max : 1);
  pl.ns = pairs * 2;
  pl.bpc = pairs;
  pl.extra = 2;
  pl.part_rows = (long long)pairs * 2 * sm100::kHeads;
  pl.needs_combine = true;
  return pl;
}

cudaError_t launch_sm100_ragged_plan(const DecodeArgs& a) {
  const int elem = a.out_dtype == MLA_DTYPE_F32 ? 4 : 2;
  int cap = a.seqlen_kv;
  if (a.block_table != nullptr && (long long)a.max_pages * a.page_size < cap) cap = a.max_pages * a.page_size;
  const QShape qs = qshape(a);
  sm100::mla_ragged_plan_kernel<<<1, 1024, 0, a.stream>>>(a.seqlens, qs.qb, qs.g, qs.hg, qs.q_len, qs.kv_heads,
                                                          cap, a.cu_tiles, a.out, a.lse, elem);
  return cudaGetLastError();
}

}  // namespace mla
