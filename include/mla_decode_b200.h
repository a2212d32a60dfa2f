/*
 * mla_decode_b200.h -- C ABI of the B200 (sm_100a) absorbed-MLA decode path.
 *
 * Layout of every tensor argument (row-major, contiguous, device pointers):
 *   q      [batch, heads, 512]        fp16 or bf16 (dtype)
 *   q_pe   [batch, heads, 64]         same dtype
 *   kv     [batch, seqlen_kv, 1, 512] same dtype  (latent: keys AND values)
 *   k_pe   [batch, seqlen_kv, 1, 64]  same dtype  (rope part of the keys)
 *   out    [batch, heads, 512]        same dtype, caller-allocated, written
 *   lse    [batch, heads]             float32 natural-log log-sum-exp, optional
 *
 * out[b,h,:] = softmax_s(([q|q_pe] . [kv|k_pe]^T) / sqrt(576)) . kv.
 *
 * Every entry point returns MLA_OK (0) or an error code; nothing throws across
 * the ABI, and mla_last_error() gives the calling thread's last message.
 * Launch entry points enqueue on `stream` (a cudaStream_t, NULL = legacy
 * default stream) and never synchronise the host.  Calls on distinct streams
 * from distinct threads are safe; per-device kernel attributes are set once.
 */
#ifndef MLA_DECODE_B200_H_
#define MLA_DECODE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLA_ABI_VERSION 1

enum MlaDtype {
  MLA_DTYPE_F16 = 0,
  MLA_DTYPE_BF16 = 1,
  MLA_DTYPE_F32 = 2   /* output only: mla_combine's `out`, mla_decode_partial's `o` */
};

enum MlaStatus {
  MLA_OK = 0,
  MLA_ERR_ARG = 1,          /* bad shape, pointer, alignment or config */
  MLA_ERR_WORKSPACE = 2,    /* workspace missing or too small */
  MLA_ERR_UNSUPPORTED = 3,  /* shape/config outside what the kernels cover */
  MLA_ERR_CUDA = 4,         /* a CUDA runtime/driver call failed */
  MLA_ERR_DEVICE = 5        /* a kernel reported a failure through its status word */
};

/* Which decode kernel runs. */
enum MlaKernelKind {
  MLA_KERNEL_AUTO = 0,   /* tensor-core kernel where it covers the shape, else SIMT */
  MLA_KERNEL_SIMT = 1,   /* CUDA-core split-KV kernel (any heads, any seqlen) */
  MLA_KERNEL_TC = 2      /* tcgen05/TMA/TMEM split-KV kernel (sm_100a) */
};

/*
 * Tuning knobs.  Same names and meaning as the reference's config dict
 * (mla_decode.py:588-598, 720-729): block_N KV rows per tile, block_H heads
 * per CTA, num_split requested KV splits per sequence, spread selects the
 * whole-wave split family of _split_plan (mla_decode.py:9-30), num_stages the
 * depth of the shared-memory pipeline.  A sequence the tensor-core kernel
 * splits between more than 3 CTA pairs is merged by a separate combine launch
 * (single pass for any combine_groups >= 0: the reference's second stage,
 * mla_decode.py:248-259, is not needed); combine_groups < 0 (an extension: the
 * reference never passes it) asks for that merge inside the decode launch
 * instead, by all of the sequence's CTA pairs in a cooperative launch.
 * softmax_scale is the factory
 * argument of the same name (mla_decode.py:38).  Zero fields mean "choose".
 */
typedef struct MlaCfg {
  int32_t block_N;
  int32_t block_H;
  int32_t num_split;
  int32_t spread;
  int32_t num_stages;
  int32_t combine_groups;
  int32_t kernel;         /* enum MlaKernelKind */
  float softmax_scale;    /* multiplies the raw scores; 0 = 1/sqrt(576) */
} MlaCfg;

/* Version of this ABI (MLA_ABI_VERSION). */
int32_t mla_abi_version(void);

/* Thread-local text of the last error returned on this thread ("" if none). */
const char* mla_last_error(void);

/*
 * _split_plan (mla_decode.py:9-30): nb = ceil(seqlen_kv / block_n) KV tiles
 * go to ns splits.  Writes {ns, blocks_per_split, extra} to out3.
 */
int32_t mla_split_plan(int32_t seqlen_kv, int32_t num_split, int32_t block_n,
                       int32_t spread, int32_t* out3);

/*
 * Bytes of device scratch mla_decode_fwd needs for this shape and config
 * (partial O and partial LSE per split, float32).  Replaces the per-call
 * T.alloc_global of glse / output_partial (mla_decode.py:73-76).
 * Clears this thread's error text on entry; returns 0 either when no
 * workspace is needed (error text stays empty) or on a bad argument (error
 * text set, see mla_last_error).
 */
size_t mla_workspace_bytes(int32_t batch, int32_t heads, int32_t seqlen_kv,
                           int32_t dtype, const MlaCfg* cfg);

/*
 * Facts about the plan mla_decode_fwd would use for this shape and config:
 *   out4[0] kernel (enum MlaKernelKind, never AUTO)
 *   out4[1] KV splits per sequence (CUDA-core kernel) or CTA pairs (tensor-core kernel)
 *   out4[2] kernel launches per call (1 or 2; the tensor-core kernel merges a
 *           sequence split between at most 3 CTA pairs itself, by the last of
 *           them; one split between more goes to a combine launch, unless
 *           cfg->combine_groups < 0 asks all of its pairs to merge it inside the
 *           kernel in a cooperative launch)
 *   out4[3] bytes at the start of the workspace that must be zero before the
 *           first call with it (the tensor-core kernel's status word and piece
 *           counters; every call leaves them zero again)
 * Mirrors the reference's split planning (mla_decode.py:9-30, 539-606).
 */
int32_t mla_describe_plan(int32_t batch, int32_t heads, int32_t seqlen_kv,
                          int32_t dtype, const MlaCfg* cfg, int64_t* out4);

/*
 * One decode call: the split-KV main kernel then the LSE combine kernel,
 * enqueued on `stream`.  Replaces the TileLang prim_func `main`
 * (mla_decode.py:65-259) that kernel(q, q_pe, kv, k_pe, out) launches, and the
 * handmade launcher mla_launch(Q, Qpe, KV, Kpe, glse, partial, out, ns)
 * (handmade/mla_handmade.py:32-53).  `workspace` must hold
 * mla_workspace_bytes(...) bytes (256-byte aligned).  lse may be NULL.
 * cfg may be NULL (all fields "choose").
 */
int32_t mla_decode_fwd(const void* q, const void* q_pe, const void* kv,
                       const void* k_pe, void* out, float* lse,
                       void* workspace, size_t workspace_bytes,
                       int32_t batch, int32_t heads, int32_t seqlen_kv,
                       int32_t dtype, const MlaCfg* cfg, void* stream);

/*
 * mla_decode_fwd in its two launches, for callers that interleave their own
 * work or events between them (same arguments and checks as mla_decode_fwd):
 * mla_decode_splitkv enqueues the split-KV main kernel (mla_decode.py:78-192),
 * which leaves per-split partials in `workspace` (or, for a single-split plan,
 * writes out/lse directly); mla_decode_combine_ws then enqueues the combine
 * kernel (mla_decode.py:194-246) over that workspace, and is a no-op for a
 * single-split plan.  Both must see the same shape, dtype and cfg.
 */
int32_t mla_decode_splitkv(const void* q, const void* q_pe, const void* kv,
                           const void* k_pe, void* out, float* lse,
                           void* workspace, size_t workspace_bytes,
                           int32_t batch, int32_t heads, int32_t seqlen_kv,
                           int32_t dtype, const MlaCfg* cfg, void* stream);
int32_t mla_decode_combine_ws(void* out, float* lse, const void* workspace,
                              size_t workspace_bytes, int32_t batch,
                              int32_t heads, int32_t seqlen_kv, int32_t dtype,
                              const MlaCfg* cfg, void* stream);

/*
 * LSE combine of num_split normalised partial results (the second kernel of
 * mla_decode.py:194-246, natural-log units):
 *   part_lse [num_split, batch, heads]       float32 (-inf = empty split)
 *   part_o   [num_split, batch, heads, 512]  float32
 * out[b,h,:] = sum_k exp(lse_k - LSE) * o_k with LSE = logsumexp_k(lse_k);
 * lse (optional) receives LSE.  dtype is the type of `out`: F16, BF16, or F32
 * (a float32 result that can itself be combined again).  Also merges per-GPU
 * results of a sequence-split decode (mla_decode_partial on each GPU's part
 * of the KV sequence) after they are gathered into one buffer.
 */
int32_t mla_combine(const float* part_lse, const float* part_o,
                    int32_t num_split, int32_t batch, int32_t heads,
                    void* out, float* lse, int32_t dtype, void* stream);

/*
 * mla_combine over partials that are not split-major: split k's LSE row r is
 * part_lse[k * lse_split_stride + r] and its O row r starts at
 * part_o + k * o_split_stride + r * 512 (strides in floats, o_split_stride a
 * multiple of 4).  The cross-GPU merge of the sequence split gathers every
 * GPU's (O, LSE) as one packed block per GPU ([O | LSE | padding]) in a single
 * all-gather and merges it in place with this call.  No reference counterpart
 * (its partials are always split-minor in one buffer, mla_decode.py:73-76).
 */
int32_t mla_combine_strided(const float* part_lse, int64_t lse_split_stride,
                            const float* part_o, int64_t o_split_stride,
                            int32_t num_split, int32_t batch, int32_t heads,
                            void* out, float* lse, int32_t dtype, void* stream);

/*
 * The sequence split's exchange over NVLink, without a collective library (no
 * reference counterpart: the reference has no multi-GPU path).  world (2..8; 1..8
 * for mla_seqsplit_decode / mla_seqsplit_merge below)
 * ranks, one GPU each on one node, each own a gather buffer of
 * mla_seqsplit_buffer_bytes(world, batch, heads) bytes (256-byte aligned, zeroed
 * once) and map every peer's buffer with mla_ipc_export / mla_ipc_import (CUDA
 * IPC; handles exchanged by the host, e.g. over the process group).  Layout of
 * a buffer: float blocks [2][world][chunk] with chunk = batch*heads*512 +
 * round_up(batch*heads, 64): block [epoch & 1][r] is rank r's (O, LSE) of call
 * `epoch` (O rows, then the LSEs); then a 256-byte header (flags, a counter, the
 * status word at byte 68: 0, or 0x201 when a wait gave up), then row words
 * uint32 pairs [2][world][round_up(batch*heads, 64)][512] and LSE words uint32
 * pairs [2][world][round_up(batch*heads, 64)] (value bits, call number).
 * For call `epoch` (1, 2, 3, ... the same on every rank), rank `rank` writes its
 * block [epoch & 1][rank] in its own buffer (mla_decode_partial into it), then
 * mla_seqsplit_exchange enqueues one launch that stores that block into every
 * peer's buffer, flags it there, and waits (at most 2 s) until every peer's block
 * has arrived in this rank's buffer; mla_combine_strided over the blocks
 * [epoch & 1][*] then merges them.  bufs holds every rank's buffer as mapped in
 * this process (bufs[rank] its own).  The launch waits on the other GPUs' launches:
 * every rank must make the call.
 */
size_t mla_seqsplit_buffer_bytes(int32_t world, int32_t batch, int32_t heads);
int32_t mla_ipc_export(const void* ptr, void* handle_out /* 64 bytes */, uint64_t* offset_out);
int32_t mla_ipc_import(const void* handle /* 64 bytes */, uint64_t offset, void** ptr_out);
int32_t mla_ipc_close(void* ptr, uint64_t offset);
int32_t mla_seqsplit_exchange(void* const* bufs, int32_t world, int32_t rank, uint32_t epoch,
                              int32_t batch, int32_t heads, void* stream);

/*
 * The sequence split in two launches per call (same buffers, IPC mapping and
 * call numbering as above; world 1..8, world 1 needing no peers).  Rank `rank`
 * decodes q against its rows [0, seqlen_part) of every sequence (kv_part /
 * k_pe_part, the layout of mla_decode_fwd; same workspace and checks) to float32
 * (O, LSE) in its block [epoch & 1][rank]; then one launch merges that result
 * row by row (straight from the decode kernel's pieces when a sequence was split
 * between many CTA pairs), stores each merged row into every peer's row words
 * over NVLink (each value paired with the call number, so no fence or flag is
 * needed), polls (at most 2 s, status word as above) until every peer's words
 * carry this call's number, and writes the LSE merge over all ranks to out
 * ([batch, heads, 512], dtype) and lse (float32 [batch, heads], optional).  Every
 * rank must make the call.  mla_seqsplit_merge is the second launch alone, for a
 * rank whose block [epoch & 1][rank] is already written (mla_decode_partial into
 * it, or O = 0 and LSE = -inf for a rank with no rows); out may be float32 there
 * (dtype 2).
 */
int32_t mla_seqsplit_decode(const void* q, const void* q_pe, const void* kv_part, const void* k_pe_part,
                            void* out, float* lse, void* workspace, size_t workspace_bytes,
                            int32_t batch, int32_t heads, int32_t seqlen_part, int32_t dtype,
                            void* const* bufs, int32_t world, int32_t rank, uint32_t epoch,
                            const MlaCfg* cfg, void* stream);
int32_t mla_seqsplit_merge(void* const* bufs, int32_t world, int32_t rank, uint32_t epoch, int32_t batch,
                           int32_t heads, void* out, float* lse, int32_t dtype, void* stream);

/*
 * mla_decode_fwd for one contiguous part of every sequence's KV cache, with a
 * float32 result: o[b,h,:] (float32 [batch, heads, 512], normalised) and
 * lse[b,h] (float32 [batch, heads], natural log, required) are the decode of
 * q against rows [0, seqlen_kv) of kv/k_pe.  Results of several parts of the
 * same sequences, stacked as [parts, batch, heads, ...], combine into the
 * decode over the whole sequence with mla_combine (the sequence split across
 * GPUs).  Same inputs, workspace and checks as mla_decode_fwd.  No
 * counterpart in the reference, which splits a sequence only inside one
 * launch (the num_split partials of mla_decode.py:73-76).
 */
int32_t mla_decode_partial(const void* q, const void* q_pe, const void* kv,
                           const void* k_pe, float* o, float* lse,
                           void* workspace, size_t workspace_bytes,
                           int32_t batch, int32_t heads, int32_t seqlen_kv,
                           int32_t dtype, const MlaCfg* cfg, void* stream);

/*
 * mla_decode_fwd over an FP8 latent KV cache: kv_fp8 [batch, seqlen_kv, 1, 512]
 * holds e4m3 (OCP FP8, 4 exponent / 3 mantissa bits, one byte per dim) values
 * whose product with kv_scale is the latent row; q, q_pe, k_pe and out stay in
 * `dtype`.  Half the latent bytes of mla_decode_fwd.  The latent rows are
 * dequantized to fp16 in shared memory (exact), Q's latent dims are rounded to
 * fp16 after multiplying by kv_scale (|q| x kv_scale must stay within fp16
 * range), P is fp16, accumulation fp32.  Tensor-core kernel only (cfg->kernel
 * auto or tc); workspace as mla_workspace_bytes(batch, heads, seqlen_kv, dtype,
 * cfg) reports for the same cfg.  No counterpart in the reference (listed as
 * untried in its notes, docs/mla_decode_best_implementation.md:1693).
 */
int32_t mla_decode_fp8kv(const void* q, const void* q_pe, const void* kv_fp8,
                         const void* k_pe, float kv_scale, void* out, float* lse,
                         void* workspace, size_t workspace_bytes,
                         int32_t batch, int32_t heads, int32_t seqlen_kv,
                         int32_t dtype, const MlaCfg* cfg, void* stream);

/*
 * Decode over KV caches of different lengths, optionally paged (the caller-side
 * format of serving decode).  No counterpart in the reference, whose kernel takes
 * one kv_ctx for the whole batch (its design notes name per-sequence lengths as
 * the next step: docs/num_split_design.md).
 *   cache_seqlens [batch] int32: KV rows of each sequence, clamped to
 *                 [0, max_seqlen_kv]; a sequence with 0 rows gets out = 0 and
 *                 lse = -inf.
 *   block_table   NULL: kv_cache [batch, max_seqlen_kv, 1, 512] and k_pe_cache
 *                 [batch, max_seqlen_kv, 1, 64], as mla_decode_fwd's kv/k_pe;
 *                 else int32 [batch, max_pages_per_seq] page ids into
 *                 kv_cache [num_pages, page_size, 1, 512] and
 *                 k_pe_cache [num_pages, page_size, 1, 64]; row r of sequence b
 *                 is row r % page_size of page block_table[b][r / page_size].
 *                 page_size is a multiple of 64; lengths are also clamped to
 *                 max_pages_per_seq x page_size; entries past a sequence's
 *                 length are not read, and rows of its last page past the length
 *                 must hold finite values (they are masked).
 * q, q_pe, out, lse, dtype and cfg as in mla_decode_fwd (tensor-core kernel only;
 * cfg->num_split = CTA pairs).  `workspace` holds mla_paged_workspace_bytes()
 * bytes, 256-byte aligned, zero before the first call (every call leaves its
 * counters zero).  Three launches: the plan kernel (tile prefix sums from
 * cache_seqlens, on the device: no host sync), the decode kernel, the combine.
 */
size_t mla_paged_workspace_bytes(int32_t batch, int32_t heads, int32_t max_seqlen_kv,
                                 int32_t dtype, const MlaCfg* cfg);
int32_t mla_decode_paged(const void* q, const void* q_pe, const void* kv_cache,
                         const void* k_pe_cache, const int32_t* block_table,
                         const int32_t* cache_seqlens, void* out, float* lse,
                         void* workspace, size_t workspace_bytes,
                         int32_t batch, int32_t heads, int32_t max_seqlen_kv,
                         int32_t page_size, int32_t num_pages,
                         int32_t max_pages_per_seq, int32_t dtype,
                         const MlaCfg* cfg, void* stream);

/*
 * mla_decode_paged for multi-token decode steps and grouped KV heads.  No
 * counterpart in the reference (baseline_mla.py:16 asserts kv_heads == 1 and
 * its query has one position per sequence); its ref_program's head grouping
 * (baseline_mla.py:179-186: query head j reads KV head j / (heads / kv_heads))
 * is kept.
 *
 *   q, out     [batch, q_len, heads, 512]   q_pe [batch, q_len, heads, 64]
 *   lse        [batch, q_len, heads] float32, optional (natural log)
 *   kv_cache   [batch, max_seqlen_kv, kv_heads, 512] (no block_table) or
 *              [num_pages, page_size, kv_heads, 512]; k_pe_cache likewise with 64
 *   cache_seqlens  int32 [batch] KV rows per sequence, or NULL (all
 *              max_seqlen_kv, capped by the page table's cover when paged)
 *
 * Query position t of a sequence with L rows attends to its first
 * L - (q_len - 1 - t) rows (the step's q_len new tokens are the last rows of the
 * cache; causal within the step); a position with no rows gets out = 0,
 * lse = -inf.  heads must be a multiple of kv_heads.  Workspace from
 * mla_decode_ext_workspace_bytes, same rules as mla_decode_paged (q_len = 1,
 * kv_heads = 1 is exactly mla_decode_paged).
 */
size_t mla_decode_ext_workspace_bytes(int32_t batch, int32_t q_len, int32_t heads, int32_t kv_heads,
                                      int32_t max_seqlen_kv, int32_t dtype, const MlaCfg* cfg);
int32_t mla_decode_ext(const void* q, const void* q_pe, const void* kv_cache, const void* k_pe_cache,
                       const int32_t* block_table, const int32_t* cache_seqlens, void* out, float* lse,
                       void* workspace, size_t workspace_bytes, int32_t batch, int32_t q_len, int32_t heads,
                       int32_t kv_heads, int32_t max_seqlen_kv, int32_t page_size, int32_t num_pages,
                       int32_t max_pages_per_seq, int32_t dtype, const MlaCfg* cfg, void* stream);

/*
 * mla_decode_ext over an FP8 latent cache: kv_fp8 (same shape and paging as
 * mla_decode_ext's kv_cache) holds e4m3 codes whose product with kv_scale is the
 * latent row, as for mla_decode_fp8kv; k_pe_cache, q, q_pe and out stay in `dtype`.
 * Same workspace as mla_decode_ext.  No counterpart in the reference.
 */
int32_t mla_decode_ext_fp8kv(const void* q, const void* q_pe, const void* kv_fp8,
                             const void* k_pe_cache, float kv_scale, const int32_t* block_table,
                             const int32_t* cache_seqlens, void* out, float* lse, void* workspace,
                             size_t workspace_bytes, int32_t batch, int32_t q_len, int32_t heads,
                             int32_t kv_heads, int32_t max_seqlen_kv, int32_t page_size,
                             int32_t num_pages, int32_t max_pages_per_seq, int32_t dtype,
                             const MlaCfg* cfg, void* stream);

/*
 * mla_decode_fwd without a workspace argument, for callers that cannot
 * allocate device memory where they decode (code running under CUDA-graph
 * capture, servers that reserve all memory up front and forbid allocation on
 * the serving path, plugin hosts whose memory another runtime owns).  No
 * counterpart in the reference: it always allocates its scratch per call.
 *
 * Same inputs, outputs, checks and result as mla_decode_fwd; the split-KV
 * scratch comes from a static device array of MLA_NOALLOC_SCRATCH_BYTES that
 * every GPU loading the library holds until exit.  Shapes whose
 * mla_workspace_bytes exceeds it (for the CUDA-core kernel: it plus a 256-byte
 * status block kept in front) return MLA_ERR_WORKSPACE.  A rejected call
 * enqueues nothing.  The array's address is looked up once per device
 * (cudaGetSymbolAddress, with that device current) by mla_noalloc_init or by
 * the first decode call on the device; make one of them before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race.
 * Allocates nothing.
 */
#define MLA_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
int32_t mla_decode_fwd_noalloc(const void* q, const void* q_pe, const void* kv,
                               const void* k_pe, void* out, float* lse,
                               int32_t batch, int32_t heads, int32_t seqlen_kv,
                               int32_t dtype, const MlaCfg* cfg, void* stream);

/*
 * Looks up the static scratch array's address on the current device, so that a
 * host can prepare before it captures its first decode into a CUDA graph.
 * Optional (the first mla_decode_fwd_noalloc on the device does the same).
 * Same reason for existing as mla_decode_fwd_noalloc; no reference counterpart.
 */
int32_t mla_noalloc_init(void);

/*
 * Enqueues on `stream` a copy of the status word of the static scratch array
 * (current device) into *status_out (device or host memory): 0 after any
 * mla_decode_fwd_noalloc call, unless that call ran the tensor-core kernel and
 * one of its bounded waits gave up: then the code it recorded (0x101..0x106, as
 * in mla_decode_fwd's workspace status word).  Read it after that call and
 * before the next, which clears it.
 * No reference counterpart.
 */
int32_t mla_noalloc_status(uint32_t* status_out, void* stream);

/*
 * Self-test of the tensor-core kernel's failure detection, for tests and health
 * checks; no reference counterpart (the reference's kernels have no bounded waits).
 * Every wait of the decode kernel on a barrier is bounded: after about 2 s it
 * raises an abort flag in both CTAs of its pair, records a code in the
 * workspace's status word (MLA_ERR_DEVICE territory: 0x101..0x106 by role) and
 * the pair winds down, so a stalled pipeline ends the kernel instead of hanging
 * the GPU.  This call runs that same wait code in one CTA pair on barriers that
 * nothing arrives on, faulting nothing: CTA 0 gives up after limit_ns (1e6..1e8)
 * and writes MLA_SELFTEST_STATUS to *status (device memory, zero before the
 * call); CTA 1 waits with 100 x the limit and must leave through the abort flag.
 * result (device, 4 x uint64): [CTA 0 gave up (1), its wait in ns, CTA 1 left
 * (1), its wait in ns].  Enqueues one launch; synchronize before reading.
 */
#define MLA_SELFTEST_STATUS 0x1ffu
int32_t mla_selftest_wait_timeout(uint32_t* status, uint64_t* result, uint64_t limit_ns,
                                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLA_DECODE_B200_H_ */
