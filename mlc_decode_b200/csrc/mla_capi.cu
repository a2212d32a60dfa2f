// extern "C" entry points of libmla_decode_b200.so (declared in
// include/mla_decode_b200.h).  Argument checking, kernel choice, split planning
// and workspace carving live here; the kernels live in their own files.
#include <stdarg.h>
#include <stdio.h>
#include <math.h>
#include <string.h>

#include <string>

#include "mla_common.cuh"
#include "mla_sm100.cuh"

namespace mla {

namespace {
thread_local std::string g_last_error;
constexpr int kSmCount = 148;
}  // namespace

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

namespace {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Resolved launch: which kernel, and the split plan it uses.
struct Resolved {
  int kernel;
  SplitPlan plan;
  int tc_variant;  // sm100 kernel variant (see mla_sm100.cuh)
};

int check_shape(int batch, int heads, int seqlen_kv, int dtype) {
  if (batch < 1 || heads < 1 || seqlen_kv < 1) {
    set_error("mla: batch, heads and seqlen_kv must be >= 1 (got %d, %d, %d)", batch, heads, seqlen_kv);
    return MLA_ERR_ARG;
  }
  if (dtype != MLA_DTYPE_F16 && dtype != MLA_DTYPE_BF16) {
    set_error("mla: dtype must be 0 (fp16) or 1 (bf16), got %d", dtype);
    return MLA_ERR_ARG;
  }
  if ((long long)batch * heads > (1ll << 30) || (long long)batch * seqlen_kv > (1ll << 40)) {
    set_error("mla: shape too large");
    return MLA_ERR_ARG;
  }
  return MLA_OK;
}

int resolve(int batch, int heads, int seqlen_kv, const MlaCfg* cfg, Resolved* r) {
  MlaCfg c{};
  if (cfg != nullptr) c = *cfg;
  int kind = c.kernel;
  if (kind != MLA_KERNEL_AUTO && kind != MLA_KERNEL_SIMT && kind != MLA_KERNEL_TC) {
    set_error("mla: unknown kernel kind %d", kind);
    return MLA_ERR_ARG;
  }
  const bool tc_ok = sm100_supports(batch, heads, seqlen_kv);
  if (kind == MLA_KERNEL_TC && !tc_ok) {
    set_error("mla: the tensor-core kernel does not cover heads=%d seqlen_kv=%d", heads, seqlen_kv);
    return MLA_ERR_UNSUPPORTED;
  }
  if (kind == MLA_KERNEL_AUTO) kind = tc_ok ? MLA_KERNEL_TC : MLA_KERNEL_SIMT;
  r->kernel = kind;
  if (c.num_split < 0 || c.block_N < 0) {
    set_error("mla: num_split and block_N must be >= 0");
    return MLA_ERR_ARG;
  }
  if (kind == MLA_KERNEL_SIMT) {
    int bn = c.block_N > 0 ? c.block_N : simt_block_n();
    if (bn % simt_block_n() != 0) {
      set_error("mla: SIMT kernel needs block_N a multiple of %d (got %d)", simt_block_n(), bn);
      return MLA_ERR_ARG;
    }
    int ns = c.num_split;
    bool spread = c.spread != 0;
    if (ns == 0) {
      // enough CTAs for two resident waves over all SMs
      const long long units = (long long)batch * ((heads + 15) / 16);
      const long long target = (long long)kSmCount * simt_ctas_per_sm() * 2;
      ns = (int)((target + units - 1) / units);
      spread = true;
    }
    r->plan = split_plan(seqlen_kv, ns, bn, spread);
    r->tc_variant = 0;
  } else {
    r->plan = sm100_plan(batch, heads, seqlen_kv, c, &r->tc_variant);
  }
  if (r->plan.ns > 8192) {
    set_error("mla: num_split %d exceeds 8192", r->plan.ns);
    return MLA_ERR_ARG;
  }
  return MLA_OK;
}

// Workspace layout:
//   tensor-core kernel: [status word, 256 B][piece counters uint32 x batch x ceil(heads/128) x 4,
//                       padded to 256 B]
//                       [partial LSE float32 x rows, padded to 256 B][partial O float32 x rows x 512]
//                       (partials only when some sequence is split between CTA pairs)
//   CUDA-core kernel:   [partial LSE][partial O] when the plan has more than one split
// The tensor-core kernel's counters must be zero before the first call (a zero-filled
// workspace); every call leaves them zero again.  The 256-byte status block holds the
// status word (bytes 0-3) and the kernel's clock probe (uint64 SM cycles, ns and calls
// at bytes 8, 16, 24, accumulated over calls).
constexpr size_t kStatusBytes = 256;

// four counters per (sequence, group of 128 heads) of the tensor-core kernel: pieces
// published and CTAs done merging, per CTA rank
size_t counter_bytes(int batch, int heads) {
  return align_up((size_t)batch * head_groups(heads) * 4 * sizeof(uint32_t), 256);
}

size_t part_rows(int batch, int heads, const Resolved& r) {
  return r.plan.part_rows > 0 ? (size_t)r.plan.part_rows : (size_t)r.plan.ns * batch * heads;
}

size_t workspace_for(int batch, int heads, const Resolved& r) {
  const size_t head = r.kernel == MLA_KERNEL_TC ? kStatusBytes + counter_bytes(batch, heads) : 0;
  if (!r.plan.needs_combine) return head;
  const size_t rows = part_rows(batch, heads, r);
  return head + align_up(rows * sizeof(float), 256) + rows * kDim * sizeof(float);
}

}  // namespace
}  // namespace mla

using namespace mla;

extern "C" {

int32_t mla_abi_version(void) { return MLA_ABI_VERSION; }

const char* mla_last_error(void) { return g_last_error.c_str(); }

int32_t mla_split_plan(int32_t seqlen_kv, int32_t num_split, int32_t block_n, int32_t spread,
                       int32_t* out3) {
  if (out3 == nullptr || seqlen_kv < 0 || block_n < 1) {
    set_error("mla_split_plan: bad argument");
    return MLA_ERR_ARG;
  }
  const SplitPlan p = split_plan(seqlen_kv, num_split, block_n, spread != 0);
  out3[0] = p.ns;
  out3[1] = p.bpc;
  out3[2] = p.extra;
  return MLA_OK;
}

int32_t mla_describe_plan(int32_t batch, int32_t heads, int32_t seqlen_kv, int32_t dtype,
                          const MlaCfg* cfg, int64_t* out4) {
  if (out4 == nullptr) {
    set_error("mla_describe_plan: null output");
    return MLA_ERR_ARG;
  }
  int rc = check_shape(batch, heads, seqlen_kv, dtype);
  if (rc != MLA_OK) return rc;
  Resolved r{};
  rc = resolve(batch, heads, seqlen_kv, cfg, &r);
  if (rc != MLA_OK) return rc;
  const bool tc = r.kernel == MLA_KERNEL_TC;
  out4[0] = r.kernel;
  out4[1] = tc ? r.plan.bpc : r.plan.ns;
  out4[2] = (r.plan.needs_combine && (!tc || r.tc_variant == 1)) ? 2 : 1;   // (variant 2: merged in-kernel)
  out4[3] = tc ? (int64_t)(kStatusBytes + counter_bytes(batch, heads)) : 0;
  return MLA_OK;
}

size_t mla_workspace_bytes(int32_t batch, int32_t heads, int32_t seqlen_kv, int32_t dtype,
                           const MlaCfg* cfg) {
  g_last_error.clear();   // a 0 result with no error text means "no workspace needed"
  if (check_shape(batch, heads, seqlen_kv, dtype) != MLA_OK) return 0;
  Resolved r{};
  if (resolve(batch, heads, seqlen_kv, cfg, &r) != MLA_OK) return 0;
  return workspace_for(batch, heads, r);
}

}  // extern "C"

namespace mla {
namespace {

// Validate one decode call and fill the launch arguments.  `need_inputs`
// is false for the combine-only entry point (q/q_pe/kv/k_pe unused).
int prepare(const char* fn, const void* q, const void* q_pe, const void* kv, const void* k_pe,
            void* out, float* lse, const void* workspace, size_t workspace_bytes, int batch,
            int heads, int seqlen_kv, int dtype, const MlaCfg* cfg, void* stream, bool need_inputs,
            DecodeArgs* a, Resolved* r, size_t* need) {
  int rc = check_shape(batch, heads, seqlen_kv, dtype);
  if (rc != MLA_OK) return rc;
  if ((need_inputs && (!q || !q_pe || !kv || !k_pe)) || !out) {
    set_error("%s: null tensor pointer", fn);
    return MLA_ERR_ARG;
  }
  if ((need_inputs && (!aligned16(q) || !aligned16(q_pe) || !aligned16(kv) || !aligned16(k_pe))) ||
      !aligned16(out)) {
    set_error("%s: tensor pointers must be 16-byte aligned", fn);
    return MLA_ERR_ARG;
  }
  rc = resolve(batch, heads, seqlen_kv, cfg, r);
  if (rc != MLA_OK) return rc;
  *need = workspace_for(batch, heads, *r);
  if (*need > 0 && (workspace == nullptr || workspace_bytes < *need ||
                    (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)) {
    set_error("%s: workspace needs %zu bytes, 256-byte aligned (got %zu at %p)", fn, *need,
              workspace_bytes, workspace);
    return MLA_ERR_WORKSPACE;
  }
  *a = DecodeArgs{};
  a->q = q;
  a->q_pe = q_pe;
  a->kv = kv;
  a->k_pe = k_pe;
  a->out = out;
  a->out_dtype = dtype;
  a->lse = lse;
  a->batch = batch;
  a->heads = heads;
  a->seqlen_kv = seqlen_kv;
  a->dtype = dtype;
  a->softmax_scale = (cfg != nullptr && cfg->softmax_scale != 0.f) ? cfg->softmax_scale
                                                                   : 1.0f / sqrtf((float)kQkDim);
  if (!(a->softmax_scale > 0.f) || !isfinite(a->softmax_scale)) {
    set_error("%s: softmax_scale must be finite and > 0", fn);
    return MLA_ERR_ARG;
  }
  a->plan = r->plan;
  a->stream = static_cast<cudaStream_t>(stream);
  if (*need > 0) {
    char* base = static_cast<char*>(const_cast<void*>(workspace));
    if (r->kernel == MLA_KERNEL_TC) {
      a->status = reinterpret_cast<uint32_t*>(base);
      a->counters = reinterpret_cast<uint32_t*>(base + kStatusBytes);
      base += kStatusBytes + counter_bytes(batch, heads);
    }
    if (r->plan.needs_combine) {
      const size_t rows = part_rows(batch, heads, *r);
      a->part_lse = reinterpret_cast<float*>(base);
      a->part_o = reinterpret_cast<float*>(base + align_up(rows * sizeof(float), 256));
    }
  }
  return MLA_OK;
}

}  // namespace

int check_decode_call(const char* fn, const void* q, const void* q_pe, const void* kv, const void* k_pe,
                      const void* out, int batch, int heads, int seqlen_kv, int dtype, const MlaCfg* cfg) {
  int rc = check_shape(batch, heads, seqlen_kv, dtype);
  if (rc != MLA_OK) return rc;
  if (!q || !q_pe || !kv || !k_pe || !out) {
    set_error("%s: null tensor pointer", fn);
    return MLA_ERR_ARG;
  }
  if (!aligned16(q) || !aligned16(q_pe) || !aligned16(kv) || !aligned16(k_pe) || !aligned16(out)) {
    set_error("%s: tensor pointers must be 16-byte aligned", fn);
    return MLA_ERR_ARG;
  }
  if (cfg != nullptr && cfg->softmax_scale != 0.f && (!(cfg->softmax_scale > 0.f) || !isfinite(cfg->softmax_scale))) {
    set_error("%s: softmax_scale must be finite and > 0", fn);
    return MLA_ERR_ARG;
  }
  Resolved r{};
  return resolve(batch, heads, seqlen_kv, cfg, &r);
}

namespace {

int run_splitkv(const char* fn, const DecodeArgs& a, const Resolved& r) {
  const cudaError_t err =
      r.kernel == MLA_KERNEL_SIMT ? launch_simt_decode(a) : launch_sm100_decode(a, r.tc_variant);
  if (err != cudaSuccess) {
    set_error("%s: decode launch failed: %s", fn, cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

int run_combine_ws(const char* fn, const DecodeArgs& a, const Resolved& r) {
  // the decode kernel wrote out/lse itself: single-split plans, and tensor-core
  // plans whose split sequences it merged (variant 0: split between a few CTA
  // pairs; variant 2: merged by all their pairs in a cooperative launch)
  if (!r.plan.needs_combine || (r.kernel == MLA_KERNEL_TC && r.tc_variant != 1)) return MLA_OK;
  const cudaError_t err =
      r.kernel == MLA_KERNEL_TC
          ? launch_sm100_combine(a)
          : launch_combine(a.part_lse, a.part_o, r.plan.ns, a.batch, a.heads, a.out, a.lse,
                           a.out_dtype, a.stream);
  if (err != cudaSuccess) {
    set_error("%s: combine launch failed: %s", fn, cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

}  // namespace
}  // namespace mla

extern "C" {

int32_t mla_decode_fwd(const void* q, const void* q_pe, const void* kv, const void* k_pe,
                       void* out, float* lse, void* workspace, size_t workspace_bytes,
                       int32_t batch, int32_t heads, int32_t seqlen_kv, int32_t dtype,
                       const MlaCfg* cfg, void* stream) {
  DecodeArgs a;
  Resolved r;
  size_t need = 0;
  int rc = prepare("mla_decode_fwd", q, q_pe, kv, k_pe, out, lse, workspace, workspace_bytes, batch,
                   heads, seqlen_kv, dtype, cfg, stream, true, &a, &r, &need);
  if (rc != MLA_OK) return rc;
  rc = run_splitkv("mla_decode_fwd", a, r);
  if (rc != MLA_OK) return rc;
  return run_combine_ws("mla_decode_fwd", a, r);
}

int32_t mla_decode_fp8kv(const void* q, const void* q_pe, const void* kv_fp8, const void* k_pe,
                         float kv_scale, void* out, float* lse, void* workspace, size_t workspace_bytes,
                         int32_t batch, int32_t heads, int32_t seqlen_kv, int32_t dtype, const MlaCfg* cfg,
                         void* stream) {
  const char* fn = "mla_decode_fp8kv";
  MlaCfg c{};
  if (cfg != nullptr) c = *cfg;
  if (c.kernel == MLA_KERNEL_SIMT) {
    set_error("%s: runs on the tensor-core kernel only (kernel = auto or tc)", fn);
    return MLA_ERR_UNSUPPORTED;
  }
  c.kernel = MLA_KERNEL_TC;
  if (!(kv_scale > 0.f) || !isfinite(kv_scale)) {
    set_error("%s: kv_scale must be finite and > 0", fn);
    return MLA_ERR_ARG;
  }
  DecodeArgs a;
  Resolved r;
  size_t need = 0;
  int rc = prepare(fn, q, q_pe, kv_fp8, k_pe, out, lse, workspace, workspace_bytes, batch, heads, seqlen_kv,
                   dtype, &c, stream, true, &a, &r, &need);
  if (rc != MLA_OK) return rc;
  a.kv_fp8 = 1;
  a.kv_scale = kv_scale;
  rc = run_splitkv(fn, a, r);
  if (rc != MLA_OK) return rc;
  return run_combine_ws(fn, a, r);
}

int32_t mla_decode_partial(const void* q, const void* q_pe, const void* kv, const void* k_pe,
                           float* o, float* lse, void* workspace, size_t workspace_bytes,
                           int32_t batch, int32_t heads, int32_t seqlen_kv, int32_t dtype,
                           const MlaCfg* cfg, void* stream) {
  if (lse == nullptr) {
    set_error("mla_decode_partial: lse is required");
    return MLA_ERR_ARG;
  }
  DecodeArgs a;
  Resolved r;
  size_t need = 0;
  int rc = prepare("mla_decode_partial", q, q_pe, kv, k_pe, o, lse, workspace, workspace_bytes, batch,
                   heads, seqlen_kv, dtype, cfg, stream, true, &a, &r, &need);
  if (rc != MLA_OK) return rc;
  a.out_dtype = MLA_DTYPE_F32;
  rc = run_splitkv("mla_decode_partial", a, r);
  if (rc != MLA_OK) return rc;
  return run_combine_ws("mla_decode_partial", a, r);
}

// The sequence split's gather buffers of a call: checks and the PeerRows view.
static int seqsplit_view(const char* fn, void* const* bufs, int32_t world, int32_t rank, uint32_t epoch,
                         int32_t batch, int32_t heads, PeerRows* x) {
  if (bufs == nullptr || world < 1 || world > kSeqMaxWorld || rank < 0 || rank >= world || epoch == 0 ||
      batch < 1 || heads < 1) {
    set_error("%s: bad argument (world %d, rank %d, epoch %u, batch %d, heads %d)", fn, world, rank, epoch, batch,
              heads);
    return MLA_ERR_ARG;
  }
  *x = PeerRows{};
  for (int q = 0; q < world; ++q) {
    if (bufs[q] == nullptr || (reinterpret_cast<uintptr_t>(bufs[q]) & 255u) != 0) {
      set_error("%s: buffer %d is null or not 256-byte aligned", fn, q);
      return MLA_ERR_ARG;
    }
    x->bufs[q] = static_cast<float*>(bufs[q]);
  }
  x->chunk = seq_chunk_floats(batch, heads);
  x->header = seq_header_offset(world, batch, heads);
  x->ll_rows = seq_ll_rows_offset(world, batch, heads);
  x->ll_lse = seq_ll_lse_offset(world, batch, heads);
  x->rows_pad = seq_rows_pad(batch, heads);
  x->world = world;
  x->rank = rank;
  x->par = (int)(epoch & 1u);
  x->epoch = epoch;
  return MLA_OK;
}

int32_t mla_seqsplit_decode(const void* q, const void* q_pe, const void* kv_part, const void* k_pe_part, void* out,
                            float* lse, void* workspace, size_t workspace_bytes, int32_t batch, int32_t heads,
                            int32_t seqlen_part, int32_t dtype, void* const* bufs, int32_t world, int32_t rank,
                            uint32_t epoch, const MlaCfg* cfg, void* stream) {
  const char* fn = "mla_seqsplit_decode";
  PeerRows x;
  int rc = seqsplit_view(fn, bufs, world, rank, epoch, batch, heads, &x);
  if (rc != MLA_OK) return rc;
  if (out == nullptr || !aligned16(out)) {
    set_error("%s: out is null or not 16-byte aligned", fn);
    return MLA_ERR_ARG;
  }
  // this rank's part decodes to float32 (O, LSE) in its own block of its own buffer
  float* own = x.bufs[rank] + ((size_t)x.par * world + rank) * x.chunk;
  float* own_lse = own + (size_t)batch * heads * kDim;
  DecodeArgs a;
  Resolved r;
  size_t need = 0;
  rc = prepare(fn, q, q_pe, kv_part, k_pe_part, own, own_lse, workspace, workspace_bytes, batch, heads, seqlen_part,
               dtype, cfg, stream, true, &a, &r, &need);
  if (rc != MLA_OK) return rc;
  a.out_dtype = MLA_DTYPE_F32;
  rc = run_splitkv(fn, a, r);
  if (rc != MLA_OK) return rc;
  // sequences split between many CTA pairs are merged from their pieces inside the
  // exchange launch; anything else is already in the block
  const bool pieces = r.kernel == MLA_KERNEL_TC && r.plan.needs_combine && r.tc_variant == 1;
  if (!pieces) {
    rc = run_combine_ws(fn, a, r);
    if (rc != MLA_OK) return rc;
  }
  const cudaError_t err = launch_seqsplit_combine(a, pieces, x, out, lse, dtype);
  if (err != cudaSuccess) {
    set_error("%s: exchange launch failed: %s", fn, cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

int32_t mla_seqsplit_merge(void* const* bufs, int32_t world, int32_t rank, uint32_t epoch, int32_t batch,
                           int32_t heads, void* out, float* lse, int32_t dtype, void* stream) {
  const char* fn = "mla_seqsplit_merge";
  PeerRows x;
  int rc = seqsplit_view(fn, bufs, world, rank, epoch, batch, heads, &x);
  if (rc != MLA_OK) return rc;
  if (out == nullptr || !aligned16(out)) {
    set_error("%s: out is null or not 16-byte aligned", fn);
    return MLA_ERR_ARG;
  }
  if (dtype != MLA_DTYPE_F16 && dtype != MLA_DTYPE_BF16 && dtype != MLA_DTYPE_F32) {
    set_error("%s: dtype must be 0, 1 or 2", fn);
    return MLA_ERR_ARG;
  }
  DecodeArgs a{};
  a.batch = batch;
  a.heads = heads;
  a.seqlen_kv = 1;
  a.stream = static_cast<cudaStream_t>(stream);
  const cudaError_t err = launch_seqsplit_combine(a, false, x, out, lse, dtype);
  if (err != cudaSuccess) {
    set_error("%s: launch failed: %s", fn, cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

int32_t mla_decode_splitkv(const void* q, const void* q_pe, const void* kv, const void* k_pe,
                           void* out, float* lse, void* workspace, size_t workspace_bytes,
                           int32_t batch, int32_t heads, int32_t seqlen_kv, int32_t dtype,
                           const MlaCfg* cfg, void* stream) {
  DecodeArgs a;
  Resolved r;
  size_t need = 0;
  const int rc = prepare("mla_decode_splitkv", q, q_pe, kv, k_pe, out, lse, workspace,
                         workspace_bytes, batch, heads, seqlen_kv, dtype, cfg, stream, true, &a, &r,
                         &need);
  if (rc != MLA_OK) return rc;
  return run_splitkv("mla_decode_splitkv", a, r);
}

int32_t mla_decode_combine_ws(void* out, float* lse, const void* workspace, size_t workspace_bytes,
                              int32_t batch, int32_t heads, int32_t seqlen_kv, int32_t dtype,
                              const MlaCfg* cfg, void* stream) {
  DecodeArgs a;
  Resolved r;
  size_t need = 0;
  const int rc = prepare("mla_decode_combine_ws", nullptr, nullptr, nullptr, nullptr, out, lse,
                         workspace, workspace_bytes, batch, heads, seqlen_kv, dtype, cfg, stream,
                         false, &a, &r, &need);
  if (rc != MLA_OK) return rc;
  return run_combine_ws("mla_decode_combine_ws", a, r);
}

int32_t mla_combine(const float* part_lse, const float* part_o, int32_t num_split, int32_t batch,
                    int32_t heads, void* out, float* lse, int32_t dtype, void* stream) {
  if (!part_lse || !part_o || !out) {
    set_error("mla_combine: null pointer");
    return MLA_ERR_ARG;
  }
  if (num_split < 1 || num_split > 8192 || batch < 1 || heads < 1) {
    set_error("mla_combine: bad num_split/batch/heads (%d, %d, %d)", num_split, batch, heads);
    return MLA_ERR_ARG;
  }
  if (dtype != MLA_DTYPE_F16 && dtype != MLA_DTYPE_BF16 && dtype != MLA_DTYPE_F32) {
    set_error("mla_combine: dtype must be 0, 1 or 2");
    return MLA_ERR_ARG;
  }
  if (!aligned16(part_o) || !aligned16(out)) {
    set_error("mla_combine: part_o and out must be 16-byte aligned");
    return MLA_ERR_ARG;
  }
  const cudaError_t err = launch_combine(part_lse, part_o, num_split, batch, heads, out, lse, dtype,
                                         static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    set_error("mla_combine: launch failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

int32_t mla_combine_strided(const float* part_lse, int64_t lse_split_stride, const float* part_o,
                            int64_t o_split_stride, int32_t num_split, int32_t batch, int32_t heads, void* out,
                            float* lse, int32_t dtype, void* stream) {
  if (!part_lse || !part_o || !out) {
    set_error("mla_combine_strided: null pointer");
    return MLA_ERR_ARG;
  }
  if (num_split < 1 || num_split > 8192 || batch < 1 || heads < 1) {
    set_error("mla_combine_strided: bad num_split/batch/heads (%d, %d, %d)", num_split, batch, heads);
    return MLA_ERR_ARG;
  }
  const int64_t rows = (int64_t)batch * heads;
  if (lse_split_stride < rows || o_split_stride < rows * kDim || o_split_stride % 4 != 0) {
    set_error("mla_combine_strided: split strides must cover a split (lse >= %lld, o >= %lld and a multiple "
              "of 4; got %lld, %lld)", (long long)rows, (long long)(rows * kDim), (long long)lse_split_stride,
              (long long)o_split_stride);
    return MLA_ERR_ARG;
  }
  if (dtype != MLA_DTYPE_F16 && dtype != MLA_DTYPE_BF16 && dtype != MLA_DTYPE_F32) {
    set_error("mla_combine_strided: dtype must be 0, 1 or 2");
    return MLA_ERR_ARG;
  }
  if (!aligned16(part_o) || !aligned16(out)) {
    set_error("mla_combine_strided: part_o and out must be 16-byte aligned");
    return MLA_ERR_ARG;
  }
  const cudaError_t err = launch_combine_strided(part_lse, (size_t)lse_split_stride, part_o, (size_t)o_split_stride,
                                                 num_split, batch, heads, out, lse, dtype,
                                                 static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    set_error("mla_combine_strided: launch failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

int32_t mla_selftest_wait_timeout(uint32_t* status, uint64_t* result, uint64_t limit_ns, void* stream) {
  if (!status || !result) {
    set_error("mla_selftest_wait_timeout: null pointer");
    return MLA_ERR_ARG;
  }
  if (limit_ns < 1000000ull || limit_ns > 100000000ull) {
    set_error("mla_selftest_wait_timeout: limit_ns must be in [1e6, 1e8] (got %llu)",
              (unsigned long long)limit_ns);
    return MLA_ERR_ARG;
  }
  const cudaError_t err = launch_wait_selftest(status, reinterpret_cast<unsigned long long*>(result), limit_ns,
                                               MLA_SELFTEST_STATUS, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    set_error("mla_selftest_wait_timeout: launch failed: %s", cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Ragged / paged decode (per-sequence KV lengths, optional page table).
// Workspace: [status 256 B][counters u32 x batch x groups x 4, padded][tile prefix
// sums u32 x (batch x groups + 1), padded][partial LSE][partial O].
// ---------------------------------------------------------------------------
namespace mla {
namespace {

struct PagedLayout {
  SplitPlan plan;
  size_t counters_off, cu_off, lse_off, o_off, total;
};

// Query side: batch x q_len x kv_heads query sequences of heads / kv_heads rows.
int paged_layout(const char* fn, int batch, int q_len, int heads, int kv_heads, int max_seqlen_kv, int dtype,
                 const MlaCfg* cfg, PagedLayout* L) {
  int rc = check_shape(batch, heads, max_seqlen_kv, dtype);
  if (rc != MLA_OK) return rc;
  if (q_len < 1 || kv_heads < 1 || heads % kv_heads != 0) {
    set_error("%s: q_len and kv_heads must be >= 1 with heads a multiple of kv_heads (q_len %d, heads %d, "
              "kv_heads %d)", fn, q_len, heads, kv_heads);
    return MLA_ERR_ARG;
  }
  MlaCfg c{};
  if (cfg != nullptr) c = *cfg;
  if (c.kernel == MLA_KERNEL_SIMT) {
    set_error("%s: runs on the tensor-core kernel only (kernel = auto or tc)", fn);
    return MLA_ERR_UNSUPPORTED;
  }
  if (!sm100_supports_ext(batch, q_len, heads, kv_heads, max_seqlen_kv)) {
    set_error("%s: shape outside the tensor-core kernel (batch %d, q_len %d, heads %d, kv_heads %d, "
              "max_seqlen_kv %d)", fn, batch, q_len, heads, kv_heads, max_seqlen_kv);
    return MLA_ERR_UNSUPPORTED;
  }
  const int qb = batch * q_len * kv_heads, g = heads / kv_heads;
  L->plan = sm100_plan_ragged(qb, g, max_seqlen_kv, c);
  const size_t vb = (size_t)qb * head_groups(g);
  const size_t rows = (size_t)L->plan.part_rows;
  L->counters_off = kStatusBytes;
  L->cu_off = L->counters_off + counter_bytes(qb, g);
  L->lse_off = L->cu_off + align_up((vb + 1) * sizeof(uint32_t), 256);
  L->o_off = L->lse_off + align_up(rows * sizeof(float), 256);
  L->total = L->o_off + rows * kDim * sizeof(float);
  return MLA_OK;
}

}  // namespace
}  // namespace mla

extern "C" {

size_t mla_paged_workspace_bytes(int32_t batch, int32_t heads, int32_t max_seqlen_kv, int32_t dtype,
                                 const MlaCfg* cfg) {
  return mla_decode_ext_workspace_bytes(batch, 1, heads, 1, max_seqlen_kv, dtype, cfg);
}

size_t mla_decode_ext_workspace_bytes(int32_t batch, int32_t q_len, int32_t heads, int32_t kv_heads,
                                      int32_t max_seqlen_kv, int32_t dtype, const MlaCfg* cfg) {
  g_last_error.clear();
  PagedLayout L;
  if (paged_layout("mla_decode_ext", batch, q_len, heads, kv_heads, max_seqlen_kv, dtype, cfg, &L) != MLA_OK)
    return 0;
  return L.total;
}

}  // extern "C"

namespace mla {
namespace {

int decode_ext(const char* fn, const void* q, const void* q_pe, const void* kv_cache, const void* k_pe_cache,
               const int32_t* block_table, const int32_t* cache_seqlens, void* out, float* lse, void* workspace,
               size_t workspace_bytes, int32_t batch, int32_t q_len, int32_t heads, int32_t kv_heads,
               int32_t max_seqlen_kv, int32_t page_size, int32_t num_pages, int32_t max_pages_per_seq,
               int32_t dtype, const MlaCfg* cfg, void* stream, bool kv_fp8 = false, float kv_scale = 1.f) {
  if (kv_fp8 && (!(kv_scale > 0.f) || !isfinite(kv_scale))) {
    set_error("%s: kv_scale must be finite and > 0", fn);
    return MLA_ERR_ARG;
  }
  PagedLayout L;
  int rc = paged_layout(fn, batch, q_len, heads, kv_heads, max_seqlen_kv, dtype, cfg, &L);
  if (rc != MLA_OK) return rc;
  if (!q || !q_pe || !kv_cache || !k_pe_cache || !out) {
    set_error("%s: null pointer", fn);
    return MLA_ERR_ARG;
  }
  if (!aligned16(q) || !aligned16(q_pe) || !aligned16(kv_cache) || !aligned16(k_pe_cache) || !aligned16(out)) {
    set_error("%s: tensor pointers must be 16-byte aligned", fn);
    return MLA_ERR_ARG;
  }
  if (block_table != nullptr) {
    if (page_size < 64 || page_size % 64 != 0 || num_pages < 1 || max_pages_per_seq < 1 ||
        (long long)num_pages * page_size >= (1ll << 31) - 256) {
      set_error("%s: page_size must be a positive multiple of 64, with num_pages x page_size rows "
                "below 2^31 (page_size %d, num_pages %d, max_pages_per_seq %d)",
                fn, page_size, num_pages, max_pages_per_seq);
      return MLA_ERR_ARG;
    }
  }
  if (workspace == nullptr || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
    set_error("%s: workspace needs %zu bytes, 256-byte aligned (got %zu at %p)", fn, L.total, workspace_bytes,
              workspace);
    return MLA_ERR_WORKSPACE;
  }
  DecodeArgs a{};
  a.q = q;
  a.q_pe = q_pe;
  a.kv = kv_cache;
  a.k_pe = k_pe_cache;
  a.out = out;
  a.out_dtype = dtype;
  a.lse = lse;
  a.batch = batch;
  a.heads = heads;
  a.q_len = q_len;
  a.kv_heads = kv_heads;
  a.kv_fp8 = kv_fp8 ? 1 : 0;
  a.kv_scale = kv_scale;
  a.seqlen_kv = max_seqlen_kv;
  a.dtype = dtype;
  a.softmax_scale = (cfg != nullptr && cfg->softmax_scale != 0.f) ? cfg->softmax_scale : 1.0f / sqrtf((float)kQkDim);
  if (!(a.softmax_scale > 0.f) || !isfinite(a.softmax_scale)) {
    set_error("%s: softmax_scale must be finite and > 0", fn);
    return MLA_ERR_ARG;
  }
  a.plan = L.plan;
  a.stream = static_cast<cudaStream_t>(stream);
  char* base = static_cast<char*>(workspace);
  a.status = reinterpret_cast<uint32_t*>(base);
  a.counters = reinterpret_cast<uint32_t*>(base + L.counters_off);
  a.cu_tiles = reinterpret_cast<uint32_t*>(base + L.cu_off);
  a.part_lse = reinterpret_cast<float*>(base + L.lse_off);
  a.part_o = reinterpret_cast<float*>(base + L.o_off);
  a.seqlens = cache_seqlens;
  a.block_table = block_table;
  a.page_size = block_table != nullptr ? page_size : 0;
  a.num_pages = block_table != nullptr ? num_pages : 0;
  a.max_pages = block_table != nullptr ? max_pages_per_seq : 0;
  // lengths clamped as the decode kernel does; sequences split between many pairs
  // merged in the kernel (cooperative launch) or by the combine launch
  const int variant = (sm100_coop_available() && cfg != nullptr && cfg->combine_groups < 0) ? 2 : 1;
  cudaError_t err = launch_sm100_ragged_plan(a);
  if (err == cudaSuccess) err = launch_sm100_decode(a, variant);
  if (err == cudaSuccess && variant == 1) err = launch_sm100_combine(a);
  if (err != cudaSuccess) {
    set_error("%s: launch failed: %s", fn, cudaGetErrorString(err));
    return MLA_ERR_CUDA;
  }
  return MLA_OK;
}

}  // namespace
}  // namespace mla

extern "C" {

int32_t mla_decode_paged(const void* q, const void* q_pe, const void* kv_cache, const void* k_pe_cache,
                         const int32_t* block_table, const int32_t* cache_seqlens, void* out, float* lse,
                         void* workspace, size_t workspace_bytes, int32_t batch, int32_t heads,
                         int32_t max_seqlen_kv, int32_t page_size, int32_t num_pages,
                         int32_t max_pages_per_seq, int32_t dtype, const MlaCfg* cfg, void* stream) {
  if (cache_seqlens == nullptr) {
    set_error("mla_decode_paged: null pointer");
    return MLA_ERR_ARG;
  }
  return decode_ext("mla_decode_paged", q, q_pe, kv_cache, k_pe_cache, block_table, cache_seqlens, out, lse,
                    workspace, workspace_bytes, batch, 1, heads, 1, max_seqlen_kv, page_size, num_pages,
                    max_pages_per_seq, dtype, cfg, stream);
}

int32_t mla_decode_ext(const void* q, const void* q_pe, const void* kv_cache, const void* k_pe_cache,
                       const int32_t* block_table, const int32_t* cache_seqlens, void* out, float* lse,
                       void* workspace, size_t workspace_bytes, int32_t batch, int32_t q_len, int32_t heads,
                       int32_t kv_heads, int32_t max_seqlen_kv, int32_t page_size, int32_t num_pages,
                       int32_t max_pages_per_seq, int32_t dtype, const MlaCfg* cfg, void* stream) {
  return decode_ext("mla_decode_ext", q, q_pe, kv_cache, k_pe_cache, block_table, cache_seqlens, out, lse,
                    workspace, workspace_bytes, batch, q_len, heads, kv_heads, max_seqlen_kv, page_size, num_pages,
                    max_pages_per_seq, dtype, cfg, stream);
}

int32_t mla_decode_ext_fp8kv(const void* q, const void* q_pe, const void* kv_fp8, const void* k_pe_cache,
                             float kv_scale, const int32_t* block_table, const int32_t* cache_seqlens, void* out,
                             float* lse, void* workspace, size_t workspace_bytes, int32_t batch, int32_t q_len,
                             int32_t heads, int32_t kv_heads, int32_t max_seqlen_kv, int32_t page_size,
                             int32_t num_pages, int32_t max_pages_per_seq, int32_t dtype, const MlaCfg* cfg,
                             void* stream) {
  return decode_ext("mla_decode_ext_fp8kv", q, q_pe, kv_fp8, k_pe_cache, block_table, cache_seqlens, out, lse,
                    workspace, workspace_bytes, batch, q_len, heads, kv_heads, max_seqlen_kv, page_size, num_pages,
                    max_pages_per_seq, dtype, cfg, stream, true, kv_scale);
}

}  // extern "C"
