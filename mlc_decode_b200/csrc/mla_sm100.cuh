// Interface of the tcgen05/TMA/TMEM decode kernel (mla_sm100.cu).
#pragma once

#include "mla_common.cuh"

namespace mla {

// Groups of 128 heads per sequence: the tensor-core kernel's work units.
int head_groups(int heads);

// True when the tensor-core kernel covers this shape (q_len query positions per
// sequence, heads query heads over kv_heads KV heads).
bool sm100_supports(int batch, int heads, int seqlen_kv);
bool sm100_supports_ext(int batch, int q_len, int heads, int kv_heads, int seqlen_kv);

// Query-side shape the kernel sees for a call (DecodeArgs q_len / kv_heads).
QShape qshape(const DecodeArgs& a);

// Split plan (and kernel variant) the tensor-core kernel uses for this shape.
// Variant 0: every sequence is whole in one CTA pair or split between at most 3
// and merged in the kernel; 1: some sequence is split between more pairs and a
// combine launch merges it; 2: such sequences are merged in the kernel by all
// their pairs together (cooperative launch; one launch per call).
SplitPlan sm100_plan(int batch, int heads, int seqlen_kv, const MlaCfg& cfg, int* variant);

// True when the current device takes cooperative launches (variant 2).
bool sm100_coop_available();

// Enqueue the tensor-core split-KV kernel; partials go to a.part_o/a.part_lse.
// Variant 2 launches cooperatively; if the driver refuses that launch, the plain
// launch and the combine launch run instead (same result).
cudaError_t launch_sm100_decode(const DecodeArgs& a, int variant);

// Plan of a ragged call (per-sequence lengths): max_seqlen_kv bounds every length.
SplitPlan sm100_plan_ragged(int batch, int heads, int max_seqlen_kv, const MlaCfg& cfg);

// Enqueue the ragged plan kernel (tile prefix sums into a.cu_tiles, empty outputs).
cudaError_t launch_sm100_ragged_plan(const DecodeArgs& a);

// Enqueue the combine of split sequences the decode kernel did not merge itself.
cudaError_t launch_sm100_combine(const DecodeArgs& a);

// Enqueue the bounded-wait self-test (one CTA pair; see mla_selftest_wait_timeout).
cudaError_t launch_wait_selftest(uint32_t* status, unsigned long long* result, uint64_t limit_ns,
                                 uint32_t code, cudaStream_t stream);

}  // namespace mla
