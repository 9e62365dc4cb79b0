// fa_noalloc.cu -- attention forward split over key ranges, with the fp32
// partial results kept in a fixed scratch array that the library owns.
//
// Who this is for: code that cannot call cudaMalloc (or any allocator) at the
// point where it runs attention -- an engine that hands every byte of device
// memory to its own pool at start-up, a latency-critical loop where an
// allocation (which can synchronise the device) is not allowed, or a plain
// C/FFI caller that only holds pointers to its own tensors.  The split form
// otherwise needs per-split partial O/LSE buffers; here they live in
// `g_split_scratch`, a file-scope device array reserved when the library is
// loaded, so the call allocates nothing.  The caller passes only q, k, v and
// the outputs, exactly as for fa_sm100_fwd.
//
// The work is: for each of n_splits contiguous key ranges, the attention
// kernel (fa_sm100_fwd with fp32 output and the range's key offset) writes a
// partial (O, LSE) into the scratch; then fa_sm100_lse_merge combines the
// parts into the caller's O and LSE.  No counterpart exists in the reference.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "fa_sm100.h"

namespace {

// 64 MiB: enough for n_splits x batch x seqlen_q x heads up to ~32K
// (row, head) pairs at 4 splits with head_dim 128.  Every GPU that loads the
// library keeps this reserved until the process exits.
constexpr size_t kSplitScratchBytes = size_t{64} << 20;
constexpr int kMaxSplits = 16;  // the merge kernel combines at most 16 parts
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_split_scratch[kSplitScratchBytes];

struct ScratchState {
  std::once_flag once;
  unsigned char* ptr = nullptr;
  int status = FA_OK;
};
ScratchState g_scratch[kMaxDevices];

// Device address of the scratch array on the current device.  In host code
// `g_split_scratch` names a host-side shadow, never the device memory; the
// real address comes from cudaGetSymbolAddress, taken once per device with
// that device current (the first call on each device does this set-up).
int scratch_on_current_device(unsigned char** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return FA_ERR_INVALID_ARG;
  ScratchState& s = g_scratch[dev];
  std::call_once(s.once, [&] {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_split_scratch) != cudaSuccess || addr == nullptr) {
      s.status = FA_ERR_CUDA;
      return;
    }
    s.ptr = static_cast<unsigned char*>(addr);
  });
  *out = s.ptr;
  return s.status;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace

extern "C" {

size_t fa_sm100_split_scratch_bytes(void) { return kSplitScratchBytes; }

int fa_sm100_fwd_split_noalloc(const FaParams* p, int32_t n_splits, void* stream) {
  int rc = fa_sm100_check_params(p);
  if (rc != FA_OK) return rc;
  if (n_splits < 1 || n_splits > kMaxSplits) return FA_ERR_INVALID_ARG;
  if (p->out_f32 != 0) return FA_ERR_UNSUPPORTED;  // the merge writes the input type
  if (p->batch == 0 || p->seqlen_q == 0) return FA_OK;
  // The merge writes LSE as (heads, seqlen_q) per batch entry: the caller's
  // LSE rows must be contiguous per head.
  if (p->lse != nullptr && p->lse_head_stride != p->seqlen_q) return FA_ERR_UNSUPPORTED;

  const int64_t b = p->batch, sq = p->seqlen_q, h = p->heads, d = p->head_dim;
  const int64_t sk = p->seqlen_k;
  // Key ranges of whole 128-key blocks, as equal as possible.
  int64_t per = (sk + n_splits - 1) / n_splits;
  per = (per + 127) / 128 * 128;
  if (per == 0) per = 128;
  const int parts = sk == 0 ? 1 : static_cast<int>((sk + per - 1) / per);

  const size_t o_part = static_cast<size_t>(b * sq * h * d) * sizeof(float);
  const size_t l_part = round_up(static_cast<size_t>(b * h * sq) * sizeof(float), 256);
  if (static_cast<size_t>(parts) * (o_part + l_part) > kSplitScratchBytes) return FA_ERR_SCRATCH_LIMIT;

  unsigned char* scratch = nullptr;
  rc = scratch_on_current_device(&scratch);
  if (rc != FA_OK) return rc;

  // Every partial is written in full (rows that see no key of a range get
  // O = 0, LSE = -inf), so nothing in the scratch has to start at zero.
  const float* o_parts[kMaxSplits];
  const float* l_parts[kMaxSplits];
  for (int i = 0; i < parts; ++i) {
    float* o_i = reinterpret_cast<float*>(scratch + static_cast<size_t>(i) * o_part);
    float* l_i = reinterpret_cast<float*>(scratch + static_cast<size_t>(parts) * o_part + static_cast<size_t>(i) * l_part);
    const int64_t k0 = static_cast<int64_t>(i) * per;
    const int64_t k1 = sk < k0 + per ? sk : k0 + per;
    FaParams q = *p;
    q.k = sk == 0 ? p->k : static_cast<const uint16_t*>(p->k) + k0 * p->k_row_stride;
    q.v = sk == 0 ? p->v : static_cast<const uint16_t*>(p->v) + k0 * p->v_row_stride;
    q.seqlen_k = static_cast<int32_t>(k1 - k0);
    q.k_pos_offset = p->k_pos_offset + k0;
    q.o = o_i;
    q.o_batch_stride = sq * h * d;
    q.o_row_stride = h * d;
    q.o_head_stride = d;
    q.out_f32 = 1;
    q.lse = l_i;
    q.lse_batch_stride = h * sq;
    q.lse_head_stride = sq;
    rc = fa_sm100_fwd(&q, stream);
    if (rc != FA_OK) return rc;
    o_parts[i] = o_i;
    l_parts[i] = l_i;
  }
  for (int64_t bi = 0; bi < b; ++bi) {
    const float* ob[kMaxSplits];
    const float* lb[kMaxSplits];
    for (int i = 0; i < parts; ++i) {
      ob[i] = o_parts[i] + bi * sq * h * d;
      lb[i] = l_parts[i] + bi * h * sq;
    }
    void* o_out = static_cast<uint16_t*>(p->o) + bi * p->o_batch_stride;
    float* lse_out = p->lse != nullptr ? p->lse + bi * p->lse_batch_stride : nullptr;
    rc = fa_sm100_lse_merge(ob, lb, parts, static_cast<int32_t>(sq), static_cast<int32_t>(h),
                            static_cast<int32_t>(d), o_out, p->o_row_stride, p->o_head_stride, p->is_bf16,
                            lse_out, stream);
    if (rc != FA_OK) return rc;
  }
  return FA_OK;
}

}  // extern "C"
