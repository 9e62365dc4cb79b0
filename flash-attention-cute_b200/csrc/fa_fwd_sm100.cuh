// fa_fwd_sm100.cuh -- warp-specialised attention forward for B200 (sm_100a).
//
// Replaces the reference's SM80 kernel (csrc/flash_fwd_kernel.cuh:32-298) and
// its tile traits (csrc/flash_fwd_traits.h:21-75).  Same mathematics: online
// softmax over key blocks with exp2 and the scale folded into one FMA
// (kernel.cuh:208-235), causal mask `key > query` (kernel.cuh:174-188), P
// rounded to the input type before the P.V product (kernel.cuh:246-252) and a
// zero-sum guard at the end (kernel.cuh:277).  Different machinery:
//
//   * one CTA owns two 128-row query tiles (256 rows) of one (batch, head);
//   * warp 8 is the TMA producer: Q tiles once, then K_j, V_j into a ring of
//     NS shared-memory slots (128-byte swizzle, mbarrier expect-tx);
//   * warp 9 is the MMA issuer: tcgen05.mma S_t = Q_t K_j^T (both operands in
//     shared memory, accumulator in TMEM) and O_t += P_t V_j (P read straight
//     from TMEM, V in shared memory as an MN-major operand -- no transpose);
//   * warps 0-3 / 4-7 are the softmax warpgroups of tile 0 / tile 1: thread r
//     owns query row r, which is TMEM lane r.  They read S with tcgen05.ld,
//     mask (tail / causal), update the running max, rescale O in TMEM only
//     when the max grew by more than 2^8 (the final division uses the same
//     stale max, so the result is exact), write P over S as 16-bit pairs and
//     finally normalise O and store O and LSE.
//
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D).
// Every mbarrier wait is bounded; on expiry the CTA records FA_ERR_TIMEOUT,
// drains its in-flight copies and MMAs, frees TMEM and exits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include "sm100_ptx.cuh"

namespace fa {

struct FwdKernelParams {
  CUtensorMap tm_q;  // (d, head, seq, batch) box (64, 1, 128, 1), 128B swizzle
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  void* o;
  float* lse;
  int32_t* error_flag;
  int64_t o_batch_stride, o_row_stride, o_head_stride;
  int64_t lse_batch_stride, lse_head_stride;
  int64_t q_pos_offset, k_pos_offset;
  uint64_t timeout_ns;
  int seqlen_q, seqlen_k, heads, batch;
  int num_m_blocks;  // ceil(seqlen_q / 256)
  float scale;       // softmax scale
  float scale_log2;  // softmax scale * log2(e)
};

constexpr int kBlockM = 128;  // query rows per tile (= TMEM lanes)
constexpr int kBlockN = 128;  // keys per block
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct FwdTraits {
  static constexpr int kTileBytes = kBlockM * D * 2;  // Q, K and V tiles are all 128 x D
  static constexpr int kBoxBytes = kBlockM * 128;     // one 64-column (128-byte) TMA box
  static constexpr int kNumBoxes = D / 64;
  static constexpr int kStages = D == 128 ? 4 : 8;
  static constexpr int kNumBarriers = 2 + 2 * kStages + 2 + 2 + 2 + 1;
  static constexpr int kSmemBytes =
      1024 /*alignment slack*/ + (2 + kStages) * kTileBytes + kNumBarriers * 8 + 16;
  static constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO0 = 256, kColO1 = 256 + D;
};

template <int D, bool kBf16, bool kCausal>
__global__ void __launch_bounds__(kThreads, 1) fa_fwd_sm100_kernel(const __grid_constant__ FwdKernelParams p) {
  using Tr = FwdTraits<D>;
  constexpr int NS = Tr::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + 2 * Tr::kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + NS * Tr::kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 2;
  uint64_t* kv_empty = kv_full + NS;
  uint64_t* s_full = kv_empty + NS;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* mma_drain = pv_done + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  volatile int* vabort = abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work unit: (m_block, head, batch); causal launches the heaviest
  // (last) query blocks first so the tail of the grid is short.
  const int bh_count = p.heads * p.batch;
  int m_block, bh;
  if constexpr (kCausal) {
    m_block = p.num_m_blocks - 1 - static_cast<int>(blockIdx.x / bh_count);
    bh = static_cast<int>(blockIdx.x % bh_count);
  } else {
    m_block = static_cast<int>(blockIdx.x % p.num_m_blocks);
    bh = static_cast<int>(blockIdx.x / p.num_m_blocks);
  }
  const int head = bh % p.heads;
  const int batch = bh / p.heads;
  const int m0 = m_block * 2 * kBlockM;

  int n_blocks = (p.seqlen_k + kBlockN - 1) / kBlockN;
  if constexpr (kCausal) {
    const int64_t last_row = static_cast<int64_t>(min(m0 + 2 * kBlockM, p.seqlen_q)) - 1;
    const int64_t max_key = p.q_pos_offset - p.k_pos_offset + last_row;  // inclusive
    if (max_key < 0) {
      n_blocks = 0;
    } else if (max_key / kBlockN + 1 < n_blocks) {
      n_blocks = static_cast<int>(max_key / kBlockN) + 1;
    }
  }

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&q_full[0]), 1);
    mbar_init(smem_u32(&q_full[1]), 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(smem_u32(&kv_full[i]), 1);
      mbar_init(smem_u32(&kv_empty[i]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&s_full[t]), 1);
      mbar_init(smem_u32(&p_full[t]), kBlockM);
      mbar_init(smem_u32(&pv_done[t]), 1);
    }
    mbar_init(smem_u32(mma_drain), 1);
    // A timeout recorded by an earlier CTA or launch makes this CTA a no-op
    // (sticky, like a CUDA sticky error) until the host clears the flag.
    const int poisoned = p.error_flag != nullptr ? *reinterpret_cast<volatile int32_t*>(p.error_flag) : 0;
    *abort_flag = poisoned != 0 ? 2 : 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint64_t tmo = p.timeout_ns;
  const bool live = *vabort == 0;
  if (!live) n_blocks = 0;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_blocks > 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      for (int t = 0; t < 2; ++t) {
        const uint32_t bar = smem_u32(&q_full[t]);
        mbar_arrive_expect_tx(bar, Tr::kTileBytes);
        for (int bx = 0; bx < Tr::kNumBoxes; ++bx) {
          tma_load_4d(smem_u32(sQ + t * Tr::kTileBytes + bx * Tr::kBoxBytes), &p.tm_q, bar, bx * 64,
                      head, m0 + t * kBlockM, batch, pol_q);
        }
      }
      int it = 0;
      bool ok = true;
      for (int j = 0; j < n_blocks && ok; ++j) {
        for (int kv = 0; kv < 2; ++kv, ++it) {
          const int slot = it % NS;
          const uint32_t fill = static_cast<uint32_t>(it / NS);
          if (!mbar_wait(smem_u32(&kv_empty[slot]), (fill & 1u) ^ 1u, vabort, tmo)) {
            ok = false;
            break;
          }
          const uint32_t bar = smem_u32(&kv_full[slot]);
          mbar_arrive_expect_tx(bar, Tr::kTileBytes);
          const CUtensorMap* tm = kv == 0 ? &p.tm_k : &p.tm_v;
          for (int bx = 0; bx < Tr::kNumBoxes; ++bx) {
            tma_load_4d(smem_u32(sKV + slot * Tr::kTileBytes + bx * Tr::kBoxBytes), tm, bar, bx * 64,
                        head, j * kBlockN, batch, pol_kv);
          }
        }
      }
      if (!ok) {
        // Error path: let every copy already issued land before the CTA exits.
        const uint64_t drain_ns = 200ull * 1000 * 1000;
        int zero = 0;
        volatile int* never = &zero;
        mbar_wait(smem_u32(&q_full[0]), 0, never, drain_ns);
        mbar_wait(smem_u32(&q_full[1]), 0, never, drain_ns);
        for (int s = 0; s < NS && s < it; ++s) {
          const int last = s + ((it - 1 - s) / NS) * NS;  // last fill index of slot s
          mbar_wait(smem_u32(&kv_full[s]), static_cast<uint32_t>(last / NS) & 1u, never, drain_ns);
        }
      }
    }
  } else if (warp == 9) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && n_blocks > 0) {
      constexpr uint32_t kIdescS = make_idesc_f16(kBlockM, kBlockN, kBf16, false);
      constexpr uint32_t kIdescO = make_idesc_f16(kBlockM, D, kBf16, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t kv_addr = smem_u32(sKV);
      bool issued = false;

      auto issue_s = [&](int t, uint32_t k_tile) {
        // S_t = Q_t K^T : reduction over D in steps of 16 (32 bytes inside
        // a 128-byte swizzle row; a new 64-column box every 4 steps).
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * Tr::kBoxBytes + (kk & 3) * 32;
          const uint64_t a = make_sw128_desc(q_addr + t * Tr::kTileBytes + off, 16, 1024);
          const uint64_t b = make_sw128_desc(k_tile + off, 16, 1024);
          umma_ss(tmem + (t ? Tr::kColS1 : Tr::kColS0), a, b, kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, uint32_t v_tile, bool acc) {
        // O_t += P_t V : reduction over the 128 keys in steps of 16.  P is
        // read from TMEM (16 keys = 8 columns of packed pairs); V is an
        // MN-major operand: 8-row groups 1024 B apart (SBO), 64-column boxes
        // kBoxBytes apart (LBO).
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          const uint64_t b = make_sw128_desc(v_tile + kk * 16 * 128, Tr::kBoxBytes, 1024);
          umma_ts(tmem + (t ? Tr::kColO1 : Tr::kColO0), tmem + (t ? Tr::kColS1 : Tr::kColS0) + kk * 8, b, kIdescO,
                  (acc || kk > 0) ? 1u : 0u);
        }
      };

      bool ok = mbar_wait(smem_u32(&q_full[0]), 0, vabort, tmo) &&
                mbar_wait(smem_u32(&q_full[1]), 0, vabort, tmo);
      int it = 0;
      if (ok) {
        const int slot = it % NS;
        ok = mbar_wait(smem_u32(&kv_full[slot]), static_cast<uint32_t>(it / NS) & 1u, vabort, tmo);
        if (ok) {
          tc_fence_after();
          const uint32_t k_tile = kv_addr + slot * Tr::kTileBytes;
          issue_s(0, k_tile);
          umma_commit(smem_u32(&s_full[0]));
          issue_s(1, k_tile);
          umma_commit(smem_u32(&s_full[1]));
          umma_commit(smem_u32(&kv_empty[slot]));
          issued = true;
          ++it;
        }
      }
      for (int j = 0; j < n_blocks && ok; ++j) {
        const uint32_t ph = static_cast<uint32_t>(j) & 1u;
        const int vslot = it % NS;
        ok = mbar_wait(smem_u32(&kv_full[vslot]), static_cast<uint32_t>(it / NS) & 1u, vabort, tmo);
        if (!ok) break;
        const uint32_t v_tile = kv_addr + vslot * Tr::kTileBytes;
        ++it;
        ok = mbar_wait(smem_u32(&p_full[0]), ph, vabort, tmo);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, v_tile, j > 0);
        umma_commit(smem_u32(&pv_done[0]));
        ok = mbar_wait(smem_u32(&p_full[1]), ph, vabort, tmo);
        if (!ok) break;
        tc_fence_after();
        issue_pv(1, v_tile, j > 0);
        umma_commit(smem_u32(&pv_done[1]));
        umma_commit(smem_u32(&kv_empty[vslot]));
        if (j + 1 < n_blocks) {
          const int kslot = it % NS;
          ok = mbar_wait(smem_u32(&kv_full[kslot]), static_cast<uint32_t>(it / NS) & 1u, vabort, tmo);
          if (!ok) break;
          const uint32_t k_tile = kv_addr + kslot * Tr::kTileBytes;
          ++it;
          // P_t of block j sits in the S_t columns: S_t of block j+1 may only
          // be written once the P.V product that reads it has completed.
          ok = mbar_wait(smem_u32(&pv_done[0]), ph, vabort, tmo);
          if (!ok) break;
          tc_fence_after();
          issue_s(0, k_tile);
          umma_commit(smem_u32(&s_full[0]));
          ok = mbar_wait(smem_u32(&pv_done[1]), ph, vabort, tmo);
          if (!ok) break;
          tc_fence_after();
          issue_s(1, k_tile);
          umma_commit(smem_u32(&s_full[1]));
          umma_commit(smem_u32(&kv_empty[kslot]));
        }
      }
      if (issued) {
        // Make sure every MMA this thread issued has finished before TMEM is
        // released (matters only on the error path).
        umma_commit(smem_u32(mma_drain));
        int zero = 0;
        volatile int* never = &zero;
        mbar_wait(smem_u32(mma_drain), 0, never, 200ull * 1000 * 1000);
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int t = warp >> 2;       // query tile of this warpgroup
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;
    const int row = m0 + t * kBlockM + r;  // local query row
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_addr + (t == 0 ? Tr::kColS0 : Tr::kColS1);
    const uint32_t tO = tmem + lane_addr + (t == 0 ? Tr::kColO0 : Tr::kColO1);
    const float c = p.scale_log2;
    // Highest key index this row may see (causal), in local key numbering.
    const int64_t key_lim = static_cast<int64_t>(row) + p.q_pos_offset - p.k_pos_offset;

    float m_run = -INFINITY;
    float l_run = 0.f;    // exact fp32 row sum (for the LSE)
    float lr_run = 0.f;   // sum of the rounded P actually multiplied (bf16 only)
    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      // Every lane polls; the outcome is made warp-uniform because the
      // tcgen05.ld / st that follow are warp-collective.
      const bool got = __all_sync(0xffffffffu,
                                  mbar_wait(smem_u32(&s_full[t]), static_cast<uint32_t>(j) & 1u, vabort, tmo));
      if (!got) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kBlockN];
      {
        uint32_t raw[32];
#pragma unroll
        for (int cc = 0; cc < kBlockN / 32; ++cc) {
          tmem_ld32(tS + cc * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[cc * 32 + i] = __uint_as_float(raw[i]);
        }
      }
      // Mask keys past the end of the sequence and, if causal, keys after the row.
      const int col0 = j * kBlockN;
      int64_t valid = static_cast<int64_t>(p.seqlen_k) - col0;
      if constexpr (kCausal) {
        const int64_t cl = key_lim - col0 + 1;
        valid = cl < valid ? cl : valid;
      }
      if (valid < kBlockN) {
#pragma unroll
        for (int i = 0; i < kBlockN; ++i) {
          if (i >= valid) s[i] = -INFINITY;
        }
      }
      float mx = s[0];
#pragma unroll
      for (int i = 1; i < kBlockN; ++i) mx = fmaxf(mx, s[i]);
      const float m_new = fmaxf(m_run, mx);
      bool warp_rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_run = m_new;
      } else {
        const bool need =
            (m_new > m_run) && (m_run == -INFINITY || (m_new - m_run) * c > kRescaleThreshold);
        warp_rescale = __any_sync(0xffffffffu, need);
        if (need) {
          alpha = ex2_approx((m_run - m_new) * c);
          m_run = m_new;
          l_run *= alpha;
          lr_run *= alpha;
        }
      }
      const float neg = (m_run == -INFINITY) ? 0.f : -m_run * c;
      float sum = 0.f;
      float sum_r = 0.f;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2_approx(fmaf(s[h * 32 + 2 * i], c, neg));
          const float p1 = ex2_approx(fmaf(s[h * 32 + 2 * i + 1], c, neg));
          pk[i] = pack2<kBf16>(p0, p1);
          sum += p0 + p1;
          if constexpr (kBf16) {
            // O is normalised by the sum of the bf16 values the MMA actually
            // uses (the reference divides by the unrounded sum, kernel.cuh:233,
            // which with bf16's 8-bit mantissa costs up to ~3e-3 on rows that
            // see few keys); the LSE keeps the exact fp32 sum.
            sum_r += __uint_as_float(pk[i] << 16) + __uint_as_float(pk[i] & 0xffff0000u);
          }
        }
        tmem_st16(tS + h * 16, pk);
      }
      if (warp_rescale) {
        // O_t of block j-1 is complete (S_t of block j was committed after its
        // P.V product) and the next P.V waits for p_full: rescale it in place.
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[32];
          tmem_ld32(tO + cc * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + cc * 32, o);
        }
      }
      tmem_wait_st();
      l_run += sum;
      lr_run += sum_r;
      tc_fence_before();
      mbar_arrive(smem_u32(&p_full[t]));
    }

    // ---- epilogue: O /= l, store O (and LSE).
    bool have_o = ok && n_blocks > 0;
    if (have_o) {
      have_o = __all_sync(0xffffffffu, mbar_wait(smem_u32(&pv_done[t]),
                                                 static_cast<uint32_t>(n_blocks - 1) & 1u, vabort, tmo));
      tc_fence_after();
    }
    const float l_norm = kBf16 ? lr_run : l_run;
    const float inv = l_norm > 0.f ? 1.f / l_norm : 0.f;
    using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
    T* orow = reinterpret_cast<T*>(p.o) + static_cast<int64_t>(batch) * p.o_batch_stride +
              static_cast<int64_t>(row) * p.o_row_stride + static_cast<int64_t>(head) * p.o_head_stride;
    const bool row_ok = live && row < p.seqlen_q;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld32(tO + cc * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (row_ok) {
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          packed[i] = pack2<kBf16>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
        }
      }
    }
    if (row_ok && p.lse != nullptr) {
      const float lse = l_run > 0.f ? fmaf(m_run, p.scale, logf(l_run)) : -INFINITY;
      p.lse[static_cast<int64_t>(batch) * p.lse_batch_stride + static_cast<int64_t>(head) * p.lse_head_stride +
            row] = lse;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *vabort == 1 && p.error_flag != nullptr) {
    atomicExch(p.error_flag, -6 /* FA_ERR_TIMEOUT */);
  }
}

}  // namespace fa
