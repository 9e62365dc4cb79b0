// fa_bwd_sm100.cuh -- attention backward for B200 (sm_100a).
//
// Gradients of O = softmax(scale * Q K^T [+ causal mask]) V given dO and the
// forward's LSE (the reference has no backward; this extends the path the
// forward's LSE output was designed for).  With P = exp(scale * S - LSE),
// D = rowsum(dO * O), dP = dO V^T and dS = P * (dP - D):
//     dV = P^T dO,   dK = scale * dS^T Q,   dQ = scale * dS K.
//
// Three kernels, no atomics (results are deterministic):
//   * fa_bwd_dot_kernel     D per (batch, head, query row);
//   * fa_bwd_dq_kernel      one 128-row query tile per CTA: for each key
//                           block, S = Q K^T and dP = dO V^T (tcgen05.mma,
//                           both operands in shared memory, accumulators in
//                           TMEM), the 8 elementwise warps form dS and write
//                           it back to TMEM as 16-bit pairs, then
//                           dQ += dS K (A read from TMEM, K as an MN-major
//                           operand -- the forward's O += P V form); K and V
//                           stream through rings of their own, since K stays
//                           in use until dQ's product and V only until dP's;
//   * fa_bwd_dkdv_kernel    one 128-key tile per CTA (all query heads of its
//                           K/V head under GQA), each step's 128 queries in
//                           two halves of 64: S^T = K Q^T and dP^T = V dO^T
//                           with keys on the TMEM lanes, the elementwise
//                           warps write P^T and dS^T as 16-bit pairs, then
//                           dV += P^T dO and dK += dS^T Q -- one half's
//                           elementwise work overlapping the other half's
//                           MMAs.
// TMA tiles, swizzles, descriptors, bounded waits and the error flag are the
// forward kernel's (fa_fwd_sm100.cuh / sm100_ptx.cuh).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include "fa_fwd_sm100.cuh"
#include "sm100_ptx.cuh"

namespace fa {

struct BwdKernelParams {
  CUtensorMap tm_q;   // (d, head, seq, batch), box (64, 1, 128, 1), SW128
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  CUtensorMap tm_do;  // same shape and layout as q
  const float* lse;   // (batch, heads, seqlen_q), row stride 1
  const float* dvec;  // D, (batch, heads, seqlen_q) contiguous
  void* dq;
  void* dk;
  void* dv;
  int32_t* error_flag;
  int64_t dq_batch_stride, dq_row_stride, dq_head_stride;
  int64_t dk_batch_stride, dk_row_stride, dk_head_stride;
  int64_t dv_batch_stride, dv_row_stride, dv_head_stride;
  int64_t lse_batch_stride, lse_head_stride;
  int64_t q_pos_offset, k_pos_offset;
  uint64_t timeout_ns;
  int seqlen_q, seqlen_k, heads, heads_k, batch, heads_per_kv;
  int num_q_blocks, num_k_blocks;  // 128-row blocks
  float scale, scale_log2;
};

// D[b, h, i] = sum_d dO[b, i, h, d] * O[b, i, h, d]  (one warp per row).
template <int D, bool kBf16>
__global__ void __launch_bounds__(256) fa_bwd_dot_kernel(const void* __restrict__ dout, const void* __restrict__ out,
                                                       float* __restrict__ dvec, int batch, int seqlen, int heads,
                                                       int64_t do_b, int64_t do_r, int64_t do_h, int64_t o_b,
                                                       int64_t o_r, int64_t o_h) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  const int64_t warp_id = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= static_cast<int64_t>(batch) * heads * seqlen) return;
  const int row = static_cast<int>(warp_id % seqlen);
  const int head = static_cast<int>((warp_id / seqlen) % heads);
  const int b = static_cast<int>(warp_id / (static_cast<int64_t>(seqlen) * heads));
  const T* a = reinterpret_cast<const T*>(dout) + b * do_b + row * do_r + head * do_h;
  const T* c = reinterpret_cast<const T*>(out) + b * o_b + row * o_r + head * o_h;
  float acc = 0.f;
#pragma unroll
  for (int e = lane; e < D; e += 32) acc = fmaf(static_cast<float>(a[e]), static_cast<float>(c[e]), acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) dvec[warp_id] = acc;  // (b, h, row) order: warp_id = (b*heads + head)*seqlen + row
}


template <int D>
struct BwdTraits {
  static constexpr int kTileBytes = kBlockM * D * 2;  // every tile is 128 rows x D
  static constexpr int kBoxBytes = kBlockM * 128;
  static constexpr int kNumBoxes = D / 64;
  // K and V have rings of their own: K_j stays in its slot until dQ += dS_j K_j
  // has run (after block j's elementwise work), V_j only until dP_j, so K gets
  // the deeper ring and its next load is not held up behind that late release.
  static constexpr int kStagesK = D == 128 ? 3 : 5;
  static constexpr int kStagesV = D == 128 ? 2 : 3;
  // q_full, k_full/empty[NK], v_full/empty[NV], s_full, s_free, ds_full[2], ds_free[2], acc_done, mma_drain
  static constexpr int kNumBarriers = 1 + 2 * (kStagesK + kStagesV) + 8;
  static constexpr int kSmemBytes =
      1024 + (2 + kStagesK + kStagesV) * kTileBytes + kNumBarriers * 8 + 16;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// P = exp2(s * c + neg) masked to the first `valid` entries, then
// dS = P * (dP - dd), packed to 16-bit pairs.  (One 64-key half row.)
// kMask = false: the caller knows every entry is visible.
template <bool kBf16, bool kMask>
__device__ __forceinline__ void ds_pack(const float (&s)[64], const float (&dp)[64], float c, float neg, float dd,
                                        int64_t valid, uint32_t (&pk)[32]) {
  const float2 c2 = make_float2(c, c);
  const float2 n2 = make_float2(neg, neg);
  const float2 d2 = make_float2(dd, dd);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 x = __ffma2_rn(make_float2(s[2 * i], s[2 * i + 1]), c2, n2);
    float2 pe = make_float2(ex2_approx(x.x), ex2_approx(x.y));
    if (kMask) {
      if (2 * i >= valid) pe.x = 0.f;
      if (2 * i + 1 >= valid) pe.y = 0.f;
    }
    const float2 g = __fmul2_rn(pe, __fadd2_rn(make_float2(dp[2 * i], dp[2 * i + 1]), make_float2(-d2.x, -d2.y)));
    pk[i] = pack2<kBf16>(g.x, g.y);
  }
}

// The dK/dV kernel's elementwise step for one thread's 32 query columns of
// a half: P^T = exp2(s * c + nl) with the first `lo` queries masked (kMask),
// dS^T = P^T * (dP^T - dd), both packed to 16-bit pairs.
template <bool kBf16, bool kMask>
__device__ __forceinline__ void pds_pack(const float (&sv)[32], const float (&dpv)[32], float c, const float* nl,
                                         const float* ddv, int64_t lo, uint32_t (&pk_p)[16], uint32_t (&pk_s)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 x = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), make_float2(c, c),
                                make_float2(nl[2 * i], nl[2 * i + 1]));
    float2 pe = make_float2(ex2_approx(x.x), ex2_approx(x.y));
    if (kMask) {
      if (2 * i < lo) pe.x = 0.f;
      if (2 * i + 1 < lo) pe.y = 0.f;
    }
    const float2 g = __fmul2_rn(pe, make_float2(dpv[2 * i] - ddv[2 * i], dpv[2 * i + 1] - ddv[2 * i + 1]));
    pk_p[i] = pack2<kBf16>(pe.x, pe.y);
    pk_s[i] = pack2<kBf16>(g.x, g.y);
  }
}

template <int D, bool kBf16, bool kCausal>
__global__ void __launch_bounds__(kThreads, 1) fa_bwd_dq_kernel(const __grid_constant__ BwdKernelParams p) {
  using Tr = BwdTraits<D>;
  constexpr int NK = Tr::kStagesK;
  constexpr int NV = Tr::kStagesV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = smem + Tr::kTileBytes;
  uint8_t* sKV = smem + 2 * Tr::kTileBytes;  // K slots [0, NK), then V slots [NK, NK + NV)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + (NK + NV) * Tr::kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + NK;
  uint64_t* v_full = k_empty + NK;
  uint64_t* v_empty = v_full + NV;
  uint64_t* s_full = v_empty + NV;  // S and dP of the block are in TMEM
  uint64_t* s_free = s_full + 1;     // the elementwise warps hold S and dP in registers
  uint64_t* ds_full = s_free + 1;    // [2] dS of the buffer's block is in TMEM
  uint64_t* ds_free = ds_full + 2;   // [2] dQ += dS K of the buffer's last block is done
  uint64_t* acc_done = ds_free + 2;  // every dQ MMA has completed
  uint64_t* mma_drain = acc_done + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  volatile int* vabort = abort_flag;
  // S, dP, the dQ accumulator and two dS buffers (16-bit pairs) all have
  // their own columns, so the next block's S and dP are computed while the
  // elementwise warps still work on this block.
  constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 256, kColDS = 256 + D;
  static_assert(kColDS + 128 <= 512, "TMEM budget");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh_count = p.heads * p.batch;
  int m_block, bh;
  if constexpr (kCausal) {
    m_block = p.num_q_blocks - 1 - static_cast<int>(blockIdx.x / bh_count);
    bh = static_cast<int>(blockIdx.x % bh_count);
  } else {
    m_block = static_cast<int>(blockIdx.x % p.num_q_blocks);
    bh = static_cast<int>(blockIdx.x / p.num_q_blocks);
  }
  const int head = bh % p.heads;
  const int batch = bh / p.heads;
  const int kv_head = head / p.heads_per_kv;
  const int m0 = m_block * kBlockM;

  int n_blocks = (p.seqlen_k + kBlockN - 1) / kBlockN;
  if constexpr (kCausal) {
    const int64_t last_row = static_cast<int64_t>(min(m0 + kBlockM, p.seqlen_q)) - 1;
    const int64_t max_key = p.q_pos_offset - p.k_pos_offset + last_row;
    if (max_key < 0) {
      n_blocks = 0;
    } else if (max_key / kBlockN + 1 < n_blocks) {
      n_blocks = static_cast<int>(max_key / kBlockN) + 1;
    }
  }

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int i = 0; i < NK; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1);
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(smem_u32(&v_full[i]), 1);
      mbar_init(smem_u32(&v_empty[i]), 1);
    }
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(s_free), 2 * kBlockM);
    mbar_init(smem_u32(&ds_full[0]), 2 * kBlockM);
    mbar_init(smem_u32(&ds_full[1]), 2 * kBlockM);
    mbar_init(smem_u32(&ds_free[0]), 1);
    mbar_init(smem_u32(&ds_free[1]), 1);
    mbar_init(smem_u32(acc_done), 1);
    mbar_init(smem_u32(mma_drain), 1);
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

  auto teardown = [&]() {
    __syncwarp();
    tc_fence_before();
    asm volatile("barrier.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (warp == 9) {
      __syncwarp();
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && *vabort == 1 && p.error_flag != nullptr) {
      atomicExch(p.error_flag, -6 /* FA_ERR_TIMEOUT */);
    }
  };

  if (warp >= 8) {
    reg_dealloc<kRegsAux>();
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, vabort, tmo));
    };
    const bool leader = lane == 0;
    if (warp == 8 && n_blocks > 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      if (leader) {
        prefetch_tmap(&p.tm_q);
        prefetch_tmap(&p.tm_do);
        prefetch_tmap(&p.tm_k);
        prefetch_tmap(&p.tm_v);
        mbar_arrive_expect_tx(smem_u32(q_full), 2 * Tr::kTileBytes);
        for (int bx = 0; bx < Tr::kNumBoxes; ++bx) {
          tma_load_4d(smem_u32(sQ + bx * Tr::kBoxBytes), &p.tm_q, smem_u32(q_full), bx * 64, head, m0, batch, pol_q);
          tma_load_4d(smem_u32(sDO + bx * Tr::kBoxBytes), &p.tm_do, smem_u32(q_full), bx * 64, head, m0, batch,
                      pol_q);
        }
      }
      int loads[2] = {0, 0};  // K and V loads issued
      bool ok = true;
      for (int j = 0; j < n_blocks && ok; ++j) {
        for (int kv = 0; kv < 2 && ok; ++kv) {  // K_j, then V_j
          const int ns = kv == 0 ? NK : NV;
          const int slot = j % ns;
          const uint32_t fill = static_cast<uint32_t>(j / ns);
          uint64_t* empty = kv == 0 ? &k_empty[slot] : &v_empty[slot];
          if (!wait_all(empty, (fill & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          if (leader) {
            const uint32_t bar = smem_u32(kv == 0 ? &k_full[slot] : &v_full[slot]);
            mbar_arrive_expect_tx(bar, Tr::kTileBytes);
            const CUtensorMap* tm = kv == 0 ? &p.tm_k : &p.tm_v;
            uint8_t* dst = sKV + (kv == 0 ? slot : NK + slot) * Tr::kTileBytes;
            for (int bx = 0; bx < Tr::kNumBoxes; ++bx) {
              tma_load_4d(smem_u32(dst + bx * Tr::kBoxBytes), tm, bar, bx * 64, kv_head, j * kBlockN, batch, pol_kv);
            }
          }
          ++loads[kv];
        }
      }
      if (!ok) {
        // Error path: let every copy already issued land before the CTA exits
        // (the last fill of each slot of both rings).
        const uint64_t drain_ns = 200ull * 1000 * 1000;
        int zero = 0;
        volatile int* never = &zero;
        mbar_wait(smem_u32(q_full), 0, never, drain_ns);
        for (int j2 = loads[0] - NK > 0 ? loads[0] - NK : 0; j2 < loads[0]; ++j2) {
          mbar_wait(smem_u32(&k_full[j2 % NK]), static_cast<uint32_t>(j2 / NK) & 1u, never, drain_ns);
        }
        for (int j2 = loads[1] - NV > 0 ? loads[1] - NV : 0; j2 < loads[1]; ++j2) {
          mbar_wait(smem_u32(&v_full[j2 % NV]), static_cast<uint32_t>(j2 / NV) & 1u, never, drain_ns);
        }
      }
    } else if (warp == 9 && n_blocks > 0) {
      // --------------------------------------------------------------- MMA
      constexpr uint32_t kIdescS = make_idesc_f16(kBlockM, kBlockN, kBf16, false);
      constexpr uint32_t kIdescDQ = make_idesc_f16(kBlockM, D, kBf16, true);
      const uint64_t desc_q = make_sw128_desc(smem_u32(sQ), 16, 1024);
      const uint64_t desc_do = make_sw128_desc(smem_u32(sDO), 16, 1024);
      const uint64_t desc_kv0 = make_sw128_desc(smem_u32(sKV), 16, 1024);              // K-major (rows = keys)
      const uint64_t desc_mn0 = make_sw128_desc(smem_u32(sKV), Tr::kBoxBytes, 1024);  // MN-major (N = d)
      constexpr uint64_t kSlotStep = Tr::kTileBytes >> 4;
      bool issued = false;
      auto issue_ss = [&](uint32_t dcol, uint64_t desc_a, int slot) {
        // D = A B^T over head_dim (the forward's S = Q K^T form)
        if (leader) {
          const uint64_t b0 = desc_kv0 + slot * kSlotStep;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t off = ((kk >> 2) * Tr::kBoxBytes + (kk & 3) * 32) >> 4;
            umma_ss(tmem + dcol, desc_a + off, b0 + off, kIdescS, kk > 0 ? 1u : 0u);
          }
        }
        __syncwarp();
      };
      auto issue_dq = [&](int kslot, uint32_t acol, bool acc) {
        // dQ += dS K: dS from TMEM (8 columns of pairs per 16 keys), K_j as an
        // MN-major operand (the forward's O += P V form).
        if (leader) {
          const uint64_t b0 = desc_mn0 + kslot * kSlotStep;
#pragma unroll
          for (int kk = 0; kk < kBlockN / 16; ++kk) {
            umma_ts(tmem + kColDQ, tmem + acol + kk * 8, b0 + kk * (2048 >> 4), kIdescDQ,
                    (acc || kk > 0) ? 1u : 0u);
          }
        }
        __syncwarp();
      };
      auto commit = [&](uint64_t* bar) {
        if (leader) umma_commit(smem_u32(bar));
        __syncwarp();
      };
      bool ok = wait_all(q_full, 0);
      int jn = 0;  // next block whose S and dP are to be issued
      int kslot_cur = 0, kslot_next = 0;
      // S and dP of block jn (block 0 first).  issue_ss takes a slot index
      // into the K slots followed by the V slots.
      auto issue_sdp = [&](int& kslot) {
        kslot = jn % NK;
        const int vslot = jn % NV;
        bool r = wait_all(&k_full[kslot], static_cast<uint32_t>(jn / NK) & 1u);
        r = r && wait_all(&v_full[vslot], static_cast<uint32_t>(jn / NV) & 1u);
        ++jn;
        if (!r) return false;
        tc_fence_after();
        issue_ss(kColS, desc_q, kslot);         // S = Q K_j^T
        issue_ss(kColDP, desc_do, NK + vslot);  // dP = dO V_j^T
        commit(s_full);
        commit(&v_empty[vslot]);
        return true;
      };
      if (ok && n_blocks > 0) {
        ok = issue_sdp(kslot_cur);
        issued = ok;
      }
      for (int j = 0; j < n_blocks && ok; ++j) {
        const uint32_t ph = static_cast<uint32_t>(j) & 1u;
        if (j + 1 < n_blocks) {
          // S/dP of block j+1 once the elementwise warps hold block j's
          ok = wait_all(s_free, ph) && issue_sdp(kslot_next);
          if (!ok) break;
        }
        // per-buffer barriers: block j's is at most one phase ahead of this wait
        ok = wait_all(&ds_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u);
        if (!ok) break;
        tc_fence_after();
        issue_dq(kslot_cur, kColDS + (j & 1) * 64, j > 0);  // dQ += dS_j K_j
        commit(&ds_free[j & 1]);
        commit(&k_empty[kslot_cur]);
        kslot_cur = kslot_next;
      }
      if (issued) {
        commit(acc_done);
        commit(mma_drain);
        int zero = 0;
        volatile int* never = &zero;
        mbar_wait(smem_u32(mma_drain), 0, never, 200ull * 1000 * 1000);
      }
    }
    teardown();
    return;
  } else {
    // --------------------------------------------------------- elementwise
    reg_alloc<kRegsSoftmax>();
    const int key_half = lane >> 4;
    const int r = 32 * (warp & 3) + 16 * (warp >> 2) + (lane & 15);
    const uint32_t lane_addr = static_cast<uint32_t>(32 * (warp & 3) + 16 * (warp >> 2)) << 16;
    constexpr int kHalfD = D / 2;
    const int row = m0 + r;
    const bool row_ok = live && row < p.seqlen_q;
    const float lse_row = row_ok ? p.lse[static_cast<int64_t>(batch) * p.lse_batch_stride +
                                         static_cast<int64_t>(head) * p.lse_head_stride + row]
                                 : -INFINITY;
    const float dd = row_ok ? p.dvec[(static_cast<int64_t>(batch) * p.heads + head) * p.seqlen_q + row] : 0.f;
    // A row with no visible key (LSE = -inf) has P = 0 everywhere.
    const bool row_live = row_ok && lse_row != -INFINITY;
    const float c = p.scale_log2;
    const float neg = row_live ? -lse_row * 1.4426950408889634f : -INFINITY;
    const int64_t key_lim = static_cast<int64_t>(row) + p.q_pos_offset - p.k_pos_offset;
    bool ok = true;
#pragma unroll 1
    for (int j = 0; j < n_blocks; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(s_full), static_cast<uint32_t>(j) & 1u, vabort, tmo))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[64], dpv[64];
      {
        uint32_t raw[64];
        tmem_ld_16x32bx2_x64_sync<64>(tmem + lane_addr + kColS, raw);
#pragma unroll
        for (int i = 0; i < 64; ++i) sv[i] = __uint_as_float(raw[i]);
        tmem_ld_16x32bx2_x64_sync<64>(tmem + lane_addr + kColDP, raw);
#pragma unroll
        for (int i = 0; i < 64; ++i) dpv[i] = __uint_as_float(raw[i]);
      }
      // S and dP are in registers: the MMA warp may compute the next block's.
      tc_fence_before();
      mbar_arrive(smem_u32(s_free));
      const int col0 = j * kBlockN + key_half * 64;
      int64_t valid = row_live ? static_cast<int64_t>(p.seqlen_k) - col0 : 0;
      if constexpr (kCausal) {
        const int64_t cl = key_lim - col0 + 1;
        valid = cl < valid ? cl : valid;
      }
      uint32_t pk[32];
      if (__any_sync(0xffffffffu, valid < 64)) {
        ds_pack<kBf16, true>(sv, dpv, c, neg, dd, valid, pk);
      } else {
        ds_pack<kBf16, false>(sv, dpv, c, neg, dd, valid, pk);
      }
      // dS buffer j&1 is free once dQ += dS_{j-2} K_{j-2} has completed.
      if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(smem_u32(&ds_free[j & 1]),
                                                      static_cast<uint32_t>((j - 2) >> 1) & 1u, vabort, tmo))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // lanes 0-15 columns [0,32) of the buffer, lanes 16-31 the same columns
      // of the second key half (32 further).
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t chunk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) chunk[i] = pk[16 * h + i];
        tmem_st_16x32bx2_x16<32>(tmem + lane_addr + kColDS + (j & 1) * 64 + h * 16, chunk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&ds_full[j & 1]));
    }
    // ---- epilogue: dQ = scale * (dS K), in the input type.
    bool have = ok && n_blocks > 0;
    if (have) {
      have = __all_sync(0xffffffffu, mbar_wait(smem_u32(acc_done), 0, vabort, tmo));
      tc_fence_after();
    }
    using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
    const float sc = have ? p.scale : 0.f;
#pragma unroll
    for (int cc = 0; cc < kHalfD / 32; ++cc) {
      uint32_t o[32];
      if (have) {
        tmem_ld_16x32bx2_x32_sync<kHalfD>(tmem + lane_addr + kColDQ + cc * 32, o);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (row_ok) {
        T* dst = reinterpret_cast<T*>(p.dq) + static_cast<int64_t>(batch) * p.dq_batch_stride +
                 static_cast<int64_t>(row) * p.dq_row_stride + static_cast<int64_t>(head) * p.dq_head_stride +
                 key_half * kHalfD + cc * 32;
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          d4[i] = make_uint4(pack2<kBf16>(__uint_as_float(o[8 * i + 0]) * sc, __uint_as_float(o[8 * i + 1]) * sc),
                             pack2<kBf16>(__uint_as_float(o[8 * i + 2]) * sc, __uint_as_float(o[8 * i + 3]) * sc),
                             pack2<kBf16>(__uint_as_float(o[8 * i + 4]) * sc, __uint_as_float(o[8 * i + 5]) * sc),
                             pack2<kBf16>(__uint_as_float(o[8 * i + 6]) * sc, __uint_as_float(o[8 * i + 7]) * sc));
        }
      }
    }
    teardown();
    return;
  }
}

template <int D>
struct BwdKVTraits {
  static constexpr int kTileBytes = kBlockM * D * 2;
  static constexpr int kBoxBytes = kBlockM * 128;
  static constexpr int kNumBoxes = D / 64;
  // stage = Q_i, dO_i tiles + 128 floats of -LSE*log2(e) + 128 floats of D
  static constexpr int kStageBytes = 2 * kTileBytes + 1024;
  static constexpr int kStages = D == 128 ? 2 : 4;
  // kv_full, st_full/empty[NS], s_full[2], p_full[2], acc_done, mma_drain
  static constexpr int kNumBarriers = 1 + 2 * kStages + 6;
  static constexpr int kSmemBytes = 1024 + 2 * kTileBytes + kStages * kStageBytes + kNumBarriers * 8 + 16;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 256 + D;
  static_assert(kColDK + D <= 512, "TMEM budget");
};

template <int D, bool kBf16, bool kCausal>
__global__ void __launch_bounds__(kThreads, 1) fa_bwd_dkdv_kernel(const __grid_constant__ BwdKernelParams p) {
  using Tr = BwdKVTraits<D>;
  constexpr int NS = Tr::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + Tr::kTileBytes;
  uint8_t* sStage = smem + 2 * Tr::kTileBytes;  // [NS] x {Q, dO, nl[128], dd[128]}
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + NS * Tr::kStageBytes);
  uint64_t* kv_full = bars;
  uint64_t* st_full = kv_full + 1;
  uint64_t* st_empty = st_full + NS;
  // Each step's 128 query columns are processed as two halves of 64, so the
  // elementwise work on one half overlaps the other half's MMAs.
  uint64_t* s_full = st_empty + NS;  // [2] S^T and dP^T of the half are in TMEM
  uint64_t* p_full = s_full + 2;     // [2] P^T and dS^T of the half are in TMEM
  uint64_t* acc_done = p_full + 2;
  uint64_t* mma_drain = acc_done + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  volatile int* vabort = abort_flag;
  auto stage_q = [&](int slot) { return sStage + slot * Tr::kStageBytes; };
  auto stage_do = [&](int slot) { return sStage + slot * Tr::kStageBytes + Tr::kTileBytes; };
  auto stage_nl = [&](int slot) { return reinterpret_cast<float*>(sStage + slot * Tr::kStageBytes + 2 * Tr::kTileBytes); };
  auto stage_dd = [&](int slot) {
    return reinterpret_cast<float*>(sStage + slot * Tr::kStageBytes + 2 * Tr::kTileBytes + 512);
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // ---- work unit: (128-key block, K/V head, batch)
  const int n_block = static_cast<int>(blockIdx.x % p.num_k_blocks);
  const int bh = static_cast<int>(blockIdx.x / p.num_k_blocks);
  const int kv_head = bh % p.heads_k;
  const int batch = bh / p.heads_k;
  const int n0 = n_block * kBlockN;
  // first query block with a row that sees a key of this block
  int i_start = 0;
  if constexpr (kCausal) {
    const int64_t t = static_cast<int64_t>(n0) + p.k_pos_offset - p.q_pos_offset - (kBlockM - 1);
    i_start = t <= 0 ? 0 : static_cast<int>((t + kBlockM - 1) / kBlockM);
  }
  const int q_blocks = i_start < p.num_q_blocks ? p.num_q_blocks - i_start : 0;
  int n_steps = q_blocks * p.heads_per_kv;  // (group head, query block) pairs

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(kv_full), 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(smem_u32(&st_full[i]), 1);
      mbar_init(smem_u32(&st_empty[i]), 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(smem_u32(&s_full[h]), 1);
      mbar_init(smem_u32(&p_full[h]), 2 * kBlockM);
    }
    mbar_init(smem_u32(acc_done), 1);
    mbar_init(smem_u32(mma_drain), 1);
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
  if (!live) n_steps = 0;

  auto teardown = [&]() {
    __syncwarp();
    tc_fence_before();
    asm volatile("barrier.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (warp == 9) {
      __syncwarp();
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && *vabort == 1 && p.error_flag != nullptr) {
      atomicExch(p.error_flag, -6 /* FA_ERR_TIMEOUT */);
    }
  };

  if (warp >= 8) {
    reg_dealloc<kRegsAux>();
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, vabort, tmo));
    };
    const bool leader = lane == 0;
    if (warp == 8 && n_steps > 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol_kv = l2_policy_evict_first();
      const uint64_t pol_q = l2_policy_evict_last();
      if (leader) {
        prefetch_tmap(&p.tm_q);
        prefetch_tmap(&p.tm_do);
        prefetch_tmap(&p.tm_k);
        prefetch_tmap(&p.tm_v);
        mbar_arrive_expect_tx(smem_u32(kv_full), 2 * Tr::kTileBytes);
        for (int bx = 0; bx < Tr::kNumBoxes; ++bx) {
          tma_load_4d(smem_u32(sK + bx * Tr::kBoxBytes), &p.tm_k, smem_u32(kv_full), bx * 64, kv_head, n0, batch,
                      pol_kv);
          tma_load_4d(smem_u32(sV + bx * Tr::kBoxBytes), &p.tm_v, smem_u32(kv_full), bx * 64, kv_head, n0, batch,
                      pol_kv);
        }
      }
      bool ok = true;
      int it = 0;
      for (; it < n_steps && ok; ++it) {
        const int g = it / q_blocks;
        const int qi = i_start + it % q_blocks;
        const int head = kv_head * p.heads_per_kv + g;
        const int slot = it % NS;
        const uint32_t fill = static_cast<uint32_t>(it / NS);
        // -LSE*log2(e) and D of the block's 128 query rows (bounded loads;
        // rows past the end, or that saw no key, get -inf so P = 0), read
        // before waiting for the slot so their latency overlaps the wait.
        float v_nl[4], v_d[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = qi * kBlockM + lane * 4 + e;
          v_nl[e] = -INFINITY;
          v_d[e] = 0.f;
          if (row < p.seqlen_q) {
            const float l = p.lse[static_cast<int64_t>(batch) * p.lse_batch_stride +
                                  static_cast<int64_t>(head) * p.lse_head_stride + row];
            v_nl[e] = l == -INFINITY ? -INFINITY : -l * 1.4426950408889634f;
            v_d[e] = p.dvec[(static_cast<int64_t>(batch) * p.heads + head) * p.seqlen_q + row];
          }
        }
        if (!wait_all(&st_empty[slot], (fill & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        float* nl = stage_nl(slot);
        float* ddv = stage_dd(slot);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          nl[lane * 4 + e] = v_nl[e];
          ddv[lane * 4 + e] = v_d[e];
        }
        __syncwarp();
        if (leader) {
          const uint32_t bar = smem_u32(&st_full[slot]);
          mbar_arrive_expect_tx(bar, 2 * Tr::kTileBytes);
          for (int bx = 0; bx < Tr::kNumBoxes; ++bx) {
            tma_load_4d(smem_u32(stage_q(slot) + bx * Tr::kBoxBytes), &p.tm_q, bar, bx * 64, head, qi * kBlockM,
                        batch, pol_q);
            tma_load_4d(smem_u32(stage_do(slot) + bx * Tr::kBoxBytes), &p.tm_do, bar, bx * 64, head,
                        qi * kBlockM, batch, pol_q);
          }
        }
      }
      if (!ok) {
        const uint64_t drain_ns = 200ull * 1000 * 1000;
        int zero = 0;
        volatile int* never = &zero;
        mbar_wait(smem_u32(kv_full), 0, never, drain_ns);
        for (int s2 = 0; s2 < NS && s2 < it; ++s2) {
          const int last = s2 + ((it - 1 - s2) / NS) * NS;
          mbar_wait(smem_u32(&st_full[s2]), static_cast<uint32_t>(last / NS) & 1u, never, drain_ns);
        }
      }
    } else if (warp == 9 && n_steps > 0) {
      // --------------------------------------------------------------- MMA
      // S^T / dP^T of one half: M = 128 keys, N = 64 queries
      constexpr uint32_t kIdescS = make_idesc_f16(kBlockN, kBlockM / 2, kBf16, false);
      constexpr uint32_t kIdescAcc = make_idesc_f16(kBlockN, D, kBf16, true);
      const uint64_t desc_k = make_sw128_desc(smem_u32(sK), 16, 1024);
      const uint64_t desc_v = make_sw128_desc(smem_u32(sV), 16, 1024);
      const uint64_t desc_st0 = make_sw128_desc(smem_u32(sStage), 16, 1024);              // K-major
      const uint64_t desc_mn0 = make_sw128_desc(smem_u32(sStage), Tr::kBoxBytes, 1024);  // MN-major (N = d)
      constexpr uint64_t kStageStep = Tr::kStageBytes >> 4;
      constexpr uint64_t kDoOff = Tr::kTileBytes >> 4;
      constexpr uint64_t kHalfRows = (64 * 128) >> 4;    // 64 rows of 128-byte-row boxes, K-major
      constexpr uint64_t kHalfRowsMN = 4 * (2048 >> 4);  // 64 rows = 4 steps of 16, MN-major
      bool issued = false;
      auto issue_ss = [&](uint32_t dcol, uint64_t desc_a, uint64_t desc_b) {
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t off = ((kk >> 2) * Tr::kBoxBytes + (kk & 3) * 32) >> 4;
            umma_ss(tmem + dcol, desc_a + off, desc_b + off, kIdescS, kk > 0 ? 1u : 0u);
          }
        }
        __syncwarp();
      };
      auto issue_acc = [&](uint32_t dcol, uint32_t acol, uint64_t desc_b, bool acc) {
        // D(keys x d) += A(keys x 64 queries, 16-bit pairs in TMEM) B(queries x d)
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kBlockM / 32; ++kk) {
            umma_ts(tmem + dcol, tmem + acol + kk * 8, desc_b + kk * (2048 >> 4), kIdescAcc,
                    (acc || kk > 0) ? 1u : 0u);
          }
        }
        __syncwarp();
      };
      auto commit = [&](uint64_t* bar) {
        if (leader) umma_commit(smem_u32(bar));
        __syncwarp();
      };
      // S^T_h = K Q_h^T and dP^T_h = V dO_h^T for query half h of stage `slot`
      auto issue_sdp = [&](int slot, int h) {
        const uint64_t dq_ = desc_st0 + slot * kStageStep + h * kHalfRows;
        issue_ss(Tr::kColS + 64 * h, desc_k, dq_);
        issue_ss(Tr::kColDP + 64 * h, desc_v, dq_ + kDoOff);
        commit(&s_full[h]);
      };
      // dV += P^T_h dO_h and dK += dS^T_h Q_h for query half h of stage `slot`
      auto issue_dvdk = [&](int slot, int h, bool acc) {
        const uint64_t mq = desc_mn0 + slot * kStageStep + h * kHalfRowsMN;
        issue_acc(Tr::kColDV, Tr::kColS + 64 * h, mq + kDoOff, acc);
        issue_acc(Tr::kColDK, Tr::kColDP + 64 * h, mq, acc);
      };
      bool ok = wait_all(kv_full, 0) && wait_all(&st_full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_sdp(0, 0);
        issue_sdp(0, 1);
        issued = true;
      }
      // Per step and half h: dV/dK of half h, then the next step's S^T/dP^T of
      // half h into the same columns (the MMAs of one issuing thread execute
      // in order, so the products read P^T_h / dS^T_h before they are
      // overwritten), while the elementwise warps work on the other half.
      for (int it = 0; it < n_steps && ok; ++it) {
        const int slot = it % NS;
        const bool more = it + 1 < n_steps;
        const int nslot = (it + 1) % NS;
        for (int h = 0; h < 2 && ok; ++h) {
          ok = wait_all(&p_full[h], static_cast<uint32_t>(it) & 1u);
          if (!ok) break;
          tc_fence_after();
          issue_dvdk(slot, h, it > 0 || h > 0);
          if (h == 1) commit(&st_empty[slot]);  // every MMA reading stage `slot` is issued
          if (more) {
            if (h == 0) {
              ok = wait_all(&st_full[nslot], static_cast<uint32_t>((it + 1) / NS) & 1u);
              if (!ok) break;
              tc_fence_after();
            }
            issue_sdp(nslot, h);
          }
        }
      }
      if (issued) {
        commit(acc_done);
        commit(mma_drain);
        int zero = 0;
        volatile int* never = &zero;
        mbar_wait(smem_u32(mma_drain), 0, never, 200ull * 1000 * 1000);
      }
    }
    teardown();
    return;
  } else {
    // --------------------------------------------------------- elementwise
    // Thread: key row r of the block (a TMEM lane) and, in each query half of
    // the step, 32 of its 64 query columns.
    reg_alloc<kRegsSoftmax>();
    const int qh = lane >> 4;
    const int r = 32 * (warp & 3) + 16 * (warp >> 2) + (lane & 15);
    const uint32_t lane_addr = static_cast<uint32_t>(32 * (warp & 3) + 16 * (warp >> 2)) << 16;
    constexpr int kHalfD = D / 2;
    const int key = n0 + r;
    const bool key_ok = live && key < p.seqlen_k;
    const int64_t key_pos = static_cast<int64_t>(key) + p.k_pos_offset;
    const float c = p.scale_log2;
    bool ok = true;
#pragma unroll 1
    for (int it = 0; it < n_steps && ok; ++it) {
      const int slot = it % NS;
      const int qi = i_start + it % q_blocks;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        // query half hh of the step: S^T_hh, dP^T_hh in columns 64 hh + [0, 64);
        // lanes 0-15 hold its queries [0, 32), lanes 16-31 queries [32, 64)
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&s_full[hh]), static_cast<uint32_t>(it) & 1u, vabort, tmo))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t col_s = Tr::kColS + 64 * hh;
        const uint32_t col_dp = Tr::kColDP + 64 * hh;
        float sv[32], dpv[32];
        {
          uint32_t raw[32];
          tmem_ld_16x32bx2_x32_sync<32>(tmem + lane_addr + col_s, raw);
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(raw[i]);
          tmem_ld_16x32bx2_x32_sync<32>(tmem + lane_addr + col_dp, raw);
#pragma unroll
          for (int i = 0; i < 32; ++i) dpv[i] = __uint_as_float(raw[i]);
        }
        // queries [q0, q0 + 32) of this thread; the first `lo` are masked
        const int64_t q0 = static_cast<int64_t>(qi) * kBlockM + 64 * hh + qh * 32;
        int64_t lo = 0;
        if constexpr (kCausal) {
          const int64_t first_vis = key_pos - p.q_pos_offset - q0;  // first query index that sees the key
          lo = first_vis < 0 ? 0 : first_vis;
        }
        if (!key_ok) lo = 32;
        const float* nl = stage_nl(slot) + 64 * hh + qh * 32;
        const float* ddv = stage_dd(slot) + 64 * hh + qh * 32;
        uint32_t pk_p[16], pk_s[16];
        if (__any_sync(0xffffffffu, lo > 0)) {
          pds_pack<kBf16, true>(sv, dpv, c, nl, ddv, lo, pk_p, pk_s);
        } else {
          pds_pack<kBf16, false>(sv, dpv, c, nl, ddv, lo, pk_p, pk_s);
        }
        // P^T_hh over the first 32 columns of S^T_hh, dS^T_hh over those of dP^T_hh
        // (query q of the half in column q / 2)
        tmem_st_16x32bx2_x16<16>(tmem + lane_addr + col_s, pk_p);
        tmem_st_16x32bx2_x16<16>(tmem + lane_addr + col_dp, pk_s);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&p_full[hh]));
      }
    }
    // ---- epilogue: dV = P^T dO, dK = scale * dS^T Q, in the input type.
    bool have = ok && n_steps > 0;
    if (have) {
      have = __all_sync(0xffffffffu, mbar_wait(smem_u32(acc_done), 0, vabort, tmo));
      tc_fence_after();
    }
    using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const uint32_t col = which == 0 ? Tr::kColDV : Tr::kColDK;
      const float sc = have ? (which == 0 ? 1.f : p.scale) : 0.f;
      T* base = reinterpret_cast<T*>(which == 0 ? p.dv : p.dk);
      const int64_t bs = which == 0 ? p.dv_batch_stride : p.dk_batch_stride;
      const int64_t rs = which == 0 ? p.dv_row_stride : p.dk_row_stride;
      const int64_t hs = which == 0 ? p.dv_head_stride : p.dk_head_stride;
#pragma unroll
      for (int cc = 0; cc < kHalfD / 32; ++cc) {
        uint32_t o[32];
        if (have) {
          tmem_ld_16x32bx2_x32_sync<kHalfD>(tmem + lane_addr + col + cc * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (live && key < p.seqlen_k) {
          uint4* d4 = reinterpret_cast<uint4*>(base + static_cast<int64_t>(batch) * bs + static_cast<int64_t>(key) * rs +
                                               static_cast<int64_t>(kv_head) * hs + qh * kHalfD + cc * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            d4[i] = make_uint4(pack2<kBf16>(__uint_as_float(o[8 * i + 0]) * sc, __uint_as_float(o[8 * i + 1]) * sc),
                               pack2<kBf16>(__uint_as_float(o[8 * i + 2]) * sc, __uint_as_float(o[8 * i + 3]) * sc),
                               pack2<kBf16>(__uint_as_float(o[8 * i + 4]) * sc, __uint_as_float(o[8 * i + 5]) * sc),
                               pack2<kBf16>(__uint_as_float(o[8 * i + 6]) * sc, __uint_as_float(o[8 * i + 7]) * sc));
          }
        }
      }
    }
    teardown();
    return;
  }
}
}  // namespace fa
