// Two-CTA (cta_group::2) variant of the grouped GEMM: a cluster of two CTAs on
// paired SMs computes a 256 x BN tile with one tcgen05.mma.cta_group::2 per
// K=16 step.  Each CTA stages its own 128 rows of A and half of B (BN/2 rows,
// or BN/2 columns for MN-major B), so per unit of MMA work each SM moves a
// third less operand data through L2 than the single-CTA 128 x BN tile.  For
// the SwiGLU gate_up tile the B halves are exactly the gate rows (leader) and
// the up rows (follower), so the accumulator layout and the epilogue are the
// single-CTA ones.
//
// Barrier protocol (both CTAs have the same shared-memory layout):
//   full[s]   leader only: armed by the leader with both CTAs' bytes; both CTAs'
//             TMA loads complete on it (.cta_group::2, leader's address)
//   empty[s]  one per CTA: the leader's MMA commit arrives on both
//   tfull[a]  one per CTA: the leader's MMA commit arrives on both
//   tempty[a] leader only: every epilogue warp of both CTAs arrives on it
//
// Row-ragged schedule: a pair tile covers two consecutive 128-row tiles of one
// expert.  An expert with an odd number of 128-row tiles ends in a pair whose
// second half lies past the expert: that half is computed (on whatever rows it
// loads) and not stored.
#pragma once

#include "grouped_gemm.cuh"

namespace b200moe {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on a barrier of another CTA of the cluster (default .release at CTA
// scope).  The epilogue's TMEM-release arrive needs no cluster-scope release:
// its TMEM reads have completed (tcgen05.wait::ld) before it.  A
// .release.cluster arrive here waited for the warp's in-flight TMA stores and
// took half of the plain-store epilogue's time.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx_u32(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// the barrier at shared::cluster address `bar_cluster` (the leader's).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* tm,
                                                 uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at this shared-memory offset in both CTAs of the pair
// once the issuing thread's prior tcgen05 operations have completed.
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

constexpr int kMaxPairExperts = 256;  // the library takes E <= 256

// Epilogues whose bf16 output goes through shared memory and TMA stores.
template <int EPI>
struct TmaOut {
  static constexpr bool value = EPI == kEpiStoreBf16 || EPI == kEpiSwigluFwd ||
                                EPI == kEpiSwigluBwd || EPI == kEpiStoreF32Tma ||
                                EPI == kEpiSwigluFwdF8 || EPI == kEpiSwigluBwdF8 ||
                                EPI == kEpiAxpby;
};

// Epilogues that read a second input tile (g and u of the SwiGLU backward)
// through TMA into per-warp buffers.
template <int EPI>
struct GuIn {
  static constexpr bool value = EPI == kEpiSwigluBwd || EPI == kEpiSwigluBwdF8 ||
                                EPI == kEpiAxpby;
};

template <int BN, int STAGES, bool TMA_OUT, bool GU_IN = false>
struct PairSmem {
  static constexpr uint32_t kABytes = 128 * 64 * 2;
  static constexpr uint32_t kBBytes = (BN / 2) * 64 * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kOutBytes = TMA_OUT ? kEpilogueWarps * kOutRing * 2048 : 0;
  static constexpr uint32_t kInBytes = GU_IN ? kEpilogueWarps * 2 * 2048 : 0;
  static constexpr uint32_t kBarrierBytes = 256;
  static constexpr uint32_t kPairTableBytes = (kMaxPairExperts + 1) * 4;
  static constexpr uint32_t kTotal =
      STAGES * kStageBytes + kOutBytes + kInBytes + kBarrierBytes + kPairTableBytes + 1024;
};

// This CTA's 128-row tile of pair tile t.  `half_ok` is false for the second
// half of an expert's last pair when the expert has an odd tile count.
template <int SCHED, int BK = 64>
__device__ __forceinline__ TileInfo decode_pair(const GemmParams& p, const int* pair_start,
                                                int t, uint32_t rank, bool& half_ok) {
  TileInfo T;
  half_ok = true;
  if (SCHED == kRowsRagged) {
    const int pt = t / p.n_tiles;
    T.n = t - pt * p.n_tiles;
    int lo = 0, hi = p.num_groups;  // largest e with pair_start[e] <= pt
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pair_start[mid] <= pt) lo = mid; else hi = mid;
    }
    T.g = lo;
    // without pad_offsets: one group of m_tiles row tiles (the router dgrad)
    const int first_tile = p.pad_offsets ? __ldg(p.pad_offsets + lo) / 128 : 0;
    const int ntiles = p.pad_offsets ? __ldg(p.pad_offsets + lo + 1) / 128 - first_tile
                                     : p.m_tiles;
    const int local = 2 * (pt - pair_start[lo]) + static_cast<int>(rank);
    half_ok = local < ntiles;
    T.m = first_tile + local;
    T.krow0 = 0;
    T.kblocks = p.k_blocks;
  } else {
    const int mp = p.m_tiles / 2;
    const int per = mp * p.n_tiles;
    const int gi = t / per;
    T.g = pair_start[gi];  // the expert order table (most rows first)
    const int r = t - gi * per;
    const int mpair = r / p.n_tiles;
    T.n = r - mpair * p.n_tiles;
    T.m = 2 * mpair + static_cast<int>(rank);
    const int s = __ldg(p.pad_offsets + T.g);
    const int e = __ldg(p.pad_offsets + T.g + 1);
    T.krow0 = s;
    T.kblocks = (e - s) / BK;
    for (int seg = 1; seg < p.k_segments; ++seg) {
      const int* po = p.pad_offsets + seg * (p.num_groups + 1) + T.g;
      T.kblocks += (__ldg(po + 1) - __ldg(po)) / BK;
    }
  }
  return T;
}

// The first row of a K-ragged tile's next k-block: rows advance by BK inside a
// segment and continue at the start of the group's next non-empty segment.
// `row` / `end` / `seg` carry the walk from one k-block to the next.
template <int BK>
__device__ __forceinline__ int kragged_next_row(const GemmParams& p, int g, int& row, int& end,
                                                int& seg) {
  while (row >= end && seg + 1 < p.k_segments) {
    ++seg;
    const int* po = p.pad_offsets + seg * (p.num_groups + 1) + g;
    row = __ldg(po);
    end = __ldg(po + 1);
  }
  const int r = row;
  row += BK;
  return r;
}

// OP: operand kind (OperandKind).  An fp8 stage carries 128 K elements in the
// bytes of a 64-element bf16 stage; MN-major fp8 tiles are one 128-element
// (128-byte) swizzle column wide, so their TMA box is 128 x 128 and the MMA's
// 32-row K step advances 4 KB.  fp8 pair tiles need BN = 256 for MN-major B.
template <int BN, bool A_MN, bool B_MN, int EPI, int SCHED, int STAGES, int OP = kOpBf16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmO0,
                             const __grid_constant__ CUtensorMap tmO1, const GemmParams p) {
  static_assert(BN == 128 || BN == 256, "BN");
  static_assert(SCHED == kRowsRagged ? !A_MN : (A_MN && B_MN), "operand majors vs schedule");
  static_assert(OP == kOpBf16 || !B_MN || BN == 256, "fp8 MN-major B needs BN = 256");
  constexpr int BM = 128;
  constexpr bool kF8 = OP != kOpBf16;
  constexpr int BK = OpTraits<OP>::kBK;
  constexpr int kMmaK = OpTraits<OP>::kMmaK;
  constexpr bool kTmaOut = TmaOut<EPI>::value;
  constexpr bool kGuIn = GuIn<EPI>::value;
  static_assert(!kGuIn || kTmaOut, "the gu input buffers come with the TMA-store ring");
  using S = PairSmem<BN, STAGES, kTmaOut, kGuIn>;
  constexpr uint32_t kTmemCols = TmemCols<BN>::value;
  constexpr uint32_t kIdesc = kF8 ? make_idesc_f8(2 * BM, BN, OpTraits<OP>::kAFmt, 0u, A_MN, B_MN)
                                  : make_idesc_bf16(2 * BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint8_t* sOut = sB + STAGES * S::kBBytes;
  uint8_t* sIn = sOut + S::kOutBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sIn + S::kInBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* in_bars = tempty + 3;  // kGuIn: one per epilogue warp, after tmem_slot / abort_flag
  static_assert(!kGuIn || (2 * STAGES + 5 + kEpilogueWarps) * 8 <= S::kBarrierBytes,
                "barrier area");
  int* pair_start = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bars) + S::kBarrierBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpilogueWarps);
    }
    if (kGuIn)
      for (int w = 0; w < kEpilogueWarps; ++w) mbar_init(&in_bars[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (SCHED == kRowsRagged && warp == 2) {
    // pair_start[e] = pairs of the experts before e (a 32-lane scan over E)
    int carry = 0;
    for (int e0 = 0; e0 <= p.num_groups; e0 += 32) {
      const int e = e0 + lane;
      int v = 0;
      if (e < p.num_groups) {
        const int nt = p.pad_offsets
                           ? (__ldg(p.pad_offsets + e + 1) - __ldg(p.pad_offsets + e)) / 128
                           : p.m_tiles;
        v = (nt + 1) / 2;
      }
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (e <= p.num_groups) pair_start[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (SCHED == kKRagged) {
    // Weight-gradient tiles run expert by expert, the experts with the most rows
    // first (ties by index), so the persistent schedule's last tiles are its
    // shortest ones: pair_start[i] = the expert of rank i.  The first A stage,
    // unused until the producer starts, holds the row counts meanwhile.
    static_assert(S::kABytes >= kMaxPairExperts * 4, "row counts fit one A stage");
    int* cnt = reinterpret_cast<int*>(sA);
    for (int e = threadIdx.x; e < p.num_groups; e += blockDim.x) {
      int c = 0;
      for (int seg = 0; seg < max(p.k_segments, 1); ++seg) {
        const int* po = p.pad_offsets + seg * (p.num_groups + 1) + e;
        c += __ldg(po + 1) - __ldg(po);
      }
      cnt[e] = c;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < p.num_groups; e += blockDim.x) {
      const int ce = cnt[e];
      int rank = 0;
      for (int j = 0; j < p.num_groups; ++j) {
        const int cj = cnt[j];
        rank += (cj > ce) || (cj == ce && j < e);
      }
      pair_start[rank] = e;
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (kTmaOut) {
      tma_prefetch_desc(&tmO0);
      tma_prefetch_desc(&tmO1);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  int num_tiles;
  if (SCHED == kRowsRagged) {
    num_tiles = pair_start[p.num_groups] * p.n_tiles;
  } else {
    num_tiles = p.num_groups * (p.m_tiles / 2) * p.n_tiles;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      B200_PROF(unsigned long long pw = 0; const long long pt0 = clock64();)
      for (int t = cluster_id; ok && t < num_tiles; t += num_clusters) {
        bool half_ok;
        const TileInfo T = decode_pair<SCHED, BK>(p, pair_start, t, rank, half_ok);
        // K-ragged: the walk over the group's row segments
        int k_row = T.krow0, k_seg = 0;
        int k_end = SCHED == kKRagged ? __ldg(p.pad_offsets + T.g + 1) : 0;
        for (int kb = 0; kb < T.kblocks; ++kb) {
          const int krow_k = SCHED == kKRagged ? kragged_next_row<BK>(p, T.g, k_row, k_end, k_seg)
                                               : 0;
          B200_PROF(const long long w0 = clock64();)
          const bool got = mbar_wait(&empty[stage], phase ^ 1u, abort_flag);
          B200_PROF(pw += clock64() - w0;)
          if (!got) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_expect_tx_u32(smem_u32(&full[stage]), 2 * S::kStageBytes);
          uint8_t* a = sA + stage * S::kABytes;
          uint8_t* b = sB + stage * S::kBBytes;
          if (!A_MN) {
            tma_load_2d_pair(a, &tmA, full_leader, kb * BK, T.m * BM);
          } else {
            const int krow = SCHED == kKRagged ? krow_k : T.krow0 + kb * BK;
            tma_load_2d_pair(a, &tmA, full_leader, T.m * BM, krow);
            if (!kF8) tma_load_2d_pair(a + 8192, &tmA, full_leader, T.m * BM + 64, krow);
          }
          if (!B_MN) {
            // this CTA's BN/2 rows of B: the gate (leader) or up (follower) rows for
            // SwiGLU, else the leader's or follower's half of the BN rows
            const int row = (EPI == kEpiSwigluFwd || EPI == kEpiSwigluFwdF8)
                                ? T.g * p.b_group_rows + static_cast<int>(rank) * p.b_half_offset +
                                      T.n * (BN / 2)
                                : T.g * p.b_group_rows + T.n * BN + static_cast<int>(rank) * (BN / 2);
            tma_load_2d_pair(b, &tmB, full_leader, kb * BK, row);
          } else {
            const int krow = (SCHED == kKRagged) ? krow_k : (T.g * p.b_group_rows + kb * BK);
            if (kF8) {
              tma_load_2d_pair(b, &tmB, full_leader, T.n * BN + static_cast<int>(rank) * (BN / 2),
                               krow);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                tma_load_2d_pair(b + j * 8192, &tmB, full_leader,
                                 T.n * BN + static_cast<int>(rank) * (BN / 2) + 64 * j, krow);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      B200_PROF(atomicAdd(&g_prof[0], pw); atomicAdd(&g_prof[1], clock64() - pt0);)
      // tail: wait until the MMA's releases of every stage this CTA filled have
      // landed, so no commit arrives on this CTA's barriers after it exits
      for (int i = 0; ok && i < STAGES; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      B200_PROF(unsigned long long we = 0, wf = 0; const long long mt0 = clock64();)
      for (int t = cluster_id; ok && t < num_tiles; t += num_clusters) {
        bool half_ok;
        const TileInfo T = decode_pair<SCHED, BK>(p, pair_start, t, rank, half_ok);
        if (T.kblocks == 0) continue;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;
        B200_PROF(long long w0 = clock64();)
        const bool got_acc = mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag);
        B200_PROF(we += clock64() - w0;)
        if (!got_acc) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < T.kblocks; ++kb) {
          B200_PROF(w0 = clock64();)
          const bool got = mbar_wait(&full[stage], phase, abort_flag);
          B200_PROF(wf += clock64() - w0;)
          if (!got) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * S::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * S::kBBytes);
#pragma unroll
          for (int kk = 0; kk < BK / kMmaK; ++kk) {
            // K-major: 32 bytes per MMA step; MN-major: kMmaK rows of 128 bytes
            const uint64_t ad = A_MN ? make_sdesc(a0 + kk * kMmaK * 128, 8192, 1024)
                                     : make_sdesc(a0 + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc(b0 + kk * kMmaK * 128, 8192, 1024)
                                     : make_sdesc(b0 + kk * 32, 16, 1024);
            if (kF8)
              umma_f8_pair(d_tmem, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
            else
              umma_bf16_pair(d_tmem, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_pair_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_pair_both(&tfull[acc]);
      }
      B200_PROF(atomicAdd(&g_prof[2], we); atomicAdd(&g_prof[3], wf);
                atomicAdd(&g_prof[4], clock64() - mt0); atomicAdd(&g_prof[8], 1ull);)
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in = q * 32 + lane;
    OutRing ring{sOut + (warp - 2) * kOutRing * 2048, 0};
    if (kGuIn) {
      ring.in = sIn + (warp - 2) * 2 * 2048;
      ring.in_bar = in_bars + (warp - 2);
      ring.abort = abort_flag;
    }
    const bool tma_out = kTmaOut && p.scatter_rows == nullptr;
    int local = 0;
    B200_PROF(unsigned long long ew = 0, eb = 0, ea = 0; const long long et0 = clock64();
              unsigned long long pacc[3] = {0, 0, 0};)
    for (int t = cluster_id; t < num_tiles; t += num_clusters) {
      bool half_ok;
      const TileInfo T = decode_pair<SCHED, BK>(p, pair_start, t, rank, half_ok);
      if (T.kblocks == 0) {
        epilogue_empty_tile<EPI, BN>(p, T, row_in, half);
        continue;
      }
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      // the first g/u chunk of this warp's part of the tile, loaded while the MMA runs
      if (kGuIn && half_ok && tma_out) {
        if (EPI == kEpiAxpby) {
          if (p.aux != nullptr)
            aux_chunk_load(ring, &tmO1, T.n * BN + half * (BN / 2),
                           T.g * p.m_tiles * 128 + T.m * 128 + q * 32, lane);
        } else {
          gu_chunk_load<EPI == kEpiSwigluBwdF8 ? 1024 : 2048>(
              ring, &tmO1, T.n * BN + half * (BN / 2), p.inter, T.m * 128 + q * 32, lane);
        }
      }
      B200_PROF(const long long w0 = clock64();)
      const bool got_acc = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag));
      B200_PROF(const long long w1 = clock64(); ew += w1 - w0;)
      if (!got_acc) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (half_ok) {
        if (tma_out)
          epilogue_tile_tma<EPI, BN, kF8>(p, T, q, lane, half, taddr, &tmO0, &tmO1, ring
                                     B200_PROF(, pacc));
        else
          epilogue_tile<EPI, BN>(p, T, row_in, half, taddr);
      }
      B200_PROF(const long long w2 = clock64();)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      B200_PROF(const long long w3 = clock64(); eb += w3 - w1; ea += w3 - w2;)
    }
    if (kTmaOut && lane == 0) bulk_wait_group_all();  // stores done before exit
    B200_PROF(if (lane == 0) {
      atomicAdd(&g_prof[5], ew);
      atomicAdd(&g_prof[6], eb);
      atomicAdd(&g_prof[7], clock64() - et0);
      atomicAdd(&g_prof[9], 1ull);
      atomicAdd(&g_prof[10], pacc[0]);
      atomicAdd(&g_prof[11], pacc[1]);
      atomicAdd(&g_prof[12], pacc[2]);
      atomicAdd(&g_prof[13], ea);
    })
  }

  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace b200moe
