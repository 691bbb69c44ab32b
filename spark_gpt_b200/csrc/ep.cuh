// Expert-parallel routing helpers: the per-rank send plan of the routed
// tokens, the packed (local expert id, routing weight) slot words that travel
// with each row, and the routing-weight gradient gathered back from the
// owners.  With P ranks and E_loc = E / P experts per rank, rank r owns
// experts [r*E_loc, (r+1)*E_loc).
//
// A token goes to each rank that owns at least one of its k experts exactly
// once (one row per (token, rank), not one per slot); its row carries k slot
// words, one per top-k slot: the slot's local expert id and bf16 routing
// weight when the expert lives on that rank, kEpNoExpert otherwise.
#pragma once

#include "common.cuh"

namespace b200moe {

constexpr unsigned kEpNoExpert = 0xFFFFu;  // low half of a slot word: no expert here
constexpr int kEpMaxRanks = 64;

// dest[t*P + r] = r when token t selected an expert of rank r, else -1 (the
// dispatch kernel skips negative ids, so dispatching dest over P "experts"
// gives the send order: rank-major, token order inside a rank).
// slot_counts[r] += slots of this block's tokens that go to rank r (zeroed by
// the caller; integer adds, so the totals do not depend on the order).
__global__ void ep_route_kernel(const long long* __restrict__ sel, long long T, int k, int E_loc,
                                int P, long long* __restrict__ dest, int* __restrict__ slot_counts) {
  __shared__ int cnt[kEpMaxRanks];
  for (int r = threadIdx.x; r < P; r += blockDim.x) cnt[r] = 0;
  __syncthreads();
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < T;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    unsigned long long mask = 0ull;
    for (int s = 0; s < k; ++s) {
      const long long e = sel[t * k + s];
      const long long r = e / E_loc;
      if (e >= 0 && r < P) {
        mask |= 1ull << r;
        atomicAdd(&cnt[r], 1);
      } else {
        raise_fault(kFaultBadExpert);
      }
    }
    for (int r = 0; r < P; ++r) dest[t * P + r] = ((mask >> r) & 1ull) ? r : -1;
  }
  __syncthreads();
  for (int r = threadIdx.x; r < P; r += blockDim.x)
    if (cnt[r]) atomicAdd(&slot_counts[r], cnt[r]);
}

// Slot words of the send rows p < pad_offsets[P] (row_flat[p] = t*P + r, or -1
// for a padding row of the send layout):
//   meta[p*k + s] = bf16bits(w[t,s]) << 16 | (sel[t,s] - r*E_loc)  if rank r owns sel[t,s]
//                 = kEpNoExpert                                    otherwise
__global__ void ep_pack_kernel(const long long* __restrict__ sel,
                               const unsigned short* __restrict__ w,
                               const int* __restrict__ row_flat, const int* __restrict__ total_rows,
                               int k, int E_loc, int P, unsigned* __restrict__ meta) {
  const long long n = static_cast<long long>(*total_rows) * k;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long p = i / k;
    const int s = static_cast<int>(i - p * k);
    const int f = row_flat[p];
    unsigned word = kEpNoExpert;
    if (f >= 0) {
      const long long t = f / P;
      const int r = f - static_cast<int>(t) * P;
      const long long e = sel[t * k + s];
      const long long lo = static_cast<long long>(r) * E_loc;
      if (e >= lo && e < lo + E_loc)
        word = (static_cast<unsigned>(w[t * k + s]) << 16) | static_cast<unsigned>(e - lo);
    }
    meta[i] = word;
  }
}

// Owner side: slot words -> selected (local expert id, -1 for none) and bf16
// routing weights (0 for none).
__global__ void ep_unpack_kernel(const unsigned* __restrict__ meta, long long n,
                                 long long* __restrict__ sel_local,
                                 unsigned short* __restrict__ w_local) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const unsigned word = meta[i];
    const unsigned id = word & 0xFFFFu;
    const bool none = id == kEpNoExpert;
    sel_local[i] = none ? -1 : static_cast<long long>(id);
    w_local[i] = none ? 0 : static_cast<unsigned short>(word >> 16);
  }
}

// Source side: the gradient of routing weight (t, s) is the owner's value for
// slot s of the row that carried token t to the owner of sel[t,s]:
//   d_w[t*k+s] = dw_rows[inv_send[t*P + sel[t,s]/E_loc] * k + s]
__global__ void ep_weight_grad_kernel(const float* __restrict__ dw_rows,
                                      const int* __restrict__ inv_send,
                                      const long long* __restrict__ sel, long long T, int k,
                                      int E_loc, int P, float* __restrict__ d_w) {
  const long long n = T * k;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = i / k;
    const int s = static_cast<int>(i - t * k);
    const long long r = sel[i] / E_loc;
    const int row = inv_send[t * P + r];
    d_w[i] = row >= 0 ? dw_rows[static_cast<long long>(row) * k + s] : 0.f;
  }
}

// d_weights[f] = 0 for the slots without an expert (inv_pad[f] < 0): the
// row-order combine backward writes only the slots that have rows.
__global__ void zero_skipped_slots_kernel(const int* __restrict__ inv_pad, long long R,
                                          float* __restrict__ d_weights) {
  for (long long f = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; f < R;
       f += static_cast<long long>(gridDim.x) * blockDim.x)
    if (inv_pad[f] < 0) d_weights[f] = 0.f;
}

}  // namespace b200moe

namespace b200moe {

// ---------------------------------------------------------------------------
// Peer-memory transport of the expert-parallel layer.  Every rank holds, in
// memory mapped by all ranks of the group (NVLink / NVSwitch peer access):
//   recv rows  (P*T_cap, H) bf16  rows other ranks send to this rank's experts
//   recv meta  (P*T_cap, k) u32   their slot words
//   back rows  (P*T_cap, H) bf16  partial rows the owners return to this rank
//   back dw    (P*T_cap, k) f32   routing-weight gradients returned with them
//   flags      (P) u64            barrier words, one per peer
// C[s][d] = rows rank s sends to rank d (unpadded), gathered on every rank.
// Layouts: at owner d, source s's rows start at recv_base[s] = sum_{s'<s}
// C[s'][d]; at source s, the rows returned by owner d start at my_back_base[d]
// = sum_{d'<d} C[s][d'] (rank-major, the source's send order).
// ---------------------------------------------------------------------------
// plan (ints): [0] n_recv | [1, 1+P) base_send[d] = sum_{s<me} C[s][d] |
// [1+P, 2+2P) recv_base[s], s = 0..P | [2+2P, 2+3P) back_base[s] = sum_{d<me} C[s][d] |
// [2+3P, 2+4P) my_back_base[d]
constexpr int ep_plan_ints(int P) { return 2 + 4 * P; }

__global__ void ep_p2p_plan_kernel(const int* __restrict__ counts, int ld, int me, int P,
                                   int* __restrict__ plan) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  auto C = [&](int s, int d) { return counts[s * ld + d]; };
  int n = 0;
  for (int s = 0; s < P; ++s) {
    plan[1 + P + s] = n;
    n += C(s, me);
  }
  plan[1 + 2 * P] = n;
  plan[0] = n;
  for (int d = 0; d < P; ++d) {
    int b = 0;
    for (int s = 0; s < me; ++s) b += C(s, d);
    plan[1 + d] = b;
  }
  for (int s = 0; s < P; ++s) {
    int b = 0;
    for (int d = 0; d < me; ++d) b += C(s, d);
    plan[2 + 2 * P + s] = b;
  }
  int b = 0;
  for (int d = 0; d < P; ++d) {
    plan[2 + 3 * P + d] = b;
    b += C(me, d);
  }
}

// Source side: token t's row goes to every rank r it selected (dest row
// inv_send[t*P+r] of the padded send layout -> row base_send[r] + (that row -
// pad_offsets[r]) of rank r's recv rows), stored straight into the peer's
// memory; with `sel`, its k slot words go to the peer's recv meta.
template <int VPL>
__global__ void ep_p2p_send_kernel(const __nv_bfloat16* __restrict__ src,
                                   const int* __restrict__ inv_send,
                                   const int* __restrict__ pad_offsets,
                                   const int* __restrict__ plan,
                                   __nv_bfloat16* const* __restrict__ peer_rows, long long T,
                                   int H, int P, const long long* __restrict__ sel,
                                   const unsigned short* __restrict__ w, int k, int E_loc,
                                   unsigned* const* __restrict__ peer_meta, int me = 0,
                                   int dest_mode = 0) {
  __shared__ int base_s[kEpMaxRanks], pad_s[kEpMaxRanks];
  for (int r = threadIdx.x; r < P; r += blockDim.x) {
    base_s[r] = plan[1 + r];
    pad_s[r] = pad_offsets[r];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    const int pl = lane < P ? inv_send[t * P + lane] : -1;
    const uint4* x = reinterpret_cast<const uint4*>(src + t * H);
    uint4 v[VPL > 0 ? VPL : 1];
    if (VPL > 0) {
#pragma unroll
      for (int j = 0; j < VPL; ++j) v[j] = __ldg(x + lane + 32 * j);
    }
    long long e = -1;
    unsigned short wb = 0;
    if (sel != nullptr && lane < k) {
      e = sel[t * k + lane];
      wb = w[t * k + lane];
    }
    for (int r = 0; r < P; ++r) {
      const int p = __shfl_sync(0xffffffffu, pl, r);
      if (p < 0) continue;
      // dest_mode 1: only this rank's own rows; 2: only the other ranks'
      if ((dest_mode == 1 && r != me) || (dest_mode == 2 && r == me)) continue;
      const long long row = base_s[r] + (p - pad_s[r]);
      uint4* dst = reinterpret_cast<uint4*>(peer_rows[r] + row * H);
      if (VPL > 0) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) dst[lane + 32 * j] = v[j];
      } else {
        for (int i = lane; i < nvec; i += 32) dst[i] = __ldg(x + i);
      }
      if (sel != nullptr && lane < k) {
        const long long lo = static_cast<long long>(r) * E_loc;
        const unsigned word = (e >= lo && e < lo + E_loc)
                                  ? ((static_cast<unsigned>(wb) << 16) | static_cast<unsigned>(e - lo))
                                  : kEpNoExpert;
        peer_meta[r][row * k + lane] = word;
      }
    }
  }
}

// Owner side: received row i (< n_recv) came from source s (recv_base[s] <= i <
// recv_base[s+1]); its result row goes back to row back_base[s] + (i -
// recv_base[s]) of s's back rows, and its k routing-weight gradients (if given)
// to the same row of s's back dw.
template <int VPL>
__global__ void ep_p2p_return_kernel(const __nv_bfloat16* __restrict__ rows,
                                     const float* __restrict__ dw, const int* __restrict__ plan,
                                     __nv_bfloat16* const* __restrict__ peer_rows,
                                     float* const* __restrict__ peer_dw, int H, int k, int P) {
  __shared__ int rb_s[kEpMaxRanks + 1], bb_s[kEpMaxRanks];
  for (int r = threadIdx.x; r <= P; r += blockDim.x) {
    rb_s[r] = plan[1 + P + r];
    if (r < P) bb_s[r] = plan[2 + 2 * P + r];
  }
  __syncthreads();
  const long long n = plan[0];
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       i < n; i += warps) {
    int s = 0;
    while (s + 1 < P && rb_s[s + 1] <= i) ++s;
    const long long row = bb_s[s] + (i - rb_s[s]);
    const uint4* x = reinterpret_cast<const uint4*>(rows + i * H);
    uint4* dst = reinterpret_cast<uint4*>(peer_rows[s] + row * H);
    if (VPL > 0) {
      uint4 v[VPL > 0 ? VPL : 1];
#pragma unroll
      for (int j = 0; j < VPL; ++j) v[j] = __ldg(x + lane + 32 * j);
#pragma unroll
      for (int j = 0; j < VPL; ++j) dst[lane + 32 * j] = v[j];
    } else {
      for (int j = lane; j < nvec; j += 32) dst[j] = __ldg(x + j);
    }
    if (dw != nullptr && lane < k) peer_dw[s][row * k + lane] = dw[i * k + lane];
  }
}

// inv_back[t*P+r]: row of the source's back rows holding owner r's result for
// token t (or -1): the padded send row minus its block start plus my_back_base[r].
__global__ void ep_p2p_back_inv_kernel(const int* __restrict__ inv_send,
                                       const int* __restrict__ pad_offsets,
                                       const int* __restrict__ plan, long long T, int P,
                                       int* __restrict__ inv_back) {
  const long long n = T * P;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i % P);
    const int p = inv_send[i];
    inv_back[i] = p >= 0 ? p - pad_offsets[r] + plan[2 + 3 * P + r] : -1;
  }
}

// Group barrier over peer memory: thread j writes `epoch` into peer j's flag
// word for this rank (release, system scope: the rows this stream stored into
// peers before are visible first), then waits until every peer has written
// `epoch` into this rank's flags (acquire).  The wait is bounded: after the
// limit it raises kFaultWaitTimeout and returns.
__global__ void ep_barrier_kernel(unsigned long long* const* __restrict__ peer_flags,
                                  unsigned long long* __restrict__ my_flags, int me, int P,
                                  unsigned long long epoch) {
  const int j = threadIdx.x;
  if (j >= P) return;
  __threadfence_system();
  unsigned long long* dst = peer_flags[j] + me;
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(epoch) : "memory");
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(my_flags + j) : "memory");
    if (v >= epoch) break;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      raise_fault(kFaultWaitTimeout);
      break;
    }
    __nanosleep(64);
  }
}

// Point-to-point completion flags of the pipelined exchange.  Each rank's flag
// area holds one word per (phase, source rank): flags[phase * kEpMaxRanks + s].
// ep_signal: thread j writes `epoch` into peer j's word (phase, me) -- every
// peer (dest < 0) or only peer `dest` -- with a system-scope release store, so
// the rows this stream stored into that peer before are visible first.
// ep_wait: waits until this rank's word (phase, src) -- or, with src < 0,
// every source's word of the phase -- reaches `epoch` (acquire), at most
// kWaitLimitNs; then it raises kFaultWaitTimeout and returns.
constexpr int kEpFlagPhases = 5;  // 0: the group barrier, 1-4: the pipelined phases

__global__ void ep_signal_kernel(unsigned long long* const* __restrict__ peer_flags, int phase,
                                 int me, int P, int dest, unsigned long long epoch) {
  const int j = threadIdx.x;
  if (j >= P || (dest >= 0 && j != dest)) return;
  __threadfence_system();
  unsigned long long* dst = peer_flags[j] + phase * kEpMaxRanks + me;
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(epoch) : "memory");
}

__global__ void ep_wait_kernel(const unsigned long long* __restrict__ my_flags, int phase, int src,
                               int P, unsigned long long epoch) {
  const int j = threadIdx.x;
  if (j >= P || (src >= 0 && j != src)) return;
  const unsigned long long* w = my_flags + phase * kEpMaxRanks + j;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
    if (v >= epoch) break;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      raise_fault(kFaultWaitTimeout);
      break;
    }
    __nanosleep(64);
  }
}

}  // namespace b200moe

namespace b200moe {

// Owner side, fused reduction + return: for received row i < plan[0], the sum
// over its slots s with a row (inv_pad[i*k+s] >= 0) of bf16(y[row] * w[i,s])
// (weights given: the combine) or of y[row] (no weights: the gather
// backward), accumulated in fp32 in slot order and rounded once, is stored
// straight into row back_base[src] + (i - recv_base[src]) of the source's back
// rows; with dw (rows, k) fp32 its k routing-weight gradients go to the same
// row of the source's back dw.  A warp takes one of SPLIT column parts of a
// received row (VPL 16-byte vectors per lane), so the fp32 accumulators stay
// few enough for four 256-thread blocks per SM at H = 2048 (four 512-column
// parts); the rows of the valid slots are loaded two at a time.
template <int VPL, int SPLIT>
__global__ void ep_p2p_reduce_return_kernel(const __nv_bfloat16* __restrict__ y,
                                            const int* __restrict__ inv_pad,
                                            const __nv_bfloat16* __restrict__ weights, int k,
                                            const float* __restrict__ dw,
                                            const int* __restrict__ plan,
                                            __nv_bfloat16* const* __restrict__ peer_rows,
                                            float* const* __restrict__ peer_dw, int H, int P,
                                            long long n_src_rows = 0, int src_fixed = -1) {
  static_assert(VPL > 0, "H in {256, 512, 1024, 2048}");
  __shared__ int rb_s[kEpMaxRanks + 1], bb_s[kEpMaxRanks];
  for (int r = threadIdx.x; r <= P; r += blockDim.x) {
    rb_s[r] = plan[1 + P + r];
    if (r < P) bb_s[r] = plan[2 + 2 * P + r];
  }
  __syncthreads();
  // src_fixed >= 0: the rows are the n_src_rows rows received from that source
  // alone (one per-source chunk of the owner's work), row i returning to row
  // back_base[src] + i; otherwise all received rows, each to its source.
  const long long n = (src_fixed >= 0 ? n_src_rows : static_cast<long long>(plan[0])) *
                      static_cast<long long>(SPLIT);
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long item = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
       item < n; item += warps) {
    const long long i = item / SPLIT;
    const int part = static_cast<int>(item - i * SPLIT);
    const int col0 = part * (H / SPLIT);  // first column of this part
    const int rl = lane < k ? inv_pad[i * k + lane] : -1;
    float wl = 1.f;
    if (weights != nullptr && lane < k) wl = __bfloat162float(weights[i * k + lane]);
    unsigned valid = __ballot_sync(0xffffffffu, rl >= 0);
    float acc[VPL][8];
#pragma unroll
    for (int j = 0; j < VPL; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[j][e] = 0.f;
    auto add_row = [&](const uint4* q, float w) {
      const __nv_bfloat162 w2 = __float2bfloat162_rn(w);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        uint4 v = q[j];
        if (weights != nullptr) {
          // bf16 x bf16 product rounded once to bf16, as the combine
          __nv_bfloat162* v2 = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
          for (int e = 0; e < 4; ++e) v2[e] = __hmul2(v2[e], w2);
        }
        acc[j][0] += bf16_lo(v.x); acc[j][1] += bf16_hi(v.x);
        acc[j][2] += bf16_lo(v.y); acc[j][3] += bf16_hi(v.y);
        acc[j][4] += bf16_lo(v.z); acc[j][5] += bf16_hi(v.z);
        acc[j][6] += bf16_lo(v.w); acc[j][7] += bf16_hi(v.w);
      }
    };
    while (valid) {
      const int s0 = __ffs(valid) - 1;
      valid &= valid - 1;
      const int s1 = valid ? __ffs(valid) - 1 : -1;
      if (s1 >= 0) valid &= valid - 1;
      const long long r0 = __shfl_sync(0xffffffffu, rl, s0);
      const float w0 = __shfl_sync(0xffffffffu, wl, s0);
      const long long r1 = __shfl_sync(0xffffffffu, rl, s1 >= 0 ? s1 : s0);
      const float w1 = __shfl_sync(0xffffffffu, wl, s1 >= 0 ? s1 : s0);
      uint4 a[VPL], b[VPL];
      const uint4* p0 = reinterpret_cast<const uint4*>(y + r0 * H + col0);
      const uint4* p1 = reinterpret_cast<const uint4*>(y + r1 * H + col0);
#pragma unroll
      for (int j = 0; j < VPL; ++j) a[j] = __ldg(p0 + lane + 32 * j);
      if (s1 >= 0) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) b[j] = __ldg(p1 + lane + 32 * j);
      }
      add_row(a, w0);
      if (s1 >= 0) add_row(b, w1);
    }
    int src = 0;
    long long row;
    if (src_fixed >= 0) {
      src = src_fixed;
      row = bb_s[src] + i;
    } else {
      while (src + 1 < P && rb_s[src + 1] <= i) ++src;
      row = bb_s[src] + (i - rb_s[src]);
    }
    uint4* dst = reinterpret_cast<uint4*>(peer_rows[src] + row * H + col0);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      uint4 o;
      o.x = pack_bf16x2(acc[j][0], acc[j][1]);
      o.y = pack_bf16x2(acc[j][2], acc[j][3]);
      o.z = pack_bf16x2(acc[j][4], acc[j][5]);
      o.w = pack_bf16x2(acc[j][6], acc[j][7]);
      dst[lane + 32 * j] = o;
    }
    if (dw != nullptr && part == 0 && lane < k) peer_dw[src][row * k + lane] = dw[i * k + lane];
  }
}

}  // namespace b200moe
