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
