// Pieces shared by the tensor-core attention kernels (forward, dQ, dK/dV):
// the drain wait used before exit and the per-thread visibility masks.
#pragma once

#include "tc_prims.cuh"

namespace sbfa {
namespace tc {

__device__ __forceinline__ bool wait_bar_drain(uint32_t bar, uint32_t parity, int* status) {
  // drains our own in-flight async work before exit: ignores the abort flag
  // but is still bounded
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      record_status(status, kStatusWaitTimeout);
      return false;
    }
  }
  return true;
}

// True when every pair of query rows [q_lo, q_lo+nq) x keys [k_lo, k_lo+nk)
// is visible (inside both sequences, lifted block mask all ones -- the plan
// marks other tiles partial -- and, when causal, inside the token rule): a
// few uniform integer tests that let the softmax phases skip the per-element
// masks on interior tiles.
__device__ __forceinline__ bool block_all_visible(const MaskParams& mp, int q_lo, int nq, int k_lo,
                                                  int nk, bool partial) {
  // branch-free, so that callers can compute it inside straight-line code
  const int q_hi = q_lo + nq - 1, k_hi = k_lo + nk - 1;
  const bool inside = !partial & (q_hi < mp.n_q) & (k_hi < mp.n_kv);
  const bool token = (mp.q_off + q_lo >= k_hi) &                        // no key after a query
                     ((k_hi < mp.sink) |                                 // sink keys only
                      (mp.q_off + q_hi - max(k_lo, mp.sink) < mp.window));
  return inside & (!mp.causal | token);
}

// Visibility of the NCOL keys [k0, k0+NCOL) for one query row, bit c of
// vis[c/32] = key k0 + c, from the sequence ends and, when causal, the token
// rule (at most two intervals: sink and window).  Branch-free.
template <int NCOL>
__device__ __forceinline__ void row_token_visibility(uint32_t (&vis)[NCOL / 32],
                                                     const MaskParams& mp, int row, int k0) {
  constexpr int W = NCOL / 32;
  const int end = row < mp.n_q ? min(mp.n_kv - k0, NCOL) : 0;
  const int qpos = mp.q_off + row;
  const int cend = min(end, qpos - k0 + 1);
  const int hi1 = mp.causal ? min(cend, mp.sink - k0) : end;
  const int lo2 = mp.causal ? max(qpos - mp.window + 1 - k0, 0) : 0;
  const int hi2 = mp.causal ? cend : 0;
#pragma unroll
  for (int w = 0; w < W; ++w) vis[w] = range_bits(0, hi1, 32 * w) | range_bits(lo2, hi2, 32 * w);
}

// Clears the keys of zero user blocks of the lifted block mask (partial tiles).
template <int NCOL>
__device__ __forceinline__ void row_block_mask(uint32_t (&vis)[NCOL / 32], const MaskParams& mp,
                                               int row, int k0) {
  constexpr int W = NCOL / 32;
  if (row >= mp.n_q) return;
  const int32_t* mrow = mp.block_mask + (size_t)(row / mp.block_m) * mp.n_kb;
  const int b0 = k0 / mp.block_n;
  const int b1 = min((k0 + NCOL - 1) / mp.block_n, mp.n_kb - 1);
  for (int b = b0; b <= b1; ++b) {
    if (__ldg(mrow + b) != 0) continue;
    const int lo = b * mp.block_n - k0, hi = lo + mp.block_n;
#pragma unroll
    for (int w = 0; w < W; ++w) vis[w] &= ~range_bits(lo, hi, 32 * w);
  }
}

// Both of the above: the full visibility of one row's NCOL keys.
template <int NCOL>
__device__ __forceinline__ void row_visibility(uint32_t (&vis)[NCOL / 32], const MaskParams& mp,
                                               int row, int k0, bool partial) {
  row_token_visibility<NCOL>(vis, mp, row, k0);
  if (partial) row_block_mask<NCOL>(vis, mp, row, k0);
}


// Visibility of the NROW query rows [q0, q0+NROW) for one key, bit c of
// vis[c/32] = row q0 + c (the column view used by the dK/dV kernel): for a
// fixed key the visible rows form one interval (causal lower end, window
// upper end unless the key is a sink), cut by the lifted block mask.
template <int NROW>
__device__ __forceinline__ void col_visibility(uint32_t (&vis)[NROW / 32], const MaskParams& mp,
                                               int key, int q0, bool partial) {
  constexpr int W = NROW / 32;
  if (key >= mp.n_kv) {
#pragma unroll
    for (int w = 0; w < W; ++w) vis[w] = 0u;
    return;
  }
  const int end = min(mp.n_q - q0, NROW);
  int lo = 0, hi = end;
  if (mp.causal) {
    lo = max(key - mp.q_off - q0, 0);                       // q >= key
    if (key >= mp.sink) hi = min(end, key + mp.window - mp.q_off - q0);  // q <= key + W - 1
  }
#pragma unroll
  for (int w = 0; w < W; ++w) vis[w] = range_bits(lo, hi, 32 * w);
  if (partial) {
    const int kb = key / mp.block_n;
    const int b0 = q0 / mp.block_m;
    const int b1 = (q0 + NROW - 1) / mp.block_m;
    const int nqb = (mp.n_q + mp.block_m - 1) / mp.block_m;
    for (int b = b0; b <= min(b1, nqb - 1); ++b) {
      if (__ldg(mp.block_mask + (size_t)b * mp.n_kb + kb) != 0) continue;
      const int rlo = b * mp.block_m - q0, rhi = rlo + mp.block_m;
#pragma unroll
      for (int w = 0; w < W; ++w) vis[w] &= ~range_bits(rlo, rhi, 32 * w);
    }
  }
}

}  // namespace tc
}  // namespace sbfa
