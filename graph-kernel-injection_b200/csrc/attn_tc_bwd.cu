// Tensor-core backward for sm_100a: separate dK/dV and dQ kernels, both
// recomputing P from the forward's log-sum-exp (upstream
// _bwd_dkdv_kernel / _bwd_dq_kernel, sparse_triton_kernel.py:395-601).
//
// Both kernels share one structure.  A CTA owns one 128-row tile of the
// "resident" operand (keys for dK/dV, queries for dQ) and walks the kept
// 128-row tiles of the other operand from the compacted plan (CSC for
// dK/dV, CSR for dQ), scoring whole 128 x 128 tiles (N = 128 MMAs run at the
// tensor pipe's full rate, N = 64 ones do not):
//   warp 0       TMA producer: the resident tiles once, then the streamed
//                tiles through a ring of kRing shared-memory entries;
//   warp 2       (dK/dV only) stages LSE*log2(e) and Delta of each streamed
//                query tile in shared memory;
//   warp 1       MMA issuer, the whole warp with one elected lane issuing
//                (warp-uniform descriptors stay in uniform registers);
//   warps 4-11   two compute groups that both work on every tile: one TMEM
//                lane (row) per thread, group g takes score columns
//                [64g, 64g+64); P = 2^(S*scale*log2e - LSE*log2e) on visible
//                pairs and dS = P * (dP - Delta), packed to 16 bits over TMEM
//                columns the group has already read, where the accumulator
//                MMAs read them as the A operand.
// The TMEM layout and MMA order of each kernel are described above it.
// Epilogue: accumulators -> 16-bit -> shared memory (128-byte swizzle) -> TMA
// store; rows past the sequence end are clipped by the tensor map.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <type_traits>
#include <utility>
#include <vector>

#include "tc_attn_common.cuh"

namespace sbfa {

int device_sm_count();

namespace {

using namespace tc;

constexpr int kT = 128;        // rows of a resident / streamed tile
constexpr int kRing = 5;       // dQ ring entries (streamed tiles in flight); DkdvLayout sets its own
constexpr int kBwdThreads = 384;
constexpr int kRegsCtl = 88;       // producer / MMA / staging warps (64 spills)
constexpr int kRegsCompute = 208;  // 128*88 + 256*208 == 384*168: the whole launch pool
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;

// TMEM column, within a 128-column score buffer, of the packed 16-bit A
// operand for k-step kk (16 score columns) of an accumulator MMA: compute
// group g packs score columns [64g, 64g+64) into buffer columns
// [64g, 64g+32).
__device__ __forceinline__ uint32_t a_col128(int kk) {
  return 64u * (uint32_t)(kk >> 2) + 8u * (uint32_t)(kk & 3);
}

// Stored dS tiles (dkdv_tc_kernel<..., DS = true> -> dq_gemm_kernel): the
// 128 x 128 16-bit tile is the A operand (M = 128 queries, K = 128 keys,
// M-major) of a tcgen05 MMA without swizzle, made of 8 x 8 core matrices of
// 128 contiguous bytes, each 8 keys x 8 consecutive queries (16 B per key).
// Core matrices follow each other along the keys (128 B apart), and each
// group of 8 queries is a 2048-byte plane: element (query q, key k) sits at
//   (q / 8) * 2048 + k * 16 + (q % 8) * 2  bytes.
// A thread holding one key's 8 consecutive queries writes one 16-byte piece,
// and the 32 keys of a warp write 512 contiguous bytes.
constexpr uint32_t kDsChunkBytes = 2048;  // one plane of 8 queries x 128 keys
__host__ __device__ constexpr uint32_t ds_tile_offset(int q, int k) {
  return (uint32_t)(q >> 3) * kDsChunkBytes + (uint32_t)k * 16u + (uint32_t)(q & 7) * 2u;
}

// ---------------------------------------------------------------------------
// dK / dV
// ---------------------------------------------------------------------------
// A CTA owns 128 keys and walks the query tiles that see them (CSC plan).
// TMEM: S_i^T = K Q_i^T at 0-127, dP_i^T = V dO_i^T at 128-255, dV at 256,
// dK at 384.  Compute group g (query columns [64g, 64g+64) of the tile)
// loads its S columns and releases them at once, so S_{i+1} is computed
// while the group runs the exponentials of step i; once it has loaded its dP
// columns it packs dS_i (16-bit) into dP columns [64g, 64g+32) and P_i into
// [64g+32, 64g+64), where the accumulator MMAs read them as the A operand.
// MMAs from one issuer run in order, so dP_{i+1} overwrites the columns
// only after dV_i and dK_i have read them:
//   [S_i loaded] S_{i+1},  [P_i, dS_i packed] dV += P_i^T dO_i,
//   dK += dS_i^T Q_i, dP_{i+1}.
// Streamed tiles share one ring of kRing entries, entry 2i = Q_i and
// 2i+1 = dO_i.  dS is computed without the softmax scale, which multiplies
// dK once in the epilogue.
//
// With DS the kernel also stores every dS_i tile (128 queries x 128 keys,
// 16-bit) to global memory for dq_gemm_kernel, at the CSC position of the
// (query head, key tile, query tile) triple, in the layout of a tcgen05
// operand without swizzle (see ds_tile_offset): each compute thread stores
// its key's 64 columns straight from registers as eight 16-byte pieces, and
// every warp-wide store covers 512 contiguous bytes.  Nothing is staged in
// shared memory, whose bandwidth the MMAs already use in full.
template <int D, bool DS = false>
struct DkdvLayout {
  // K, V and a 5-entry ring of 128-column tiles fill 224 KB; 64-column
  // tiles leave room for 6 ring entries.
  static constexpr int kRing = D > 64 ? 5 : 6;
  static constexpr uint32_t kTile = kT * D * 2;
  static constexpr uint32_t K = 0;
  static constexpr uint32_t V = K + kTile;
  static constexpr uint32_t RING = V + kTile;               // kRing streamed tiles
  static constexpr uint32_t LS = RING + kRing * kTile;       // 2 x 128 floats (LSE * log2 e)
  static constexpr uint32_t DL = LS + 2 * kT * 4;            // 2 x 128 floats (Delta)
  static constexpr uint32_t BAR = DL + 2 * kT * 4;
  static constexpr int kKVFull = 0;
  static constexpr int kRFull = 1;                   // [kRing]
  static constexpr int kREmpty = 1 + kRing;          // [kRing]
  static constexpr int kLFull = 1 + 2 * kRing;       // [2] LSE / Delta slot staged
  static constexpr int kLEmpty = 3 + 2 * kRing;      // [2] slot read by the compute groups
  static constexpr int kSFull = 5 + 2 * kRing;       // S_i written
  static constexpr int kSFree = 6 + 2 * kRing;       // S_i loaded by the compute groups
  static constexpr int kDPFull = 7 + 2 * kRing;      // dP_i written
  static constexpr int kDSReady = 8 + 2 * kRing;     // P_i and dS_i packed in TMEM
  static constexpr int kDone = 9 + 2 * kRing;
  static constexpr int kDrain = 10 + 2 * kRing;
  static constexpr int kNumBars = 11 + 2 * kRing;
  static constexpr uint32_t MISC = BAR + kNumBars * 8;
  static constexpr uint32_t kBytes = MISC + 16;
  // D = 128 leaves no room to align the window by hand: the kernel checks
  // that the runtime placed it on a 1024-byte boundary (it does when the
  // kernel has no static shared memory) and reports otherwise.
  static constexpr bool kAlignInKernel = kBytes + 1024 <= 232448;
  static constexpr uint32_t kAlloc = kAlignInKernel ? kBytes + 1024 : kBytes;
};

template <typename T, int D, bool DS>
__global__ void __launch_bounds__(kBwdThreads, 1)
    dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                   const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                   const __grid_constant__ CUtensorMap tmdk,
                   const __grid_constant__ CUtensorMap tmdv,
                   T* __restrict__ ds, int nnz, T* __restrict__ dk,
                   T* __restrict__ dv, const float* __restrict__ lse,
                   const float* __restrict__ delta, float scale, float scale_log2, MaskParams mp,
                   const int32_t* __restrict__ col_ptr, const int32_t* __restrict__ row_idx, int BH,
                   int n_tj, int heads, int kv_group, Strides3 sdk, Strides3 sdv,
                   float* __restrict__ part_ws, int sink_parts, int* status) {
  using L = DkdvLayout<D, DS>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = idesc_f16(kBF16, kT, kT, false, false);   // M=128 keys, N=128 q
  constexpr uint32_t kIdescAcc = idesc_f16(kBF16, kT, D, false, true);   // M=128 keys, N=D
  constexpr int kBoxes = D / 64;
  constexpr uint32_t kTS = 0, kTDP = 128, kTDV = 256, kTDK = 384;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if (L::kAlignInKernel) {
    smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  } else if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) record_status(status, kStatusBadSmemAlign);
    return;
  }
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sb + L::BAR + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // BH counts (batch, key/value head) units.  The sink key tiles (seen by
  // every query tile) first; then each unit's remaining key tiles in order,
  // so CTAs running side by side stream the same query tiles through L2.
  // With grouped-query attention the kv_group query heads of a unit are
  // streamed one after another and all accumulate into its dK, dV, except
  // for the sink tile when sink_parts > 1: its column is as long as the
  // whole sequence for every query head of the group, so sink_parts CTAs per
  // unit take one query head each and leave fp32 partial dV, dK in part_ws
  // for dkdv_sink_reduce_kernel.
  int tj, bh, head_lo = 0, n_heads = kv_group;
  bool split = false;
  if ((int)blockIdx.x < BH * sink_parts) {
    tj = 0;
    bh = blockIdx.x / sink_parts;
    if (sink_parts > 1) {
      split = true;
      head_lo = blockIdx.x % sink_parts;
      n_heads = 1;
    }
  } else {
    const int idx = blockIdx.x - BH * sink_parts;
    bh = idx / (n_tj - 1);
    tj = 1 + idx % (n_tj - 1);
  }
  const int kv_heads = heads / kv_group;
  const int hh = bh % kv_heads, bb = bh / kv_heads;  // TMA coordinates of the K/V plane
  const int n_ti = ceil_div_dev(mp.n_q, kT);  // query tiles (plan rows)
  const PlanSpan span = plan_span(col_ptr, tj, n_ti, (int64_t)n_ti * n_tj, status);
  const int e0 = span.e0;
  const int nq = span.n;                 // query tiles per query head
  // streamed tiles: tile i is query tile i % nq of query head
  // hh * kv_group + head_lo + i / nq
  const int ntot = nq * n_heads;
  // partials of this CTA when split: [dV | dK] x 128 keys x D fp32
  float* part = split ? part_ws + (size_t)blockIdx.x * 2 * kT * D : nullptr;

  if (nq == 0 && split) {  // no query sees the sink tile: zero partials
    for (int idx = threadIdx.x; idx < 2 * kT * D / 4; idx += blockDim.x)
      reinterpret_cast<float4*>(part)[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  if (nq == 0) {  // no query sees this key tile: dK = dV = 0
    for (int idx = threadIdx.x; idx < kT * (D / 8); idx += blockDim.x) {
      const int rr = idx / (D / 8), cc = idx % (D / 8);
      const int key = tj * kT + rr;
      if (key < mp.n_kv) {
        reinterpret_cast<uint4*>(dk + bb * sdk.b + hh * sdk.h + (int64_t)key * sdk.n)[cc] =
            make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(dv + bb * sdv.b + hh * sdv.h + (int64_t)key * sdv.n)[cc] =
            make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(bar(L::kKVFull), 1);
    for (int s = 0; s < L::kRing; ++s) {
      mbar_init(bar(L::kRFull + s), 1);
      mbar_init(bar(L::kREmpty + s), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bar(L::kLFull + x), 1);
      mbar_init(bar(L::kLEmpty + x), 256);
    }
    mbar_init(bar(L::kSFull), 1);
    mbar_init(bar(L::kSFree), 256);
    mbar_init(bar(L::kDPFull), 1);
    mbar_init(bar(L::kDSReady), 256);
    mbar_init(bar(L::kDone), 1);
    mbar_init(bar(L::kDrain), 1);
    *abort_flag = 0;
    mbar_init_fence();
    // the resident K, V tiles are requested before the TMEM allocation and
    // the CTA-wide sync, so their latency overlaps them
    mbar_expect_tx(bar(L::kKVFull), 2 * L::kTile);
    for (int r = 0; r < kBoxes; ++r) {
      tma_load_4d(sb + L::K + r * 16384u, &tmk, bar(L::kKVFull), 64 * r, tj * kT, hh, bb);
      tma_load_4d(sb + L::V + r * 16384u, &tmv, bar(L::kKVFull), 64 * r, tj * kT, hh, bb);
    }
    // ... and so are the first ring entries, Q_0 and dO_0 (fresh slots 0, 1)
    const int ti0 = plan_index(plan_entry(row_idx, e0, n_ti, status));
    for (int part = 0; part < 2; ++part) {
      mbar_expect_tx(bar(L::kRFull + part), L::kTile);
      for (int r = 0; r < kBoxes; ++r)
        tma_load_4d(sb + L::RING + part * L::kTile + r * 16384u, part ? &tmdo : &tmq,
                    bar(L::kRFull + part), 64 * r, ti0 * kT, hh * kv_group + head_lo, bb);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    regs_dec<kRegsCtl>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      // (K, V, Q_0 and dO_0 were requested by this thread right after the
      // barrier set-up)
      int issued = 2;
      int next_ent = ntot > 1 ? plan_entry(row_idx, e0 + (1 % nq), n_ti, status) : 0;
      bool ok = true;
      for (int i = 1; ok && i < ntot; ++i) {
        const int ti = plan_index(next_ent);
        const int hq = hh * kv_group + head_lo + i / nq;  // query head of tile i
        if (i + 1 < ntot)
          next_ent = plan_entry(row_idx, e0 + (i + 1) % nq, n_ti, status);  // prefetch
        for (int part = 0; part < 2; ++part) {           // Q_i, then dO_i
          const int e = 2 * i + part, s = e % L::kRing, f = e / L::kRing;
          if (f > 0 && !wait_bar_w(bar(L::kREmpty + s), (uint32_t)((f - 1) & 1), abort_flag,
                                   status)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            mbar_expect_tx(bar(L::kRFull + s), L::kTile);
            for (int r = 0; r < kBoxes; ++r)
              tma_load_4d(sb + L::RING + s * L::kTile + r * 16384u, part ? &tmdo : &tmq,
                          bar(L::kRFull + s), 64 * r, ti * kT, hq, bb);
          }
          issued = e + 1;
        }
      }
      if (lane == 0) {
        wait_bar_drain(bar(L::kKVFull), 0, status);
        for (int s = 0; s < L::kRing; ++s) {
          const int fills = issued > s ? (issued - 1 - s) / L::kRing + 1 : 0;
          if (fills) wait_bar_drain(bar(L::kRFull + s), (uint32_t)((fills - 1) & 1), status);
        }
      }
    } else if (warp == 2) {
      // ------------------------------------------- LSE (log2 units) / Delta
      // a warp of its own, so the latency of these loads never delays the
      // tensor copies
      for (int i = 0; i < ntot; ++i) {
        const int slot = i & 1;
        const int ti = plan_index(plan_entry(row_idx, e0 + i % nq, n_ti, status));
        const int row0 = ti * kT;
        const size_t qbh = (size_t)bb * heads + hh * kv_group + head_lo + i / nq;  // query (b, h)
        float lv[kT / 32], dv2[kT / 32];
#pragma unroll
        for (int c = 0; c < kT / 32; ++c) {  // loads first, then the wait for the slot
          const int row = row0 + 32 * c + lane;
          const bool in = row < mp.n_q;
          lv[c] = in ? lse[qbh * mp.n_q + row] * kLog2e : 0.f;
          dv2[c] = in ? delta[qbh * mp.n_q + row] : 0.f;
        }
        if (i >= 2 && !wait_bar_w(bar(L::kLEmpty + slot), (uint32_t)(((i >> 1) - 1) & 1),
                                  abort_flag, status))
          break;
        float* ls = reinterpret_cast<float*>(smem + L::LS) + slot * kT;
        float* dl = reinterpret_cast<float*>(smem + L::DL) + slot * kT;
#pragma unroll
        for (int c = 0; c < kT / 32; ++c) {
          ls[32 * c + lane] = lv[c];
          dl[32 * c + lane] = dv2[c];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(L::kLFull + slot));
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------- MMA issuer
      const uint64_t d_k = desc_kmajor(sb + L::K), d_v = desc_kmajor(sb + L::V);
      const uint64_t d_r = desc_kmajor(sb + L::RING);
      const uint64_t m_r = desc_mnmajor(sb + L::RING, 16384u);
      auto ring = [&](int e) -> bool {
        if (!wait_bar_w(bar(L::kRFull + e % L::kRing), (uint32_t)((e / L::kRing) & 1), abort_flag,
                        status))
          return false;
        tc_fence_after();
        return true;
      };
      // tdst[128 keys x 128 q] = A (K or V, K-major) * (ring entry e)^T
      auto scores = [&](uint32_t tdst, uint64_t da, int e) {
        const uint64_t db = desc_advance(d_r, (uint32_t)(e % L::kRing) * L::kTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
          mma_f16_ss_w(tmem + tdst, desc_advance(da, off), desc_advance(db, off), kIdescS,
                       kk > 0 ? 1u : 0u);
        }
      };
      // tacc[128 keys x D] += packed A (TMEM columns tsrc + a_col128) * ring entry e
      auto accum = [&](uint32_t tacc, uint32_t tsrc, int e, bool acc) {
        const uint64_t mb = desc_advance(m_r, (uint32_t)(e % L::kRing) * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)
          mma_f16_ts_w(tmem + tacc, tmem + tsrc + a_col128(kk),
                       desc_advance(mb, (uint32_t)kk * 2048u), kIdescAcc,
                       (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = wait_bar_w(bar(L::kKVFull), 0, abort_flag, status) && ring(0);
      if (ok) {
        scores(kTS, d_k, 0);  // S_0
        tc_commit_w(bar(L::kSFull));
        ok = ring(1);
      }
      if (ok) {
        scores(kTDP, d_v, 1);  // dP_0
        tc_commit_w(bar(L::kDPFull));
      }
      for (int i = 0; ok && i < ntot; ++i) {
        const uint32_t ph = (uint32_t)(i & 1);
        if (i + 1 < ntot) {  // S_{i+1} as soon as the compute groups have loaded S_i
          if (!ring(2 * i + 2) || !wait_bar_w(bar(L::kSFree), ph, abort_flag, status)) break;
          tc_fence_after();
          scores(kTS, d_k, 2 * i + 2);
          tc_commit_w(bar(L::kSFull));
        }
        // dO_{i+1} is checked before the wait for dS_i, off the critical path
        if ((i + 1 < ntot && !ring(2 * i + 3)) ||
            !wait_bar_w(bar(L::kDSReady), ph, abort_flag, status))
          break;
        tc_fence_after();
        accum(kTDV, kTDP + 32u, 2 * i + 1, i > 0);  // dV += P_i^T dO_i
        tc_commit_w(bar(L::kREmpty + (2 * i + 1) % L::kRing));
        accum(kTDK, kTDP, 2 * i, i > 0);            // dK += dS_i^T Q_i (unscaled)
        tc_commit_w(bar(L::kREmpty + (2 * i) % L::kRing));
        if (i + 1 < ntot) {
          scores(kTDP, d_v, 2 * i + 3);  // dP_{i+1}, after dV_i and dK_i have read P_i, dS_i
          tc_commit_w(bar(L::kDPFull));
        }
      }
      tc_commit_w(bar(L::kDone));
      tc_commit_w(bar(L::kDrain));
      wait_bar_drain(bar(L::kDrain), 0, status);
    }
  } else {
    regs_inc<kRegsCompute>();
    // ------------------------------------------------------------ compute
    const int grp = (warp - 4) >> 2;  // query columns [64*grp, 64*grp + 64) of every tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int key = tj * kT + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    int32_t ent_next = plan_entry(row_idx, e0, n_ti, status);
    int pos_next = nq > 1 ? 1 : 0;  // (i + 1) % nq, kept as a counter (no division)
    int pos_i = 0, head_i = 0;      // i % nq and i / nq
    for (int i = 0; i < ntot; ++i) {
      const int slot = i & 1;
      const uint32_t ph = (uint32_t)(i & 1);
      const int32_t ent = ent_next;
      if (i + 1 < ntot) ent_next = plan_entry(row_idx, e0 + pos_next, n_ti, status);  // in flight
      pos_next = pos_next + 1 == nq ? 0 : pos_next + 1;
      const int q0 = plan_index(ent) * kT + 64 * grp;
      uint32_t vis[2] = {0xffffffffu, 0xffffffffu};
      const bool all_vis = block_all_visible(mp, q0, 64, tj * kT, kT, plan_partial(ent));
      if (!all_vis) col_visibility<64>(vis, mp, key, q0, plan_partial(ent));
      ok = wait_bar_w(bar(L::kLFull + slot), (uint32_t)((i >> 1) & 1), abort_flag, status) &&
           wait_bar_w(bar(L::kSFull), ph, abort_flag, status);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = tmem + lane_base + kTS + 64u * grp;
      const uint32_t t_dp = tmem + lane_base + kTDP + 64u * grp;
      const float4* ls4 = reinterpret_cast<const float4*>(smem + L::LS) + (slot * kT + 64 * grp) / 4;
      const float4* dl4 = reinterpret_cast<const float4*>(smem + L::DL) + (slot * kT + 64 * grp) / 4;
      // P = 2^(S * scale * log2 e - LSE * log2 e) on visible pairs, packed to
      // 16 bits while the exponentials are in flight
      float p[64];
      uint32_t pk[32];
      {
        uint32_t sv[64];
        tmem_ld32(t_s, sv);
        tmem_ld32(t_s + 32u, sv + 32);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(bar(L::kSFree));  // S_{i+1} may overwrite the slot
        if (all_vis) {
#pragma unroll
          for (int q4 = 0; q4 < 16; ++q4) {
            const float4 l4 = ls4[q4];
            p[4 * q4 + 0] = ex2(fmaf(__uint_as_float(sv[4 * q4 + 0]), scale_log2, -l4.x));
            p[4 * q4 + 1] = ex2(fmaf(__uint_as_float(sv[4 * q4 + 1]), scale_log2, -l4.y));
            p[4 * q4 + 2] = ex2(fmaf(__uint_as_float(sv[4 * q4 + 2]), scale_log2, -l4.z));
            p[4 * q4 + 3] = ex2(fmaf(__uint_as_float(sv[4 * q4 + 3]), scale_log2, -l4.w));
          }
        } else {
#pragma unroll
          for (int q4 = 0; q4 < 16; ++q4) {
            const float4 l4 = ls4[q4];
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int cc = 4 * q4 + e;
              const bool on = (vis[cc >> 5] >> (cc & 31)) & 1u;
              p[cc] = on ? ex2(fmaf(__uint_as_float(sv[cc]), scale_log2, -lv[e])) : 0.f;
            }
          }
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) pk[c] = pack2<T>(p[2 * c], p[2 * c + 1]);
      }
      // dS = P * (dP - Delta), in two 32-column halves
      ok = wait_bar_w(bar(L::kDPFull), ph, abort_flag, status);
      if (!ok) break;
      tc_fence_after();
      uint32_t dsk[32];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t dpv[32];
        tmem_ld32(t_dp + 32u * hf, dpv);
        tmem_wait_ld();
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const float4 d4 = dl4[8 * hf + q4];
          const int c = 32 * hf + 4 * q4;
          const float a0 = p[c + 0] * (__uint_as_float(dpv[4 * q4 + 0]) - d4.x);
          const float a1 = p[c + 1] * (__uint_as_float(dpv[4 * q4 + 1]) - d4.y);
          const float a2 = p[c + 2] * (__uint_as_float(dpv[4 * q4 + 2]) - d4.z);
          const float a3 = p[c + 3] * (__uint_as_float(dpv[4 * q4 + 3]) - d4.w);
          dsk[16 * hf + 2 * q4] = pack2<T>(a0, a1);
          dsk[16 * hf + 2 * q4 + 1] = pack2<T>(a2, a3);
        }
      }
      mbar_arrive(bar(L::kLEmpty + slot));  // the LSE / Delta slot has been read
      tmem_st32(t_dp + 32u, pk);  // P_i over dP columns [64g+32, 64g+64), already read
      tmem_st32(t_dp, dsk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(L::kDSReady));
      if constexpr (DS) {
        // this key's 64 columns of dS_i, straight from registers (tile
        // (query (b, h)) * nnz + CSC position; see ds_tile_offset)
        T* dst = ds + (size_t)((bb * heads + hh * kv_group + head_lo + head_i) * nnz + e0 + pos_i) *
                          (kT * kT) +
                 ds_tile_offset(64 * grp, r) / sizeof(T);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(dst + c * (kDsChunkBytes / sizeof(T))) =
              make_uint4(dsk[4 * c], dsk[4 * c + 1], dsk[4 * c + 2], dsk[4 * c + 3]);
      }
      if (++pos_i == nq) {
        pos_i = 0;
        ++head_i;
      }
    }
    // epilogue: group 0 writes dV (staged in K's buffer), group 1 writes
    // dK * scale (staged in V's buffer); both buffers are free once every
    // MMA is done
    if (ok) ok = wait_bar_w(bar(L::kDone), 0, abort_flag, status);
    if (ok && split) {
      // one part of a split sink tile: raw fp32 dV (group 0) / dK (group 1)
      // rows straight from TMEM, summed and scaled by dkdv_sink_reduce_kernel
      tc_fence_after();
      const uint32_t t_acc = tmem + lane_base + (grp == 0 ? kTDV : kTDK);
      float4* dst = reinterpret_cast<float4*>(part + ((size_t)grp * kT + r) * D);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t t[32];
        tmem_ld32(t_acc + 32u * c, t);
        tmem_wait_ld();
#pragma unroll
        for (int i2 = 0; i2 < 8; ++i2)
          dst[8 * c + i2] = make_float4(__uint_as_float(t[4 * i2]), __uint_as_float(t[4 * i2 + 1]),
                                        __uint_as_float(t[4 * i2 + 2]),
                                        __uint_as_float(t[4 * i2 + 3]));
      }
      ok = false;  // nothing left to store
    }
    if (ok) {
      tc_fence_after();
      const uint32_t t_acc = tmem + lane_base + (grp == 0 ? kTDV : kTDK);
      const float mul = grp == 0 ? 1.f : scale;
      const uint32_t stage = sb + (grp == 0 ? L::K : L::V);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t t[32];
        tmem_ld32(t_acc + 32u * c, t);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2)
          w[i2] = pack2<T>(__uint_as_float(t[2 * i2]) * mul, __uint_as_float(t[2 * i2 + 1]) * mul);
        const uint32_t region = stage + (uint32_t)((32 * c) >> 6) * 16384u;
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2) {
          const uint32_t addr =
              region + sw128_offset((uint32_t)r, (uint32_t)((32 * c) & 63) + 8u * i2);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * i2]),
                       "r"(w[4 * i2 + 1]), "r"(w[4 * i2 + 2]), "r"(w[4 * i2 + 3])
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1 + grp, 128);
      if (r == 0) {
        for (int b = 0; b < kBoxes; ++b)
          tma_store_4d(grp == 0 ? &tmdv : &tmdk, stage + (uint32_t)b * 16384u, 64 * b, tj * kT,
                       hh, bb);
        bulk_commit();
        bulk_wait_read0();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// dV, dK of the sink key tile of every (batch, key/value head) unit from the
// fp32 partials of its `parts` CTAs (one per query head of the group):
// summed in part order, dK scaled, rounded to 16 bits, rows past n_kv
// skipped.  One CTA per unit.
template <typename T, int D>
__global__ void __launch_bounds__(256) dkdv_sink_reduce_kernel(
    const float* __restrict__ part_ws, T* __restrict__ dk, T* __restrict__ dv, int parts,
    int kv_heads, int n_kv, float scale, Strides3 sdk, Strides3 sdv) {
  const int u = blockIdx.x;
  const int hh = u % kv_heads, bb = u / kv_heads;
  const float4* base = reinterpret_cast<const float4*>(part_ws) + (size_t)u * parts * 2 * kT * D / 4;
  for (int idx = threadIdx.x; idx < kT * D / 4; idx += blockDim.x) {
    const int key = idx / (D / 4), c4 = idx % (D / 4);
    if (key >= n_kv) continue;
    float4 sv = make_float4(0.f, 0.f, 0.f, 0.f), sk = sv;
    for (int p = 0; p < parts; ++p) {
      const float4 a = base[(size_t)p * 2 * kT * D / 4 + idx];
      const float4 b = base[(size_t)p * 2 * kT * D / 4 + kT * D / 4 + idx];
      sv = make_float4(sv.x + a.x, sv.y + a.y, sv.z + a.z, sv.w + a.w);
      sk = make_float4(sk.x + b.x, sk.y + b.y, sk.z + b.z, sk.w + b.w);
    }
    const uint2 ov = make_uint2(pack2<T>(sv.x, sv.y), pack2<T>(sv.z, sv.w));
    const uint2 ok = make_uint2(pack2<T>(sk.x * scale, sk.y * scale),
                                pack2<T>(sk.z * scale, sk.w * scale));
    *reinterpret_cast<uint2*>(dv + bb * sdv.b + hh * sdv.h + (int64_t)key * sdv.n + 4 * c4) = ov;
    *reinterpret_cast<uint2*>(dk + bb * sdk.b + hh * sdk.h + (int64_t)key * sdk.n + 4 * c4) = ok;
  }
}

// ---------------------------------------------------------------------------
// dQ
// ---------------------------------------------------------------------------
// A CTA owns 128 queries and walks the key tiles they see (CSR plan).
// TMEM: S[0] 0-127, S[1] 128-255, dP 256-383, dQ 384-.  Streamed tiles
// share one ring of kRing entries, entry 2j = V_j and 2j+1 = K_j: V_j is
// only read by dP(j) and is released early, so the ring refills with the
// next tiles while dQ_j still reads K_j.
// MMA order: S(0) dP(0) | [dP(j) read] S(j+1), dP(j+1); [dS_j ready] dQ_j
// for j = 0, 1, ...: K_{j+1} is first needed when the compute groups have
// read dP(j), a ring slot's time later than if S(j+1) followed dQ_{j-1}.
// Compute group g takes keys [64g, 64g+64) of every tile and writes its
// packed dS over S columns [64g, 64g+32) of the same slot.
template <int D>
struct DqLayout {
  static constexpr uint32_t kTile = kT * D * 2;
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t DO = Q + kTile;
  static constexpr uint32_t RING = DO + kTile;       // kRing streamed tiles
  static constexpr uint32_t BAR = RING + kRing * kTile;
  static constexpr int kQFull = 0;
  static constexpr int kRFull = 1;                   // [kRing]
  static constexpr int kREmpty = 1 + kRing;          // [kRing]
  static constexpr int kSDFull = 1 + 2 * kRing;      // [2] S(j) and dP(j) written
  static constexpr int kDPFree = 3 + 2 * kRing;      // compute read dP(j)
  static constexpr int kPReady = 4 + 2 * kRing;      // [2] compute wrote dS(j) into S[j&1]
  static constexpr int kDone = 6 + 2 * kRing;
  static constexpr int kDrain = 7 + 2 * kRing;
  static constexpr int kNumBars = 8 + 2 * kRing;
  static constexpr uint32_t MISC = BAR + kNumBars * 8;
  static constexpr uint32_t kAlloc = MISC + 16 + 1024;
};

template <typename T, int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    dq_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                 const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmdo,
                 const __grid_constant__ CUtensorMap tmdq, T* __restrict__ dq,
                 const float* __restrict__ lse, const float* __restrict__ delta, float scale,
                 float scale_log2, MaskParams mp, const int32_t* __restrict__ row_ptr,
                 const int32_t* __restrict__ col_idx, int heads, int kv_group, Strides3 sdq,
                 int* status) {
  using L = DqLayout<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = idesc_f16(kBF16, kT, kT, false, false);   // M=128 q, N=128 keys
  constexpr uint32_t kIdescAcc = idesc_f16(kBF16, kT, D, false, true);   // M=128 q, N=D
  constexpr int kBoxes = D / 64;
  constexpr uint32_t kTS0 = 0, kTDP = 256, kTDQ = 384;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sb + L::BAR + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ti = blockIdx.x;
  const int bh = blockIdx.y;
  const int hh = bh % heads, bb = bh / heads;  // TMA coordinates of the (batch, head) plane
  const int n_tj = ceil_div_dev(mp.n_kv, kT);  // key tiles (plan columns)
  const PlanSpan span = plan_span(row_ptr, ti, n_tj, (int64_t)gridDim.x * n_tj, status);
  const int e0 = span.e0;
  const int nk = span.n;

  if (nk == 0) {  // the tile's rows see no key: dQ = 0
    for (int idx = threadIdx.x; idx < kT * (D / 8); idx += blockDim.x) {
      const int rr = idx / (D / 8), cc = idx % (D / 8);
      const int row = ti * kT + rr;
      if (row < mp.n_q)
        reinterpret_cast<uint4*>(dq + bb * sdq.b + hh * sdq.h + (int64_t)row * sdq.n)[cc] =
            make_uint4(0, 0, 0, 0);
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(bar(L::kQFull), 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar(L::kRFull + s), 1);
      mbar_init(bar(L::kREmpty + s), 1);
    }
    mbar_init(bar(L::kSDFull), 1);
    mbar_init(bar(L::kSDFull + 1), 1);
    mbar_init(bar(L::kDPFree), 256);
    mbar_init(bar(L::kPReady), 256);
    mbar_init(bar(L::kPReady + 1), 256);
    mbar_init(bar(L::kDone), 1);
    mbar_init(bar(L::kDrain), 1);
    *abort_flag = 0;
    mbar_init_fence();
    // the resident Q, dO tiles are requested before the TMEM allocation and
    // the CTA-wide sync, so their latency overlaps them
    mbar_expect_tx(bar(L::kQFull), 2 * L::kTile);
    for (int r = 0; r < kBoxes; ++r) {
      tma_load_4d(sb + L::Q + r * 16384u, &tmq, bar(L::kQFull), 64 * r, ti * kT, hh, bb);
      tma_load_4d(sb + L::DO + r * 16384u, &tmdo, bar(L::kQFull), 64 * r, ti * kT, hh, bb);
    }
    // ... and so are the first ring entries, K_0 (entry 1) and V_0 (entry 0)
    const int kt0 = plan_index(plan_entry(col_idx, e0, n_tj, status));
    for (int part = 1; part >= 0; --part) {
      mbar_expect_tx(bar(L::kRFull + part), L::kTile);
      for (int r = 0; r < kBoxes; ++r)
        tma_load_4d(sb + L::RING + part * L::kTile + r * 16384u, part ? &tmk : &tmv,
                    bar(L::kRFull + part), 64 * r, kt0 * kT, hh / kv_group, bb);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    regs_dec<kRegsCtl>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- producer
      // (Q, dO, K_0 and V_0 were requested by this thread right after the
      // barrier set-up)
      int fills[kRing] = {1, 1};  // copies issued per ring slot
      int next_ent = nk > 1 ? plan_entry(col_idx, e0 + 1, n_tj, status) : 0;
      bool ok = true;
      for (int j = 1; ok && j < nk; ++j) {
        const int kt = plan_index(next_ent);
        if (j + 1 < nk) next_ent = plan_entry(col_idx, e0 + j + 1, n_tj, status);  // prefetch
        // K_j (entry 2j+1) before V_j (entry 2j): K_j is read first (by S(j),
        // issued a tile before dP(j)), and its slot was freed earlier (by
        // V_{j-2}, released as soon as dP(j-2) was issued).  Each slot is still
        // filled in entry order, so the per-slot parities hold.
        for (int part = 1; part >= 0; --part) {
          const int e = 2 * j + part, s = e % kRing, f = e / kRing;
          if (f > 0 &&
              !wait_bar(bar(L::kREmpty + s), (uint32_t)((f - 1) & 1), abort_flag, status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(bar(L::kRFull + s), L::kTile);
          for (int r = 0; r < kBoxes; ++r)
            tma_load_4d(sb + L::RING + s * L::kTile + r * 16384u, part ? &tmk : &tmv,
                        bar(L::kRFull + s), 64 * r, kt * kT, hh / kv_group, bb);
          ++fills[s];
        }
      }
      wait_bar_drain(bar(L::kQFull), 0, status);
      for (int s = 0; s < kRing; ++s)
        if (fills[s]) wait_bar_drain(bar(L::kRFull + s), (uint32_t)((fills[s] - 1) & 1), status);
    } else if (warp == 1) {
      // ---------------------------------------------------------- MMA issuer
      // base descriptors, built once; MMAs add constant offsets
      const uint64_t d_q = desc_kmajor(sb + L::Q), d_g = desc_kmajor(sb + L::DO);
      const uint64_t d_r = desc_kmajor(sb + L::RING);
      const uint64_t m_r = desc_mnmajor(sb + L::RING, 16384u);
      auto ring = [&](int e) -> bool {
        if (!wait_bar_w(bar(L::kRFull + e % kRing), (uint32_t)((e / kRing) & 1), abort_flag,
                        status))
          return false;
        tc_fence_after();
        return true;
      };
      // scores: tdst[128 x 128] = A (resident, K-major) * ring entry e^T
      auto scores = [&](uint32_t tdst, uint64_t da_in, int e) {
        const uint64_t da = opaque(da_in);
        const uint64_t db = desc_advance(d_r, (uint32_t)(e % kRing) * L::kTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
          mma_f16_ss_w(tmem + tdst, desc_advance(da, off), desc_advance(db, off), kIdescS,
                       kk > 0 ? 1u : 0u);
        }
      };
      bool ok = wait_bar_w(bar(L::kQFull), 0, abort_flag, status) && ring(1);
      if (ok) {
        scores(kTS0, d_q, 1);  // S(0) = Q K_0^T
        ok = ring(0);
      }
      if (ok) {
        scores(kTDP, d_g, 0);  // dP(0) = dO V_0^T
        tc_commit_w(bar(L::kSDFull));
        tc_commit_w(bar(L::kREmpty + 0));
      }
      for (int j = 0; ok && j < nk; ++j) {
        if (j + 1 < nk) {  // S(j+1) and dP(j+1) once the compute groups have read dP(j)
          // K_{j+1} is checked first, while the compute groups are still on
          // dP(j), so the check stays off the critical path
          if (!ring(2 * j + 3) ||
              !wait_bar_w(bar(L::kDPFree), (uint32_t)(j & 1), abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // S(j+1) goes into the slot dQ_{j-1} has read (MMAs run in order)
          scores(kTS0 + 128u * (uint32_t)((j + 1) & 1), d_q, 2 * j + 3);
          if (!ring(2 * j + 2)) {
            ok = false;
            break;
          }
          scores(kTDP, d_g, 2 * j + 2);
          tc_commit_w(bar(L::kSDFull + ((j + 1) & 1)));
          tc_commit_w(bar(L::kREmpty + (2 * j + 2) % kRing));
        }
        if (!wait_bar_w(bar(L::kPReady + (j & 1)), (uint32_t)((j >> 1) & 1), abort_flag,
                        status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t mk = opaque(desc_advance(m_r, (uint32_t)((2 * j + 1) % kRing) * L::kTile));
        const uint32_t ts = (uint32_t)opaque(tmem + kTS0 + 128u * (uint32_t)(j & 1));
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)  // dQ += dS_j K_j
          mma_f16_ts_w(tmem + kTDQ, ts + a_col128(kk), desc_advance(mk, (uint32_t)kk * 2048u),
                       kIdescAcc, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit_w(bar(L::kREmpty + (2 * j + 1) % kRing));
      }
      tc_commit_w(bar(L::kDone));
      tc_commit_w(bar(L::kDrain));
      wait_bar_drain(bar(L::kDrain), 0, status);
    }
  } else {
    regs_inc<kRegsCompute>();
    // ------------------------------------------------------------ compute
    const int grp = (warp - 4) >> 2;  // key half of every tile this group takes
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int row = ti * kT + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const bool in = row < mp.n_q;
    const float lse2 = in ? lse[(size_t)bh * mp.n_q + row] * kLog2e : 0.f;
    const float dl = in ? delta[(size_t)bh * mp.n_q + row] : 0.f;
    bool ok = true;
    int32_t ent_next = plan_entry(col_idx, e0, n_tj, status);
    for (int j = 0; j < nk; ++j) {
      const int32_t ent = ent_next;
      if (j + 1 < nk) ent_next = plan_entry(col_idx, e0 + j + 1, n_tj, status);  // in flight
      const int k0 = plan_index(ent) * kT + 64 * grp;
      uint32_t vis[2] = {0xffffffffu, 0xffffffffu};
      const bool all_vis = block_all_visible(mp, ti * kT, kT, k0, 64, plan_partial(ent));
      if (!all_vis) row_visibility<64>(vis, mp, row, k0, plan_partial(ent));
      ok = wait_bar_w(bar(L::kSDFull + (j & 1)), (uint32_t)((j >> 1) & 1), abort_flag, status);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = tmem + lane_base + kTS0 + 128u * (uint32_t)(j & 1) + 64u * grp;
      const uint32_t t_dp = tmem + lane_base + kTDP + 64u * grp;
      uint32_t sv[64], dpv[64];
      tmem_ld32(t_s, sv);
      tmem_ld32(t_s + 32u, sv + 32);
      tmem_ld32(t_dp, dpv);
      tmem_ld32(t_dp + 32u, dpv + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar(L::kDPFree));
      // dS = P * (dP - Delta); the softmax scale multiplies dQ in the epilogue
      uint32_t ds2[32];
      if (all_vis) {
        // packed fp32x2 arithmetic for the exponents and dS
        const float2 sc2 = make_float2(scale_log2, scale_log2);
        const float2 nl2 = make_float2(-lse2, -lse2), nd2 = make_float2(-dl, -dl);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float2 x = __ffma2_rn(
              make_float2(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1])), sc2, nl2);
          const float2 p = make_float2(ex2(x.x), ex2(x.y));
          const float2 d = __fmul2_rn(
              p, __fadd2_rn(make_float2(__uint_as_float(dpv[2 * c]),
                                        __uint_as_float(dpv[2 * c + 1])),
                            nd2));
          ds2[c] = pack2<T>(d.x, d.y);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          float d[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int cc = 2 * c + e;
            const bool on = (vis[cc >> 5] >> (cc & 31)) & 1u;
            const float p = on ? ex2(fmaf(__uint_as_float(sv[cc]), scale_log2, -lse2)) : 0.f;
            d[e] = p * (__uint_as_float(dpv[cc]) - dl);
          }
          ds2[c] = pack2<T>(d[0], d[1]);
        }
      }
      tmem_st32(t_s, ds2);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(L::kPReady + (j & 1)));
    }
    // epilogue: dQ columns [64*grp, 64*grp + 64) staged in Q's buffer
    if (ok) ok = wait_bar_w(bar(L::kDone), 0, abort_flag, status);
    if (ok && 64 * grp < D) {
      tc_fence_after();
      const uint32_t t_acc = tmem + lane_base + kTDQ + 64u * grp;
      const uint32_t region = sb + L::Q + (uint32_t)grp * 16384u;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t t[32];
        tmem_ld32(t_acc + 32u * c, t);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2)
          w[i2] = pack2<T>(__uint_as_float(t[2 * i2]) * scale, __uint_as_float(t[2 * i2 + 1]) * scale);
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2) {
          const uint32_t addr = region + sw128_offset((uint32_t)r, 32u * c + 8u * i2);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * i2]),
                       "r"(w[4 * i2 + 1]), "r"(w[4 * i2 + 2]), "r"(w[4 * i2 + 3])
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1 + grp, 128);
      if (r == 0) {
        tma_store_4d(&tmdq, region, 64 * grp, ti * kT, hh, bb);
        bulk_commit();
        bulk_wait_read0();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// dQ from stored dS (after dkdv_tc_kernel<..., DS = true>)
// ---------------------------------------------------------------------------
// dQ_i = scale * sum_j dS_ij K_j over the key tiles j query tile i sees (CSR
// plan), with dS_ij read from the tile dkdv_tc_kernel stored at
// (query (b, h)) * nnz + csc_pos[p] for CSR entry p.  No exponentials, no
// recomputed S or dP: the kernel moves 32 KB of dS per kept tile and is
// bound by HBM.  Persistent: one CTA per SM walks the (query tile,
// query (b, h)) items head-major, so its load pipeline never drains between
// items:
//   warp 0      streams (dS_ij, K_j) pairs of item after item through a
//               ring (dS by one 32 KB bulk copy, byte for byte in its stored
//               layout; K_j by TMA);
//   warp 1      issues the 128 x D x 128 MMAs (A = dS_ij, M-major without
//               swizzle; B = K_j, N-major) into one of two TMEM
//               accumulators, alternating per item;
//   warps 4-7   write an item's dQ (one query row per thread: TMEM ->
//               16-bit -> a swizzled staging tile -> TMA store) while the
//               next item accumulates in the other buffer.
template <int D>
struct DqGemmLayout {
  static constexpr int kStages = D > 64 ? 3 : 4;
  static constexpr uint32_t kDsTile = kT * kT * 2;   // dS [128 queries x 128 keys], ds_tile_offset
  static constexpr uint32_t kKTile = kT * D * 2;     // K_j [128 keys][D]
  static constexpr uint32_t kStage = kDsTile + kKTile;
  static constexpr uint32_t RING = 0;
  static constexpr uint32_t OUT = RING + kStages * kStage;  // dQ staging: D/64 swizzled [128][64] boxes
  static constexpr uint32_t BAR = OUT + kT * D * 2;
  static constexpr int kFull = 0;                     // [kStages]
  static constexpr int kEmpty = kStages;              // [kStages]
  static constexpr int kAccFull = 2 * kStages;        // [2] an item's last MMA done
  static constexpr int kAccFree = 2 * kStages + 2;    // [2] the epilogue has read the accumulator
  static constexpr int kDrain = 2 * kStages + 4;
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr uint32_t MISC = BAR + kNumBars * 8;
  static constexpr uint32_t kAlloc = MISC + 16 + 1024;
  static constexpr uint32_t kCols = 2 * D;            // two fp32 dQ accumulators
  static_assert(kAlloc <= 232448, "dQ GEMM shared memory exceeds the 227 KB per CTA");
};
constexpr int kDqGemmThreads = 256;  // warps 2-3 idle

template <typename T, int D>
__global__ void __launch_bounds__(kDqGemmThreads, 1)
    dq_gemm_kernel(const T* __restrict__ ds, const __grid_constant__ CUtensorMap tmk,
                   const __grid_constant__ CUtensorMap tmdq, T* __restrict__ dq, float scale,
                   MaskParams mp, const int32_t* __restrict__ row_ptr,
                   const int32_t* __restrict__ col_idx, const int32_t* __restrict__ csc_pos,
                   int nnz, int heads, int kv_group, int BH, Strides3 sdq, int* status) {
  using L = DqGemmLayout<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdesc = idesc_f16(kBF16, kT, D, true, true);  // M=128 q, N=D
  constexpr int kBoxes = D / 64;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sb + L::BAR + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_ti = ceil_div_dev(mp.n_q, kT);
  const int n_tj = ceil_div_dev(mp.n_kv, kT);
  const int n_items = n_ti * BH;
  // item it: query tile ti of query (b, h) bh, the kept key tiles
  // [e0, e0 + nk) of its CSR row
  struct Item {
    int ti, bh, e0, nk;
  };
  auto item = [&](int it) -> Item {
    Item w;
    w.bh = it / n_ti;
    w.ti = it - w.bh * n_ti;
    const PlanSpan span = plan_span(row_ptr, w.ti, n_tj, (int64_t)n_ti * n_tj, status);
    w.e0 = span.e0;
    w.nk = span.n;
    return w;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(bar(L::kFull + s), 1);
      mbar_init(bar(L::kEmpty + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar(L::kAccFull + a), 1);
      mbar_init(bar(L::kAccFree + a), 128);
    }
    mbar_init(bar(L::kDrain), 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t gp = 0;  // (dS, K) pairs loaded by this CTA so far
      bool run = true;
      for (int it = blockIdx.x; run && it < n_items; it += gridDim.x) {
        const Item w = item(it);
        const int hh = w.bh % heads, bb = w.bh / heads;
        const int64_t tile0 = (int64_t)w.bh * nnz;  // the query (b, h)'s first stored dS tile
        for (int p = 0; p < w.nk; ++p, ++gp) {
          const uint32_t s = gp % L::kStages, f = gp / L::kStages;
          if (f > 0 && !wait_bar(bar(L::kEmpty + s), (f - 1) & 1u, abort_flag, status)) {
            run = false;
            break;
          }
          const int kt = plan_index(plan_entry(col_idx, w.e0 + p, n_tj, status));
          const int cp = bounded(__ldg(csc_pos + w.e0 + p), nnz, status);
          const uint32_t dst = sb + L::RING + s * L::kStage;
          mbar_expect_tx(bar(L::kFull + s), L::kStage);
          bulk_load(dst, ds + (size_t)(tile0 + cp) * (kT * kT), L::kDsTile, bar(L::kFull + s));
          for (int b = 0; b < kBoxes; ++b)
            tma_load_4d(dst + L::kDsTile + (uint32_t)b * 16384u, &tmk, bar(L::kFull + s), 64 * b,
                        kt * kT, hh / kv_group, bb);
        }
      }
      // every copy this thread issued lands before the CTA can exit
      for (uint32_t s = 0; s < (uint32_t)L::kStages; ++s) {
        const uint32_t fills = gp > s ? (gp - 1 - s) / L::kStages + 1 : 0;
        if (fills) wait_bar_drain(bar(L::kFull + s), (fills - 1) & 1u, status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    uint32_t gc = 0;  // pairs consumed
    uint32_t ai = 0;  // items accumulated (items with no kept tile take no buffer)
    bool run = true;
    for (int it = blockIdx.x; run && it < n_items; it += gridDim.x) {
      const Item w = item(it);
      if (w.nk == 0) continue;
      const uint32_t a = ai & 1u;
      if (ai >= 2 && !wait_bar_w(bar(L::kAccFree + a), ((ai >> 1) - 1) & 1u, abort_flag, status))
        break;
      tc_fence_after();
      const uint32_t acc = tmem + a * (uint32_t)D;
      for (int p = 0; p < w.nk; ++p, ++gc) {
        const uint32_t s = gc % L::kStages;
        if (!wait_bar_w(bar(L::kFull + s), (gc / L::kStages) & 1u, abort_flag, status)) {
          run = false;
          break;
        }
        tc_fence_after();
        // A: 16 keys per k-step = ds_tile_offset(0, 16 kk); core matrices 128 B
        // apart along the keys, 2048 B apart along the queries
        const uint64_t da = smem_desc_noswizzle(sb + L::RING + s * L::kStage, 128u, kDsChunkBytes);
        const uint64_t db = desc_mnmajor(sb + L::RING + s * L::kStage + L::kDsTile, 16384u);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)
          mma_f16_ss_w(acc, desc_advance(da, ds_tile_offset(0, 16 * kk)),
                       desc_advance(db, (uint32_t)kk * 2048u), kIdesc,
                       (p > 0 || kk > 0) ? 1u : 0u);
        tc_commit_w(bar(L::kEmpty + s));
      }
      if (!run) break;
      tc_commit_w(bar(L::kAccFull + a));
      ++ai;
    }
    tc_commit_w(bar(L::kDrain));
    wait_bar_drain(bar(L::kDrain), 0, status);
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // thread r holds query row r of the item's dQ: TMEM -> 16-bit registers
    // (the accumulator is then released to the MMA warp) -> the staging tile
    // as D/64 swizzled [128][64] boxes -> TMA store, which overlaps the next
    // item's accumulation
    const int r = threadIdx.x - 128;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t ai = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item w = item(it);
      const int hh = w.bh % heads, bb = w.bh / heads;
      if (w.nk == 0) {  // the tile's rows see no key: dQ = 0
        const int row = w.ti * kT + r;
        if (row < mp.n_q) {
          uint4* dst = reinterpret_cast<uint4*>(dq + bb * sdq.b + hh * sdq.h + (int64_t)row * sdq.n);
          for (int cc = 0; cc < D / 8; ++cc) dst[cc] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const uint32_t a = ai & 1u;
      bool ok = wait_bar(bar(L::kAccFull + a), (ai >> 1) & 1u, abort_flag, status);
      if (!named_bar_and(1, 128, ok && !*abort_flag)) break;
      tc_fence_after();
      uint32_t packed[D / 2];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t t[32];
        tmem_ld32(tmem + lane_base + a * (uint32_t)D + 32u * c, t);
        tmem_wait_ld();
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2)
          packed[16 * c + i2] =
              pack2<T>(__uint_as_float(t[2 * i2]) * scale, __uint_as_float(t[2 * i2 + 1]) * scale);
      }
      tc_fence_before();
      mbar_arrive(bar(L::kAccFree + a));
      // the previous item's store has finished reading the staging tile
      if (r == 0) bulk_wait_read0();
      named_bar_sync(1, 128);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint32_t addr = sb + L::OUT + (uint32_t)(c >> 3) * 16384u +
                              sw128_offset((uint32_t)r, (uint32_t)(8 * c) & 63u);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(packed[4 * c]),
                     "r"(packed[4 * c + 1]), "r"(packed[4 * c + 2]), "r"(packed[4 * c + 3])
                     : "memory");
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (r == 0) {
        for (int b = 0; b < kBoxes; ++b)
          tma_store_4d(&tmdq, sb + L::OUT + (uint32_t)b * 16384u, 64 * b, w.ti * kT, hh, bb);
        bulk_commit();
      }
      ++ai;
    }
    if (r == 0) bulk_wait_read0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kCols);
  }
}

// Integer tuning knob from the environment (dflt when unset or empty).
int env_int(const char* name, int dflt) {
  const char* e = std::getenv(name);
  return e != nullptr && *e != '\0' ? std::atoi(e) : dflt;
}

template <typename T, int D>
int launch_bwd_tc(const void* q, const void* k, const void* v, const void* dout, void* dq,
                  void* dk, void* dv, const float* lse, const float* delta, int BH, float scale,
                  const MaskParams& mp, const Views& vw, const int32_t* dq_rp,
                  const int32_t* dq_ci, const int32_t* kv_cp, const int32_t* kv_ri,
                  float* part_ws, int sink_parts, const int32_t* csc_pos, int nnz, void* ds_ws,
                  int* status, cudaStream_t s, cudaStream_t s_dq = nullptr, int dq_grid = 0) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv, mdo, mdq, mdk, mdv;
  const uint64_t nq = (uint64_t)mp.n_q, nkv = (uint64_t)mp.n_kv;
  const uint64_t nh = (uint64_t)vw.heads, nb = (uint64_t)(BH / vw.heads);
  const uint64_t nhk = nh / (uint64_t)vw.kv_group;  // key/value heads
  if (int rc = make_tmap_4d(&mq, q, kBF16, D, nq, nh, nb, vw.q, kT)) return rc;
  if (int rc = make_tmap_4d(&mdo, dout, kBF16, D, nq, nh, nb, vw.dout, kT)) return rc;
  if (int rc = make_tmap_4d(&mk, k, kBF16, D, nkv, nhk, nb, vw.k, kT)) return rc;
  if (int rc = make_tmap_4d(&mv, v, kBF16, D, nkv, nhk, nb, vw.v, kT)) return rc;
  if (int rc = make_tmap_4d(&mdq, dq, kBF16, D, nq, nh, nb, vw.dq, kT)) return rc;
  if (int rc = make_tmap_4d(&mdk, dk, kBF16, D, nkv, nhk, nb, vw.dk, kT)) return rc;
  if (int rc = make_tmap_4d(&mdv, dv, kBF16, D, nkv, nhk, nb, vw.dv, kT)) return rc;
  // stored dS: BH * nnz tiles of 128 queries x 128 keys, 16-bit, 32 KB each
  // in the layout of ds_tile_offset
  const bool ds = ds_ws != nullptr;
  const float sl = scale * kLog2e;
  auto run_dkdv = [&](auto ds_tag) -> int {
    constexpr bool DS = decltype(ds_tag)::value;
    using L = DkdvLayout<D, DS>;
    auto kern = dkdv_tc_kernel<T, D, DS>;
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)L::kAlloc),
                            "cudaFuncSetAttribute(dkdv_tc)"))
      return rc;
    const int n_tj = ceil_div_i(mp.n_kv, kT);
    const int units = BH / vw.kv_group;  // (batch, key/value head) pairs
    {
      LaunchScope ls("dkdv_tc_kernel", s);
      kern<<<(n_tj - 1 + sink_parts) * units, kBwdThreads, L::kAlloc, s>>>(
          mq, mk, mv, mdo, mdk, mdv, (T*)ds_ws, nnz, (T*)dk, (T*)dv, lse, delta, scale, sl, mp,
          kv_cp,
          kv_ri, units, n_tj, vw.heads, vw.kv_group, vw.dk, vw.dv, part_ws, sink_parts, status);
    }
    return check_launch("dkdv_tc_kernel");
  };
  {
    const int n_tj = ceil_div_i(mp.n_kv, kT);
    const int units = BH / vw.kv_group;  // (batch, key/value head) pairs
    if (int rc = ds ? run_dkdv(std::true_type{}) : run_dkdv(std::false_type{})) return rc;
    if (sink_parts > 1) {
      LaunchScope ls("dkdv_sink_reduce_kernel", s);
      dkdv_sink_reduce_kernel<T, D><<<units, 256, 0, s>>>(part_ws, (T*)dk, (T*)dv, sink_parts,
                                                          vw.heads / vw.kv_group, mp.n_kv, scale,
                                                          vw.dk, vw.dv);
    }
  }
  if (int rc = check_launch("dkdv_sink_reduce_kernel")) return rc;
  if (ds) {
    using L = DqGemmLayout<D>;
    auto kern = dq_gemm_kernel<T, D>;
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)L::kAlloc),
                            "cudaFuncSetAttribute(dq_gemm)"))
      return rc;
    // on the side stream when given: it waits for this call's dK/dV pass
    // and then runs beside the next group's
    cudaStream_t sq = s;
    if (s_dq != nullptr && s_dq != s) {
      cudaEvent_t ev = nullptr;
      if (int rc = check_cuda(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming),
                              "cudaEventCreateWithFlags"))
        return rc;
      cudaError_t e = cudaEventRecord(ev, s);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(s_dq, ev, 0);
      cudaEventDestroy(ev);
      if (int rc = check_cuda(e, "dQ side stream: wait for the dK/dV pass")) return rc;
      sq = s_dq;
    }
    // persistent: one CTA per SM (or dq_grid CTAs) over the (query tile,
    // query (b, h)) items
    const int64_t items = (int64_t)ceil_div_i(mp.n_q, kT) * BH;
    if (items >= (1LL << 31))  // the kernel counts items in 32-bit integers
      return fail(SBFA_ERR_UNSUPPORTED, "dQ GEMM: B * H * ceil(n_q / 128) must be < 2^31");
    const int cap = dq_grid > 0 ? std::min(dq_grid, device_sm_count()) : device_sm_count();
    const int grid = (int)std::min<int64_t>(items, cap);
    LaunchScope ls("dq_gemm_kernel", sq);
    // the priority travels with the launch itself, so a captured CUDA graph
    // keeps it too
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kDqGemmThreads);
    cfg.dynamicSmemBytes = L::kAlloc;
    cfg.stream = sq;
    cudaLaunchAttribute attr[1];
    int least = 0, greatest = 0;
    if (sq != s && env_int("SBFA_DQ_PRIO", 1) != 0 &&
        cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess) {
      attr[0].id = cudaLaunchAttributePriority;
      attr[0].val.priority = greatest;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    }
    return check_cuda(cudaLaunchKernelEx(&cfg, kern, (const T*)ds_ws, mk, mdq, (T*)dq, scale, mp,
                                         dq_rp, dq_ci, csc_pos, nnz, vw.heads, vw.kv_group, BH,
                                         vw.dq, status),
                      "dq_gemm_kernel");
  }
  {
    using L = DqLayout<D>;
    auto kern = dq_tc_kernel<T, D>;
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)L::kAlloc),
                            "cudaFuncSetAttribute(dq_tc)"))
      return rc;
    dim3 grid(ceil_div_i(mp.n_q, kT), BH);
    LaunchScope ls("dq_tc_kernel", s);
    kern<<<grid, kBwdThreads, L::kAlloc, s>>>(mq, mk, mv, mdo, mdq, (T*)dq, lse, delta, scale, sl,
                                              mp, dq_rp, dq_ci, vw.heads, vw.kv_group, vw.dq,
                                              status);
  }
  return check_launch("dq_tc_kernel");
}


// Side stream for the dQ GEMM of calls on caller stream `s`: one per (device,
// caller stream), created on first use at the highest priority, so that the
// GEMM's CTAs take SMs as the dK/dV pass frees them.  Calls on different
// caller streams never share a side stream (a CUDA-graph capture of one
// caller stream takes in only its own).  nullptr (no overlap) past 64 caller
// streams or when creation fails.
cudaStream_t dq_side_stream(cudaStream_t s) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, cudaStream_t>, cudaStream_t>> table;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& e : table)
    if (e.first.first == dev && e.first.second == s) return e.second;
  if (table.size() >= 64) return nullptr;
  int least = 0, greatest = 0;
  if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) greatest = 0;
  cudaStream_t st = nullptr;
  if (cudaStreamCreateWithPriority(&st, cudaStreamNonBlocking, greatest) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  table.push_back({{dev, s}, st});
  return st;
}

// The backward over the stored dS, overlapped: the (b, h) units are cut into
// groups (whole batch elements, or head ranges of one when there are fewer
// batch elements than groups); group g's dK/dV pass runs on the caller's
// stream and its dQ GEMM, an HBM-bound kernel, on the side stream beside the
// tensor-bound dK/dV pass of group g + 1, on 3/8 of the SMs (the last
// group's on all of them, with nothing left to overlap).  Every group reads
// and writes only its own rows, so the order between groups does not matter;
// the caller's stream waits for the side stream before it returns, and a
// CUDA-graph capture of the caller's stream takes the side stream in and
// joins it again.  Four groups once the problem has at least 64 items per SM
// (at 14-55 per SM the extra launches and group tails cost as much as the
// overlap gains or more: -0.4 % at 28, -1 % at 55, -24 % at 14 items per SM
// forced to four groups);
// SBFA_BWD_GROUPS and SBFA_DQ_GRID override the group count and the dQ
// GEMM's CTA count (SBFA_BWD_GROUPS=1: one dK/dV pass, then dQ on the
// caller's stream).
template <typename T, int D>
int run_bwd_tc(const void* q, const void* k, const void* v, const void* dout, void* dq, void* dk,
               void* dv, const float* lse, const float* delta, int BH, float scale,
               const MaskParams& mp, const Views& vw, const int32_t* dq_rp, const int32_t* dq_ci,
               const int32_t* kv_cp, const int32_t* kv_ri, float* part_ws, int sink_parts,
               const int32_t* csc_pos, int nnz, void* ds_ws, int* status, cudaStream_t s) {
  const int sms = device_sm_count();
  const int64_t items = (int64_t)ceil_div_i(mp.n_q, kT) * BH;
  int want = env_int("SBFA_BWD_GROUPS", 0);
  if (want <= 0) want = items >= 64LL * sms ? 4 : 1;
  int dq_grid = env_int("SBFA_DQ_GRID", 0);
  if (dq_grid <= 0) dq_grid = std::max(1, sms * 3 / 8);
  const int H = vw.heads, B = BH / H, g = vw.kv_group;
  cudaStream_t side = ds_ws != nullptr && want > 1 ? dq_side_stream(s) : nullptr;
  if (side == nullptr)
    return launch_bwd_tc<T, D>(q, k, v, dout, dq, dk, dv, lse, delta, BH, scale, mp, vw, dq_rp,
                               dq_ci, kv_cp, kv_ri, part_ws, sink_parts, csc_pos, nnz, ds_ws,
                               status, s);
  int hsplit = std::max(1, want / std::max(B, 1));
  while (hsplit > 1 && (H % hsplit != 0 || (H / hsplit) % g != 0)) --hsplit;
  const int Hg = H / hsplit;
  Views vg = vw;
  vg.heads = Hg;
  const int64_t es = (int64_t)sizeof(T);
  int rc_groups = SBFA_OK;
  for (int bi = 0; bi < B && rc_groups == SBFA_OK; ++bi) {
    for (int hs = 0; hs < hsplit; ++hs) {
      const int h0 = hs * Hg;
      const int64_t u = (int64_t)bi * H + h0;  // the group's first query (b, h)
      auto qo = [&](const Strides3& st) { return (bi * st.b + (int64_t)h0 * st.h) * es; };
      auto ko = [&](const Strides3& st) { return (bi * st.b + (int64_t)(h0 / g) * st.h) * es; };
      const bool last = bi == B - 1 && hs == hsplit - 1;
      if (int rc = launch_bwd_tc<T, D>(
              static_cast<const char*>(q) + qo(vw.q), static_cast<const char*>(k) + ko(vw.k),
              static_cast<const char*>(v) + ko(vw.v), static_cast<const char*>(dout) + qo(vw.dout),
              static_cast<char*>(dq) + qo(vw.dq), static_cast<char*>(dk) + ko(vw.dk),
              static_cast<char*>(dv) + ko(vw.dv), lse + u * mp.n_q, delta + u * mp.n_q, Hg, scale,
              mp, vg, dq_rp, dq_ci, kv_cp, kv_ri,
              part_ws != nullptr ? part_ws + (u / g) * sink_parts * 2 * kT * D : nullptr,
              sink_parts, csc_pos, nnz,
              static_cast<char*>(ds_ws) + u * nnz * (int64_t)(kT * kT * 2), status, s, side,
              last ? 0 : dq_grid)) {
        rc_groups = rc;
        break;
      }
    }
  }
  // join even after a failed launch, so that nothing queued on the side
  // stream outlives the call unordered with the caller's stream
  cudaEvent_t ev = nullptr;
  cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if (e == cudaSuccess) {
    e = cudaEventRecord(ev, side);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ev, 0);
    cudaEventDestroy(ev);
  } else {
    e = cudaStreamSynchronize(side);  // no event to order with: wait for it here
  }
  if (rc_groups != SBFA_OK) return rc_groups;
  return check_cuda(e, "dQ side stream: join");
}

}  // namespace

int generic_delta(int dtype, const void* o, const void* dout, float* delta, int BH, int n_q,
                  int D, const Views& vw, cudaStream_t s);

// Bytes of fp32 partials the split sink tile needs under grouped-query
// attention (0 without grouping: the sink CTA of a unit then streams a single
// query head, as every other key tile's CTA does).
int64_t tc_bwd_split_bytes(int64_t BH, int kv_group, int64_t D) {
  if (kv_group <= 1) return 0;
  return BH / kv_group * (int64_t)kv_group * 2 * kT * D * (int64_t)sizeof(float);
}

// Bytes of the stored dS tiles (16-bit [128 keys][128 queries] per query
// (b, h) and kept 128 x 128 tile), or 0 where the dS path does not apply
// (head_dim 64 keeps the recomputing dQ kernel).
int64_t tc_bwd_ds_bytes(int64_t BH, int64_t nnz, int64_t D) {
  if (D != 128 || BH <= 0 || nnz <= 0 || BH * nnz >= (1ll << 31)) return 0;
  return BH * nnz * (int64_t)kT * kT * 2;
}

int tc_bwd(int dtype, int D, const void* q, const void* k, const void* v, const void* o,
           const float* lse, const void* dout, void* dq, void* dk, void* dv, float* delta, int BH,
           float scale, const MaskParams& mp, const Views& vw, const int32_t* dq_rp,
           const int32_t* dq_ci, const int32_t* kv_cp, const int32_t* kv_ri, void* split_ws,
           int64_t split_ws_bytes, const int32_t* csc_pos, int64_t nnz, void* ds_ws,
           int64_t ds_ws_bytes, int* status, cudaStream_t s) {
  if (int rc = generic_delta(dtype, o, dout, delta, BH, mp.n_q, D, vw, s)) return rc;
  const bool bf = dtype == SBFA_BF16;
  // split the sink tile over the group's query heads when the caller gave
  // room for the partials (else one CTA per unit streams every head)
  const int64_t need = tc_bwd_split_bytes(BH, vw.kv_group, D);
  const bool split = need > 0 && split_ws != nullptr && split_ws_bytes >= need &&
                     ((uintptr_t)split_ws & 15u) == 0;
  float* part = split ? static_cast<float*>(split_ws) : nullptr;
  const int parts = split ? vw.kv_group : 1;
  // dQ from stored dS when the caller gave room for it
  const int64_t ds_need = tc_bwd_ds_bytes(BH, nnz, D);
  const bool use_ds = ds_need > 0 && ds_ws != nullptr && csc_pos != nullptr &&
                      ds_ws_bytes >= ds_need && ((uintptr_t)ds_ws & 15u) == 0;
  void* dsw = use_ds ? ds_ws : nullptr;
  const int nz = use_ds ? (int)nnz : 0;
#define SBFA_BWD(TT, DD)                                                                       \
  return run_bwd_tc<TT, DD>(q, k, v, dout, dq, dk, dv, lse, delta, BH, scale, mp, vw, dq_rp,  \
                            dq_ci, kv_cp, kv_ri, part, parts, csc_pos, nz, dsw, status, s)
  if (D == 128) {
    if (bf) SBFA_BWD(__nv_bfloat16, 128);
    SBFA_BWD(__half, 128);
  }
  if (D == 64) {
    if (bf) SBFA_BWD(__nv_bfloat16, 64);
    SBFA_BWD(__half, 64);
  }
#undef SBFA_BWD
  return fail(SBFA_ERR_UNSUPPORTED, "tensor-core backward: head_dim must be 64 or 128");
}

}  // namespace sbfa
