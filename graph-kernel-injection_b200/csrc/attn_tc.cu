// Tensor-core block-sparse attention for sm_100a: TMA + tcgen05 + TMEM.
//
// Forward (replaces upstream _fwd_kernel, sparse_triton_kernel.py:231-352).
// One CTA per (pair of 128-row query tiles A/B, batch*head), 384 threads in
// three warpgroups (registers rebalanced with setmaxnreg: 88 / 208 / 208):
//   warp 0      TMA producer: Q_A, Q_B once, then K_j, V_j of every kept key
//               tile (plan CSR row, 256x128 tiles) into one STAGES-deep ring
//               that alternates K and V tiles;
//   warps 1, 2  MMA issuers for tile A and tile B (whole warp, one elected
//               lane issuing): S_X = Q_X K^T into TMEM, O_X += P_X V with
//               P_X read straight from TMEM;
//   warp 3      idle;
//   warps 4-7   softmax for tile A, warps 8-11 for tile B: thread t of a group
//               owns query row t (its TMEM lane).
// Every key tile is processed as two 64-key half-steps u = 2j + h so that S_X
// is double buffered: TMEM S_A [0,128) and S_B [128,256) each hold two 64-
// column slots, O_A [256,384), O_B [384,512).  Per half-step the softmax
// thread loads its 64 scores with tcgen05.ld, masks them (uniform all-visible
// test, else a 64-bit mask from token-rule intervals, the sequence end and
// the lifted block mask on partial tiles), runs the online softmax in base 2,
// rescales its O row in TMEM only when the running max grew by more than
// 2^8, and writes P (bf16/fp16) packed over the first 32 columns of the slot.
// MMA warp X per half-step: [P_X(u) ready] PV_X(u), QK_X(u+2) into the same
// slot.  MMAs from one thread execute in issue order, so QK_X(u+2) overwrites
// the slot only after PV_X(u) has read P_X(u); the softmax of u+1 (other
// slot) overlaps both.  An O rescale first waits for PV_X(u-1).
// Epilogue: O rows are normalised, staged in the Q buffer (128-byte swizzle)
// and written with a TMA store; LSE rows are stored directly.
// Numerics as upstream: natural-log LSE = m + log(l), empty rows give
// O = 0 and LSE = 0, P is rounded to the input type before P V.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "tc_attn_common.cuh"

namespace sbfa {
namespace {

using namespace tc;

constexpr int kTM = 128;   // rows per query tile (one TMEM lane per row)
constexpr int kPair = 2;   // query tiles per CTA
constexpr int kTN = 128;   // keys per key tile
constexpr int kHalf = 64;  // keys per half-step (one 64-column S slot)
constexpr int kFwdThreads = 384;
constexpr int kRegsCtl = 88;       // producer / MMA warpgroup (64 spills descriptor math)
constexpr int kRegsSoftmax = 208;  // each softmax warpgroup (128*88 + 256*208 == 384*168)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;
constexpr uint32_t kTmemCols = 512;  // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)

template <int D, int STAGES>
struct FwdLayout {
  static constexpr uint32_t kTile = kTM * D * 2;       // 128 rows x D, 16-bit
  static constexpr uint32_t Q = 0;                     // Q_A, Q_B; O staging in the epilogue
  static constexpr uint32_t KV = Q + kPair * kTile;    // ring: K_0, V_0, K_1, V_1, ...
  static constexpr uint32_t BAR = KV + STAGES * kTile;
  static constexpr int kQFull = 0;
  static constexpr int kKVFull = 1;
  static constexpr int kKVEmpty = 1 + STAGES;
  // S and P barriers are per (tile x, slot h) at 2x + h: a softmax group
  // may run one step ahead of the MMA warp, never two on the same slot
  static constexpr int kSFull = 1 + 2 * STAGES;   // [4]
  static constexpr int kPFull = 5 + 2 * STAGES;   // [4]
  static constexpr int kPVDone = 9 + 2 * STAGES;  // [2]
  static constexpr int kOFull = 11 + 2 * STAGES;  // [2]
  static constexpr int kDrain = 13 + 2 * STAGES;  // [2]
  static constexpr int kNumBars = 15 + 2 * STAGES;
  static constexpr uint32_t MISC = BAR + kNumBars * 8;  // [0] TMEM base, [1] abort flag
  static constexpr uint32_t kBytes = MISC + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;     // room to align the base to 1 KB
};

template <typename T, int D, int STAGES>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmo,
                  T* __restrict__ o, float* __restrict__ lse, float scale_log2, MaskParams mp,
                  const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx,
                  int heads, int kv_group, Strides3 so, int* status) {
  using L = FwdLayout<D, STAGES>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescQK = idesc_f16(kBF16, kTM, kHalf, false, false);
  constexpr uint32_t kIdescPV = idesc_f16(kBF16, kTM, D, false, true);
  constexpr int kBoxes = D / 64;  // 64-column boxes per tile row

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sb + L::BAR + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x;
  const int bh = blockIdx.y;
  const int hh = bh % heads, bb = bh / heads;  // TMA coordinates of the (batch, head) plane
  const int row0 = pair * kPair * kTM;
  const int n_tj = ceil_div_dev(mp.n_kv, kTN);  // key tiles (plan columns)
  const PlanSpan span = plan_span(row_ptr, pair, n_tj, (int64_t)gridDim.x * n_tj, status);
  const int e0 = span.e0;
  const int n = span.n;

  if (n == 0) {  // no kept key tile: O = 0, LSE = 0 for every row of the pair
    for (int idx = threadIdx.x; idx < kPair * kTM * (D / 8); idx += blockDim.x) {
      const int rr = idx / (D / 8), cc = idx % (D / 8);
      const int row = row0 + rr;
      if (row < mp.n_q)
        reinterpret_cast<uint4*>(o + bb * so.b + hh * so.h + (int64_t)row * so.n)[cc] =
            make_uint4(0, 0, 0, 0);
    }
    for (int rr = threadIdx.x; rr < kPair * kTM; rr += blockDim.x) {
      const int row = row0 + rr;
      if (row < mp.n_q) lse[(size_t)bh * mp.n_q + row] = 0.f;
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(bar(L::kQFull), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(L::kKVFull + s), 1);
      mbar_init(bar(L::kKVEmpty + s), kPair);  // released by both MMA warps
    }
    for (int x = 0; x < kPair; ++x) {
      mbar_init(bar(L::kSFull + 2 * x), 1);
      mbar_init(bar(L::kSFull + 2 * x + 1), 1);
      mbar_init(bar(L::kPFull + 2 * x), 128);
      mbar_init(bar(L::kPFull + 2 * x + 1), 128);
      mbar_init(bar(L::kPVDone + x), 1);
      mbar_init(bar(L::kOFull + x), 1);
    }
    mbar_init(bar(L::kDrain), 1);
    mbar_init(bar(L::kDrain + 1), 1);
    *abort_flag = 0;
    mbar_init_fence();
    // the resident Q_A, Q_B tiles are requested before the TMEM allocation
    // and the CTA-wide sync, so their latency overlaps them
    mbar_expect_tx(bar(L::kQFull), kPair * L::kTile);
    for (int x = 0; x < kPair; ++x)
      for (int r = 0; r < kBoxes; ++r)
        tma_load_4d(sb + L::Q + x * L::kTile + r * 16384u, &tmq, bar(L::kQFull), 64 * r,
                    row0 + x * kTM, hh, bb);
    // ... and so are the first ring entries, K_0 and V_0 (fresh slots 0, 1)
    const int kt0 = plan_index(plan_entry(col_idx, e0, n_tj, status));
    for (int part = 0; part < 2; ++part) {
      mbar_expect_tx(bar(L::kKVFull + part), L::kTile);
      for (int r = 0; r < kBoxes; ++r)
        tma_load_4d(sb + L::KV + part * L::kTile + r * 16384u, part == 0 ? &tmk : &tmv,
                    bar(L::kKVFull + part), 64 * r, kt0 * kTN, hh / kv_group, bb);
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
    // ------------------------------------------------------------ producer
      // (Q_A, Q_B, K_0 and V_0 were requested by this thread right after the
      // barrier set-up)
      int issued = 2;  // ring entries issued: entry 2j = K_j, 2j + 1 = V_j
      bool ok = true;
      int next_ent = n > 1 ? plan_entry(col_idx, e0 + 1, n_tj, status) : 0;
      for (int j = 1; ok && j < n; ++j) {
        const int kt = plan_index(next_ent);
        if (j + 1 < n) next_ent = plan_entry(col_idx, e0 + j + 1, n_tj, status);  // prefetch
        for (int part = 0; part < 2; ++part) {
          const int e = 2 * j + part;
          const int s = e % STAGES, f = e / STAGES;
          if (f > 0 && !wait_bar(bar(L::kKVEmpty + s), (uint32_t)((f - 1) & 1), abort_flag, status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(bar(L::kKVFull + s), L::kTile);
          for (int r = 0; r < kBoxes; ++r)
            tma_load_4d(sb + L::KV + s * L::kTile + r * 16384u, part == 0 ? &tmk : &tmv,
                        bar(L::kKVFull + s), 64 * r, kt * kTN, hh / kv_group, bb);
          issued = e + 1;
        }
      }
      // wait for our own copies still in flight (all consumed on success)
      wait_bar_drain(bar(L::kQFull), 0, status);
      for (int s = 0; s < STAGES; ++s) {
        const int fills = issued > s ? (issued - 1 - s) / STAGES + 1 : 0;
        if (fills) wait_bar_drain(bar(L::kKVFull + s), (uint32_t)((fills - 1) & 1), status);
      }
   } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    // warp 1 issues tile A's MMAs, warp 2 tile B's: each waits only on its
    // own softmax group, so one group's delay never holds the other's MMAs
    {
      const int x = warp - 1;
      auto kv_wait = [&](int e) -> bool {
        if (!wait_bar_w(bar(L::kKVFull + e % STAGES), (uint32_t)((e / STAGES) & 1), abort_flag,
                        status))
          return false;
        tc_fence_after();
        return true;
      };
      // base descriptors, built once; MMAs add constant offsets
      const uint64_t dq0 = desc_kmajor(sb + L::Q);
      const uint64_t dkv_k = desc_kmajor(sb + L::KV);
      const uint64_t dkv_v = desc_mnmajor(sb + L::KV, 16384u);
      const int U = 2 * n;  // half-steps: u = 2j + h covers keys [64h, 64h + 64) of tile j
      // S_X slot h = Q_X (K_j rows [64h, 64h + 64))^T
      auto qk = [&](int x, int u) {
        const int j = u >> 1, h = u & 1;
        const uint64_t dq = desc_advance(dq0, (uint32_t)x * L::kTile);
        const uint64_t dk =
            desc_advance(dkv_k, (uint32_t)((2 * j) % STAGES) * L::kTile + (uint32_t)h * 8192u);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
          mma_f16_ss_w(tmem + 128u * x + 64u * h, desc_advance(dq, off), desc_advance(dk, off),
                       kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      // O_X += P_X(u) V_j rows [64h, 64h + 64), P_X(u) packed in slot h
      auto pv = [&](int x, int u) {
        const int j = u >> 1, h = u & 1;
        const uint64_t dv = desc_advance(dkv_v, (uint32_t)((2 * j + 1) % STAGES) * L::kTile +
                                                    (uint32_t)h * 8192u);
#pragma unroll
        for (int kk = 0; kk < kHalf / 16; ++kk)
          mma_f16_ts_w(tmem + 256u + 128u * x, tmem + 128u * x + 64u * h + 8u * kk,
                       desc_advance(dv, (uint32_t)kk * 2048u), kIdescPV,
                       (u > 0 || kk > 0) ? 1u : 0u);
      };
      bool ok = wait_bar_w(bar(L::kQFull), 0, abort_flag, status) && kv_wait(0);
      if (ok) {
        for (int h = 0; h < 2; ++h) {
          qk(x, h);
          tc_commit_w(bar(L::kSFull + 2 * x + h));
        }
        tc_commit_w(bar(L::kKVEmpty + 0));  // K_0 fully read (one of the two arrivals)
      }
      for (int u = 0; ok && u < U; ++u) {
        const int j = u >> 1, h = u & 1;
        const bool more = u + 2 < U;
        if (h == 0 && !(kv_wait(2 * j + 1) && (!more || kv_wait(2 * j + 2)))) break;  // V_j, K_{j+1}
        if (!wait_bar_w(bar(L::kPFull + 2 * x + h), (uint32_t)((u >> 1) & 1), abort_flag,
                        status))
          break;
        tc_fence_after();
        pv(x, u);
        tc_commit_w(bar(L::kPVDone + x));
        if (more) {  // S_X(u+2) into the slot PV_X(u) has just read (MMAs run in order)
          qk(x, u + 2);
          tc_commit_w(bar(L::kSFull + 2 * x + h));
        }
        if (h == 1) {
          tc_commit_w(bar(L::kKVEmpty + (2 * j + 1) % STAGES));            // V_j fully read
          if (more) tc_commit_w(bar(L::kKVEmpty + (2 * j + 2) % STAGES));  // K_{j+1} too
        }
      }
      tc_commit_w(bar(L::kOFull + x));
      tc_commit_w(bar(L::kDrain + x));
      wait_bar_drain(bar(L::kDrain + x), 0, status);
    }
   }
  } else {
    regs_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax A / B
    const int x = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int row = row0 + x * kTM + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t t_sx = tmem + lane_base + 128u * x;
    const uint32_t t_o = tmem + lane_base + 256u + 128u * x;
    const int U = 2 * n;
    float m_run = -INFINITY, l_run = 0.f;
    bool settled = false;  // warp-uniform: every row of this warp has a finite running max
    bool ok = true;
    int32_t ent = 0, ent_next = plan_entry(col_idx, e0, n_tj, status);
    for (int u = 0; u < U; ++u) {
      const int j = u >> 1, h = u & 1;
      if (h == 0) {
        ent = ent_next;
        if (j + 1 < n) ent_next = plan_entry(col_idx, e0 + j + 1, n_tj, status);  // in flight
      }
      const int k0 = plan_index(ent) * kTN + kHalf * h;
      const bool partial = plan_partial(ent);
      uint32_t vis[2] = {0xffffffffu, 0xffffffffu};
      const bool all_vis = block_all_visible(mp, row0 + x * kTM, kTM, k0, kHalf, partial);
      if (!all_vis) row_visibility<kHalf>(vis, mp, row, k0, partial);
      ok = wait_bar_w(bar(L::kSFull + 2 * x + h), (uint32_t)((u >> 1) & 1), abort_flag, status);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = t_sx + 64u * h;
      uint32_t sv[kHalf];
      tmem_ld32(t_s, sv);
      tmem_ld32(t_s + 32u, sv + 32);
      tmem_wait_ld();
      if (!all_vis) {
#pragma unroll
        for (int c = 0; c < kHalf; ++c)
          if (!((vis[c >> 5] >> (c & 31)) & 1u)) sv[c] = __float_as_uint(-INFINITY);
      }
      if (!settled) {
        // some row of this warp has seen no visible key yet: its running
        // maximum starts at this step's maximum (stays -inf if none visible)
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = __uint_as_float(sv[i]);
#pragma unroll
        for (int c = 8; c < kHalf; ++c) mx[c & 7] = fmaxf(mx[c & 7], __uint_as_float(sv[c]));
        const float rm = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        if (m_run == -INFINITY) m_run = rm * scale_log2;
        settled = __all_sync(0xffffffffu, m_run != -INFINITY);
      }
      // Exponentials against the running maximum, with this step's maximum
      // reduced alongside them: a row whose maximum grew by more than 2^8
      // (rare after the first tiles) is redone below.  A row with nothing
      // visible so far has only -inf scores, so m_use = 0 gives p = 0.
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      float mx[4];
      float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t pk[kHalf / 2];
#pragma unroll
      for (int i = 0; i < 4; ++i) mx[i] = -INFINITY;
      const float2 sc2 = make_float2(scale_log2, scale_log2);
      const float2 nm2 = make_float2(-m_use, -m_use);
      // packed fp32x2 arithmetic (masked scores are -inf: 2^-inf = 0)
#pragma unroll
      for (int i = 0; i < kHalf / 2; ++i) {
        const float s0 = __uint_as_float(sv[2 * i]), s1 = __uint_as_float(sv[2 * i + 1]);
        mx[i & 3] = max3f(mx[i & 3], s0, s1);
        const float2 x2 = __ffma2_rn(make_float2(s0, s1), sc2, nm2);
        const float2 p = make_float2(ex2(x2.x), ex2(x2.y));
        acc[i & 1] = __fadd2_rn(acc[i & 1], p);
        pk[i] = pack2<T>(p.x, p.y);
      }
      const float rm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      const float m_new = rm * scale_log2;
      const bool need = (m_run != -INFINITY) && (m_new > m_run + kRescaleLog2);
      float rsum = (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
      if (!__any_sync(0xffffffffu, need)) {
        tmem_st16(t_s, pk);
        tmem_st16(t_s + 16u, pk + 16);
      } else {
        // O_X holds PV_X(0 .. u-1) once PV_X(u-1) has completed; the S_X(u)
        // barrier already implies PV_X(u-2), so this parity wait is exact
        ok = __all_sync(0xffffffffu, u == 0 || wait_bar(bar(L::kPVDone + x),
                                                        (uint32_t)((u - 1) & 1), abort_flag,
                                                        status));
        if (!ok) break;
        tc_fence_after();
        const float alpha = need ? ex2(m_run - m_new) : 1.f;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t t[32];
          tmem_ld32(t_o + 32u * c, t);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
          tmem_st32(t_o + 32u * c, t);
        }
        if (need) {
          l_run *= alpha;
          m_run = m_new;
        }
        // recompute P against the new maximum, 32 scores at a time from the
        // slot (P chunk c overwrites score columns that chunk c has read)
        rsum = 0.f;
        const float m_re = (m_run == -INFINITY) ? 0.f : m_run;
#pragma unroll 1
        for (int c = 0; c < kHalf / 32; ++c) {
          uint32_t t[32], w[16];
          tmem_ld32(t_s + 32u * c, t);
          tmem_wait_ld();
          const uint32_t vb = c == 0 ? vis[0] : vis[1];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float s0 = ((vb >> (2 * i)) & 1u) ? __uint_as_float(t[2 * i]) : -INFINITY;
            const float s1 = ((vb >> (2 * i + 1)) & 1u) ? __uint_as_float(t[2 * i + 1]) : -INFINITY;
            const float p0 = ex2(fmaf(s0, scale_log2, -m_re));
            const float p1 = ex2(fmaf(s1, scale_log2, -m_re));
            rsum += p0 + p1;
            w[i] = pack2<T>(p0, p1);
          }
          tmem_st16(t_s + 16u * c, w);
        }
      }
      tmem_wait_st();
      l_run += rsum;
      tc_fence_before();
      mbar_arrive(bar(L::kPFull + 2 * x + h));
    }
    if (ok) ok = wait_bar_w(bar(L::kOFull + x), 0, abort_flag, status);
    if (ok) {
      tc_fence_after();
      const bool valid = l_run > 0.f;
      const float inv = valid ? 1.f / l_run : 0.f;
      const uint32_t stage = sb + L::Q + (uint32_t)x * L::kTile;  // Q_X is no longer read
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t t[32];
        tmem_ld32(t_o + 32u * c, t);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack2<T>(__uint_as_float(t[2 * i]) * inv, __uint_as_float(t[2 * i + 1]) * inv);
        const uint32_t region = stage + (uint32_t)((32 * c) >> 6) * 16384u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t addr = region + sw128_offset((uint32_t)r, (uint32_t)((32 * c) & 63) + 8u * i);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * i]),
                       "r"(w[4 * i + 1]), "r"(w[4 * i + 2]), "r"(w[4 * i + 3])
                       : "memory");
        }
      }
      if (row < mp.n_q)
        lse[(size_t)bh * mp.n_q + row] = valid ? (m_run + log2f(l_run)) * kLn2 : 0.f;
      fence_proxy_async_smem();
      named_bar_sync(1 + x, 128);
      if (r == 0) {
        for (int b = 0; b < kBoxes; ++b)
          tma_store_4d(&tmo, stage + (uint32_t)b * 16384u, 64 * b, row0 + x * kTM, hh, bb);
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
// host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

template <typename T, int D, int STAGES>
int launch_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int BH,
                  float scale, const MaskParams& mp, const Views& vw, const int32_t* rp,
                  const int32_t* ci, int* status, cudaStream_t s) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv, mo;
  const uint64_t nh = (uint64_t)vw.heads, nb = (uint64_t)(BH / vw.heads);
  const uint64_t nhk = nh / (uint64_t)vw.kv_group;  // key/value heads
  if (int rc = tc::make_tmap_4d(&mq, q, kBF16, D, (uint64_t)mp.n_q, nh, nb, vw.q, kTM)) return rc;
  if (int rc = tc::make_tmap_4d(&mk, k, kBF16, D, (uint64_t)mp.n_kv, nhk, nb, vw.k, kTN)) return rc;
  if (int rc = tc::make_tmap_4d(&mv, v, kBF16, D, (uint64_t)mp.n_kv, nhk, nb, vw.v, kTN)) return rc;
  if (int rc = tc::make_tmap_4d(&mo, o, kBF16, D, (uint64_t)mp.n_q, nh, nb, vw.o, kTM)) return rc;
  using L = FwdLayout<D, STAGES>;
  auto kern = fwd_tc_kernel<T, D, STAGES>;
  if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)L::kAlloc),
                          "cudaFuncSetAttribute(fwd_tc)"))
    return rc;
  dim3 grid(ceil_div_i(mp.n_q, kPair * kTM), BH);
  {
    LaunchScope ls("fwd_tc_kernel", s);
    kern<<<grid, kFwdThreads, L::kAlloc, s>>>(mq, mk, mv, mo, (T*)o, lse, scale * kLog2e, mp, rp,
                                             ci, vw.heads, vw.kv_group, vw.o, status);
  }
  return check_launch("fwd_tc_kernel");
}

}  // namespace

namespace tc {
bool tma_compatible(const void* base, const Strides3& st) {
  return ((uintptr_t)base & 15u) == 0 && st.b % 8 == 0 && st.h % 8 == 0 && st.n % 8 == 0 &&
         st.b > 0 && st.h > 0 && st.n > 0;
}

int make_tmap_4d(CUtensorMap* map, const void* base, bool bf16, uint64_t cols, uint64_t rows,
                 uint64_t heads, uint64_t batch, const Strides3& st, uint32_t box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(SBFA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (!tma_compatible(base, st))
    return fail(SBFA_ERR_INVALID,
                "tensor-core path: tensors must be 16-byte aligned with batch, head and row "
                "strides that are positive multiples of 8 elements");
  cuuint64_t dims[4] = {cols, rows, heads, batch};
  cuuint64_t strides[3] = {(cuuint64_t)st.n * 2, (cuuint64_t)st.h * 2, (cuuint64_t)st.b * 2};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SBFA_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return SBFA_OK;
}
}  // namespace tc

bool tc_supports(int pass, int dtype, int64_t D) {
  if (dtype != SBFA_F16 && dtype != SBFA_BF16) return false;
  if (D != 64 && D != 128) return false;
  return pass >= 0 && pass <= 2;
}

int tc_tiles(int pass, int64_t* tm, int64_t* tn) {
  *tm = pass == 0 ? kPair * kTM : kTM;
  *tn = kTN;
  return SBFA_OK;
}

int tc_fwd(int dtype, int D, const void* q, const void* k, const void* v, void* o, float* lse,
           int BH, float scale, const MaskParams& mp, const Views& vw, const int32_t* rp,
           const int32_t* ci, int* status, cudaStream_t s) {
  const bool bf = dtype == SBFA_BF16;
  if (D == 128)
    return bf ? launch_fwd_tc<__nv_bfloat16, 128, 5>(q, k, v, o, lse, BH, scale, mp, vw, rp, ci,
                                                     status, s)
              : launch_fwd_tc<__half, 128, 5>(q, k, v, o, lse, BH, scale, mp, vw, rp, ci, status, s);
  if (D == 64)
    return bf ? launch_fwd_tc<__nv_bfloat16, 64, 8>(q, k, v, o, lse, BH, scale, mp, vw, rp, ci,
                                                    status, s)
              : launch_fwd_tc<__half, 64, 8>(q, k, v, o, lse, BH, scale, mp, vw, rp, ci, status, s);
  return fail(SBFA_ERR_UNSUPPORTED, "tensor-core forward: head_dim must be 64 or 128");
}


}  // namespace sbfa
