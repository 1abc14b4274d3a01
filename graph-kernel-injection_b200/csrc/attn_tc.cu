// Tensor-core block-sparse attention for sm_100a: TMA + tcgen05 + TMEM.
//
// Forward (replaces upstream _fwd_kernel, sparse_triton_kernel.py:231-352).
// One CTA per (128-row query tile, batch*head), 192 threads:
//   warp 0      TMA producer: Q once, then K and V tiles of the kept key
//               tiles (plan CSR row) into STAGES-deep rings;
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM
//               S buffers, O += P_j V_j into the TMEM O accumulator;
//   warps 2-5   softmax: thread t owns query row t (the TMEM lane it may
//               read), loads its 128 scores with tcgen05.ld, applies the
//               token rule on boundary tiles only, runs the online softmax
//               in base 2, rescales its O row in TMEM only when the running
//               max grew by more than 2^8, writes P (bf16/fp16) to shared
//               memory in the 128-byte-swizzled K-major layout the MMA reads.
// Pipelining: QK_{j+2} is issued as soon as softmax released S buffer j%2,
// so the tensor core computes the next scores while softmax runs.
// Numerics as upstream: natural-log LSE = m + log(l), empty rows give
// O = 0 and LSE = 0, P is rounded to the input type before P V.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "tc_prims.cuh"

namespace sbfa {
namespace {

using namespace tc;

constexpr int kTM = 128;  // query rows per tile
constexpr int kTN = 128;  // keys per tile
constexpr int kFwdThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;

template <int D, int STAGES>
struct FwdLayout {
  static constexpr uint32_t kTile = kTM * D * 2;  // one 128-row tile of Q, K or V
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t K0 = Q + kTile;
  static constexpr uint32_t V0 = K0 + STAGES * kTile;
  static constexpr uint32_t P = V0 + STAGES * kTile;
  static constexpr uint32_t BAR = P + kTM * kTN * 2;
  // barrier slots
  static constexpr int kQFull = 0;
  static constexpr int kKFull = 1;
  static constexpr int kKEmpty = 1 + STAGES;
  static constexpr int kVFull = 1 + 2 * STAGES;
  static constexpr int kVEmpty = 1 + 3 * STAGES;
  static constexpr int kSFull = 1 + 4 * STAGES;   // 2
  static constexpr int kSEmpty = 3 + 4 * STAGES;  // 2
  static constexpr int kPFull = 5 + 4 * STAGES;
  static constexpr int kPVDone = 6 + 4 * STAGES;
  static constexpr int kDrain = 7 + 4 * STAGES;
  static constexpr int kNumBars = 8 + 4 * STAGES;
  static constexpr uint32_t MISC = BAR + kNumBars * 8;  // [0] TMEM base, [1] abort flag
  static constexpr uint32_t kBytes = MISC + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;     // room to align the base to 1 KB
};

constexpr uint32_t kTmemCols = 512;  // S0 [0,128), S1 [128,256), O [256, 256+D)

__device__ __forceinline__ bool wait_bar_drain(uint32_t bar, uint32_t parity, int* status) {
  // used only to drain our own in-flight async work before exit: ignores the
  // abort flag but is still bounded
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

template <typename T, int D, int STAGES>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, T* __restrict__ o,
                  float* __restrict__ lse, float scale_log2, MaskParams mp,
                  const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx,
                  int* status) {
  using L = FwdLayout<D, STAGES>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescQK = idesc_f16(kBF16, kTM, kTN, false, false);
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
  const int ti = blockIdx.x;
  const int bh = blockIdx.y;
  const int e0 = row_ptr[ti];
  const int n = row_ptr[ti + 1] - e0;

  if (n == 0) {  // no kept key tile: O = 0, LSE = 0 for every row of the tile
    for (int idx = threadIdx.x; idx < kTM * (D / 8); idx += blockDim.x) {
      const int rr = idx / (D / 8), cc = idx % (D / 8);
      const int row = ti * kTM + rr;
      if (row < mp.n_q)
        reinterpret_cast<uint4*>(o + ((size_t)bh * mp.n_q + row) * D)[cc] = make_uint4(0, 0, 0, 0);
    }
    for (int rr = threadIdx.x; rr < kTM; rr += blockDim.x) {
      const int row = ti * kTM + rr;
      if (row < mp.n_q) lse[(size_t)bh * mp.n_q + row] = 0.f;
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(bar(L::kQFull), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(L::kKFull + s), 1);
      mbar_init(bar(L::kKEmpty + s), 1);
      mbar_init(bar(L::kVFull + s), 1);
      mbar_init(bar(L::kVEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(L::kSFull + b), 1);
      mbar_init(bar(L::kSEmpty + b), 128);
    }
    mbar_init(bar(L::kPFull), 128);
    mbar_init(bar(L::kPVDone), 1);
    mbar_init(bar(L::kDrain), 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_expect_tx(bar(L::kQFull), L::kTile);
      for (int r = 0; r < kBoxes; ++r)
        tma_load_3d(sb + L::Q + r * 16384u, &tmq, bar(L::kQFull), 64 * r, ti * kTM, bh);
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (uint32_t)((j / STAGES) & 1);
        const int kt = plan_index(col_idx[e0 + j]);
        if (j >= STAGES && !wait_bar(bar(L::kKEmpty + s), ph ^ 1u, abort_flag, status)) break;
        mbar_expect_tx(bar(L::kKFull + s), L::kTile);
        for (int r = 0; r < kBoxes; ++r)
          tma_load_3d(sb + L::K0 + s * L::kTile + r * 16384u, &tmk, bar(L::kKFull + s), 64 * r,
                      kt * kTN, bh);
        k_issued = j + 1;
        if (j >= STAGES && !wait_bar(bar(L::kVEmpty + s), ph ^ 1u, abort_flag, status)) break;
        mbar_expect_tx(bar(L::kVFull + s), L::kTile);
        for (int r = 0; r < kBoxes; ++r)
          tma_load_3d(sb + L::V0 + s * L::kTile + r * 16384u, &tmv, bar(L::kVFull + s), 64 * r,
                      kt * kTN, bh);
        v_issued = j + 1;
      }
      // wait for our own copies still in flight (all consumed on success)
      wait_bar_drain(bar(L::kQFull), 0, status);
      for (int s = 0; s < STAGES; ++s) {
        const int fk = k_issued > s ? (k_issued - 1 - s) / STAGES + 1 : 0;
        const int fv = v_issued > s ? (v_issued - 1 - s) / STAGES + 1 : 0;
        if (fk) wait_bar_drain(bar(L::kKFull + s), (uint32_t)((fk - 1) & 1), status);
        if (fv) wait_bar_drain(bar(L::kVFull + s), (uint32_t)((fv - 1) & 1), status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = wait_bar(bar(L::kQFull), 0, abort_flag, status);
      auto issue_qk = [&](int t) -> bool {
        const int s = t % STAGES, b = t & 1;
        if (!wait_bar(bar(L::kKFull + s), (uint32_t)((t / STAGES) & 1), abort_flag, status))
          return false;
        if (t >= 2 &&
            !wait_bar(bar(L::kSEmpty + b), (uint32_t)(((t - 2) >> 1) & 1), abort_flag, status))
          return false;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)b * 128u;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
          mma_f16_ss(d_tmem, desc_kmajor(sb + L::Q + off),
                     desc_kmajor(sb + L::K0 + s * L::kTile + off), kIdescQK, kk > 0 ? 1u : 0u);
        }
        tc_commit(bar(L::kSFull + b));
        tc_commit(bar(L::kKEmpty + s));
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && n > 1) ok = issue_qk(1);
      for (int j = 0; ok && j < n; ++j) {
        const int s = j % STAGES;
        if (!wait_bar(bar(L::kPFull), (uint32_t)(j & 1), abort_flag, status)) break;
        if (!wait_bar(bar(L::kVFull + s), (uint32_t)((j / STAGES) & 1), abort_flag, status)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTN / 16; ++kk) {
          const uint32_t poff = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
          mma_f16_ss(tmem + 256u, desc_kmajor(sb + L::P + poff),
                     desc_mnmajor(sb + L::V0 + s * L::kTile + (uint32_t)kk * 2048u, 16384u),
                     kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(bar(L::kPVDone));
        tc_commit(bar(L::kVEmpty + s));
        if (j + 2 < n) ok = issue_qk(j + 2);
      }
      tc_commit(bar(L::kDrain));
      wait_bar_drain(bar(L::kDrain), 0, status);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int row = ti * kTM + r;
    const int qpos = mp.q_off + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int32_t ent = col_idx[e0 + j];
      const int kt = plan_index(ent);
      const bool partial = plan_partial(ent);
      const int b = j & 1;
      ok = __all_sync(0xffffffffu,
                      wait_bar(bar(L::kSFull + b), (uint32_t)((j >> 1) & 1), abort_flag, status));
      if (!ok) break;
      tc_fence_after();
      float x[kTN];
      {
        uint32_t xr[kTN];
#pragma unroll
        for (int c = 0; c < kTN / 32; ++c)
          tmem_ld32(tmem + lane_base + (uint32_t)b * 128u + 32u * c, xr + 32 * c);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kTN; ++c) x[c] = __uint_as_float(xr[c]);
      }
      tc_fence_before();
      mbar_arrive(bar(L::kSEmpty + b));

      const int k0 = kt * kTN;
      const bool full = row < mp.n_q && k0 + kTN - 1 < mp.n_kv && !partial &&
                        (!mp.causal || (k0 + kTN - 1 <= qpos &&
                                        (k0 + kTN - 1 < mp.sink || k0 >= qpos - mp.window + 1)));
      if (!full) {
#pragma unroll
        for (int c = 0; c < kTN; ++c)
          if (!visible(mp, row, k0 + c, partial)) x[c] = -INFINITY;
      }
      float rmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTN; ++c) {
        x[c] *= scale_log2;
        rmax = fmaxf(rmax, x[c]);
      }
      const float m_new = fmaxf(m_run, rmax);
      const bool need = (m_run != -INFINITY) && (m_new > m_run + kRescaleLog2);
      bool pv_waited = false;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        ok = __all_sync(0xffffffffu, wait_bar(bar(L::kPVDone), (uint32_t)((j - 1) & 1),
                                              abort_flag, status));
        if (!ok) break;
        pv_waited = true;
        tc_fence_after();
        const float alpha = need ? ex2(m_run - m_new) : 1.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t t[32];
          tmem_ld32(tmem + lane_base + 256u + 32u * c, t);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
          tmem_st32(tmem + lane_base + 256u + 32u * c, t);
        }
        tmem_wait_st();
      }
      if (need) {
        l_run *= ex2(m_run - m_new);
        m_run = m_new;
      }
      if (m_run == -INFINITY) m_run = m_new;  // first visible key: O row and l are still 0
      const bool dead = (m_run == -INFINITY);
      uint32_t pk[kTN / 2];
      float rsum = 0.f;
#pragma unroll
      for (int c = 0; c < kTN / 2; ++c) {
        const float p0 = dead ? 0.f : ex2(x[2 * c] - m_run);
        const float p1 = dead ? 0.f : ex2(x[2 * c + 1] - m_run);
        rsum += p0 + p1;
        pk[c] = pack2<T>(p0, p1);
      }
      l_run += rsum;
      if (j > 0 && !pv_waited) {  // the single P buffer is free once P_{j-1} V_{j-1} is done
        ok = __all_sync(0xffffffffu, wait_bar(bar(L::kPVDone), (uint32_t)((j - 1) & 1),
                                              abort_flag, status));
        if (!ok) break;
      }
#pragma unroll
      for (int ch = 0; ch < kTN / 8; ++ch) {
        const uint32_t addr = sb + L::P + (uint32_t)(ch >> 3) * 16384u +
                              sw128_offset((uint32_t)r, (uint32_t)(ch & 7) * 8u);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * ch]),
                     "r"(pk[4 * ch + 1]), "r"(pk[4 * ch + 2]), "r"(pk[4 * ch + 3])
                     : "memory");
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(L::kPFull));
    }
    if (ok)
      ok = __all_sync(0xffffffffu, wait_bar(bar(L::kPVDone), (uint32_t)((n - 1) & 1), abort_flag,
                                            status));
    if (ok) {
      tc_fence_after();
      const bool valid = l_run > 0.f;
      const float inv = valid ? 1.f / l_run : 0.f;
      T* orow = o + ((size_t)bh * mp.n_q + row) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t t[32];
        tmem_ld32(tmem + lane_base + 256u + 32u * c, t);
        tmem_wait_ld();
        if (row < mp.n_q) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack2<T>(__uint_as_float(t[2 * i]) * inv, __uint_as_float(t[2 * i + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + 32 * c);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      if (row < mp.n_q)
        lse[(size_t)bh * mp.n_q + row] = valid ? (m_run + log2f(l_run)) * kLn2 : 0.f;
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
                  float scale, const MaskParams& mp, const int32_t* rp, const int32_t* ci,
                  int* status, cudaStream_t s) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv;
  if (int rc = tc::make_tmap_3d(&mq, q, kBF16, D, (uint64_t)mp.n_q, (uint64_t)BH, kTM)) return rc;
  if (int rc = tc::make_tmap_3d(&mk, k, kBF16, D, (uint64_t)mp.n_kv, (uint64_t)BH, kTN)) return rc;
  if (int rc = tc::make_tmap_3d(&mv, v, kBF16, D, (uint64_t)mp.n_kv, (uint64_t)BH, kTN)) return rc;
  using L = FwdLayout<D, STAGES>;
  auto kern = fwd_tc_kernel<T, D, STAGES>;
  if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)L::kAlloc),
                          "cudaFuncSetAttribute(fwd_tc)"))
    return rc;
  dim3 grid(ceil_div_i(mp.n_q, kTM), BH);
  {
    LaunchScope ls("fwd_tc_kernel", s);
    kern<<<grid, kFwdThreads, L::kAlloc, s>>>(mq, mk, mv, (T*)o, lse, scale * kLog2e, mp, rp, ci,
                                             status);
  }
  return check_launch("fwd_tc_kernel");
}

}  // namespace

namespace tc {
int make_tmap_3d(CUtensorMap* map, const void* base, bool bf16, uint64_t cols, uint64_t rows,
                 uint64_t planes, uint32_t box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(SBFA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (((uintptr_t)base & 15u) != 0)
    return fail(SBFA_ERR_INVALID, "tensor-core path: tensors must be 16-byte aligned");
  cuuint64_t dims[3] = {cols, rows, planes};
  cuuint64_t strides[2] = {cols * 2, cols * rows * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
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
  return pass == 0;
}

int tc_tiles(int pass, int64_t* tm, int64_t* tn) {
  (void)pass;
  *tm = kTM;
  *tn = kTN;
  return SBFA_OK;
}

int tc_fwd(int dtype, int D, const void* q, const void* k, const void* v, void* o, float* lse,
           int BH, float scale, const MaskParams& mp, const int32_t* rp, const int32_t* ci,
           int* status, cudaStream_t s) {
  const bool bf = dtype == SBFA_BF16;
  if (D == 128)
    return bf ? launch_fwd_tc<__nv_bfloat16, 128, 2>(q, k, v, o, lse, BH, scale, mp, rp, ci, status, s)
              : launch_fwd_tc<__half, 128, 2>(q, k, v, o, lse, BH, scale, mp, rp, ci, status, s);
  if (D == 64)
    return bf ? launch_fwd_tc<__nv_bfloat16, 64, 3>(q, k, v, o, lse, BH, scale, mp, rp, ci, status, s)
              : launch_fwd_tc<__half, 64, 3>(q, k, v, o, lse, BH, scale, mp, rp, ci, status, s);
  return fail(SBFA_ERR_UNSUPPORTED, "tensor-core forward: head_dim must be 64 or 128");
}

int tc_bwd(int, int, const void*, const void*, const void*, const void*, const float*,
           const void*, void*, void*, void*, float*, int, float, const MaskParams&,
           const int32_t*, const int32_t*, const int32_t*, const int32_t*, int*, cudaStream_t) {
  return fail(SBFA_ERR_UNSUPPORTED, "tensor-core backward not built");
}

}  // namespace sbfa
