// CUDA-core ("generic") block-sparse attention kernels.
//
// These cover every dtype (fp16, bf16, fp32, fp64) and head dims up to 256
// (128 for fp64) with exact fp32 (fp64 for fp64 inputs) arithmetic.  The
// tensor-core kernels in attn_tc.cu take the bf16/fp16 hot shapes; these
// take everything else (the upstream fp32 verification tiers, fp64
// gradcheck, head dims 16/32, tiny tiles).
//
// Semantics follow sparse_triton_kernel.py exactly:
//   forward  :231-352  online softmax, natural exp, LSE = m + log(l), empty
//                      rows -> O = 0, LSE = 0
//   delta    :355-392  Delta = rowsum(O * dO) in fp32
//   dK/dV    :395-509  P = exp(S - LSE), dV += P^T dO, dS = P (dP - Delta) s,
//                      dK += dS^T Q
//   dQ       :512-601  dQ += dS K
// but each kernel walks a compacted list of kept tiles (sbfa_build_plan)
// instead of scanning the whole mask row/column.
//
// Tiling: forward and dQ use 16 query rows x 64 keys per CTA step (4 warps,
// 4 rows per warp, lanes over keys for QK^T and over head-dim for PV);
// dK/dV uses 16 keys x 64 query rows.
#include <algorithm>

#include "sbfa_common.cuh"

namespace sbfa {
namespace {

constexpr int kRows = 16;      // query rows per CTA (fwd, dQ)
constexpr int kKeys = 64;      // keys per tile (fwd, dQ)
constexpr int kKvKeys = 16;    // keys per CTA (dK/dV)
constexpr int kKvRows = 64;    // query rows per tile (dK/dV)
constexpr int kThreads = 128;

template <typename A>
__device__ __forceinline__ A warp_max(A x) {
  for (int o = 16; o > 0; o >>= 1) x = max(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
template <typename A>
__device__ __forceinline__ A warp_sum(A x) {
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Load `rows` rows of an [N, D] slice (global row stride `sn` elements)
// starting at row r0 into smem (row stride `ld`), converting to the
// accumulator type; rows >= n are zero.
template <typename T, typename A>
__device__ __forceinline__ void load_rows(A* dst, int ld, const T* src, int64_t sn, int r0,
                                          int rows, int n, int D) {
  for (int i = threadIdx.x; i < rows * D; i += blockDim.x) {
    int r = i / D, d = i - r * D;
    int gr = r0 + r;
    dst[r * ld + d] = gr < n ? Elem<T>::to(src[(int64_t)gr * sn + d]) : A(0);
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T, int DPL>
__global__ void __launch_bounds__(kThreads) fwd_generic_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    T* __restrict__ o, float* __restrict__ lse, int D, double scale_f, MaskParams mp, Views vw,
    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx, int* status) {
  using A = typename Elem<T>::acc;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  A* Qs = reinterpret_cast<A*>(smem_raw);   // [kRows][D]
  A* Ks = Qs + kRows * D;                   // [kKeys][D+1]
  A* Vs = Ks + kKeys * (D + 1);             // [kKeys][D]
  const int ti = blockIdx.x;
  const size_t bh = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const A scale = (A)scale_f;
  const T* qb = q + vw.at(vw.q, (int)bh, 0);
  const T* kb = k + vw.at_kv(vw.k, (int)bh, 0);
  const T* vb = v + vw.at_kv(vw.v, (int)bh, 0);
  const int row0 = ti * kRows;
  load_rows<T, A>(Qs, D, qb, vw.q.n, row0, kRows, mp.n_q, D);

  A m[4], l[4], acc[4][DPL];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m[r] = neg_inf<A>();
    l[r] = 0;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[r][i] = 0;
  }
  const int n_tj = ceil_div_dev(mp.n_kv, kKeys);  // key tiles (plan columns)
  const PlanSpan span = plan_span(row_ptr, ti, n_tj, (int64_t)gridDim.x * n_tj, status);
  const int e0 = span.e0, e1 = span.e0 + span.n;
  for (int e = e0; e < e1; ++e) {
    const int32_t ent = plan_entry(col_idx, e, n_tj, status);
    const int tj = plan_index(ent);
    const bool partial = plan_partial(ent);
    const int k0 = tj * kKeys;
    __syncthreads();
    load_rows<T, A>(Ks, D + 1, kb, vw.k.n, k0, kKeys, mp.n_kv, D);
    load_rows<T, A>(Vs, D, vb, vw.v.n, k0, kKeys, mp.n_kv, D);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int lr = warp * 4 + r;
      const int row = row0 + lr;
      A s0 = 0, s1 = 0;
      const A* qr = Qs + lr * D;
      const A* k0r = Ks + lane * (D + 1);
      const A* k1r = Ks + (lane + 32) * (D + 1);
      for (int d = 0; d < D; ++d) {
        A qd = qr[d];
        s0 += qd * k0r[d];
        s1 += qd * k1r[d];
      }
      const bool v0 = visible(mp, row, k0 + lane, partial);
      const bool v1 = visible(mp, row, k0 + lane + 32, partial);
      s0 = v0 ? s0 * scale : neg_inf<A>();
      s1 = v1 ? s1 * scale : neg_inf<A>();
      const A m_new = max(m[r], warp_max(max(s0, s1)));
      if (m_new == neg_inf<A>()) continue;  // nothing visible yet (warp-uniform)
      const A alpha = (m[r] == neg_inf<A>()) ? A(0) : acc_exp<A>(m[r] - m_new);
      const A p0 = v0 ? acc_exp<A>(s0 - m_new) : A(0);
      const A p1 = v1 ? acc_exp<A>(s1 - m_new) : A(0);
      l[r] = l[r] * alpha + warp_sum(p0 + p1);
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[r][i] *= alpha;
      for (int j = 0; j < 32; ++j) {
        const A pj0 = __shfl_sync(0xffffffffu, p0, j);
        const A pj1 = __shfl_sync(0xffffffffu, p1, j);
        const A* va = Vs + j * D;
        const A* vc = Vs + (j + 32) * D;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int d = lane + 32 * i;
          if (d < D) acc[r][i] += pj0 * va[d] + pj1 * vc[d];
        }
      }
      m[r] = m_new;
    }
  }
  T* ob = o + vw.at(vw.o, (int)bh, 0);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = row0 + warp * 4 + r;
    if (row >= mp.n_q) continue;
    const bool valid = l[r] > A(0);
    const A inv = valid ? A(1) / l[r] : A(1);
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) ob[(int64_t)row * vw.o.n + d] = Elem<T>::from(valid ? acc[r][i] * inv : A(0));
    }
    if (lane == 0)
      lse[bh * mp.n_q + row] = valid ? (float)(m[r] + acc_log<A>(l[r])) : 0.0f;
  }
}

// ---------------------------------------------------------------------------
// Backward: Delta = rowsum(O * dO)
// ---------------------------------------------------------------------------
// One block row per (row tile, bh): no index division per row.  When a row
// is a whole number of 16-byte vectors (D * sizeof(T) % 16 == 0, at most 32
// of them), `g` = D / vec lanes share a row with one vector load each and
// 32 / g rows run per warp; otherwise a warp takes a row with scalar loads.
constexpr int kDeltaRows = 4;  // rows per lane group in the vectorised Delta path

template <typename T>
__global__ void delta_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                             float* __restrict__ delta, int n_q, int D, int g, Views vw) {
  using A = typename Elem<T>::acc;
  constexpr int kVec = 16 / sizeof(T);
  const int bh = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T* ob = o + vw.at(vw.o, bh, 0);
  const T* gb = dout + vw.at(vw.dout, bh, 0);
  float* db = delta + (int64_t)bh * n_q;
  if (g > 0) {
    // kDeltaRows rows per lane group, all loads issued before any use so each
    // thread keeps 2 * kDeltaRows 16-byte loads in flight
    const int per_warp = 32 / g;
    const int rows_per_block = (blockDim.x >> 5) * per_warp;
    const int row0 = (blockIdx.x * kDeltaRows * (blockDim.x >> 5) + warp) * per_warp + lane / g;
    const int sub = lane % g;
    uint4 a[kDeltaRows], b[kDeltaRows];
#pragma unroll
    for (int k = 0; k < kDeltaRows; ++k) {
      const int row = row0 + k * rows_per_block;
      if (row < n_q) {
        a[k] = *reinterpret_cast<const uint4*>(ob + (int64_t)row * vw.o.n + sub * kVec);
        b[k] = *reinterpret_cast<const uint4*>(gb + (int64_t)row * vw.dout.n + sub * kVec);
      } else {
        a[k] = make_uint4(0, 0, 0, 0);
        b[k] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int k = 0; k < kDeltaRows; ++k) {
      const int row = row0 + k * rows_per_block;
      const T* ta = reinterpret_cast<const T*>(&a[k]);
      const T* tb = reinterpret_cast<const T*>(&b[k]);
      A s = 0;
#pragma unroll
      for (int i = 0; i < kVec; ++i) s += Elem<T>::to(ta[i]) * Elem<T>::to(tb[i]);
      for (int off = g >> 1; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (row < n_q && sub == 0) db[row] = (float)s;
    }
  } else {
    const int row = blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= n_q) return;
    A s = 0;
    for (int d = lane; d < D; d += 32)
      s += Elem<T>::to(ob[(int64_t)row * vw.o.n + d]) * Elem<T>::to(gb[(int64_t)row * vw.dout.n + d]);
    s = warp_sum(s);
    if (lane == 0) db[row] = (float)s;
  }
}

// Launch of delta_kernel for any dtype; vector loads when every row start
// is 16-byte aligned.
template <typename T>
int launch_delta(const void* o, const void* dout, float* delta, int BH, int n_q, int D,
                 const Views& vw, cudaStream_t s) {
  constexpr int kVec = 16 / sizeof(T);
  const bool vec_ok = D % kVec == 0 && D / kVec <= 32 && ((D / kVec) & (D / kVec - 1)) == 0 &&
                      ((uintptr_t)o % 16 == 0) && ((uintptr_t)dout % 16 == 0) &&
                      vw.o.n % kVec == 0 && vw.o.h % kVec == 0 && vw.o.b % kVec == 0 &&
                      vw.dout.n % kVec == 0 && vw.dout.h % kVec == 0 && vw.dout.b % kVec == 0;
  const int g = vec_ok ? D / kVec : 0;
  const int rows_per_block = g > 0 ? 8 * (32 / g) * kDeltaRows : 8;
  dim3 grid(ceil_div_i(n_q, rows_per_block), BH);
  {
    LaunchScope ls("delta_kernel", s);
    delta_kernel<T><<<grid, 256, 0, s>>>((const T*)o, (const T*)dout, delta, n_q, D, g, vw);
  }
  return check_launch("delta_kernel");
}

// ---------------------------------------------------------------------------
// Backward: dQ
// ---------------------------------------------------------------------------
template <typename T, int DPL>
__global__ void __launch_bounds__(kThreads) dq_generic_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ delta, T* __restrict__ dq, int D, double scale_f, MaskParams mp,
    Views vw, const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx,
    int* status) {
  using A = typename Elem<T>::acc;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  A* Qs = reinterpret_cast<A*>(smem_raw);   // [kRows][D]
  A* dOs = Qs + kRows * D;                  // [kRows][D]
  A* Ks = dOs + kRows * D;                  // [kKeys][D+1]
  A* Vs = Ks + kKeys * (D + 1);             // [kKeys][D+1]
  const int ti = blockIdx.x;
  const size_t bh = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const A scale = (A)scale_f;
  const T* kb = k + vw.at_kv(vw.k, (int)bh, 0);
  const T* vb = v + vw.at_kv(vw.v, (int)bh, 0);
  const int row0 = ti * kRows;
  load_rows<T, A>(Qs, D, q + vw.at(vw.q, (int)bh, 0), vw.q.n, row0, kRows, mp.n_q, D);
  load_rows<T, A>(dOs, D, dout + vw.at(vw.dout, (int)bh, 0), vw.dout.n, row0, kRows, mp.n_q, D);
  A lse_r[4], del_r[4], acc[4][DPL];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = row0 + warp * 4 + r;
    lse_r[r] = row < mp.n_q ? (A)lse[bh * mp.n_q + row] : A(0);
    del_r[r] = row < mp.n_q ? (A)delta[bh * mp.n_q + row] : A(0);
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[r][i] = 0;
  }
  const int n_tj = ceil_div_dev(mp.n_kv, kKeys);  // key tiles (plan columns)
  const PlanSpan span = plan_span(row_ptr, ti, n_tj, (int64_t)gridDim.x * n_tj, status);
  const int e0 = span.e0, e1 = span.e0 + span.n;
  for (int e = e0; e < e1; ++e) {
    const int32_t ent = plan_entry(col_idx, e, n_tj, status);
    const int tj = plan_index(ent);
    const bool partial = plan_partial(ent);
    const int k0 = tj * kKeys;
    __syncthreads();
    load_rows<T, A>(Ks, D + 1, kb, vw.k.n, k0, kKeys, mp.n_kv, D);
    load_rows<T, A>(Vs, D + 1, vb, vw.v.n, k0, kKeys, mp.n_kv, D);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int lr = warp * 4 + r;
      const int row = row0 + lr;
      const A* qr = Qs + lr * D;
      const A* dor = dOs + lr * D;
      A s0 = 0, s1 = 0, dp0 = 0, dp1 = 0;
      const A* k0r = Ks + lane * (D + 1);
      const A* k1r = Ks + (lane + 32) * (D + 1);
      const A* v0r = Vs + lane * (D + 1);
      const A* v1r = Vs + (lane + 32) * (D + 1);
      for (int d = 0; d < D; ++d) {
        const A qd = qr[d], gd = dor[d];
        s0 += qd * k0r[d];
        s1 += qd * k1r[d];
        dp0 += gd * v0r[d];
        dp1 += gd * v1r[d];
      }
      const bool vis0 = visible(mp, row, k0 + lane, partial);
      const bool vis1 = visible(mp, row, k0 + lane + 32, partial);
      const A p0 = vis0 ? acc_exp<A>(s0 * scale - lse_r[r]) : A(0);
      const A p1 = vis1 ? acc_exp<A>(s1 * scale - lse_r[r]) : A(0);
      const A ds0 = p0 * (dp0 - del_r[r]) * scale;
      const A ds1 = p1 * (dp1 - del_r[r]) * scale;
      for (int j = 0; j < 32; ++j) {
        const A a0 = __shfl_sync(0xffffffffu, ds0, j);
        const A a1 = __shfl_sync(0xffffffffu, ds1, j);
        const A* ka = Ks + j * (D + 1);
        const A* kc = Ks + (j + 32) * (D + 1);
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int d = lane + 32 * i;
          if (d < D) acc[r][i] += a0 * ka[d] + a1 * kc[d];
        }
      }
    }
  }
  T* dqb = dq + vw.at(vw.dq, (int)bh, 0);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = row0 + warp * 4 + r;
    if (row >= mp.n_q) continue;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) dqb[(int64_t)row * vw.dq.n + d] = Elem<T>::from(acc[r][i]);
    }
  }
}

// ---------------------------------------------------------------------------
// Backward: dK, dV
// ---------------------------------------------------------------------------
template <typename T, int DPL>
__global__ void __launch_bounds__(kThreads) dkdv_generic_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ delta, T* __restrict__ dk, T* __restrict__ dv, int D,
    double scale_f, MaskParams mp, Views vw, const int32_t* __restrict__ col_ptr,
    const int32_t* __restrict__ row_idx, int* status) {
  using A = typename Elem<T>::acc;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  A* Ks = reinterpret_cast<A*>(smem_raw);   // [kKvKeys][D]
  A* Vs = Ks + kKvKeys * D;                 // [kKvKeys][D]
  A* Qs = Vs + kKvKeys * D;                 // [kKvRows][D+1]
  A* dOs = Qs + kKvRows * (D + 1);          // [kKvRows][D+1]
  A* Ls = dOs + kKvRows * (D + 1);          // [kKvRows]
  A* Dl = Ls + kKvRows;                     // [kKvRows]
  // one CTA per (key tile, batch, key/value head): the query heads of the
  // group all accumulate into the same dK, dV rows
  const int tj = blockIdx.x;
  const int kv_heads = vw.heads / vw.kv_group;
  const int bh0 = (int)(blockIdx.y / kv_heads) * vw.heads +
                  (int)(blockIdx.y % kv_heads) * vw.kv_group;  // first query head's bh
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const A scale = (A)scale_f;
  const int key0 = tj * kKvKeys;
  load_rows<T, A>(Ks, D, k + vw.at_kv(vw.k, bh0, 0), vw.k.n, key0, kKvKeys, mp.n_kv, D);
  load_rows<T, A>(Vs, D, v + vw.at_kv(vw.v, bh0, 0), vw.v.n, key0, kKvKeys, mp.n_kv, D);
  A adk[4][DPL], adv[4][DPL];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int i = 0; i < DPL; ++i) adk[c][i] = adv[c][i] = 0;
  const int n_ti = ceil_div_dev(mp.n_q, kKvRows);  // query tiles (plan rows)
  const PlanSpan span = plan_span(col_ptr, tj, n_ti, (int64_t)n_ti * gridDim.x, status);
  const int e0 = span.e0, ne = span.n;
  for (int it = 0; it < ne * vw.kv_group; ++it) {
    const int bh = bh0 + it / ne;
    const T* qb = q + vw.at(vw.q, bh, 0);
    const T* gb = dout + vw.at(vw.dout, bh, 0);
    const int32_t ent = plan_entry(row_idx, e0 + it % ne, n_ti, status);
    const int ti = plan_index(ent);
    const bool partial = plan_partial(ent);
    const int r0 = ti * kKvRows;
    __syncthreads();
    load_rows<T, A>(Qs, D + 1, qb, vw.q.n, r0, kKvRows, mp.n_q, D);
    load_rows<T, A>(dOs, D + 1, gb, vw.dout.n, r0, kKvRows, mp.n_q, D);
    for (int i = threadIdx.x; i < kKvRows; i += blockDim.x) {
      const int row = r0 + i;
      Ls[i] = row < mp.n_q ? (A)lse[(int64_t)bh * mp.n_q + row] : A(0);
      Dl[i] = row < mp.n_q ? (A)delta[(int64_t)bh * mp.n_q + row] : A(0);
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int lk = warp * 4 + c;
      const int key = key0 + lk;
      const A* kr = Ks + lk * D;
      const A* vr = Vs + lk * D;
      const A* q0r = Qs + lane * (D + 1);
      const A* q1r = Qs + (lane + 32) * (D + 1);
      const A* g0r = dOs + lane * (D + 1);
      const A* g1r = dOs + (lane + 32) * (D + 1);
      A s0 = 0, s1 = 0, dp0 = 0, dp1 = 0;
      for (int d = 0; d < D; ++d) {
        const A kd = kr[d], vd = vr[d];
        s0 += q0r[d] * kd;
        s1 += q1r[d] * kd;
        dp0 += g0r[d] * vd;
        dp1 += g1r[d] * vd;
      }
      const bool vis0 = visible(mp, r0 + lane, key, partial);
      const bool vis1 = visible(mp, r0 + lane + 32, key, partial);
      const A p0 = vis0 ? acc_exp<A>(s0 * scale - Ls[lane]) : A(0);
      const A p1 = vis1 ? acc_exp<A>(s1 * scale - Ls[lane + 32]) : A(0);
      const A ds0 = p0 * (dp0 - Dl[lane]) * scale;
      const A ds1 = p1 * (dp1 - Dl[lane + 32]) * scale;
      for (int j = 0; j < 32; ++j) {
        const A pa = __shfl_sync(0xffffffffu, p0, j);
        const A pb = __shfl_sync(0xffffffffu, p1, j);
        const A sa = __shfl_sync(0xffffffffu, ds0, j);
        const A sb = __shfl_sync(0xffffffffu, ds1, j);
        const A* ga = dOs + j * (D + 1);
        const A* gc = dOs + (j + 32) * (D + 1);
        const A* qa = Qs + j * (D + 1);
        const A* qc = Qs + (j + 32) * (D + 1);
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int d = lane + 32 * i;
          if (d < D) {
            adv[c][i] += pa * ga[d] + pb * gc[d];
            adk[c][i] += sa * qa[d] + sb * qc[d];
          }
        }
      }
    }
  }
  T* dkb = dk + vw.at_kv(vw.dk, bh0, 0);
  T* dvb = dv + vw.at_kv(vw.dv, bh0, 0);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int key = key0 + warp * 4 + c;
    if (key >= mp.n_kv) continue;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) {
        dkb[(int64_t)key * vw.dk.n + d] = Elem<T>::from(adk[c][i]);
        dvb[(int64_t)key * vw.dv.n + d] = Elem<T>::from(adv[c][i]);
      }
    }
  }
}

template <typename T>
size_t fwd_smem(int D) {
  return sizeof(typename Elem<T>::acc) * ((size_t)kRows * D + kKeys * (D + 1) + kKeys * D);
}
template <typename T>
size_t dq_smem(int D) {
  return sizeof(typename Elem<T>::acc) * (2 * (size_t)kRows * D + 2 * kKeys * (D + 1));
}
template <typename T>
size_t dkdv_smem(int D) {
  return sizeof(typename Elem<T>::acc) *
         (2 * (size_t)kKvKeys * D + 2 * kKvRows * (D + 1) + 2 * kKvRows);
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
  return check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bytes),
                    "cudaFuncSetAttribute(generic)");
}

template <typename T, int DPL>
int launch_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int BH,
               int D, double scale, const MaskParams& mp, const Views& vw, const int32_t* row_ptr,
               const int32_t* col_idx, cudaStream_t s) {
  auto kern = fwd_generic_kernel<T, DPL>;
  size_t sm = fwd_smem<T>(D);
  if (int rc = set_smem(kern, sm)) return rc;
  dim3 grid(ceil_div_i(mp.n_q, kRows), BH);
  {
    LaunchScope ls("fwd_generic_kernel", s);
    kern<<<grid, kThreads, sm, s>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, lse, D,
                                    scale, mp, vw, row_ptr, col_idx, device_status_ptr());
  }
  return check_launch("fwd_generic_kernel");
}

template <typename T, int DPL>
int launch_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
               const void* dout, void* dq, void* dk, void* dv, float* delta, int BH, int D,
               double scale, const MaskParams& mp, const Views& vw, const int32_t* dq_row_ptr,
               const int32_t* dq_col_idx, const int32_t* kv_col_ptr,
               const int32_t* kv_row_idx, cudaStream_t s) {
  if (int rc = launch_delta<T>(o, dout, delta, BH, mp.n_q, D, vw, s)) return rc;
  {
    auto kern = dkdv_generic_kernel<T, DPL>;
    size_t sm = dkdv_smem<T>(D);
    if (int rc = set_smem(kern, sm)) return rc;
    dim3 grid(ceil_div_i(mp.n_kv, kKvKeys), BH / vw.kv_group);
    {
      LaunchScope ls("dkdv_generic_kernel", s);
      kern<<<grid, kThreads, sm, s>>>((const T*)q, (const T*)k, (const T*)v, (const T*)dout,
                                      lse, delta, (T*)dk, (T*)dv, D, scale, mp, vw,
                                      kv_col_ptr, kv_row_idx, device_status_ptr());
    }
    if (int rc = check_launch("dkdv_generic_kernel")) return rc;
  }
  {
    auto kern = dq_generic_kernel<T, DPL>;
    size_t sm = dq_smem<T>(D);
    if (int rc = set_smem(kern, sm)) return rc;
    dim3 grid(ceil_div_i(mp.n_q, kRows), BH);
    {
      LaunchScope ls("dq_generic_kernel", s);
      kern<<<grid, kThreads, sm, s>>>((const T*)q, (const T*)k, (const T*)v, (const T*)dout,
                                      lse, delta, (T*)dq, D, scale, mp, vw, dq_row_ptr,
                                      dq_col_idx, device_status_ptr());
    }
    return check_launch("dq_generic_kernel");
  }
}

template <typename T>
int dispatch_fwd(int D, const void* q, const void* k, const void* v, void* o, float* lse,
                 int BH, double scale, const MaskParams& mp, const Views& vw, const int32_t* rp,
                 const int32_t* ci, cudaStream_t s) {
  if (D <= 32) return launch_fwd<T, 1>(q, k, v, o, lse, BH, D, scale, mp, vw, rp, ci, s);
  if (D <= 64) return launch_fwd<T, 2>(q, k, v, o, lse, BH, D, scale, mp, vw, rp, ci, s);
  if (D <= 128) return launch_fwd<T, 4>(q, k, v, o, lse, BH, D, scale, mp, vw, rp, ci, s);
  return launch_fwd<T, 8>(q, k, v, o, lse, BH, D, scale, mp, vw, rp, ci, s);
}

template <typename T>
int dispatch_bwd(int D, const void* q, const void* k, const void* v, const void* o,
                 const float* lse, const void* dout, void* dq, void* dk, void* dv, float* delta,
                 int BH, double scale, const MaskParams& mp, const Views& vw, const int32_t* a,
                 const int32_t* b, const int32_t* c, const int32_t* d, cudaStream_t s) {
  if (D <= 32)
    return launch_bwd<T, 1>(q, k, v, o, lse, dout, dq, dk, dv, delta, BH, D, scale, mp, vw, a, b, c, d, s);
  if (D <= 64)
    return launch_bwd<T, 2>(q, k, v, o, lse, dout, dq, dk, dv, delta, BH, D, scale, mp, vw, a, b, c, d, s);
  if (D <= 128)
    return launch_bwd<T, 4>(q, k, v, o, lse, dout, dq, dk, dv, delta, BH, D, scale, mp, vw, a, b, c, d, s);
  return launch_bwd<T, 8>(q, k, v, o, lse, dout, dq, dk, dv, delta, BH, D, scale, mp, vw, a, b, c, d, s);
}

}  // namespace

// Delta = rowsum(O * dO) in fp32 (used by the tensor-core backward too).
int generic_delta(int dtype, const void* o, const void* dout, float* delta, int BH, int n_q,
                  int D, const Views& vw, cudaStream_t s) {
  switch (dtype) {
    case SBFA_F16: return launch_delta<__half>(o, dout, delta, BH, n_q, D, vw, s);
    case SBFA_BF16: return launch_delta<__nv_bfloat16>(o, dout, delta, BH, n_q, D, vw, s);
    case SBFA_F32: return launch_delta<float>(o, dout, delta, BH, n_q, D, vw, s);
    case SBFA_F64: return launch_delta<double>(o, dout, delta, BH, n_q, D, vw, s);
  }
  return fail(SBFA_ERR_INVALID, "unknown dtype");
}

// Entry points used by capi.cu.
int generic_tiles(int pass, int64_t* tm, int64_t* tn) {
  if (pass == 2) { *tm = kKvRows; *tn = kKvKeys; }
  else { *tm = kRows; *tn = kKeys; }
  return SBFA_OK;
}

bool generic_supports(int dtype, int64_t D) {
  if (D <= 0) return false;
  if (dtype == SBFA_F64) return D <= 128;
  return D <= 256;
}

int generic_fwd(int dtype, int D, const void* q, const void* k, const void* v, void* o,
                float* lse, int BH, double scale, const MaskParams& mp, const Views& vw,
                const int32_t* rp, const int32_t* ci, cudaStream_t s) {
  switch (dtype) {
    case SBFA_F16: return dispatch_fwd<__half>(D, q, k, v, o, lse, BH, scale, mp, vw, rp, ci, s);
    case SBFA_BF16:
      return dispatch_fwd<__nv_bfloat16>(D, q, k, v, o, lse, BH, scale, mp, vw, rp, ci, s);
    case SBFA_F32: return dispatch_fwd<float>(D, q, k, v, o, lse, BH, scale, mp, vw, rp, ci, s);
    case SBFA_F64: return dispatch_fwd<double>(D, q, k, v, o, lse, BH, scale, mp, vw, rp, ci, s);
  }
  return fail(SBFA_ERR_INVALID, "unknown dtype");
}

int generic_bwd(int dtype, int D, const void* q, const void* k, const void* v, const void* o,
                const float* lse, const void* dout, void* dq, void* dk, void* dv, float* delta,
                int BH, double scale, const MaskParams& mp, const Views& vw, const int32_t* a,
                const int32_t* b, const int32_t* c, const int32_t* d, cudaStream_t s) {
  switch (dtype) {
    case SBFA_F16:
      return dispatch_bwd<__half>(D, q, k, v, o, lse, dout, dq, dk, dv, delta, BH, scale, mp, vw, a, b, c, d, s);
    case SBFA_BF16:
      return dispatch_bwd<__nv_bfloat16>(D, q, k, v, o, lse, dout, dq, dk, dv, delta, BH, scale, mp, vw, a, b, c, d, s);
    case SBFA_F32:
      return dispatch_bwd<float>(D, q, k, v, o, lse, dout, dq, dk, dv, delta, BH, scale, mp, vw, a, b, c, d, s);
    case SBFA_F64:
      return dispatch_bwd<double>(D, q, k, v, o, lse, dout, dq, dk, dv, delta, BH, scale, mp, vw, a, b, c, d, s);
  }
  return fail(SBFA_ERR_INVALID, "unknown dtype");
}

}  // namespace sbfa
