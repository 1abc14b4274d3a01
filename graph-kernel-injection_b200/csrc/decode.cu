// Split-KV decode for a single query per (batch, head).
//
// Upstream has no decode kernel: benchmark.py:799-804 clamps block_m to 1
// and runs the prefill _fwd_kernel (sparse_triton_kernel.py:231-352) with
// N_Q = 1, which scans all ceil(N_KV/BN) mask entries per (b, h).  Here:
//
//  * the kept key tiles of mask row 0 come from a compacted plan (pass 3,
//    64-key tiles), so only kept tiles are touched;
//  * inside a kept tile, a key is loaded only if the query can see it
//    (bounds, lifted block mask on partial tiles, StreamingLLM token rule),
//    so HBM traffic is exactly the visible K/V rows;
//  * each key row is read by a group of G lanes with 16-byte loads
//    (G = D * sizeof(T) / 16; 16 lanes for D = 128 fp16), fully coalesced,
//    U keys in flight per group;
//  * with grouped-query attention a CTA serves up to 4 query heads of one
//    key/value head, so each K/V row is read once for all of them;
//  * every CTA keeps an online-softmax partial (m, l, acc[D]) per lane group,
//    merges its groups through shared memory and either writes O / LSE
//    directly (one split) or a partial to the workspace, merged by
//    decode_merge_kernel (several splits).
#include <algorithm>
#include <mutex>

#include "sbfa_common.cuh"

namespace sbfa {

int decode_group(int dtype, int64_t D);
int decode_heads_per_cta(int group);
int check_decode_args(const void* q, const void* k, const void* v, const void* o, int64_t B,
                      int64_t H, int64_t n_kv, int64_t head_dim, int dtype, int64_t sink,
                      int64_t window, const int32_t* block_mask, int64_t block_m,
                      int64_t block_n, int64_t kv_heads);

namespace {

constexpr int kDecThreads = 128;
constexpr int kDecTile = 64;   // keys per plan tile (pass 3)

// Grouped-query decode tuning: query heads per CTA at most (1, 2 or 4), keys
// per lane group and iteration, and whether the next iteration's rows are
// loaded before the current one is computed.  Measured at config-4 geometry
// with 8 and 4 K/V heads (fp16, B=64): 4 heads, 2 keys, prefetch 2498 GB/s;
// 4 heads, 4 keys 2392; 4 heads, 4 keys, prefetch 2106; 2 heads, 4 keys
// 2231; one head per CTA (rows re-read per query head) 1753.
#ifndef SBFA_DECODE_MAX_QG
#define SBFA_DECODE_MAX_QG 4
#endif
#ifndef SBFA_DECODE_GQA_UNROLL
#define SBFA_DECODE_GQA_UNROLL 2
#endif
#ifndef SBFA_DECODE_GQA_PREFETCH
#define SBFA_DECODE_GQA_PREFETCH 1
#endif
constexpr int kMaxQG = SBFA_DECODE_MAX_QG;
constexpr int kGqaUnroll = SBFA_DECODE_GQA_UNROLL;
constexpr bool kGqaPrefetch = SBFA_DECODE_GQA_PREFETCH != 0;
static_assert(kMaxQG == 1 || kMaxQG == 2 || kMaxQG == 4, "heads per CTA: 1, 2 or 4");

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& w, float* f) {
  if constexpr (sizeof(T) == 2) {
    const T* h = reinterpret_cast<const T*>(&w);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to(h[i]);
  } else {
    const float* x = reinterpret_cast<const float*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = x[i];
  }
}

// Where the candidate keys of a decode query come from.  total() candidates
// t = 0 .. total()-1; key(t, &row) gives the cache row of candidate t and
// whether the query sees it.
//
// PlanKeys: the kept 64-key tiles of mask row 0 (a full-length cache).
struct PlanKeys {
  MaskParams mp;
  const int32_t* row_ptr;
  const int32_t* col_idx;
  int* status;  // debug builds record out-of-range plan indices here
  __device__ __forceinline__ PlanSpan span() const {
    const int n_tiles = ceil_div_dev(mp.n_kv, kDecTile);
    return plan_span(row_ptr, 0, n_tiles, n_tiles, status);
  }
  __device__ __forceinline__ int total() const { return span().n * kDecTile; }
  __device__ __forceinline__ bool key(int t, int* row) const {
    const int32_t ent =
        plan_entry(col_idx, span().e0 + t / kDecTile, ceil_div_dev(mp.n_kv, kDecTile), status);
    const int kk = plan_index(ent) * kDecTile + (t % kDecTile);
    *row = kk;
    return visible(mp, 0, kk, plan_partial(ent));
  }
};

// RingKeys: a StreamingLLM ring-buffer cache.  Rows [0, sink) hold positions
// [0, sink); rows [sink, sink + window) hold positions p >= sink at
// sink + (p - sink) % window.  The visible positions of the query at
// seq_len - 1 are the n_sink sinks followed by the n_win window positions,
// whose first one sits at ring offset slot0; all of them are visible.
struct RingKeys {
  int n_sink, n_win, slot0, sink, window;
  __device__ __forceinline__ int total() const { return n_sink + n_win; }
  __device__ __forceinline__ bool key(int t, int* row) const {
    if (t < n_sink) {
      *row = t;
    } else {
      int x = slot0 + (t - n_sink);
      if (x >= window) x -= window;
      *row = sink + x;
    }
    return true;
  }
};

// Partial record layout in the workspace: [m, l, acc[0..D)] floats, one per
// (query (batch, head), split).
//
// A CTA serves QG query heads that share one key/value head (grouped-query
// attention: query head h reads key/value head h / group; QG divides the
// group, QG = group = 1 without grouping), so every K/V row it loads is
// used by all QG queries.  Lane l of a G-lane group holds elements
// [l*EPV, (l+1)*EPV) of the row for every one of the QG queries; dot
// products and accumulators use packed fp32x2 FMAs.
template <typename T, int G, int QG, int U, bool PF, typename Keys>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    T* __restrict__ o, float* __restrict__ lse, float* __restrict__ ws, int D, float scale,
    Keys keys, int64_t kv_rows, int nsplit, int heads, int group) {
  constexpr int EPV = 16 / sizeof(T);      // elements per 16-byte vector
  constexpr int E2 = EPV / 2;              // fp32 pairs per vector
  constexpr int GPW = 32 / G;              // lane groups per warp
  constexpr int NG = (kDecThreads / 32) * GPW;
  __shared__ float sm_m[QG][NG], sm_l[QG][NG];
  extern __shared__ float sm_acc[];        // [QG][NG][D]

  const int split = blockIdx.x;
  const size_t bh0 = (size_t)blockIdx.y * QG;   // first query (batch, head) of the CTA
  const size_t kvh = (bh0 / heads) * (size_t)(heads / group) + (bh0 % heads) / group;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane / G, gl = lane % G;
  const int gid = warp * GPW + grp;

  // query slices of this lane, pre-scaled
  float2 qv[QG][E2];
#pragma unroll
  for (int j = 0; j < QG; ++j) {
    float f[EPV];
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(q + (bh0 + j) * (size_t)D) + gl);
    unpack16<T>(w, f);
#pragma unroll
    for (int i = 0; i < E2; ++i) qv[j][i] = make_float2(f[2 * i] * scale, f[2 * i + 1] * scale);
  }
  // this split's candidates: [t_lo, t_hi), in whole 64-key tiles
  const int all = keys.total();
  const int per = ((all + nsplit - 1) / nsplit + kDecTile - 1) / kDecTile * kDecTile;
  const int t_lo = split * per;
  const int total = max(0, min(all, t_lo + per) - t_lo);
  const uint4* kb = reinterpret_cast<const uint4*>(k + kvh * (size_t)kv_rows * D);
  const uint4* vb = reinterpret_cast<const uint4*>(v + kvh * (size_t)kv_rows * D);
  const int vec_per_row = D / EPV;   // == G

  float m[QG], l[QG];
  float2 acc[QG][E2];
#pragma unroll
  for (int j = 0; j < QG; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int i = 0; i < E2; ++i) acc[j][i] = make_float2(0.f, 0.f);
  }

  // U keys per lane group and iteration; with PF the next iteration's rows
  // are requested before this one's arithmetic, so loads stay in flight
  // while the CTA computes.
  const int step = NG * U;
  auto fetch = [&](int base, uint4 (&kw)[U], uint4 (&vw)[U], bool (&vis)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u * NG + gid;
      vis[u] = false;
      kw[u] = make_uint4(0u, 0u, 0u, 0u);
      vw[u] = kw[u];
      if (t < total) {
        int key = 0;
        vis[u] = keys.key(t_lo + t, &key);
        if (vis[u]) {
          kw[u] = __ldg(kb + (size_t)key * vec_per_row + gl);
          vw[u] = __ldg(vb + (size_t)key * vec_per_row + gl);
        }
      }
    }
  };
  uint4 kn[U], vn[U];
  bool visn[U];
  if (PF) fetch(0, kn, vn, visn);
  for (int base = 0; base < total; base += step) {
    uint4 kw[U], vw[U];
    bool vis[U];
    if (PF) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        kw[u] = kn[u];
        vw[u] = vn[u];
        vis[u] = visn[u];
      }
      if (base + step < total) fetch(base + step, kn, vn, visn);
    } else {
      fetch(base, kw, vw, vis);
    }
    float s[U][QG];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kf[EPV];
      unpack16<T>(kw[u], kf);
#pragma unroll
      for (int j = 0; j < QG; ++j) {
        float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < E2; ++i) d2 = __ffma2_rn(qv[j][i], make_float2(kf[2 * i], kf[2 * i + 1]), d2);
        float d = d2.x + d2.y;
#pragma unroll
        for (int off = G / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        s[u][j] = vis[u] ? d : -INFINITY;
      }
    }
    // No shuffles below this point in the iteration.  A query whose keys so
    // far are all invisible keeps m = -inf; the exponents then use 0 as
    // their reference so that no -inf - -inf appears (every p is 0).
    float mref[QG];
#pragma unroll
    for (int j = 0; j < QG; ++j) {
      float tmax = s[0][j];
#pragma unroll
      for (int u = 1; u < U; ++u) tmax = fmaxf(tmax, s[u][j]);
      const float m_new = fmaxf(m[j], tmax);
      mref[j] = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = __expf(m[j] - mref[j]);
      l[j] *= alpha;
#pragma unroll
      for (int i = 0; i < E2; ++i) acc[j][i] = __fmul2_rn(acc[j][i], make_float2(alpha, alpha));
      m[j] = m_new;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (!vis[u]) continue;
      float vf[EPV];
      unpack16<T>(vw[u], vf);
#pragma unroll
      for (int j = 0; j < QG; ++j) {
        const float p = __expf(s[u][j] - mref[j]);
        l[j] += p;
#pragma unroll
        for (int i = 0; i < E2; ++i)
          acc[j][i] = __ffma2_rn(make_float2(p, p), make_float2(vf[2 * i], vf[2 * i + 1]), acc[j][i]);
      }
    }
  }

  // merge the lane groups of the CTA, per query
#pragma unroll
  for (int j = 0; j < QG; ++j) {
    if (gl == 0) { sm_m[j][gid] = m[j]; sm_l[j][gid] = l[j]; }
#pragma unroll
    for (int i = 0; i < E2; ++i) {
      sm_acc[((size_t)j * NG + gid) * D + gl * EPV + 2 * i] = acc[j][i].x;
      sm_acc[((size_t)j * NG + gid) * D + gl * EPV + 2 * i + 1] = acc[j][i].y;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < QG * D; idx += blockDim.x) {
    const int j = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int g = 0; g < NG; ++g) M = fmaxf(M, sm_m[j][g]);
    float L = 0.f, a = 0.f;
    for (int g = 0; g < NG; ++g)
      if (sm_m[j][g] != -INFINITY) {
        const float w = __expf(sm_m[j][g] - M);
        L += sm_l[j][g] * w;
        a += sm_acc[((size_t)j * NG + g) * D + d] * w;
      }
    const size_t bh = bh0 + j;
    if (nsplit == 1) {
      const bool valid = L > 0.f;
      o[bh * D + d] = Elem<T>::from(valid ? a / L : 0.f);
      if (d == 0 && lse) lse[bh] = valid ? M + logf(L) : 0.f;
    } else {
      float* rec = ws + (bh * nsplit + split) * (size_t)(D + 2);
      rec[2 + d] = a;
      if (d == 0) { rec[0] = M; rec[1] = L; }
    }
  }
}

template <typename T>
__global__ void decode_merge_kernel(const float* __restrict__ ws, T* __restrict__ o,
                                    float* __restrict__ lse, int D, int nsplit) {
  const size_t bh = blockIdx.x;
  const float* recs = ws + bh * nsplit * (size_t)(D + 2);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, recs[s * (D + 2)]);
  float L = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = recs[s * (D + 2)];
    if (ms != -INFINITY) L += recs[s * (D + 2) + 1] * __expf(ms - M);
  }
  const bool valid = L > 0.f;
  const float inv = valid ? 1.f / L : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    if (valid)
      for (int s = 0; s < nsplit; ++s) {
        const float ms = recs[s * (D + 2)];
        if (ms != -INFINITY) a += recs[s * (D + 2) + 2 + d] * __expf(ms - M);
      }
    o[bh * D + d] = Elem<T>::from(a * inv);
  }
  if (threadIdx.x == 0 && lse) lse[bh] = valid ? M + logf(L) : 0.f;
}

template <typename T, int G, int QG, typename Keys>
int launch_decode(const void* q, const void* k, const void* v, void* o, float* lse, float* ws,
                  int BH, int D, float scale, const Keys& keys, int64_t kv_rows, int nsplit,
                  int heads, int group, cudaStream_t s) {
  constexpr int NG = (kDecThreads / 32) * (32 / G);
  constexpr int U = QG > 1 ? kGqaUnroll : 4;       // keys per lane group and iteration
  constexpr bool PF = QG > 1 ? kGqaPrefetch : false;
  const size_t sm = sizeof(float) * QG * NG * D;
  auto kern = decode_split_kernel<T, G, QG, U, PF, Keys>;
  if (sm > 48 * 1024) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)sm), "cudaFuncSetAttribute(decode)"))
      return rc;
  }
  dim3 grid(nsplit, BH / QG);
  {
    LaunchScope ls("decode_split_kernel", s);
    kern<<<grid, kDecThreads, sm, s>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, lse, ws,
                                       D, scale, keys, kv_rows, nsplit, heads, group);
  }
  if (int rc = check_launch("decode_split_kernel")) return rc;
  if (nsplit > 1) {
    {
      LaunchScope ls("decode_merge_kernel", s);
      decode_merge_kernel<T><<<BH, 128, 0, s>>>(ws, (T*)o, lse, D, nsplit);
    }
    return check_launch("decode_merge_kernel");
  }
  return SBFA_OK;
}

template <typename T, int G, typename Keys>
int launch_decode_qg(int qg, const void* q, const void* k, const void* v, void* o, float* lse,
                     float* ws, int BH, int D, float scale, const Keys& keys, int64_t kv_rows,
                     int nsplit, int heads, int group, cudaStream_t s) {
  switch (qg) {
    case 1: return launch_decode<T, G, 1>(q, k, v, o, lse, ws, BH, D, scale, keys, kv_rows, nsplit, heads, group, s);
    case 2: return launch_decode<T, G, 2>(q, k, v, o, lse, ws, BH, D, scale, keys, kv_rows, nsplit, heads, group, s);
    case 4: return launch_decode<T, G, 4>(q, k, v, o, lse, ws, BH, D, scale, keys, kv_rows, nsplit, heads, group, s);
  }
  return fail(SBFA_ERR_UNSUPPORTED, "decode: unsupported heads per CTA");
}

template <typename T, typename Keys>
int dispatch_decode(int G, int qg, const void* q, const void* k, const void* v, void* o,
                    float* lse, float* ws, int BH, int D, float scale, const Keys& keys,
                    int64_t kv_rows, int nsplit, int heads, int group, cudaStream_t s) {
#define SBFA_DEC(GG)                                                                          \
  case GG:                                                                                    \
    return launch_decode_qg<T, GG>(qg, q, k, v, o, lse, ws, BH, D, scale, keys, kv_rows,       \
                                   nsplit, heads, group, s);
  switch (G) {
    SBFA_DEC(1)
    SBFA_DEC(2)
    SBFA_DEC(4)
    SBFA_DEC(8)
    SBFA_DEC(16)
    SBFA_DEC(32)
  }
#undef SBFA_DEC
  return fail(SBFA_ERR_UNSUPPORTED, "decode: unsupported head_dim for the vector layout");
}

template <typename Keys>
int decode_any(int dtype, const void* q, const void* k, const void* v, void* o, float* lse,
               void* ws, int BH, int D, float scale, const Keys& keys, int64_t kv_rows,
               int nsplit, int heads, int group, cudaStream_t s) {
  const int G = decode_group(dtype, D);
  const int qg = decode_heads_per_cta(group);
  float* w = (float*)ws;
  switch (dtype) {
    case SBFA_F16:
      return dispatch_decode<__half>(G, qg, q, k, v, o, lse, w, BH, D, scale, keys, kv_rows,
                                     nsplit, heads, group, s);
    case SBFA_BF16:
      return dispatch_decode<__nv_bfloat16>(G, qg, q, k, v, o, lse, w, BH, D, scale, keys,
                                            kv_rows, nsplit, heads, group, s);
    case SBFA_F32:
      return dispatch_decode<float>(G, qg, q, k, v, o, lse, w, BH, D, scale, keys, kv_rows,
                                    nsplit, heads, group, s);
  }
  return fail(SBFA_ERR_UNSUPPORTED, "decode: unsupported dtype");
}

}  // namespace

int decode_tile() { return kDecTile; }

// Kept tiles the decode query can touch: every tile when the block mask is
// the only limit, else the tiles holding the sink and window keys (+2 for
// boundary tiles).
int64_t decode_est_tiles(int64_t n_kv, int is_causal, int64_t sink, int64_t window) {
  const int64_t t = kDecTile;
  const int64_t all = (n_kv + t - 1) / t;
  if (!is_causal) return all;
  const int64_t vis = std::min<int64_t>(n_kv, sink) + std::min<int64_t>(n_kv, window);
  return std::min<int64_t>(all, (vis + t - 1) / t + 2);
}

// Lanes per key row, or 0 when the head dim does not map onto 16-byte
// vectors (the caller then uses the generic forward).
int decode_group(int dtype, int64_t D) {
  int es = (dtype == SBFA_F32) ? 4 : (dtype == SBFA_F64 ? 8 : 2);
  if (dtype == SBFA_F64) return 0;
  int64_t bytes = D * es;
  if (bytes % 16 != 0) return 0;
  int64_t g = bytes / 16;
  if (g == 1 || g == 2 || g == 4 || g == 8 || g == 16 || g == 32) return (int)g;
  return 0;
}

int device_sm_count();

// Query heads one CTA serves for a grouped-query factor: the largest power
// of two up to 4 that divides the group (1 without grouping).  Four keeps
// the kernel at ~150 registers, three CTAs (12 warps, 48 KB of loads in
// flight) per SM; eight would need ~250 and leave two.  A group of 8 is
// served by two CTAs side by side, whose second read of each row is mostly
// an L2 hit.
int decode_heads_per_cta(int group) {
  for (int qg = kMaxQG; qg > 1; qg >>= 1)
    if (group % qg == 0) return qg;
  return 1;
}

// Number of splits per (b, h): enough CTAs for ~16 per SM of this device
// over `ctas` CTAs per split, never more than the tiles a row can hold.
int decode_nsplit(int64_t ctas, int64_t est_tiles) {
  const int64_t target = (int64_t)device_sm_count() * 16;
  int64_t ns = (target + ctas - 1) / std::max<int64_t>(1, ctas);
  ns = std::max<int64_t>(1, std::min<int64_t>(ns, std::max<int64_t>(1, est_tiles)));
  return (int)std::min<int64_t>(ns, 64);
}

int64_t decode_ws_bytes(int64_t BH, int64_t D, int nsplit) {
  return nsplit <= 1 ? 0 : BH * nsplit * (D + 2) * (int64_t)sizeof(float);
}

int decode_run(int dtype, const void* q, const void* k, const void* v, void* o, float* lse,
               void* ws, int BH, int D, float scale, const MaskParams& mp, const int32_t* rp,
               const int32_t* ci, int nsplit, int heads, int group, cudaStream_t s) {
  const PlanKeys keys{mp, rp, ci, device_status_ptr()};
  return decode_any(dtype, q, k, v, o, lse, ws, BH, D, scale, keys, (int64_t)mp.n_kv, nsplit,
                    heads, group, s);
}

}  // namespace sbfa

// ---------------------------------------------------------------------------
// Allocation-free decode
// ---------------------------------------------------------------------------
// Scratch for sbfa_decode_noalloc: the decode plan (row_ptr, col_idx, nnz)
// followed by the split-KV partials.  A file-scope device array, so every
// GPU that loads libsbfa holds these bytes until the process exits.
namespace sbfa {
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];
std::mutex g_scratch_mu;
unsigned char* g_scratch_addr[64] = {nullptr};

// Device address of g_decode_scratch on the current device, resolved once
// per device (the host-side symbol is only a stand-in and must never be
// handed to a kernel).
int scratch_base(unsigned char** out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(SBFA_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_decode_scratch),
                            "cudaGetSymbolAddress(decode scratch)"))
      return rc;
    g_scratch_addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_addr[dev];
  return SBFA_OK;
}
}  // namespace
}  // namespace sbfa

extern "C" int sbfa_decode_noalloc(const void* q, const void* k, const void* v, void* o,
                                   float* lse, int64_t B, int64_t H, int64_t n_kv,
                                   int64_t head_dim, int dtype, double softmax_scale,
                                   int is_causal, int64_t sink, int64_t window,
                                   const int32_t* block_mask, int64_t block_m, int64_t block_n,
                                   void* stream) {
  using namespace sbfa;
  // the same checks as sbfa_decode, all before anything touches the shared
  // scratch or launches a kernel
  if (int rc = check_decode_args(q, k, v, o, B, H, n_kv, head_dim, dtype, sink, window,
                                 block_mask, block_m, block_n, H))
    return rc;
  const int64_t n_tiles = (n_kv + kDecTile - 1) / kDecTile;
  // plan: row_ptr[2], col_idx[n_tiles], nnz[1]; partials start on a 256-byte boundary
  const int64_t plan_bytes = ((2 + n_tiles + 1) * (int64_t)sizeof(int32_t) + 255) / 256 * 256;
  const int ns = decode_nsplit(B * H, decode_est_tiles(n_kv, is_causal, sink, window));
  const int64_t ws_bytes = decode_ws_bytes(B * H, head_dim, ns);
  if (plan_bytes + ws_bytes > (int64_t)kNoAllocScratchBytes)
    return fail(SBFA_ERR_INVALID,
                "sbfa_decode_noalloc: this shape needs " + std::to_string(plan_bytes + ws_bytes) +
                    " bytes of scratch, more than the static " +
                    std::to_string(kNoAllocScratchBytes) +
                    "-byte buffer; use sbfa_decode with a caller-provided workspace");
  unsigned char* base = nullptr;
  if (int rc = scratch_base(&base)) return rc;
  int32_t* row_ptr = reinterpret_cast<int32_t*>(base);
  int32_t* col_idx = row_ptr + 2;
  int32_t* nnz = col_idx + n_tiles;
  // every scratch byte read below is written first in stream order: the plan
  // kernels write row_ptr (scan sets row_ptr[0] = 0) and the kept col_idx
  // entries; each split writes its whole partial record before the merge
  if (int rc = sbfa_build_plan(block_mask, 1, n_kv, block_m, block_n, 1, kDecTile, row_ptr,
                               col_idx, nullptr, nullptr, nnz, stream))
    return rc;
  return sbfa_decode(q, k, v, o, lse, B, H, n_kv, head_dim, dtype, softmax_scale, is_causal, sink,
                     window, block_mask, block_m, block_n, row_ptr, col_idx,
                     ws_bytes > 0 ? base + plan_bytes : nullptr, ws_bytes, H, stream);
}

// ---------------------------------------------------------------------------
// StreamingLLM ring-buffer KV cache
// ---------------------------------------------------------------------------
namespace sbfa {
namespace {

// Copies the new tokens' K and V rows into their ring rows, skipping the
// positions a later token of the same call overwrites (so no two threads
// write one row).  One 16-byte vector per thread and step.
template <typename T>
__global__ void ring_append_kernel(T* __restrict__ kc, T* __restrict__ vc,
                                   const T* __restrict__ kn, const T* __restrict__ vn, int D,
                                   int64_t rows, int64_t n_new, int64_t pos0, int64_t sink,
                                   int64_t window) {
  constexpr int kVec = 16 / sizeof(T);
  const int vpr = D / kVec;
  const int64_t bh = blockIdx.y;
  const int64_t end = pos0 + n_new;
  const int64_t n = n_new * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vpr;
    const int c = (int)(i % vpr);
    const int64_t p = pos0 + t;
    if (p >= sink && p < end - window) continue;  // overwritten within this call
    const int64_t row = p < sink ? p : sink + (p - sink) % window;
    const int64_t src = (bh * n_new + t) * D;
    const int64_t dst = (bh * rows + row) * D;
    reinterpret_cast<uint4*>(kc + dst)[c] = reinterpret_cast<const uint4*>(kn + src)[c];
    reinterpret_cast<uint4*>(vc + dst)[c] = reinterpret_cast<const uint4*>(vn + src)[c];
  }
}

RingKeys ring_keys(int64_t sink, int64_t window, int64_t seq_len) {
  const int64_t n_sink = std::min(sink, seq_len);
  const int64_t lo = std::max(sink, seq_len - window);
  const int64_t n_win = std::max<int64_t>(0, seq_len - lo);
  const int64_t slot0 = window > 0 ? (lo - sink) % window : 0;
  return RingKeys{(int)n_sink, (int)n_win, (int)slot0, (int)sink, (int)window};
}

int check_ring(int64_t B, int64_t H, int64_t D, int dtype, int64_t sink, int64_t window) {
  if (B <= 0 || H <= 0 || D <= 0)
    return fail(SBFA_ERR_INVALID, "B, H and head_dim must be positive");
  if (B * H > 65535) return fail(SBFA_ERR_UNSUPPORTED, "B * H must be <= 65535");
  if (sink < 0 || window < 0)
    return fail(SBFA_ERR_INVALID, "sink_size and window_size must be non-negative");
  if (sink + window <= 0 || sink + window >= (1ll << 30))
    return fail(SBFA_ERR_INVALID, "sink_size + window_size must be in [1, 2^30)");
  if (decode_group(dtype, D) == 0)
    return fail(SBFA_ERR_UNSUPPORTED,
                "ring cache: dtype must be float16/bfloat16/float32 with head_dim * element "
                "size a multiple of 16 bytes (at most 512 bytes)");
  return SBFA_OK;
}

}  // namespace
}  // namespace sbfa

extern "C" int sbfa_ring_append(void* k_cache, void* v_cache, const void* k_new,
                                const void* v_new, int64_t B, int64_t H, int64_t head_dim,
                                int dtype, int64_t sink, int64_t window, int64_t pos0,
                                int64_t n_new, void* stream) {
  using namespace sbfa;
  if (int rc = check_ring(B, H, head_dim, dtype, sink, window)) return rc;
  if (!k_cache || !v_cache || !k_new || !v_new)
    return fail(SBFA_ERR_INVALID, "sbfa_ring_append: NULL tensor pointer");
  if (pos0 < 0 || n_new < 0) return fail(SBFA_ERR_INVALID, "pos0 and n_new must be >= 0");
  if (n_new == 0) return SBFA_OK;
  for (const void* p : {(const void*)k_cache, (const void*)v_cache, k_new, v_new})
    if ((uintptr_t)p % 16) return fail(SBFA_ERR_INVALID, "ring cache tensors must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t rows = sink + window;
  const int es = dtype == SBFA_F32 ? 4 : 2;
  const int64_t vecs = n_new * (head_dim * es / 16);
  dim3 grid((unsigned)std::min<int64_t>((vecs + 255) / 256, 1024), (unsigned)(B * H));
  LaunchScope ls("ring_append_kernel", s);
  switch (dtype) {
    case SBFA_F16:
      ring_append_kernel<__half><<<grid, 256, 0, s>>>((__half*)k_cache, (__half*)v_cache,
                                                      (const __half*)k_new, (const __half*)v_new,
                                                      (int)head_dim, rows, n_new, pos0, sink,
                                                      window);
      break;
    case SBFA_BF16:
      ring_append_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, (const __nv_bfloat16*)k_new,
          (const __nv_bfloat16*)v_new, (int)head_dim, rows, n_new, pos0, sink, window);
      break;
    case SBFA_F32:
      ring_append_kernel<float><<<grid, 256, 0, s>>>((float*)k_cache, (float*)v_cache,
                                                     (const float*)k_new, (const float*)v_new,
                                                     (int)head_dim, rows, n_new, pos0, sink,
                                                     window);
      break;
    default: return fail(SBFA_ERR_UNSUPPORTED, "ring cache: unsupported dtype");
  }
  return check_launch("ring_append_kernel");
}

extern "C" int64_t sbfa_ring_decode_workspace_bytes(int64_t B, int64_t H, int64_t head_dim,
                                                    int64_t sink, int64_t window) {
  using namespace sbfa;
  if (B <= 0 || H <= 0 || head_dim <= 0 || sink < 0 || window < 0) return 0;
  const int ns = decode_nsplit(B * H, (sink + window + kDecTile - 1) / kDecTile);
  return decode_ws_bytes(B * H, head_dim, ns);
}

extern "C" int sbfa_ring_decode(const void* q, const void* k_cache, const void* v_cache, void* o,
                                float* lse, int64_t B, int64_t H, int64_t head_dim, int dtype,
                                double softmax_scale, int64_t sink, int64_t window,
                                int64_t seq_len, void* split_ws, int64_t split_ws_bytes,
                                void* stream) {
  using namespace sbfa;
  if (int rc = check_ring(B, H, head_dim, dtype, sink, window)) return rc;
  if (!q || !k_cache || !v_cache || !o)
    return fail(SBFA_ERR_INVALID, "sbfa_ring_decode: NULL tensor pointer");
  if (seq_len <= 0 || seq_len >= (1ll << 31))
    return fail(SBFA_ERR_INVALID, "seq_len must be in [1, 2^31)");
  for (const void* p : {q, k_cache, v_cache, (const void*)o})
    if ((uintptr_t)p % 16) return fail(SBFA_ERR_INVALID, "ring cache tensors must be 16-byte aligned");
  const RingKeys keys = ring_keys(sink, window, seq_len);
  const int64_t BH = B * H;
  const int ns = decode_nsplit(BH, (keys.n_sink + keys.n_win + kDecTile - 1) / kDecTile);
  const int64_t need = decode_ws_bytes(BH, head_dim, ns);
  if (need > 0 && (split_ws == nullptr || split_ws_bytes < need))
    return fail(SBFA_ERR_INVALID, "sbfa_ring_decode: split workspace too small (need " +
                                      std::to_string(need) + " bytes)");
  return decode_any(dtype, q, k_cache, v_cache, o, lse, split_ws, (int)BH, (int)head_dim,
                    (float)softmax_scale, keys, sink + window, ns, (int)H, 1,
                    (cudaStream_t)stream);
}
