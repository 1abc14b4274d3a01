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
//  * every CTA keeps an online-softmax partial (m, l, acc[D]) per lane group,
//    merges its groups through shared memory and either writes O / LSE
//    directly (one split) or a partial to the workspace, merged by
//    decode_merge_kernel (several splits);
//  * with grouped-query attention a CTA serves several query heads of one
//    key/value head, so each K/V row is read once for all of them: up to 16
//    on the tensor cores (decode_gqa_kernel, fp16/bf16 with D = 64 or 128),
//    up to 4 on the CUDA cores otherwise.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "sbfa_common.cuh"

namespace sbfa {

int decode_group(int dtype, int64_t D);
int decode_heads_per_cta(int group);
bool decode_uses_mma(int dtype, int64_t D, int group);
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
  // The same per tile: first() once, then tile(first, i) for candidate
  // tile i (a plan entry, loaded ahead of its use) and tile_key(entry, j)
  // for its key j.
  __device__ __forceinline__ int first() const { return span().e0; }
  __device__ __forceinline__ int32_t tile(int e0, int i) const {
    return plan_entry(col_idx, e0 + i, ceil_div_dev(mp.n_kv, kDecTile), status);
  }
  __device__ __forceinline__ bool tile_key(int32_t ent, int j, int* row) const {
    const int kk = plan_index(ent) * kDecTile + j;
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
  __device__ __forceinline__ int first() const { return 0; }
  __device__ __forceinline__ int32_t tile(int, int i) const { return i; }
  __device__ __forceinline__ bool tile_key(int32_t i, int j, int* row) const {
    return key(i * kDecTile + j, row);
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

// ---------------------------------------------------------------------------
// Grouped-query decode on the tensor cores (fp16/bf16, D = 64 or 128).
//
// A CTA serves up to 16 query heads of one key/value head (one M = 16 MMA
// tile; rows past the group's heads are zero) over one split of the kept
// keys.  Each of its four warps owns 16 keys of every 64-key stage and runs
// its own pipeline of kGqaStages shared-memory buffers:
//  * the warp's lanes copy its 16 K rows and 16 V rows with 16-byte
//    `cp.async` (a half-warp per 256-byte row), into rows whose 16-byte
//    chunks are XOR-swizzled by (row % 8) so that the `ldmatrix` reads below
//    are free of bank conflicts; a key the query cannot see is zero-filled
//    without reading global memory, so HBM traffic is the visible rows;
//  * S = Q K^T: 2 key tiles x D/16 steps of `mma.sync.m16n8k16` (fp32
//    accumulators), K fragments by `ldmatrix`;
//  * online softmax per head in base 2 on the accumulator fragments (a quad
//    of lanes holds a head's 16 scores), P rounded to the input type, as
//    the prefill kernels do before P V;
//  * O += P V: D/8 MMAs, V fragments by `ldmatrix.trans`.
// The warps' partial (m, l, O) are merged through shared memory; one split
// writes O and LSE, several write partial records for decode_merge_kernel.
// The decode is HBM-bound: the tensor cores only replace the per-key
// CUDA-core dot products and lane-group reductions that made the grouped
// kernel above issue-bound, and the staging keeps 2 x 4 x (stages - 1) x
// 8 KB of loads in flight per SM (two CTAs) without holding them in
// registers.  tcgen05 would need M >= 64 (16 heads at most here) and a TMEM
// round trip per stage.
constexpr int kGqaWarps = 4;
constexpr int kGqaThreads = kGqaWarps * 32;
constexpr int kGqaKeys = 16;                   // keys per warp and stage
constexpr int kGqaStageKeys = kGqaWarps * kGqaKeys;
static_assert(kGqaStageKeys == kDecTile, "a stage is one plan tile");
#ifndef SBFA_DECODE_GQA_STAGES
#define SBFA_DECODE_GQA_STAGES 3
#endif
constexpr int kGqaStages = SBFA_DECODE_GQA_STAGES;
constexpr int kGqaRows = 16;                   // query heads per MMA tile
constexpr int kGqaMaxCtasPerSm = 4;            // bound used by the workspace size

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
// C[16x8] += A[16x16] (row) * B[16x8] (col), fp32 accumulators
template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
// two floats as a packed pair of T (x in the low half)
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Shared memory of decode_gqa_kernel: the stage buffers, later reused for
// the merge of the warps' partials.
template <int D>
constexpr size_t gqa_smem_bytes() {
  constexpr size_t stages = (size_t)kGqaWarps * kGqaStages * 2 * kGqaKeys * D * 2;
  constexpr size_t merge = (size_t)kGqaWarps * kGqaRows * (D + 2) * sizeof(float);
  return stages > merge ? stages : merge;
}

template <typename T, int D, typename Keys>
__global__ void __launch_bounds__(kGqaThreads, 2) decode_gqa_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    T* __restrict__ o, float* __restrict__ lse, float* __restrict__ ws, float scale_log2,
    Keys keys, int64_t kv_rows, int nsplit, int group, int qh, int chunks) {
  constexpr int CPR = D * 2 / 16;          // 16-byte chunks per row
  constexpr int RB = D * 2;                // bytes per row
  constexpr int KSTEPS = D / 16;
  constexpr int NT = D / 8;                // output column tiles
  constexpr uint32_t kFull = 0xffffffffu;
  extern __shared__ __align__(128) unsigned char gqa_smem[];
  __shared__ uint32_t vis_s[kGqaWarps][kGqaStages];

  const int split = blockIdx.x;
  const int kvu = blockIdx.y / chunks;             // (batch, key/value head)
  const int h0 = (blockIdx.y % chunks) * qh;       // first head of the group served here
  const int nrows = min(qh, group - h0);
  const size_t bh0 = (size_t)kvu * group + h0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;

  // Q fragments (rows g and g + 8 of the 16-row tile), zero past nrows
  uint32_t qa[KSTEPS][4];
  {
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(q + (bh0 + g) * D);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(q + (bh0 + g + 8) * D);
    const bool r0 = g < nrows, r1 = g + 8 < nrows;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const int c0 = kk * 8 + t4, c1 = kk * 8 + 4 + t4;   // pair indices
      qa[kk][0] = r0 ? __ldg(q0 + c0) : 0u;
      qa[kk][1] = r1 ? __ldg(q1 + c0) : 0u;
      qa[kk][2] = r0 ? __ldg(q0 + c1) : 0u;
      qa[kk][3] = r1 ? __ldg(q1 + c1) : 0u;
    }
  }

  const int all = keys.total();
  const int per = ((all + nsplit - 1) / nsplit + kDecTile - 1) / kDecTile * kDecTile;
  const int t_lo = split * per;
  const int total = max(0, min(all, t_lo + per) - t_lo);
  const int nstage = (total + kGqaStageKeys - 1) / kGqaStageKeys;
  const T* kb = k + (size_t)kvu * kv_rows * D;
  const T* vb = v + (size_t)kvu * kv_rows * D;
  const uint32_t ks0 =
      smem_u32(gqa_smem) + (uint32_t)(warp * kGqaStages * 2 * kGqaKeys * RB);

  // Stage s is candidate tile t_lo / 64 + s; its plan entry is loaded one
  // iteration before the stage is issued, so that the issue does not wait
  // on it.
  const int e0 = keys.first();
  const int tile0 = t_lo / kDecTile;
  auto entry = [&](int s) { return s < nstage ? keys.tile(e0, tile0 + s) : 0; };
  // copies this warp's 16 keys of stage s (plan entry ent) into buffer `slot`
  auto issue = [&](int s, int32_t ent, int slot) {
    int rowinfo = -1;                              // cache row, or -1 if not visible
    if (s < nstage) {
      const int j = warp * kGqaKeys + (lane & (kGqaKeys - 1));
      int row = 0;
      if (s * kGqaStageKeys + j < total && keys.tile_key(ent, j, &row)) rowinfo = row;
    }
    const uint32_t vis = __ballot_sync(kFull, lane < kGqaKeys && rowinfo >= 0);
    if (lane == 0) vis_s[warp][slot] = vis;
    if (vis != 0) {
      const uint32_t kd = ks0 + (uint32_t)(slot * 2 * kGqaKeys * RB);
      const uint32_t vd = kd + (uint32_t)(kGqaKeys * RB);
#pragma unroll
      for (int j = 0; j < CPR / 2; ++j) {
        const int flat = j * 32 + lane;
        const int r = flat / CPR, c = flat % CPR;
        const int ri = __shfl_sync(kFull, rowinfo, r);
        const size_t off = (size_t)(ri >= 0 ? ri : 0) * D + c * 8;
        const uint32_t so = (uint32_t)(r * RB + ((c ^ (r & 7)) << 4));
        const int nb = ri >= 0 ? 16 : 0;
        cp_async16(kd + so, kb + off, nb);
        cp_async16(vd + so, vb + off, nb);
      }
    }
    cp_async_commit();
  };

  float oacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // rows g, g + 8

#pragma unroll
  for (int s = 0; s < kGqaStages - 1; ++s) issue(s, entry(s), s);
  int32_t ent_next = entry(kGqaStages - 1);
  for (int s = 0; s < nstage; ++s) {
    cp_async_wait<kGqaStages - 2>();
    __syncwarp();
    issue(s + kGqaStages - 1, ent_next, (s + kGqaStages - 1) % kGqaStages);
    ent_next = entry(s + kGqaStages);
    const int slot = s % kGqaStages;
    const uint32_t vis = vis_s[warp][slot];
    if (vis == 0) continue;
    const uint32_t kd = ks0 + (uint32_t)(slot * 2 * kGqaKeys * RB);
    const uint32_t vd = kd + (uint32_t)(kGqaKeys * RB);

    // S = Q K^T for the warp's 16 keys (two 8-key column tiles)
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      const int r = nt * 8 + (lane & 7);
#pragma unroll
      for (int kp = 0; kp < KSTEPS / 2; ++kp) {
        const int c = kp * 4 + (lane >> 3);
        uint32_t b[4];
        ldsm_x4(kd + (uint32_t)(r * RB + ((c ^ (r & 7)) << 4)), b);
        mma16816<T>(sc[nt], qa[2 * kp], b[0], b[1]);
        mma16816<T>(sc[nt], qa[2 * kp + 1], b[2], b[3]);
      }
    }
    // online softmax in base 2; invisible keys are -inf
    float x[2][4];
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = nt * 8 + 2 * t4 + (e & 1);
        x[nt][e] = ((vis >> key) & 1u) ? sc[nt][e] * scale_log2 : -INFINITY;
        if (e < 2) mx0 = fmaxf(mx0, x[nt][e]); else mx1 = fmaxf(mx1, x[nt][e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    // a head with nothing visible so far keeps m = -inf; 0 is then the
    // exponent reference, so no -inf - -inf appears (every p is 0)
    const float r0 = n0 == -INFINITY ? 0.f : n0, r1 = n1 == -INFINITY ? 0.f : n1;
    const float a0 = exp2f(m0 - r0), a1 = exp2f(m1 - r1);
    m0 = n0;
    m1 = n1;
    float p[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      p[nt][0] = exp2f(x[nt][0] - r0);
      p[nt][1] = exp2f(x[nt][1] - r0);
      p[nt][2] = exp2f(x[nt][2] - r1);
      p[nt][3] = exp2f(x[nt][3] - r1);
    }
    l0 = l0 * a0 + (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
    l1 = l1 * a1 + (p[0][2] + p[0][3]) + (p[1][2] + p[1][3]);
    uint32_t pa[4];
    pa[0] = pack2<T>(p[0][0], p[0][1]);
    pa[1] = pack2<T>(p[0][2], p[0][3]);
    pa[2] = pack2<T>(p[1][0], p[1][1]);
    pa[3] = pack2<T>(p[1][2], p[1][3]);
    // O = alpha O + P V
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      oacc[j][0] *= a0;
      oacc[j][1] *= a0;
      oacc[j][2] *= a1;
      oacc[j][3] *= a1;
    }
    {
      const int mi = lane >> 3;
      const int r = (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        const int c = j + (mi >> 1);
        uint32_t b[4];
        ldsm_x4_t(vd + (uint32_t)(r * RB + ((c ^ (r & 7)) << 4)), b);
        mma16816<T>(oacc[j], pa, b[0], b[1]);
        mma16816<T>(oacc[j + 1], pa, b[2], b[3]);
      }
    }
  }
  cp_async_wait<0>();
  // row sums over the quad
  l0 += __shfl_xor_sync(kFull, l0, 1);
  l0 += __shfl_xor_sync(kFull, l0, 2);
  l1 += __shfl_xor_sync(kFull, l1, 1);
  l1 += __shfl_xor_sync(kFull, l1, 2);
  __syncthreads();   // every warp is done with its stage buffers

  // merge the warps: [warp][row] m, l, then [warp][row][D] O
  float* sm_m = reinterpret_cast<float*>(gqa_smem);
  float* sm_l = sm_m + kGqaWarps * kGqaRows;
  float* sm_o = sm_l + kGqaWarps * kGqaRows;
  if (t4 == 0) {
    sm_m[warp * kGqaRows + g] = m0;
    sm_m[warp * kGqaRows + g + 8] = m1;
    sm_l[warp * kGqaRows + g] = l0;
    sm_l[warp * kGqaRows + g + 8] = l1;
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    float* o0 = sm_o + ((size_t)warp * kGqaRows + g) * D + j * 8 + 2 * t4;
    *reinterpret_cast<float2*>(o0) = make_float2(oacc[j][0], oacc[j][1]);
    *reinterpret_cast<float2*>(o0 + 8 * D) = make_float2(oacc[j][2], oacc[j][3]);
  }
  __syncthreads();
  constexpr float kLn2 = 0.6931471805599453f;
  for (int idx = threadIdx.x; idx < nrows * D; idx += kGqaThreads) {
    const int row = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kGqaWarps; ++w) M = fmaxf(M, sm_m[w * kGqaRows + row]);
    float L = 0.f, a = 0.f;
#pragma unroll
    for (int w = 0; w < kGqaWarps; ++w) {
      const float mw = sm_m[w * kGqaRows + row];
      if (mw != -INFINITY) {
        const float wt = exp2f(mw - M);
        L += sm_l[w * kGqaRows + row] * wt;
        a += sm_o[((size_t)w * kGqaRows + row) * D + d] * wt;
      }
    }
    const size_t bh = bh0 + row;
    if (nsplit == 1) {
      const bool valid = L > 0.f;
      o[bh * D + d] = Elem<T>::from(valid ? a / L : 0.f);
      if (d == 0 && lse) lse[bh] = valid ? (M + log2f(L)) * kLn2 : 0.f;
    } else {
      // partial record in the natural-log domain of decode_merge_kernel
      float* rec = ws + (bh * nsplit + split) * (size_t)(D + 2);
      rec[2 + d] = a;
      if (d == 0) { rec[0] = M * kLn2; rec[1] = L; }
    }
  }
}

// Query heads per tensor-core decode CTA for a grouped-query factor: the
// group split into ceil(group / 16) near-equal chunks.
int gqa_rows(int group) {
  const int chunks = (group + kGqaRows - 1) / kGqaRows;
  return (group + chunks - 1) / chunks;
}

template <typename T, int D, typename Keys>
int launch_decode_gqa(const void* q, const void* k, const void* v, void* o, float* lse,
                      float* ws, int BH, float scale, const Keys& keys, int64_t kv_rows,
                      int nsplit, int group, cudaStream_t s) {
  const int qh = gqa_rows(group);
  const int chunks = (group + qh - 1) / qh;
  const size_t sm = gqa_smem_bytes<D>();
  auto kern = decode_gqa_kernel<T, D, Keys>;
  if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)sm), "cudaFuncSetAttribute(decode_gqa)"))
    return rc;
  dim3 grid(nsplit, (BH / group) * chunks);
  constexpr float kLog2e = 1.4426950408889634f;
  {
    LaunchScope ls("decode_gqa_kernel", s);
    kern<<<grid, kGqaThreads, sm, s>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, lse, ws,
                                       scale * kLog2e, keys, kv_rows, nsplit, group, qh, chunks);
  }
  if (int rc = check_launch("decode_gqa_kernel")) return rc;
  if (nsplit > 1) {
    {
      LaunchScope ls("decode_merge_kernel", s);
      decode_merge_kernel<T><<<BH, 128, 0, s>>>(ws, (T*)o, lse, D, nsplit);
    }
    return check_launch("decode_merge_kernel");
  }
  return SBFA_OK;
}

// Resident decode_gqa_kernel CTAs per SM for head dim D on the current
// device (occupancy query, cached per device; 2 when no device answers).
int gqa_ctas_per_sm(int D) {
  static std::mutex mu;
  static int cached[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 2;
  const int w = D == 64 ? 0 : 1;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev][w] == 0) {
    int n = 0;
    cudaError_t e;
    if (w == 0) {
      auto kern = decode_gqa_kernel<__half, 64, PlanKeys>;
      const size_t sm = gqa_smem_bytes<64>();
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kGqaThreads, sm);
    } else {
      auto kern = decode_gqa_kernel<__half, 128, PlanKeys>;
      const size_t sm = gqa_smem_bytes<128>();
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kGqaThreads, sm);
    }
    if (e != cudaSuccess) (void)cudaGetLastError();
    cached[dev][w] = (e == cudaSuccess && n > 0) ? std::min(n, kGqaMaxCtasPerSm) : 2;
  }
  return cached[dev][w];
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
  if (decode_uses_mma(dtype, D, group)) {
#define SBFA_GQA(TT, DD)                                                                     \
  return launch_decode_gqa<TT, DD>(q, k, v, o, lse, w, BH, scale, keys, kv_rows, nsplit, group, s);
    if (dtype == SBFA_F16) {
      if (D == 64) SBFA_GQA(__half, 64)
      SBFA_GQA(__half, 128)
    }
    if (D == 64) SBFA_GQA(__nv_bfloat16, 64)
    SBFA_GQA(__nv_bfloat16, 128)
#undef SBFA_GQA
  }
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

// Whether a decode call runs decode_gqa_kernel (the tensor-core grouped-query
// kernel): fp16/bf16, head dim 64 or 128, at least two query heads per K/V head.
#ifndef SBFA_DECODE_GQA_MMA
#define SBFA_DECODE_GQA_MMA 1
#endif
bool decode_uses_mma(int dtype, int64_t D, int group) {
  return SBFA_DECODE_GQA_MMA && (dtype == SBFA_F16 || dtype == SBFA_BF16) &&
         (D == 64 || D == 128) && group >= 2;
}

constexpr int kDecCtasPerSm = 16;

// Number of splits per (b, h): enough CTAs for ~per_sm per SM of this device
// over `ctas` CTAs per split, never more than the tiles a row can hold.
int decode_nsplit(int64_t ctas, int64_t est_tiles, int per_sm) {
  const int64_t target = (int64_t)device_sm_count() * per_sm;
  int64_t ns = (target + ctas - 1) / std::max<int64_t>(1, ctas);
  ns = std::max<int64_t>(1, std::min<int64_t>(ns, std::max<int64_t>(1, est_tiles)));
  return (int)std::min<int64_t>(ns, 64);
}

// Splits of the tensor-core grouped decode: its CTAs stream long runs of
// tiles, so splitting only pays where it fills the GPU.  The split count
// minimises a wave model: ceil(CTAs / resident slots) waves, each as long
// as a CTA's tiles plus about one tile of set-up (Q, plan entries, the
// first loads, the merge of the warps), plus ~4 tiles for the merge launch
// when there are several splits.  At config 4 with 8 K/V heads (512 CTAs,
// 33 tiles, 296 slots) it picks 1 split; measured kernel fractions of HBM
// were 0.91 / 0.85 / 0.84 / 0.80 / 0.69 for 1 / 2 / 3 / 5 / 10 splits.
constexpr int kGqaSetupTiles = 1;
constexpr int kGqaMergeTiles = 4;
int gqa_splits(int64_t ctas, int64_t est_tiles, int64_t slots) {
  const int64_t T = std::max<int64_t>(1, est_tiles);
  const int64_t cap = std::min<int64_t>(
      {T, 64, std::max<int64_t>(1, (2 * slots + ctas - 1) / std::max<int64_t>(1, ctas))});
  int best = 1;
  int64_t best_cost = INT64_MAX;
  for (int64_t ns = 1; ns <= cap; ++ns) {
    const int64_t waves = (ctas * ns + slots - 1) / slots;
    const int64_t cost =
        waves * ((T + ns - 1) / ns + kGqaSetupTiles) + (ns > 1 ? kGqaMergeTiles : 0);
    if (cost < best_cost) { best_cost = cost; best = (int)ns; }
  }
  return best;
}

// Splits of a decode call over BH query (batch, head) pairs with `group`
// query heads per K/V head.
int decode_splits(int64_t BH, int group, int dtype, int64_t D, int64_t est_tiles) {
  if (decode_uses_mma(dtype, D, group)) {
    const int qh = gqa_rows(group);
    const int64_t ctas = std::max<int64_t>(1, BH / group * ((group + qh - 1) / qh));
    return gqa_splits(ctas, est_tiles, (int64_t)device_sm_count() * gqa_ctas_per_sm((int)D));
  }
  return decode_nsplit(std::max<int64_t>(1, BH / decode_heads_per_cta(group)), est_tiles,
                       kDecCtasPerSm);
}

// The most splits any grouping of BH query pairs can give, which sizes the
// worst-case workspace: the CUDA-core kernel's rule at its fewest CTAs (4
// query heads per CTA), or the grouped kernel's cap at its fewest (16 query
// heads per CTA, the most resident CTAs per SM it can reach).
int decode_max_splits(int64_t BH, int64_t est_tiles) {
  const int a = decode_nsplit(std::max<int64_t>(1, BH / kMaxQG), est_tiles, kDecCtasPerSm);
  const int64_t ctas = std::max<int64_t>(1, BH / kGqaRows);
  const int64_t slots = (int64_t)device_sm_count() * kGqaMaxCtasPerSm;
  const int64_t b = std::min<int64_t>(
      {std::max<int64_t>(1, est_tiles), 64, std::max<int64_t>(1, (2 * slots + ctas - 1) / ctas)});
  return std::max<int>(a, (int)b);
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
  const int ns = decode_splits(B * H, 1, dtype, head_dim,
                               decode_est_tiles(n_kv, is_causal, sink, window));
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
  const int ns =
      decode_splits(B * H, 1, SBFA_F32, head_dim, (sink + window + kDecTile - 1) / kDecTile);
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
  const int ns = decode_splits(BH, 1, dtype, head_dim,
                               (keys.n_sink + keys.n_win + kDecTile - 1) / kDecTile);
  const int64_t need = decode_ws_bytes(BH, head_dim, ns);
  if (need > 0 && (split_ws == nullptr || split_ws_bytes < need))
    return fail(SBFA_ERR_INVALID, "sbfa_ring_decode: split workspace too small (need " +
                                      std::to_string(need) + " bytes)");
  return decode_any(dtype, q, k_cache, v_cache, o, lse, split_ws, (int)BH, (int)head_dim,
                    (float)softmax_scale, keys, sink + window, ns, (int)H, 1,
                    (cudaStream_t)stream);
}
