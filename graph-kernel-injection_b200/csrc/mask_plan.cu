// Mask construction and kept-tile compaction on the GPU.
//
//  * sbfa_streaming_mask / sbfa_dense_mask: the int32 block masks of
//    make_streaming_mask / make_dense_mask (sparse_triton_kernel.py:104-210),
//    one thread per entry, bit-exact (pure integer arithmetic in int64).
//  * sbfa_build_plan: CSR + CSC lists of kept (query tile, key tile) pairs
//    for a block mask re-tiled to the kernel's tile sizes.  The upstream
//    kernels scan every mask entry per tile (sparse_triton_kernel.py:283-285,
//    448-449, 563-565); the lists let the attention kernels visit only kept
//    tiles.  Three launches: per-line counts, an exclusive scan, and an
//    order-preserving compaction (one CTA per tile row / tile column).
#include <algorithm>

#include "sbfa_common.cuh"

namespace sbfa {
namespace {

__global__ void streaming_mask_kernel(int64_t n_qb, int64_t n_kb, int64_t q_off,
                                      int64_t sink, int64_t window, int64_t bm,
                                      int64_t bn, int32_t* out) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = n_qb * n_kb;
  for (; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t i = idx / n_kb, j = idx - i * n_kb;
    int64_t q_lo = i * bm + q_off, q_hi = q_lo + bm;
    int64_t k_lo = j * bn, k_hi = k_lo + bn;
    bool causal = q_hi > k_lo;
    bool sink_b = k_lo < sink;
    bool win_b = (k_hi - 1) >= (q_lo - window + 1);
    out[idx] = (causal && (sink_b || win_b)) ? 1 : 0;
  }
}

__global__ void dense_mask_kernel(int64_t n_qb, int64_t n_kb, int64_t bm, int64_t bn,
                                  int causal, int32_t* out) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = n_qb * n_kb;
  for (; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t i = idx / n_kb, j = idx - i * n_kb;
    out[idx] = causal ? ((j * bn < (i + 1) * bm) ? 1 : 0) : 1;
  }
}

struct PlanGeom {
  const int32_t* mask;
  int n_q, n_kv, bm, bn, n_kb;  // user mask geometry
  int tm, tn, n_ti, n_tj;       // tile geometry
};

// kept = any overlapped user block nonzero, full = all nonzero.
__device__ __forceinline__ void tile_flags(const PlanGeom& g, int ti, int tj, bool& kept,
                                           bool& full) {
  int r0 = ti * g.tm, r1 = min((ti + 1) * g.tm, g.n_q);
  int c0 = tj * g.tn, c1 = min((tj + 1) * g.tn, g.n_kv);
  int b0 = r0 / g.bm, b1 = (r1 - 1) / g.bm;
  int d0 = c0 / g.bn, d1 = (c1 - 1) / g.bn;
  bool any = false, all = true;
  for (int b = b0; b <= b1; ++b) {
    const int32_t* row = g.mask + (size_t)b * g.n_kb;
    for (int d = d0; d <= d1; ++d) {
      bool on = __ldg(row + d) != 0;
      any |= on;
      all &= on;
    }
  }
  kept = any;
  full = all;
}

// Block x < n_ti handles tile row x (CSR); block x >= n_ti handles tile
// column x - n_ti (CSC).  Pass 0 writes counts to ptr[line + 1]; pass 1
// writes the compacted, ascending index list starting at ptr[line].
template <int PASS>
__global__ void plan_line_kernel(PlanGeom g, int32_t* row_ptr, int32_t* col_idx,
                                 int32_t* col_ptr, int32_t* row_idx) {
  const bool is_row = blockIdx.x < (unsigned)g.n_ti;
  const int line = is_row ? blockIdx.x : blockIdx.x - g.n_ti;
  int32_t* ptr = is_row ? row_ptr : col_ptr;
  int32_t* idx = is_row ? col_idx : row_idx;
  if (ptr == nullptr) return;
  const int len = is_row ? g.n_tj : g.n_ti;
  __shared__ int warp_tot[32];
  __shared__ int base;
  if (threadIdx.x == 0) base = (PASS == 1) ? ptr[line] : 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int start = 0; start < len; start += blockDim.x) {
    int other = start + threadIdx.x;
    bool kept = false, full = false;
    if (other < len) {
      if (is_row) tile_flags(g, line, other, kept, full);
      else tile_flags(g, other, line, kept, full);
    }
    unsigned ballot = __ballot_sync(0xffffffffu, kept);
    if (lane == 0) warp_tot[warp] = __popc(ballot);
    __syncthreads();
    int before = 0, chunk = 0;
    for (int w = 0; w < nwarps; ++w) {
      if (w < warp) before += warp_tot[w];
      chunk += warp_tot[w];
    }
    if (PASS == 1 && kept) {
      int pos = base + before + __popc(ballot & ((1u << lane) - 1u));
      idx[pos] = (int32_t)((uint32_t)other | (full ? 0u : kPartialBit));
    }
    __syncthreads();
    if (threadIdx.x == 0) base += chunk;
    __syncthreads();
  }
  if (PASS == 0 && threadIdx.x == 0) ptr[line + 1] = base;
}

// In-place exclusive scan of counts stored at ptr[1..n] (ptr[0] := 0), one
// CTA per array; writes the total to *nnz when given.
__global__ void plan_scan_kernel(int32_t* row_ptr, int n_rows, int32_t* col_ptr, int n_cols,
                                 int32_t* nnz) {
  int32_t* ptr = blockIdx.x == 0 ? row_ptr : col_ptr;
  const int n = blockIdx.x == 0 ? n_rows : n_cols;
  if (ptr == nullptr) return;
  __shared__ int carry;
  __shared__ int warp_sum[32];
  if (threadIdx.x == 0) { carry = 0; ptr[0] = 0; }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int start = 0; start < n; start += blockDim.x) {
    int i = start + threadIdx.x;
    int v = i < n ? ptr[i + 1] : 0;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sum[warp] = x;
    __syncthreads();
    int pre = 0, tot = 0;
    for (int w = 0; w < nwarps; ++w) {
      if (w < warp) pre += warp_sum[w];
      tot += warp_sum[w];
    }
    if (i < n) ptr[i + 1] = carry + pre + x;
    __syncthreads();
    if (threadIdx.x == 0) carry += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0 && nnz != nullptr && (blockIdx.x == 0 || row_ptr == nullptr)) *nnz = carry;
}

// For every CSR entry (tile row i, tile column j) of a plan, the position of
// the same tile in the CSC lists: a binary search for i in column j's
// ascending row list.  One CTA per tile row (grid-strided).
__global__ void plan_csc_pos_kernel(const int32_t* __restrict__ row_ptr,
                                    const int32_t* __restrict__ col_idx,
                                    const int32_t* __restrict__ col_ptr,
                                    const int32_t* __restrict__ row_idx, int n_ti,
                                    int32_t* __restrict__ csc_pos) {
  for (int i = blockIdx.x; i < n_ti; i += gridDim.x) {
    const int p1 = row_ptr[i + 1];
    for (int p = row_ptr[i] + threadIdx.x; p < p1; p += blockDim.x) {
      const int j = plan_index(col_idx[p]);
      int lo = col_ptr[j], hi = col_ptr[j + 1];
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (plan_index(row_idx[mid]) < i) lo = mid + 1; else hi = mid;
      }
      csc_pos[p] = lo;
    }
  }
}

int grid_for(int64_t total) {
  int64_t g = (total + 255) / 256;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 32));
}

}  // namespace
}  // namespace sbfa

using namespace sbfa;

extern "C" int sbfa_streaming_mask(int64_t n_q, int64_t n_kv, int64_t sink, int64_t window,
                                   int64_t block_m, int64_t block_n, int32_t* mask_out,
                                   void* stream) {
  if (n_q <= 0 || n_kv <= 0) return fail(SBFA_ERR_INVALID, "n_q and n_kv must be positive");
  if (sink < 0 || window < 0)
    return fail(SBFA_ERR_INVALID, "sink_size and window_size must be non-negative");
  if (block_m <= 0 || block_n <= 0) return fail(SBFA_ERR_INVALID, "block sizes must be positive");
  if (mask_out == nullptr) return fail(SBFA_ERR_INVALID, "mask_out is NULL");
  int64_t n_qb = (n_q + block_m - 1) / block_m, n_kb = (n_kv + block_n - 1) / block_n;
  {
    LaunchScope ls("streaming_mask_kernel", (cudaStream_t)stream);
    streaming_mask_kernel<<<grid_for(n_qb * n_kb), 256, 0, (cudaStream_t)stream>>>(
        n_qb, n_kb, n_kv - n_q, sink, window, block_m, block_n, mask_out);
  }
  return check_launch("streaming_mask_kernel");
}

extern "C" int sbfa_dense_mask(int64_t n_q, int64_t n_kv, int64_t block_m, int64_t block_n,
                               int causal, int32_t* mask_out, void* stream) {
  if (block_m <= 0 || block_n <= 0) return fail(SBFA_ERR_INVALID, "block sizes must be positive");
  if (n_q % block_m != 0 || n_kv % block_n != 0)
    return fail(SBFA_ERR_INVALID, "block_m / block_n must divide n_q / n_kv");
  if (mask_out == nullptr) return fail(SBFA_ERR_INVALID, "mask_out is NULL");
  int64_t n_qb = n_q / block_m, n_kb = n_kv / block_n;
  if (n_qb * n_kb == 0) return SBFA_OK;
  {
    LaunchScope ls("dense_mask_kernel", (cudaStream_t)stream);
    dense_mask_kernel<<<grid_for(n_qb * n_kb), 256, 0, (cudaStream_t)stream>>>(
        n_qb, n_kb, block_m, block_n, causal, mask_out);
  }
  return check_launch("dense_mask_kernel");
}

extern "C" int sbfa_build_plan(const int32_t* block_mask, int64_t n_q, int64_t n_kv,
                               int64_t block_m, int64_t block_n, int64_t tile_m,
                               int64_t tile_n, int32_t* row_ptr, int32_t* col_idx,
                               int32_t* col_ptr, int32_t* row_idx, int32_t* nnz_out,
                               void* stream) {
  if (block_mask == nullptr) return fail(SBFA_ERR_INVALID, "block_mask is NULL");
  if (n_q <= 0 || n_kv <= 0 || block_m <= 0 || block_n <= 0 || tile_m <= 0 || tile_n <= 0)
    return fail(SBFA_ERR_INVALID, "sizes must be positive");
  if (n_q >= (1ll << 31) || n_kv >= (1ll << 31))
    return fail(SBFA_ERR_INVALID, "sequence lengths must fit in int32");
  if ((row_ptr == nullptr) != (col_idx == nullptr) || (col_ptr == nullptr) != (row_idx == nullptr))
    return fail(SBFA_ERR_INVALID, "CSR / CSC arrays must be given in pairs");
  PlanGeom g;
  g.mask = block_mask;
  g.n_q = (int)n_q;
  g.n_kv = (int)n_kv;
  g.bm = (int)block_m;
  g.bn = (int)block_n;
  g.n_kb = ceil_div_i(n_kv, block_n);
  g.tm = (int)tile_m;
  g.tn = (int)tile_n;
  g.n_ti = ceil_div_i(n_q, tile_m);
  g.n_tj = ceil_div_i(n_kv, tile_n);
  cudaStream_t s = (cudaStream_t)stream;
  const int lines = g.n_ti + g.n_tj;
  {
    LaunchScope ls("plan_count_kernel", s);
    plan_line_kernel<0><<<lines, 256, 0, s>>>(g, row_ptr, col_idx, col_ptr, row_idx);
  }
  if (int rc = check_launch("plan_line_kernel<count>")) return rc;
  {
    LaunchScope ls("plan_scan_kernel", s);
    plan_scan_kernel<<<2, 1024, 0, s>>>(row_ptr, g.n_ti, col_ptr, g.n_tj, nnz_out);
  }
  if (int rc = check_launch("plan_scan_kernel")) return rc;
  {
    LaunchScope ls("plan_fill_kernel", s);
    plan_line_kernel<1><<<lines, 256, 0, s>>>(g, row_ptr, col_idx, col_ptr, row_idx);
  }
  return check_launch("plan_line_kernel<fill>");
}

extern "C" int sbfa_plan_csc_positions(const int32_t* row_ptr, const int32_t* col_idx,
                                       const int32_t* col_ptr, const int32_t* row_idx,
                                       int64_t n_ti, int32_t* csc_pos, void* stream) {
  if (!row_ptr || !col_idx || !col_ptr || !row_idx || !csc_pos)
    return fail(SBFA_ERR_INVALID, "sbfa_plan_csc_positions: NULL plan pointer");
  if (n_ti <= 0 || n_ti >= (1ll << 31)) return fail(SBFA_ERR_INVALID, "n_ti out of range");
  cudaStream_t s = (cudaStream_t)stream;
  {
    LaunchScope ls("plan_csc_pos_kernel", s);
    plan_csc_pos_kernel<<<(int)std::min<int64_t>(n_ti, 148 * 8), 128, 0, s>>>(
        row_ptr, col_idx, col_ptr, row_idx, (int)n_ti, csc_pos);
  }
  return check_launch("plan_csc_pos_kernel");
}
