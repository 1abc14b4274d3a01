// extern "C" entry points of libsbfa.so (declared in include/sbfa.h):
// argument validation mirroring the upstream bridge
// (sparse_triton_kernel.py:631-650), error strings, the per-device status
// word, and selection between the tensor-core and generic kernels by
// dtype / head dim (one backend, shape-based selection).
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "sbfa_common.cuh"

namespace sbfa {

// attn_generic.cu
int generic_tiles(int pass, int64_t* tm, int64_t* tn);
bool generic_supports(int dtype, int64_t D);
int generic_fwd(int dtype, int D, const void* q, const void* k, const void* v, void* o,
                float* lse, int BH, double scale, const MaskParams& mp, const Views& vw,
                const int32_t* rp, const int32_t* ci, cudaStream_t s);
int generic_bwd(int dtype, int D, const void* q, const void* k, const void* v, const void* o,
                const float* lse, const void* dout, void* dq, void* dk, void* dv, float* delta,
                int BH, double scale, const MaskParams& mp, const Views& vw, const int32_t* a,
                const int32_t* b, const int32_t* c, const int32_t* d, cudaStream_t s);
// decode.cu
int decode_tile();
int64_t decode_est_tiles(int64_t n_kv, int is_causal, int64_t sink, int64_t window);
int decode_group(int dtype, int64_t D);
int decode_splits(int64_t BH, int group, int dtype, int64_t D, int64_t est_tiles);
int decode_max_splits(int64_t BH, int64_t est_tiles);
int64_t decode_ws_bytes(int64_t BH, int64_t D, int nsplit);
int decode_run(int dtype, const void* q, const void* k, const void* v, void* o, float* lse,
               void* ws, int BH, int D, float scale, const MaskParams& mp, const int32_t* rp,
               const int32_t* ci, int nsplit, int heads, int group, cudaStream_t s);
// attn_tc.cu
bool tc_supports(int pass, int dtype, int64_t D);
int tc_tiles(int pass, int64_t* tm, int64_t* tn);
int tc_fwd(int dtype, int D, const void* q, const void* k, const void* v, void* o, float* lse,
           int BH, float scale, const MaskParams& mp, const Views& vw, const int32_t* rp,
           const int32_t* ci, int* status, cudaStream_t s);
int tc_bwd(int dtype, int D, const void* q, const void* k, const void* v, const void* o,
           const float* lse, const void* dout, void* dq, void* dk, void* dv, float* delta,
           int BH, float scale, const MaskParams& mp, const Views& vw, const int32_t* dq_rp,
           const int32_t* dq_ci, const int32_t* kv_cp, const int32_t* kv_ri, void* split_ws,
           int64_t split_ws_bytes, const int32_t* csc_pos, int64_t nnz, void* ds_ws,
           int64_t ds_ws_bytes, int* status, cudaStream_t s);
int64_t tc_bwd_split_bytes(int64_t BH, int kv_group, int64_t D);
int64_t tc_bwd_ds_bytes(int64_t BH, int64_t nnz, int64_t D);
namespace tc {
bool tma_compatible(const void* base, const Strides3& st);
}

namespace {
thread_local std::string g_last_error;
__device__ int g_status_word;
std::mutex g_status_mu;
int* g_status_ptr[64] = {nullptr};

std::atomic<int64_t> g_launches{0};
std::atomic<bool> g_timing{false};
struct TimedLaunch {
  const char* name;
  cudaEvent_t start, stop;
};
std::mutex g_timing_mu;
std::vector<TimedLaunch> g_timed;
}  // namespace

LaunchScope::LaunchScope(const char* name, cudaStream_t s) : name_(name), stream_(s) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (g_timing.load(std::memory_order_relaxed)) {
    if (cudaEventCreate(&start_) == cudaSuccess) {
      if (cudaEventRecord(start_, stream_) != cudaSuccess) {
        cudaEventDestroy(start_);
        start_ = nullptr;
      }
    } else {
      start_ = nullptr;
    }
  }
}

LaunchScope::~LaunchScope() {
  if (start_ == nullptr) return;
  cudaEvent_t stop = nullptr;
  if (cudaEventCreate(&stop) == cudaSuccess && cudaEventRecord(stop, stream_) == cudaSuccess) {
    std::lock_guard<std::mutex> lock(g_timing_mu);
    g_timed.push_back({name_, start_, stop});
    return;
  }
  if (stop) cudaEventDestroy(stop);
  cudaEventDestroy(start_);
}

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SBFA_OK;
  return fail(SBFA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

int device_sm_count() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    cached[dev] =
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0
            ? n
            : 148;
  }
  return cached[dev];
}

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = (int*)p;
  }
  return g_status_ptr[dev];
}

namespace {

int elem_size(int dtype) {
  switch (dtype) {
    case SBFA_F16: case SBFA_BF16: return 2;
    case SBFA_F32: return 4;
    case SBFA_F64: return 8;
  }
  return 0;
}

int check_common(int64_t B, int64_t H, int64_t n_q, int64_t n_kv, int64_t D, int dtype,
                 int64_t sink, int64_t window, const int32_t* block_mask, int64_t bm,
                 int64_t bn) {
  if (elem_size(dtype) == 0) return fail(SBFA_ERR_INVALID, "unknown dtype code");
  if (B <= 0 || H <= 0 || n_q <= 0 || n_kv <= 0 || D <= 0)
    return fail(SBFA_ERR_INVALID, "B, H, n_q, n_kv and head_dim must be positive");
  if (n_q >= (1ll << 31) || n_kv >= (1ll << 31))
    return fail(SBFA_ERR_INVALID, "sequence lengths must fit in int32");
  if (B * H > 65535) return fail(SBFA_ERR_UNSUPPORTED, "B * H must be <= 65535");
  if (sink < 0 || window < 0)
    return fail(SBFA_ERR_INVALID, "sink_size and window_size must be non-negative");
  if (bm <= 0 || bn <= 0) return fail(SBFA_ERR_INVALID, "block sizes must be positive");
  if (block_mask == nullptr) return fail(SBFA_ERR_INVALID, "block_mask is NULL");
  return SBFA_OK;
}

MaskParams make_mp(int64_t n_q, int64_t n_kv, int is_causal, int64_t sink, int64_t window,
                   const int32_t* block_mask, int64_t bm, int64_t bn) {
  MaskParams mp;
  mp.block_mask = block_mask;
  mp.n_q = (int)n_q;
  mp.n_kv = (int)n_kv;
  mp.q_off = (int)(n_kv - n_q);
  mp.block_m = (int)std::min<int64_t>(bm, 1ll << 30);
  mp.block_n = (int)std::min<int64_t>(bn, 1ll << 30);
  mp.n_kb = ceil_div_i(n_kv, bn);
  mp.sink = (int)std::min<int64_t>(sink, n_kv);
  mp.window = (int)std::min<int64_t>(window, n_kv + 1);
  mp.causal = is_causal ? 1 : 0;
  return mp;
}

bool use_tc(int pass, int dtype, int64_t D) { return tc_supports(pass, dtype, D); }

// Views of a call: strides == NULL means every tensor is contiguous
// [B, H or H_kv, N, D]; otherwise strides holds (batch, head, row) element
// strides for each of the `count` tensors in the order of Views' members.
// kv_heads <= 0 means H (no grouping); else H must be a multiple of it.
int make_views(const int64_t* strides, int count, int64_t H, int64_t kv_heads, int64_t n_q,
               int64_t n_kv, int64_t D, Views* vw) {
  if (kv_heads <= 0) kv_heads = H;
  if (H % kv_heads != 0)
    return fail(SBFA_ERR_INVALID, "the query head count must be a multiple of kv_heads");
  Strides3* dst[8] = {&vw->q, &vw->k, &vw->v, &vw->o, &vw->dout, &vw->dq, &vw->dk, &vw->dv};
  const bool kv_side[8] = {false, true, true, false, false, false, true, true};
  vw->heads = (int)H;
  vw->kv_group = (int)(H / kv_heads);
  for (int t = 0; t < 8; ++t) {
    const int64_t n = kv_side[t] ? n_kv : n_q;
    const int64_t h = kv_side[t] ? kv_heads : H;
    if (strides == nullptr || t >= count) {
      *dst[t] = Strides3{h * n * D, n * D, D};
    } else {
      const int64_t* st = strides + 3 * t;
      if (st[0] < 0 || st[1] < 0 || st[2] < D)
        return fail(SBFA_ERR_INVALID,
                    "strides must be non-negative and rows at least head_dim apart");
      *dst[t] = Strides3{st[0], st[1], st[2]};
    }
  }
  return SBFA_OK;
}

// The tensor-core kernels read every tensor through TMA maps.
int check_tma(const void* const* ptrs, const Strides3* const* st, int count, const char* who) {
  for (int t = 0; t < count; ++t)
    if (!tc::tma_compatible(ptrs[t], *st[t]))
      return fail(SBFA_ERR_INVALID,
                  std::string(who) + ": for float16/bfloat16 with head_dim 64 or 128 every "
                  "tensor must be 16-byte aligned with batch, head and row strides that are "
                  "positive multiples of 8 elements");
  return SBFA_OK;
}

}  // namespace
}  // namespace sbfa

using namespace sbfa;

extern "C" int sbfa_abi_version(void) { return 5; }

extern "C" int64_t sbfa_launch_count(void) { return g_launches.load(); }

extern "C" int sbfa_timing_enable(int on) {
  g_timing.store(on != 0);
  return SBFA_OK;
}

extern "C" int sbfa_timing_read(int max_kernels, char* names, double* total_ms,
                                int64_t* launches, int* n_out) {
  std::vector<TimedLaunch> rec;
  {
    std::lock_guard<std::mutex> lock(g_timing_mu);
    rec.swap(g_timed);
  }
  std::vector<std::string> keys;
  std::vector<double> ms;
  std::vector<int64_t> cnt;
  int rc = SBFA_OK;
  for (auto& r : rec) {
    float t = 0.f;
    if (rc == SBFA_OK) rc = check_cuda(cudaEventSynchronize(r.stop), "timing sync");
    if (rc == SBFA_OK) rc = check_cuda(cudaEventElapsedTime(&t, r.start, r.stop), "timing read");
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
    size_t i = 0;
    while (i < keys.size() && keys[i] != r.name) ++i;
    if (i == keys.size()) {
      keys.emplace_back(r.name);
      ms.push_back(0.0);
      cnt.push_back(0);
    }
    ms[i] += t;
    cnt[i] += 1;
  }
  if (rc != SBFA_OK) return rc;
  const int n = (int)std::min<size_t>(keys.size(), (size_t)std::max(0, max_kernels));
  for (int i = 0; i < n; ++i) {
    if (names) {
      std::memset(names + 64 * i, 0, 64);
      std::strncpy(names + 64 * i, keys[i].c_str(), 63);
    }
    if (total_ms) total_ms[i] = ms[i];
    if (launches) launches[i] = cnt[i];
  }
  if (n_out) *n_out = n;
  return SBFA_OK;
}

extern "C" int sbfa_last_error(char* buf, size_t len) {
  const std::string& e = g_last_error;
  if (buf && len) {
    size_t n = std::min(len - 1, e.size());
    std::memcpy(buf, e.data(), n);
    buf[n] = '\0';
  }
  return (int)e.size();
}

extern "C" int sbfa_device_status(int* status_out) {
  int* p = device_status_ptr();
  if (p == nullptr) return fail(SBFA_ERR_CUDA, "cannot resolve the device status word");
  int v = 0;
  if (int rc = check_cuda(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost),
                          "read device status"))
    return rc;
  if (v != 0) {
    int zero = 0;
    if (int rc = check_cuda(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice),
                            "clear device status"))
      return rc;
  }
  if (status_out) *status_out = v;
  return SBFA_OK;
}

extern "C" int sbfa_plan_tiles(int pass, int dtype, int64_t head_dim, int64_t n_q,
                               int64_t* tile_m, int64_t* tile_n) {
  if (tile_m == nullptr || tile_n == nullptr) return fail(SBFA_ERR_INVALID, "NULL output");
  if (pass < 0 || pass > 3) return fail(SBFA_ERR_INVALID, "pass must be 0..3");
  if (pass == 3) {
    *tile_m = 1;
    *tile_n = decode_tile();
    return SBFA_OK;
  }
  (void)n_q;
  if (use_tc(pass, dtype, head_dim)) return tc_tiles(pass, tile_m, tile_n);
  return generic_tiles(pass, tile_m, tile_n);
}

extern "C" int sbfa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                        int64_t B, int64_t H, int64_t n_q, int64_t n_kv, int64_t head_dim,
                        int dtype, double softmax_scale, int is_causal, int64_t sink,
                        int64_t window, const int32_t* block_mask, int64_t block_m,
                        int64_t block_n, const int32_t* row_ptr, const int32_t* col_idx,
                        const int64_t* strides, int64_t kv_heads, void* stream) {
  if (int rc = check_common(B, H, n_q, n_kv, head_dim, dtype, sink, window, block_mask,
                            block_m, block_n))
    return rc;
  if (!q || !k || !v || !o || !lse || !row_ptr || !col_idx)
    return fail(SBFA_ERR_INVALID, "sbfa_fwd: NULL tensor or plan pointer");
  Views vw;
  if (int rc = make_views(strides, 4, H, kv_heads, n_q, n_kv, head_dim, &vw)) return rc;
  MaskParams mp = make_mp(n_q, n_kv, is_causal, sink, window, block_mask, block_m, block_n);
  cudaStream_t s = (cudaStream_t)stream;
  const int BH = (int)(B * H);
  if (use_tc(0, dtype, head_dim)) {
    const void* ptrs[4] = {q, k, v, o};
    const Strides3* st[4] = {&vw.q, &vw.k, &vw.v, &vw.o};
    if (int rc = check_tma(ptrs, st, 4, "sbfa_fwd")) return rc;
    return tc_fwd(dtype, (int)head_dim, q, k, v, o, lse, BH, softmax_scale, mp, vw, row_ptr,
                  col_idx, device_status_ptr(), s);
  }
  if (!generic_supports(dtype, head_dim))
    return fail(SBFA_ERR_UNSUPPORTED, "head_dim too large (max 256; 128 for float64)");
  return generic_fwd(dtype, (int)head_dim, q, k, v, o, lse, BH, softmax_scale, mp, vw, row_ptr,
                     col_idx, s);
}

extern "C" int sbfa_bwd(const void* q, const void* k, const void* v, const void* o,
                        const float* lse, const void* dout, void* dq, void* dk, void* dv,
                        float* delta_ws, int64_t B, int64_t H, int64_t n_q, int64_t n_kv,
                        int64_t head_dim, int dtype, double softmax_scale, int is_causal,
                        int64_t sink, int64_t window, const int32_t* block_mask,
                        int64_t block_m, int64_t block_n, const int32_t* dq_row_ptr,
                        const int32_t* dq_col_idx, const int32_t* kv_col_ptr,
                        const int32_t* kv_row_idx, const int64_t* strides, int64_t kv_heads,
                        void* split_ws, int64_t split_ws_bytes, const int32_t* dq_csc_pos,
                        int64_t nnz, void* ds_ws, int64_t ds_ws_bytes, void* stream) {
  if (int rc = check_common(B, H, n_q, n_kv, head_dim, dtype, sink, window, block_mask,
                            block_m, block_n))
    return rc;
  if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv || !delta_ws)
    return fail(SBFA_ERR_INVALID, "sbfa_bwd: NULL tensor pointer");
  if (!dq_row_ptr || !dq_col_idx || !kv_col_ptr || !kv_row_idx)
    return fail(SBFA_ERR_INVALID, "sbfa_bwd: NULL plan pointer");
  Views vw;
  if (int rc = make_views(strides, 8, H, kv_heads, n_q, n_kv, head_dim, &vw)) return rc;
  MaskParams mp = make_mp(n_q, n_kv, is_causal, sink, window, block_mask, block_m, block_n);
  cudaStream_t s = (cudaStream_t)stream;
  const int BH = (int)(B * H);
  if (use_tc(1, dtype, head_dim)) {
    const void* ptrs[7] = {q, k, v, dout, dq, dk, dv};
    const Strides3* st[7] = {&vw.q, &vw.k, &vw.v, &vw.dout, &vw.dq, &vw.dk, &vw.dv};
    if (int rc = check_tma(ptrs, st, 7, "sbfa_bwd")) return rc;
    return tc_bwd(dtype, (int)head_dim, q, k, v, o, lse, dout, dq, dk, dv, delta_ws, BH,
                  softmax_scale, mp, vw, dq_row_ptr, dq_col_idx, kv_col_ptr, kv_row_idx,
                  split_ws, split_ws_bytes, dq_csc_pos, nnz, ds_ws, ds_ws_bytes,
                  device_status_ptr(), s);
  }
  if (!generic_supports(dtype, head_dim))
    return fail(SBFA_ERR_UNSUPPORTED, "head_dim too large (max 256; 128 for float64)");
  return generic_bwd(dtype, (int)head_dim, q, k, v, o, lse, dout, dq, dk, dv, delta_ws, BH,
                     softmax_scale, mp, vw, dq_row_ptr, dq_col_idx, kv_col_ptr, kv_row_idx, s);
}


namespace sbfa {
// Every check sbfa_decode makes on its tensors and shape, before anything is
// launched (shared with sbfa_decode_noalloc, which builds its plan only once
// these pass).
int check_decode_args(const void* q, const void* k, const void* v, const void* o, int64_t B,
                      int64_t H, int64_t n_kv, int64_t head_dim, int dtype, int64_t sink,
                      int64_t window, const int32_t* block_mask, int64_t block_m,
                      int64_t block_n, int64_t kv_heads) {
  if (int rc = check_common(B, H, 1, n_kv, head_dim, dtype, sink, window, block_mask, block_m,
                            block_n))
    return rc;
  if (!q || !k || !v || !o) return fail(SBFA_ERR_INVALID, "decode: NULL tensor pointer");
  if (kv_heads > 0 && (kv_heads > H || H % kv_heads != 0))
    return fail(SBFA_ERR_INVALID, "the query head count must be a multiple of kv_heads");
  if (decode_group(dtype, head_dim) == 0)
    return fail(SBFA_ERR_UNSUPPORTED,
                "decode: head_dim * element size must be 16..512 bytes in powers of two "
                "(fp16/bf16/fp32)");
  for (const void* p : {q, k, v, o})
    if (((uintptr_t)p & 15u) != 0)
      return fail(SBFA_ERR_UNSUPPORTED, "decode: tensors must be 16-byte aligned");
  return SBFA_OK;
}
}  // namespace sbfa

extern "C" int64_t sbfa_bwd_workspace_bytes(int64_t B, int64_t H, int64_t head_dim, int dtype,
                                            int64_t kv_heads) {
  if (B <= 0 || H <= 0 || head_dim <= 0) return 0;
  if (kv_heads <= 0) kv_heads = H;
  if (kv_heads > H || H % kv_heads != 0 || !use_tc(1, dtype, head_dim)) return 0;
  return tc_bwd_split_bytes(B * H, (int)(H / kv_heads), head_dim);
}

extern "C" int64_t sbfa_bwd_ds_workspace_bytes(int64_t B, int64_t H, int64_t head_dim,
                                               int dtype, int64_t nnz) {
  if (B <= 0 || H <= 0 || !use_tc(1, dtype, head_dim)) return 0;
  return tc_bwd_ds_bytes(B * H, nnz, head_dim);
}

extern "C" int64_t sbfa_decode_workspace_bytes(int64_t B, int64_t H, int64_t n_kv,
                                               int64_t head_dim, int64_t block_n) {
  (void)block_n;
  // sized for the worst case over masks (non-causal: every tile may be kept)
  // and over head groupings (the most query heads per CTA, so the fewest
  // CTAs per split and the most splits)
  if (B <= 0 || H <= 0 || head_dim <= 0 || n_kv <= 0) return 0;
  const int ns = decode_max_splits(B * H, decode_est_tiles(n_kv, 0, 0, 0));
  return decode_ws_bytes(B * H, head_dim, ns);
}

extern "C" int sbfa_decode(const void* q, const void* k, const void* v, void* o, float* lse,
                           int64_t B, int64_t H, int64_t n_kv, int64_t head_dim, int dtype,
                           double softmax_scale, int is_causal, int64_t sink, int64_t window,
                           const int32_t* block_mask, int64_t block_m, int64_t block_n,
                           const int32_t* row_ptr, const int32_t* col_idx, void* split_ws,
                           int64_t split_ws_bytes, int64_t kv_heads, void* stream) {
  if (int rc = check_decode_args(q, k, v, o, B, H, n_kv, head_dim, dtype, sink, window,
                                 block_mask, block_m, block_n, kv_heads))
    return rc;
  if (!row_ptr || !col_idx) return fail(SBFA_ERR_INVALID, "sbfa_decode: NULL plan pointer");
  if (kv_heads <= 0) kv_heads = H;
  const int group = (int)(H / kv_heads);
  const int ns = decode_splits(B * H, group, dtype, head_dim,
                               decode_est_tiles(n_kv, is_causal, sink, window));
  const int64_t need = decode_ws_bytes(B * H, head_dim, ns);
  if (need > 0 && (split_ws == nullptr || split_ws_bytes < need))
    return fail(SBFA_ERR_INVALID, "sbfa_decode: split workspace too small (need " +
                                      std::to_string(need) + " bytes)");
  MaskParams mp = make_mp(1, n_kv, is_causal, sink, window, block_mask, block_m, block_n);
  return decode_run(dtype, q, k, v, o, lse, split_ws, (int)(B * H), (int)head_dim,
                    softmax_scale, mp, row_ptr, col_idx, ns, (int)H, group,
                    (cudaStream_t)stream);
}

extern "C" int sbfa_decode_supported(int dtype, int64_t head_dim) {
  return decode_group(dtype, head_dim) != 0 ? 1 : 0;
}
