// Shared device/host helpers for libsbfa: element types, the StreamingLLM
// token rule, the per-device status word and host-side error reporting.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "sbfa.h"

namespace sbfa {

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------

template <typename T> struct Elem;
template <> struct Elem<__half> {
  using acc = float;
  static __device__ __forceinline__ float to(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  using acc = float;
  static __device__ __forceinline__ float to(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<float> {
  using acc = float;
  static __device__ __forceinline__ float to(float x) { return x; }
  static __device__ __forceinline__ float from(float x) { return x; }
};
template <> struct Elem<double> {
  using acc = double;
  static __device__ __forceinline__ double to(double x) { return x; }
  static __device__ __forceinline__ double from(double x) { return x; }
};

template <typename A> __device__ __forceinline__ A acc_exp(A x);
template <> __device__ __forceinline__ float acc_exp<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double acc_exp<double>(double x) { return exp(x); }
template <typename A> __device__ __forceinline__ A acc_log(A x);
template <> __device__ __forceinline__ float acc_log<float>(float x) { return logf(x); }
template <> __device__ __forceinline__ double acc_log<double>(double x) { return log(x); }
template <typename A> __device__ __forceinline__ A neg_inf();
template <> __device__ __forceinline__ float neg_inf<float>() { return -INFINITY; }
template <> __device__ __forceinline__ double neg_inf<double>() { return -(double)INFINITY; }

// ---------------------------------------------------------------------------
// Mask semantics (one place, used by every kernel)
// ---------------------------------------------------------------------------

// Per-call mask parameters.  sink/window are pre-clamped on the host to
// [0, n_kv] / [0, n_kv + 1] so every position fits in int32 and the rule is
// unchanged (a window longer than q + 1 already admits every k <= q).
struct MaskParams {
  const int32_t* block_mask;  // [n_qb, n_kb] int32
  int n_q, n_kv;
  int q_off;                  // n_kv - n_q
  int block_m, block_n, n_kb;
  int sink, window;
  int causal;
};

// Element strides (batch, head, row) of one [B, H, N, D] tensor whose last
// dimension is unit-stride (upstream makes every input contiguous first,
// sparse_triton_kernel.py:834; here views are read in place).
struct Strides3 {
  int64_t b, h, n;
};

// Strides of every tensor of a call, the query head count that splits the
// flattened (batch, query head) index bh into (bh / heads, bh % heads), and
// the grouped-query factor: query head h reads key/value head h / kv_group
// (kv_group = 1 without grouping).  k, v, dk, dv have heads / kv_group heads.
struct Views {
  Strides3 q, k, v, o, dout, dq, dk, dv;
  int heads;
  int kv_group;
  // element offset of row `row` of query-side tensor s for bh
  __host__ __device__ __forceinline__ int64_t at(const Strides3& s, int bh, int64_t row) const {
    return (int64_t)(bh / heads) * s.b + (int64_t)(bh % heads) * s.h + row * s.n;
  }
  // element offset of row `row` of key/value-side tensor s for query bh
  __host__ __device__ __forceinline__ int64_t at_kv(const Strides3& s, int bh, int64_t row) const {
    return (int64_t)(bh / heads) * s.b + (int64_t)((bh % heads) / kv_group) * s.h + row * s.n;
  }
};

// Token rule of sparse_triton_kernel.py:315-319 at absolute positions.
__device__ __forceinline__ bool token_visible(int qpos, int k, int sink, int window) {
  return (k <= qpos) && (k < sink || k >= qpos - window + 1);
}

// Lifted block-mask entry for (query row, key) (sparse_triton_kernel.py:877-879).
__device__ __forceinline__ bool lifted_visible(const MaskParams& mp, int row, int k) {
  return __ldg(mp.block_mask + (size_t)(row / mp.block_m) * mp.n_kb + (k / mp.block_n)) != 0;
}

// Full visibility of element (row, k): bounds, lifted block mask (only when
// the tile is partial), token rule (only when causal).
__device__ __forceinline__ bool visible(const MaskParams& mp, int row, int k, bool partial) {
  if (row >= mp.n_q || k >= mp.n_kv) return false;
  if (partial && !lifted_visible(mp, row, k)) return false;
  if (mp.causal && !token_visible(mp.q_off + row, k, mp.sink, mp.window)) return false;
  return true;
}

constexpr uint32_t kPartialBit = 0x80000000u;
__device__ __forceinline__ int plan_index(int32_t e) { return (int)((uint32_t)e & ~kPartialBit); }
__device__ __forceinline__ bool plan_partial(int32_t e) { return ((uint32_t)e & kPartialBit) != 0; }

// ---------------------------------------------------------------------------
// Host-side error plumbing
// ---------------------------------------------------------------------------

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);

// Device address of the status word of the current device (allocated once
// per device inside libsbfa, zero-initialised).
int* device_status_ptr();

// Status codes a kernel may record (first writer wins).
constexpr int kStatusWaitTimeout = 1;
constexpr int kStatusBadSmemAlign = 2;
constexpr int kStatusBoundsCheck = 3;  // debug builds: an index was out of range
__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------------------
// Bounds checks of the debug build (compiled with SBFA_DEBUG_BOUNDS)
// ---------------------------------------------------------------------------
// Every index a kernel reads from a plan (list offsets, list lengths, tile
// indices) and the tile coordinates derived from it go through these.  In
// the debug build a value outside its range is recorded in the status word
// (kStatusBoundsCheck) and replaced by the nearest value in range, so the
// access it feeds stays inside its buffer and no pipeline changes shape; in
// release builds they return the value unchanged.
__device__ __forceinline__ int bounded(int v, int hi, int* status) {
#ifdef SBFA_DEBUG_BOUNDS
  if (v < 0 || v >= hi) {
    record_status(status, kStatusBoundsCheck);
    return v < 0 ? 0 : max(hi - 1, 0);
  }
#endif
  (void)hi;
  (void)status;
  return v;
}

// The list [e0, e0 + n) of line i of a compacted plan (CSR row_ptr or CSC
// col_ptr): e0 within the cap entries of the list array, n within the
// n_other tiles of the crossing dimension and the array's end.
struct PlanSpan {
  int e0, n;
};
__device__ __forceinline__ PlanSpan plan_span(const int32_t* ptr, int i, int n_other,
                                              int64_t cap, int* status) {
  PlanSpan s{ptr[i], ptr[i + 1] - ptr[i]};
#ifdef SBFA_DEBUG_BOUNDS
  const int icap = (int)min(cap, (int64_t)0x7fffffff - 1);
  s.e0 = bounded(s.e0, icap + 1, status);
  s.n = bounded(s.n, min(n_other, icap - s.e0) + 1, status);
#endif
  (void)n_other;
  (void)cap;
  return s;
}

// Plan entry e of a list: tile index checked against the n_other tiles of
// the crossing dimension, the partial bit kept.
__device__ __forceinline__ int32_t plan_entry(const int32_t* list, int e, int n_other,
                                              int* status) {
  const int32_t ent = list[e];
#ifdef SBFA_DEBUG_BOUNDS
  const int idx = bounded((int)((uint32_t)ent & 0x7fffffffu), n_other, status);
  return (int32_t)(((uint32_t)ent & 0x80000000u) | (uint32_t)idx);
#else
  (void)n_other;
  (void)status;
  return ent;
#endif
}

inline int ceil_div_i(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }
__device__ __forceinline__ int ceil_div_dev(int a, int b) {
  return (int)(((int64_t)a + b - 1) / b);
}

// Wraps one kernel launch: counts it, and when timing is enabled
// (sbfa_timing_enable) records a CUDA event pair around it on its stream,
// tagged with `name`, for sbfa_timing_read.
class LaunchScope {
 public:
  LaunchScope(const char* name, cudaStream_t s);
  ~LaunchScope();
  LaunchScope(const LaunchScope&) = delete;
  LaunchScope& operator=(const LaunchScope&) = delete;

 private:
  const char* name_;
  cudaStream_t stream_;
  cudaEvent_t start_ = nullptr;
};

}  // namespace sbfa
