/*
 * sbfa.h - C ABI of libsbfa.so, the B200 (sm_100a) kernels for StreamingLLM
 * sink+window block-sparse attention.
 *
 * Conventions shared by every entry point
 *   - All tensor pointers are DEVICE pointers on the current CUDA device.
 *   - Q/K/V/O/dO/dQ/dK/dV are logical [B, H, N, D] tensors with a unit-stride
 *     last dimension.  sbfa_fwd and sbfa_bwd take an optional host array of
 *     (batch, head, row) element strides per tensor (NULL = contiguous), so
 *     transposed views are read and written in place; the tensor-core kernels
 *     (float16/bfloat16, head_dim 64 or 128) then need 16-byte aligned
 *     tensors whose strides are positive multiples of 8 elements.  The decode
 *     and ring-cache entry points take contiguous tensors.  LSE and Delta are
 *     always contiguous fp32 [B, H, N_Q].  (The upstream Python bridge forces
 *     .contiguous() on every input, sparse_triton_kernel.py:834,707.)
 *   - `stream` is a cudaStream_t passed as void*; every launch is
 *     asynchronous on it.  NULL means the legacy default stream.
 *   - Return value: SBFA_OK (0) or an SBFA_ERR_* code; sbfa_last_error()
 *     gives the message of the last failure on the calling thread.
 *   - Block masks are int32 [ceil(n_q/block_m), ceil(n_kv/block_n)], nonzero
 *     = keep, shared by every (batch, head) exactly as upstream
 *     (sparse_triton_kernel.py:645-650).
 *   - Queries are bottom-right aligned: query row r sits at absolute
 *     position (n_kv - n_q) + r (sparse_triton_kernel.py:655-660).
 *   - With is_causal != 0 a kept block additionally applies the token rule
 *     visible(q,k) = (k <= q) && (k < sink || k >= q - window + 1)
 *     (sparse_triton_kernel.py:315-322); with is_causal == 0 only the block
 *     mask (and sequence bounds) apply.
 *   - A query row with no visible key produces O = 0 and LSE = 0
 *     (sparse_triton_kernel.py:341-352) and zero gradients.
 */
#ifndef SBFA_H_
#define SBFA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum sbfa_status {
  SBFA_OK = 0,
  SBFA_ERR_INVALID = 1,     /* bad argument (shape, pointer, size) */
  SBFA_ERR_UNSUPPORTED = 2, /* valid request this build has no kernel for */
  SBFA_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  SBFA_ERR_DEVICE = 4       /* a kernel reported a failure through the status word */
};

enum sbfa_dtype { SBFA_F16 = 0, SBFA_BF16 = 1, SBFA_F32 = 2, SBFA_F64 = 3 };

/* ABI version of this header (bumped on any signature change). */
int sbfa_abi_version(void);

/* Copy the calling thread's last error message (NUL-terminated, truncated to
 * len) into buf.  Returns the full message length. */
int sbfa_last_error(char* buf, size_t len);

/* Read and clear the device status word of the current device (a blocking
 * device->host read of 4 bytes).  0 = no kernel reported a failure since
 * the last call; otherwise the first failure code a kernel recorded
 * (1 = a bounded wait on a pipeline barrier expired, 2 = a kernel found its
 * dynamic shared memory window not 1024-byte aligned and wrote nothing). */
int sbfa_device_status(int* status_out);

/* Failure-path self-test (no upstream counterpart): launches one block
 * whose bounded wait on a barrier that nothing completes gives up after
 * limit_ns (1e6 .. 1e9), exactly as every pipeline wait of the tensor-core
 * kernels does; it records status 1 for sbfa_device_status and returns, and
 * the context stays usable. */
int sbfa_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* Total kernel launches issued by this library in this process. */
int64_t sbfa_launch_count(void);

/* Per-kernel device timing (no upstream counterpart; upstream times whole
 * calls with torch.cuda.Event, benchmark.py:438-492).  While enabled, every
 * launch records a CUDA event pair around itself on its own stream.
 * sbfa_timing_read waits for the recorded events, writes up to max_kernels
 * aggregated rows (name as a NUL-terminated string in a 64-byte slot of
 * names, summed milliseconds, launch count), returns the row count through
 * n_out and clears the record. */
int sbfa_timing_enable(int on);
int sbfa_timing_read(int max_kernels, char* names, double* total_ms, int64_t* launches,
                     int* n_out);

/* ---------------------------------------------------------------------------
 * Masks and plans
 * ------------------------------------------------------------------------- */

/* Dense int32 block mask, bit-exact with make_streaming_mask
 * (sparse_triton_kernel.py:104-181): entry (i, j) is
 *   (q_hi > k_lo) & ((k_lo < sink) | (k_hi - 1 >= q_lo - window + 1))
 * with q_lo = i*block_m + (n_kv - n_q), q_hi = q_lo + block_m,
 * k_lo = j*block_n, k_hi = k_lo + block_n (unclamped).
 * mask_out: int32[ceil(n_q/block_m) * ceil(n_kv/block_n)]. */
int sbfa_streaming_mask(int64_t n_q, int64_t n_kv, int64_t sink, int64_t window,
                        int64_t block_m, int64_t block_n, int32_t* mask_out,
                        void* stream);

/* Dense (causal=0) or dense-causal block mask, bit-exact with
 * make_dense_mask (sparse_triton_kernel.py:184-210). */
int sbfa_dense_mask(int64_t n_q, int64_t n_kv, int64_t block_m, int64_t block_n,
                    int causal, int32_t* mask_out, void* stream);

/* Compacted kept-tile lists of a block mask re-tiled to (tile_m, tile_n).
 * Replaces the per-iteration mask scans of the upstream kernels
 * (sparse_triton_kernel.py:283-285, 448-449, 563-565).
 * Tile (I, J) covers rows [I*tile_m, (I+1)*tile_m) and keys
 * [J*tile_n, (J+1)*tile_n), clipped to n_q / n_kv; it is kept iff any user
 * block it overlaps is nonzero.  Index entries carry bit 31 set when some
 * overlapped user block is zero ("partial" tile: the kernel must test the
 * lifted block mask per element).
 *   row_ptr: int32[n_ti + 1], col_idx: int32[n_ti * n_tj]   (CSR, by query tile)
 *   col_ptr: int32[n_tj + 1], row_idx: int32[n_ti * n_tj]   (CSC, by key tile)
 *   nnz_out: int32[1] (device), number of kept tiles.
 * Any of the CSR / CSC pairs may be NULL to skip it. */
int sbfa_build_plan(const int32_t* block_mask, int64_t n_q, int64_t n_kv,
                    int64_t block_m, int64_t block_n, int64_t tile_m, int64_t tile_n,
                    int32_t* row_ptr, int32_t* col_idx, int32_t* col_ptr,
                    int32_t* row_idx, int32_t* nnz_out, void* stream);

/* For every CSR entry p of a plan (both lists built by sbfa_build_plan), the
 * position in row_idx of the same tile: csc_pos: int32[nnz].  Used by
 * sbfa_bwd to find the dS tile the dK/dV pass stored for CSR entry p. */
int sbfa_plan_csc_positions(const int32_t* row_ptr, const int32_t* col_idx,
                            const int32_t* col_ptr, const int32_t* row_idx, int64_t n_ti,
                            int32_t* csc_pos, void* stream);

/* Tile sizes (tile_m, tile_n) whose plan the given pass expects.
 * pass: 0 = forward, 1 = backward dQ (CSR), 2 = backward dK/dV (CSC),
 * 3 = decode (n_q == 1). */
int sbfa_plan_tiles(int pass, int dtype, int64_t head_dim, int64_t n_q,
                    int64_t* tile_m, int64_t* tile_n);

/* ---------------------------------------------------------------------------
 * Attention
 * ------------------------------------------------------------------------- */

/* Common shape/semantic arguments, in this order, for the calls below:
 *   B, H, n_q, n_kv, head_dim, dtype, softmax_scale, is_causal, sink, window,
 *   block_mask, block_m, block_n
 *
 * Tensor layout: logical [B, H, N, head_dim] with a unit-stride last
 * dimension.  strides == NULL means every tensor is contiguous; otherwise it
 * points to host int64 element strides (batch, head, row) for each tensor,
 * three per tensor, in the order the call lists (sbfa_fwd: q, k, v, o;
 * sbfa_bwd: q, k, v, o, dout, dq, dk, dv), so transposed views such as the
 * [B, N, H, D] memory behind Llama-style attention are read in place (upstream
 * copies them with .contiguous(), sparse_triton_kernel.py:707, 834).  For
 * float16/bfloat16 with head_dim 64 or 128 (the tensor-core kernels, which read
 * through TMA) every tensor must be 16-byte aligned and its strides positive
 * multiples of 8 elements, else SBFA_ERR_INVALID.  lse and delta_ws are always
 * contiguous [B, H, n_q].
 *
 * kv_heads: grouped-query attention (no upstream counterpart; upstream
 * requires equal head counts, sparse_triton_kernel.py:636-641).  k, v, dk,
 * dv have kv_heads heads and query head h reads key/value head
 * h / (H / kv_heads); dk, dv sum over each group's query heads.  kv_heads <= 0
 * means H.
 */

/* Forward: O = softmax(Q K^T * scale  masked) V, LSE = natural-log
 * log-sum-exp per row (0 for empty rows).  Replaces _fwd_kernel and its
 * launch in _BlockSparseFlashAttention.forward
 * (sparse_triton_kernel.py:231-352, 652-682).
 * row_ptr/col_idx: plan of pass 0 for this mask. */
int sbfa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
             int64_t B, int64_t H, int64_t n_q, int64_t n_kv, int64_t head_dim,
             int dtype, double softmax_scale, int is_causal, int64_t sink,
             int64_t window, const int32_t* block_mask, int64_t block_m,
             int64_t block_n, const int32_t* row_ptr, const int32_t* col_idx,
             const int64_t* strides, int64_t kv_heads, void* stream);

/* Backward: dQ, dK, dV (written, not accumulated) from Q, K, V, O, dO and
 * the forward's LSE.  Replaces _bwd_preprocess_kernel, _bwd_dkdv_kernel,
 * _bwd_dq_kernel and their launches (sparse_triton_kernel.py:355-601,
 * 694-779).  delta_ws: caller scratch, fp32[B*H*n_q].
 * dq_row_ptr/dq_col_idx: plan of pass 1; kv_col_ptr/kv_row_idx: plan of
 * pass 2 (may be the same plan when the tiles agree).
 * split_ws: optional caller scratch (16-byte aligned) of
 * sbfa_bwd_workspace_bytes() bytes.  With grouped-query attention the first
 * key tile (the sinks) is seen by every query tile of every query head of a
 * group; given this scratch, its dK/dV work is split over one CTA per query
 * head and the fp32 partials are summed by a second kernel, instead of one
 * CTA streaming all of them.  NULL (or too small) keeps the single CTA;
 * results agree to rounding.
 * ds_ws: optional caller scratch (16-byte aligned) of
 * sbfa_bwd_ds_workspace_bytes() bytes, with dq_csc_pos from
 * sbfa_plan_csc_positions() and nnz the plan's kept-tile count (the dQ and
 * dK/dV plans must then be the same plan).  Given it, the dK/dV pass also
 * stores every 16-bit dS tile there and dQ becomes a GEMM over the stored
 * tiles, instead of a third pass that recomputes S, P and dP; NULL keeps that
 * pass.  The two give the same dQ to rounding (the dS values are the dK/dV
 * pass's).  With the stored tiles and a large enough problem (64 or more
 * 128-row query tiles x B*H per SM) the dQ GEMM of one group of (b, h) units
 * runs on a library-owned high-priority side stream beside the next group's
 * dK/dV pass; the side stream belongs to `stream` (one per device and
 * caller stream), waits on it through events and is joined back into it
 * before the call returns, so work queued after the call, and a CUDA-graph
 * capture of `stream`, see one stream.  Results are bit-identical with and
 * without the overlap.  Environment: SBFA_BWD_GROUPS=n forces n groups (1
 * switches the overlap off), SBFA_DQ_GRID=n the dQ GEMM's CTA count while
 * it overlaps (default 3/8 of the SMs). */
int sbfa_bwd(const void* q, const void* k, const void* v, const void* o,
             const float* lse, const void* dout, void* dq, void* dk, void* dv,
             float* delta_ws, int64_t B, int64_t H, int64_t n_q, int64_t n_kv,
             int64_t head_dim, int dtype, double softmax_scale, int is_causal,
             int64_t sink, int64_t window, const int32_t* block_mask,
             int64_t block_m, int64_t block_n, const int32_t* dq_row_ptr,
             const int32_t* dq_col_idx, const int32_t* kv_col_ptr,
             const int32_t* kv_row_idx, const int64_t* strides, int64_t kv_heads,
             void* split_ws, int64_t split_ws_bytes, const int32_t* dq_csc_pos,
             int64_t nnz, void* ds_ws, int64_t ds_ws_bytes, void* stream);

/* Bytes of the stored dS tiles sbfa_bwd can use for this shape: B * H * nnz
 * tiles of 128 x 128 16-bit elements (nnz = kept 128 x 128 tiles of the
 * plan), or 0 where that path does not apply (dtype / head_dim other than
 * fp16 / bf16 with head_dim 128, or B * H * nnz >= 2^31).  No upstream
 * counterpart (upstream recomputes dS in its dQ kernel,
 * sparse_triton_kernel.py:512-601). */
int64_t sbfa_bwd_ds_workspace_bytes(int64_t B, int64_t H, int64_t head_dim, int dtype,
                                    int64_t nnz);

/* Scratch bytes of the split first key tile in sbfa_bwd (0 when nothing is
 * split: no grouping, or a dtype / head_dim the tensor-core kernels do not
 * take).  No upstream counterpart (upstream has no grouped-query attention). */
int64_t sbfa_bwd_workspace_bytes(int64_t B, int64_t H, int64_t head_dim, int dtype,
                                 int64_t kv_heads);

/* Split-KV decode for n_q == 1 (the upstream path is _fwd_kernel with
 * N_Q = 1, BLOCK_M = 1: benchmark.py:799-804 -> sparse_triton_kernel.py:231).
 * Reads only the K/V rows the query can see.  row_ptr/col_idx: plan of
 * pass 3.  split_ws: caller scratch of sbfa_decode_workspace_bytes() bytes.
 * lse may be NULL.  q, o: contiguous [B, H, 1, D]; k, v: contiguous
 * [B, kv_heads, n_kv, D] (kv_heads <= 0 means H).  With kv_heads < H a CTA
 * serves several query heads of one K/V head, so each K/V row is read once
 * per 16 query heads of its group (fp16/bf16 with head_dim 64 or 128, on the
 * tensor cores) or per 4 (other dtypes and head dims). */
int sbfa_decode(const void* q, const void* k, const void* v, void* o, float* lse,
                int64_t B, int64_t H, int64_t n_kv, int64_t head_dim, int dtype,
                double softmax_scale, int is_causal, int64_t sink, int64_t window,
                const int32_t* block_mask, int64_t block_m, int64_t block_n,
                const int32_t* row_ptr, const int32_t* col_idx, void* split_ws,
                int64_t split_ws_bytes, int64_t kv_heads, void* stream);

/* Scratch bytes sbfa_decode needs for this shape (any kv_heads). */
int64_t sbfa_decode_workspace_bytes(int64_t B, int64_t H, int64_t n_kv,
                                    int64_t head_dim, int64_t block_n);

/* 1 if sbfa_decode has a kernel for (dtype, head_dim), else 0 (callers then
 * run sbfa_fwd with n_q == 1, as upstream does). */
int sbfa_decode_supported(int dtype, int64_t head_dim);

/* ---------------------------------------------------------------------------
 * StreamingLLM ring-buffer KV cache (no upstream counterpart: upstream keeps
 * the whole cache and decodes through _fwd_kernel with N_Q = 1,
 * benchmark.py:799-804).  The query at position p sees positions [0, sink)
 * and (p - window, p], so a cache needs only sink + window rows per
 * (batch, head): K and V caches are contiguous [B, H, sink + window, D];
 * row r < sink holds position r, and position p >= sink lives in row
 * sink + (p - sink) % window.  Same results as sbfa_decode over a full cache
 * under the streaming rule (block mask with block_m = 1, causal), at
 * (sink + window) / n_kv of its memory.
 * ------------------------------------------------------------------------- */

/* Writes K/V of positions [pos0, pos0 + n_new) (k_new, v_new: contiguous
 * [B, H, n_new, D]) into their ring rows; positions that a later token of the
 * same call would overwrite are skipped.  Positions must be appended in
 * order across calls (pos0 = tokens already cached). */
int sbfa_ring_append(void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                     int64_t B, int64_t H, int64_t head_dim, int dtype, int64_t sink,
                     int64_t window, int64_t pos0, int64_t n_new, void* stream);

/* Split-KV decode of the query at position seq_len - 1 (q, o: contiguous
 * [B, H, 1, D]; lse may be NULL) over a ring cache holding positions
 * [0, seq_len).  split_ws: caller scratch of
 * sbfa_ring_decode_workspace_bytes() bytes (may be NULL when that is 0). */
int sbfa_ring_decode(const void* q, const void* k_cache, const void* v_cache, void* o,
                     float* lse, int64_t B, int64_t H, int64_t head_dim, int dtype,
                     double softmax_scale, int64_t sink, int64_t window, int64_t seq_len,
                     void* split_ws, int64_t split_ws_bytes, void* stream);

/* Scratch bytes sbfa_ring_decode needs for this cache geometry (any seq_len). */
int64_t sbfa_ring_decode_workspace_bytes(int64_t B, int64_t H, int64_t head_dim, int64_t sink,
                                         int64_t window);

/* sbfa_decode without any device allocation by anyone.  No counterpart in
 * the upstream project, which has no decode entry point at all.
 *
 * For callers that cannot allocate device memory around a decode step: a
 * serving loop that reserved all of its memory up front, or runs the step
 * under a fixed budget, and so may not call cudaMalloc (or grow a caching
 * allocator) per token; a host embedding libsbfa through a plain C FFI with
 * no device allocator of its own.  They pass only Q, K, V, the outputs and
 * the block mask (same meaning as sbfa_decode); the decode plan and the
 * split-KV partials live in an 8 MiB array inside the library, present on
 * every GPU that loads it until the process exits.
 *  - Shapes whose plan plus partials exceed 8 MiB are rejected with
 *    SBFA_ERR_INVALID before any launch; use sbfa_decode for those.
 *  - The first call on each device resolves that device's copy of the
 *    array (cudaGetSymbolAddress); make that first call before capturing
 *    the stream into a graph.
 *  - All calls on a device share the one array and it keeps the last call's
 *    contents (each call rewrites what it reads first); calls that can run
 *    at the same time on the GPU (different streams, or graphs replayed
 *    concurrently) race on it and must be serialised by the caller. */
int sbfa_decode_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                        int64_t B, int64_t H, int64_t n_kv, int64_t head_dim, int dtype,
                        double softmax_scale, int is_causal, int64_t sink, int64_t window,
                        const int32_t* block_mask, int64_t block_m, int64_t block_n,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SBFA_H_ */
