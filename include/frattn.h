/*
 * frattn.h — C ABI of the B200 (sm_100a) fused 2D-RoPE + varlen attention
 * forward kernel.
 *
 * Everything here takes plain device pointers, sizes and a CUDA stream handle
 * passed as `void*` (a cudaStream_t / CUstream); no framework types cross the
 * boundary. All entry points return 0 on success, a negative FRATTN_E* code for
 * an invalid argument (nothing was launched), or a positive code for a launch or
 * driver failure.
 *
 * Reference interface replaced (sdan/fused-rope-attn):
 *   fused_attn.py:139-232  fused_rope_attention(q, k, v, cos, sin, cu_seqlens, *, out)
 *                          -> frattn_fwd
 *   fused_attn.py:33-136   compute_rope_2d(...) (cos/sin from (h, w) grid ids)
 *                          -> frattn_fwd_pos takes the (h, w) ids directly
 *   fused_attn.py:246-423  fused_attn_kernel (Triton) -> the sm_100a kernels
 *                          launched by frattn_fwd / frattn_fwd_pos
 */
#ifndef FRATTN_H_
#define FRATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (values of the *_dtype arguments). */
enum {
  FRATTN_F32 = 0,
  FRATTN_F16 = 1,
  FRATTN_BF16 = 2
};

/* Return codes. */
enum {
  FRATTN_OK = 0,
  FRATTN_E_SHAPE = -1,     /* bad T / H / D / nseg                          */
  FRATTN_E_DTYPE = -2,     /* unsupported q/k/v or cos/sin element type     */
  FRATTN_E_ALIGN = -3,     /* a pointer is not 16-byte aligned              */
  FRATTN_E_NULL = -4,      /* a required pointer is NULL                    */
  FRATTN_E_WORKSPACE = -5, /* workspace smaller than frattn_workspace_bytes */
  FRATTN_E_NOALLOC_LIMIT = -6, /* T above FRATTN_NOALLOC_MAX_TOKENS (frattn_fwd_noalloc) */
  FRATTN_E_CUDA = 1,       /* CUDA runtime / driver error at launch         */
  FRATTN_E_TMAP = 2        /* cuTensorMapEncodeTiled rejected a descriptor  */
};

/* Device status word codes (written by the kernels into *status, first error
 * wins; read it back after the stream has synchronised). */
enum {
  FRATTN_STATUS_OK = 0,
  FRATTN_STATUS_WAIT_TIMEOUT = 0x100, /* | role << 4 | barrier group        */
  FRATTN_STATUS_BAD_SEQLENS = 0x200,  /* cu_seqlens not non-decreasing in [0,T] */
  FRATTN_STATUS_BAD_POSITIONS = 0x400 /* a pos_hw value outside [0, max_position) */
};

/* Library version (major * 10000 + minor * 100 + patch). */
int frattn_version(void);

/* Human-readable text for a return code or a device status code. */
const char* frattn_error_string(int code);

/* Bytes of device workspace frattn_fwd / frattn_fwd_pos need for `total_tokens`
 * packed tokens split into `num_segments` cu_seqlens segments. The workspace
 * holds the work list the on-device scheduler builds from cu_seqlens on every
 * call (no host synchronisation). Replaces the reference's host-side
 * `window_lens.max().item()` and grid computation (fused_attn.py:209-218). */
int frattn_workspace_bytes(int total_tokens, int num_segments, size_t* bytes);

/* Extra workspace bytes that enable the rotated-K path for long segments:
 * pass workspace_bytes >= frattn_workspace_bytes(...) (or _pos) + this value
 * and the K rows of segments longer than 128 tokens are rotated once per call
 * into the workspace by a short pre-pass, instead of once per 128-row q tile
 * inside the attention kernel. Short segments (windows) always rotate K in the
 * attention kernel. A workspace of only the base size is valid and keeps every
 * rotation inside the attention kernel. No counterpart in the reference (its
 * kernel re-rotates K for every q block, fused_attn.py:365-390). */
int frattn_workspace_bytes_rotated_k(int total_tokens, int num_heads, int head_dim, size_t* bytes);

/* Fused RoPE + varlen attention forward (fused_attn.py:139-232 semantics):
 *   for every segment s = [cu[s], cu[s+1]) and head h:
 *     O[s,h] = softmax(R(Q[s,h]) R(K[s,h])^T / sqrt(D)) V[s,h]
 *   with R the rotate-half rotary embedding using cos/sin rows of the token:
 *     x0' = x0 cos - x1 sin, x1' = x0 sin + x1 cos  (x0 = x[:D/2], x1 = x[D/2:]),
 *   computed in fp32 and rounded to the q/k/v element type before the product.
 *
 *   q, k, v, out : [T, H, D] contiguous, element type in_dtype (F16 or BF16)
 *   cos, sin     : [T, D/2] contiguous, element type cs_dtype (F32, F16, BF16)
 *   cu_seqlens   : [nseg + 1] int32, non-decreasing, values in [0, T]
 *   max_seqlen   : optional hint (<= 0: unknown). A value <= 128 skips the K
 *                  pre-rotation pass (no segment is long); results do not depend on it
 *   workspace    : >= frattn_workspace_bytes(T, nseg) bytes of device memory
 *   status       : device int32 (may be NULL); set non-zero on a device error
 *   stream       : cudaStream_t the kernels are launched on
 * Rows of `out` outside [cu[0], cu[nseg]) are written with zeros (this makes an
 * all-empty cu_seqlens return zeros, matching fused_attn.py:212-213).
 * Supported D: every multiple of 8 in [32, 128]. A D that is not a multiple of
 * 16 runs on tiles rounded up to the next multiple of 16; TMA fills the extra
 * columns with zeros, so they add nothing to QK^T and are never stored. (The
 * Python wrapper reaches any other even D up to 128 by zero-padding each
 * rotate-half half; this ABI takes the kernel dims only.)
 */
int frattn_fwd(const void* q, const void* k, const void* v, const void* cos, const void* sin,
               int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
               int max_seqlen, int in_dtype, void* out, void* workspace, size_t workspace_bytes,
               int32_t* status, void* stream);

/* frattn_fwd for q, k, v whose token rows are spread out: element (t, h, d)
 * of q is q[t * q_stride + h * D + d] (likewise k, v), e.g. the three views
 * of one fused [T, 3, H, D] QKV projection output (strides 3 H D). Strides are
 * in elements, at least H * D and multiples of 8 (16-byte row starts, a TMA
 * requirement; FRATTN_E_ALIGN otherwise). The reference copies such inputs to
 * contiguous tensors first (fused_attn.py:187-193); here the tensor maps read
 * them in place. out stays contiguous [T, H, D]. */
int frattn_fwd_strided(const void* q, const void* k, const void* v, long long q_stride,
                       long long k_stride, long long v_stride, const void* cos, const void* sin,
                       int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
                       int max_seqlen, int in_dtype, void* out, void* workspace,
                       size_t workspace_bytes, int32_t* status, void* stream);

/* Same operation with the 2D rotary angles generated in the kernel from integer
 * (h, w) patch positions instead of materialised cos/sin tables
 * (compute_rope_2d, fused_attn.py:77-116, without the dtype cast):
 *   inv_freq[i] = theta^(-2i / (D/2)),  i < D/4
 *   angle[t, i]        = pos_hw[t, 0] * inv_freq[i]   (i < D/4)
 *   angle[t, D/4 + i]  = pos_hw[t, 1] * inv_freq[i]
 *   pos_hw : [T, 2] int32, 0 <= value < max_position (max_position <= 65536).
 * The per-position cos/sin table (max_position rows) lives in the workspace, so
 * this entry point needs frattn_workspace_bytes_pos(...) bytes instead. The
 * scheduler kernel checks every position against the table; on a value outside
 * it nothing is computed and *status is set to FRATTN_STATUS_BAD_POSITIONS. */
int frattn_workspace_bytes_pos(int total_tokens, int num_segments, int max_position, int D,
                               size_t* bytes);
int frattn_fwd_pos(const void* q, const void* k, const void* v, const int32_t* pos_hw,
                   int max_position, float theta, const int32_t* cu_seqlens, int nseg, int T,
                   int H, int D, int max_seqlen, int in_dtype, void* out, void* workspace,
                   size_t workspace_bytes, int32_t* status, void* stream);

/* ---- Rotation in the QKV projection (the reference's caller rotates q/k in
 * a separate elementwise pass after the projection, bench.py:72-78, or the
 * fused kernel rotates them per q block, fused_attn.py:340-345, 385-390).
 *
 * frattn_qkv_rope: qkv = x W^T + bias on the tensor cores (tcgen05, fp32
 * accumulation in TMEM) with the rotary embedding applied in the epilogue:
 *   x    : [T, K] rows of x_stride elements (0: K), element type in_dtype
 *   w    : [3 H D, K] contiguous (nn.Linear weight layout, q rows, then k, then v)
 *   bias : [3 H D] or NULL
 *   cos, sin : [T, D/2] (cs_dtype F32 / F16 / BF16), rows of token t
 *   qkv  : [T, 3, H, D] contiguous output; q and k heads rotated, v as projected
 * Each output value is acc + bias rounded to in_dtype; q/k values are then
 * rotated in fp32 and rounded once more (what frattn_fwd does to a stored q/k).
 * D a multiple of 16 in [32, 128]; K and x_stride multiples of 8.
 *
 * frattn_fwd_rotated: frattn_fwd_strided for q and k that are already rotated
 * (e.g. the q/k views of frattn_qkv_rope's output, strides 3 H D; 0 means
 * contiguous): no tables are read and no rotation runs. Workspace as frattn_fwd.
 */
int frattn_qkv_rope(const void* x, long long x_stride, const void* w, const void* bias,
                    const void* cos, const void* sin, int cs_dtype, int T, int K, int H, int D,
                    int in_dtype, void* qkv, int32_t* status, void* stream);
/* Kernel choice of frattn_qkv_rope (no counterpart in the reference): enable != 0
 * (default) runs the GEMM on CTA pairs (tcgen05 cta_group::2, one M = 256 MMA over
 * two SMs, each loading half of the weight tile), 0 on single CTAs (M = 128).
 * Both give the same values (same accumulation order per output element). */
int frattn_qkv_rope_set_pairs(int enable);
int frattn_fwd_rotated(const void* q, const void* k, const void* v, long long q_stride,
                       long long k_stride, long long v_stride, const int32_t* cu_seqlens, int nseg,
                       int T, int H, int D, int max_seqlen, int in_dtype, void* out,
                       void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* ---- Training (the reference is forward-only, fused_attn.py:246-423).
 *
 * frattn_fwd_lse: frattn_fwd that also writes lse [T, H] fp32, the base-2
 * log-sum-exp of the scaled scores of each row and head
 * (log2 sum_j 2^(s_ij log2(e) / sqrt(D)), s = R(q) R(k)^T); the backward pass
 * recomputes the softmax from it. Values of rows outside every segment are
 * unspecified.
 *
 * frattn_bwd: gradients of out = frattn_fwd(q, k, v, cos, sin, cu_seqlens) with
 * respect to q, k and v, given dout [T, H, D], the forward's out and lse:
 *   dv = P^T dout, dS = P o (dout v^T - rowsum(dout o out)),
 *   dq = R^T(dS R(k)) / sqrt(D), dk = R^T(dS^T R(q)) / sqrt(D),
 * P = softmax(R(q) R(k)^T / sqrt(D)) per segment and head, R^T the inverse
 * rotation. cos/sin are constants (no gradient). Rows outside every segment
 * get zero gradients. All tensors contiguous [T, H, D] (cos/sin [T, D/2]);
 * D a multiple of 16 in [32, 128]; workspace >= frattn_workspace_bytes_bwd(T, H, D)
 * bytes (rotated q and k, the row terms and an fp32 dq accumulator). */
int frattn_fwd_lse(const void* q, const void* k, const void* v, const void* cos, const void* sin,
                   int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
                   int max_seqlen, int in_dtype, void* out, float* lse, void* workspace,
                   size_t workspace_bytes, int32_t* status, void* stream);
int frattn_workspace_bytes_bwd(int total_tokens, int num_heads, int head_dim, size_t* bytes);
int frattn_bwd(const void* q, const void* k, const void* v, const void* cos, const void* sin,
               int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D, int in_dtype,
               const void* out, const void* dout, const float* lse, void* dq, void* dk, void* dv,
               void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* ---- FP8 (e4m3) q / k for long segments (the reference computes QK^T in
 * the input type, fused_attn.py:394).
 *
 * frattn_fwd_fp8: the frattn_fwd operation with S = R(q) R(k)^T on the FP8
 * tensor cores (tcgen05 kind::f8f6f4). A pre-pass rotates q and k in fp32 and
 * rounds them to e4m3 with one scale per (token, head) row of q and one per head
 * of k (scale = max |value| / 448); the scales are folded into the softmax
 * exponent. P V stays in the input type. Same arguments as frattn_fwd; the
 * workspace must hold frattn_workspace_bytes_fp8(T, nseg, H, D) bytes (the
 * work list, the e4m3 copies of q and k and the scales) and be 256-byte
 * aligned. D a multiple of 16 in [32, 128]. Accuracy: e4m3 keeps 3 mantissa bits, so scores carry about 2^-5
 * relative error per product; on N(0, 1) inputs the output stays within
 * max-abs 2e-2 / mean-abs 2e-3 of the fp32 path for long segments. Intended for
 * long segments (all segments take the work-list path; windows gain nothing). */
int frattn_workspace_bytes_fp8(int total_tokens, int num_segments, int num_heads, int head_dim,
                               size_t* bytes);
int frattn_fwd_fp8(const void* q, const void* k, const void* v, const void* cos, const void* sin,
                   int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
                   int max_seqlen, int in_dtype, void* out, void* workspace, size_t workspace_bytes,
                   int32_t* status, void* stream);

/* Allocation-free variant of frattn_fwd (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory at the point of the call: a
 * host runtime whose allocator is owned by someone else (a plugin inside another
 * framework with no access to its caching allocator), code running where
 * cudaMalloc would synchronise the device or is forbidden (latency-critical
 * serving loops, some embedded/FFI hosts), or bindings that only see raw
 * pointers. The work list that frattn_fwd keeps in the caller's workspace lives
 * instead in one fixed device array inside this library
 * (FRATTN_NOALLOC_SCRATCH_BYTES per GPU, held until the process exits), so the
 * caller passes only inputs, outputs and a stream. Nothing is allocated: no
 * cudaMalloc / cudaFree and no allocating library routine.
 *
 * Limits and rules:
 *   - T (total_tokens) <= FRATTN_NOALLOC_MAX_TOKENS, else FRATTN_E_NOALLOC_LIMIT;
 *   - the first call on a device looks up the array's device address (once,
 *     with that device current) and caches it; make that first call before any
 *     stream capture. A cudaDeviceReset destroys the array with the context,
 *     and the cached address then no longer names it: do not call this entry
 *     point on a device after resetting it;
 *   - all rotation runs inside the attention kernel (the array never holds a
 *     rotated-K copy); for long segments this is slower than frattn_fwd with a
 *     rotated-K workspace;
 *   - every call on a device shares the one array: calls whose kernels overlap
 *     on the GPU (e.g. on two streams without ordering) race and may produce
 *     wrong output. Order such calls on one stream or use frattn_fwd.
 * Arguments and results are otherwise those of frattn_fwd. */
#define FRATTN_NOALLOC_MAX_TOKENS 65536
#define FRATTN_NOALLOC_SCRATCH_BYTES 65536
int frattn_fwd_noalloc(const void* q, const void* k, const void* v, const void* cos,
                       const void* sin, int cs_dtype, const int32_t* cu_seqlens, int nseg, int T,
                       int H, int D, int max_seqlen, int in_dtype, void* out, int32_t* status,
                       void* stream);

/* ---- Window plan on the device (no host-side index arithmetic, no large
 * host->device copies). Replaces the host producers of the kernel's inputs:
 *   utils.py:12-102        get_window_index(grid_thw, window_size, merge, patch)
 *   utils.py:105-153       window_shuffle / window_unshuffle
 *   fused_attn.py:125-134  compute_rope_2d(..., window_idx=...) window-ordered tables
 * grid_thw is a HOST array [num_images][3] of (t, h, w) patch counts (h, w
 * divisible by merge). Windows are window_size / merge / patch_size merge units
 * on a side, visited row-major per frame, units row-major inside a window, edge
 * windows truncated (the reference's order; no window is ever empty).
 *
 * frattn_window_plan_sizes: number of merge units U (= T / merge^2), windows W
 * and the device workspace the plan needs.
 * frattn_window_plan writes (device pointers, stream-ordered):
 *   window_index [U] int64  source merge unit of each window-order slot
 *   cu_seqlens   [W + 1] int32 token offsets of the windows
 *   pos_hw       [T, 2] int32 (h, w) patch position of each token in window
 *                order, or NULL (input of frattn_fwd_pos)
 *   cos_table, sin_table [T, rotary_dim] fp32 in window order, or both NULL:
 *                index i < rotary_dim/2 uses h, the rest w, with
 *                inv_freq[i] = theta^(-2i / rotary_dim) (rotary_dim = head_dim / 2)
 * frattn_window_shuffle: rows of row_bytes (multiple of 16) bytes;
 *   inverse = 0: out[p m2 + j] = x[window_index[p] m2 + j] (into window order),
 *   inverse = 1: out[window_index[p] m2 + j] = x[p m2 + j] (back), m2 = merge^2.
 *   x and out must not overlap. */
int frattn_window_plan_sizes(const int32_t* grid_thw, int num_images, int window_size, int merge,
                             int patch_size, int64_t* units, int64_t* windows,
                             size_t* workspace_bytes);
int frattn_window_plan(const int32_t* grid_thw, int num_images, int window_size, int merge,
                       int patch_size, int64_t* window_index, int32_t* cu_seqlens, int32_t* pos_hw,
                       float* cos_table, float* sin_table, int rotary_dim, float theta,
                       void* workspace, size_t workspace_bytes, void* stream);
int frattn_window_shuffle(const void* x, const int64_t* window_index, int64_t units, int merge_unit,
                          int64_t row_bytes, int inverse, void* out, void* stream);

/* Test hook for the bounded-wait failure path: launches one CTA that waits on
 * an mbarrier nothing ever arrives on, with a `limit_ns` bound, and returns
 * through *status (FRATTN_STATUS_WAIT_TIMEOUT | ...) without faulting or
 * hanging the GPU. No counterpart in the reference (which has no failure
 * detection). */
int frattn_selftest_wait_timeout(int32_t* status, uint64_t limit_ns, void* stream);

/* Measurement hook (no counterpart in the reference): the next frattn_fwd /
 * frattn_fwd_strided / frattn_fwd_pos call from this host thread records the
 * two CUDA events (cudaEvent_t) on its stream around its attention kernels
 * (the K pre-rotation and the attention kernel, or the window kernel), not
 * around the work-list kernel. Recorded during stream capture they become
 * event nodes of the graph. The events are forgotten after that call. */
int frattn_set_timing_events(void* start_event, void* stop_event);

/* Upper bound (nanoseconds) of every mbarrier wait inside the kernels;
 * default 2e9. A wait that exceeds it sets *status and the kernel returns. */
int frattn_set_wait_limit_ns(uint64_t limit_ns);

#ifdef __cplusplus
}
#endif
#endif /* FRATTN_H_ */
