// Host side of the C ABI (include/frattn.h): argument checks, workspace layout,
// TMA tensor maps and the launches of the kernels in frattn_kernel.cuh. The
// kernels of each supported head dimension live in their own object
// (frattn_inst.cu compiled with -DFRATTN_D=<D>); this file picks one by D.
#include "frattn_kernel.cuh"

// Head dimensions with compiled kernels: multiples of 8 in [32, 128].
#define FRATTN_HEAD_DIMS(X) \
  X(32) X(40) X(48) X(56) X(64) X(72) X(80) X(88) X(96) X(104) X(112) X(120) X(128)

namespace frattn {

#define FRATTN_DECL(DD)                                                                       \
  int attn_d##DD(const Params& prm, int mode, int in_dtype, int cs_dtype, cudaStream_t st);   \
  int window_d##DD(const Params& prm, int in_dtype, int cs_dtype, bool rotated, cudaStream_t st); \
  int prep_d##DD(const int32_t* cu, int nseg, int T, int H, WorkItem* items, int* header,     \
                 void* out, int32_t* status, const int32_t* pos_hw, float* pos_tab,           \
                 int pos_rows, float theta, int in_dtype, cudaStream_t st);
#ifdef FRATTN_FAST_BUILD
FRATTN_DECL(80)
#else
FRATTN_HEAD_DIMS(FRATTN_DECL)
#endif
#undef FRATTN_DECL

// Failure-path self test: wait on a barrier nothing arrives on.
__global__ void wait_timeout_kernel(int32_t* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t b;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&b), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  Params p;
  memset(&p, 0, sizeof(p));
  p.status = status;
  p.wait_limit_ns = limit_ns;
  bounded_wait(smem_u32(&b), 0, p, &abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0xF0);
}

}  // namespace frattn

// ====================================================================== host
using namespace frattn;

namespace {

using PFN_encodeTiled = TmapEncodeFn;
PFN_encodeTiled get_encode_fn() { return tmap_encoder(); }

unsigned long long g_wait_limit_ns = 2000000000ull;

// Events recorded around the attention kernel of the next call on this host
// thread (frattn_set_timing_events); cleared by that call.
thread_local cudaEvent_t g_ev_start = nullptr, g_ev_stop = nullptr;

// (external records: during stream capture they become event-record nodes
// whose timestamps the host can read after a replay)
// (outside a capture the external flag is not accepted: plain records there)
void timing_record(cudaEvent_t ev, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, st);
}
void timing_begin(cudaStream_t st) {
  if (g_ev_start) timing_record(g_ev_start, st);
}
void timing_end(cudaStream_t st) {
  if (g_ev_stop) timing_record(g_ev_stop, st);
  g_ev_start = g_ev_stop = nullptr;
}

// [T, H, D] tensor viewed as 3-D {D, H, T}; box {16, 1, 128}, 32-B swizzle.
int make_qkv_map(CUtensorMap* m, const void* base, int T, int H, int D, bool bf16,
                 long long row_stride) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return FRATTN_E_TMAP;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(T)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(row_stride) * 2};
  cuuint32_t box[3] = {16, 1, static_cast<cuuint32_t>(kTileM)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FRATTN_E_TMAP;
}

// [T, D/2] cos or sin table; box {D/2, 128}, no swizzle.
int make_cs_map(CUtensorMap* m, const void* base, int T, int D, int cs_dtype) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return FRATTN_E_TMAP;
  const int esz = cs_dtype == FRATTN_F32 ? 4 : 2;
  const CUtensorMapDataType dt = cs_dtype == FRATTN_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : cs_dtype == FRATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D / 2), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(D / 2) * esz};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(D / 2), static_cast<cuuint32_t>(kTileM)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FRATTN_E_TMAP;
}

// [T, H, D16] e4m3 rows (D16 bytes per head, zero-padded) viewed as 3-D {D16, H, T};
// box {32, 1, 128} (32 e4m3 = 32 bytes per column block), 32-B swizzle.
int make_fp8_map(CUtensorMap* m, const void* base, int T, int H, int D16) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return FRATTN_E_TMAP;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D16), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D16), static_cast<cuuint64_t>(H) * D16};
  cuuint32_t box[3] = {32, 1, static_cast<cuuint32_t>(kTileM)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FRATTN_E_TMAP;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Attention kernels of head dimension D.
int dispatch_head_dim(const Params& prm, int mode, int D, int in_dtype, int cs_dtype,
                      cudaStream_t st) {
  switch (D) {
#define FRATTN_CASE(DD) \
    case DD: return attn_d##DD(prm, mode, in_dtype, cs_dtype, st);
#ifdef FRATTN_FAST_BUILD
    FRATTN_CASE(80)
#else
    FRATTN_HEAD_DIMS(FRATTN_CASE)
#endif
#undef FRATTN_CASE
    default: return FRATTN_E_SHAPE;
  }
}

// Window kernel of head dimension D (FRATTN_E_SHAPE: none for this D / type).
int dispatch_window(const Params& prm, int D, int in_dtype, int cs_dtype, bool rotated,
                    cudaStream_t st) {
  switch (D) {
#define FRATTN_CASE(DD) \
    case DD: return window_d##DD(prm, in_dtype, cs_dtype, rotated, st);
#ifdef FRATTN_FAST_BUILD
    FRATTN_CASE(80)
#else
    FRATTN_HEAD_DIMS(FRATTN_CASE)
#endif
#undef FRATTN_CASE
    default: return FRATTN_E_SHAPE;
  }
}

// Work-list kernel of head dimension D.
int launch_prep(const int32_t* cu, int nseg, int T, int H, int D, WorkItem* items, int* header,
                void* out, int32_t* status, const int32_t* pos_hw, float* pos_tab, int pos_rows,
                float theta, int in_dtype, cudaStream_t st) {
  switch (D) {
#define FRATTN_CASE(DD)                                                                       \
    case DD:                                                                                  \
      return prep_d##DD(cu, nseg, T, H, items, header, out, status, pos_hw, pos_tab, pos_rows, \
                        theta, in_dtype, st);
#ifdef FRATTN_FAST_BUILD
    FRATTN_CASE(80)
#else
    FRATTN_HEAD_DIMS(FRATTN_CASE)
#endif
#undef FRATTN_CASE
    default: return FRATTN_E_SHAPE;
  }
}

bool supported_head_dim(int D) {
#ifdef FRATTN_FAST_BUILD
  return D == 80;
#else
  return D % 8 == 0 && D >= 32 && D <= 128;
#endif
}

size_t pos_table_bytes(int max_position, int D) {
  return (static_cast<size_t>(max_position) * (D / 4) * 2 * sizeof(float) + 255) & ~size_t(255);
}

int common_checks(const void* q, const void* k, const void* v, const int32_t* cu, int nseg, int T,
                  int H, int D, int in_dtype, void* out, void* ws) {
  if (!q || !k || !v || !cu || !out || !ws) return FRATTN_E_NULL;
  if (T < 0 || H <= 0 || nseg < 1) return FRATTN_E_SHAPE;
  if (!supported_head_dim(D)) return FRATTN_E_SHAPE;
  if (in_dtype != FRATTN_BF16 && in_dtype != FRATTN_F16) return FRATTN_E_DTYPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(ws))
    return FRATTN_E_ALIGN;
  if (static_cast<long long>(T) * H * D >= (1ll << 31)) return FRATTN_E_SHAPE;
  return 0;
}

template <int MODE>
int fwd_impl(const void* q, const void* k, const void* v, const void* cos, const void* sin,
             int cs_dtype, const int32_t* pos_hw, int max_position, float theta,
             const int32_t* cu, int nseg, int T, int H, int D, int in_dtype, void* out,
             void* workspace, size_t ws_bytes, int32_t* status, void* stream,
             int max_seqlen = 0, long long q_stride = 0, long long k_stride = 0,
             long long v_stride = 0, float* lse = nullptr, const float* qscale = nullptr,
             const float* kscale = nullptr) {
  int rc = common_checks(q, k, v, cu, nseg, T, H, D, in_dtype, out, workspace);
  if (rc) return rc;
  // token strides of q, k, v in elements (0: contiguous [T, H, D]); TMA needs
  // every row start 16-byte aligned
  const long long hd = static_cast<long long>(H) * D;
  if (q_stride == 0) q_stride = hd;
  if (k_stride == 0) k_stride = hd;
  if (v_stride == 0) v_stride = hd;
  if (MODE != kRopeFp8) {  // (FP8: q_stride / k_stride carry the padded e4m3 head width)
    if (q_stride < hd || k_stride < hd || v_stride < hd) return FRATTN_E_SHAPE;
    if ((q_stride | k_stride | v_stride) & 7) return FRATTN_E_ALIGN;
  }
  size_t need = 0;
  if (MODE == kRopeTable) {
    frattn_workspace_bytes(T, nseg, &need);
    if (!cos || !sin) return FRATTN_E_NULL;
    if (cs_dtype != FRATTN_F32 && cs_dtype != FRATTN_F16 && cs_dtype != FRATTN_BF16)
      return FRATTN_E_DTYPE;
    if (!aligned16(cos) || !aligned16(sin)) return FRATTN_E_ALIGN;
  } else if (MODE == kRopeNone || MODE == kRopeFp8) {
    frattn_workspace_bytes(T, nseg, &need);
  } else {
    if (!pos_hw) return FRATTN_E_NULL;
    if (max_position <= 0 || max_position > 65536) return FRATTN_E_SHAPE;
    if (reinterpret_cast<uintptr_t>(pos_hw) & 7u) return FRATTN_E_ALIGN;
    frattn_workspace_bytes_pos(T, nseg, max_position, D, &need);
  }
  if (ws_bytes < need) return FRATTN_E_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* header = reinterpret_cast<int*>(ws);
  WorkItem* items = reinterpret_cast<WorkItem*>(ws + kHeaderBytes);
  float* pos_tab = nullptr;
  if (MODE == kRopePos) {
    size_t base = kHeaderBytes + max_items(T) * sizeof(WorkItem);
    base = (base + 255) & ~size_t(255);
    pos_tab = reinterpret_cast<float*>(ws + base);
  }
  if (T == 0)
    return launch_prep(cu, nseg, T, H, D, items, header, out, status, pos_hw, pos_tab,
                       max_position, theta, in_dtype, st);

  Params prm;
  memset(&prm, 0, sizeof(prm));
  const bool bf16 = in_dtype == FRATTN_BF16;
  if (MODE == kRopeFp8) {  // q, k: e4m3 rows of q_stride bytes per head (the padded head dim)
    if (make_fp8_map(&prm.tmq, q, T, H, static_cast<int>(q_stride)) ||
        make_fp8_map(&prm.tmk, k, T, H, static_cast<int>(k_stride)) ||
        make_qkv_map(&prm.tmv, v, T, H, D, bf16, v_stride))
      return FRATTN_E_TMAP;
  } else if (make_qkv_map(&prm.tmq, q, T, H, D, bf16, q_stride) ||
             make_qkv_map(&prm.tmk, k, T, H, D, bf16, k_stride) ||
             make_qkv_map(&prm.tmv, v, T, H, D, bf16, v_stride)) {
    return FRATTN_E_TMAP;
  }
  // Rotated-K buffer after the work list (and table) when the workspace has
  // room. A caller's max_seqlen <= one tile says no segment is long, so the
  // pre-rotation pass would find nothing to do and is not launched. The hint
  // only selects that path: long segments are still correct without it
  // (their K tiles are then rotated inside the attention kernel).
  const size_t krot_off = (need + 255) & ~size_t(255);
  const size_t krot_bytes = static_cast<size_t>(T) * H * D * 2;
  const bool no_long = max_seqlen > 0 && max_seqlen <= kTileM;
  if (MODE != kRopeNone && MODE != kRopeFp8 && ws_bytes >= krot_off + krot_bytes && !no_long) {
    prm.krot = ws + krot_off;
    if (make_qkv_map(&prm.tmk_rot, prm.krot, T, H, D, bf16, static_cast<long long>(H) * D))
      return FRATTN_E_TMAP;
  }
  // cos/sin rows are staged through TMA only when a row is a multiple of 16 bytes
  // (the kernel's Cfg::CS_BYTES makes the same decision).
  const int cs_esz = cs_dtype == FRATTN_F32 ? 4 : 2;
  if (MODE == kRopeTable && ((D / 2) * cs_esz) % 16 == 0 &&
      (make_cs_map(&prm.tmcos, cos, T, D, cs_dtype) || make_cs_map(&prm.tmsin, sin, T, D, cs_dtype)))
    return FRATTN_E_TMAP;
  prm.k = k;
  prm.k_stride = k_stride;
  prm.cos = cos;
  prm.sin = sin;
  prm.pos_hw = pos_hw;
  prm.pos_tab = pos_tab;
  prm.pos_rows = max_position;
  prm.cu = cu;
  prm.nseg = nseg;
  prm.out = out;
  prm.items = items;
  prm.header = header;
  prm.T = T;
  prm.H = H;
  prm.status = status;
  prm.wait_limit_ns = g_wait_limit_ns;
  prm.lse = lse;
  prm.qscale = qscale;
  prm.kscale = kscale;
  // Window regime (the caller says no segment exceeds one tile): one kernel,
  // no work list. Head dims / element types without a window kernel, and the
  // position entry point, take the general path below.
  if ((MODE == kRopeTable || MODE == kRopeNone) && no_long) {
    timing_begin(st);  // the window kernel is then the only launch of the call
    rc = dispatch_window(prm, D, in_dtype, cs_dtype, MODE == kRopeNone, st);
    if (rc != FRATTN_E_SHAPE) {
      timing_end(st);
      return rc;
    }
  }
  rc = launch_prep(cu, nseg, T, H, D, items, header, out, status, pos_hw, pos_tab, max_position,
                   theta, in_dtype, st);
  if (rc) return rc;
  timing_begin(st);  // around the K pre-rotation (if any) and the attention kernel
  rc = dispatch_head_dim(prm, MODE, D, in_dtype, cs_dtype, st);
  timing_end(st);
  return rc;
}

}  // namespace

namespace frattn {
// Bounded-wait limit shared by every kernel of the library (frattn_set_wait_limit_ns).
unsigned long long frattn_wait_limit_ns() { return g_wait_limit_ns; }

// Attention over q / k already rotated and quantised to e4m3 (frattn_fp8.cu):
// rows of D16 bytes per head, dequantisation scales per q row and per k head.
int attn_fp8_prequantized(const void* q8, const void* k8, const void* v, const float* qscale,
                          const float* kscale, int D16, const int32_t* cu, int nseg, int T, int H, int D,
                          int in_dtype, void* out, void* workspace, size_t ws_bytes, int32_t* status,
                          cudaStream_t st) {
  if (!qscale || !kscale) return FRATTN_E_NULL;
  return fwd_impl<kRopeFp8>(q8, k8, v, nullptr, nullptr, FRATTN_F32, nullptr, 0, 0.f, cu, nseg, T, H, D,
                            in_dtype, out, workspace, ws_bytes, status, st, 0, D16, D16, 0, nullptr, qscale,
                            kscale);
}
}  // namespace frattn

// ---------------------------------------------------------------- no-alloc variant
// Work-list storage for frattn_fwd_noalloc: a fixed device array that every GPU
// loading this library keeps until the process exits. It is large enough for
// FRATTN_NOALLOC_MAX_TOKENS packed tokens.
static __device__ __align__(256) uint8_t g_noalloc_scratch[FRATTN_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_scratch on the current device (the symbol's name
// in host code is only a host-side handle). Resolved once per device.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FRATTN_E_CUDA;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return FRATTN_E_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}
}  // namespace

extern "C" {

int frattn_version(void) { return 100; }

const char* frattn_error_string(int code) {
  switch (code) {
    case FRATTN_OK: return "ok";
    case FRATTN_E_SHAPE: return "invalid shape (T, H, D or nseg)";
    case FRATTN_E_DTYPE: return "unsupported element type";
    case FRATTN_E_ALIGN: return "pointer not 16-byte aligned";
    case FRATTN_E_NULL: return "required pointer is NULL";
    case FRATTN_E_WORKSPACE: return "workspace too small";
    case FRATTN_E_CUDA: return "CUDA launch error";
    case FRATTN_E_TMAP: return "tensor map encoding failed";
    case FRATTN_E_NOALLOC_LIMIT:
      return "total_tokens exceeds FRATTN_NOALLOC_MAX_TOKENS for frattn_fwd_noalloc";
    case FRATTN_STATUS_BAD_SEQLENS: return "cu_seqlens is not non-decreasing within [0, T]";
    case FRATTN_STATUS_BAD_POSITIONS: return "a pos_hw value is outside [0, max_position)";
    default:
      if ((code & 0xF00) == FRATTN_STATUS_WAIT_TIMEOUT) return "device wait timed out";
      return "unknown error";
  }
}

int frattn_workspace_bytes(int total_tokens, int num_segments, size_t* bytes) {
  if (!bytes) return FRATTN_E_NULL;
  if (total_tokens < 0 || num_segments < 1) return FRATTN_E_SHAPE;
  *bytes = kHeaderBytes + max_items(total_tokens) * sizeof(WorkItem);
  return 0;
}

int frattn_workspace_bytes_rotated_k(int total_tokens, int num_heads, int head_dim,
                                     size_t* bytes) {
  if (!bytes) return FRATTN_E_NULL;
  if (total_tokens < 0 || num_heads <= 0 || head_dim <= 0) return FRATTN_E_SHAPE;
  *bytes = 256 + static_cast<size_t>(total_tokens) * num_heads * head_dim * 2;
  return 0;
}

int frattn_workspace_bytes_pos(int total_tokens, int num_segments, int max_position, int D,
                               size_t* bytes) {
  if (!bytes) return FRATTN_E_NULL;
  if (total_tokens < 0 || num_segments < 1 || max_position <= 0 || max_position > 65536)
    return FRATTN_E_SHAPE;
  size_t base = kHeaderBytes + max_items(total_tokens) * sizeof(WorkItem);
  base = (base + 255) & ~size_t(255);
  *bytes = base + pos_table_bytes(max_position, D);
  return 0;
}

int frattn_fwd(const void* q, const void* k, const void* v, const void* cos, const void* sin,
               int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
               int max_seqlen, int in_dtype, void* out, void* workspace, size_t workspace_bytes,
               int32_t* status, void* stream) {
  return fwd_impl<kRopeTable>(q, k, v, cos, sin, cs_dtype, nullptr, 0, 0.f, cu_seqlens, nseg, T,
                              H, D, in_dtype, out, workspace, workspace_bytes, status, stream,
                              max_seqlen);
}

int frattn_fwd_strided(const void* q, const void* k, const void* v, long long q_stride,
                       long long k_stride, long long v_stride, const void* cos, const void* sin,
                       int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
                       int max_seqlen, int in_dtype, void* out, void* workspace,
                       size_t workspace_bytes, int32_t* status, void* stream) {
  if (q_stride <= 0 || k_stride <= 0 || v_stride <= 0) return FRATTN_E_SHAPE;
  return fwd_impl<kRopeTable>(q, k, v, cos, sin, cs_dtype, nullptr, 0, 0.f, cu_seqlens, nseg, T,
                              H, D, in_dtype, out, workspace, workspace_bytes, status, stream,
                              max_seqlen, q_stride, k_stride, v_stride);
}

int frattn_fwd_pos(const void* q, const void* k, const void* v, const int32_t* pos_hw,
                   int max_position, float theta, const int32_t* cu_seqlens, int nseg, int T,
                   int H, int D, int max_seqlen, int in_dtype, void* out, void* workspace,
                   size_t workspace_bytes, int32_t* status, void* stream) {
  return fwd_impl<kRopePos>(q, k, v, nullptr, nullptr, FRATTN_F32, pos_hw, max_position, theta,
                            cu_seqlens, nseg, T, H, D, in_dtype, out, workspace, workspace_bytes,
                            status, stream, max_seqlen);
}

int frattn_fwd_lse(const void* q, const void* k, const void* v, const void* cos, const void* sin,
                   int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
                   int max_seqlen, int in_dtype, void* out, float* lse, void* workspace,
                   size_t workspace_bytes, int32_t* status, void* stream) {
  if (!lse) return FRATTN_E_NULL;
  if (reinterpret_cast<uintptr_t>(lse) & 3u) return FRATTN_E_ALIGN;
  return fwd_impl<kRopeTable>(q, k, v, cos, sin, cs_dtype, nullptr, 0, 0.f, cu_seqlens, nseg, T,
                              H, D, in_dtype, out, workspace, workspace_bytes, status, stream,
                              max_seqlen, 0, 0, 0, lse);
}

int frattn_fwd_rotated(const void* q, const void* k, const void* v, long long q_stride,
                       long long k_stride, long long v_stride, const int32_t* cu_seqlens, int nseg,
                       int T, int H, int D, int max_seqlen, int in_dtype, void* out,
                       void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (q_stride < 0 || k_stride < 0 || v_stride < 0) return FRATTN_E_SHAPE;
  return fwd_impl<kRopeNone>(q, k, v, nullptr, nullptr, FRATTN_F32, nullptr, 0, 0.f, cu_seqlens,
                             nseg, T, H, D, in_dtype, out, workspace, workspace_bytes, status,
                             stream, max_seqlen, q_stride, k_stride, v_stride);
}

int frattn_selftest_wait_timeout(int32_t* status, uint64_t limit_ns, void* stream) {
  if (!status) return FRATTN_E_NULL;
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_ns);
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

int frattn_fwd_noalloc(const void* q, const void* k, const void* v, const void* cos,
                       const void* sin, int cs_dtype, const int32_t* cu_seqlens, int nseg, int T,
                       int H, int D, int max_seqlen, int in_dtype, void* out, int32_t* status,
                       void* stream) {
  (void)max_seqlen;
  if (T < 0) return FRATTN_E_SHAPE;
  if (T > FRATTN_NOALLOC_MAX_TOKENS) return FRATTN_E_NOALLOC_LIMIT;
  size_t need = 0;
  int rc = frattn_workspace_bytes(T, nseg, &need);
  if (rc) return rc;
  if (need > FRATTN_NOALLOC_SCRATCH_BYTES) return FRATTN_E_NOALLOC_LIMIT;
  void* ws = nullptr;
  rc = noalloc_scratch(&ws);
  if (rc) return rc;
  // The scheduler kernel rewrites the header and every item it uses on each
  // call, so nothing in the array has to be cleared first. Only the work-list
  // bytes are handed over (never room for a rotated-K copy): every rotation
  // stays inside the attention kernel.
  return fwd_impl<kRopeTable>(q, k, v, cos, sin, cs_dtype, nullptr, 0, 0.f, cu_seqlens, nseg, T,
                              H, D, in_dtype, out, ws, need, status, stream);
}


int frattn_set_timing_events(void* start_event, void* stop_event) {
  if ((start_event == nullptr) != (stop_event == nullptr)) return FRATTN_E_NULL;
  g_ev_start = static_cast<cudaEvent_t>(start_event);
  g_ev_stop = static_cast<cudaEvent_t>(stop_event);
  return 0;
}

int frattn_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns == 0) return FRATTN_E_SHAPE;
  g_wait_limit_ns = limit_ns;
  return 0;
}

}  // extern "C"
