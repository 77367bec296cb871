// Kernels of one head dimension D (this file is compiled once per supported D
// with -DFRATTN_D=<D>; the host code in frattn.cu picks the object by D).
#include "frattn_kernel.cuh"

#ifndef FRATTN_D
#error "compile with -DFRATTN_D=<head dim>"
#endif
#define FRATTN_CAT2(a, b) a##b
#define FRATTN_CAT(a, b) FRATTN_CAT2(a, b)

namespace frattn {

// Attention launch (K pre-rotation when prm.krot is set, then the persistent
// attention kernel) for element types in_dtype / cs_dtype.
int FRATTN_CAT(attn_d, FRATTN_D)(const Params& prm, int mode, int in_dtype, int cs_dtype,
                                 cudaStream_t st) {
#ifdef FRATTN_FAST_BUILD  // experiment builds: table mode only
  if (mode != kRopeTable) return FRATTN_E_SHAPE;
  return dispatch_in<FRATTN_D, kRopeTable>(prm, in_dtype, cs_dtype, st);
#else
  if (mode == kRopePos) return dispatch_in<FRATTN_D, kRopePos>(prm, in_dtype, cs_dtype, st);
  if (mode == kRopeNone) return dispatch_in<FRATTN_D, kRopeNone>(prm, in_dtype, cs_dtype, st);
  if (mode == kRopeFp8) return dispatch_in<FRATTN_D, kRopeFp8>(prm, in_dtype, cs_dtype, st);
  return dispatch_in<FRATTN_D, kRopeTable>(prm, in_dtype, cs_dtype, st);
#endif
}

// Window-regime kernel (every segment at most 128 tokens); FRATTN_E_SHAPE when
// this head dim or element type has none.
// `rotated`: q and k arrive rotated (no tables are read).
int FRATTN_CAT(window_d, FRATTN_D)(const Params& prm, int in_dtype, int cs_dtype, bool rotated,
                                   cudaStream_t st) {
  if (in_dtype == FRATTN_BF16) return window_cs<FRATTN_D, __nv_bfloat16>(prm, cs_dtype, st, rotated);
#ifndef FRATTN_FAST_BUILD
  if (in_dtype == FRATTN_F16) return window_cs<FRATTN_D, __half>(prm, cs_dtype, st, rotated);
#endif
  return FRATTN_E_DTYPE;
}

// Work-list (scheduler) kernel of this head dimension.
int FRATTN_CAT(prep_d, FRATTN_D)(const int32_t* cu, int nseg, int T, int H, WorkItem* items,
                                 int* header, void* out, int32_t* status, const int32_t* pos_hw,
                                 float* pos_tab, int pos_rows, float theta, int in_dtype,
                                 cudaStream_t st) {
  if (in_dtype == FRATTN_BF16)
    build_worklist<__nv_bfloat16, FRATTN_D><<<1, kPrepThreads, 0, st>>>(
        cu, nseg, T, H, items, header, static_cast<__nv_bfloat16*>(out), status, pos_hw, pos_tab,
        pos_rows, theta);
  else
    build_worklist<__half, FRATTN_D><<<1, kPrepThreads, 0, st>>>(
        cu, nseg, T, H, items, header, static_cast<__half*>(out), status, pos_hw, pos_tab, pos_rows,
        theta);
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

}  // namespace frattn

#if defined(FRATTN_TRACE) && FRATTN_D == 80
extern "C" int frattn_trace_read(unsigned long long* host, int words) {
  if (words > frattn::kTraceWords) words = frattn::kTraceWords;
  return cudaMemcpyFromSymbol(host, frattn::g_trace, words * sizeof(unsigned long long)) ==
                 cudaSuccess
             ? 0
             : 1;
}
#endif
