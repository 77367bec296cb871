// FP8 (e4m3) q / k variant of the fused RoPE attention forward (sm_100a).
//
// For long segments S = R(Q) R(K)^T is the tensor-core half of the work; with
// q and k rotated and quantised to e4m3 once per call it runs as
// tcgen05.mma kind::f8f6f4 (twice the 16-bit rate). P V stays 16-bit (P in
// [0, 1] has too few e4m3 mantissa bits to spare). Scales: one per (token,
// head) row of q, folded into that row's softmax exponent factor, and one per
// head for k (k rows are columns of S, so a per-row k scale would cost a
// multiply per score).
//
//   fp8_k_amax   one thread per (token, head): max |R(k)| per head (atomicMax
//                on the fp32 bit pattern, values are non-negative)
//   fp8_quantize one thread per (token, head): R(q) / s_q(t,h) and R(k) / s_k(h)
//                rounded to e4m3 (saturating), rows padded with zeros to a
//                multiple of 16 bytes; s = amax / 448 (the e4m3 maximum).
//                Eight lanes per row (one 8-element chunk of each half each,
//                16-byte loads, shuffle-reduced row maxima; head dims that are
//                multiples of 16).
// then the persistent attention kernel in its kRopeFp8 mode (work list as for
// frattn_fwd, no rotation, no K pre-rotation pass).
#include <cuda_fp8.h>

#include "frattn_kernel.cuh"

namespace frattn {

int attn_fp8_prequantized(const void* q8, const void* k8, const void* v, const float* qscale,
                          const float* kscale, int D16, const int32_t* cu, int nseg, int T, int H, int D,
                          int in_dtype, void* out, void* workspace, size_t ws_bytes, int32_t* status,
                          cudaStream_t st);  // frattn.cu

namespace {

constexpr float kE4M3Max = 448.f;

// Eight lanes per (token, head) row: lane c < D/16 owns the 8-element chunk c of
// each rotate-half half (16-byte loads), rotates it in fp32 and the row's
// max |value| is reduced over the eight lanes with shuffles.
template <int D, typename TI, typename TC>
__device__ __forceinline__ void rotated_chunk(const TI* __restrict__ x, const TC* __restrict__ cs,
                                              const TC* __restrict__ sn, int c, float (&y0)[8], float (&y1)[8]) {
  float c8[8], s8[8], x0[8], x1[8];
  load8<TC>(cs + 8 * c, c8);
  load8<TC>(sn + 8 * c, s8);
  unpack8<TI>(__ldg(reinterpret_cast<const uint4*>(x + 8 * c)), x0);
  unpack8<TI>(__ldg(reinterpret_cast<const uint4*>(x + D / 2 + 8 * c)), x1);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    y0[e] = x0[e] * c8[e] - x1[e] * s8[e];
    y1[e] = x0[e] * s8[e] + x1[e] * c8[e];
  }
}

__device__ __forceinline__ float max8_lanes(float m) {
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

__device__ __forceinline__ uint2 pack8_e4m3(const float (&y)[8], float inv) {
  uint32_t w[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(y[4 * u] * inv, y[4 * u + 1] * inv), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(y[4 * u + 2] * inv, y[4 * u + 3] * inv), __NV_SATFINITE, __NV_E4M3);
    w[u] = lo | (hi << 16);
  }
  return make_uint2(w[0], w[1]);
}

template <int D, typename TI, typename TC>
__global__ void __launch_bounds__(256) fp8_k_amax(const TI* __restrict__ k, const TC* __restrict__ cos,
                                                  const TC* __restrict__ sin, int T, int H,
                                                  unsigned int* __restrict__ kamax) {
  // per-head maxima of the block's rows in shared memory first, then one global
  // atomic per head and block (non-negative floats order as their bit patterns)
  __shared__ unsigned int smax[256];
  smax[threadIdx.x] = 0u;
  __syncthreads();
  const long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long i = g >> 3;  // row (token, head)
  const int c = static_cast<int>(g & 7);
  const bool in = i < static_cast<long long>(T) * H;
  const int h = static_cast<int>(i % H);
  float m = 0.f;
  if (in && c < D / 16) {
    const int t = static_cast<int>(i / H);
    float y0[8], y1[8];
    rotated_chunk<D, TI, TC>(k + static_cast<size_t>(i) * D, cos + static_cast<size_t>(t) * (D / 2),
                             sin + static_cast<size_t>(t) * (D / 2), c, y0, y1);
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, fmaxf(fabsf(y0[e]), fabsf(y1[e])));
  }
  m = max8_lanes(m);
  if (in && c == 0) {
    if (H <= 256)
      atomicMax(smax + h, __float_as_uint(m));
    else
      atomicMax(kamax + h, __float_as_uint(m));
  }
  __syncthreads();
  if (H <= 256 && static_cast<int>(threadIdx.x) < H && smax[threadIdx.x] != 0u)
    atomicMax(kamax + threadIdx.x, smax[threadIdx.x]);
}

template <int D, typename TI, typename TC>
__global__ void __launch_bounds__(256) fp8_quantize(const TI* __restrict__ q, const TI* __restrict__ k,
                                                    const TC* __restrict__ cos, const TC* __restrict__ sin,
                                                    int T, int H, const unsigned int* __restrict__ kamax,
                                                    uint8_t* __restrict__ q8, uint8_t* __restrict__ k8,
                                                    float* __restrict__ qscale, float* __restrict__ kscale) {
  constexpr int D16 = (D + 15) / 16 * 16;  // == D (head dims here are multiples of 16)
  static_assert(D16 == D, "multiples of 16");
  const long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long i = g >> 3;
  const int c = static_cast<int>(g & 7);
  const bool in = i < static_cast<long long>(T) * H;
  const bool act = in && c < D / 16;
  const int t = in ? static_cast<int>(i / H) : 0, h = static_cast<int>(i % H);
  const TC* cs = cos + static_cast<size_t>(t) * (D / 2);
  const TC* sn = sin + static_cast<size_t>(t) * (D / 2);
  float y0[8], y1[8];
  float m = 0.f;
  if (act) {
    rotated_chunk<D, TI, TC>(q + static_cast<size_t>(i) * D, cs, sn, c, y0, y1);
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, fmaxf(fabsf(y0[e]), fabsf(y1[e])));
  }
  m = max8_lanes(m);
  const float sq = m > 0.f ? m / kE4M3Max : 1.f;
  if (act) {
    uint8_t* row = q8 + static_cast<size_t>(i) * D;
    *reinterpret_cast<uint2*>(row + 8 * c) = pack8_e4m3(y0, 1.f / sq);
    *reinterpret_cast<uint2*>(row + D / 2 + 8 * c) = pack8_e4m3(y1, 1.f / sq);
    if (c == 0) qscale[i] = sq;
    const float mk = __uint_as_float(__ldg(kamax + h));
    const float sk = mk > 0.f ? mk / kE4M3Max : 1.f;
    rotated_chunk<D, TI, TC>(k + static_cast<size_t>(i) * D, cs, sn, c, y0, y1);
    uint8_t* krow = k8 + static_cast<size_t>(i) * D;
    *reinterpret_cast<uint2*>(krow + 8 * c) = pack8_e4m3(y0, 1.f / sk);
    *reinterpret_cast<uint2*>(krow + D / 2 + 8 * c) = pack8_e4m3(y1, 1.f / sk);
    if (t == 0 && c == 0) kscale[h] = sk;
  }
}

struct Fp8Layout {
  size_t base, q8, k8, qs, ks, kamax, total;
};
size_t al256(size_t x) { return (x + 255) & ~size_t(255); }
Fp8Layout fp8_layout(int T, int nseg, int H, int D) {
  Fp8Layout l;
  size_t base = 0;
  frattn_workspace_bytes(T, nseg, &base);
  const size_t rows = static_cast<size_t>(T) * H;
  const int D16 = (D + 15) / 16 * 16;
  l.base = 0;
  l.q8 = al256(base);
  l.k8 = al256(l.q8 + rows * D16);
  l.qs = al256(l.k8 + rows * D16);
  l.ks = al256(l.qs + rows * 4);
  l.kamax = al256(l.ks + static_cast<size_t>(H) * 4);
  l.total = al256(l.kamax + static_cast<size_t>(H) * 4);
  return l;
}

template <int D, typename TI, typename TC>
int quantize_d(const void* q, const void* k, const void* cos, const void* sin, int T, int H, uint8_t* ws,
               const Fp8Layout& L, cudaStream_t st) {
  const long long rows = static_cast<long long>(T) * H;
  const int blocks = static_cast<int>((rows * 8 + 255) / 256);  // eight lanes per row
  unsigned int* kamax = reinterpret_cast<unsigned int*>(ws + L.kamax);
  if (cudaMemsetAsync(kamax, 0, static_cast<size_t>(H) * 4, st) != cudaSuccess) return FRATTN_E_CUDA;
  fp8_k_amax<D, TI, TC><<<blocks, 256, 0, st>>>(static_cast<const TI*>(k), static_cast<const TC*>(cos),
                                                static_cast<const TC*>(sin), T, H, kamax);
  fp8_quantize<D, TI, TC><<<blocks, 256, 0, st>>>(
      static_cast<const TI*>(q), static_cast<const TI*>(k), static_cast<const TC*>(cos), static_cast<const TC*>(sin),
      T, H, kamax, ws + L.q8, ws + L.k8, reinterpret_cast<float*>(ws + L.qs), reinterpret_cast<float*>(ws + L.ks));
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

// Head dims with a 16-byte-chunked rotation (D / 2 a multiple of 8).
template <typename TI, typename TC>
int quantize(const void* q, const void* k, const void* cos, const void* sin, int T, int H, int D, uint8_t* ws,
             const Fp8Layout& L, cudaStream_t st) {
  switch (D) {
    case 32: return quantize_d<32, TI, TC>(q, k, cos, sin, T, H, ws, L, st);
    case 48: return quantize_d<48, TI, TC>(q, k, cos, sin, T, H, ws, L, st);
    case 64: return quantize_d<64, TI, TC>(q, k, cos, sin, T, H, ws, L, st);
    case 80: return quantize_d<80, TI, TC>(q, k, cos, sin, T, H, ws, L, st);
    case 96: return quantize_d<96, TI, TC>(q, k, cos, sin, T, H, ws, L, st);
    case 112: return quantize_d<112, TI, TC>(q, k, cos, sin, T, H, ws, L, st);
    case 128: return quantize_d<128, TI, TC>(q, k, cos, sin, T, H, ws, L, st);
    default: return FRATTN_E_SHAPE;
  }
}

template <typename TI>
int quantize_cs(int cs_dtype, const void* q, const void* k, const void* cos, const void* sin, int T, int H, int D,
                uint8_t* ws, const Fp8Layout& L, cudaStream_t st) {
  switch (cs_dtype) {
    case FRATTN_F32: return quantize<TI, float>(q, k, cos, sin, T, H, D, ws, L, st);
    case FRATTN_BF16: return quantize<TI, __nv_bfloat16>(q, k, cos, sin, T, H, D, ws, L, st);
    case FRATTN_F16: return quantize<TI, __half>(q, k, cos, sin, T, H, D, ws, L, st);
    default: return FRATTN_E_DTYPE;
  }
}

}  // namespace
}  // namespace frattn

extern "C" int frattn_workspace_bytes_fp8(int total_tokens, int num_segments, int num_heads, int head_dim,
                                          size_t* bytes) {
  if (!bytes) return FRATTN_E_NULL;
  if (total_tokens < 0 || num_segments < 1 || num_heads <= 0 || head_dim <= 0) return FRATTN_E_SHAPE;
  *bytes = frattn::fp8_layout(total_tokens, num_segments, num_heads, head_dim).total;
  return 0;
}

extern "C" int frattn_fwd_fp8(const void* q, const void* k, const void* v, const void* cos, const void* sin,
                              int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
                              int max_seqlen, int in_dtype, void* out, void* workspace, size_t workspace_bytes,
                              int32_t* status, void* stream) {
  using namespace frattn;
  (void)max_seqlen;
  if (!q || !k || !v || !cos || !sin || !cu_seqlens || !out || !workspace) return FRATTN_E_NULL;
  if (T < 0 || H <= 0 || nseg < 1 || D % 16 != 0 || D < 32 || D > 128) return FRATTN_E_SHAPE;
  if (in_dtype != FRATTN_BF16 && in_dtype != FRATTN_F16) return FRATTN_E_DTYPE;
  if (cs_dtype != FRATTN_F32 && cs_dtype != FRATTN_BF16 && cs_dtype != FRATTN_F16) return FRATTN_E_DTYPE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return FRATTN_E_ALIGN;
  const Fp8Layout L = fp8_layout(T, nseg, H, D);
  if (workspace_bytes < L.total) return FRATTN_E_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (T > 0) {
    const int rc = in_dtype == FRATTN_BF16
                       ? quantize_cs<__nv_bfloat16>(cs_dtype, q, k, cos, sin, T, H, D, ws, L, st)
                       : quantize_cs<__half>(cs_dtype, q, k, cos, sin, T, H, D, ws, L, st);
    if (rc) return rc;
  }
  return attn_fp8_prequantized(ws + L.q8, ws + L.k8, v, reinterpret_cast<const float*>(ws + L.qs),
                               reinterpret_cast<const float*>(ws + L.ks), (D + 15) / 16 * 16, cu_seqlens, nseg, T,
                               H, D, in_dtype, out, ws, L.q8, status, st);
}
