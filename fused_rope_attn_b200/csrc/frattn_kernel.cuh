// Fused 2D-RoPE + variable-length attention forward for B200 (sm_100a).
//
// Operation (reference: sdan/fused-rope-attn fused_attn.py:246-423, the Triton
// `fused_attn_kernel`, and its wrapper fused_attn.py:139-232):
//   for each cu_seqlens segment s and head h,
//     O = softmax(R(Q) R(K)^T / sqrt(D)) V
//   with R = rotate-half RoPE, computed in fp32 and rounded to the input type
//   before the product (fused_attn.py:340-345, 385-390), fp32 online softmax in
//   base 2 (fused_attn.py:353-405), fp32 accumulation and a final 1/l
//   (fused_attn.py:417-423).
//
// Design (B200-native, not a translation of the Triton program grid):
//   * An on-device scheduler kernel (`build_worklist`) turns cu_seqlens into a
//     work list in the workspace, so no host sync is needed:
//       - "long" items: 256-row q ranges (two 128-row tiles) of segments longer
//         than 128 tokens, attending to their whole segment;
//       - "packed" items: the rows of all short (<= 128 token) segments that
//         lie in one 128-row chunk of the packed sequence, batched into one
//         M=128 tile with a per-row segment mask (two 64-token windows share
//         one tensor-core tile instead of two half-empty ones).
//   * One persistent CTA per SM walks units. A unit fills two 128-row q "slots"
//     A and B: two q tiles of one (segment, head) sharing every K/V tile (long
//     items), or heads 2g and 2g+1 of one packed item. The softmax of one slot
//     overlaps the tensor-core work of the other.
//   * 512 threads = 4 warpgroups with a setmaxnreg register split:
//       WG0  warp 0 TMA producer (Q, K, V tiles; 32-B swizzle, 16-column
//            blocks), warp 1 tcgen05 MMA issuer + TMEM owner
//       WG1  RoPE: rotates raw Q/K tiles in shared memory in place, one tile row
//            per thread, loads of a batch issued up front
//       WG2  softmax + O rescale + epilogue of slot A (row = TMEM lane)
//       WG3  the same for slot B
//   * S = Q K^T (M=128, N=128, K=D, both operands in smem) and O += P V
//     (M=128, N=D, K=128, P read from TMEM where it overwrites S) run on the
//     5th-gen tensor cores with fp32 accumulators in TMEM.
//   * The exponent reference max only moves when the row max grows by > 2^8,
//     so O is rescaled rarely.
//   * Every mbarrier wait is bounded; on timeout the kernel records a status
//     code and returns instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <type_traits>

#include "../../include/frattn.h"
#include "frattn_ptx.cuh"

namespace frattn {

constexpr int kTileM = 128;   // q rows per tile (TMEM lanes)
constexpr int kTileN = 128;   // kv rows per tile
constexpr int kThreads = 512; // 16 warps = 4 warpgroups
constexpr int kRopeThreads = 128;

#ifndef FRATTN_POLY_OF_8
#define FRATTN_POLY_OF_8 0  // pairs (of every 8) whose exp2 runs on the FMA pipe
#endif
#ifndef FRATTN_REG_CTRL
#define FRATTN_REG_CTRL 80
#endif
#ifndef FRATTN_REG_ROPE
#define FRATTN_REG_ROPE 80
#endif
#ifndef FRATTN_REG_SOFTMAX
#define FRATTN_REG_SOFTMAX 176
#endif
constexpr int kSoftmaxThreads = 128;
constexpr int kBlkBytes = kTileM * 32;  // one 16-column (32 B) block of a 128-row tile

enum ItemKind : int { kItemLong = 0, kItemPacked = 1 };

struct __align__(16) WorkItem {
  int q0, q1;      // q rows [q0, q1) stored by this item
  int kv0, kv1;    // kv rows [kv0, kv1) attended to
  int seg_lo, seg_hi;  // segment index range covered (packed items)
  int kind, pad;
};

// The work list, its header and the position table are written by
// build_worklist in the same call. The kernels that read them start early
// (programmatic dependent launch) and may be resident before those writes, so
// they read them through L2 (ld.global.cg), never through the non-coherent
// read-only path, which may keep lines from before the writes.
__device__ __forceinline__ WorkItem load_item(const WorkItem* it) {
  const int4 a = __ldcg(reinterpret_cast<const int4*>(it));
  const int4 b = __ldcg(reinterpret_cast<const int4*>(it) + 1);
  WorkItem w;
  w.q0 = a.x; w.q1 = a.y; w.kv0 = a.z; w.kv1 = a.w;
  w.seg_lo = b.x; w.seg_hi = b.y; w.kind = b.z; w.pad = b.w;
  return w;
}

constexpr int kHeaderBytes = 128;
__host__ __device__ inline size_t max_items(int T) {
  const size_t chunks = (static_cast<size_t>(T) + kTileM - 1) / kTileM;
  return 3 * chunks + 2;
}

// Rotary angle source: materialised tables (reference API), (h, w) ids, or
// none (q and k arrive rotated, e.g. from the QKV projection's epilogue).
// kRopeFp8: q and k arrive rotated and quantised to e4m3 (per-row q scales,
// per-head k scales); S = Q K^T runs as an FP8 MMA, P V stays 16-bit.
enum RopeMode : int { kRopeTable = 0, kRopePos = 1, kRopeNone = 2, kRopeFp8 = 3 };

struct Params {
  CUtensorMap tmq, tmk, tmv;
  CUtensorMap tmk_rot;
  CUtensorMap tmcos, tmsin; // [T, D/2] cos/sin tables, box {D/2, 128} (table mode)      // rotated K in the workspace (long segments), when krot != nullptr
  const void* k;            // [T, H, D] raw K (token stride k_stride elements)
  long long k_stride;
  void* krot;               // [T, H, D] K rotated once, rows of long segments only
  const void* cos;          // [T, D/2] (table mode)
  const void* sin;
  const int32_t* pos_hw;    // [T, 2] (pos mode)
  const float* pos_tab;     // [P, D/4] cos then [P, D/4] sin (pos mode)
  int pos_rows;
  const int32_t* cu;
  int nseg;
  void* out;
  const WorkItem* items;
  const int* header;
  int T, H;
  int32_t* status;
  unsigned long long wait_limit_ns;
  float* lse;               // [T, H] base-2 log-sum-exp of the scaled scores, or nullptr
  const float* qscale;      // [T, H] e4m3 dequantisation scales of q rows (kRopeFp8)
  const float* kscale;      // [H] e4m3 dequantisation scale of k (kRopeFp8)
};

// ------------------------------------------------------------------ helpers
struct Ctl {
  uint32_t tmem_base;
  int abort;
};

// Timeline trace (build with -DFRATTN_TRACE): SM clock stamps of pipeline
// events of CTA 0's first two units, read back with frattn_trace_read.
#ifdef FRATTN_TRACE
constexpr int kTraceWords = 8192;
static __device__ unsigned long long g_trace[kTraceWords];
#define FR_TRACE(ui, ev, idx)                                                          \
  do {                                                                                 \
    if (blockIdx.x == 0 && (ui) < 2 && (idx) < 128)                                    \
      g_trace[(ui) * 4096 + (ev) * 128 + (idx)] = clock64();                           \
  } while (0)
#else
#define FR_TRACE(ui, ev, idx) do { } while (0)
#endif

__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity, const Params& p,
                                             volatile int* abort_flag, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > p.wait_limit_ns) {
        *abort_flag = 1;
        if (p.status) atomicCAS(reinterpret_cast<int*>(p.status), 0, code);
        return false;
      }
    }
  }
  return true;
}

// Warp-uniform bounded wait (every lane polls; the warp agrees on the result so
// that the following .sync.aligned tcgen05 instructions never diverge).
__device__ __forceinline__ bool bounded_wait_warp(uint32_t bar, uint32_t parity, const Params& p,
                                                  volatile int* abort_flag, int code) {
  const bool ok = bounded_wait(bar, parity, p, abort_flag, code);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs (Blackwell f32x2 instructions) and exp2 on the FMA pipe
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t add2_rm(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair of arguments on the FMA pipe (offloads the MUFU unit):
//   n = floor(x) via a round-down add of 1.5 * 2^23, f = x - n in [0, 1),
//   2^f by a cubic fitted here (Lawson-iterated least squares on Chebyshev
//   nodes, max relative error 7.5e-5, below the bf16/fp16 rounding of P),
//   then n is added to the exponent field. Arguments are clamped at -126 so
//   masked (-inf) entries give (nearly) 0; results are exact enough for P and
//   the row sums (2^-13.7 relative).
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  float x0, x1;
  f2unpack(x, x0, x1);
  x = f2pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t magic = f2pack(kMagic, kMagic);
  const uint64_t t = add2_rm(x, magic);           // floor(x) + magic, exactly
  const uint64_t f = sub2(x, sub2(t, magic));     // x - floor(x)
  uint64_t y = fma2(f2pack(0.0780244916677475f, 0.0780244916677475f), f,
                    f2pack(0.22606723010540009f, 0.22606723010540009f));
  y = fma2(y, f, f2pack(0.6958335041999817f, 0.6958335041999817f));
  y = fma2(y, f, f2pack(0.9999251961708069f, 0.9999251961708069f));
  float t0, t1, y0, y1;
  f2unpack(t, t0, t1);
  f2unpack(y, y0, y1);
  // bits(t) << 23 == floor(x) << 23 (mod 2^32): the magic's low 9 bits are 0
  const uint32_t r0 = __float_as_uint(y0) + (__float_as_uint(t0) << 23);
  const uint32_t r1 = __float_as_uint(y1) + (__float_as_uint(t1) << 23);
  return f2pack(__uint_as_float(r0), __uint_as_float(r1));
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

// Load 8 consecutive values of a cos/sin table row as fp32.
template <typename TC>
__device__ __forceinline__ void load8(const TC* src, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* src, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(src));
  const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* src, float (&v)[8]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* src, float (&v)[8]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
  const __half2* h = reinterpret_cast<const __half2*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Load 8 consecutive cos/sin values from shared memory as fp32.
template <typename TC>
__device__ __forceinline__ void load8_smem(const TC* src, float (&v)[8]) {
  if constexpr (std::is_same<TC, float>::value) {
    const float4 a = reinterpret_cast<const float4*>(src)[0];
    const float4 b = reinterpret_cast<const float4*>(src)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    const TC* h = reinterpret_cast<const TC*>(&a);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32<TC>(h[i]);
  }
}

template <typename TI>
__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]);
template <>
__device__ __forceinline__ void unpack8<__nv_bfloat16>(const uint4& u, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void unpack8<__half>(const uint4& u, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename TI>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Address of the 16-byte chunk `c` (8 elements) of row r inside a 128-row tile
// stored as [column block][row][32 B] with the TMA/UMMA 32-byte swizzle
// (16-byte halves of rows 4..7 of every 8-row group are swapped).
__device__ __forceinline__ uint32_t chunk_off(int r, int c) {
  return static_cast<uint32_t>((c >> 1) * kBlkBytes + r * 32 +
                               ((((c & 1) ^ (r >> 2)) & 1) << 4));
}

// Rotary cos/sin for 8 consecutive rotary indices [i0, i0+8) of token `row`.
template <int D, int MODE, typename TC>
__device__ __forceinline__ void rope_coeffs(const Params& p, int row, int i0, float (&cs)[8],
                                            float (&sn)[8]) {
  if constexpr (MODE == kRopeTable) {
    const TC* c = static_cast<const TC*>(p.cos) + static_cast<size_t>(row) * (D / 2) + i0;
    const TC* s = static_cast<const TC*>(p.sin) + static_cast<size_t>(row) * (D / 2) + i0;
    load8<TC>(c, cs);
    load8<TC>(s, sn);
  } else {
    constexpr int Q4 = D / 4;
    const int2 hw = __ldg(reinterpret_cast<const int2*>(p.pos_hw) + row);
    const float* ct = p.pos_tab;
    const float* st = p.pos_tab + static_cast<size_t>(p.pos_rows) * Q4;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = i0 + e;
      const int pos = i < Q4 ? hw.x : hw.y;
      const int j = i < Q4 ? i : i - Q4;
      const size_t idx = static_cast<size_t>(pos) * Q4 + j;
      cs[e] = __ldcg(ct + idx);
      sn[e] = __ldcg(st + idx);
    }
  }
}

// Rotate chunk pair (c, c + D/16) of row r of a 128 x D tile in place
// (rotate-half RoPE in fp32, one rounding to the element type,
// fused_attn.py:340-345). cos/sin come from the staged rows when given.
template <int D, int MODE, typename TI, typename TC>
__device__ __forceinline__ void rope_pair(uint8_t* tile, int row0, const Params& p, int r,
                                          const uint8_t* cs_smem, int c) {
  constexpr int NP = D / 16;
  const uint4 ua = *reinterpret_cast<const uint4*>(tile + chunk_off(r, c));
  const uint4 ub = *reinterpret_cast<const uint4*>(tile + chunk_off(r, c + NP));
  float cs[8], sn[8];
  if (MODE == kRopeTable && cs_smem != nullptr) {
    const TC* cst = reinterpret_cast<const TC*>(cs_smem) + r * (D / 2) + c * 8;
    load8_smem<TC>(cst, cs);
    load8_smem<TC>(cst + kTileM * (D / 2), sn);
  } else {
    rope_coeffs<D, MODE, TC>(p, min(row0 + r, p.T - 1), c * 8, cs, sn);  // rows >= T hold TMA zeros
  }
  float x0[8], x1[8];
  unpack8<TI>(ua, x0);
  unpack8<TI>(ub, x1);
  uint4 oa, ob;
  uint32_t* wa = reinterpret_cast<uint32_t*>(&oa);
  uint32_t* wb = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    wa[e / 2] = pack2<TI>(x0[e] * cs[e] - x1[e] * sn[e], x0[e + 1] * cs[e + 1] - x1[e + 1] * sn[e + 1]);
    wb[e / 2] = pack2<TI>(x0[e] * sn[e] + x1[e] * cs[e], x0[e + 1] * sn[e + 1] + x1[e + 1] * cs[e + 1]);
  }
  *reinterpret_cast<uint4*>(tile + chunk_off(r, c)) = oa;
  *reinterpret_cast<uint4*>(tile + chunk_off(r, c + NP)) = ob;
}

// cos/sin of rotary index i for token `row` (scalar; used when D/2 is not a
// multiple of 8, e.g. D = 72).
template <int D, int MODE, typename TC>
__device__ __forceinline__ void rope_coeff1(const Params& p, int row, int i, const TC* cs_row, float& c,
                                            float& s) {
  if (MODE == kRopeTable && cs_row != nullptr) {
    c = to_f32<TC>(cs_row[i]);
    s = to_f32<TC>(cs_row[kTileM * (D / 2) + i]);
  } else if constexpr (MODE == kRopeTable) {
    c = to_f32<TC>(__ldg(static_cast<const TC*>(p.cos) + static_cast<size_t>(row) * (D / 2) + i));
    s = to_f32<TC>(__ldg(static_cast<const TC*>(p.sin) + static_cast<size_t>(row) * (D / 2) + i));
  } else {
    constexpr int Q4 = D / 4;
    const int2 hw = __ldg(reinterpret_cast<const int2*>(p.pos_hw) + row);
    const int pos = i < Q4 ? hw.x : hw.y;
    const size_t idx = static_cast<size_t>(pos) * Q4 + (i < Q4 ? i : i - Q4);
    c = __ldcg(p.pos_tab + idx);
    s = __ldcg(p.pos_tab + static_cast<size_t>(p.pos_rows) * Q4 + idx);
  }
}

// Element-wise rotation of row r (pairs j, j + D/2 that straddle 8-element
// chunks), for head dims with D/2 not a multiple of 8.
template <int D, int MODE, typename TI, typename TC>
__device__ __forceinline__ void rope_row_elementwise(uint8_t* tile, int row0, const Params& p, int r,
                                                     const uint8_t* cs_smem) {
  const int row = row0 + r;
  if (row >= p.T) return;
  const TC* cs_row = cs_smem ? reinterpret_cast<const TC*>(cs_smem) + r * (D / 2) : nullptr;
  auto at = [&](int e) -> TI* {
    return reinterpret_cast<TI*>(tile + chunk_off(r, e >> 3) + (e & 7) * 2);
  };
#pragma unroll 4
  for (int j = 0; j < D / 2; ++j) {
    TI* pa = at(j);
    TI* pb = at(j + D / 2);
    const float x0 = to_f32<TI>(*pa), x1 = to_f32<TI>(*pb);
    float c, sn;
    rope_coeff1<D, MODE, TC>(p, row, j, cs_row, c, sn);
    const float a = x0 * c - x1 * sn;
    const float b = x0 * sn + x1 * c;
    *pa = from_f32<TI>(a);
    *pb = from_f32<TI>(b);
  }
}

// Rotate the rows of a raw 128 x D tile owned by this rope thread.
template <int D, int MODE, typename TI, typename TC>
__device__ __forceinline__ void rope_tile(uint8_t* tile, int row0, const Params& p, int r0,
                                          const uint8_t* cs_smem = nullptr) {
  if constexpr (MODE == kRopeNone || MODE == kRopeFp8) {
    return;  // already rotated
  } else if constexpr (D % 16 == 0) {
    // One chunk pair per iteration, as a real loop: the rotation shares the
    // SM's instruction caches with the softmax code, and the unrolled form
    // (D/16 copies at each call site) measured slower in the window regime.
    constexpr int NP = D / 16;
#pragma unroll 1
    for (int c = 0; c < NP; ++c) rope_pair<D, MODE, TI, TC>(tile, row0, p, r0, cs_smem, c);
  } else {
    rope_row_elementwise<D, MODE, TI, TC>(tile, row0, p, r0, cs_smem);
  }
}

// Rotate row r of a raw 128 x D Q tile (shared memory) into TMEM lane r at
// column qcol: element e of the rotated row goes to column qcol + e / 2 as a
// packed pair, the A-operand layout of a TMEM-sourced MMA. The smem tile is
// only read. Warp-converged (tcgen05.st is .sync.aligned).
template <int D, int MODE, typename TI, typename TC>
__device__ __forceinline__ void rope_q_to_tmem(const uint8_t* tile, int row0, const Params& p, int r,
                                               const uint8_t* cs_smem, uint32_t qcol) {
  static_assert(D % 16 == 0, "whole 8-element chunks");
  constexpr int NP = D / 16;
#pragma unroll 1
  for (int c = 0; c < NP; ++c) {
    const uint4 ua = *reinterpret_cast<const uint4*>(tile + chunk_off(r, c));
    const uint4 ub = *reinterpret_cast<const uint4*>(tile + chunk_off(r, c + NP));
    if constexpr (MODE == kRopeNone) {  // already rotated: copy
      tmem_st4(qcol + 4 * c, ua);
      tmem_st4(qcol + 4 * (c + NP), ub);
      continue;
    }
    float cs[8], sn[8];
    if (MODE == kRopeTable && cs_smem != nullptr) {
      const TC* cst = reinterpret_cast<const TC*>(cs_smem) + r * (D / 2) + c * 8;
      load8_smem<TC>(cst, cs);
      load8_smem<TC>(cst + kTileM * (D / 2), sn);
    } else {
      rope_coeffs<D, MODE, TC>(p, min(row0 + r, p.T - 1), c * 8, cs, sn);
    }
    float x0[8], x1[8];
    unpack8<TI>(ua, x0);
    unpack8<TI>(ub, x1);
    uint4 oa, ob;
    uint32_t* wa = reinterpret_cast<uint32_t*>(&oa);
    uint32_t* wb = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      wa[e / 2] = pack2<TI>(x0[e] * cs[e] - x1[e] * sn[e], x0[e + 1] * cs[e + 1] - x1[e + 1] * sn[e + 1]);
      wb[e / 2] = pack2<TI>(x0[e] * sn[e] + x1[e] * cs[e], x0[e + 1] * sn[e + 1] + x1[e + 1] * cs[e + 1]);
    }
    tmem_st4(qcol + 4 * c, oa);
    tmem_st4(qcol + 4 * (c + NP), ob);
  }
}

__device__ __forceinline__ int upper_bound_cu(const int32_t* cu, int lo, int hi, int x) {
  // first index i in [lo, hi) with cu[i] > x (hi if none)
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(cu + mid) > x) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// ------------------------------------------------------------------ K pre-rotation
// Rows of segments longer than one tile are read by every q tile of their
// segment: rotating those K rows once per call (instead of once per q tile in
// the attention kernel) turns L/128 rotations of each K tile into one, at the
// cost of reading K and writing the rotated copy once (HBM-bound, a few us).
// Short segments keep the fully fused path (their K tiles are used once).
// Same arithmetic as rope_pair: fp32 rotation, one rounding.
template <int D, int MODE, typename TI, typename TC>
__global__ void __launch_bounds__(256) rotate_k_long(const __grid_constant__ Params p) {
  constexpr int NP = D / 16;
  griddep_wait();               // work list of this call is complete
  griddep_launch_dependents();  // let the attention kernel start its prologue
  const int n_long = __ldcg(p.header + 1);
  const TI* kin = static_cast<const TI*>(p.k);
  TI* kout = static_cast<TI*>(p.krot);
  // One thread per (row, head) of the long items (each covers at most 256 rows):
  // the whole 2*D-byte K row and its cos/sin row are loaded before any math.
  const int per_item = 2 * kTileM * p.H;
  const long long total = static_cast<long long>(n_long) * per_item;
  for (long long e = blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(e / per_item);
    const int rem = static_cast<int>(e % per_item);
    const int h = rem % p.H;
    const int row = __ldcg(&p.items[i].q0) + rem / p.H;
    if (row >= __ldcg(&p.items[i].q1)) continue;
    const size_t base = (static_cast<size_t>(row) * p.H + h) * D;  // rotated copy: contiguous
    const size_t ibase = static_cast<size_t>(row) * p.k_stride + static_cast<size_t>(h) * D;
    if constexpr (D % 16 != 0) {
      for (int j = 0; j < D / 2; ++j) {
        const float x0 = to_f32<TI>(kin[ibase + j]), x1 = to_f32<TI>(kin[ibase + D / 2 + j]);
        float c, sn;
        rope_coeff1<D, MODE, TC>(p, row, j, static_cast<const TC*>(nullptr), c, sn);
        kout[base + j] = from_f32<TI>(x0 * c - x1 * sn);
        kout[base + D / 2 + j] = from_f32<TI>(x0 * sn + x1 * c);
      }
    } else {
      uint4 ua[NP], ub[NP];
#pragma unroll
      for (int c = 0; c < NP; ++c) {
        ua[c] = __ldg(reinterpret_cast<const uint4*>(kin + ibase + 8 * c));
        ub[c] = __ldg(reinterpret_cast<const uint4*>(kin + ibase + D / 2 + 8 * c));
      }
#pragma unroll
      for (int c = 0; c < NP; ++c) {
        float x0[8], x1[8], cs[8], sn[8];
        unpack8<TI>(ua[c], x0);
        unpack8<TI>(ub[c], x1);
        rope_coeffs<D, MODE, TC>(p, row, 8 * c, cs, sn);
        uint4 oa, ob;
        uint32_t* wa = reinterpret_cast<uint32_t*>(&oa);
        uint32_t* wb = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
        for (int q = 0; q < 8; q += 2) {
          const float a0 = x0[q] * cs[q] - x1[q] * sn[q];
          const float a1 = x0[q + 1] * cs[q + 1] - x1[q + 1] * sn[q + 1];
          const float b0 = x0[q] * sn[q] + x1[q] * cs[q];
          const float b1 = x0[q + 1] * sn[q + 1] + x1[q + 1] * cs[q + 1];
          wa[q / 2] = pack2<TI>(a0, a1);
          wb[q / 2] = pack2<TI>(b0, b1);
        }
        *reinterpret_cast<uint4*>(kout + base + 8 * c) = oa;
        *reinterpret_cast<uint4*>(kout + base + D / 2 + 8 * c) = ob;
      }
    }
  }
}

// ------------------------------------------------------------------ kernel
// A unit of work: one or two 128-row q tiles ("slots" A and B) that the CTA
// runs concurrently so that the softmax of one slot overlaps the tensor-core
// work of the other.
//   long item  (segment > 128 tokens): slots A/B = consecutive q tiles of one
//              (segment, head); they share every K/V tile.
//   packed item: slots A/B = heads 2g and 2g+1 of the same packed rows; each
//              slot has its own K/V tiles.
struct Unit {
  int q0a, q1a, q0b, q1b;
  int ha, hb;
  int kv0, kv1, seg_lo, seg_hi, kind;
  bool has_b, shared;
};

__device__ __forceinline__ Unit decode_unit(const Params& p, int u, int n_long) {
  Unit U;
  const int hp = (p.H + 1) >> 1;
  WorkItem it;
  if (u < n_long * p.H) {
    it = load_item(p.items + u / p.H);
    const int h = u % p.H;
    U.q0a = it.q0;
    U.q1a = min(it.q0 + kTileM, it.q1);
    U.q0b = it.q0 + kTileM;
    U.q1b = it.q1;
    U.ha = U.hb = h;
    U.has_b = U.q0b < U.q1b;
    U.shared = true;
  } else {
    const int v = u - n_long * p.H;
    it = load_item(p.items + n_long + v / hp);
    const int g = v % hp;
    U.q0a = U.q0b = it.q0;
    U.q1a = U.q1b = it.q1;
    U.ha = 2 * g;
    U.hb = 2 * g + 1;
    U.has_b = U.hb < p.H;
    U.shared = false;
  }
  U.kv0 = it.kv0;
  U.kv1 = it.kv1;
  U.seg_lo = it.seg_lo;
  U.seg_hi = it.seg_hi;
  U.kind = it.kind;
  return U;
}

template <int D, int CSB, bool FP8 = false>
struct Cfg {
  static_assert(D % 8 == 0 && D >= 32 && D <= 128, "D must be a multiple of 8 in [32,128]");
  static constexpr int DP = (D + 15) / 16 * 16;      // tile width: D rounded up to the MMA K step
  static constexpr int KB = DP / 16;                 // 32-byte column blocks per row
  static constexpr int TILE_BYTES = kTileM * DP * 2; // one 128 x DP tile (TMA zero-fills D..DP)
  // cos/sin rows of the current unit staged in smem (table mode): [128][D/2] x 2
  // (only when a cos/sin row is a whole number of 16-byte units, as TMA requires)
  static constexpr int CS_BYTES = ((D / 2) * CSB) % 16 == 0 ? 2 * kTileM * (D / 2) * CSB : 0;
  static constexpr int BAR_BYTES = 512;
  static constexpr int kBudget = 232448 - BAR_BYTES - 1024;
  static constexpr bool fits(int qb, int st) {
    return (2 * qb + 2 * st) * TILE_BYTES + CS_BYTES <= kBudget;
  }
  static constexpr int STAGES = fits(1, D <= 80 ? 3 : 2) ? (D <= 80 ? 3 : 2) : 1;  // K/V ring
  static constexpr int QBUF = fits(2, STAGES) ? 2 : 1;                             // Q per slot
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * QBUF * TILE_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * TILE_BYTES;
  static constexpr int OFF_CS = OFF_V + STAGES * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_CS + ((CS_BYTES + 1023) & ~1023);
  static constexpr int SMEM_BYTES = OFF_BAR + BAR_BYTES + 1024;  // +1024 alignment slack
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  // TMEM columns: S/P of slot X at 128 X, O of slot X at 256 + 128 X.
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t TMEM_S = 0;
  static constexpr uint32_t TMEM_O = 256;
  // Rotated Q of slot X lives in TMEM behind O_X (columns DP .. DP + DP/2 of
  // the 128-column O region) when it fits; S then takes its A operand from
  // TMEM and the rotation never writes shared memory.
  static constexpr bool Q_TMEM = !FP8 && (D % 16 == 0) && (DP + DP / 2 <= 128);
  // FP8 q / k tiles: 32-element (32-byte) column blocks, zero-filled past D
  static constexpr int KB8 = (D + 31) / 32;
  static constexpr uint32_t TMEM_Q = TMEM_O + DP;
};

template <int ST, int QB>
struct Bars {
  static constexpr int Q_FULL = 0;                   // [2][QB]
  static constexpr int Q_READY = Q_FULL + 2 * QB;    // [2][QB]
  static constexpr int Q_EMPTY = Q_READY + 2 * QB;   // [2][QB]
  static constexpr int K_FULL = Q_EMPTY + 2 * QB;    // [ST]
  static constexpr int K_READY = K_FULL + ST;
  static constexpr int K_EMPTY = K_READY + ST;
  static constexpr int V_FULL = K_EMPTY + ST;
  static constexpr int V_EMPTY = V_FULL + ST;
  static constexpr int S_FULL = V_EMPTY + ST;        // [2] S of slot X in TMEM
  static constexpr int P_FULL = S_FULL + 2;          // [2] P of slot X in TMEM (S consumed)
  static constexpr int O_FULL = P_FULL + 2;          // [2] last PV of the unit done
  static constexpr int CS_FULL = O_FULL + 2;          // cos/sin of the unit staged
  static constexpr int CS_EMPTY = CS_FULL + 1;         // ... and no longer needed
  static constexpr int DONE = CS_EMPTY + 1;
  static constexpr int QT_FREE = DONE + 1;            // [2] Q columns of slot X in TMEM reusable
  static constexpr int COUNT = QT_FREE + 2;
};

// Register split (setmaxnreg): 128 x (REG_CTRL + REG_ROPE) + 256 x REG_SOFTMAX
// must not exceed the 512 x 128 launch budget.
constexpr uint32_t REG_CTRL = FRATTN_REG_CTRL;
constexpr uint32_t REG_ROPE = FRATTN_REG_ROPE;
constexpr uint32_t REG_SOFTMAX = FRATTN_REG_SOFTMAX;
#ifndef FRATTN_REG_EXPERIMENT
static_assert(128 * (REG_CTRL + REG_ROPE) + 256 * REG_SOFTMAX <= 512 * 128, "register split");
#endif

template <int D, int MODE, typename TI, typename TC>
__global__ void __launch_bounds__(kThreads, 1) fused_rope_attn_kernel(const __grid_constant__ Params p) {
  using C = Cfg<D, MODE == kRopeTable ? static_cast<int>(sizeof(TC)) : 0, MODE == kRopeFp8>;
  constexpr bool kFp8 = MODE == kRopeFp8;
  constexpr uint32_t IDESC_S8 = make_idesc_f16(false, kTileM, kTileN, false);  // e4m3 x e4m3 (format 0)
  constexpr int QK_BYTES = kFp8 ? C::KB8 * kBlkBytes : C::TILE_BYTES;         // one q / k tile
  constexpr int ST = C::STAGES;
  constexpr int QB = C::QBUF;
  using B = Bars<ST, QB>;
  constexpr bool kBF16 = std::is_same<TI, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = make_idesc_f16(kBF16, kTileM, kTileN, false);
  constexpr uint32_t IDESC_O = make_idesc_f16(kBF16, kTileM, C::DP, true);
  constexpr uint32_t SW32 = 6;
  static_assert(B::COUNT * 8 + 16 <= C::BAR_BYTES, "barrier area");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * static_cast<uint32_t>(i); };
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + C::OFF_BAR + 8 * B::COUNT);
  volatile int* abort_flag = &ctl->abort;
  auto qbuf = [&](int x, int b) -> uint32_t { return C::OFF_Q + (x * QB + b) * C::TILE_BYTES; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int x = 0; x < 2; ++x) {
      for (int b = 0; b < QB; ++b) {
        mbar_init(bar(B::Q_FULL + x * QB + b), 1);
        mbar_init(bar(B::Q_READY + x * QB + b), kRopeThreads);
        // Q in TMEM: the rope warpgroup releases the smem buffer once it has
        // read it; otherwise the last S MMA of the unit does.
        mbar_init(bar(B::Q_EMPTY + x * QB + b), C::Q_TMEM ? kRopeThreads : 1);
      }
      mbar_init(bar(B::S_FULL + x), 1);
      mbar_init(bar(B::QT_FREE + x), 1);
      mbar_init(bar(B::P_FULL + x), kSoftmaxThreads);
      mbar_init(bar(B::O_FULL + x), 1);
    }
    for (int i = 0; i < ST; ++i) {
      mbar_init(bar(B::K_FULL + i), 1);
      mbar_init(bar(B::K_READY + i), kRopeThreads);
      mbar_init(bar(B::K_EMPTY + i), 1);
      mbar_init(bar(B::V_FULL + i), 1);
      mbar_init(bar(B::V_EMPTY + i), 1);
    }
    mbar_init(bar(B::CS_FULL), 1);
    mbar_init(bar(B::CS_EMPTY), kRopeThreads);
    mbar_init(bar(B::DONE), 1);
    ctl->abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmq);
    tma_prefetch_desc(&p.tmk);
    tma_prefetch_desc(&p.tmv);
    if (p.krot) tma_prefetch_desc(&p.tmk_rot);
    if (C::CS_BYTES) {
      tma_prefetch_desc(&p.tmcos);
      tma_prefetch_desc(&p.tmsin);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  // Everything above overlaps the previous kernel of this call (programmatic
  // dependent launch); the work list and rotated K are read only after this.
  griddep_wait();
  const int n_items = __ldcg(p.header);
  const int n_long = __ldcg(p.header + 1);
  const int n_units = n_long * p.H + (n_items - n_long) * ((p.H + 1) >> 1);
  const int wg = warp >> 2;

  if (wg == 0) {
    regs_dec<REG_CTRL>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- TMA producer
      uint32_t q_it[2] = {0, 0}, k_it = 0, v_it = 0, cs_it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Unit U = decode_unit(p, u, n_long);
        const int ns = U.has_b ? 2 : 1;
        if constexpr (C::CS_BYTES != 0) {
          ok = bounded_wait(bar(B::CS_EMPTY), (cs_it & 1) ^ 1, p, abort_flag,
                            FRATTN_STATUS_WAIT_TIMEOUT | 0x03);
          if (!ok) break;
          mbar_arrive_expect_tx(bar(B::CS_FULL), C::CS_BYTES);
          tma_load_2d(sbase + C::OFF_CS, &p.tmcos, bar(B::CS_FULL), 0, U.q0a);
          tma_load_2d(sbase + C::OFF_CS + C::CS_BYTES / 2, &p.tmsin, bar(B::CS_FULL), 0, U.q0a);
          ++cs_it;
        }
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (x >= ns || !ok) break;
          const int qs = q_it[x] % QB;
          ok = bounded_wait(bar(B::Q_EMPTY + x * QB + qs), ((q_it[x] / QB) & 1) ^ 1, p, abort_flag,
                            FRATTN_STATUS_WAIT_TIMEOUT | 0x00);
          if (!ok) break;
          const uint32_t fb = bar(B::Q_FULL + x * QB + qs);
          mbar_arrive_expect_tx(fb, QK_BYTES);
#pragma unroll
          for (int b = 0; b < (kFp8 ? C::KB8 : C::KB); ++b)
            tma_load_3d(sbase + qbuf(x, qs) + b * kBlkBytes, &p.tmq, fb, (kFp8 ? 32 : 16) * b, x ? U.hb : U.ha,
                        x ? U.q0b : U.q0a);
          ++q_it[x];
        }
        const int nkv = (U.kv1 - U.kv0 + kTileN - 1) / kTileN;
        const int nk = U.shared ? 1 : ns;
        const CUtensorMap* kmap = (U.shared && p.krot) ? &p.tmk_rot : &p.tmk;
        for (int j = 0; j < nkv && ok; ++j) {
          const int row = U.kv0 + j * kTileN;
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (x >= nk || !ok) break;
            const int hx = x ? U.hb : U.ha;
            const int ks = k_it % ST;
            ok = bounded_wait(bar(B::K_EMPTY + ks), ((k_it / ST) & 1) ^ 1, p, abort_flag,
                              FRATTN_STATUS_WAIT_TIMEOUT | 0x01);
            if (!ok) break;
            FR_TRACE((u - (int)blockIdx.x) / (int)gridDim.x, 0, j * 2 + x);
            mbar_arrive_expect_tx(bar(B::K_FULL + ks), QK_BYTES);
#pragma unroll
            for (int b = 0; b < (kFp8 ? C::KB8 : C::KB); ++b)
              tma_load_3d(sbase + C::OFF_K + ks * C::TILE_BYTES + b * kBlkBytes, kmap,
                          bar(B::K_FULL + ks), (kFp8 ? 32 : 16) * b, hx, row);
            ++k_it;
            const int vs = v_it % ST;
            ok = bounded_wait(bar(B::V_EMPTY + vs), ((v_it / ST) & 1) ^ 1, p, abort_flag,
                              FRATTN_STATUS_WAIT_TIMEOUT | 0x02);
            if (!ok) break;
            mbar_arrive_expect_tx(bar(B::V_FULL + vs), C::TILE_BYTES);
#pragma unroll
            for (int b = 0; b < C::KB; ++b)
              tma_load_3d(sbase + C::OFF_V + vs * C::TILE_BYTES + b * kBlkBytes, &p.tmv,
                          bar(B::V_FULL + vs), 16 * b, hx, row);
            ++v_it;
          }
        }
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------- MMA issuer
      if (lane == 0) {
        uint32_t q_it[2] = {0, 0}, k_it = 0, v_it = 0, p_it[2] = {0, 0};
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
          const Unit U = decode_unit(p, u, n_long);
          const int ui = (u - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x);
          (void)ui;
          const int ns = U.has_b ? 2 : 1;
          const int nk = U.shared ? 1 : ns;
          const int nkv = (U.kv1 - U.kv0 + kTileN - 1) / kTileN;
          int qs[2] = {0, 0};
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (x >= ns || !ok) break;
            qs[x] = q_it[x] % QB;
            ok = bounded_wait(bar(B::Q_READY + x * QB + qs[x]), (q_it[x] / QB) & 1, p, abort_flag,
                              FRATTN_STATUS_WAIT_TIMEOUT | 0x10);
          }
          if (!ok) break;
          uint32_t vprev[2] = {0, 0};
          for (int j = 0; j <= nkv && ok; ++j) {
#pragma unroll
            for (int x = 0; x < 2; ++x) {
              if (x >= ns || !ok) break;
              const uint32_t s_col = tmem + C::TMEM_S + 128u * x;
              if (j > 0) {
                // O_x (+)= P_x(j-1) V(j-1); P is read from TMEM (it aliases S_x).
                ok = bounded_wait(bar(B::P_FULL + x), p_it[x] & 1, p, abort_flag,
                                  FRATTN_STATUS_WAIT_TIMEOUT | 0x11);
                if (!ok) break;
                FR_TRACE(ui, 1, (j - 1) * 2 + x);
                ++p_it[x];
                const uint32_t vi = vprev[x];
                ok = bounded_wait(bar(B::V_FULL + vi % ST), (vi / ST) & 1, p, abort_flag,
                                  FRATTN_STATUS_WAIT_TIMEOUT | 0x12);
                if (!ok) break;
                FR_TRACE(ui, 2, (j - 1) * 2 + x);
                tc_fence_after();
                const uint32_t vaddr = sbase + C::OFF_V + (vi % ST) * C::TILE_BYTES;
                const uint64_t vdesc = make_sdesc(vaddr, kBlkBytes, 256, SW32);
#pragma unroll
                for (int kk = 0; kk < kTileN / 16; ++kk) {
                  // descriptor of the kk-th 16-row group: advance the start-address field
                  const uint64_t bd = vdesc + static_cast<uint64_t>((kk * 512) >> 4);
                  umma_ts(tmem + C::TMEM_O + 128u * x, s_col + kk * 8, bd, IDESC_O,
                          (j > 1 || kk > 0) ? 1u : 0u);
                }
                FR_TRACE(ui, 10, (j - 1) * 2 + x);
                if (!U.shared || x == ns - 1) umma_commit(bar(B::V_EMPTY + vi % ST));
                if (j == nkv) umma_commit(bar(B::O_FULL + x));
              }
              if (j < nkv) {
                // S_x(j) = Q_x K(j)^T
                const uint32_t ki = k_it + (U.shared ? 0 : x);
                ok = bounded_wait(bar(B::K_READY + ki % ST), (ki / ST) & 1, p, abort_flag,
                                  FRATTN_STATUS_WAIT_TIMEOUT | 0x13);
                if (!ok) break;
                FR_TRACE(ui, 3, j * 2 + x);
                tc_fence_after();
                const uint32_t qaddr = sbase + qbuf(x, qs[x]);
                const uint32_t kaddr = sbase + C::OFF_K + (ki % ST) * C::TILE_BYTES;
                const uint64_t qdesc = make_sdesc(qaddr, 16, 256, SW32);
                const uint64_t kdesc = make_sdesc(kaddr, 16, 256, SW32);
                if constexpr (kFp8) {
#pragma unroll
                  for (int kb = 0; kb < C::KB8; ++kb) {  // K = 32 e4m3 elements per MMA
                    const uint64_t o = static_cast<uint64_t>((kb * kBlkBytes) >> 4);
                    umma_ss_f8(s_col, qdesc + o, kdesc + o, IDESC_S8, kb > 0 ? 1u : 0u);
                  }
                } else {
#pragma unroll
                  for (int kb = 0; kb < C::KB; ++kb) {
                    const uint64_t bd = kdesc + static_cast<uint64_t>((kb * kBlkBytes) >> 4);
                    if constexpr (C::Q_TMEM) {
                      umma_ts(s_col, tmem + C::TMEM_Q + 128u * x + kb * 8, bd, IDESC_S, kb > 0 ? 1u : 0u);
                    } else {
                      const uint64_t ad = qdesc + static_cast<uint64_t>((kb * kBlkBytes) >> 4);
                      umma_ss(s_col, ad, bd, IDESC_S, kb > 0 ? 1u : 0u);
                    }
                  }
                }
                FR_TRACE(ui, 11, j * 2 + x);
                umma_commit(bar(B::S_FULL + x));
                FR_TRACE(ui, 4, j * 2 + x);
                if (!U.shared || x == ns - 1) umma_commit(bar(B::K_EMPTY + ki % ST));
                if (j == nkv - 1)
                  umma_commit(bar(C::Q_TMEM ? B::QT_FREE + x : B::Q_EMPTY + x * QB + qs[x]));
                vprev[x] = v_it + (U.shared ? 0 : x);
              }
            }
            if (j < nkv) {
              k_it += nk;
              v_it += nk;
            }
          }
          ++q_it[0];
          if (ns > 1) ++q_it[1];
        }
        // Drain: every issued MMA completes before TMEM is released.
        umma_commit(bar(B::DONE));
        bounded_wait(bar(B::DONE), 0, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x15);
      }
      __syncwarp();
    }
  } else if (wg == 1) {
    // ------------------------------------------------------------ RoPE warpgroup
    regs_dec<REG_ROPE>();
    const int r = threadIdx.x - 128;
    uint32_t q_it[2] = {0, 0}, k_it = 0, cs_it = 0;
    bool ok = true;
    const uint8_t* cs_tile = C::CS_BYTES ? smem + C::OFF_CS : nullptr;
    const uint32_t q_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);  // TMEM lane of row r
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const Unit U = decode_unit(p, u, n_long);
      const int ns = U.has_b ? 2 : 1;
      if constexpr (C::CS_BYTES != 0) {
        ok = bounded_wait(bar(B::CS_FULL), cs_it & 1, p, abort_flag,
                          FRATTN_STATUS_WAIT_TIMEOUT | 0x22);
        if (!ok) break;
        ++cs_it;
      }
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (x >= ns || !ok) break;
        const int qs = q_it[x] % QB;
        // warp-uniform result: the TMEM stores below are .sync.aligned
        ok = bounded_wait_warp(bar(B::Q_FULL + x * QB + qs), (q_it[x] / QB) & 1, p, abort_flag,
                               FRATTN_STATUS_WAIT_TIMEOUT | 0x20);
        if (!ok) break;
        const int qrow = x ? U.q0b : U.q0a;
        if constexpr (C::Q_TMEM) {
          // The slot's Q columns are free once the previous Q of this slot is
          // no longer read: its last S MMA committed QT_FREE.
          if (q_it[x] > 0) {
            ok = bounded_wait_warp(bar(B::QT_FREE + x), (q_it[x] - 1) & 1, p, abort_flag,
                                   FRATTN_STATUS_WAIT_TIMEOUT | 0x23);
            if (!ok) break;
          }
          tc_fence_after();
          rope_q_to_tmem<D, MODE, TI, TC>(smem + qbuf(x, qs), qrow, p, r,
                                          qrow == U.q0a ? cs_tile : nullptr,
                                          q_lane + C::TMEM_Q + 128u * x);
          mbar_arrive(bar(B::Q_EMPTY + x * QB + qs));  // smem tile read: reusable
          tmem_st_wait();
          tc_fence_before();
        } else {
          rope_tile<D, MODE, TI, TC>(smem + qbuf(x, qs), qrow, p, r,
                                     qrow == U.q0a ? cs_tile : nullptr);
          fence_proxy_async_smem();
        }
        mbar_arrive(bar(B::Q_READY + x * QB + qs));
        ++q_it[x];
      }
      const int nkv = (U.kv1 - U.kv0 + kTileN - 1) / kTileN;
      const int nk = U.shared ? 1 : ns;
      for (int j = 0; j < nkv && ok; ++j) {
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (x >= nk || !ok) break;
          const int ks = k_it % ST;
          ok = bounded_wait(bar(B::K_FULL + ks), (k_it / ST) & 1, p, abort_flag,
                            FRATTN_STATUS_WAIT_TIMEOUT | 0x21);
          if (!ok) break;
          const int krow = U.kv0 + j * kTileN;
          if (!(U.shared && p.krot))  // long segments: K arrives pre-rotated
            rope_tile<D, MODE, TI, TC>(smem + C::OFF_K + ks * C::TILE_BYTES, krow, p, r,
                                       krow == U.q0a ? cs_tile : nullptr);
          fence_proxy_async_smem();
          mbar_arrive(bar(B::K_READY + ks));
          ++k_it;
        }
      }
      if (C::CS_BYTES != 0 && ok) mbar_arrive(bar(B::CS_EMPTY));
    }
  } else {
    // ------------------------------------------------------------ softmax WGs
    regs_inc<REG_SOFTMAX>();
    const int x = wg - 2;                      // slot
    const int t = ((warp & 3) << 5) | lane;    // q row within the tile == TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_addr = lane_addr + C::TMEM_S + 128u * x;
    const uint32_t o_addr = lane_addr + C::TMEM_O + 128u * x;
    const float sl2_base = 1.4426950408889634f * rsqrtf(static_cast<float>(D));
    constexpr float kRescaleLog2 = 8.0f;  // move the reference max only when it grows by 2^8
    constexpr int kPolyOf8 = FRATTN_POLY_OF_8;
    uint32_t s_it = 0, o_it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const Unit U = decode_unit(p, u, n_long);
      const int ui = (u - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x);
      (void)ui;
      if (x == 1 && !U.has_b) continue;
      const int h = x ? U.hb : U.ha;
      const int q0x = x ? U.q0b : U.q0a;
      const int q1x = x ? U.q1b : U.q1a;
      const int nkv = (U.kv1 - U.kv0 + kTileN - 1) / kTileN;
      const int row = q0x + t;
      int lo = 0, hi = 0;
      if (row < q1x) {
        if (U.kind == kItemLong) {
          lo = U.kv0;
          hi = U.kv1;
        } else {
          const int s = upper_bound_cu(p.cu, U.seg_lo, U.seg_hi + 2, row) - 1;
          lo = __ldg(p.cu + s);
          hi = __ldg(p.cu + s + 1);
        }
      }
      float m_ref = -INFINITY, l = 0.f;
      // exponent factor of the raw scores (FP8: times the dequantisation scales)
      float sl2 = sl2_base;
      if constexpr (kFp8)
        sl2 *= __ldg(p.qscale + static_cast<size_t>(min(row, p.T - 1)) * p.H + h) * __ldg(p.kscale + h);
      for (int j = 0; j < nkv; ++j) {
        ok = bounded_wait_warp(bar(B::S_FULL + x), s_it & 1, p, abort_flag,
                               FRATTN_STATUS_WAIT_TIMEOUT | 0x30);
        if (!ok) break;
        if (t == 0) FR_TRACE(ui, 5, j * 2 + x);
        ++s_it;
        tc_fence_after();
        float s[kTileN];
#pragma unroll
        for (int c = 0; c < kTileN / 32; ++c) {
          uint32_t rr[32];
          tmem_ld32(s_addr + c * 32, rr);
#pragma unroll
          for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(rr[e]);
        }
        tmem_ld_wait();
        if (t == 0) FR_TRACE(ui, 6, j * 2 + x);

        const int c0 = U.kv0 + j * kTileN;
        const int lo_r = lo - c0, hi_r = hi - c0;
        if (lo_r > 0 || hi_r < kTileN) {
#pragma unroll
          for (int i = 0; i < kTileN; ++i)
            if (i < lo_r || i >= hi_r) s[i] = -INFINITY;
        }
        float mxq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) mxq[q] = fmaxf(s[2 * q], s[2 * q + 1]);
#pragma unroll
        for (int i = 8; i < kTileN; i += 8) {
#pragma unroll
          for (int q = 0; q < 4; ++q) mxq[q] = max3(mxq[q], s[i + 2 * q], s[i + 2 * q + 1]);
        }
        const float mx = max3(fmaxf(mxq[0], mxq[1]), mxq[2], mxq[3]);
        // The exponent reference only moves when the running max grows by more
        // than 2^8 (or is still -inf); the final 1/l uses the same reference,
        // so the result is exact up to rounding.
        float alpha = 1.f;
        bool rescale = false;
        if (mx > m_ref && (m_ref == -INFINITY || (mx - m_ref) * sl2 > kRescaleLog2)) {
          alpha = (m_ref == -INFINITY) ? 0.f : ex2((m_ref - mx) * sl2);
          rescale = l > 0.f;
          m_ref = mx;
        }
        const float mb = (m_ref == -INFINITY ? 0.f : m_ref) * sl2;
        // p = 2^(s*scale - ref): pairs in fp32x2; kPolyOf8 of every 8 pairs go
        // through the FMA-pipe exp2, the rest through MUFU ex2. P is written as
        // packed pairs over the first 64 TMEM columns of the S region (already
        // consumed into registers), 32 columns at a time.
        const uint64_t scale2 = f2pack(sl2, sl2);
        const uint64_t bias2 = f2pack(-mb, -mb);
        uint64_t sp2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int c = 0; c < kTileN / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint64_t xa = fma2(f2pack(s[c * 32 + 2 * e], s[c * 32 + 2 * e + 1]), scale2, bias2);
            uint64_t pp;
            if ((e & 7) < kPolyOf8) {
              pp = exp2_poly2(xa);
            } else {
              float a0, a1;
              f2unpack(xa, a0, a1);
              pp = f2pack(ex2(a0), ex2(a1));
            }
            sp2[e & 3] = add2(sp2[e & 3], pp);
            float p0, p1;
            f2unpack(pp, p0, p1);
            pk[e] = pack2<TI>(p0, p1);
          }
          tmem_st16(s_addr + c * 16, pk);
        }
        float sa, sb, sc, sd;
        f2unpack(add2(sp2[0], sp2[1]), sa, sb);
        f2unpack(add2(sp2[2], sp2[3]), sc, sd);
        const float sum = (sa + sb) + (sc + sd);
        l = l * alpha + sum;
        // O holds PV(j-1) complete: S_FULL(j) was committed after it.
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < C::DP / 16; ++c) {
            uint32_t rr[16];
            tmem_ld16(o_addr + c * 16, rr);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
            tmem_st16(o_addr + c * 16, rr);
          }
        }
        if (t == 0) FR_TRACE(ui, 7, j * 2 + x);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(B::P_FULL + x));
        if (t == 0) FR_TRACE(ui, 8, j * 2 + x);
      }
      if (!ok) break;
      // Epilogue: last PV of this slot done -> normalise and store the row.
      ok = bounded_wait_warp(bar(B::O_FULL + x), o_it & 1, p, abort_flag,
                             FRATTN_STATUS_WAIT_TIMEOUT | 0x32);
      if (!ok) break;
      ++o_it;
      if (t == 0) FR_TRACE(ui, 9, x);
      tc_fence_after();
      const bool store = lo < hi;
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      if (p.lse && row < q1x)  // log2 of the softmax denominator of the scaled scores
        p.lse[static_cast<size_t>(row) * p.H + h] =
            (store && l > 0.f) ? m_ref * sl2 + log2f(l) : -INFINITY;
      TI* orow = static_cast<TI*>(p.out) + (static_cast<size_t>(row) * p.H + h) * D;
      uint32_t oo[C::DP / 16][16];
#pragma unroll
      for (int c = 0; c < C::DP / 16; ++c) tmem_ld16(o_addr + c * 16, oo[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < C::DP / 16; ++c) {
        const uint32_t (&rr)[16] = oo[c];
        if (store) {
          uint4 w0, w1;
          w0.x = pack2<TI>(__uint_as_float(rr[0]) * inv_l, __uint_as_float(rr[1]) * inv_l);
          w0.y = pack2<TI>(__uint_as_float(rr[2]) * inv_l, __uint_as_float(rr[3]) * inv_l);
          w0.z = pack2<TI>(__uint_as_float(rr[4]) * inv_l, __uint_as_float(rr[5]) * inv_l);
          w0.w = pack2<TI>(__uint_as_float(rr[6]) * inv_l, __uint_as_float(rr[7]) * inv_l);
          w1.x = pack2<TI>(__uint_as_float(rr[8]) * inv_l, __uint_as_float(rr[9]) * inv_l);
          w1.y = pack2<TI>(__uint_as_float(rr[10]) * inv_l, __uint_as_float(rr[11]) * inv_l);
          w1.z = pack2<TI>(__uint_as_float(rr[12]) * inv_l, __uint_as_float(rr[13]) * inv_l);
          w1.w = pack2<TI>(__uint_as_float(rr[14]) * inv_l, __uint_as_float(rr[15]) * inv_l);
          if (c * 16 < D) reinterpret_cast<uint4*>(orow + c * 16)[0] = w0;
          if (c * 16 + 8 < D) reinterpret_cast<uint4*>(orow + c * 16)[1] = w1;
        }
      }
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ scheduler
// One CTA of 256 threads builds the work list from cu_seqlens (see the file
// header). Long items come first (largest kv ranges first per segment order),
// packed items after them.
constexpr int kPrepThreads = 256;

__device__ __forceinline__ int block_exclusive_scan(int v, int* tmp, int* total) {
  // Warp-shuffle scan, then a scan of the 32 warp totals by warp 0.
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) tmp[w] = x;
  __syncthreads();
  if (w == 0) {
    int y = lane < kPrepThreads / 32 ? tmp[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int z = __shfl_up_sync(0xffffffffu, y, off);
      if (lane >= off) y += z;
    }
    tmp[32 + lane] = y;  // inclusive scan of warp totals
  }
  __syncthreads();
  const int incl = x + (w > 0 ? tmp[32 + w - 1] : 0);
  *total = tmp[32 + kPrepThreads / 32 - 1];
  __syncthreads();
  return incl - v;
}

// upper_bound over cu_seqlens held in shared or global memory (plain loads).
__device__ __forceinline__ int upper_bound_any(const int32_t* cu, int lo, int hi, int x) {
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] > x) hi = mid; else lo = mid + 1;
  }
  return lo;
}

template <typename TI, int D>
__global__ void __launch_bounds__(kPrepThreads, 1)
    build_worklist(const int32_t* __restrict__ cu, int nseg, int T, int H, WorkItem* items,
                   int* header, TI* out, int32_t* status, const int32_t* pos_hw,
                   float* pos_tab, int pos_rows, float theta) {
  griddep_launch_dependents();  // dependents only start prologues; they wait for completion
  __shared__ int tmp[64];
  constexpr int kCuSmem = 8192;  // cu_seqlens entries staged in shared memory
  __shared__ int32_t s_cu[kCuSmem];
  const int tid = threadIdx.x;
  const bool cu_in_smem = nseg + 1 <= kCuSmem;
  if (cu_in_smem)
    for (int i = tid; i <= nseg; i += kPrepThreads) s_cu[i] = cu[i];
  __syncthreads();
  const int32_t* cuv = cu_in_smem ? s_cu : cu;

  // Validate cu_seqlens: non-decreasing, inside [0, T].
  int bad = 0;
  for (int s = tid; s <= nseg; s += kPrepThreads) {
    const int a = cuv[s];
    if (a < 0 || a > T) bad = 1;
    if (s < nseg && cuv[s + 1] < a) bad = 1;
  }
  bad = __syncthreads_or(bad);
  // (h, w) positions index a table of pos_rows rows: every one must be inside it.
  int bad_pos = 0;
  if (pos_hw != nullptr && !bad)
    for (int e = tid; e < 2 * T; e += kPrepThreads) {
      const int v = pos_hw[e];
      if (v < 0 || v >= pos_rows) bad_pos = 1;
    }
  bad_pos = __syncthreads_or(bad_pos);
  if (bad || bad_pos) {
    if (tid == 0) {
      header[0] = 0;
      header[1] = 0;
      if (status)
        atomicCAS(reinterpret_cast<int*>(status), 0,
                  bad ? FRATTN_STATUS_BAD_SEQLENS : FRATTN_STATUS_BAD_POSITIONS);
    }
    return;
  }

  // Rotary table for the (h, w)-position entry point: [P, D/4] cos, then sin.
  if (pos_tab != nullptr) {
    constexpr int Q4 = D / 4;
    for (int e = tid; e < pos_rows * Q4; e += kPrepThreads) {
      const int pos = e / Q4, i = e % Q4;
      // inv_freq[i] = 1 / theta^(2i / (D/2)), evaluated in fp32 like torch does
      const float inv = 1.0f / powf(theta, static_cast<float>(2 * i) / static_cast<float>(D / 2));
      const float ang = static_cast<float>(pos) * inv;
      float sv, cv;
      sincosf(ang, &sv, &cv);
      pos_tab[e] = cv;
      pos_tab[static_cast<size_t>(pos_rows) * Q4 + e] = sv;
    }
  }

  const int c_first = cuv[0], c_last = cuv[nseg];
  // Zero rows not covered by any segment.
  {
    const size_t row_elems = static_cast<size_t>(H) * D;  // multiple of 8
    const size_t n0 = static_cast<size_t>(c_first) * row_elems / 8;
    const size_t n1 = static_cast<size_t>(T - c_last) * row_elems / 8;
    uint4 z = make_uint4(0, 0, 0, 0);
    uint4* o0 = reinterpret_cast<uint4*>(out);
    uint4* o1 = reinterpret_cast<uint4*>(out + static_cast<size_t>(c_last) * row_elems);
    for (size_t i = tid; i < n0; i += kPrepThreads) o0[i] = z;
    for (size_t i = tid; i < n1; i += kPrepThreads) o1[i] = z;
  }

  int base = 0, total = 0;
  // Long items.
  for (int s0 = 0; s0 < nseg; s0 += kPrepThreads) {
    const int s = s0 + tid;
    int a = 0, b = 0, n = 0;
    if (s < nseg) {
      a = cuv[s];
      b = cuv[s + 1];
      if (b - a > kTileM) n = (b - a + 2 * kTileM - 1) / (2 * kTileM);
    }
    const int off = block_exclusive_scan(n, tmp, &total);
    for (int i = 0; i < n; ++i) {
      WorkItem w;
      w.q0 = a + i * 2 * kTileM;
      w.q1 = min(a + (i + 1) * 2 * kTileM, b);
      w.kv0 = a;
      w.kv1 = b;
      w.seg_lo = s;
      w.seg_hi = s;
      w.kind = kItemLong;
      w.pad = 0;
      items[base + off + i] = w;
    }
    base += total;
  }
  const int n_long = base;
  // Packed items: per 128-row chunk, the rows of short segments inside it.
  const int nch = (T + kTileM - 1) / kTileM;
  for (int c0 = 0; c0 < nch; c0 += kPrepThreads) {
    const int c = c0 + tid;
    int has = 0;
    WorkItem w;
    if (c < nch && c_first < c_last) {
      int a = max(c * kTileM, c_first);
      int e = min(c * kTileM + kTileM, min(T, c_last));
      if (a < e) {
        int sa = upper_bound_any(cuv, 0, nseg + 1, a) - 1;
        if (cuv[sa + 1] - cuv[sa] > kTileM) {
          a = cuv[sa + 1];
          if (a < e) sa = upper_bound_any(cuv, 0, nseg + 1, a) - 1;
        }
        if (a < e && cuv[sa + 1] - cuv[sa] <= kTileM) {
          int se = upper_bound_any(cuv, 0, nseg + 1, e - 1) - 1;
          if (cuv[se + 1] - cuv[se] > kTileM) {
            e = cuv[se];
            if (a < e) se = upper_bound_any(cuv, 0, nseg + 1, e - 1) - 1;
          }
          if (a < e) {
            has = 1;
            w.q0 = a;
            w.q1 = e;
            w.kv0 = cuv[sa];
            w.kv1 = cuv[se + 1];
            w.seg_lo = sa;
            w.seg_hi = se;
            w.kind = kItemPacked;
            w.pad = 0;
          }
        }
      }
    }
    const int off = block_exclusive_scan(has, tmp, &total);
    if (has) items[base + off] = w;
    base += total;
  }
  if (tid == 0) {
    header[0] = base;
    header[1] = n_long;
  }
}

// ------------------------------------------------------------------ launch
// cuTensorMapEncodeTiled from the driver (looked up once per process; nullptr
// when the driver does not provide it).
typedef CUresult (*TmapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
inline TmapEncodeFn tmap_encoder() {
  static TmapEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<TmapEncodeFn>(f);
  });
  return fn;
}

inline int sm_count_for_current_device() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

template <int D, int MODE, typename TI, typename TC>
int launch_attn(const Params& prm, cudaStream_t st) {
  using C = Cfg<D, MODE == kRopeTable ? static_cast<int>(sizeof(TC)) : 0, MODE == kRopeFp8>;
  auto kern = fused_rope_attn_kernel<D, MODE, TI, TC>;
  // Per-device flag; setting the attribute twice is harmless, so races are benign.
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
        cudaSuccess)
      return FRATTN_E_CUDA;
    attr_set |= bit;
  }
  const int grid = sm_count_for_current_device();
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t lc = {};
  lc.stream = st;
  lc.attrs = &attr;
  lc.numAttrs = 1;
  if (MODE != kRopeNone && MODE != kRopeFp8 && prm.krot) {
    lc.gridDim = dim3(2 * grid);
    lc.blockDim = dim3(256);
    lc.dynamicSmemBytes = 0;
    if constexpr (MODE != kRopeNone && MODE != kRopeFp8)
      if (cudaLaunchKernelEx(&lc, rotate_k_long<D, MODE, TI, TC>, prm) != cudaSuccess) return FRATTN_E_CUDA;
  }
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(kThreads);
  lc.dynamicSmemBytes = C::SMEM_BYTES;
  if (cudaLaunchKernelEx(&lc, kern, prm) != cudaSuccess) return FRATTN_E_CUDA;
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

template <int D, int MODE, typename TI>
int dispatch_cs(const Params& prm, int cs_dtype, cudaStream_t st) {
  if constexpr (MODE != kRopeTable) {  // no tables are read: one instantiation
    return launch_attn<D, MODE, TI, float>(prm, st);
  } else {
#ifdef FRATTN_FAST_BUILD  // experiment builds: fp32 tables only
    if (cs_dtype != FRATTN_F32) return FRATTN_E_DTYPE;
    return launch_attn<D, MODE, TI, float>(prm, st);
#else
    switch (cs_dtype) {
      case FRATTN_F32: return launch_attn<D, MODE, TI, float>(prm, st);
      case FRATTN_BF16: return launch_attn<D, MODE, TI, __nv_bfloat16>(prm, st);
      case FRATTN_F16: return launch_attn<D, MODE, TI, __half>(prm, st);
      default: return FRATTN_E_DTYPE;
    }
#endif
  }
}

template <int D, int MODE>
int dispatch_in(const Params& prm, int in_dtype, int cs_dtype, cudaStream_t st) {
  if (in_dtype == FRATTN_BF16) return dispatch_cs<D, MODE, __nv_bfloat16>(prm, cs_dtype, st);
#ifndef FRATTN_FAST_BUILD
  if (in_dtype == FRATTN_F16) return dispatch_cs<D, MODE, __half>(prm, cs_dtype, st);
#endif
  return FRATTN_E_DTYPE;
}

// ------------------------------------------------------------------ window kernel
// Window regime (every segment at most one tile long, e.g. the 8x8-patch
// windows of the vision tower): one CTA per (128-row chunk of the packed
// sequence, head), no work list and no persistent loop. Two CTAs share an SM
// (256 TMEM columns each), so the hardware overlaps one CTA's loads with the
// other's rotation, MMAs and softmax. The chunk's q rows attend to the
// segments that contain them: kv rows [kv0, kv1) from the first to the last of
// those segments, in 128-row K/V tiles (online softmax over the tiles, so any
// segmentation is handled; windows of up to 64 tokens give one tile).
// 128 threads, one q row each: RoPE of its Q row (into TMEM) and K row (in
// shared memory), softmax of its row, epilogue. Thread 0 also issues the TMA
// loads and the tcgen05 MMAs; the phases of a tile are separated by CTA
// barriers (the work of a CTA is one serial chain; overlap comes from the
// other CTA on the SM). 128 threads, because registers are charged per four
// warps: a fifth warp would cost a whole second group and halve residency.
constexpr int kWinThreads = 128;
constexpr int kWinStage = 1024;  // cu_seqlens entries staged in shared memory

// First index i in [0, n) with v[i] > x (n if none), v non-decreasing.
__device__ __forceinline__ int upper_bound_smem(const int* v, int n, int x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (v[mid] > x) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// First index i in [0, n) with cu[i] > x (n if none), cu non-decreasing: a
// 32-way search by one warp (every lane returns the result).
__device__ __forceinline__ int warp_upper_bound(const int32_t* cu, int n, int x, int lane) {
  int lo = 0, hi = n;  // the answer lies in [lo, hi]
  while (hi - lo > 32) {
    const int step = (hi - lo + 31) / 32;
    const int idx = lo + lane * step;
    const bool gt = idx >= hi || __ldg(cu + idx) > x;  // probes past the range count as above
    const uint32_t m = __ballot_sync(0xffffffffu, gt);
    const int f = m ? __ffs(m) - 1 : 32;  // first probe above x
    if (f == 0) return lo;
    const int nlo = lo + (f - 1) * step + 1;
    hi = f < 32 ? min(hi, lo + f * step) : hi;
    lo = nlo;
  }
  const int idx = lo + lane;
  const bool gt = idx < hi && __ldg(cu + idx) > x;
  const uint32_t m = __ballot_sync(0xffffffffu, gt);
  return m ? lo + __ffs(m) - 1 : hi;
}
constexpr int kWinSmemMin = 80 * 1024;  // keeps at most two CTAs (512 TMEM columns) per SM

template <int D, int CSB>
struct WinCfg {
  using C = Cfg<D, CSB>;
  static_assert(C::Q_TMEM, "window kernel: Q lives in TMEM behind O");
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + C::TILE_BYTES;
  static constexpr int OFF_V = OFF_K + C::TILE_BYTES;
  static constexpr int OFF_BAR = OFF_V + C::TILE_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int RAW = OFF_BAR + BAR_BYTES + 1024;  // +1024 alignment slack
  static constexpr int SMEM_BYTES = RAW < kWinSmemMin ? kWinSmemMin : RAW;
  static constexpr uint32_t TMEM_COLS = 256;
  static constexpr uint32_t TMEM_S = 0;    // S / P
  static constexpr uint32_t TMEM_O = 128;  // O (DP columns), rotated Q behind it
  static constexpr uint32_t TMEM_Q = TMEM_O + C::DP;
  static_assert(TMEM_Q + C::DP / 2 <= TMEM_COLS, "TMEM columns");
  // barriers (all single-arrival: TMA transactions or tcgen05 commits)
  static constexpr int Q_FULL = 0, K_FULL = 1, V_FULL = 2, S_FULL = 3, KV_EMPTY = 4, O_FULL = 5,
                       COUNT = 6;
};

// Rotate row r of a raw 128 x D tile with cos/sin held in registers (fp32,
// one rounding to the element type): into TMEM at column qcol as packed pairs
// (TO_TMEM) or in place in shared memory.
template <int D, typename TI, bool TO_TMEM, bool ROT = true>
__device__ __forceinline__ void rope_row_regs(uint8_t* tile, int r, const float (&cr)[D / 2],
                                              const float (&sr)[D / 2], uint32_t qcol) {
  static_assert(D % 16 == 0, "whole 8-element chunks");
  constexpr int NP = D / 16;
#pragma unroll
  for (int c = 0; c < NP; ++c) {
    const uint4 ua = *reinterpret_cast<const uint4*>(tile + chunk_off(r, c));
    const uint4 ub = *reinterpret_cast<const uint4*>(tile + chunk_off(r, c + NP));
    if constexpr (!ROT) {  // already rotated: copy to TMEM (in place: nothing to do)
      if constexpr (TO_TMEM) {
        tmem_st4(qcol + 4 * c, ua);
        tmem_st4(qcol + 4 * (c + NP), ub);
      }
      continue;
    }
    float x0[8], x1[8];
    unpack8<TI>(ua, x0);
    unpack8<TI>(ub, x1);
    uint4 oa, ob;
    uint32_t* wa = reinterpret_cast<uint32_t*>(&oa);
    uint32_t* wb = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const int i = 8 * c + e;
      wa[e / 2] = pack2<TI>(x0[e] * cr[i] - x1[e] * sr[i], x0[e + 1] * cr[i + 1] - x1[e + 1] * sr[i + 1]);
      wb[e / 2] = pack2<TI>(x0[e] * sr[i] + x1[e] * cr[i], x0[e + 1] * sr[i + 1] + x1[e + 1] * cr[i + 1]);
    }
    if constexpr (TO_TMEM) {
      tmem_st4(qcol + 4 * c, oa);
      tmem_st4(qcol + 4 * (c + NP), ob);
    } else {
      *reinterpret_cast<uint4*>(tile + chunk_off(r, c)) = oa;
      *reinterpret_cast<uint4*>(tile + chunk_off(r, c + NP)) = ob;
    }
  }
}

template <int D, typename TI, typename TC, int MODE = kRopeTable>
__global__ void __launch_bounds__(kWinThreads, 2) window_attn_kernel(const __grid_constant__ Params p) {
  static_assert(MODE == kRopeTable || MODE == kRopeNone, "window kernel: tables or pre-rotated");
  constexpr bool kRot = MODE == kRopeTable;
  using C = Cfg<D, static_cast<int>(sizeof(TC))>;
  using W = WinCfg<D, static_cast<int>(sizeof(TC))>;
  constexpr bool kBF16 = std::is_same<TI, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = make_idesc_f16(kBF16, kTileM, kTileN, false);
  constexpr uint32_t IDESC_O = make_idesc_f16(kBF16, kTileM, C::DP, true);
  constexpr uint32_t SW32 = 6;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + W::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * static_cast<uint32_t>(i); };
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + W::OFF_BAR + 8 * W::COUNT);
  volatile int* abort_flag = &ctl->abort;
  __shared__ int s_unit[6];        // kv0, kv1, first row, end row, staged cu entries, their first index
  __shared__ int s_cu[kWinStage];  // cu_seqlens, or cu_seqlens[sa .. se + 1] when long

  const int t = threadIdx.x;  // q row within the chunk == TMEM lane
  const int warp = t >> 5;
  const int lane = t & 31;
  const int h = blockIdx.x;
  const int q0 = blockIdx.y * kTileM;
  const int q1 = min(q0 + kTileM, p.T);
#ifdef FRATTN_TRACE
  // per-CTA global-timer stamps: [cta][event], events 0 entry, 1 unit known,
  // 2 Q rotated, 3 K arrived, 4 S ready, 5 P stored, 6 O ready, 7 exit
  const int tr_cta = blockIdx.y * gridDim.x + blockIdx.x;
#define WIN_TRACE(ev) \
  do { if (tr_cta < kTraceWords / 8) g_trace[tr_cta * 8 + (ev)] = globaltimer_ns(); } while (0)
#else
#define WIN_TRACE(ev) do { } while (0)
#endif
  if (t == 0) WIN_TRACE(0);

  // cos/sin of this thread's q row straight into registers (reused for its K
  // row when the K tile is the chunk itself, as for windows that do not cross
  // a chunk boundary); issued first so that the latency overlaps the rest.
  constexpr int RD = D / 2;
  float cr[RD], sr[RD];
  if constexpr (kRot) {
    const int rr = min(q0 + t, p.T - 1);
    const TC* cp = static_cast<const TC*>(p.cos) + static_cast<size_t>(rr) * RD;
    const TC* sp = static_cast<const TC*>(p.sin) + static_cast<size_t>(rr) * RD;
    if constexpr (RD % 8 == 0) {
#pragma unroll
      for (int i = 0; i < RD; i += 8) {
        float a[8], b[8];
        load8<TC>(cp + i, a);
        load8<TC>(sp + i, b);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          cr[i + e] = a[e];
          sr[i + e] = b[e];
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < RD; ++i) {
        cr[i] = to_f32<TC>(__ldg(cp + i));
        sr[i] = to_f32<TC>(__ldg(sp + i));
      }
    }
  }
  const int n_all = p.nseg + 1;
  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < W::COUNT; ++i) mbar_init(bar(i), 1);
      ctl->abort = 0;
      fence_mbar_init();
      fence_proxy_async_smem();
      // Q does not depend on the segmentation: load first.
      mbar_arrive_expect_tx(bar(W::Q_FULL), C::TILE_BYTES);
#pragma unroll
      for (int b = 0; b < C::KB; ++b)
        tma_load_3d(sbase + W::OFF_Q + b * kBlkBytes, &p.tmq, bar(W::Q_FULL), 16 * b, h, q0);
    }
    __syncwarp();
    tmem_alloc(smem_u32(&ctl->tmem_base), W::TMEM_COLS);
    tmem_relinquish();
  }
  // cu_seqlens into shared memory in one round of loads when it is short (the
  // usual case: a few hundred windows); a longer one is searched by warp 0.
  if (n_all <= kWinStage)
    for (int i = t; i < n_all; i += kWinThreads) s_cu[i] = __ldg(p.cu + i);
  if (warp == 1 && blockIdx.x == 0 && blockIdx.y == 0) {
    // cu_seqlens check (non-decreasing, inside [0, T]) by one warp per call.
    int bad = 0;
    for (int sg = lane; sg <= p.nseg; sg += 32) {
      const int v0 = __ldg(p.cu + sg);
      if (v0 < 0 || v0 > p.T) bad = 1;
      if (sg < p.nseg && __ldg(p.cu + sg + 1) < v0) bad = 1;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0 && p.status)
      atomicCAS(reinterpret_cast<int*>(p.status), 0, FRATTN_STATUS_BAD_SEQLENS);
  }
  __syncthreads();
  if (warp == 0) {
    // Segments of this chunk: [sa, se] contain rows [a, e) = [q0, q1) clipped
    // to [cu[0], cu[nseg]); kv rows [cu[sa], cu[se + 1]). Values are clamped
    // to [0, T] so that a malformed cu_seqlens (reported above) cannot send a
    // load or store out of bounds.
    const bool small = n_all <= kWinStage;
    auto cu_at = [&](int i) -> int { return small ? s_cu[i] : __ldg(p.cu + i); };
    const int cu_first = min(max(cu_at(0), 0), p.T);
    const int cu_last = min(max(cu_at(p.nseg), 0), p.T);
    const int a = max(q0, cu_first), e = min(q1, cu_last);
    int kv0 = 0, kv1 = 0, sa = 0, se = -1;
    if (a < e) {
      if (small) {
        sa = upper_bound_smem(s_cu, n_all, a) - 1;
        se = upper_bound_smem(s_cu, n_all, e - 1) - 1;
      } else {
        sa = warp_upper_bound(p.cu, n_all, a, lane) - 1;
        se = warp_upper_bound(p.cu, n_all, e - 1, lane) - 1;
      }
      sa = min(max(sa, 0), p.nseg - 1);
      se = min(max(se, sa), p.nseg - 1);
      kv0 = min(max(cu_at(sa), 0), p.T);
      kv1 = min(max(cu_at(se + 1), 0), p.T);
      if (kv1 < kv0) kv1 = kv0;
    }
    const int n_stage = se - sa + 2;  // entries cu[sa .. se + 1]
    if (lane == 0) {
      s_unit[0] = kv0;
      s_unit[1] = kv1;
      s_unit[2] = a;
      s_unit[3] = e;
      // staged entries for the row lookups: all of cu (base 0) or this chunk's
      s_unit[4] = a < e ? (small ? n_all : (n_stage <= kWinStage ? n_stage : 0)) : 0;
      s_unit[5] = small ? 0 : sa;
      if (kv1 > kv0) {  // first K/V tile right away
        mbar_arrive_expect_tx(bar(W::K_FULL), C::TILE_BYTES);
#pragma unroll
        for (int b = 0; b < C::KB; ++b)
          tma_load_3d(sbase + W::OFF_K + b * kBlkBytes, &p.tmk, bar(W::K_FULL), 16 * b, h, kv0);
        mbar_arrive_expect_tx(bar(W::V_FULL), C::TILE_BYTES);
#pragma unroll
        for (int b = 0; b < C::KB; ++b)
          tma_load_3d(sbase + W::OFF_V + b * kBlkBytes, &p.tmv, bar(W::V_FULL), 16 * b, h, kv0);
      }
    }
    __syncwarp();
    if (!small && a < e && n_stage <= kWinStage)
      for (int i = lane; i < n_stage; i += 32) s_cu[i] = __ldg(p.cu + sa + i);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int kv0 = s_unit[0], kv1 = s_unit[1], ra = s_unit[2], re = s_unit[3], n_cu = s_unit[4];
  const int cu_base = s_unit[5];
  const int nkv = (kv1 - kv0 + kTileN - 1) / kTileN;
  if (t == 0) WIN_TRACE(1);

  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const uint32_t s_addr = lane_addr + W::TMEM_S;
  const uint32_t o_addr = lane_addr + W::TMEM_O;
  const int row = q0 + t;
  int lo = 0, hi = 0;  // kv rows this q row attends to
  if (row >= ra && row < re) {
    if (n_cu > 0) {  // staged entries cu[cu_base .. cu_base + n_cu)
      const int i = min(max(upper_bound_smem(s_cu, n_cu, row), 1), n_cu - 1);
      lo = max(s_cu[i - 1], kv0);
      hi = min(s_cu[i], kv1);
      (void)cu_base;
    } else {
      const int sg = upper_bound_cu(p.cu, 0, p.nseg + 1, row) - 1;
      lo = max(__ldg(p.cu + sg), kv0);
      hi = min(__ldg(p.cu + sg + 1), kv1);
    }
  }
  bool ok = true;
  float m_ref = -INFINITY, l = 0.f;
  if (nkv > 0) {
    // rotated Q of row t into TMEM (A operand of S)
    ok = bounded_wait_warp(bar(W::Q_FULL), 0, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x58);
    if (ok) {
      rope_row_regs<D, TI, true, kRot>(smem + W::OFF_Q, t, cr, sr, lane_addr + W::TMEM_Q);
      tmem_st_wait();
    }
    if (t == 0) WIN_TRACE(2);
    // K tile 0: rotated before the tile loop, with the register cos/sin when the
    // tile is this chunk (they are dead afterwards).
    ok = ok && bounded_wait_warp(bar(W::K_FULL), 0, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x59);
    if (ok) {
      if (t == 0) WIN_TRACE(3);
      if (kv0 == q0)
        rope_row_regs<D, TI, false, kRot>(smem + W::OFF_K, t, cr, sr, 0);
      else
        rope_tile<D, MODE, TI, TC>(smem + W::OFF_K, kv0, p, t, nullptr);
      fence_proxy_async_smem();
    }
    const float sl2 = 1.4426950408889634f * rsqrtf(static_cast<float>(D));
    constexpr float kRescaleLog2 = 8.0f;
    for (int j = 0; j < nkv; ++j) {
      const int krow = kv0 + j * kTileN;
      if (j > 0 && t == 0) {  // next K/V tile once PV(j-1) has released the buffers
        ok = bounded_wait(bar(W::KV_EMPTY), (j - 1) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x51);
        if (ok) {
          mbar_arrive_expect_tx(bar(W::K_FULL), C::TILE_BYTES);
#pragma unroll
          for (int b = 0; b < C::KB; ++b)
            tma_load_3d(sbase + W::OFF_K + b * kBlkBytes, &p.tmk, bar(W::K_FULL), 16 * b, h, krow);
          mbar_arrive_expect_tx(bar(W::V_FULL), C::TILE_BYTES);
#pragma unroll
          for (int b = 0; b < C::KB; ++b)
            tma_load_3d(sbase + W::OFF_V + b * kBlkBytes, &p.tmv, bar(W::V_FULL), 16 * b, h, krow);
        }
      }
      // rotated K row t (in place, shared memory); tile 0 was rotated above
      if (j > 0) {
        ok = ok && bounded_wait_warp(bar(W::K_FULL), j & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x59);
        if (ok) {
          rope_tile<D, MODE, TI, TC>(smem + W::OFF_K, krow, p, t, nullptr);
          fence_proxy_async_smem();
        }
      }
      tc_fence_before();
      ok = __syncthreads_and(ok);
      tc_fence_after();
      if (!ok) break;
      if (t == 0) {  // S = Q K^T (Q from TMEM)
        const uint64_t kdesc = make_sdesc(sbase + W::OFF_K, 16, 256, SW32);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
          umma_ts(tmem + W::TMEM_S, tmem + W::TMEM_Q + kb * 8,
                  kdesc + static_cast<uint64_t>((kb * kBlkBytes) >> 4), IDESC_S, kb > 0 ? 1u : 0u);
        umma_commit(bar(W::S_FULL));
      }
      ok = bounded_wait_warp(bar(W::S_FULL), j & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x5A);
      if (!ok) break;
      if (t == 0 && j == 0) WIN_TRACE(4);
      tc_fence_after();
      const int lo_r = lo - krow, hi_r = hi - krow;
      // 32-column chunks that no row of this warp attends to keep P = 0 and
      // cost no exponentials (the other windows of the tile).
      uint32_t live = 0;
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c)
        if (__any_sync(0xffffffffu, lo_r < 32 * c + 32 && hi_r > 32 * c)) live |= 1u << c;
      float s[kTileN];
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t rr[32];
        if (live & (1u << c)) {
          tmem_ld32(s_addr + c * 32, rr);
#pragma unroll
          for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(rr[e]);
        }
      }
      tmem_ld_wait();
      float mxq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c) {
        if (!(live & (1u << c))) continue;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int i = c * 32 + e;
          if (i < lo_r || i >= hi_r) s[i] = -INFINITY;
        }
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            mxq[q] = max3(mxq[q], s[c * 32 + e + 2 * q], s[c * 32 + e + 2 * q + 1]);
        }
      }
      const float mx = max3(fmaxf(mxq[0], mxq[1]), mxq[2], mxq[3]);
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_ref && (m_ref == -INFINITY || (mx - m_ref) * sl2 > kRescaleLog2)) {
        alpha = (m_ref == -INFINITY) ? 0.f : ex2((m_ref - mx) * sl2);
        rescale = l > 0.f;
        m_ref = mx;
      }
      const float mb = (m_ref == -INFINITY ? 0.f : m_ref) * sl2;
      const uint64_t scale2 = f2pack(sl2, sl2);
      const uint64_t bias2 = f2pack(-mb, -mb);
      uint64_t sp2[4] = {0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t pk[16];
        if (live & (1u << c)) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint64_t xa = fma2(f2pack(s[c * 32 + 2 * e], s[c * 32 + 2 * e + 1]), scale2, bias2);
            float a0, a1;
            f2unpack(xa, a0, a1);
            const uint64_t pp = f2pack(ex2(a0), ex2(a1));
            sp2[e & 3] = add2(sp2[e & 3], pp);
            float p0, p1;
            f2unpack(pp, p0, p1);
            pk[e] = pack2<TI>(p0, p1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = 0u;
        }
        tmem_st16(s_addr + c * 16, pk);
      }
      float sa_, sb_, sc_, sd_;
      f2unpack(add2(sp2[0], sp2[1]), sa_, sb_);
      f2unpack(add2(sp2[2], sp2[3]), sc_, sd_);
      l = l * alpha + ((sa_ + sb_) + (sc_ + sd_));
      // O holds PV(j-1) complete: S(j) was issued after it by the same thread.
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < C::DP / 16; ++c) {
          uint32_t rr[16];
          tmem_ld16(o_addr + c * 16, rr);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
          tmem_st16(o_addr + c * 16, rr);
        }
      }
      if (t == 0 && j == 0) WIN_TRACE(5);
      tmem_st_wait();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (t == 0) {  // O += P V (P from TMEM, where it overwrote S)
        ok = bounded_wait(bar(W::V_FULL), j & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x54);
        if (ok) {
          const uint64_t vdesc = make_sdesc(sbase + W::OFF_V, kBlkBytes, 256, SW32);
#pragma unroll
          for (int kk = 0; kk < kTileN / 16; ++kk)
            umma_ts(tmem + W::TMEM_O, tmem + W::TMEM_S + kk * 8,
                    vdesc + static_cast<uint64_t>((kk * 512) >> 4), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(bar(W::KV_EMPTY));
          if (j == nkv - 1) umma_commit(bar(W::O_FULL));
        }
      }
    }
    ok = __syncthreads_and(ok);
    if (ok) ok = bounded_wait_warp(bar(W::O_FULL), 0, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x5B);
    if (t == 0) WIN_TRACE(6);
    tc_fence_after();
  }
  // Epilogue: normalise and store the row; rows outside every segment are 0.
  // (The TMEM loads are warp-wide; only the stores depend on the row.)
  {
    TI* orow = static_cast<TI*>(p.out) + (static_cast<size_t>(min(row, p.T - 1)) * p.H + h) * D;
    const bool has = ok && lo < hi && l > 0.f;
    const float inv_l = has ? 1.f / l : 0.f;
    if (p.lse && row < p.T)
      p.lse[static_cast<size_t>(row) * p.H + h] =
          has ? m_ref * (1.4426950408889634f * rsqrtf(static_cast<float>(D))) + log2f(l) : -INFINITY;
    uint32_t oo[C::DP / 16][16];
    if (nkv > 0) {
#pragma unroll
      for (int c = 0; c < C::DP / 16; ++c) tmem_ld16(o_addr + c * 16, oo[c]);
      tmem_ld_wait();
    }
#pragma unroll
    for (int c = 0; c < C::DP / 16; ++c) {
      const uint32_t (&rr)[16] = oo[c];
      uint4 w0, w1;
      w0.x = pack2<TI>(has ? __uint_as_float(rr[0]) * inv_l : 0.f, has ? __uint_as_float(rr[1]) * inv_l : 0.f);
      w0.y = pack2<TI>(has ? __uint_as_float(rr[2]) * inv_l : 0.f, has ? __uint_as_float(rr[3]) * inv_l : 0.f);
      w0.z = pack2<TI>(has ? __uint_as_float(rr[4]) * inv_l : 0.f, has ? __uint_as_float(rr[5]) * inv_l : 0.f);
      w0.w = pack2<TI>(has ? __uint_as_float(rr[6]) * inv_l : 0.f, has ? __uint_as_float(rr[7]) * inv_l : 0.f);
      w1.x = pack2<TI>(has ? __uint_as_float(rr[8]) * inv_l : 0.f, has ? __uint_as_float(rr[9]) * inv_l : 0.f);
      w1.y = pack2<TI>(has ? __uint_as_float(rr[10]) * inv_l : 0.f, has ? __uint_as_float(rr[11]) * inv_l : 0.f);
      w1.z = pack2<TI>(has ? __uint_as_float(rr[12]) * inv_l : 0.f, has ? __uint_as_float(rr[13]) * inv_l : 0.f);
      w1.w = pack2<TI>(has ? __uint_as_float(rr[14]) * inv_l : 0.f, has ? __uint_as_float(rr[15]) * inv_l : 0.f);
      if (row < q1) {
        if (c * 16 < D) reinterpret_cast<uint4*>(orow + c * 16)[0] = w0;
        if (c * 16 + 8 < D) reinterpret_cast<uint4*>(orow + c * 16)[1] = w1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, W::TMEM_COLS);
  }
  if (t == 0) WIN_TRACE(7);
#undef WIN_TRACE
}

// Launch of the window kernel; FRATTN_E_SHAPE when this head dim has none
// (the caller then uses the general path).
template <int D, typename TI, typename TC, int MODE = kRopeTable>
int launch_window(const Params& prm, cudaStream_t st) {
  if constexpr (!(Cfg<D, static_cast<int>(sizeof(TC))>::Q_TMEM)) {
    return FRATTN_E_SHAPE;
  } else {
    using W = WinCfg<D, static_cast<int>(sizeof(TC))>;
    auto kern = window_attn_kernel<D, TI, TC, MODE>;
    static unsigned long long attr_set = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set & bit)) {
      // two CTAs per SM need the largest shared-memory carve-out
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, W::SMEM_BYTES) !=
              cudaSuccess ||
          cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) !=
              cudaSuccess)
        return FRATTN_E_CUDA;
      attr_set |= bit;
    }
    const dim3 grid(prm.H, (prm.T + kTileM - 1) / kTileM);
    kern<<<grid, kWinThreads, W::SMEM_BYTES, st>>>(prm);
    return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
  }
}

template <int D, typename TI>
int window_cs(const Params& prm, int cs_dtype, cudaStream_t st, bool rotated = false) {
  if (rotated) return launch_window<D, TI, float, kRopeNone>(prm, st);
#ifdef FRATTN_FAST_BUILD
  if (cs_dtype != FRATTN_F32) return FRATTN_E_SHAPE;
  return launch_window<D, TI, float>(prm, st);
#else
  switch (cs_dtype) {
    case FRATTN_F32: return launch_window<D, TI, float>(prm, st);
    case FRATTN_BF16: return launch_window<D, TI, __nv_bfloat16>(prm, st);
    case FRATTN_F16: return launch_window<D, TI, __half>(prm, st);
    default: return FRATTN_E_DTYPE;
  }
#endif
}

}  // namespace frattn
