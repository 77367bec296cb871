// Backward pass of the fused 2D-RoPE + varlen attention (sm_100a).
//
// The reference is forward-only (fused_attn.py:246-423); this computes the
// gradients of O = softmax(R(Q) R(K)^T / sqrt(D)) V per cu_seqlens segment with
// respect to q, k and v (cos/sin are constants of the positions):
//   S = R(Q) R(K)^T, P = softmax(S / sqrt(D)) (recomputed from the forward's
//   base-2 log-sum-exp), dV = P^T dO, dP = dO V^T, dS = P o (dP - rowsum(dO o O)),
//   dR(Q) = dS R(K) / sqrt(D), dR(K) = dS^T R(Q) / sqrt(D), dq = R^T dR(Q), dk = R^T dR(K)
// with R^T the inverse rotation (x0 = y0 c + y1 s, x1 = -y0 s + y1 c).
//
// Kernels (one call):
//   bwd_prep      one thread per (token, head): rotated q and k into the
//                 workspace (fp32 math, one rounding, as the forward), the row
//                 term rowsum(dO o O), and a zeroed fp32 dq accumulator row
//   bwd_main      one CTA per (128-key chunk of the packed sequence, head),
//                 head dims that are multiples of 16 up to 128:
//                 the chunk's keys attend to the queries of their own segments,
//                 so the CTA walks the q tiles of the segments that overlap the
//                 chunk (windows: one tile; a long segment: all of its tiles).
//                 Per q tile, on the tensor cores (tcgen05, fp32 in TMEM):
//                   S^T = K Q^T and dP^T = V dO^T      (SS, keys = TMEM lanes)
//                   dV += P^T dO, dK += dS^T Q          (TS: P^T, dS^T from TMEM)
//                   dQ_tile = dS K                      (SS: dS^T written to smem
//                                                        as an MN-major A operand)
//                 The 256 compute threads (one key row and half of the columns
//                 each) turn S^T, dP^T into P^T and dS^T; 128 dQ threads add the
//                 dQ tile (q rows = TMEM lanes) to the fp32 [H, T, D] accumulator
//                 with vector atomics, one row per lane. dK is scaled and inverse-
//                 rotated in the epilogue; dV is stored as is.
//   bwd_dq        one thread per (token, head): dq = R^T(dq_acc / sqrt(D))
// Warp roles of bwd_main (448 threads): warp 0 TMA producer (K, V once; Q, dO
// per q tile, two stages), warp 1 TMEM owner + MMA issuer, warps 2-9 compute,
// warps 10-13 dQ (TMEM read and atomics, overlapping the next tile's compute).
// Every mbarrier wait is bounded (status code, unwind, TMEM freed).
#include "frattn_kernel.cuh"

namespace frattn {

unsigned long long frattn_wait_limit_ns();  // frattn.cu

struct BwdParams {
  CUtensorMap tmq, tmk, tmv, tmdo;  // rotated q, rotated k, v, dO: [T, H, D], box {16, 1, 128}
  const int32_t* cu;
  int nseg, T, H;
  const float* lse;     // [T, H] base-2 log-sum-exp of the scaled scores (forward)
  const float* delta;   // [H, T] rowsum(dO o O)
  float* dq_acc;        // [H, T, D] fp32
  void* dk;             // [T, H, D]
  void* dv;
  const void* cos;      // [T, D/2]
  const void* sin;
  int32_t* status;
  unsigned long long wait_limit_ns;
};

template <int D>
struct BwdCfg {
  static_assert(D % 16 == 0 && D >= 32 && D <= 128, "backward: D a multiple of 16 in [32, 128]");
  static constexpr int KB = D / 16;
  static constexpr int TILE = kTileM * D * 2;       // one 128 x D tile
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int DS_BYTES = 128 * 128 * 2;
  // Q / dO stages: two when they fit in 227 KB, else one (D = 128)
  static constexpr int QS = (2 + 4) * TILE + DS_BYTES + 2048 + 256 + 1024 <= 232448 ? 2 : 1;
  static constexpr int OFF_Q = OFF_V + TILE;         // [QS] stages
  static constexpr int OFF_DO = OFF_Q + QS * TILE;   // [QS]
  static constexpr int OFF_DS = OFF_DO + QS * TILE;  // dS^T as an MN-major [128 q x 128 keys] operand
  static constexpr int OFF_VEC = OFF_DS + DS_BYTES; // lse2, delta of the q tile: [2][2][128] fp32
  static constexpr int OFF_BAR = OFF_VEC + 2 * 2 * 128 * 4;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static_assert(SMEM <= 232448, "shared memory");
  // TMEM columns (every accumulator starts on a 128-column boundary): S^T / P^T,
  // then the dQ tile once dV has read P^T; dP^T / dS^T; dV; dK
  static constexpr uint32_t T_S = 0, T_DQ = 0, T_DP = 128, T_DV = 256, T_DK = 384;
  static_assert(D <= 128, "TMEM columns");
};

namespace {

__device__ __forceinline__ bool bwd_wait(uint32_t bar, uint32_t parity, const BwdParams& p,
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
__device__ __forceinline__ bool bwd_wait_warp(uint32_t bar, uint32_t parity, const BwdParams& p,
                                              volatile int* abort_flag, int code) {
  return __all_sync(0xffffffffu, bwd_wait(bar, parity, p, abort_flag, code));
}
__device__ __forceinline__ void bwd_drain(uint32_t bar, uint32_t parity, unsigned long long limit) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > limit) return;
}

// Segment s with cu[s] <= x < cu[s+1] (non-empty), or -1 when x lies outside [cu[0], cu[nseg]).
__device__ __forceinline__ int segment_of(const int32_t* cu, int nseg, int x) {
  if (x < __ldg(cu) || x >= __ldg(cu + nseg)) return -1;
  int lo = 0, hi = nseg + 1;  // first i with cu[i] > x
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(cu + mid) > x) hi = mid; else lo = mid + 1;
  }
  return lo - 1;
}

}  // namespace

// ------------------------------------------------------------------ prep
template <int D, typename TI, typename TC>
__global__ void __launch_bounds__(256) bwd_prep(const TI* __restrict__ q, const TI* __restrict__ k,
                                                const TI* __restrict__ o, const TI* __restrict__ dout,
                                                const TC* __restrict__ cos, const TC* __restrict__ sin,
                                                int T, int H, TI* __restrict__ qr, TI* __restrict__ kr,
                                                float* __restrict__ delta, float* __restrict__ dq_acc) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;  // (token, head)
  if (i >= static_cast<long long>(T) * H) return;
  const int t = static_cast<int>(i / H);
  const size_t base = static_cast<size_t>(i) * D;
  constexpr int NP = D / 16;
#pragma unroll 1
  for (int c = 0; c < NP; ++c) {
    float cs[8], sn[8];
    load8<TC>(cos + static_cast<size_t>(t) * (D / 2) + 8 * c, cs);
    load8<TC>(sin + static_cast<size_t>(t) * (D / 2) + 8 * c, sn);
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const TI* src = which ? k : q;
      TI* dst = which ? kr : qr;
      float x0[8], x1[8];
      unpack8<TI>(__ldg(reinterpret_cast<const uint4*>(src + base + 8 * c)), x0);
      unpack8<TI>(__ldg(reinterpret_cast<const uint4*>(src + base + D / 2 + 8 * c)), x1);
      uint4 a, b;
      uint32_t* wa = reinterpret_cast<uint32_t*>(&a);
      uint32_t* wb = reinterpret_cast<uint32_t*>(&b);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        wa[e / 2] = pack2<TI>(x0[e] * cs[e] - x1[e] * sn[e], x0[e + 1] * cs[e + 1] - x1[e + 1] * sn[e + 1]);
        wb[e / 2] = pack2<TI>(x0[e] * sn[e] + x1[e] * cs[e], x0[e + 1] * sn[e + 1] + x1[e + 1] * cs[e + 1]);
      }
      *reinterpret_cast<uint4*>(dst + base + 8 * c) = a;
      *reinterpret_cast<uint4*>(dst + base + D / 2 + 8 * c) = b;
    }
  }
  float acc = 0.f;
#pragma unroll 1
  for (int c = 0; c < D / 8; ++c) {
    float a[8], b[8];
    unpack8<TI>(__ldg(reinterpret_cast<const uint4*>(o + base + 8 * c)), a);
    unpack8<TI>(__ldg(reinterpret_cast<const uint4*>(dout + base + 8 * c)), b);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf(a[e], b[e], acc);
  }
  const int hh = static_cast<int>(i % H);
  delta[static_cast<size_t>(hh) * T + t] = acc;  // [H, T]
  float4* z = reinterpret_cast<float4*>(dq_acc + (static_cast<size_t>(hh) * T + t) * D);
#pragma unroll
  for (int c = 0; c < D / 4; ++c) z[c] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// ------------------------------------------------------------------ dq
template <int D, typename TI, typename TC>
__global__ void __launch_bounds__(256) bwd_dq(const float* __restrict__ dq_acc, const TC* __restrict__ cos,
                                              const TC* __restrict__ sin, int T, int H, TI* __restrict__ dq) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(T) * H) return;
  const int t = static_cast<int>(i / H);
  const size_t base = static_cast<size_t>(i) * D;
  const size_t abase = (static_cast<size_t>(i % H) * T + t) * D;  // accumulator is [H, T, D]
  const float scale = rsqrtf(static_cast<float>(D));
#pragma unroll 1
  for (int c = 0; c < D / 16; ++c) {
    float cs[8], sn[8];
    load8<TC>(cos + static_cast<size_t>(t) * (D / 2) + 8 * c, cs);
    load8<TC>(sin + static_cast<size_t>(t) * (D / 2) + 8 * c, sn);
    const float4* a4 = reinterpret_cast<const float4*>(dq_acc + abase + 8 * c);
    const float4* b4 = reinterpret_cast<const float4*>(dq_acc + abase + D / 2 + 8 * c);
    const float4 a0 = a4[0], a1 = a4[1], b0 = b4[0], b1 = b4[1];
    const float y0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float y1[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    uint4 oa, ob;
    uint32_t* wa = reinterpret_cast<uint32_t*>(&oa);
    uint32_t* wb = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      wa[e / 2] = pack2<TI>((y0[e] * cs[e] + y1[e] * sn[e]) * scale,
                            (y0[e + 1] * cs[e + 1] + y1[e + 1] * sn[e + 1]) * scale);
      wb[e / 2] = pack2<TI>((y1[e] * cs[e] - y0[e] * sn[e]) * scale,
                            (y1[e + 1] * cs[e + 1] - y0[e + 1] * sn[e + 1]) * scale);
    }
    *reinterpret_cast<uint4*>(dq + base + 8 * c) = oa;
    *reinterpret_cast<uint4*>(dq + base + D / 2 + 8 * c) = ob;
  }
}

// ------------------------------------------------------------------ main
// Timeline trace (build with -DFRATTN_BWD_TRACE): SM clock stamps of CTA 0's
// first 32 q tiles, read back with frattn_bwd_trace_read.
#ifdef FRATTN_BWD_TRACE
static __device__ unsigned long long g_bwd_trace[16 * 32];
#define BT(ev, i) do { if (blockIdx.x == 0 && blockIdx.y == 0 && (i) < 32) g_bwd_trace[(ev) * 32 + (i)] = clock64(); } while (0)
#else
#define BT(ev, i) do { } while (0)
#endif
// warp 0 TMA, warp 1 MMA, warps 2-9 compute, warps 10-13 dQ (144 registers per
// thread at one CTA per SM)
constexpr int kBwdThreads = 448;
template <int D, typename TI, typename TC>
__global__ void __launch_bounds__(kBwdThreads, 1) bwd_main(const __grid_constant__ BwdParams p) {
  using C = BwdCfg<D>;
  constexpr bool kBF16 = std::is_same<TI, __nv_bfloat16>::value;
  constexpr uint32_t SW32 = 6;
  constexpr uint32_t IDESC_SS = make_idesc_f16(kBF16, kTileM, kTileN, false);  // S^T, dP^T
  constexpr uint32_t IDESC_TS = make_idesc_f16(kBF16, kTileM, D, true);        // dV, dK (B MN-major)
  constexpr uint32_t IDESC_DQ = IDESC_TS | (1u << 15);                         // dQ: A MN-major too

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  enum { KV_FULL = 0, FULL = 1, EMPTY = 3, SD_FULL = 5, DS_READY = 6, DQ_FULL = 7, DQ_FREE = 8,
         DS_FREE = 9, ACC_FULL = 10, DRAIN = 11, VEC_READY = 12, NBAR = 14 };
  auto bar = [&](int i) { return smem_u32(bars + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* vec = reinterpret_cast<float*>(smem + C::OFF_VEC);  // [buf][lse2 | delta][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int kc0 = blockIdx.x * kTileM;
  const int kc1 = min(kc0 + kTileM, p.T);
  // q range: the segments that contain a key of this chunk
  const int cu0 = __ldg(p.cu), cun = __ldg(p.cu + p.nseg);
  const int kf = max(kc0, cu0), kl = min(kc1, cun) - 1;
  int qa = 0, qb = 0;
  if (kf <= kl) {
    qa = __ldg(p.cu + segment_of(p.cu, p.nseg, kf));
    qb = __ldg(p.cu + segment_of(p.cu, p.nseg, kl) + 1);
  }
  const int nq = (qb - qa + kTileM - 1) / kTileM;
  // The key chunks of one segment visit its q tiles in rotated orders, so that
  // their dQ additions land on different rows at any moment.
  const int q_first = nq > 0 ? static_cast<int>(blockIdx.x) % nq : 0;
  auto q_tile = [&](int i) { return qa + ((i + q_first) % nq) * kTileM; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < NBAR; ++i)
      mbar_init(bar(i), (i == DS_READY || i >= VEC_READY) ? 256 : i == DQ_FREE ? 128 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nq > 0) {
      // ------------------------------------------------------------ producer
      mbar_arrive_expect_tx(bar(KV_FULL), 2 * C::TILE);
#pragma unroll
      for (int b = 0; b < C::KB; ++b) {
        tma_load_3d(sbase + C::OFF_K + b * kBlkBytes, &p.tmk, bar(KV_FULL), 16 * b, h, kc0);
        tma_load_3d(sbase + C::OFF_V + b * kBlkBytes, &p.tmv, bar(KV_FULL), 16 * b, h, kc0);
      }
      int i = 0;
      for (; i < nq; ++i) {
        const int s = i % C::QS;
        if (!bwd_wait(bar(EMPTY + s), ((i / C::QS) & 1) ^ 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x61))
          break;
        const int q0 = q_tile(i);
        mbar_arrive_expect_tx(bar(FULL + s), 2 * C::TILE);
#pragma unroll
        for (int b = 0; b < C::KB; ++b) {
          tma_load_3d(sbase + C::OFF_Q + s * C::TILE + b * kBlkBytes, &p.tmq, bar(FULL + s), 16 * b, h, q0);
          tma_load_3d(sbase + C::OFF_DO + s * C::TILE + b * kBlkBytes, &p.tmdo, bar(FULL + s), 16 * b, h, q0);
        }
      }
      // copies in flight land before the CTA exits
      bwd_drain(bar(KV_FULL), 0, p.wait_limit_ns);
      for (int j = max(0, i - C::QS); j < i; ++j) bwd_drain(bar(FULL + j % C::QS), (j / C::QS) & 1, p.wait_limit_ns);
    }
  } else if (warp == 1) {
    if (lane == 0 && nq > 0) {
      // ------------------------------------------------------------ MMA issuer
      bool ok = bwd_wait(bar(KV_FULL), 0, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x62);
      const uint32_t kaddr = sbase + C::OFF_K, vaddr = sbase + C::OFF_V;
      const uint64_t k_k = make_sdesc(kaddr, 16, 256, SW32);          // K as a K-major operand
      const uint64_t v_k = make_sdesc(vaddr, 16, 256, SW32);
      const uint64_t k_mn = make_sdesc(kaddr, kBlkBytes, 256, SW32);  // K as an MN-major B
      const uint64_t ds_mn = make_sdesc(sbase + C::OFF_DS, kBlkBytes, 256, SW32);
      for (int i = 0; i < nq && ok; ++i) {
        const int s = i % C::QS;
        ok = bwd_wait(bar(FULL + s), (i / C::QS) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x63);
        BT(0, i);
        if (!ok) break;
        tc_fence_after();
        const uint32_t qaddr = sbase + C::OFF_Q + s * C::TILE, doaddr = sbase + C::OFF_DO + s * C::TILE;
        const uint64_t q_k = make_sdesc(qaddr, 16, 256, SW32), do_k = make_sdesc(doaddr, 16, 256, SW32);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb) {  // dP^T = V dO^T (dK(i-1) has read dS^T: in order)
          const uint64_t o = static_cast<uint64_t>((kb * kBlkBytes) >> 4);
          umma_ss(tmem + C::T_DP, v_k + o, do_k + o, IDESC_SS, kb > 0);
        }
        if (i > 0) {  // the S columns hold dQ(i-1) until the compute threads have read it
          ok = bwd_wait(bar(DQ_FREE), (i - 1) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x65);
          if (!ok) break;
          tc_fence_after();
        }
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb) {  // S^T = K Q^T
          const uint64_t o = static_cast<uint64_t>((kb * kBlkBytes) >> 4);
          umma_ss(tmem + C::T_S, k_k + o, q_k + o, IDESC_SS, kb > 0);
        }
        umma_commit(bar(SD_FULL));
        BT(1, i);
        ok = bwd_wait(bar(DS_READY), i & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x64);
        BT(2, i);
        if (!ok) break;
        tc_fence_after();
        const uint64_t do_mn = make_sdesc(doaddr, kBlkBytes, 256, SW32);
        const uint64_t q_mn = make_sdesc(qaddr, kBlkBytes, 256, SW32);
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {  // dV += P^T dO, dK += dS^T Q
          const uint64_t o = static_cast<uint64_t>((kk * 512) >> 4);
          const uint32_t acol = kk < 4 ? kk * 8 : 96 + (kk - 4) * 8;  // packed q columns 16 kk ..
          umma_ts(tmem + C::T_DV, tmem + C::T_S + acol, do_mn + o, IDESC_TS, (i > 0 || kk > 0));
          umma_ts(tmem + C::T_DK, tmem + C::T_DP + acol, q_mn + o, IDESC_TS, (i > 0 || kk > 0));
        }
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {  // dQ = dS K over the S columns (after dV read P^T)
          const uint64_t o = static_cast<uint64_t>((kk * 512) >> 4);
          umma_ss(tmem + C::T_DQ, ds_mn + o, k_mn + o, IDESC_DQ, kk > 0);
        }
        umma_commit(bar(DQ_FULL));
        BT(3, i);
        umma_commit(bar(EMPTY + s));
        umma_commit(bar(DS_FREE));
      }
      if (ok) umma_commit(bar(ACC_FULL));
      umma_commit(bar(DRAIN));
      bwd_drain(bar(DRAIN), 0, p.wait_limit_ns);
    }
  } else if (warp < 10) {
    // -------------------------------------------------------------- compute
    // 8 warps: warp w reads TMEM lane quarter w & 3 (rows t); the two warps of
    // a quarter split the work by column halves (hf = 0, 1).
    const int t = ((warp & 3) << 5) | lane;  // TMEM lane: key row (S^T, dP^T, dV, dK), q row (dQ)
    const int hf = (warp - 2) >> 2;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int key = kc0 + t;
    int klo = 0, khi = 0;
    if (key < kc1) {
      const int sk = segment_of(p.cu, p.nseg, key);
      if (sk >= 0) {
        klo = __ldg(p.cu + sk);
        khi = __ldg(p.cu + sk + 1);
      }
    }
    const float sl2 = 1.4426950408889634f * rsqrtf(static_cast<float>(D));
    // this thread's lse (half 0) or delta (half 1) value of row t of a q tile,
    // loaded one tile ahead
    auto row_term = [&](int q0) -> float {
      const int q = q0 + t;
      if (q >= qb) return 0.f;
      return hf ? __ldg(p.delta + static_cast<size_t>(h) * p.T + q)
                : __ldg(p.lse + static_cast<size_t>(q) * p.H + h);
    };
    float term = nq > 0 ? row_term(q_tile(0)) : 0.f;
    bool ok = true;
    for (int i = 0; i < nq && ok; ++i) {
      const int b = i & 1;
      const int q0 = q_tile(i);
      float* lsev = vec + b * 256;
      float* delv = lsev + 128;
      (hf ? delv : lsev)[t] = term;
      // (bounded barrier of the 256 compute threads: the tile's lse2 / delta are staged)
      mbar_arrive(bar(VEC_READY + b));
      ok = bwd_wait_warp(bar(VEC_READY + b), (i >> 1) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x6A);
      if (t == 0 && hf == 0) BT(4, i);
      if (ok) ok = bwd_wait_warp(bar(SD_FULL), i & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x66);
      if (t == 0 && hf == 0) BT(5, i);
      if (ok && i > 0)
        ok = bwd_wait_warp(bar(DS_FREE), (i - 1) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x67);
      if (!ok) break;
      tc_fence_after();
      const int lo_r = klo - q0, hi_r = khi - q0;  // valid q columns of this key row
      // Packed P^T / dS^T of 32-column chunk c go to TMEM columns pcol(c) (16 wide).
      // Half 0 (chunks 0, 1) writes columns 0..31, over S columns it has already
      // read; half 1 (chunks 3, then 2) writes 96..127, over its own chunk 3. The
      // two halves never write a column the other still has to read.
#pragma unroll 1
      for (int n = 0; n < 2; ++n) {
        const int c = hf ? 3 - n : n;
        const uint32_t pcol = hf ? 96u + 16u * (c - 2) : 16u * c;
        uint32_t sr[32], dr[32];
        tmem_ld32(lane_addr + C::T_S + 32 * c, sr);
        tmem_ld32(lane_addr + C::T_DP + 32 * c, dr);
        tmem_ld_wait();
        uint32_t pk[16], dk[16];
#pragma unroll
        for (int e4 = 0; e4 < 32; e4 += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(lsev + 32 * c + e4);
          const float4 d4 = *reinterpret_cast<const float4*>(delv + 32 * c + e4);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dl[4] = {d4.x, d4.y, d4.z, d4.w};
          float pv[4], dv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int col = 32 * c + e4 + u;
            const bool valid = col >= lo_r && col < hi_r;
            const float pe = valid ? ex2(__uint_as_float(sr[e4 + u]) * sl2 - lv[u]) : 0.f;
            pv[u] = pe;
            dv[u] = pe * (__uint_as_float(dr[e4 + u]) - dl[u]);
          }
          pk[e4 / 2] = pack2<TI>(pv[0], pv[1]);
          pk[e4 / 2 + 1] = pack2<TI>(pv[2], pv[3]);
          dk[e4 / 2] = pack2<TI>(dv[0], dv[1]);
          dk[e4 / 2 + 1] = pack2<TI>(dv[2], dv[3]);
        }
        tmem_st16(lane_addr + C::T_S + pcol, pk);
        tmem_st16(lane_addr + C::T_DP + pcol, dk);
        // dS^T row t, q columns [32c, 32c + 32): chunks 4c .. 4c + 3 of the MN-major operand
        uint8_t* ds = smem + C::OFF_DS;
#pragma unroll
        for (int m = 0; m < 4; ++m)
          *reinterpret_cast<uint4*>(ds + chunk_off(t, 4 * c + m)) =
              make_uint4(dk[4 * m], dk[4 * m + 1], dk[4 * m + 2], dk[4 * m + 3]);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(DS_READY));
      if (t == 0 && hf == 0) BT(6, i);
      if (i + 1 < nq) term = row_term(q_tile(i + 1));  // latency hidden by the dQ phase
    }
    // epilogue: half 0 stores dV as is, half 1 stores dK scaled and rotated back;
    // keys outside every segment get 0
    if (ok && nq > 0) ok = bwd_wait_warp(bar(ACC_FULL), 0, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x69);
    tc_fence_after();
    // (8-column TMEM chunks: a few registers at a time; loads are warp-wide,
    // stores only for rows that are keys of this chunk)
    const bool loaded = ok && nq > 0;
    const bool store = key < kc1 && (ok || nq == 0);
    const bool has = nq > 0 && klo < khi;
    const size_t base = (static_cast<size_t>(key) * p.H + h) * D;
    if (hf == 0) {
      TI* dvp = static_cast<TI*>(p.dv) + base;
#pragma unroll 1
      for (int c = 0; c < D / 8; ++c) {
        uint32_t a8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (loaded) {
          tmem_ld8(lane_addr + C::T_DV + 8 * c, a8);
          tmem_ld_wait();
        }
        uint4 w;
        uint32_t* ww = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 8; e += 2)
          ww[e / 2] = pack2<TI>(has ? __uint_as_float(a8[e]) : 0.f, has ? __uint_as_float(a8[e + 1]) : 0.f);
        if (store) *reinterpret_cast<uint4*>(dvp + 8 * c) = w;
      }
    } else {
      TI* dkp = static_cast<TI*>(p.dk) + base;
      const float scale = rsqrtf(static_cast<float>(D));
      const int krow = store ? key : 0;
      const TC* cr = static_cast<const TC*>(p.cos) + static_cast<size_t>(krow) * (D / 2);
      const TC* sr = static_cast<const TC*>(p.sin) + static_cast<size_t>(krow) * (D / 2);
#pragma unroll 1
      for (int c = 0; c < D / 16; ++c) {
        uint32_t y0r[8] = {0, 0, 0, 0, 0, 0, 0, 0}, y1r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (loaded) {
          tmem_ld8(lane_addr + C::T_DK + 8 * c, y0r);
          tmem_ld8(lane_addr + C::T_DK + D / 2 + 8 * c, y1r);
          tmem_ld_wait();
        }
        float cs[8], sn[8];
        load8<TC>(cr + 8 * c, cs);
        load8<TC>(sr + 8 * c, sn);
        uint4 oa, ob;
        uint32_t* wa = reinterpret_cast<uint32_t*>(&oa);
        uint32_t* wb = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float a[2], bb[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float y0 = has ? __uint_as_float(y0r[e + u]) * scale : 0.f;
            const float y1 = has ? __uint_as_float(y1r[e + u]) * scale : 0.f;
            a[u] = y0 * cs[e + u] + y1 * sn[e + u];
            bb[u] = y1 * cs[e + u] - y0 * sn[e + u];
          }
          wa[e / 2] = pack2<TI>(a[0], a[1]);
          wb[e / 2] = pack2<TI>(bb[0], bb[1]);
        }
        if (store) {
          *reinterpret_cast<uint4*>(dkp + 8 * c) = oa;
          *reinterpret_cast<uint4*>(dkp + D / 2 + 8 * c) = ob;
        }
      }
    }
  } else {
    // -------------------------------------------------------------- dQ warps
    // Read each q tile's dQ (TMEM lane = q row), free the columns for the next
    // S^T, and add the row to the fp32 [H, T, D] accumulator with vector atomics
    // (one row per lane: 32 different cache lines per instruction; same-line
    // vector atomics serialise in L2, and a staged bulk reduce-add drained its
    // shared memory at a few bytes per clock). The compute warps meanwhile go on
    // with the next tile.
    const int t = ((warp & 3) << 5) | lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    float* dq_head = p.dq_acc + static_cast<size_t>(h) * p.T * D;  // [T, D] of head h
    for (int i = 0; i < nq; ++i) {
      if (!bwd_wait_warp(bar(DQ_FULL), i & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x68)) break;
      tc_fence_after();
      // head dims up to 80 in one pass (registers); larger ones in two halves,
      // the columns freed after the second
      constexpr int NP = D <= 80 ? 1 : 2, W = D / NP;
      const int q = q_tile(i) + t;
      float4* dst = reinterpret_cast<float4*>(dq_head + static_cast<size_t>(q < qb ? q : 0) * D);
#pragma unroll 1
      for (int part = 0; part < NP; ++part) {
        uint32_t dq[W];
        static_assert(W % 8 == 0, "8-column TMEM chunks");
#pragma unroll
        for (int c = 0; c < W / 8; ++c)
          tmem_ld8(lane_addr + C::T_DQ + part * W + 8 * c, *reinterpret_cast<uint32_t(*)[8]>(&dq[8 * c]));
        tmem_ld_wait();
        if (part == NP - 1) {
          tc_fence_before();
          mbar_arrive(bar(DQ_FREE));  // the S columns may take the next S^T
        }
        if (q < qb) {
#pragma unroll
          for (int c = 0; c < W / 4; ++c)
            atomicAdd(dst + part * (W / 4) + c,
                      make_float4(__uint_as_float(dq[4 * c]), __uint_as_float(dq[4 * c + 1]),
                                  __uint_as_float(dq[4 * c + 2]), __uint_as_float(dq[4 * c + 3])));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host
static int make_rows_map(CUtensorMap* m, const void* base, int T, int H, int D, bool bf16) {
  const TmapEncodeFn enc = tmap_encoder();
  if (!enc) return FRATTN_E_TMAP;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {16, 1, static_cast<cuuint32_t>(kTileM)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FRATTN_E_TMAP;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct BwdLayout {
  size_t qr, kr, delta, dq_acc, total;
};
static BwdLayout bwd_layout(int T, int H, int D) {
  const size_t rows = static_cast<size_t>(T) * H;
  BwdLayout l;
  l.qr = 0;
  l.kr = align256(l.qr + rows * D * 2);
  l.delta = align256(l.kr + rows * D * 2);
  l.dq_acc = align256(l.delta + rows * 4);
  l.total = align256(l.dq_acc + rows * D * 4);
  return l;
}

template <int D, typename TI, typename TC>
static int launch_bwd(const void* q, const void* k, const void* v, const void* cos, const void* sin,
                      const int32_t* cu, int nseg, int T, int H, const void* out, const void* dout,
                      const float* lse, void* dq, void* dk, void* dv, uint8_t* ws, int32_t* status,
                      cudaStream_t st) {
  using C = BwdCfg<D>;
  const BwdLayout L = bwd_layout(T, H, D);
  TI* qr = reinterpret_cast<TI*>(ws + L.qr);
  TI* kr = reinterpret_cast<TI*>(ws + L.kr);
  float* delta = reinterpret_cast<float*>(ws + L.delta);
  float* dq_acc = reinterpret_cast<float*>(ws + L.dq_acc);
  const long long rows = static_cast<long long>(T) * H;
  const int pb = static_cast<int>((rows + 255) / 256);
  bwd_prep<D, TI, TC><<<pb, 256, 0, st>>>(static_cast<const TI*>(q), static_cast<const TI*>(k),
                                          static_cast<const TI*>(out), static_cast<const TI*>(dout),
                                          static_cast<const TC*>(cos), static_cast<const TC*>(sin), T, H, qr,
                                          kr, delta, dq_acc);
  if (cudaGetLastError() != cudaSuccess) return FRATTN_E_CUDA;
  BwdParams p;
  memset(&p, 0, sizeof(p));
  const bool bf16 = std::is_same<TI, __nv_bfloat16>::value;
  if (make_rows_map(&p.tmq, qr, T, H, D, bf16) || make_rows_map(&p.tmk, kr, T, H, D, bf16) ||
      make_rows_map(&p.tmv, v, T, H, D, bf16) || make_rows_map(&p.tmdo, dout, T, H, D, bf16))
    return FRATTN_E_TMAP;
  p.cu = cu;
  p.nseg = nseg;
  p.T = T;
  p.H = H;
  p.lse = lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk = dk;
  p.dv = dv;
  p.cos = cos;
  p.sin = sin;
  p.status = status;
  p.wait_limit_ns = frattn_wait_limit_ns();
  auto kern = bwd_main<D, TI, TC>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bitv = 1ull << (dev & 63);
  if (!(attr_set & bitv)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return FRATTN_E_CUDA;
    attr_set |= bitv;
  }
  kern<<<dim3((T + kTileM - 1) / kTileM, H), kBwdThreads, C::SMEM, st>>>(p);
  if (cudaGetLastError() != cudaSuccess) return FRATTN_E_CUDA;
  bwd_dq<D, TI, TC><<<pb, 256, 0, st>>>(dq_acc, static_cast<const TC*>(cos), static_cast<const TC*>(sin), T, H,
                                        static_cast<TI*>(dq));
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

template <int D, typename TI>
static int bwd_cs(int cs_dtype, const void* q, const void* k, const void* v, const void* cos, const void* sin,
                  const int32_t* cu, int nseg, int T, int H, const void* out, const void* dout, const float* lse,
                  void* dq, void* dk, void* dv, uint8_t* ws, int32_t* status, cudaStream_t st) {
  switch (cs_dtype) {
    case FRATTN_F32:
      return launch_bwd<D, TI, float>(q, k, v, cos, sin, cu, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    case FRATTN_BF16:
      return launch_bwd<D, TI, __nv_bfloat16>(q, k, v, cos, sin, cu, nseg, T, H, out, dout, lse, dq, dk, dv, ws,
                                              status, st);
    case FRATTN_F16:
      return launch_bwd<D, TI, __half>(q, k, v, cos, sin, cu, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    default: return FRATTN_E_DTYPE;
  }
}

template <int D>
static int bwd_in(int in_dtype, int cs_dtype, const void* q, const void* k, const void* v, const void* cos,
                  const void* sin, const int32_t* cu, int nseg, int T, int H, const void* out, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, uint8_t* ws, int32_t* status, cudaStream_t st) {
  if (in_dtype == FRATTN_BF16)
    return bwd_cs<D, __nv_bfloat16>(cs_dtype, q, k, v, cos, sin, cu, nseg, T, H, out, dout, lse, dq, dk, dv, ws,
                                    status, st);
  if (in_dtype == FRATTN_F16)
    return bwd_cs<D, __half>(cs_dtype, q, k, v, cos, sin, cu, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status,
                             st);
  return FRATTN_E_DTYPE;
}

}  // namespace frattn

extern "C" int frattn_workspace_bytes_bwd(int total_tokens, int num_heads, int head_dim, size_t* bytes) {
  if (!bytes) return FRATTN_E_NULL;
  if (total_tokens < 0 || num_heads <= 0 || head_dim <= 0) return FRATTN_E_SHAPE;
  *bytes = frattn::bwd_layout(total_tokens, num_heads, head_dim).total + 256;
  return 0;
}

extern "C" int frattn_bwd(const void* q, const void* k, const void* v, const void* cos, const void* sin,
                          int cs_dtype, const int32_t* cu_seqlens, int nseg, int T, int H, int D,
                          int in_dtype, const void* out, const void* dout, const float* lse, void* dq,
                          void* dk, void* dv, void* workspace, size_t workspace_bytes, int32_t* status,
                          void* stream) {
  using namespace frattn;
  if (!q || !k || !v || !cos || !sin || !cu_seqlens || !out || !dout || !lse || !dq || !dk || !dv || !workspace)
    return FRATTN_E_NULL;
  if (T < 0 || H <= 0 || nseg < 1) return FRATTN_E_SHAPE;
  if (D % 16 != 0 || D < 32 || D > 128) return FRATTN_E_SHAPE;
  if (static_cast<long long>(T) * H * D >= (1ll << 31)) return FRATTN_E_SHAPE;
  if (in_dtype != FRATTN_BF16 && in_dtype != FRATTN_F16) return FRATTN_E_DTYPE;
  if (cs_dtype != FRATTN_F32 && cs_dtype != FRATTN_BF16 && cs_dtype != FRATTN_F16) return FRATTN_E_DTYPE;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(q) || !a16(k) || !a16(v) || !a16(cos) || !a16(sin) || !a16(out) || !a16(dout) || !a16(dq) ||
      !a16(dk) || !a16(dv) || !a16(workspace) || (reinterpret_cast<uintptr_t>(lse) & 3u))
    return FRATTN_E_ALIGN;
  size_t need = 0;
  frattn_workspace_bytes_bwd(T, H, D, &need);
  if (workspace_bytes < need - 256) return FRATTN_E_WORKSPACE;
  if (T == 0) return 0;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (D) {
    case 32: return bwd_in<32>(in_dtype, cs_dtype, q, k, v, cos, sin, cu_seqlens, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    case 48: return bwd_in<48>(in_dtype, cs_dtype, q, k, v, cos, sin, cu_seqlens, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    case 64: return bwd_in<64>(in_dtype, cs_dtype, q, k, v, cos, sin, cu_seqlens, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    case 80: return bwd_in<80>(in_dtype, cs_dtype, q, k, v, cos, sin, cu_seqlens, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    case 96: return bwd_in<96>(in_dtype, cs_dtype, q, k, v, cos, sin, cu_seqlens, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    case 112: return bwd_in<112>(in_dtype, cs_dtype, q, k, v, cos, sin, cu_seqlens, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    case 128: return bwd_in<128>(in_dtype, cs_dtype, q, k, v, cos, sin, cu_seqlens, nseg, T, H, out, dout, lse, dq, dk, dv, ws, status, st);
    default: return FRATTN_E_SHAPE;
  }
}

#ifdef FRATTN_BWD_TRACE
extern "C" int frattn_bwd_trace_read(unsigned long long* host, int words) {
  if (words > 16 * 32) words = 16 * 32;
  return cudaMemcpyFromSymbol(host, frattn::g_bwd_trace, words * sizeof(unsigned long long)) == cudaSuccess ? 0 : 1;
}
#endif
