// QKV projection with rotary embedding applied in the GEMM epilogue (sm_100a).
//
//   qkv[t, :] = x[t, :] · Wᵀ + b         (W: [3·H·D, K], nn.Linear layout)
//   q, k heads of qkv rotated in place with cos/sin of token t (rotate-half)
//
// The reference's caller (bench.py:72-78 of sdan/fused-rope-attn) takes q, k
// from a projection and rotates them in a separate elementwise pass (or, in the
// fused kernel, once per q tile inside attention, fused_attn.py:340-345,
// 385-390). Here the projection's epilogue writes Q and K already rotated, so
// the attention that follows reads them as they are (frattn_fwd_rotated).
//
// Numerics: the fp32 accumulator plus bias is rounded to the element type (the
// value a plain projection would store), then rotated in fp32 and rounded once
// more, which is exactly what the rotation inside the attention kernels does
// to a stored q/k. V is stored as projected.
//
// Design (one persistent CTA per SM, 192 threads):
//   warp 0     TMA producer: 128 x 64 tiles of x and BN x 64 tiles of W
//              (128-byte swizzle, K-major) into an ST-stage ring
//   warp 1     TMEM owner + tcgen05.mma issuer: D[128 x BN] += A·Bᵀ, 4 MMAs
//              (K = 16) per stage, fp32 accumulators in TMEM, two accumulator
//              buffers of 256 columns so the epilogue of tile i overlaps the
//              main loop of tile i + 1
//   warps 2-5  epilogue: one output row per thread (TMEM lane), whole heads per
//              N tile (BN = floor(256 / D) heads), bias, rounding, rotation of
//              q / k heads, 16-byte stores
// Every mbarrier wait is bounded; on timeout the kernel records a status code,
// waits (bounded) for its own copies and MMAs in flight, frees TMEM and returns.
#include "frattn_kernel.cuh"

namespace frattn {

unsigned long long frattn_wait_limit_ns();  // frattn.cu

// Kernel choice for frattn_qkv_rope: CTA pairs (default) or single CTAs.
static int g_qkv_pairs = 1;
static bool qkv_use_pairs() { return g_qkv_pairs != 0; }

#ifndef FRATTN_QKV_EPI_WARPS
#define FRATTN_QKV_EPI_WARPS 4
#endif
// Epilogue warps: 4 (one per TMEM lane quarter) or 8 (two per quarter, taking
// alternate heads of a tile; 8 measured slower: register spills at 320 threads).
constexpr int kEpiWarps = FRATTN_QKV_EPI_WARPS;
constexpr int kHeadStep = kEpiWarps / 4;
constexpr int kQkvThreads = 64 + 32 * kEpiWarps;  // warp 0 TMA, warp 1 MMA, the rest epilogue

struct QkvParams {
  CUtensorMap tma_x, tma_w;
  CUtensorMap tma_out;  // [T, N] output, box {D, 128} (one head of one tile)
  const void* bias;  // [N] or nullptr
  const void* cos;   // [T, D/2]
  const void* sin;
  void* out;         // [T, N] (= [T, 3, H, D])
  int T, N, K, H;
  int n_tiles_n, n_tiles;
  int32_t* status;
  unsigned long long wait_limit_ns;
};

template <int D>
struct QkvCfg {
  static constexpr int HPT = 256 / D;  // whole heads per N tile
  static constexpr int BN = HPT * D;
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STG_BYTES = BM * BN * 2;  // output staging of one tile
  static constexpr int ST_FIT = (227 * 1024 - 2048 - STG_BYTES) / STAGE;
  static constexpr int ST = ST_FIT > 6 ? 6 : ST_FIT;
  static constexpr int OFF_STG = ST * STAGE;
  static constexpr int OFF_BAR = OFF_STG + STG_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;  // barriers + 1024-B alignment slack
  static_assert(BN % 16 == 0 && BN <= 256, "UMMA N");
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "128-B swizzle atoms");
  static_assert(ST >= 2, "pipeline depth");
};

namespace {

__device__ __forceinline__ bool qkv_wait(uint32_t bar, uint32_t parity, const QkvParams& p,
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

// Drain wait used while unwinding: ignores the abort flag, gives up after limit.
__device__ __forceinline__ void qkv_drain(uint32_t bar, uint32_t parity, unsigned long long limit) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > limit) return;
}

template <typename TI>
__device__ __forceinline__ void load8_in(const TI* src, float (&v)[8]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
  unpack8<TI>(a, v);
}

}  // namespace

// Epilogue of one tile for the thread of accumulator row `row` (row r of the
// CTA's 128): whole heads of the N tile [n0, n0 + HPT D) from TMEM columns acc..
// (bias, rounding to the input type, rotation of q / k heads) into the
// shared-memory staging boxes [HPT][128][D] that TMA stores then write out
// (rows of 32 threads land in one box: coalesced, full-sector writes, where
// per-thread row stores wrote 32 separate half sectors per instruction).
// cos / sin of the token of accumulator row `row`, loaded into registers before
// the tile's accumulator is ready (their latency then hides behind the main
// loop). Head dims above 80 load them per head instead (register budget).
template <int D>
struct QkvRowCs {
  static constexpr bool kPrefetch = D <= 80;
  float c[kPrefetch ? D / 2 : 1], s[kPrefetch ? D / 2 : 1];
};

template <int D, typename TC>
__device__ __forceinline__ void qkv_row_cs(const QkvParams& p, int row, int n0, QkvRowCs<D>& cs) {
  if constexpr (QkvRowCs<D>::kPrefetch) {
    if (row >= p.T || n0 >= 2 * p.H * D) return;  // no q / k head in this tile
    const TC* cr = static_cast<const TC*>(p.cos) + static_cast<size_t>(row) * (D / 2);
    const TC* sr = static_cast<const TC*>(p.sin) + static_cast<size_t>(row) * (D / 2);
#pragma unroll
    for (int c = 0; c < D / 16; ++c) {
      float a[8], b[8];
      load8<TC>(cr + 8 * c, a);
      load8<TC>(sr + 8 * c, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        cs.c[8 * c + e] = a[e];
        cs.s[8 * c + e] = b[e];
      }
    }
  }
}

// The tile's accumulator columns are released (lane 0 arrives on empty_bar, a
// shared::cluster address) as soon as the last head has been read from TMEM.
template <int D, int HPT, typename TI, typename TC>
__device__ __forceinline__ void qkv_tile_epilogue(const QkvParams& p, uint32_t acc, int row, int n0, uint8_t* stg,
                                                  int r, const QkvRowCs<D>& cs, uint32_t empty_bar, int h0) {
  const TI* bias = static_cast<const TI*>(p.bias);
#pragma unroll 1
  for (int hh = h0; hh < HPT; hh += kHeadStep) {
    const int n = n0 + hh * D;
    if (n >= p.N) break;
    uint32_t v[D];  // accumulator, then the finished values (fp32 bit patterns)
#pragma unroll
    for (int c = 0; c < D / 16; ++c) {
      uint32_t (&chunk)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[16 * c]);
      tmem_ld16(acc + hh * D + 16 * c, chunk);
    }
    tmem_ld_wait();
    if (hh + kHeadStep >= HPT || n + kHeadStep * D >= p.N) {  // this warp's last head: TMEM no longer read
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(empty_bar);
    }
    if (row >= p.T) continue;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      float b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (bias) load8_in<TI>(bias + n + 8 * c, b);
#pragma unroll
      for (int e = 0; e < 8; ++e)  // the value a plain projection stores
        v[8 * c + e] = __float_as_uint(to_f32<TI>(from_f32<TI>(__uint_as_float(v[8 * c + e]) + b[e])));
    }
    const int part = (n / D) / p.H;  // 0 q, 1 k, 2 v
    if (part < 2) {
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        float c8[8], s8[8];
        if constexpr (QkvRowCs<D>::kPrefetch) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            c8[e] = cs.c[8 * c + e];
            s8[e] = cs.s[8 * c + e];
          }
        } else {
          load8<TC>(static_cast<const TC*>(p.cos) + static_cast<size_t>(row) * (D / 2) + 8 * c, c8);
          load8<TC>(static_cast<const TC*>(p.sin) + static_cast<size_t>(row) * (D / 2) + 8 * c, s8);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x0 = __uint_as_float(v[8 * c + e]), x1 = __uint_as_float(v[8 * c + e + D / 2]);
          v[8 * c + e] = __float_as_uint(x0 * c8[e] - x1 * s8[e]);
          v[8 * c + e + D / 2] = __float_as_uint(x0 * s8[e] + x1 * c8[e]);
        }
      }
    }
    // row r of head hh's [128][D] staging box (written to global by a TMA store)
    uint4* dst = reinterpret_cast<uint4*>(stg + (static_cast<size_t>(hh) * 128 + r) * D * 2);
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      uint4 w;
      w.x = pack2<TI>(__uint_as_float(v[8 * c + 0]), __uint_as_float(v[8 * c + 1]));
      w.y = pack2<TI>(__uint_as_float(v[8 * c + 2]), __uint_as_float(v[8 * c + 3]));
      w.z = pack2<TI>(__uint_as_float(v[8 * c + 4]), __uint_as_float(v[8 * c + 5]));
      w.w = pack2<TI>(__uint_as_float(v[8 * c + 6]), __uint_as_float(v[8 * c + 7]));
      dst[c] = w;
    }
  }
}

template <int D, typename TI, typename TC>
__global__ void __launch_bounds__(kQkvThreads, 1) qkv_rope_gemm_kernel(const __grid_constant__ QkvParams p) {
  using C = QkvCfg<D>;
  constexpr int ST = C::ST;
  constexpr bool kBF16 = std::is_same<TI, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = make_idesc_f16(kBF16, C::BM, C::BN, false);
  constexpr uint32_t SW128 = 2;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  // full[ST] empty[ST] acc_full[2] acc_empty[2] drain
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int FULL = 0, EMPTY = ST, ACC_FULL = 2 * ST, ACC_EMPTY = 2 * ST + 2, DRAIN = 2 * ST + 4;
  const int STG_FREE = 2 * ST + 5, STG_FULL = 2 * ST + 6;  // output staging reusable / written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), kEpiWarps);
    }
    mbar_init(bar(DRAIN), 1);
    mbar_init(bar(STG_FREE), 1);
    mbar_init(bar(STG_FULL), 32 * kEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tma_x);
    tma_prefetch_desc(&p.tma_w);
    tma_prefetch_desc(&p.tma_out);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nk = (p.K + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.n_tiles_n) * C::BM, n0 = (t % p.n_tiles_n) * C::BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % ST;
          if (!qkv_wait(bar(EMPTY + s), ((it / ST) & 1) ^ 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x31)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + s * C::STAGE;
          mbar_arrive_expect_tx(bar(FULL + s), C::STAGE);
          tma_load_2d(smem_u32(a), &p.tma_x, bar(FULL + s), kb * C::BK, m0);
          tma_load_2d(smem_u32(a + C::A_BYTES), &p.tma_w, bar(FULL + s), kb * C::BK, n0);
        }
      }
      // copies still in flight land before the CTA exits (normally none)
      const uint32_t first = it > static_cast<uint32_t>(ST) ? it - ST : 0;
      for (uint32_t i = first; i < it; ++i) qkv_drain(bar(FULL + i % ST), (i / ST) & 1, p.wait_limit_ns);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!qkv_wait(bar(ACC_EMPTY + buf), ((lt >> 1) & 1) ^ 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x32))
          break;
        tc_fence_after();
        const uint32_t d = tmem + buf * 256u;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % ST;
          if (!qkv_wait(bar(FULL + s), (it / ST) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x33)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * C::STAGE);
          const uint64_t ad = make_sdesc(a, 16, 1024, SW128);
          const uint64_t bd = make_sdesc(a + C::A_BYTES, 16, 1024, SW128);
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk)  // +32 B per K=16 step inside the swizzle atom
            umma_ss(d, ad + 2 * kk, bd + 2 * kk, IDESC, (kb | kk) != 0);
          umma_commit(bar(EMPTY + s));
        }
        if (ok) umma_commit(bar(ACC_FULL + buf));
      }
      // every MMA issued above has finished before TMEM is freed
      umma_commit(bar(DRAIN));
      qkv_drain(bar(DRAIN), 0, p.wait_limit_ns);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int ew = warp & 3;  // TMEM lane quarter this warp may access
    const int r = ew * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(ew * 32) << 16);
    const bool store_leader = warp == 2 && lane == 0;  // issues the tile's TMA stores
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      const int m0p = (t / p.n_tiles_n) * C::BM, n0p = (t % p.n_tiles_n) * C::BN;
      QkvRowCs<D> rcs;
      qkv_row_cs<D, TC>(p, m0p + r, n0p, rcs);  // before the accumulator wait
      const bool ok = qkv_wait(bar(ACC_FULL + buf), (lt >> 1) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x34);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m0 = (t / p.n_tiles_n) * C::BM, n0 = (t % p.n_tiles_n) * C::BN;
      // the staging boxes are free once the previous tile's TMA stores have read them
      if (lt > 0) {
        if (store_leader) {
          bulk_wait_read_all();
          mbar_arrive(bar(STG_FREE));
        }
        if (!__all_sync(0xffffffffu, qkv_wait(bar(STG_FREE), (lt - 1) & 1, p, abort_flag,
                                              FRATTN_STATUS_WAIT_TIMEOUT | 0x3A)))
          break;
      }
      qkv_tile_epilogue<D, C::HPT, TI, TC>(p, lane_base + buf * 256u, m0 + r, n0, smem + C::OFF_STG, r, rcs,
                                           mapa_shared(bar(ACC_EMPTY + buf), cluster_ctarank()), (warp - 2) >> 2);
      fence_proxy_async_smem();  // staging writes visible to the TMA stores
      mbar_arrive(bar(STG_FULL));
      if (store_leader) {
        if (!qkv_wait(bar(STG_FULL), lt & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x3B)) break;
#pragma unroll 1
        for (int hh = 0; hh < C::HPT; ++hh)
          if (n0 + hh * D < p.N)
            tma_store_2d(&p.tma_out, smem_u32(smem + C::OFF_STG) + hh * 128 * D * 2, n0 + hh * D, m0);
        bulk_commit_group();
      }
    }
    if (store_leader) bulk_wait_all();  // output written before the CTA ends
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ CTA pairs
// The same GEMM on CTA pairs (cluster of 2, tcgen05 cta_group::2): one MMA of
// M = 256 spans both CTAs. Each CTA loads its own 128 rows of x and half of the
// N tile's W rows (BN/2), so a pair moves 2 x (16 + BN/16) KB per 64-wide K step
// for twice the FLOPs of one CTA: a third less operand traffic per FLOP than the
// single-CTA kernel. Each CTA's TMEM holds its 128 accumulator rows x BN columns
// (two buffers); both CTAs run the epilogue of their rows. The leader CTA (rank
// 0) owns the stage barriers that count both CTAs' TMA bytes and issues the
// MMAs; its commits arrive on both CTAs' barriers (multicast commit); the peer's
// epilogue warps arrive on the leader's accumulator-free barrier.
template <int D>
struct QkvPairCfg {
  static constexpr int HPT = 256 / D;
  static constexpr int BN = HPT * D;  // N tile of the pair
  static constexpr int BNH = BN / 2;  // W rows loaded by each CTA
  static constexpr int BK = 64;
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = BNH * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STG_BYTES = 128 * BN * 2;  // output staging of the CTA's 128 rows
  static constexpr int ST_FIT = (227 * 1024 - 2048 - STG_BYTES) / STAGE;
  static constexpr int ST = ST_FIT > 6 ? 6 : ST_FIT;
  static constexpr int OFF_STG = ST * STAGE;
  static constexpr int OFF_BAR = OFF_STG + STG_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static_assert(BN % 16 == 0 && BN <= 256 && BNH % 8 == 0, "UMMA N / swizzle atoms");
  static_assert(B_BYTES % 1024 == 0, "128-B swizzle atoms");
};

template <int D, typename TI, typename TC>
__global__ void __launch_bounds__(kQkvThreads, 1) qkv_rope_gemm_pair_kernel(const __grid_constant__ QkvParams p) {
  using C = QkvPairCfg<D>;
  constexpr int ST = C::ST;
  constexpr bool kBF16 = std::is_same<TI, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = make_idesc_f16(kBF16, 256, C::BN, false);
  constexpr uint32_t SW128 = 2;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int FULL = 0, EMPTY = ST, ACC_FULL = 2 * ST, ACC_EMPTY = 2 * ST + 2, DRAIN = 2 * ST + 4;
  const int STG_FREE = 2 * ST + 5, STG_FULL = 2 * ST + 6;  // output staging reusable / written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(bar(FULL + i), 1);   // the leader's producer arrives; both CTAs' bytes complete it
      mbar_init(bar(EMPTY + i), 1);  // multicast commit of the leader's MMAs
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), 2 * kEpiWarps);  // epilogue warps of both CTAs (used in the leader)
    }
    mbar_init(bar(DRAIN), 1);
    mbar_init(bar(STG_FREE), 1);
    mbar_init(bar(STG_FULL), 32 * kEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tma_x);
    tma_prefetch_desc(&p.tma_w);
    tma_prefetch_desc(&p.tma_out);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nk = (p.K + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer (both CTAs)
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; t < p.n_tiles && ok; t += npairs) {
        const int m0 = (t / p.n_tiles_n) * 256 + 128 * static_cast<int>(rank);
        const int n0 = (t % p.n_tiles_n) * C::BN + C::BNH * static_cast<int>(rank);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % ST;
          if (!qkv_wait(bar(EMPTY + s), ((it / ST) & 1) ^ 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x35)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(bar(FULL + s), 2 * C::STAGE);
          const uint32_t full0 = mapa_shared(bar(FULL + s), 0);  // the leader's stage barrier
          uint8_t* a = smem + s * C::STAGE;
          tma_load_2d_pair(smem_u32(a), &p.tma_x, full0, kb * C::BK, m0);
          tma_load_2d_pair(smem_u32(a + C::A_BYTES), &p.tma_w, full0, kb * C::BK, n0);
        }
      }
      if (leader) {  // copies of both CTAs still in flight land before the pair exits
        const uint32_t first = it > static_cast<uint32_t>(ST) ? it - ST : 0;
        for (uint32_t i = first; i < it; ++i) qkv_drain(bar(FULL + i % ST), (i / ST) & 1, p.wait_limit_ns);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------------------------------------------------- MMA issuer (leader)
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = pair; t < p.n_tiles && ok; t += npairs, ++lt) {
        const int buf = lt & 1;
        if (!qkv_wait(bar(ACC_EMPTY + buf), ((lt >> 1) & 1) ^ 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x36))
          break;
        tc_fence_after();
        const uint32_t d = tmem + buf * 256u;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % ST;
          if (!qkv_wait(bar(FULL + s), (it / ST) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x37)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * C::STAGE);
          const uint64_t ad = make_sdesc(a, 16, 1024, SW128);
          const uint64_t bd = make_sdesc(a + C::A_BYTES, 16, 1024, SW128);
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk)
            umma_ss_pair(d, ad + 2 * kk, bd + 2 * kk, IDESC, (kb | kk) != 0);
          umma_commit_pair_mc(bar(EMPTY + s), 0x3);
        }
        if (ok) umma_commit_pair_mc(bar(ACC_FULL + buf), 0x3);
      }
      umma_commit_pair_mc(bar(DRAIN), 0x1);
      qkv_drain(bar(DRAIN), 0, p.wait_limit_ns);
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int ew = warp & 3;
    const int r = ew * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(ew * 32) << 16);
    const uint32_t acc_empty0 = mapa_shared(bar(ACC_EMPTY), 0);
    const bool store_leader = warp == 2 && lane == 0;  // issues the tile's TMA stores
    uint32_t lt = 0;
    for (int t = pair; t < p.n_tiles; t += npairs, ++lt) {
      const int buf = lt & 1;
      const int m0p = (t / p.n_tiles_n) * 256 + 128 * static_cast<int>(rank), n0p = (t % p.n_tiles_n) * C::BN;
      QkvRowCs<D> rcs;
      qkv_row_cs<D, TC>(p, m0p + r, n0p, rcs);  // before the accumulator wait
      const bool ok = qkv_wait(bar(ACC_FULL + buf), (lt >> 1) & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x38);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m0 = (t / p.n_tiles_n) * 256 + 128 * static_cast<int>(rank), n0 = (t % p.n_tiles_n) * C::BN;
      // the staging boxes are free once the previous tile's TMA stores have read them
      if (lt > 0) {
        if (store_leader) {
          bulk_wait_read_all();
          mbar_arrive(bar(STG_FREE));
        }
        if (!__all_sync(0xffffffffu, qkv_wait(bar(STG_FREE), (lt - 1) & 1, p, abort_flag,
                                              FRATTN_STATUS_WAIT_TIMEOUT | 0x3A)))
          break;
      }
      qkv_tile_epilogue<D, C::HPT, TI, TC>(p, lane_base + buf * 256u, m0 + r, n0, smem + C::OFF_STG, r, rcs,
                                           acc_empty0 + 8u * buf, (warp - 2) >> 2);
      fence_proxy_async_smem();  // staging writes visible to the TMA stores
      mbar_arrive(bar(STG_FULL));
      if (store_leader) {
        if (!qkv_wait(bar(STG_FULL), lt & 1, p, abort_flag, FRATTN_STATUS_WAIT_TIMEOUT | 0x3B)) break;
#pragma unroll 1
        for (int hh = 0; hh < C::HPT; ++hh)
          if (n0 + hh * D < p.N)
            tma_store_2d(&p.tma_out, smem_u32(smem + C::OFF_STG) + hh * 128 * D * 2, n0 + hh * D, m0);
        bulk_commit_group();
      }
    }
    if (store_leader) bulk_wait_all();  // output written before the CTA ends
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its pair may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// [rows, K] row-major matrix (row stride ld elements) as a 2-D TMA map with
// box {64, box_rows} and 128-byte swizzle.
static int make_kmajor_map(CUtensorMap* m, const void* base, int rows, int K, long long ld,
                           int box_rows, bool bf16) {
  const TmapEncodeFn enc = tmap_encoder();
  if (!enc) return FRATTN_E_TMAP;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FRATTN_E_TMAP;
}

// [T, N] output as a 2-D TMA map with box {D, 128} (one head of a 128-row tile),
// no swizzle: the staging boxes are dense [128][D] rows.
static int make_out_map(CUtensorMap* m, void* base, int T, int N, int D, bool bf16) {
  const TmapEncodeFn enc = tmap_encoder();
  if (!enc) return FRATTN_E_TMAP;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(D), 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FRATTN_E_TMAP;
}

// CTA-pair launch (cluster of 2).
template <int D, typename TI, typename TC>
static int launch_qkv_pair(QkvParams& p, const void* x, long long ldx, const void* w, bool bf16,
                           cudaStream_t st) {
  using C = QkvPairCfg<D>;
  if (make_kmajor_map(&p.tma_x, x, p.T, p.K, ldx, 128, bf16) ||
      make_kmajor_map(&p.tma_w, w, p.N, p.K, p.K, C::BNH, bf16) || make_out_map(&p.tma_out, p.out, p.T, p.N, D, bf16))
    return FRATTN_E_TMAP;
  p.n_tiles_n = (p.N + C::BN - 1) / C::BN;
  p.n_tiles = ((p.T + 255) / 256) * p.n_tiles_n;
  auto kern = qkv_rope_gemm_pair_kernel<D, TI, TC>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bitv = 1ull << (dev & 63);
  if (!(attr_set & bitv)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return FRATTN_E_CUDA;
    attr_set |= bitv;
  }
  const int pairs = sm_count_for_current_device() / 2;
  const int np = p.n_tiles < pairs ? p.n_tiles : pairs;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(2 * np);
  lc.blockDim = dim3(kQkvThreads);
  lc.dynamicSmemBytes = C::SMEM;
  lc.stream = st;
  lc.attrs = &attr;
  lc.numAttrs = 1;
  if (cudaLaunchKernelEx(&lc, kern, p) != cudaSuccess) return FRATTN_E_CUDA;
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

template <int D, typename TI, typename TC>
static int launch_qkv(QkvParams& p, const void* x, long long ldx, const void* w, bool bf16,
                      cudaStream_t st) {
  if (qkv_use_pairs()) return launch_qkv_pair<D, TI, TC>(p, x, ldx, w, bf16, st);
  using C = QkvCfg<D>;
  if (make_kmajor_map(&p.tma_x, x, p.T, p.K, ldx, C::BM, bf16) ||
      make_kmajor_map(&p.tma_w, w, p.N, p.K, p.K, C::BN, bf16) || make_out_map(&p.tma_out, p.out, p.T, p.N, D, bf16))
    return FRATTN_E_TMAP;
  p.n_tiles_n = (p.N + C::BN - 1) / C::BN;
  p.n_tiles = ((p.T + C::BM - 1) / C::BM) * p.n_tiles_n;
  auto kern = qkv_rope_gemm_kernel<D, TI, TC>;
  static unsigned long long attr_set = 0;  // per device; setting twice is harmless
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bitv = 1ull << (dev & 63);
  if (!(attr_set & bitv)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return FRATTN_E_CUDA;
    attr_set |= bitv;
  }
  const int sms = sm_count_for_current_device();
  const int grid = p.n_tiles < sms ? p.n_tiles : sms;
  kern<<<grid, kQkvThreads, C::SMEM, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

template <int D, typename TI>
static int qkv_cs(QkvParams& p, const void* x, long long ldx, const void* w, int cs_dtype, bool bf16,
                  cudaStream_t st) {
  switch (cs_dtype) {
    case FRATTN_F32: return launch_qkv<D, TI, float>(p, x, ldx, w, bf16, st);
    case FRATTN_BF16: return launch_qkv<D, TI, __nv_bfloat16>(p, x, ldx, w, bf16, st);
    case FRATTN_F16: return launch_qkv<D, TI, __half>(p, x, ldx, w, bf16, st);
    default: return FRATTN_E_DTYPE;
  }
}

template <int D>
static int qkv_in(QkvParams& p, const void* x, long long ldx, const void* w, int in_dtype, int cs_dtype,
                  cudaStream_t st) {
  if (in_dtype == FRATTN_BF16) return qkv_cs<D, __nv_bfloat16>(p, x, ldx, w, cs_dtype, true, st);
  if (in_dtype == FRATTN_F16) return qkv_cs<D, __half>(p, x, ldx, w, cs_dtype, false, st);
  return FRATTN_E_DTYPE;
}

}  // namespace frattn

extern "C" int frattn_qkv_rope(const void* x, long long x_stride, const void* w, const void* bias,
                               const void* cos, const void* sin, int cs_dtype, int T, int K, int H,
                               int D, int in_dtype, void* qkv, int32_t* status, void* stream) {
  using namespace frattn;
  if (!x || !w || !cos || !sin || !qkv) return FRATTN_E_NULL;
  if (T < 0 || K <= 0 || H <= 0 || D % 16 != 0 || D < 32 || D > 128) return FRATTN_E_SHAPE;
  if (x_stride == 0) x_stride = K;
  if (x_stride < K || (x_stride & 7) || (K & 7)) return x_stride < K ? FRATTN_E_SHAPE : FRATTN_E_ALIGN;
  if (in_dtype != FRATTN_BF16 && in_dtype != FRATTN_F16) return FRATTN_E_DTYPE;
  if (cs_dtype != FRATTN_F32 && cs_dtype != FRATTN_BF16 && cs_dtype != FRATTN_F16) return FRATTN_E_DTYPE;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(x) || !a16(w) || !a16(cos) || !a16(sin) || !a16(qkv) || (bias && !a16(bias)))
    return FRATTN_E_ALIGN;
  const long long N = 3ll * H * D;
  if (static_cast<long long>(T) * N >= (1ll << 31) || N * K >= (1ll << 31)) return FRATTN_E_SHAPE;
  if (T == 0) return 0;
  QkvParams p;
  memset(&p, 0, sizeof(p));
  p.bias = bias;
  p.cos = cos;
  p.sin = sin;
  p.out = qkv;
  p.T = T;
  p.N = static_cast<int>(N);
  p.K = K;
  p.H = H;
  p.status = status;
  p.wait_limit_ns = frattn_wait_limit_ns();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (D) {
    case 32: return qkv_in<32>(p, x, x_stride, w, in_dtype, cs_dtype, st);
    case 48: return qkv_in<48>(p, x, x_stride, w, in_dtype, cs_dtype, st);
    case 64: return qkv_in<64>(p, x, x_stride, w, in_dtype, cs_dtype, st);
    case 80: return qkv_in<80>(p, x, x_stride, w, in_dtype, cs_dtype, st);
    case 96: return qkv_in<96>(p, x, x_stride, w, in_dtype, cs_dtype, st);
    case 112: return qkv_in<112>(p, x, x_stride, w, in_dtype, cs_dtype, st);
    case 128: return qkv_in<128>(p, x, x_stride, w, in_dtype, cs_dtype, st);
    default: return FRATTN_E_SHAPE;
  }
}

extern "C" int frattn_qkv_rope_set_pairs(int enable) {
  frattn::g_qkv_pairs = enable ? 1 : 0;
  return 0;
}
