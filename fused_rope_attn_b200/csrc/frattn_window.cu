// Window plan on the device: the Qwen2.5-VL window permutation of merge units,
// its token-space cu_seqlens, the (h, w) patch position of every token in
// window order, optionally the rotary cos/sin tables in window order, and the
// shuffle / unshuffle of [T, ...] rows into and out of window order.
//
// Reference (sdan/fused-rope-attn): get_window_index (utils.py:12-102),
// window_shuffle / window_unshuffle (utils.py:105-153) and the window-ordered
// tables of compute_rope_2d (fused_attn.py:33-136, window_idx argument). The
// reference builds these with host-side torch ops on every image set; here
// every output element has a closed form, so one thread per merge unit (or
// per window, per row chunk) writes it directly into device memory.
//
// Layout (per image i with t frames of gh x gw merge units, vw = window side in
// units): windows are visited row-major per frame, units row-major inside a
// window, edge windows truncated. For unit (frame f, row r, col c) in window
// (wr, wc) = (r / vw, c / vw):
//   hh = min(vw, gh - wr vw), ww = min(vw, gw - wc vw)
//   position in frame = wr vw gw + hh wc vw + (r - wr vw) ww + (c - wc vw)
// and window (wr, wc) starts at unit wr vw gw + hh wc vw of its frame.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "../../include/frattn.h"

namespace frattn_window {

struct ImgPlan {
  int t, gh, gw, nwh, nww;
  int unit_base;  // first merge unit of the image
  int win_base;   // first window of the image
  int pad;
};

// Last image whose base is <= x (bases ascending).
template <bool kWindows>
__device__ __forceinline__ int find_image(const ImgPlan* img, int n, int x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    const int b = kWindows ? img[mid].win_base : img[mid].unit_base;
    if (b <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Source unit (frame, row, col) of window-order slot s (closed-form inverse of
// the slot formula in the file header): full window rows hold vw gw units;
// inside window row wr every window but the last holds hh vw units.
struct UnitRC {
  int u, r, c;
};
__device__ __forceinline__ UnitRC slot_unit(const ImgPlan* img, int n_img, int slot, int vw) {
  const ImgPlan I = img[find_image<false>(img, n_img, slot)];
  const int per_frame = I.gh * I.gw;
  const int rel = slot - I.unit_base;
  const int f = rel / per_frame, s = rel - f * per_frame;
  const int wr = s / (vw * I.gw);
  const int hh = min(vw, I.gh - wr * vw);
  const int in_row = s - wr * vw * I.gw;
  const int wc = in_row / (hh * vw);
  const int ww = min(vw, I.gw - wc * vw);
  const int inner = in_row - wc * hh * vw;
  UnitRC o;
  o.r = wr * vw + inner / ww;
  o.c = wc * vw + inner % ww;
  o.u = I.unit_base + f * per_frame + o.r * I.gw + o.c;
  return o;
}

// window_index (one thread per slot), pos_hw (one per token row) and the
// cos/sin tables (one per table element), all written in window order with
// coalesced stores.
__global__ void plan_units(const ImgPlan* __restrict__ img, int n_img, int units, int vw, int m,
                           int64_t* __restrict__ window_index, int32_t* __restrict__ pos_hw,
                           float* __restrict__ cos_t, float* __restrict__ sin_t, int rd,
                           float theta) {
  extern __shared__ float inv_freq[];  // [rd / 2]
  const int q4 = rd / 2;
  if (cos_t != nullptr)
    for (int i = threadIdx.x; i < q4; i += blockDim.x)
      inv_freq[i] = 1.0f / powf(theta, static_cast<float>(2 * i) / static_cast<float>(rd));
  __syncthreads();
  const int mu = m * m;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  for (int64_t sl = first; sl < units; sl += stride)
    window_index[sl] = slot_unit(img, n_img, static_cast<int>(sl), vw).u;
  const int64_t rows = static_cast<int64_t>(units) * mu;
  if (pos_hw != nullptr)
    for (int64_t p = first; p < rows; p += stride) {
      const int j = static_cast<int>(p % mu);
      const UnitRC o = slot_unit(img, n_img, static_cast<int>(p / mu), vw);
      pos_hw[2 * p] = o.r * m + j / m;  // merge order inside the unit
      pos_hw[2 * p + 1] = o.c * m + j % m;
    }
  if (cos_t != nullptr)
    for (int64_t e = first; e < rows * rd; e += stride) {
      const int64_t p = e / rd;
      const int i = static_cast<int>(e - p * rd);
      const int j = static_cast<int>(p % mu);
      const UnitRC o = slot_unit(img, n_img, static_cast<int>(p / mu), vw);
      const int pos = i < q4 ? o.r * m + j / m : o.c * m + j % m;
      const float ang = static_cast<float>(pos) * inv_freq[i < q4 ? i : i - q4];
      float sv, cv;
      sincosf(ang, &sv, &cv);
      cos_t[e] = cv;
      sin_t[e] = sv;
    }
}

// One thread per window: cu_seqlens (token offsets) in window order.
__global__ void plan_windows(const ImgPlan* __restrict__ img, int n_img, int windows, int units,
                             int vw, int mu, int32_t* __restrict__ cu) {
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w <= windows; w += gridDim.x * blockDim.x) {
    if (w == windows) {
      cu[w] = units * mu;
      continue;
    }
    const ImgPlan I = img[find_image<true>(img, n_img, w)];
    const int per_frame = I.nwh * I.nww;
    const int rel = w - I.win_base;
    const int f = rel / per_frame, rem = rel - f * per_frame;
    const int wr = rem / I.nww, wc = rem - wr * I.nww;
    const int hh = min(vw, I.gh - wr * vw);
    cu[w] = (I.unit_base + f * I.gh * I.gw + wr * vw * I.gw + hh * wc * vw) * mu;
  }
}

// out row (p mu + j) = x row (idx[p] mu + j) (gather), or the inverse scatter.
__global__ void shuffle_rows(const uint4* __restrict__ x, const int64_t* __restrict__ idx,
                             int64_t units, int mu, int64_t row_vec, int inverse,
                             uint4* __restrict__ out) {
  const int64_t total = units * mu * row_vec;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = e / row_vec, col = e - row * row_vec;
    const int64_t p = row / mu, j = row - p * mu;
    const int64_t src_row = __ldg(idx + p) * mu + j;
    if (inverse)
      out[src_row * row_vec + col] = __ldg(x + e);
    else
      out[e] = __ldg(x + src_row * row_vec + col);
  }
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int build_plan(const int32_t* grid_thw, int num_images, int window_size, int merge,
               int patch_size, std::vector<ImgPlan>* plan, int64_t* units, int64_t* windows,
               int* vw_out) {
  if (!grid_thw) return FRATTN_E_NULL;
  if (num_images < 1 || window_size <= 0 || merge <= 0 || patch_size <= 0) return FRATTN_E_SHAPE;
  const int vw = window_size / merge / patch_size;
  if (vw <= 0) return FRATTN_E_SHAPE;
  int64_t u = 0, w = 0;
  plan->clear();
  for (int i = 0; i < num_images; ++i) {
    const int t = grid_thw[3 * i], h = grid_thw[3 * i + 1], wd = grid_thw[3 * i + 2];
    if (t <= 0 || h <= 0 || wd <= 0 || h % merge || wd % merge) return FRATTN_E_SHAPE;
    ImgPlan I;
    I.t = t;
    I.gh = h / merge;
    I.gw = wd / merge;
    I.nwh = (I.gh + vw - 1) / vw;
    I.nww = (I.gw + vw - 1) / vw;
    I.unit_base = static_cast<int>(u);
    I.win_base = static_cast<int>(w);
    I.pad = 0;
    plan->push_back(I);
    u += static_cast<int64_t>(t) * I.gh * I.gw;
    w += static_cast<int64_t>(t) * I.nwh * I.nww;
    if (u * merge * merge >= (1ll << 31) || w >= (1ll << 31)) return FRATTN_E_SHAPE;
  }
  *units = u;
  *windows = w;
  *vw_out = vw;
  return 0;
}

}  // namespace frattn_window

using namespace frattn_window;

extern "C" {

int frattn_window_plan_sizes(const int32_t* grid_thw, int num_images, int window_size, int merge,
                             int patch_size, int64_t* units, int64_t* windows,
                             size_t* workspace_bytes) {
  if (!units || !windows || !workspace_bytes) return FRATTN_E_NULL;
  std::vector<ImgPlan> plan;
  int vw = 0;
  const int rc = build_plan(grid_thw, num_images, window_size, merge, patch_size, &plan, units,
                            windows, &vw);
  if (rc) return rc;
  *workspace_bytes = (plan.size() * sizeof(ImgPlan) + 255) & ~size_t(255);
  return 0;
}

int frattn_window_plan(const int32_t* grid_thw, int num_images, int window_size, int merge,
                       int patch_size, int64_t* window_index, int32_t* cu_seqlens, int32_t* pos_hw,
                       float* cos_table, float* sin_table, int rotary_dim, float theta,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!window_index || !cu_seqlens || !workspace) return FRATTN_E_NULL;
  if ((cos_table == nullptr) != (sin_table == nullptr)) return FRATTN_E_NULL;
  if (cos_table && (rotary_dim <= 0 || rotary_dim % 2 || rotary_dim > 256)) return FRATTN_E_SHAPE;
  std::vector<ImgPlan> plan;
  int64_t units = 0, windows = 0;
  int vw = 0;
  int rc = build_plan(grid_thw, num_images, window_size, merge, patch_size, &plan, &units,
                      &windows, &vw);
  if (rc) return rc;
  if (workspace_bytes < plan.size() * sizeof(ImgPlan)) return FRATTN_E_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ImgPlan* d_plan = static_cast<ImgPlan*>(workspace);
  // Pageable source: the copy is staged before cudaMemcpyAsync returns, so the
  // host vector may go out of scope afterwards.
  if (cudaMemcpyAsync(d_plan, plan.data(), plan.size() * sizeof(ImgPlan), cudaMemcpyHostToDevice,
                      st) != cudaSuccess)
    return FRATTN_E_CUDA;
  const int grid = 4 * sm_count();
  const int threads = 256;
  const size_t smem = cos_table ? sizeof(float) * (rotary_dim / 2) : 0;
  plan_units<<<grid, threads, smem, st>>>(d_plan, num_images, static_cast<int>(units), vw, merge,
                                          window_index, pos_hw, cos_table, sin_table, rotary_dim,
                                          theta);
  plan_windows<<<grid, threads, 0, st>>>(d_plan, num_images, static_cast<int>(windows),
                                         static_cast<int>(units), vw, merge * merge, cu_seqlens);
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

int frattn_window_shuffle(const void* x, const int64_t* window_index, int64_t units, int merge_unit,
                          int64_t row_bytes, int inverse, void* out, void* stream) {
  if (!x || !window_index || !out) return FRATTN_E_NULL;
  if (units < 0 || merge_unit <= 0 || row_bytes <= 0 || row_bytes % 16) return FRATTN_E_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) return FRATTN_E_ALIGN;
  if (units == 0) return 0;
  const int grid = 4 * sm_count();
  shuffle_rows<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(x), window_index, units, merge_unit, row_bytes / 16, inverse,
      static_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : FRATTN_E_CUDA;
}

}  // extern "C"
