// Optimizer-side sphere kernels of nGPT training: the exact retraction of the
// normalised weight matrices onto their unit rows / columns and the tangent
// projection of their gradients (engpt/kernels.py:32-136, used by
// NGPTAdamW, engpt/optim.py:74-109).  All four work in place, compute in
// fp32 and store in the tensor's dtype (fp32 or bf16).
//
//   rows     x[r, :] /= max(|x[r, :]|, eps)            g[r, :] -= (g[r, :] . w[r, :]) w[r, :]
//   columns  x[:, c] /= max(|x[:, c]|, eps)            g[:, c] -= (g[:, c] . w[:, c]) w[:, c]
//
// Rows: one warp per row, 16-byte loads where the row allows them, the
// reduction by shuffles, the row read a second time (from L1/L2) to write.
// Columns: coalesced tiles of 64 columns (each lane two adjacent columns,
// one 128-256 byte segment per warp and row); the rows of a tile are split
// over enough blocks to fill the GPU.  Pass 1 writes each block's partial
// column sums to caller scratch [splits, cols]; pass 2 adds a tile's partials
// and rewrites its rows.
#include "common.cuh"

namespace engpt {
namespace sphere {

template <typename T>
__device__ __forceinline__ float ld1(const T* p);
template <>
__device__ __forceinline__ float ld1<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld1<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
__device__ __forceinline__ void st1(T* p, float v);
template <>
__device__ __forceinline__ void st1<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st1<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// 16-byte vector of a row: 4 fp32 or 8 bf16 values
template <typename T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* v) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  }
  __device__ static void store(float* p, const float* v) { *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]); }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float* v) { unpack8(*reinterpret_cast<const uint4*>(p), v); }
  __device__ static void store(__nv_bfloat16* p, const float* v) { *reinterpret_cast<uint4*>(p) = pack8(v); }
};

// One warp per row.  PROJECT: g -= (g.w) w on `x` = g with weight w; else x /= max(|x|, eps).
template <typename T, bool PROJECT, bool VEC>
__global__ void __launch_bounds__(256) rows_kernel(T* __restrict__ x, const T* __restrict__ w, int64_t rows,
                                                   int64_t cols, float eps) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  T* xr = x + row * cols;
  const T* wr = PROJECT ? w + row * cols : nullptr;
  constexpr int N = Vec<T>::N;
  float acc = 0.f;
  if (VEC) {
    for (int64_t c = (int64_t)lane * N; c < cols; c += 32 * N) {
      float a[N];
      Vec<T>::load(xr + c, a);
      if (PROJECT) {
        float b[N];
        Vec<T>::load(wr + c, b);
#pragma unroll
        for (int i = 0; i < N; ++i) acc = fmaf(a[i], b[i], acc);
      } else {
#pragma unroll
        for (int i = 0; i < N; ++i) acc = fmaf(a[i], a[i], acc);
      }
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float a = ld1(xr + c);
      acc = fmaf(a, PROJECT ? ld1(wr + c) : a, acc);
    }
  }
  acc = warp_sum_xor<32>(acc);
  // normalise: divide by max(|x|, eps) (sqrt(max(ss, eps^2)) is the same number); project: subtract acc * w
  const float den = PROJECT ? 1.f : fmaxf(sqrtf(acc), eps);
  if (VEC) {
    for (int64_t c = (int64_t)lane * N; c < cols; c += 32 * N) {
      float a[N];
      Vec<T>::load(xr + c, a);
      if (PROJECT) {
        float b[N];
        Vec<T>::load(wr + c, b);
#pragma unroll
        for (int i = 0; i < N; ++i) a[i] = fmaf(-acc, b[i], a[i]);
      } else {
#pragma unroll
        for (int i = 0; i < N; ++i) a[i] = a[i] / den;
      }
      Vec<T>::store(xr + c, a);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float a = ld1(xr + c);
      st1(xr + c, PROJECT ? fmaf(-acc, ld1(wr + c), a) : a / den);
    }
  }
}

constexpr int kColTile = 64;   // columns per tile: two per lane
constexpr int kColWarps = 8;

// Rows [r0, r1) of split `s` for a tile: contiguous, ragged-safe.
__device__ __forceinline__ void split_rows(int64_t rows, int splits, int s, int64_t& r0, int64_t& r1) {
  const int64_t base = rows / splits, extra = rows % splits;
  r0 = s * base + (s < extra ? s : extra);
  r1 = r0 + base + (s < extra ? 1 : 0);
}

// Pass 1: partial column sums (|x|^2, or g.w) of a tile's rows in this split -> part[s, c].
template <typename T, bool PROJECT>
__global__ void __launch_bounds__(kColWarps * 32) cols_partial_kernel(const T* __restrict__ x,
                                                                      const T* __restrict__ w, int64_t rows,
                                                                      int64_t cols, float* __restrict__ part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * kColTile + 2 * lane;
  int64_t r0, r1;
  split_rows(rows, gridDim.y, blockIdx.y, r0, r1);
  float a0 = 0.f, a1 = 0.f;
  const bool in0 = c0 < cols, in1 = c0 + 1 < cols;
  for (int64_t r = r0 + warp; r < r1; r += kColWarps) {
    const T* xr = x + r * cols;
    if (in0) {
      const float v = ld1(xr + c0);
      a0 = fmaf(v, PROJECT ? ld1(w + r * cols + c0) : v, a0);
    }
    if (in1) {
      const float v = ld1(xr + c0 + 1);
      a1 = fmaf(v, PROJECT ? ld1(w + r * cols + c0 + 1) : v, a1);
    }
  }
  __shared__ float red[kColWarps][kColTile];
  red[warp][2 * lane] = a0;
  red[warp][2 * lane + 1] = a1;
  __syncthreads();
  if (threadIdx.x < kColTile) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kColWarps; ++i) s += red[i][threadIdx.x];
    const int64_t c = (int64_t)blockIdx.x * kColTile + threadIdx.x;
    if (c < cols) part[(int64_t)blockIdx.y * cols + c] = s;
  }
}

// Pass 2: the tile's column sums from every split's partials, then rewrite this split's rows.
template <typename T, bool PROJECT>
__global__ void __launch_bounds__(kColWarps * 32) cols_apply_kernel(T* __restrict__ x, const T* __restrict__ w,
                                                                    int64_t rows, int64_t cols, float eps,
                                                                    const float* __restrict__ part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ float coef[kColTile];
  if (threadIdx.x < kColTile) {
    const int64_t c = (int64_t)blockIdx.x * kColTile + threadIdx.x;
    float s = 0.f;
    if (c < cols)
      for (int i = 0; i < (int)gridDim.y; ++i) s += part[(int64_t)i * cols + c];
    coef[threadIdx.x] = PROJECT ? s : fmaxf(sqrtf(s), eps);   // the dot product, or the column's norm
  }
  __syncthreads();
  const int64_t c0 = (int64_t)blockIdx.x * kColTile + 2 * lane;
  const float k0 = coef[2 * lane], k1 = coef[2 * lane + 1];
  const bool in0 = c0 < cols, in1 = c0 + 1 < cols;
  int64_t r0, r1;
  split_rows(rows, gridDim.y, blockIdx.y, r0, r1);
  // four rows per iteration, every load issued before the first store, so each warp keeps several rows'
  // reads in flight (one row at a time left the pass latency-bound); the same arithmetic per element
  constexpr int U = 4;
  int64_t r = r0 + warp;
  for (; r + (U - 1) * kColWarps < r1; r += U * kColWarps) {
    float v0[U], v1[U], g0[U], g1[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t o = (r + u * kColWarps) * cols + c0;
      v0[u] = in0 ? ld1(x + o) : 0.f;
      v1[u] = in1 ? ld1(x + o + 1) : 0.f;
      if (PROJECT) {
        g0[u] = in0 ? ld1(w + o) : 0.f;
        g1[u] = in1 ? ld1(w + o + 1) : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t o = (r + u * kColWarps) * cols + c0;
      if (in0) st1(x + o, PROJECT ? fmaf(-k0, g0[u], v0[u]) : v0[u] / k0);
      if (in1) st1(x + o + 1, PROJECT ? fmaf(-k1, g1[u], v1[u]) : v1[u] / k1);
    }
  }
  for (; r < r1; r += kColWarps) {
    T* xr = x + r * cols;
    if (in0) {
      const float v = ld1(xr + c0);
      st1(xr + c0, PROJECT ? fmaf(-k0, ld1(w + r * cols + c0), v) : v / k0);
    }
    if (in1) {
      const float v = ld1(xr + c0 + 1);
      st1(xr + c0 + 1, PROJECT ? fmaf(-k1, ld1(w + r * cols + c0 + 1), v) : v / k1);
    }
  }
}

// Row splits of a column launch: enough (tile, split) blocks for two waves over the SMs, at least 8 rows each.
inline int col_splits(int64_t rows, int64_t cols) {
  const int64_t tiles = (cols + kColTile - 1) / kColTile;
  int64_t want = (2 * (int64_t)num_sms() + tiles - 1) / tiles;
  const int64_t max_by_rows = rows / 8 > 0 ? rows / 8 : 1;
  if (want > max_by_rows) want = max_by_rows;
  if (want > 256) want = 256;
  if (want < 1) want = 1;
  return (int)want;
}

template <typename T, bool PROJECT>
int launch_rows(T* x, const T* w, int64_t rows, int64_t cols, float eps, cudaStream_t st) {
  const int64_t blocks = (rows * 32 + 255) / 256;
  ENGPT_REQUIRE(blocks <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "sphere rows: too many rows");
  const bool vec = (cols % Vec<T>::N) == 0 && aligned(x, 16) && (!PROJECT || aligned(w, 16));
  if (vec)
    rows_kernel<T, PROJECT, true><<<(unsigned)blocks, 256, 0, st>>>(x, w, rows, cols, eps);
  else
    rows_kernel<T, PROJECT, false><<<(unsigned)blocks, 256, 0, st>>>(x, w, rows, cols, eps);
  return check_launch(PROJECT ? "project_row_grad" : "normalize_rows");
}

template <typename T, bool PROJECT>
int launch_cols(T* x, const T* w, int64_t rows, int64_t cols, float eps, float* scratch, cudaStream_t st) {
  const int splits = col_splits(rows, cols);
  const int64_t tiles = (cols + kColTile - 1) / kColTile;
  ENGPT_REQUIRE(tiles <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "sphere columns: too many columns");
  dim3 grid((unsigned)tiles, (unsigned)splits);
  cols_partial_kernel<T, PROJECT><<<grid, kColWarps * 32, 0, st>>>(x, w, rows, cols, scratch);
  int rc = check_launch(PROJECT ? "project_column_grad (partials)" : "normalize_columns (partials)");
  if (rc) return rc;
  cols_apply_kernel<T, PROJECT><<<grid, kColWarps * 32, 0, st>>>(x, w, rows, cols, eps, scratch);
  return check_launch(PROJECT ? "project_column_grad" : "normalize_columns");
}

}  // namespace sphere
}  // namespace engpt

using namespace engpt;
using namespace engpt::sphere;

extern "C" {

int64_t engpt_column_scratch_floats(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (int64_t)col_splits(rows, cols) * cols;
}

int engpt_normalize_rows(void* x, int dtype, int64_t rows, int64_t cols, float eps, void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows >= 0 && cols > 0, ENGPT_ERR_SHAPE, "normalize_rows: rows=%lld cols=%lld", (long long)rows,
                (long long)cols);
  if (rows == 0) return ENGPT_OK;
  ENGPT_REQUIRE(x != nullptr, ENGPT_ERR_ARG, "normalize_rows: null pointer");
  cudaStream_t st = as_stream(stream);
  if (dtype == ENGPT_F32) return launch_rows<float, false>((float*)x, nullptr, rows, cols, eps, st);
  if (dtype == ENGPT_BF16) return launch_rows<__nv_bfloat16, false>((__nv_bfloat16*)x, nullptr, rows, cols, eps, st);
  return set_error(ENGPT_ERR_DTYPE, "normalize_rows: dtype %d", dtype);
}

int engpt_project_row_grad(const void* weight, void* grad, int dtype, int64_t rows, int64_t cols, void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows >= 0 && cols > 0, ENGPT_ERR_SHAPE, "project_row_grad: rows=%lld cols=%lld", (long long)rows,
                (long long)cols);
  if (rows == 0) return ENGPT_OK;
  ENGPT_REQUIRE(weight && grad, ENGPT_ERR_ARG, "project_row_grad: null pointer");
  cudaStream_t st = as_stream(stream);
  if (dtype == ENGPT_F32) return launch_rows<float, true>((float*)grad, (const float*)weight, rows, cols, 0.f, st);
  if (dtype == ENGPT_BF16)
    return launch_rows<__nv_bfloat16, true>((__nv_bfloat16*)grad, (const __nv_bfloat16*)weight, rows, cols, 0.f, st);
  return set_error(ENGPT_ERR_DTYPE, "project_row_grad: dtype %d", dtype);
}

int engpt_normalize_columns(void* x, int dtype, int64_t rows, int64_t cols, float eps, float* scratch, void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows > 0 && cols >= 0, ENGPT_ERR_SHAPE, "normalize_columns: rows=%lld cols=%lld", (long long)rows,
                (long long)cols);
  if (cols == 0) return ENGPT_OK;
  ENGPT_REQUIRE(x && scratch, ENGPT_ERR_ARG, "normalize_columns: null pointer");
  cudaStream_t st = as_stream(stream);
  if (dtype == ENGPT_F32) return launch_cols<float, false>((float*)x, nullptr, rows, cols, eps, scratch, st);
  if (dtype == ENGPT_BF16)
    return launch_cols<__nv_bfloat16, false>((__nv_bfloat16*)x, nullptr, rows, cols, eps, scratch, st);
  return set_error(ENGPT_ERR_DTYPE, "normalize_columns: dtype %d", dtype);
}

int engpt_project_column_grad(const void* weight, void* grad, int dtype, int64_t rows, int64_t cols, float* scratch,
                              void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows > 0 && cols >= 0, ENGPT_ERR_SHAPE, "project_column_grad: rows=%lld cols=%lld", (long long)rows,
                (long long)cols);
  if (cols == 0) return ENGPT_OK;
  ENGPT_REQUIRE(weight && grad && scratch, ENGPT_ERR_ARG, "project_column_grad: null pointer");
  cudaStream_t st = as_stream(stream);
  if (dtype == ENGPT_F32)
    return launch_cols<float, true>((float*)grad, (const float*)weight, rows, cols, 0.f, scratch, st);
  if (dtype == ENGPT_BF16)
    return launch_cols<__nv_bfloat16, true>((__nv_bfloat16*)grad, (const __nv_bfloat16*)weight, rows, cols, 0.f,
                                            scratch, st);
  return set_error(ENGPT_ERR_DTYPE, "project_column_grad: dtype %d", dtype);
}

}  // extern "C"
