// Library-wide plumbing (error reporting, device status word) and the small
// memory-bound kernels around the hot path: rotary tables, the carried
// embedding, the SwiGLU epilogue, the output-head weight scaling and the
// token cross-entropy.
#include "common.cuh"

#include <string.h>


namespace engpt {

static thread_local char t_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_err[0] = '\0'; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(ENGPT_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return ENGPT_OK;
}

__device__ int g_device_status = 0;

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// ------------------------------------------------------------ rotary tables
// rotary_frequencies (engpt/kernels.py:355-374): inv_freq = 1 / theta^(2i/rd)
// and the angle pos * inv_freq are formed in fp32, then cos/sin.
__global__ void rotary_tables_kernel(int T, int half, int rd, float theta, float* cos_out, float* sin_out) {
  int64_t n = (int64_t)T * half;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    int t = (int)(e / half);
    int i = (int)(e % half);
    // theta^(2i/rd) rounded once to fp32 (double pow, then one rounding), fp32
    // reciprocal and fp32 angle, as the reference forms them in float32;
    // cos/sin of the fp32 angle evaluated in double and rounded once.
    float expo = (float)(2 * i) / (float)rd;
    float powed = (float)pow((double)theta, (double)expo);
    float inv = 1.0f / powed;
    float f = (float)t * inv;
    cos_out[e] = (float)cos((double)f);
    sin_out[e] = (float)sin((double)f);
  }
}

// --------------------------------------------------------- carried embedding
__global__ void embed_kernel(const int64_t* __restrict__ idx, const float* __restrict__ emb, int64_t n, int d,
                             int64_t vocab, float* __restrict__ y, float* __restrict__ rho,
                             __nv_bfloat16* __restrict__ aux) {
  // one warp per token row
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (row >= n) return;
  int64_t tok = idx[row];
  bool ok = tok >= 0 && tok < vocab;
  if (!ok && lane == 0) record_device_error(ENGPT_ERR_ARG, 1);
  const float* src = emb + (ok ? tok : 0) * (int64_t)d;
  float* dst = y + row * (int64_t)d;
  if ((d & 3) == 0) {
    for (int c = lane * 4; c < d; c += 128) {
      float4 v = ok ? *reinterpret_cast<const float4*>(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(dst + c) = v;
      if (aux) {
        __nv_bfloat162* a = reinterpret_cast<__nv_bfloat162*>(aux + row * (int64_t)d + c);
        a[0] = __floats2bfloat162_rn(v.x, v.y);
        a[1] = __floats2bfloat162_rn(v.z, v.w);
      }
    }
  } else {
    for (int c = lane; c < d; c += 32) {
      float v = ok ? src[c] : 0.f;
      dst[c] = v;
      if (aux) aux[row * (int64_t)d + c] = __float2bfloat16_rn(v);
    }
  }
  if (lane == 0) rho[row] = 1.0f;
}

// ------------------------------------------------------------ SwiGLU epilogue
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// SiLU on the hot path: MUFU exp and approximate reciprocal (a few ulp in
// fp32, far below the bf16 rounding of the result).  For x -> -inf the
// denominator overflows and __fdividef returns 0, the limit of x*sigmoid(x).
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float load_as_f32(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float load_as_f32(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ void store_f32(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void store_f32(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

// Vector path: bf16 in, bf16 out, width % 8 == 0.  A block owns whole rows
// (blockIdx.x: row group, threads: 8-column chunks); each thread keeps
// kSwiRows rows' loads in flight before computing.
constexpr int kSwiRows = 4;

__global__ void __launch_bounds__(256, 3) swiglu_bf16_vec_kernel(const __nv_bfloat16* __restrict__ ug,
                                                                 const float* __restrict__ s_u,
                                                                 const float* __restrict__ s_gate, float u_mult,
                                                                 float gate_mult, int64_t rows, int width,
                                                                 __nv_bfloat16* __restrict__ out) {
  const int chunks = width >> 3;
  for (int ch = threadIdx.x; ch < chunks; ch += blockDim.x) {
    const int c = ch << 3;
    float4 su0 = *reinterpret_cast<const float4*>(s_u + c);
    float4 su1 = *reinterpret_cast<const float4*>(s_u + c + 4);
    float4 sg0 = *reinterpret_cast<const float4*>(s_gate + c);
    float4 sg1 = *reinterpret_cast<const float4*>(s_gate + c + 4);
    const float su[8] = {su0.x, su0.y, su0.z, su0.w, su1.x, su1.y, su1.z, su1.w};
    const float sg[8] = {sg0.x, sg0.y, sg0.z, sg0.w, sg1.x, sg1.y, sg1.z, sg1.w};
    for (int64_t r0 = (int64_t)blockIdx.x * kSwiRows; r0 < rows; r0 += (int64_t)gridDim.x * kSwiRows) {
      uint4 ru[kSwiRows], rg[kSwiRows];
#pragma unroll
      for (int k = 0; k < kSwiRows; ++k) {
        if (r0 + k < rows) {
          const __nv_bfloat16* row = ug + (r0 + k) * (int64_t)(2 * width);
          ru[k] = ld_stream(row + c);
          rg[k] = ld_stream(row + width + c);
        }
      }
#pragma unroll
      for (int k = 0; k < kSwiRows; ++k) {
        if (r0 + k < rows) {
          float u[8], g[8], o[8];
          unpack8(ru[k], u);
          unpack8(rg[k], g);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float uu = (u[i] * su[i]) * u_mult;
            const float gg = (g[i] * sg[i]) * gate_mult;
            o[i] = uu * silu_fast(gg);
          }
          st_stream(out + (r0 + k) * (int64_t)width + c, pack8(o));
        }
      }
    }
  }
}

template <typename TI, typename TO>
__global__ void swiglu_generic_kernel(const TI* __restrict__ ug, const float* __restrict__ s_u,
                                      const float* __restrict__ s_gate, float u_mult, float gate_mult,
                                      int64_t rows, int width, TO* __restrict__ out) {
  int64_t total = rows * width;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e / width;
    int c = (int)(e - r * width);
    float uu = (load_as_f32(ug, r * 2 * width + c) * s_u[c]) * u_mult;
    float gg = (load_as_f32(ug, r * 2 * width + width + c) * s_gate[c]) * gate_mult;
    store_f32(out, e, uu * silu_f(gg));
  }
}

// -------------------------------------------------------- row-scaled casting
template <typename TO>
__global__ void scale_rows_cast_kernel(const float* __restrict__ src, const float* __restrict__ scale, float mult,
                                       int64_t rows, int64_t cols, TO* __restrict__ out) {
  int64_t total = rows * cols;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e / cols;
    float v = src[e];
    if (scale) v = v * (scale[r] * mult);
    store_f32(out, e, v);
  }
}

__global__ void scale_rows_cast_bf16_vec_kernel(const float* __restrict__ src, const float* __restrict__ scale,
                                                float mult, int64_t rows, int64_t cols,
                                                __nv_bfloat16* __restrict__ out) {
  int64_t total8 = rows * cols / 8;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total8; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t base = e * 8;
    int64_t r = base / cols;
    float4 a = *reinterpret_cast<const float4*>(src + base);
    float4 b = *reinterpret_cast<const float4*>(src + base + 4);
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (scale) {
      float s = scale[r] * mult;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = v[i] * s;
    }
    *reinterpret_cast<uint4*>(out + base) = pack8(v);
  }
}

// ---------------------------------------------------- batched fp32->bf16 cast
constexpr int kCastMax = 64;
struct CastList {
  const float* src[kCastMax];
  __nv_bfloat16* dst[kCastMax];
  int64_t count[kCastMax];
  int block0[kCastMax + 1];   // tensor i owns blocks [block0[i], block0[i + 1]) of the 1-D grid
  int m;
};

constexpr int kCastVecPerThread = 4;   // 8-element vectors per thread and block-stride step

// grid.y = tensor, grid.x strides over that tensor in 8-element chunks
__global__ void __launch_bounds__(256) cast_many_kernel(const __grid_constant__ CastList L) {
  // this block's tensor: the last i with block0[i] <= blockIdx.x (blocks in proportion to the tensor sizes)
  int lo = 0, hi = L.m - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (L.block0[mid] <= (int)blockIdx.x) lo = mid; else hi = mid - 1;
  }
  const int t = lo;
  const float* __restrict__ src = L.src[t];
  __nv_bfloat16* __restrict__ dst = L.dst[t];
  const int64_t n = L.count[t];
  const int64_t n8 = n / 8;
  const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  const int nb = L.block0[t + 1] - L.block0[t];
  const int64_t stride = (int64_t)nb * blockDim.x;
  const int64_t first = (int64_t)(blockIdx.x - L.block0[t]) * blockDim.x + threadIdx.x;
  if (vec) {
    for (int64_t e = first; e < n8; e += stride) {
      float4 a = *reinterpret_cast<const float4*>(src + e * 8);
      float4 b = *reinterpret_cast<const float4*>(src + e * 8 + 4);
      float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      *reinterpret_cast<uint4*>(dst + e * 8) = pack8(v);
    }
    for (int64_t e = n8 * 8 + first; e < n; e += stride) dst[e] = __float2bfloat16_rn(src[e]);
  } else {
    for (int64_t e = first; e < n; e += stride) dst[e] = __float2bfloat16_rn(src[e]);
  }
}

// ------------------------------------------------------------ cross-entropy
// Log-sum-exp state in base 2: m = running max of x * log2(e), s = sum of 2^(x * log2(e) - m).
// The running max is raised only when a value exceeds it, so the common step is one FFMA and one
// MUFU ex2 per logit.
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void lse_push(float& m, float& s, float x) {
  const float xl = x * kLog2e;
  if (xl > m) {
    s = s * ex2_fast(m - xl) + 1.0f;
    m = xl;
  } else {
    s += ex2_fast(xl - m);
  }
}
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = s * ex2_fast(m - mm) + s2 * ex2_fast(m2 - mm);
  m = mm;
}

// One CTA per row: online log-sum-exp over the row (16-byte loads for bf16), then the
// target's term.  ignore_index (-100) rows contribute 0.
template <typename T>
__global__ void __launch_bounds__(256) cross_entropy_rows_kernel(const T* __restrict__ logits, int64_t rows,
                                                                 int64_t vocab, int64_t ld,
                                                                 const int64_t* __restrict__ targets,
                                                                 float* __restrict__ row_loss) {
  int64_t r = blockIdx.x;
  if (r >= rows) return;
  const T* row = logits + r * ld;
  float m = -INFINITY, s = 0.f;
  int64_t head = 0;
  if (sizeof(T) == 2) {
    // bf16: align the body to 16 bytes, then 8 elements per load.
    uintptr_t addr = reinterpret_cast<uintptr_t>(row);
    head = ((16 - (addr & 15)) & 15) / 2;
    if (head > vocab) head = vocab;
    for (int64_t c = threadIdx.x; c < head; c += blockDim.x) lse_push(m, s, load_as_f32(row, c));
    int64_t nvec = (vocab - head) / 8;
    const uint4* body = reinterpret_cast<const uint4*>(row + head);
    for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) {
      float x[8];
      unpack8(ld_stream(body + v), x);
      float cm = fmaxf(fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])), fmaxf(fmaxf(x[4], x[5]), fmaxf(x[6], x[7])));
      const float cml = cm * kLog2e;
      if (cml > m) {   // rare after the first few vectors of a thread
        s *= ex2_fast(m - cml);
        m = cml;
      }
      const float nm = -m;
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        s0 += ex2_fast(fmaf(x[i], kLog2e, nm));
        s1 += ex2_fast(fmaf(x[i + 1], kLog2e, nm));
      }
      s += s0 + s1;
    }
    for (int64_t c = head + nvec * 8 + threadIdx.x; c < vocab; c += blockDim.x) lse_push(m, s, load_as_f32(row, c));
  } else {
    for (int64_t c = threadIdx.x; c < vocab; c += blockDim.x) lse_push(m, s, load_as_f32(row, c));
  }
  // warp combine
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  __shared__ float sm[8], ss[8];
  int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) lse_merge(M, S, sm[i], ss[i]);
    int64_t t = targets[r];
    float loss = 0.f;
    if (t == -100) {
      loss = 0.f;  // ignore_index of F.cross_entropy
    } else if (t < 0 || t >= vocab) {
      record_device_error(ENGPT_ERR_ARG, 2);
      loss = NAN;
    } else {
      loss = (M + log2f(S)) * 0.6931471805599453f - load_as_f32(row, t);   // logsumexp - logit[t]
    }
    row_loss[r] = loss;
  }
}

__global__ void __launch_bounds__(1024) mean_loss_kernel(const float* __restrict__ row_loss,
                                                         const int64_t* __restrict__ targets, int64_t rows,
                                                         float* __restrict__ out) {
  double acc = 0.0;
  long long cnt = 0;
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    if (targets[r] != -100) {
      acc += (double)row_loss[r];
      ++cnt;
    }
  }
  __shared__ double sacc[1024];
  __shared__ long long scnt[1024];
  sacc[threadIdx.x] = acc;
  scnt[threadIdx.x] = cnt;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) {
      sacc[threadIdx.x] += sacc[threadIdx.x + o];
      scnt[threadIdx.x] += scnt[threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[0] = scnt[0] > 0 ? (float)(sacc[0] / (double)scnt[0]) : NAN;
}

int launch_mean_loss(const float* row_loss, const int64_t* targets, int64_t rows, float* loss_out, cudaStream_t st) {
  mean_loss_kernel<<<1, 1024, 0, st>>>(row_loss, targets, rows, loss_out);
  return check_launch("cross_entropy_mean");
}

static int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

}  // namespace engpt

using namespace engpt;

extern "C" {

const char* engpt_last_error(void) { return t_err; }

int engpt_abi_version(void) { return 101; }

int engpt_device_status(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(ENGPT_ERR_LAUNCH, "device sync: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  if (e != cudaSuccess) return set_error(ENGPT_ERR_LAUNCH, "read status: %s", cudaGetErrorString(e));
  return v;
}

int engpt_clear_device_status(void) {
  int z = 0;
  cudaError_t e = cudaMemcpyToSymbol(g_device_status, &z, sizeof(int));
  if (e != cudaSuccess) return set_error(ENGPT_ERR_LAUNCH, "clear status: %s", cudaGetErrorString(e));
  return ENGPT_OK;
}

int engpt_rotary_tables(int T, int Dh, float theta, float* cos_out, float* sin_out, void* stream) {
  clear_error();
  ENGPT_REQUIRE(T > 0 && Dh > 0, ENGPT_ERR_SHAPE, "rotary_tables: T=%d Dh=%d", T, Dh);
  int rd = Dh - (Dh % 2);
  int half = rd / 2;
  if (half == 0) return ENGPT_OK;
  ENGPT_REQUIRE(cos_out && sin_out, ENGPT_ERR_ARG, "rotary_tables: null output");
  int64_t n = (int64_t)T * half;
  rotary_tables_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(T, half, rd, theta, cos_out, sin_out);
  return check_launch("rotary_tables");
}

int engpt_embed_carried(const int64_t* idx, const float* emb, int64_t n_tokens, int d, int64_t vocab, float* y_out,
                        float* rho_out, void* aux_bf16, void* stream) {
  clear_error();
  ENGPT_REQUIRE(n_tokens >= 0 && d > 0 && vocab > 0, ENGPT_ERR_SHAPE, "embed: n=%lld d=%d", (long long)n_tokens, d);
  if (n_tokens == 0) return ENGPT_OK;
  ENGPT_REQUIRE(idx && emb && y_out && rho_out, ENGPT_ERR_ARG, "embed: null pointer");
  if ((d & 3) == 0)
    ENGPT_REQUIRE(aligned(emb, 16) && aligned(y_out, 16) && (!aux_bf16 || aligned(aux_bf16, 8)), ENGPT_ERR_ALIGN,
                  "embed: vector path needs 16-byte aligned rows");
  int64_t threads = n_tokens * 32;
  int blocks = (int)((threads + 255) / 256);
  embed_kernel<<<blocks, 256, 0, as_stream(stream)>>>(idx, emb, n_tokens, d, vocab, y_out, rho_out,
                                                      reinterpret_cast<__nv_bfloat16*>(aux_bf16));
  return check_launch("embed_carried");
}

int engpt_swiglu(const void* ug, int dtype, const float* s_u, const float* s_gate, float u_mult, float gate_mult,
                 int64_t rows, int width, void* out, int out_dtype, void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows >= 0 && width > 0, ENGPT_ERR_SHAPE, "swiglu: rows=%lld width=%d", (long long)rows, width);
  if (rows == 0) return ENGPT_OK;
  ENGPT_REQUIRE(ug && s_u && s_gate && out, ENGPT_ERR_ARG, "swiglu: null pointer");
  cudaStream_t st = as_stream(stream);
  if (dtype == ENGPT_BF16 && out_dtype == ENGPT_BF16 && (width % 8) == 0 && aligned(ug, 16) && aligned(out, 16) &&
      aligned(s_u, 16) && aligned(s_gate, 16)) {
    const int64_t groups = (rows + kSwiRows - 1) / kSwiRows;
    const int threads = (width / 8) < 256 ? (((width / 8) + 31) / 32) * 32 : 256;
    const int64_t cap = (int64_t)num_sms() * 8 * (256 / threads);
    const int blocks = (int)(groups < cap ? groups : cap);
    swiglu_bf16_vec_kernel<<<blocks, threads, 0, st>>>((const __nv_bfloat16*)ug, s_u, s_gate, u_mult, gate_mult,
                                                        rows, width, (__nv_bfloat16*)out);
  } else if (dtype == ENGPT_BF16 && out_dtype == ENGPT_BF16) {
    swiglu_generic_kernel<__nv_bfloat16, __nv_bfloat16><<<grid_for(rows * width, 256), 256, 0, st>>>(
        (const __nv_bfloat16*)ug, s_u, s_gate, u_mult, gate_mult, rows, width, (__nv_bfloat16*)out);
  } else if (dtype == ENGPT_F32 && out_dtype == ENGPT_F32) {
    swiglu_generic_kernel<float, float><<<grid_for(rows * width, 256), 256, 0, st>>>(
        (const float*)ug, s_u, s_gate, u_mult, gate_mult, rows, width, (float*)out);
  } else if (dtype == ENGPT_BF16 && out_dtype == ENGPT_F32) {
    swiglu_generic_kernel<__nv_bfloat16, float><<<grid_for(rows * width, 256), 256, 0, st>>>(
        (const __nv_bfloat16*)ug, s_u, s_gate, u_mult, gate_mult, rows, width, (float*)out);
  } else {
    return set_error(ENGPT_ERR_DTYPE, "swiglu: dtype %d -> %d not supported", dtype, out_dtype);
  }
  return check_launch("swiglu");
}

int engpt_scale_rows_cast(const float* src, const float* scale, float mult, int64_t rows, int64_t cols, void* out,
                          int out_dtype, void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows >= 0 && cols > 0, ENGPT_ERR_SHAPE, "scale_rows_cast: rows=%lld cols=%lld", (long long)rows,
                (long long)cols);
  if (rows == 0) return ENGPT_OK;
  ENGPT_REQUIRE(src && out, ENGPT_ERR_ARG, "scale_rows_cast: null pointer");
  cudaStream_t st = as_stream(stream);
  if (out_dtype == ENGPT_BF16) {
    if ((cols % 8) == 0 && aligned(src, 16) && aligned(out, 16)) {
      scale_rows_cast_bf16_vec_kernel<<<grid_for(rows * cols / 8, 256), 256, 0, st>>>(src, scale, mult, rows, cols,
                                                                                    (__nv_bfloat16*)out);
    } else {
      scale_rows_cast_kernel<__nv_bfloat16><<<grid_for(rows * cols, 256), 256, 0, st>>>(src, scale, mult, rows, cols,
                                                                                        (__nv_bfloat16*)out);
    }
  } else if (out_dtype == ENGPT_F32) {
    scale_rows_cast_kernel<float><<<grid_for(rows * cols, 256), 256, 0, st>>>(src, scale, mult, rows, cols,
                                                                              (float*)out);
  } else {
    return set_error(ENGPT_ERR_DTYPE, "scale_rows_cast: out dtype %d", out_dtype);
  }
  return check_launch("scale_rows_cast");
}

int engpt_cast_f32_bf16_many(const void* const* src, void* const* dst, const int64_t* counts, int n,
                             void* stream) {
  clear_error();
  ENGPT_REQUIRE(n >= 0, ENGPT_ERR_SHAPE, "cast_many: n=%d", n);
  if (n == 0) return ENGPT_OK;
  ENGPT_REQUIRE(src && dst && counts, ENGPT_ERR_ARG, "cast_many: null pointer array");
  cudaStream_t st = as_stream(stream);
  for (int base = 0; base < n; base += kCastMax) {
    const int m = (n - base) < kCastMax ? (n - base) : kCastMax;
    CastList L;
    for (int i = 0; i < m; ++i) {
      ENGPT_REQUIRE(counts[base + i] >= 0, ENGPT_ERR_SHAPE, "cast_many: count[%d] < 0", base + i);
      ENGPT_REQUIRE(counts[base + i] == 0 || (src[base + i] && dst[base + i]), ENGPT_ERR_ARG,
                    "cast_many: null tensor %d", base + i);
      L.src[i] = static_cast<const float*>(src[base + i]);
      L.dst[i] = static_cast<__nv_bfloat16*>(dst[base + i]);
      L.count[i] = counts[base + i];
    }
    for (int i = m; i < kCastMax; ++i) {
      L.src[i] = nullptr;
      L.dst[i] = nullptr;
      L.count[i] = 0;
    }
    // blocks in proportion to each tensor's size (every tensor at least one), so the whole batch finishes
    // together with the GPU full until the end
    int64_t nblk = 0;
    for (int i = 0; i < m; ++i) {
      L.block0[i] = (int)nblk;
      const int64_t vecs = (L.count[i] + 7) / 8;
      int64_t b = (vecs + 256 * kCastVecPerThread - 1) / (256 * kCastVecPerThread);
      if (b < 1) b = 1;
      nblk += b;
      ENGPT_REQUIRE(nblk <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "cast_many: too many blocks");
    }
    for (int i = m; i <= kCastMax; ++i) L.block0[i] = (int)nblk;
    L.m = m;
    cast_many_kernel<<<(unsigned)nblk, 256, 0, st>>>(L);
    int rc = check_launch("cast_f32_bf16_many");
    if (rc) return rc;
  }
  return ENGPT_OK;
}

int engpt_cross_entropy(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t ld,
                        const int64_t* targets, float* row_loss, float* loss_out, void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows > 0 && vocab > 0 && ld >= vocab, ENGPT_ERR_SHAPE, "cross_entropy: rows=%lld vocab=%lld ld=%lld",
                (long long)rows, (long long)vocab, (long long)ld);
  ENGPT_REQUIRE(rows <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "cross_entropy: too many rows");
  ENGPT_REQUIRE(logits && targets && row_loss && loss_out, ENGPT_ERR_ARG, "cross_entropy: null pointer");
  cudaStream_t st = as_stream(stream);
  if (dtype == ENGPT_BF16) {
    cross_entropy_rows_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, st>>>((const __nv_bfloat16*)logits, rows, vocab,
                                                                             ld, targets, row_loss);
  } else if (dtype == ENGPT_F32) {
    cross_entropy_rows_kernel<float><<<(unsigned)rows, 256, 0, st>>>((const float*)logits, rows, vocab, ld, targets,
                                                                     row_loss);
  } else {
    return set_error(ENGPT_ERR_DTYPE, "cross_entropy: dtype %d", dtype);
  }
  int rc = check_launch("cross_entropy_rows");
  if (rc) return rc;
  mean_loss_kernel<<<1, 1024, 0, st>>>(row_loss, targets, rows, loss_out);
  return check_launch("cross_entropy_mean");
}

// ------------------------------------------------ cross-entropy, no allocation
// Per-row loss scratch for engpt_cross_entropy_noalloc, resident in the
// library's device memory (one copy per device that loads the library).
static __device__ __align__(256) float g_ce_noalloc_rows[ENGPT_CE_NOALLOC_MAX_ROWS];

// Device address of g_ce_noalloc_rows on the current device.  In host code the
// array's name is only a host-side stand-in, never a device address, so the
// address is looked up with the device current.  It is looked up on every
// call (a cheap runtime query once the module is loaded) rather than cached,
// so it stays valid across a cudaDeviceReset that rebuilds the context.
static int ce_noalloc_scratch(float** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_ce_noalloc_rows);
  if (e != cudaSuccess || p == nullptr)
    return set_error(ENGPT_ERR_LAUNCH, "cross_entropy_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  *out = static_cast<float*>(p);
  return ENGPT_OK;
}

int engpt_cross_entropy_noalloc(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t ld,
                                const int64_t* targets, float* loss_out, void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows > 0 && vocab > 0 && ld >= vocab, ENGPT_ERR_SHAPE,
                "cross_entropy_noalloc: rows=%lld vocab=%lld ld=%lld", (long long)rows, (long long)vocab,
                (long long)ld);
  ENGPT_REQUIRE(rows <= ENGPT_CE_NOALLOC_MAX_ROWS, ENGPT_ERR_SHAPE,
                "cross_entropy_noalloc: %lld rows exceed the fixed scratch of %d rows; use engpt_cross_entropy "
                "with a caller-provided row buffer", (long long)rows, ENGPT_CE_NOALLOC_MAX_ROWS);
  ENGPT_REQUIRE(logits && targets && loss_out, ENGPT_ERR_ARG, "cross_entropy_noalloc: null pointer");
  ENGPT_REQUIRE(dtype == ENGPT_BF16 || dtype == ENGPT_F32, ENGPT_ERR_DTYPE, "cross_entropy_noalloc: dtype %d",
                dtype);
  float* row_loss = nullptr;
  int rc = ce_noalloc_scratch(&row_loss);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  if (dtype == ENGPT_BF16) {
    cross_entropy_rows_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, st>>>((const __nv_bfloat16*)logits, rows, vocab,
                                                                             ld, targets, row_loss);
  } else {
    cross_entropy_rows_kernel<float><<<(unsigned)rows, 256, 0, st>>>((const float*)logits, rows, vocab, ld, targets,
                                                                     row_loss);
  }
  rc = check_launch("cross_entropy_noalloc_rows");
  if (rc) return rc;
  mean_loss_kernel<<<1, 1024, 0, st>>>(row_loss, targets, rows, loss_out);
  return check_launch("cross_entropy_noalloc_mean");
}

}  // extern "C"
