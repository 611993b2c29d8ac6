// Fused QKV epilogue: per-head L2 norm of raw q/k + interleaved RoPE +
// s_qk scale, and V / rho, in one HBM pass.
//
// Restates qkv_postprocess_from_carried (engpt/kernels.py:139-179) with the
// RoPE of apply_rope_inplace (engpt/kernels.py:399-414):
//   q_den = max(|q_raw|, rho * eps)  (norm taken before RoPE; RoPE keeps it)
//   q = RoPE(q_raw) / q_den * s_qk_eff,  k likewise,  v = v_raw / rho.
// The reference issues ~20 eager launches (norms, clones, rotations, copies,
// divides, multiplies); here a group of Dh/8 lanes owns one (token, q|k|v,
// head) row: 16-byte loads, an fp32 sum of squares reduced with shuffles, the
// rotation on register pairs and one 16-byte store per lane.  Outputs go to
// [B,T,H,Dh] or directly to the head-major [B,H,T,Dh] layout the attention
// kernel's TMA reads, so no transpose pass follows.
#include "common.cuh"

namespace engpt {

struct QkvArgs {
  const void* qkv;
  const float* rho;
  const float* cos_tab;
  const float* sin_tab;
  int rope_half;
  const float* qk_scale;
  float qk_mult;
  float eps;
  int B, T, H, Dh;
  void* q;
  void* k;
  void* v;
  int layout;  // 0: [B,T,H,Dh], 1: [B,H,T,Dh]
};

// token index n < 2^31 (checked on the host), so the split into (b, t) is 32-bit
__device__ __forceinline__ int64_t out_offset(const QkvArgs& a, int64_t n, int h) {
  if (a.layout == 0) return (n * a.H + h) * (int64_t)a.Dh;
  const int ni = (int)n;
  const int b = ni / a.T;
  const int t = ni - b * a.T;
  return ((int64_t)(b * a.H + h) * a.T + t) * a.Dh;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* x);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* x) {
  unpack8(ld_stream(p), x);
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* x) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float* x);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float* x) {
  *reinterpret_cast<uint4*>(p) = pack8(x);
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float* x) {
  *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

// One CTA per token: thread e8 of the 3*d/8 threads owns 8 consecutive
// elements of the token's [3, H, Dh] slice, i.e. (s, h, sub) with LPR lanes
// (Dh = 8 * LPR, LPR divides 32) per (s, h) row.
template <typename T, int LPR>
__global__ void __launch_bounds__(768) qkv_vec_kernel(QkvArgs a) {
  const int64_t n = blockIdx.x;                   // token = b * T + t
  const int e8 = threadIdx.x;                     // < 3 * H * LPR
  const int row = e8 / LPR;                       // s * H + h
  const int sub = e8 - row * LPR;
  const int s = row / a.H;
  const int h = row - s * a.H;
  const int e0 = sub * 8;
  const T* src = reinterpret_cast<const T*>(a.qkv) + (n * 3 * a.H + row) * (int64_t)a.Dh + e0;

  float x[8];
  load8<T>(src, x);
  const float rho = a.rho[n];
  // sum of squares across the LPR lanes of this row (groups are lane-aligned)
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);

  float outv[8];
  if (s == 2) {
#pragma unroll
    for (int i = 0; i < 8; ++i) outv[i] = x[i] / rho;
  } else {
    float den = sqrtf(ss);
    if (a.eps > 0.f) den = fmaxf(den, rho * a.eps);
    const int t = (int)n - ((int)n / a.T) * a.T;
    const int p0 = e0 >> 1;  // first pair index of this lane
    float c[4], sn[4];
    if ((a.rope_half & 3) == 0 && p0 + 4 <= a.rope_half) {
      float4 cv = *reinterpret_cast<const float4*>(a.cos_tab + (int64_t)t * a.rope_half + p0);
      float4 sv = *reinterpret_cast<const float4*>(a.sin_tab + (int64_t)t * a.rope_half + p0);
      c[0] = cv.x; c[1] = cv.y; c[2] = cv.z; c[3] = cv.w;
      sn[0] = sv.x; sn[1] = sv.y; sn[2] = sv.z; sn[3] = sv.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool rot = p0 + i < a.rope_half;
        c[i] = rot ? a.cos_tab[(int64_t)t * a.rope_half + p0 + i] : 1.f;
        sn[i] = rot ? a.sin_tab[(int64_t)t * a.rope_half + p0 + i] : 0.f;
      }
    }
    const float* sc = a.qk_scale + (int64_t)h * a.Dh + e0;
    float4 s0 = *reinterpret_cast<const float4*>(sc);
    float4 s1 = *reinterpret_cast<const float4*>(sc + 4);
    float scl[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float xe = x[2 * i], xo = x[2 * i + 1];
      float re, ro;
      if (p0 + i < a.rope_half) {
        re = xe * c[i] - xo * sn[i];
        ro = xe * sn[i] + xo * c[i];
      } else {
        re = xe;
        ro = xo;
      }
      outv[2 * i] = (re / den) * (scl[2 * i] * a.qk_mult);
      outv[2 * i + 1] = (ro / den) * (scl[2 * i + 1] * a.qk_mult);
    }
  }
  T* dst = reinterpret_cast<T*>(s == 0 ? a.q : (s == 1 ? a.k : a.v)) + out_offset(a, n, h) + e0;
  store8<T>(dst, outv);
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(p[i]);
  else return p[i];
}
template <typename T>
__device__ __forceinline__ void stf(T* p, int64_t i, float v) {
  if constexpr (sizeof(T) == 2) p[i] = __float2bfloat16_rn(v);
  else p[i] = v;
}

// Generic path: any Dh.  One warp per (token, q|k|v, head) row.
template <typename T>
__global__ void __launch_bounds__(256) qkv_generic_kernel(QkvArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t task = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t ntask = (int64_t)a.B * a.T * 3 * a.H;
  if (task >= ntask) return;
  const int h = (int)(task % a.H);
  const int64_t ns = task / a.H;
  const int s = (int)(ns % 3);
  const int64_t n = ns / 3;
  const T* src = reinterpret_cast<const T*>(a.qkv) + task * (int64_t)a.Dh;
  T* dst = reinterpret_cast<T*>(s == 0 ? a.q : (s == 1 ? a.k : a.v)) + out_offset(a, n, h);
  const float rho = a.rho[n];
  if (s == 2) {
    for (int e = lane; e < a.Dh; e += 32) stf<T>(dst, e, ldf<T>(src, e) / rho);
    return;
  }
  float ss = 0.f;
  for (int e = lane; e < a.Dh; e += 32) {
    float v = ldf<T>(src, e);
    ss += v * v;
  }
  ss = warp_sum_xor<32>(ss);
  float den = sqrtf(ss);
  if (a.eps > 0.f) den = fmaxf(den, rho * a.eps);
  const int t = (int)(n % a.T);
  const float* sc = a.qk_scale + (int64_t)h * a.Dh;
  const int npairs = (a.Dh + 1) / 2;
  for (int p = lane; p < npairs; p += 32) {
    const int e = 2 * p;
    if (p < a.rope_half) {
      const float c = a.cos_tab[(int64_t)t * a.rope_half + p];
      const float sn = a.sin_tab[(int64_t)t * a.rope_half + p];
      const float xe = ldf<T>(src, e), xo = ldf<T>(src, e + 1);
      stf<T>(dst, e, ((xe * c - xo * sn) / den) * (sc[e] * a.qk_mult));
      stf<T>(dst, e + 1, ((xe * sn + xo * c) / den) * (sc[e + 1] * a.qk_mult));
    } else {
      stf<T>(dst, e, (ldf<T>(src, e) / den) * (sc[e] * a.qk_mult));
      if (e + 1 < a.Dh) stf<T>(dst, e + 1, (ldf<T>(src, e + 1) / den) * (sc[e + 1] * a.qk_mult));
    }
  }
}

}  // namespace engpt

using namespace engpt;

extern "C" int engpt_qkv_postprocess(const void* qkv, int dtype, const float* rho, const float* cos_tab,
                                     const float* sin_tab, int rope_half, const float* qk_scale, float qk_mult,
                                     float norm_eps, int B, int T, int H, int Dh, void* q_out, void* k_out,
                                     void* v_out, int out_layout, void* stream) {
  clear_error();
  ENGPT_REQUIRE(B >= 0 && T >= 0 && H > 0 && Dh > 0, ENGPT_ERR_SHAPE, "qkv_postprocess: B=%d T=%d H=%d Dh=%d", B, T,
                H, Dh);
  ENGPT_REQUIRE(rope_half >= 0 && 2 * rope_half <= Dh, ENGPT_ERR_SHAPE, "qkv_postprocess: rope_half=%d Dh=%d",
                rope_half, Dh);
  ENGPT_REQUIRE(out_layout == 0 || out_layout == 1, ENGPT_ERR_ARG, "qkv_postprocess: layout %d", out_layout);
  ENGPT_REQUIRE(dtype == ENGPT_BF16 || dtype == ENGPT_F32, ENGPT_ERR_DTYPE, "qkv_postprocess: dtype %d", dtype);
  if ((int64_t)B * T == 0) return ENGPT_OK;
  ENGPT_REQUIRE(qkv && rho && qk_scale && q_out && k_out && v_out, ENGPT_ERR_ARG, "qkv_postprocess: null pointer");
  ENGPT_REQUIRE(rope_half == 0 || (cos_tab && sin_tab), ENGPT_ERR_ARG, "qkv_postprocess: null rope table");
  QkvArgs a{qkv, rho, cos_tab, sin_tab, rope_half, qk_scale, qk_mult, norm_eps, B, T, H, Dh, q_out, k_out, v_out,
            out_layout};
  const int64_t ntask = (int64_t)B * T * 3 * H;
  cudaStream_t st = as_stream(stream);
  const int esz = dtype == ENGPT_BF16 ? 2 : 4;
  const bool vec_ok = (Dh == 8 || Dh == 16 || Dh == 32 || Dh == 64 || Dh == 128 || Dh == 256) &&
                      aligned(qkv, 16) && aligned(q_out, 16) && aligned(k_out, 16) && aligned(v_out, 16) &&
                      aligned(qk_scale, 16) && (rope_half == 0 || (aligned(cos_tab, 16) && aligned(sin_tab, 16))) &&
                      ((int64_t)Dh * esz) % 16 == 0;
  const int threads_per_token = 3 * H * (Dh / 8);
  if (vec_ok && threads_per_token <= 768 && threads_per_token % 32 == 0) {
    const int lpr = Dh / 8;
    const int64_t blocks = (int64_t)B * T;
    ENGPT_REQUIRE(blocks <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "qkv_postprocess: too large");
#define ENGPT_QKV_LAUNCH(L)                                                                                  \
  case L:                                                                                                    \
    if (dtype == ENGPT_BF16)                                                                                 \
      qkv_vec_kernel<__nv_bfloat16, L><<<(unsigned)blocks, threads_per_token, 0, st>>>(a);                   \
    else                                                                                                     \
      qkv_vec_kernel<float, L><<<(unsigned)blocks, threads_per_token, 0, st>>>(a);                           \
    break;
    switch (lpr) {
      ENGPT_QKV_LAUNCH(1)
      ENGPT_QKV_LAUNCH(2)
      ENGPT_QKV_LAUNCH(4)
      ENGPT_QKV_LAUNCH(8)
      ENGPT_QKV_LAUNCH(16)
      ENGPT_QKV_LAUNCH(32)
      default:
        return set_error(ENGPT_ERR_UNSUPPORTED, "qkv_postprocess: lpr %d", lpr);
    }
#undef ENGPT_QKV_LAUNCH
  } else {
    const int64_t blocks = (ntask * 32 + 255) / 256;
    ENGPT_REQUIRE(blocks <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "qkv_postprocess: too large");
    if (dtype == ENGPT_BF16) qkv_generic_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(a);
    else qkv_generic_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(a);
  }
  return check_launch("qkv_postprocess");
}
