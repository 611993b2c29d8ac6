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
// [B,T,H,Dh], to the head-major [B,H,T,Dh], or back over qkv itself
// ([B,T,3,H,Dh], as the reference's no-grad path does), which the attention
// kernel's TMA reads through strided tensor maps.
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
  int layout;  // ENGPT_QKV_BTHD, ENGPT_QKV_BHTD or ENGPT_QKV_INPLACE
};

// Element offset of row (token n, part s, head h) in the output of part s.
// Token index n < 2^31 (checked on the host), so the (b, t) split is 32-bit.
__device__ __forceinline__ int64_t out_offset(const QkvArgs& a, int64_t n, int s, int h) {
  if (a.layout == ENGPT_QKV_INPLACE) return ((n * 3 + s) * a.H + h) * (int64_t)a.Dh;
  if (a.layout == ENGPT_QKV_BTHD) return (n * a.H + h) * (int64_t)a.Dh;
  const int ni = (int)n;
  const int b = ni / a.T;
  const int t = ni - b * a.T;
  return ((int64_t)(b * a.H + h) * a.T + t) * a.Dh;
}

// Eight raw elements as loaded (bf16: one 16-byte word), converted to fp32 only when used, so a thread
// keeps its tokens' rows in few registers and more CTAs (more loads in flight) fit on an SM.
template <typename T>
struct Raw8;
template <>
struct Raw8<__nv_bfloat16> {
  uint4 v;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { v = ld_once(p); }  // coherent: may be in place
  __device__ __forceinline__ void zero() { v = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ void to_float(float* x) const { unpack8(v, x); }
};
template <>
struct Raw8<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = *reinterpret_cast<const float4*>(p);
    b = *reinterpret_cast<const float4*>(p + 4);
  }
  __device__ __forceinline__ void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void to_float(float* x) const {
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
};

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

// A CTA owns kQkvTok consecutive tokens; its threads form an (H * LPR, 3)
// block: threadIdx.y is q|k|v, threadIdx.x / LPR the head and threadIdx.x % LPR
// the 8-element slice (Dh = 8 * LPR, LPR a power of two dividing 32), so every
// index is a shift.  All global loads (the tokens' qkv slices, rho, and the
// tokens' rotary rows, staged in shared memory) are issued before any is used.
// The kernel is instruction-bound at HBM speed, so per-token work is kept
// minimal: scales are loaded once, bf16 results use the MUFU reciprocal forms
// (about 2 ulp, far below bf16 rounding; fp32 results use IEEE sqrt and
// division), and an in-place result reuses its load address.  In place is
// safe: each thread writes only the elements it read, after reading them.
constexpr int kQkvTok = 2;
constexpr int kQkvMaxHalf = 128;   // rotary pairs staged per token (head_dim <= 256)

template <typename T, int LPR>
__global__ void __launch_bounds__(768, 2) qkv_vec_kernel(QkvArgs a) {
  __shared__ __align__(16) float s_cos[kQkvTok][kQkvMaxHalf];
  __shared__ __align__(16) float s_sin[kQkvTok][kQkvMaxHalf];
  constexpr bool kFast = sizeof(T) == 2;
  const int ntok = a.B * a.T;
  const int n0 = blockIdx.x * kQkvTok;
  const int s = threadIdx.y;                      // 0: q, 1: k, 2: v
  const int h = threadIdx.x / LPR;
  const int sub = threadIdx.x % LPR;
  const int e0 = sub * 8;
  const int row = s * a.H + h;
  const int64_t tok_stride = (int64_t)3 * a.H * a.Dh;
  T* src = const_cast<T*>(reinterpret_cast<const T*>(a.qkv)) + ((int64_t)n0 * 3 * a.H + row) * a.Dh + e0;

  Raw8<T> raw[kQkvTok];
  float rho[kQkvTok];
#pragma unroll
  for (int k = 0; k < kQkvTok; ++k) {
    if (n0 + k < ntok) {
      raw[k].load(src + k * tok_stride);
      rho[k] = a.rho[n0 + k];
    } else {
      raw[k].zero();
      rho[k] = 1.f;
    }
  }
  // rotary rows of the CTA's tokens -> shared memory
  const int half = a.rope_half;
  const int t0 = n0 % a.T;
  for (int pi = threadIdx.y * blockDim.x + threadIdx.x; pi < half; pi += blockDim.x * blockDim.y) {
#pragma unroll
    for (int k = 0; k < kQkvTok; ++k) {
      int t = t0 + k;
      while (t >= a.T) t -= a.T;  // tokens of the next sequence
      const bool live = n0 + k < ntok;
      s_cos[k][pi] = live ? a.cos_tab[(int64_t)t * half + pi] : 1.f;
      s_sin[k][pi] = live ? a.sin_tab[(int64_t)t * half + pi] : 0.f;
    }
  }
  float scl[8];
  if (s < 2) {
    const float* sc = a.qk_scale + (int64_t)h * a.Dh + e0;
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(sc));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(sc + 4));
    scl[0] = s0.x * a.qk_mult; scl[1] = s0.y * a.qk_mult; scl[2] = s0.z * a.qk_mult; scl[3] = s0.w * a.qk_mult;
    scl[4] = s1.x * a.qk_mult; scl[5] = s1.y * a.qk_mult; scl[6] = s1.z * a.qk_mult; scl[7] = s1.w * a.qk_mult;
  }
  __syncthreads();
  T* base = reinterpret_cast<T*>(s == 0 ? a.q : (s == 1 ? a.k : a.v));
  const bool inplace = a.layout == ENGPT_QKV_INPLACE;
  const int p0 = e0 >> 1;      // first rotary pair of this lane (a multiple of 4)
  const bool rot = p0 < half;  // half is a multiple of 4: a lane's 4 pairs rotate together or not at all
#pragma unroll
  for (int k = 0; k < kQkvTok; ++k) {
    const int n = n0 + k;
    float x[8];
    raw[k].to_float(x);
    // sum of squares across the LPR lanes of this row (groups are lane-aligned; all lanes take part)
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (n >= ntok) continue;
    float outv[8];
    if (s == 2) {
      const float inv_rho = kFast ? __fdividef(1.0f, rho[k]) : 1.0f / rho[k];
#pragma unroll
      for (int i = 0; i < 8; ++i) outv[i] = x[i] * inv_rho;
    } else {
      // 1 / max(|q|, rho*eps): one reciprocal per row, then multiplies
      float inv_den;
      if (kFast) {
        inv_den = rsqrtf(ss);
        if (a.eps > 0.f) inv_den = fminf(inv_den, __fdividef(1.0f, rho[k] * a.eps));
      } else {
        float den = sqrtf(ss);
        if (a.eps > 0.f) den = fmaxf(den, rho[k] * a.eps);
        inv_den = 1.0f / den;
      }
      if (rot) {
        const float4 c4 = *reinterpret_cast<const float4*>(&s_cos[k][p0]);
        const float4 s4 = *reinterpret_cast<const float4*>(&s_sin[k][p0]);
        const float c[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float xe = x[2 * i], xo = x[2 * i + 1];
          outv[2 * i] = ((xe * c[i] - xo * sn[i]) * inv_den) * scl[2 * i];
          outv[2 * i + 1] = ((xe * sn[i] + xo * c[i]) * inv_den) * scl[2 * i + 1];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) outv[i] = (x[i] * inv_den) * scl[i];
      }
    }
    store8<T>(inplace ? src + k * tok_stride : base + out_offset(a, n, s, h) + e0, outv);
  }
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
  T* dst = reinterpret_cast<T*>(s == 0 ? a.q : (s == 1 ? a.k : a.v)) + out_offset(a, n, s, h);
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
  ENGPT_REQUIRE(out_layout >= ENGPT_QKV_BTHD && out_layout <= ENGPT_QKV_INPLACE, ENGPT_ERR_ARG,
                "qkv_postprocess: layout %d", out_layout);
  if (out_layout == ENGPT_QKV_INPLACE) {
    // q, k, v are written over qkv: their pointers must be null or the qkv buffer itself
    ENGPT_REQUIRE((!q_out || q_out == qkv) && (!k_out || k_out == qkv) && (!v_out || v_out == qkv),
                  ENGPT_ERR_ARG, "qkv_postprocess: in-place outputs must be the qkv buffer");
    q_out = k_out = v_out = const_cast<void*>(qkv);
  }
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
                      rope_half <= kQkvMaxHalf && rope_half % 4 == 0 &&
                      aligned(qkv, 16) && aligned(q_out, 16) && aligned(k_out, 16) && aligned(v_out, 16) &&
                      aligned(qk_scale, 16) && (rope_half == 0 || (aligned(cos_tab, 16) && aligned(sin_tab, 16))) &&
                      ((int64_t)Dh * esz) % 16 == 0;
  const int threads_per_token = 3 * H * (Dh / 8);
  if (vec_ok && threads_per_token <= 768 && threads_per_token % 32 == 0) {
    const int lpr = Dh / 8;
    ENGPT_REQUIRE((int64_t)B * T <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "qkv_postprocess: too large");
    const int64_t blocks = ((int64_t)B * T + kQkvTok - 1) / kQkvTok;
#define ENGPT_QKV_LAUNCH(L)                                                                                  \
  case L:                                                                                                    \
    if (dtype == ENGPT_BF16)                                                                                 \
      qkv_vec_kernel<__nv_bfloat16, L><<<(unsigned)blocks, dim3(H * L, 3), 0, st>>>(a);                       \
    else                                                                                                     \
      qkv_vec_kernel<float, L><<<(unsigned)blocks, dim3(H * L, 3), 0, st>>>(a);                               \
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
