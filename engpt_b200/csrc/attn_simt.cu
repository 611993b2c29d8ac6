// Causal attention on CUDA cores (fp32 or bf16 in/out, any head_dim <= 256).
//
// This is the exact-arithmetic path of causal_sdpa (engpt/kernels.py:417-431)
// used for fp32 mode (where tensor-core tf32/bf16 rounding would exceed the
// 1e-5 fp32 tolerance) and for head dims the tcgen05 kernel does not cover.
// A CTA owns 32 consecutive queries of one (batch, head); K/V tiles of 32
// keys are staged in shared memory as fp32; each warp keeps four query rows
// with an online softmax (running max and sum) in fp32.
#include "common.cuh"

namespace engpt {

constexpr int kSimtQ = 32;   // queries per CTA
constexpr int kSimtK = 32;   // keys per tile
constexpr int kSimtWarps = 8;
constexpr int kRowsPerWarp = kSimtQ / kSimtWarps;

struct SimtAttnArgs {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int B, T, H, Dh;
  float scale;
  int64_t qs[3], ks[3], vs[3], os[3];
};

template <typename T>
__device__ __forceinline__ float ldv(const T* p, int64_t i) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(p[i]);
  else return p[i];
}

template <typename T, int MAXV>  // MAXV = ceil(Dh / 32)
__global__ void __launch_bounds__(kSimtWarps * 32) attn_simt_kernel(SimtAttnArgs a) {
  extern __shared__ float smem[];
  const int ldk = a.Dh + 1;
  float* sK = smem;                       // [kSimtK][Dh+1]
  float* sV = sK + kSimtK * ldk;          // [kSimtK][Dh+1]
  float* sQ = sV + kSimtK * ldk;          // [kSimtQ][Dh]

  const int nqb = (a.T + kSimtQ - 1) / kSimtQ;
  // heaviest query blocks first
  const int64_t lin = blockIdx.x;
  const int bh = (int)(lin % ((int64_t)a.B * a.H));
  const int qb = nqb - 1 - (int)(lin / ((int64_t)a.B * a.H));
  const int b = bh / a.H, h = bh % a.H;
  const int q0 = qb * kSimtQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const T* Q = reinterpret_cast<const T*>(a.q) + b * a.qs[0] + h * a.qs[2];
  const T* K = reinterpret_cast<const T*>(a.k) + b * a.ks[0] + h * a.ks[2];
  const T* V = reinterpret_cast<const T*>(a.v) + b * a.vs[0] + h * a.vs[2];
  T* O = reinterpret_cast<T*>(a.o) + b * a.os[0] + h * a.os[2];

  for (int i = threadIdx.x; i < kSimtQ * a.Dh; i += blockDim.x) {
    int r = i / a.Dh, c = i % a.Dh;
    int t = q0 + r;
    sQ[i] = t < a.T ? ldv(Q, (int64_t)t * a.qs[1] + c) : 0.f;
  }

  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][MAXV];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) acc[r][i] = 0.f;
  }

  const int kend = min(a.T, q0 + kSimtQ);  // keys needed by this block
  for (int k0 = 0; k0 < kend; k0 += kSimtK) {
    __syncthreads();
    for (int i = threadIdx.x; i < kSimtK * a.Dh; i += blockDim.x) {
      int r = i / a.Dh, c = i % a.Dh;
      int t = k0 + r;
      sK[r * ldk + c] = t < a.T ? ldv(K, (int64_t)t * a.ks[1] + c) : 0.f;
      sV[r * ldk + c] = t < a.T ? ldv(V, (int64_t)t * a.vs[1] + c) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int qr = warp * kRowsPerWarp + r;
      const int tq = q0 + qr;
      if (tq >= a.T || k0 > tq) continue;  // warp-uniform
      const int key = k0 + lane;
      float s = 0.f;
      const float* qrow = sQ + qr * a.Dh;
      const float* krow = sK + lane * ldk;
      for (int c = 0; c < a.Dh; ++c) s += qrow[c] * krow[c];
      s *= a.scale;
      const bool valid = key <= tq && key < a.T;
      s = valid ? s : -INFINITY;
      const float tmax = warp_max(s);
      const float mnew = fmaxf(m[r], tmax);
      const float p = valid ? expf(s - mnew) : 0.f;
      const float corr = expf(m[r] - mnew);  // m = -inf at start -> 0
      l[r] = l[r] * corr + warp_sum_xor<32>(p);
      m[r] = mnew;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) acc[r][i] *= corr;
      for (int j = 0; j < kSimtK; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        if (pj != 0.f) {
#pragma unroll
          for (int i = 0; i < MAXV; ++i) {
            const int c = lane + 32 * i;
            if (c < a.Dh) acc[r][i] += pj * sV[j * ldk + c];
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int tq = q0 + warp * kRowsPerWarp + r;
    if (tq >= a.T) continue;
    const float inv = 1.0f / l[r];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < a.Dh) {
        const float v = acc[r][i] * inv;
        if constexpr (sizeof(T) == 2) O[(int64_t)tq * a.os[1] + c] = __float2bfloat16_rn(v);
        else O[(int64_t)tq * a.os[1] + c] = v;
      }
    }
  }
}

int launch_attn_simt(const void* q, const void* k, const void* v, void* o, int dtype, int B, int T, int H, int Dh,
                     float scale, const int64_t* strides, cudaStream_t st) {
  ENGPT_REQUIRE(Dh <= 256, ENGPT_ERR_UNSUPPORTED, "attention (simt): head_dim %d > 256", Dh);
  SimtAttnArgs a;
  a.q = q; a.k = k; a.v = v; a.o = o;
  a.B = B; a.T = T; a.H = H; a.Dh = Dh; a.scale = scale;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = strides[i];
    a.ks[i] = strides[3 + i];
    a.vs[i] = strides[6 + i];
    a.os[i] = strides[9 + i];
  }
  const int nqb = (T + kSimtQ - 1) / kSimtQ;
  const int64_t blocks = (int64_t)nqb * B * H;
  ENGPT_REQUIRE(blocks <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "attention (simt): grid too large");
  const size_t smem = sizeof(float) * (size_t)(2 * kSimtK * (Dh + 1) + kSimtQ * Dh);
  const int maxv = (Dh + 31) / 32;
#define ENGPT_SIMT_CASE(MV)                                                                              \
  if (maxv <= MV) {                                                                                      \
    if (dtype == ENGPT_BF16) {                                                                           \
      auto kern = attn_simt_kernel<__nv_bfloat16, MV>;                                                   \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                \
      kern<<<(unsigned)blocks, kSimtWarps * 32, smem, st>>>(a);                                          \
    } else {                                                                                             \
      auto kern = attn_simt_kernel<float, MV>;                                                           \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                \
      kern<<<(unsigned)blocks, kSimtWarps * 32, smem, st>>>(a);                                          \
    }                                                                                                    \
    return check_launch("attention (simt)");                                                             \
  }
  ENGPT_SIMT_CASE(1)
  ENGPT_SIMT_CASE(2)
  ENGPT_SIMT_CASE(4)
  ENGPT_SIMT_CASE(8)
#undef ENGPT_SIMT_CASE
  return set_error(ENGPT_ERR_UNSUPPORTED, "attention (simt): head_dim %d", Dh);
}

}  // namespace engpt
