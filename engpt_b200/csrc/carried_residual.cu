// Fused carried-radius residual + exact gauge (one HBM pass).
//
// Restates carried_residual_gauge (engpt/kernels.py:277-324): per row
//   beta = 1 - alpha
//   R0 = sum b^2, R1 = sum beta^2 y^2, R2 = sum alpha^2 b^2, R3 = sum alpha beta y b
//   c_b = max(sqrt R0, eps_b);  |u|^2 = c_b^2 R1 + rho^2 R2 + 2 rho c_b R3
//   rho+ = max(|u|, eps_r rho c_b);  u = beta c_b y + alpha rho b
//   g = max(rho+ / max_radius, 1)  (skipped when max_radius <= 0)
//   Y' = u / g,  rho' = rho+ / g
// The reference runs ~15 full-width eager passes with [B,T,d] temporaries;
// here one warp owns one row (four warps in small launches, see below): the row's Y (fp32) and branch (bf16/fp32) are
// loaded once into registers with 16-byte loads, the four sums are reduced
// with warp shuffles, and Y', rho' and the next GEMM's operand are written
// in the same pass.  Bytes per row: 4d (Y) + 2d or 4d (branch) + 4d (Y') +
// 8 (rho in/out) + aux (2d for a bf16 operand).
#include "common.cuh"
#include "carried_residual.cuh"

namespace engpt {

struct ResidualArgs {
  const float* y;
  const float* rho;
  const void* branch;
  const float* alpha;
  float alpha_mult;
  int alpha_abs;
  float branch_eps;
  float residual_eps;
  float max_radius;
  int64_t rows;
  int d;
  float* y_out;
  float* rho_out;
  void* aux;
  int aux_mode;
};

__device__ __forceinline__ float eff_alpha(const ResidualArgs& a, float raw) {
  return (a.alpha_abs ? fabsf(raw) : raw) * a.alpha_mult;
}

__device__ __forceinline__ RowScalars finish_row(const ResidualArgs& a, float rho, float r0, float r1, float r2,
                                                 float r3) {
  return residual_row_scalars(a.branch_eps, a.residual_eps, a.max_radius, rho, r0, r1, r2, r3);
}

// Vector path: d % 8 == 0, d <= 256 * MAXCH.  Lane owns 8-column chunks
// (lane, lane + 32, ...).  BT = branch element type.
template <int MAXCH, typename BT>
__global__ void __launch_bounds__(256, (MAXCH <= 4 ? 3 : 1)) residual_vec_kernel(ResidualArgs a) {
  const int lane = threadIdx.x & 31;
  // rows from the last to the first: the GEMM that wrote the branch just before finished on its last rows,
  // which are the ones still in L2
  const int64_t rr = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (rr >= a.rows) return;
  const int64_t row = a.rows - 1 - rr;
  const int nch = a.d >> 3;
  const float* yrow = a.y + row * a.d;
  const BT* brow = reinterpret_cast<const BT*>(a.branch) + row * a.d;

  // the whole row is loaded before any use: Y as fp32, the branch kept in its
  // storage type (bf16 stays packed, 4 registers per 8 values)
  constexpr int BW = sizeof(BT) == 2 ? 4 : 8;  // 32-bit words per 8 branch values
  float yv[MAXCH][8];
  uint32_t bw[MAXCH][BW];
  float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int ch = k * 32 + lane;
    if (ch < nch) {
      const int c = ch << 3;
      float4 y0 = *reinterpret_cast<const float4*>(yrow + c);
      float4 y1 = *reinterpret_cast<const float4*>(yrow + c + 4);
      yv[k][0] = y0.x; yv[k][1] = y0.y; yv[k][2] = y0.z; yv[k][3] = y0.w;
      yv[k][4] = y1.x; yv[k][5] = y1.y; yv[k][6] = y1.z; yv[k][7] = y1.w;
      if constexpr (sizeof(BT) == 2) {
        uint4 raw = ld_stream(brow + c);
        bw[k][0] = raw.x; bw[k][1] = raw.y; bw[k][2] = raw.z; bw[k][3] = raw.w;
      } else {
        uint4 b0 = *reinterpret_cast<const uint4*>(brow + c);
        uint4 b1 = *reinterpret_cast<const uint4*>(brow + c + 4);
        bw[k][0] = b0.x; bw[k][1] = b0.y; bw[k][2] = b0.z; bw[k][3] = b0.w;
        bw[k][4] = b1.x; bw[k][5] = b1.y; bw[k][6] = b1.z; bw[k][7] = b1.w;
      }
    }
  }
  auto bval = [&](int k, int i) -> float {
    if constexpr (sizeof(BT) == 2) {
      const uint32_t w = bw[k][i >> 1];
      return __uint_as_float((i & 1) ? (w & 0xffff0000u) : (w << 16));
    } else {
      return __uint_as_float(bw[k][i]);
    }
  };
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int ch = k * 32 + lane;
    if (ch < nch) {
      const int c = ch << 3;
      float4 a0 = *reinterpret_cast<const float4*>(a.alpha + c);
      float4 a1 = *reinterpret_cast<const float4*>(a.alpha + c + 4);
      float al[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float alpha = eff_alpha(a, al[i]);
        float beta = 1.0f - alpha;
        float y = yv[k][i], b = bval(k, i);
        float bsq = b * b;
        r0 += bsq;
        r1 += (beta * beta) * (y * y);
        r2 += (alpha * alpha) * bsq;
        r3 += ((alpha * beta) * y) * b;
      }
    }
  }
  r0 = warp_sum_xor<32>(r0);
  r1 = warp_sum_xor<32>(r1);
  r2 = warp_sum_xor<32>(r2);
  r3 = warp_sum_xor<32>(r3);
  const RowScalars s = finish_row(a, a.rho[row], r0, r1, r2, r3);

  float* yo = a.y_out + row * a.d;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int ch = k * 32 + lane;
    if (ch < nch) {
      const int c = ch << 3;
      float4 a0 = *reinterpret_cast<const float4*>(a.alpha + c);
      float4 a1 = *reinterpret_cast<const float4*>(a.alpha + c + 4);
      float al[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = out_value(eff_alpha(a, al[i]), yv[k][i], bval(k, i), s);
      *reinterpret_cast<float4*>(yo + c) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(yo + c + 4) = make_float4(o[4], o[5], o[6], o[7]);
      if (a.aux_mode == ENGPT_AUX_BF16_Y) {
        st_stream(reinterpret_cast<__nv_bfloat16*>(a.aux) + row * a.d + c, pack8(o));
      } else if (a.aux_mode == ENGPT_AUX_BF16_H || a.aux_mode == ENGPT_AUX_F32_H) {
        float h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = o[i] * s.inv_rho;
        if (a.aux_mode == ENGPT_AUX_BF16_H) {
          st_stream(reinterpret_cast<__nv_bfloat16*>(a.aux) + row * a.d + c, pack8(h));
        } else {
          float* ho = reinterpret_cast<float*>(a.aux) + row * a.d + c;
          *reinterpret_cast<float4*>(ho) = make_float4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<float4*>(ho + 4) = make_float4(h[4], h[5], h[6], h[7]);
        }
      }
    }
  }
  if (lane == 0) a.rho_out[row] = s.rho_new;
}

__device__ __forceinline__ float ld_branch(const void* p, int bt, int64_t i) {
  return bt == ENGPT_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                          : reinterpret_cast<const float*>(p)[i];
}

// Generic path: any d.  One warp per row, two strided passes (the second
// re-reads the row, which stays in L1/L2 for the row sizes this serves).
// In-place safe: every element is read in both passes by the lane that
// writes it, and the first pass ends (warp reduction) before any write.
__global__ void __launch_bounds__(256) residual_generic_kernel(ResidualArgs a, int bt) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= a.rows) return;
  const float* yrow = a.y + row * a.d;
  float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
  for (int c = lane; c < a.d; c += 32) {
    float alpha = eff_alpha(a, a.alpha[c]);
    float beta = 1.0f - alpha;
    float y = yrow[c];
    float b = ld_branch(a.branch, bt, row * a.d + c);
    float bsq = b * b;
    r0 += bsq;
    r1 += (beta * beta) * (y * y);
    r2 += (alpha * alpha) * bsq;
    r3 += ((alpha * beta) * y) * b;
  }
  r0 = warp_sum_xor<32>(r0);
  r1 = warp_sum_xor<32>(r1);
  r2 = warp_sum_xor<32>(r2);
  r3 = warp_sum_xor<32>(r3);
  const RowScalars s = finish_row(a, a.rho[row], r0, r1, r2, r3);
  for (int c = lane; c < a.d; c += 32) {
    float alpha = eff_alpha(a, a.alpha[c]);
    float o = out_value(alpha, yrow[c], ld_branch(a.branch, bt, row * a.d + c), s);
    a.y_out[row * a.d + c] = o;
    if (a.aux_mode == ENGPT_AUX_BF16_Y) {
      reinterpret_cast<__nv_bfloat16*>(a.aux)[row * a.d + c] = __float2bfloat16_rn(o);
    } else if (a.aux_mode == ENGPT_AUX_BF16_H) {
      reinterpret_cast<__nv_bfloat16*>(a.aux)[row * a.d + c] = __float2bfloat16_rn(o * s.inv_rho);
    } else if (a.aux_mode == ENGPT_AUX_F32_H) {
      reinterpret_cast<float*>(a.aux)[row * a.d + c] = o * s.inv_rho;
    }
  }
  if (lane == 0) a.rho_out[row] = s.rho_new;
}

// Small launches: four warps share a row (two rows per 256-thread block), thread t of the row owning the
// 8-column chunks t, t + 128, ...  With one warp per row a launch of a few thousand rows is only two or three
// waves of resident blocks, and its partial last wave costs up to a third of the time (8192 rows at d = 1024:
// 1024 blocks over 444 resident); four times the warps spread the same rows evenly.  The four warps' partial
// sums meet in shared memory and every thread of the row adds them in the same order.  In-place safe: a
// thread writes only the elements it read, after the barrier, and the row's rho is read before it.
constexpr int kSplitWarps = 4;

template <int MAXCH, typename BT>
__global__ void __launch_bounds__(256) residual_split_kernel(ResidualArgs a) {
  __shared__ float part[2][kSplitWarps][4];
  const int lane = threadIdx.x & 31;
  const int wrow = (threadIdx.x >> 5) & (kSplitWarps - 1);   // warp within its row
  const int rib = threadIdx.x >> 7;                           // row within the block
  const int t = wrow * 32 + lane;                             // thread within the row
  const int64_t rr = (int64_t)blockIdx.x * 2 + rib;
  const bool valid = rr < a.rows;
  // rows from the last to the first, as the one-warp kernel
  const int64_t row = valid ? a.rows - 1 - rr : 0;
  const int nch = a.d >> 3;
  const float* yrow = a.y + row * a.d;
  const BT* brow = reinterpret_cast<const BT*>(a.branch) + row * a.d;
  constexpr int BW = sizeof(BT) == 2 ? 4 : 8;
  float yv[MAXCH][8];
  uint32_t bw[MAXCH][BW];
  float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int ch = k * 32 * kSplitWarps + t;
    if (valid && ch < nch) {
      const int c = ch << 3;
      float4 y0 = *reinterpret_cast<const float4*>(yrow + c);
      float4 y1 = *reinterpret_cast<const float4*>(yrow + c + 4);
      yv[k][0] = y0.x; yv[k][1] = y0.y; yv[k][2] = y0.z; yv[k][3] = y0.w;
      yv[k][4] = y1.x; yv[k][5] = y1.y; yv[k][6] = y1.z; yv[k][7] = y1.w;
      if constexpr (sizeof(BT) == 2) {
        uint4 raw = ld_stream(brow + c);
        bw[k][0] = raw.x; bw[k][1] = raw.y; bw[k][2] = raw.z; bw[k][3] = raw.w;
      } else {
        uint4 b0 = *reinterpret_cast<const uint4*>(brow + c);
        uint4 b1 = *reinterpret_cast<const uint4*>(brow + c + 4);
        bw[k][0] = b0.x; bw[k][1] = b0.y; bw[k][2] = b0.z; bw[k][3] = b0.w;
        bw[k][4] = b1.x; bw[k][5] = b1.y; bw[k][6] = b1.z; bw[k][7] = b1.w;
      }
    }
  }
  const float rho = valid ? a.rho[row] : 1.0f;
  auto bval = [&](int k, int i) -> float {
    if constexpr (sizeof(BT) == 2) {
      const uint32_t w = bw[k][i >> 1];
      return __uint_as_float((i & 1) ? (w & 0xffff0000u) : (w << 16));
    } else {
      return __uint_as_float(bw[k][i]);
    }
  };
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int ch = k * 32 * kSplitWarps + t;
    if (valid && ch < nch) {
      const int c = ch << 3;
      float4 a0 = *reinterpret_cast<const float4*>(a.alpha + c);
      float4 a1 = *reinterpret_cast<const float4*>(a.alpha + c + 4);
      float al[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float alpha = eff_alpha(a, al[i]);
        float beta = 1.0f - alpha;
        float y = yv[k][i], b = bval(k, i);
        float bsq = b * b;
        r0 += bsq;
        r1 += (beta * beta) * (y * y);
        r2 += (alpha * alpha) * bsq;
        r3 += ((alpha * beta) * y) * b;
      }
    }
  }
  r0 = warp_sum_xor<32>(r0);
  r1 = warp_sum_xor<32>(r1);
  r2 = warp_sum_xor<32>(r2);
  r3 = warp_sum_xor<32>(r3);
  if (lane == 0) {
    part[rib][wrow][0] = r0;
    part[rib][wrow][1] = r1;
    part[rib][wrow][2] = r2;
    part[rib][wrow][3] = r3;
  }
  __syncthreads();
  if (!valid) return;
  float sum[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) sum[q] = (part[rib][0][q] + part[rib][1][q]) + (part[rib][2][q] + part[rib][3][q]);
  const RowScalars s = finish_row(a, rho, sum[0], sum[1], sum[2], sum[3]);

  float* yo = a.y_out + row * a.d;
#pragma unroll
  for (int k = 0; k < MAXCH; ++k) {
    const int ch = k * 32 * kSplitWarps + t;
    if (ch < nch) {
      const int c = ch << 3;
      float4 a0 = *reinterpret_cast<const float4*>(a.alpha + c);
      float4 a1 = *reinterpret_cast<const float4*>(a.alpha + c + 4);
      float al[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = out_value(eff_alpha(a, al[i]), yv[k][i], bval(k, i), s);
      *reinterpret_cast<float4*>(yo + c) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(yo + c + 4) = make_float4(o[4], o[5], o[6], o[7]);
      if (a.aux_mode == ENGPT_AUX_BF16_Y) {
        st_stream(reinterpret_cast<__nv_bfloat16*>(a.aux) + row * a.d + c, pack8(o));
      } else if (a.aux_mode == ENGPT_AUX_BF16_H || a.aux_mode == ENGPT_AUX_F32_H) {
        float h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = o[i] * s.inv_rho;
        if (a.aux_mode == ENGPT_AUX_BF16_H) {
          st_stream(reinterpret_cast<__nv_bfloat16*>(a.aux) + row * a.d + c, pack8(h));
        } else {
          float* ho = reinterpret_cast<float*>(a.aux) + row * a.d + c;
          *reinterpret_cast<float4*>(ho) = make_float4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<float4*>(ho + 4) = make_float4(h[4], h[5], h[6], h[7]);
        }
      }
    }
  }
  if (t == 0) a.rho_out[row] = s.rho_new;
}

}  // namespace engpt

using namespace engpt;

extern "C" int engpt_carried_residual_gauge(const float* y, const float* rho, const void* branch, int branch_dtype,
                                            const float* alpha, float alpha_mult, int alpha_abs, float branch_eps,
                                            float residual_eps, float max_radius, int64_t rows, int d,
                                            float* y_out, float* rho_out, void* aux_out, int aux_mode,
                                            void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows >= 0 && d > 0, ENGPT_ERR_SHAPE, "carried_residual_gauge: rows=%lld d=%d", (long long)rows, d);
  if (rows == 0) return ENGPT_OK;
  ENGPT_REQUIRE(y && rho && branch && alpha && y_out && rho_out, ENGPT_ERR_ARG,
                "carried_residual_gauge: null pointer");
  ENGPT_REQUIRE(branch_dtype == ENGPT_BF16 || branch_dtype == ENGPT_F32, ENGPT_ERR_DTYPE,
                "carried_residual_gauge: branch dtype %d", branch_dtype);
  ENGPT_REQUIRE(aux_mode >= ENGPT_AUX_NONE && aux_mode <= ENGPT_AUX_F32_H, ENGPT_ERR_ARG,
                "carried_residual_gauge: aux_mode %d", aux_mode);
  ENGPT_REQUIRE(aux_mode == ENGPT_AUX_NONE || aux_out, ENGPT_ERR_ARG, "carried_residual_gauge: aux_out is null");
  ResidualArgs a{y, rho, branch, alpha, alpha_mult, alpha_abs, branch_eps, residual_eps, max_radius,
                 rows, d, y_out, rho_out, aux_out, aux_mode};
  const int threads = 256;
  const int64_t blocks64 = (rows * 32 + threads - 1) / threads;
  ENGPT_REQUIRE(blocks64 <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "carried_residual_gauge: too many rows");
  const int blocks = (int)blocks64;
  cudaStream_t st = as_stream(stream);
  const bool vec_ok = (d % 8) == 0 && d <= 2048 && aligned(y, 16) && aligned(y_out, 16) && aligned(branch, 16) &&
                      aligned(alpha, 16) && (aux_mode == ENGPT_AUX_NONE || aligned(aux_out, 16));
  // one warp per row would fill fewer than four waves of its resident blocks (three per SM): four warps per row
  const bool split = vec_ok && blocks64 < 4 * 3 * (int64_t)num_sms();
  if (split) {
    const unsigned sblocks = (unsigned)((rows + 1) / 2);
    if ((d / 8 + 127) / 128 <= 1) {
      if (branch_dtype == ENGPT_BF16)
        residual_split_kernel<1, __nv_bfloat16><<<sblocks, threads, 0, st>>>(a);
      else
        residual_split_kernel<1, float><<<sblocks, threads, 0, st>>>(a);
    } else {
      if (branch_dtype == ENGPT_BF16)
        residual_split_kernel<2, __nv_bfloat16><<<sblocks, threads, 0, st>>>(a);
      else
        residual_split_kernel<2, float><<<sblocks, threads, 0, st>>>(a);
    }
  } else if (vec_ok) {
    const int nch = d / 8;
    const int maxch = (nch + 31) / 32;
#define ENGPT_RES_LAUNCH(MC)                                                                  \
  if (branch_dtype == ENGPT_BF16)                                                             \
    residual_vec_kernel<MC, __nv_bfloat16><<<blocks, threads, 0, st>>>(a);                    \
  else                                                                                        \
    residual_vec_kernel<MC, float><<<blocks, threads, 0, st>>>(a);
    if (maxch <= 1) {
      ENGPT_RES_LAUNCH(1)
    } else if (maxch <= 2) {
      ENGPT_RES_LAUNCH(2)
    } else if (maxch <= 4) {
      ENGPT_RES_LAUNCH(4)
    } else {
      ENGPT_RES_LAUNCH(8)
    }
#undef ENGPT_RES_LAUNCH
  } else {
    residual_generic_kernel<<<blocks, threads, 0, st>>>(a, branch_dtype);
  }
  return check_launch("carried_residual_gauge");
}
