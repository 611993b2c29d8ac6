// Per-row arithmetic of the carried residual + gauge (engpt/kernels.py:277-324),
// shared by the standalone residual kernel and the GEMM epilogue that fuses it.
//   c_b = max(sqrt R0, eps_b);  |u|^2 = c_b^2 R1 + rho^2 R2 + 2 rho c_b R3
//   rho+ = max(|u|, eps_r rho c_b);  g = max(rho+ / max_radius, 1)  (max_radius > 0)
//   Y' = (beta c_b y + alpha rho b) / g,  rho' = rho+ / g
#pragma once

#include "common.cuh"

namespace engpt {

struct RowScalars {
  float coef_y;   // c_b (gauge folded in at write time)
  float coef_b;   // rho
  float g;        // gauge divisor (1 when inactive)
  float inv_g;    // 1 / g
  float rho_new;
  float inv_rho;  // 1 / rho_new, for the Y/rho side output
};

__device__ __forceinline__ RowScalars residual_row_scalars(float branch_eps, float residual_eps, float max_radius,
                                                           float rho, float r0, float r1, float r2, float r3) {
  float cb = sqrtf(fmaxf(r0, 0.0f));
  if (branch_eps > 0.f) cb = fmaxf(cb, branch_eps);
  float rho_cb = rho * cb;
  float u2 = cb * cb * r1 + rho * rho * r2 + 2.0f * rho_cb * r3;
  float rho_plus = sqrtf(fmaxf(u2, 0.0f));
  if (residual_eps > 0.f) rho_plus = fmaxf(rho_plus, residual_eps * rho_cb);
  float g = 1.0f;
  if (max_radius > 0.f) g = fmaxf(rho_plus / max_radius, 1.0f);
  RowScalars s;
  s.coef_y = cb;
  s.coef_b = rho;
  s.g = g;
  s.inv_g = 1.0f / g;
  s.rho_new = (g == 1.0f) ? rho_plus : rho_plus / g;
  s.inv_rho = 1.0f / s.rho_new;
  return s;
}

// u / g, with the per-row reciprocal (exact when the gauge is inactive, within 1 ulp otherwise)
__device__ __forceinline__ float out_value(float alpha, float y, float b, const RowScalars& s) {
  float beta = 1.0f - alpha;
  float u = beta * s.coef_y * y + alpha * s.coef_b * b;
  return u * s.inv_g;
}

}  // namespace engpt
