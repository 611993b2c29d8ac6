// Persistent tcgen05 GEMM for B200 (sm_100a) with a fused epilogue:
//   C[M, N] = A[M, K] * B[N, K]^T   (bf16 operands, K contiguous; fp32 accumulation in TMEM)
//
// The dense projections of the enGPT block (engpt/models.py:140-182) are this
// shape with A = the activations and B = an nn.Linear weight.  A CTA owns one
// SM and walks 128 x 256 output tiles (tile t = blockIdx.x + i * gridDim.x,
// row-block major, so the 256 KB A row-block a wave of CTAs shares stays in
// L2).  Warp roles (192 threads):
//   warp 0      TMA producer: 64-wide K slices of A (128 rows) and B (256 rows)
//               into a 4-stage shared-memory ring (128-byte swizzle)
//   warp 1      TMEM allocator + MMA issuer (the whole warp runs the loop; one
//               elected lane issues): 4 x tcgen05.mma M128 N256 K16 per slice
//               into one of two 256-column fp32 accumulators
//   warps 2..5  epilogue: thread = output row (TMEM lane); reads the finished
//               accumulator 32 columns at a time with tcgen05.ld, applies the
//               epilogue functor and stores, while the MMAs of the next tile
//               fill the other accumulator.
// Every wait is bounded (mbar_wait); on a timeout the kernel records
// ENGPT_ERR_TIMEOUT in the device status word, drains its copies and MMAs,
// frees TMEM and returns.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace engpt {
namespace gemm {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kABytes = BM * BK * 2;   // 16 KB
constexpr int kBBytes = BN * BK * 2;   // 32 KB

constexpr int kOutBytes = BM * 64 * 2;   // one 64-column bf16 output chunk of the tile (16 KB)

struct Layout {
  static constexpr int A = 0;
  static constexpr int B = A + kStages * kABytes;
  static constexpr int OUT = B + kStages * kBBytes;        // 2 output staging buffers
  static constexpr int BAR = OUT + 2 * kOutBytes;
  static constexpr int kBars = 16;
  static constexpr int MISC = BAR + kBars * 8;
  static constexpr int TOTAL = MISC + 16;
  static constexpr int kDynSmem = TOTAL + 1024;
};
static_assert(Layout::kDynSmem <= 227 * 1024, "shared memory");

enum { B_FULL = 0, B_EMPTY = B_FULL + kStages, B_ACC_FULL = B_EMPTY + kStages, B_ACC_EMPTY = B_ACC_FULL + 2,
       B_FINAL = B_ACC_EMPTY + 2 };
static_assert(B_FINAL < Layout::kBars, "barrier slots");

struct Shape {
  int M, N, K;
  int tiles_n, tiles;   // output tiles along N, total
  // B rows of tile column tn: [b0 + tn * b_step, +128) and [b1 + tn * b_step, +128) fill the 256 B rows
  // (accumulator columns 0-127 and 128-255).  Plain GEMM: b0 = 0, b1 = 128, b_step = 256.  Up/gate with
  // SwiGLU: b0 = 0, b1 = width (the gate half of the weight), b_step = 128.
  int b0, b1, b_step;
};

// Output staging: each epilogue thread writes its row's 64 bf16 results of one output chunk (128 bytes)
// into a 128B-swizzled shared buffer; one thread then stores the 64 x 128 box with TMA (clipped at the
// tensor's end), so the global writes are full lines instead of 32 scattered rows per warp instruction.
// Two buffers alternate; a buffer is rewritten only after the store that read it has finished reading.
struct OutStage {
  uint8_t* buf;            // 2 x kOutBytes
  uint32_t sbuf;
  const CUtensorMap* map;
  int r;                   // this thread's row in the tile
  bool leader;             // issues the stores
  int count;
  __device__ __forceinline__ void put(int col, int row0, const uint4* v8) {
    const int b = count & 1;
    if (leader) bulk_wait_group_read<1>();
    bar_sync_named(1, 128);
    uint8_t* rowp = buf + b * kOutBytes + r * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(rowp + ((j ^ (r & 7)) << 4)) = v8[j];
    fence_proxy_async_smem();
    bar_sync_named(1, 128);
    if (leader) {
      tma_store_2d(map, col, row0, sbuf + b * kOutBytes);
      bulk_commit_group();
    }
    ++count;
  }
};

__device__ __forceinline__ void load_acc32(uint32_t taddr, float* v) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld32(r);
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Epilogues: tile(m0, m, tn, tacc, out) runs on every epilogue thread for row m = m0 + r of tile column tn;
// tacc is the TMEM address of this thread's accumulator row (column 0 of the 256).

// Plain bf16 output: C[m, 256 tn + c] = acc[c].
struct StoreBf16 {
  __device__ __forceinline__ void tile(int m0, int m, int tn, uint32_t tacc, OutStage& out) const {
#pragma unroll 1
    for (int oc = 0; oc < BN / 64; ++oc) {
      float v[64];
      load_acc32(tacc + 64 * oc, v);
      load_acc32(tacc + 64 * oc + 32, v + 32);
      uint4 o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = pack8(v + 8 * j);
      out.put(tn * BN + 64 * oc, m0, o);
    }
  }
};

// QKV projection + qkv_postprocess_from_carried (engpt/kernels.py:139-179) on the fp32 accumulator:
// per (token, head) of q and k: divide by max(|x|, rho * eps) (the norm before RoPE; RoPE keeps it),
// rotate interleaved pairs (2i, 2i+1) by the token's angle (i < rope_half), scale by s_qk * qk_mult;
// v is divided by rho.  Written bf16 into the packed [M, 3, H, Dh] rows that the attention kernel reads.
// Needs Dh = 64 and d a multiple of 256 (a 256-column tile is 4 whole heads of one of q, k, v).
struct QkvEpi {
  const float* rho;          // [M]
  const float* cos_tab;      // [T, rope_half]
  const float* sin_tab;
  const float* qk_scale;     // [H, Dh]
  float qk_mult, eps;
  int M, T, d, rope_half;
  __device__ __forceinline__ void tile(int m0, int m, int tn, uint32_t tacc, OutStage& out) const {
    const int col0 = tn * BN;
    const int part = col0 / d;            // 0: q, 1: k, 2: v (a 256-column tile lies inside one)
    const bool live = m < M;
    const float rho_m = live ? __ldg(rho + m) : 1.f;
    if (part == 2) {
      const float inv = __fdividef(1.0f, rho_m);
#pragma unroll 1
      for (int hh = 0; hh < BN / 64; ++hh) {
        float x[64];
        load_acc32(tacc + 64 * hh, x);
        load_acc32(tacc + 64 * hh + 32, x + 32);
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] *= inv;
        uint4 o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = pack8(x + 8 * j);
        out.put(col0 + 64 * hh, m0, o);
      }
      return;
    }
    // this token's rotary row, once for the tile's four heads (pairs >= rope_half: cos 1, sin 0)
    float cs[32], sn[32];
    {
      const int t = live ? m % T : 0;
      const float* crow = cos_tab + (int64_t)t * rope_half;
      const float* srow = sin_tab + (int64_t)t * rope_half;
      if (rope_half == 32) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 c4 = __ldg(reinterpret_cast<const float4*>(crow + i));
          const float4 s4 = __ldg(reinterpret_cast<const float4*>(srow + i));
          cs[i] = c4.x; cs[i + 1] = c4.y; cs[i + 2] = c4.z; cs[i + 3] = c4.w;
          sn[i] = s4.x; sn[i + 1] = s4.y; sn[i + 2] = s4.z; sn[i + 3] = s4.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          cs[i] = i < rope_half ? __ldg(crow + i) : 1.f;
          sn[i] = i < rope_half ? __ldg(srow + i) : 0.f;
        }
      }
    }
#pragma unroll 1
    for (int hh = 0; hh < BN / 64; ++hh) {
      float x[64];
      load_acc32(tacc + 64 * hh, x);
      load_acc32(tacc + 64 * hh + 32, x + 32);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) ss = fmaf(x[i], x[i], ss);
      float inv_den = rsqrtf(ss);
      if (eps > 0.f) inv_den = fminf(inv_den, __fdividef(1.0f, rho_m * eps));
      const float f = inv_den * qk_mult;
      const float* sc = qk_scale + (col0 + 64 * hh - part * d);   // s_qk[h, 0..63]
      uint4 o[8];
#pragma unroll
      for (int i = 0; i < 64; i += 8) {
        const float4 s0 = __ldg(reinterpret_cast<const float4*>(sc + i));
        const float4 s1 = __ldg(reinterpret_cast<const float4*>(sc + i + 4));
        const float scl[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
          const int pi = (i + k) >> 1;
          const float xe = x[i + k], xo = x[i + k + 1];
          v[k] = ((xe * cs[pi] - xo * sn[pi]) * f) * scl[k];
          v[k + 1] = ((xe * sn[pi] + xo * cs[pi]) * f) * scl[k + 1];
        }
        o[i / 8] = pack8(v);
      }
      out.put(col0 + 64 * hh, m0, o);
    }
  }
};

// Up/gate projection + SwiGLU (engpt/kernels.py:182-206): accumulator columns 0-127 are u and 128-255 the
// gate for hidden columns 128 tn .. 128 tn + 127:  hidden = (u * s_u * u_mult) * silu(gate * s_gate * gate_mult).
struct SwiGluEpi {
  const float* s_u;
  const float* s_gate;
  float u_mult, gate_mult;
  __device__ __forceinline__ void tile(int m0, int m, int tn, uint32_t tacc, OutStage& out) const {
#pragma unroll 1
    for (int oc = 0; oc < 2; ++oc) {
      const int c0 = tn * 128 + 64 * oc;
      uint4 o[8];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float u[32], g[32];
        load_acc32(tacc + 64 * oc + 32 * half, u);
        load_acc32(tacc + 128 + 64 * oc + 32 * half, g);
        const int cb = c0 + 32 * half;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          const float4 su0 = __ldg(reinterpret_cast<const float4*>(s_u + cb + i));
          const float4 su1 = __ldg(reinterpret_cast<const float4*>(s_u + cb + i + 4));
          const float4 sg0 = __ldg(reinterpret_cast<const float4*>(s_gate + cb + i));
          const float4 sg1 = __ldg(reinterpret_cast<const float4*>(s_gate + cb + i + 4));
          const float su[8] = {su0.x, su0.y, su0.z, su0.w, su1.x, su1.y, su1.z, su1.w};
          const float sg[8] = {sg0.x, sg0.y, sg0.z, sg0.w, sg1.x, sg1.y, sg1.z, sg1.w};
          float v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float uu = (u[i + k] * su[k]) * u_mult;
            const float gg = (g[i + k] * sg[k]) * gate_mult;
            v[k] = uu * __fdividef(gg, 1.0f + __expf(-gg));
          }
          o[4 * half + i / 8] = pack8(v);
        }
      }
      out.put(c0, m0, o);
    }
  }
};

template <typename Epi>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const Shape sh, const Epi epi) {
  using L = Layout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sbase + L::BAR + 8 * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC + 8);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kb_n = (sh.K + BK - 1) / BK;
  const int my_tiles = blockIdx.x < sh.tiles ? (sh.tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_FULL + s), 1);
      mbar_init(bar(B_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(B_ACC_FULL + b), 1);
      mbar_init(bar(B_ACC_EMPTY + b), 128);
    }
    mbar_init(bar(B_FINAL), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int it = 0;
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int t = blockIdx.x + i * gridDim.x;
        const int m0 = (t / sh.tiles_n) * BM;
        const int tn = t % sh.tiles_n;
        const int nb0 = sh.b0 + tn * sh.b_step;
        const int nb1 = sh.b1 + tn * sh.b_step;
        for (int kb = 0; kb < kb_n; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages) {
            ok = mbar_wait(bar(B_EMPTY + s), ((it / kStages) - 1) & 1, abort_flag, 50);
            if (!ok) break;
          }
          mbar_expect_tx(bar(B_FULL + s), kABytes + kBBytes);
          tma_load_2d(sbase + L::A + s * kABytes, &tmA, kb * BK, m0, bar(B_FULL + s));
          tma_load_2d(sbase + L::B + s * kBBytes, &tmB, kb * BK, nb0, bar(B_FULL + s));
          tma_load_2d(sbase + L::B + s * kBBytes + kBBytes / 2, &tmB, kb * BK, nb1, bar(B_FULL + s));
        }
      }
      if (!ok || *abort_flag) {
        // drain the copies still in flight before the CTA exits
        volatile int never = 0;
        for (int j = (it - kStages > 0 ? it - kStages : 0); j < it; ++j)
          mbar_wait(bar(B_FULL + j % kStages), (j / kStages) & 1, &never, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN, false, false);
    const uint64_t da0 = sw128_desc(sbase + L::A, 16, 1024);
    const uint64_t db0 = sw128_desc(sbase + L::B, 16, 1024);
    int it = 0;
    bool ok = true;
    for (int i = 0; ok && i < my_tiles; ++i) {
      const int ab = i & 1;
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ACC_EMPTY + ab), ((i >> 1) - 1) & 1, abort_flag, 51));
        if (!ok) break;
      }
      tc_fence_after();
      const uint32_t td = tmem + BN * ab;
      for (int kb = 0; kb < kb_n; ++kb, ++it) {
        const int s = it % kStages;
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_FULL + s), (it / kStages) & 1, abort_flag, 52));
        if (!ok) break;
        tc_fence_after();
        const uint64_t da = desc_add(da0, s * kABytes);
        const uint64_t db = desc_add(db0, s * kBBytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_f16_ss_w(td, desc_add(da, kk * 32), desc_add(db, kk * 32), kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit_w(bar(B_EMPTY + s));
      }
      if (!ok) break;
      umma_commit_w(bar(B_ACC_FULL + ab));
    }
    umma_commit_w(bar(B_FINAL));
    volatile int never = 0;
    mbar_wait(bar(B_FINAL), 0, &never, 53);
  } else {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;                    // TMEM lane quarter of this warp
    const int r = wq * 32 + lane;               // row within the tile
    const uint32_t t_lane = (uint32_t)(wq * 32) << 16;
    OutStage out{smem + L::OUT, sbase + L::OUT, &tmC, r, threadIdx.x == 64, 0};
    if (out.leader) tma_prefetch_desc(&tmC);
    for (int i = 0; i < my_tiles; ++i) {
      const int ab = i & 1;
      const int t = blockIdx.x + i * gridDim.x;
      const int m0 = (t / sh.tiles_n) * BM;
      const int tn = t % sh.tiles_n;
      const bool ok = mbar_wait(bar(B_ACC_FULL + ab), (i >> 1) & 1, abort_flag, 54);
      if (bar_red_or(1, 128, !ok)) break;     // the four epilogue warps leave together
      tc_fence_after();
      epi.tile(m0, m0 + r, tn, tmem + BN * ab + t_lane, out);
      tc_fence_before();
      mbar_arrive(bar(B_ACC_EMPTY + ab));
    }
    if (out.leader) bulk_wait_group<0>();      // stores done before shared memory goes away
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// --------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encode() {
  if (g_encode) return ENGPT_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return set_error(ENGPT_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return ENGPT_OK;
}

// 2-D view [rows, K] of a bf16 matrix with row stride ld (elements); box 64 (K) x box_rows.
static int make_map(CUtensorMap* m, const void* base, int rows, int K, int64_t ld, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ENGPT_ERR_ALIGN, "gemm: tensor map encode failed (%d)", (int)r);
  return ENGPT_OK;
}

// M x (tiles_n tiles) output; B has b_rows rows, read per tile as two 128-row boxes (see Shape).
template <typename Epi>
static int launch(const void* a, int64_t lda, const void* b, int64_t ldb, int b_rows, int M, int tiles_n, int K,
                  int b0, int b1, int b_step, void* c, int64_t ldc, int c_cols, const Epi& epi, cudaStream_t st) {
  int rc = get_encode();
  if (rc) return rc;
  ENGPT_REQUIRE(aligned(a, 16) && aligned(b, 16) && (lda * 2) % 16 == 0 && (ldb * 2) % 16 == 0 && K % 8 == 0,
                ENGPT_ERR_ALIGN, "gemm: operands need 16-byte aligned rows (K multiple of 8)");
  CUtensorMap ma, mb;
  if ((rc = make_map(&ma, a, M, K, lda, BM))) return rc;
  if ((rc = make_map(&mb, b, b_rows, K, ldb, BN / 2))) return rc;
  ENGPT_REQUIRE(aligned(c, 16) && (ldc * 2) % 16 == 0, ENGPT_ERR_ALIGN, "gemm: output needs 16-byte aligned rows");
  CUtensorMap mc;
  if ((rc = make_map(&mc, c, M, c_cols, ldc, BM))) return rc;   // output boxes: 64 columns x 128 rows
  Shape sh;
  sh.M = M;
  sh.N = tiles_n * BN;
  sh.K = K;
  sh.tiles_n = tiles_n;
  sh.b0 = b0;
  sh.b1 = b1;
  sh.b_step = b_step;
  const int64_t tiles = (int64_t)((M + BM - 1) / BM) * sh.tiles_n;
  ENGPT_REQUIRE(tiles <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "gemm: too many tiles");
  sh.tiles = (int)tiles;
  const int grid = (int)std::min<int64_t>(tiles, num_sms());
  auto kern = gemm_kernel<Epi>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout::kDynSmem);
  if (e != cudaSuccess) return set_error(ENGPT_ERR_LAUNCH, "gemm: smem attribute: %s", cudaGetErrorString(e));
  kern<<<grid, kThreads, Layout::kDynSmem, st>>>(ma, mb, mc, sh, epi);
  return check_launch("gemm (tcgen05)");
}

}  // namespace gemm
}  // namespace engpt

using namespace engpt;

extern "C" int engpt_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc, int M,
                               int N, int K, void* stream) {
  clear_error();
  ENGPT_REQUIRE(M >= 0 && N >= 0 && K > 0, ENGPT_ERR_SHAPE, "gemm: M=%d N=%d K=%d", M, N, K);
  if ((int64_t)M * N == 0) return ENGPT_OK;
  ENGPT_REQUIRE(a && b && c, ENGPT_ERR_ARG, "gemm: null pointer");
  ENGPT_REQUIRE(lda >= K && ldb >= K && ldc >= N, ENGPT_ERR_SHAPE, "gemm: leading dimensions");
  gemm::StoreBf16 epi;
  return gemm::launch(a, lda, b, ldb, N, M, (N + gemm::BN - 1) / gemm::BN, K, 0, gemm::BN / 2, gemm::BN, c, ldc, N,
                      epi, as_stream(stream));
}

extern "C" int engpt_qkv_projection(const void* x, const void* w_qkv, const float* rho, const float* cos_tab,
                                    const float* sin_tab, int rope_half, const float* qk_scale, float qk_mult,
                                    float norm_eps, int B, int T, int H, int Dh, void* qkv_out, void* stream) {
  clear_error();
  ENGPT_REQUIRE(B >= 0 && T > 0 && H > 0 && Dh == 64, ENGPT_ERR_UNSUPPORTED,
                "qkv_projection: head_dim %d (the fused tile needs 64)", Dh);
  const int d = H * Dh;
  ENGPT_REQUIRE(d % gemm::BN == 0, ENGPT_ERR_UNSUPPORTED, "qkv_projection: d=%d not a multiple of 256", d);
  ENGPT_REQUIRE(rope_half >= 0 && 2 * rope_half <= Dh, ENGPT_ERR_SHAPE, "qkv_projection: rope_half=%d", rope_half);
  const int64_t M = (int64_t)B * T;
  if (M == 0) return ENGPT_OK;
  ENGPT_REQUIRE(M <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "qkv_projection: too many tokens");
  ENGPT_REQUIRE(x && w_qkv && rho && qk_scale && qkv_out && (rope_half == 0 || (cos_tab && sin_tab)), ENGPT_ERR_ARG,
                "qkv_projection: null pointer");
  ENGPT_REQUIRE(aligned(qkv_out, 16), ENGPT_ERR_ALIGN, "qkv_projection: output not 16-byte aligned");
  gemm::QkvEpi epi{rho, cos_tab, sin_tab, qk_scale, qk_mult, norm_eps, (int)M, T, d, rope_half};
  return gemm::launch(x, d, w_qkv, d, 3 * d, (int)M, 3 * d / gemm::BN, d, 0, gemm::BN / 2, gemm::BN, qkv_out, 3 * d,
                      3 * d, epi, as_stream(stream));
}

extern "C" int engpt_up_gate_swiglu(const void* x, const void* w_ug, const float* s_u, const float* s_gate,
                                    float u_mult, float gate_mult, int64_t rows, int d, int width, void* hidden,
                                    void* stream) {
  clear_error();
  ENGPT_REQUIRE(rows >= 0 && d > 0 && width > 0, ENGPT_ERR_SHAPE, "up_gate_swiglu: rows=%lld d=%d width=%d",
                (long long)rows, d, width);
  ENGPT_REQUIRE(width % 128 == 0 && d % 8 == 0, ENGPT_ERR_UNSUPPORTED,
                "up_gate_swiglu: width %d not a multiple of 128 or d %d not a multiple of 8", width, d);
  if (rows == 0) return ENGPT_OK;
  ENGPT_REQUIRE(rows <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "up_gate_swiglu: too many rows");
  ENGPT_REQUIRE(x && w_ug && s_u && s_gate && hidden, ENGPT_ERR_ARG, "up_gate_swiglu: null pointer");
  ENGPT_REQUIRE(aligned(hidden, 16), ENGPT_ERR_ALIGN, "up_gate_swiglu: output not 16-byte aligned");
  gemm::SwiGluEpi epi{s_u, s_gate, u_mult, gate_mult};
  return gemm::launch(x, d, w_ug, d, 2 * width, (int)rows, width / 128, d, 0, width, 128, hidden, width, width, epi,
                      as_stream(stream));
}
