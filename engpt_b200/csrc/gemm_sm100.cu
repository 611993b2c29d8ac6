// Persistent tcgen05 GEMM for B200 (sm_100a) with a fused epilogue:
//   C[M, N] = A[M, K] * B[N, K]^T   (bf16 operands, K contiguous; fp32 accumulation in TMEM)
//
// The dense projections of the enGPT block (engpt/models.py:140-182) are this
// shape with A = the activations and B = an nn.Linear weight.  A CTA owns one
// SM and walks 128 x 256 output tiles (tile t = blockIdx.x + i * gridDim.x,
// in groups of 64 row blocks with the tile columns outer inside a group, so
// the A row blocks of a group stay in L2 while B streams past them once).
// Warp roles (192 threads):
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

#include "carried_residual.cuh"
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
  int row_blocks;       // ceil(M / BM)
  int group;            // row blocks per raster group (tile order below)
  // Tile t -> (row block, tile column): groups of `group` row blocks, tile columns outer inside a group, so
  // the tiles in flight at once share a few row blocks of A and a narrow band of B columns (a large B, such
  // as the 50k-row output head, then stays in L2 while the group's row blocks reuse it).
  __device__ __forceinline__ void coords(int t, int& m0, int& tn) const {
    const int per_group = group * tiles_n;
    const int g = t / per_group;
    const int rem = t - g * per_group;
    const int rb0 = g * group;
    const int gs = min(group, row_blocks - rb0);
    tn = rem / gs;
    m0 = (rb0 + rem - tn * gs) * BM;
  }
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
  int M, T, d, rope_half, dh;   // dh: head_dim, 64 or 128
  // q or k heads of head_dim 128 (two per 256-column tile): the norm over the head's 128 accumulator columns,
  // then two 64-column halves rotated (pairs 32 half ..), scaled and stored
  __device__ __forceinline__ void tile128(int m0, int m, int col0, int part, uint32_t tacc, float rho_m,
                                          OutStage& out) const {
    const int t = m < M ? m % T : 0;
#pragma unroll 1
    for (int hh = 0; hh < BN / 128; ++hh) {
      const uint32_t th = tacc + 128 * hh;
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32];
        load_acc32(th + 32 * c, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) ss = fmaf(x[i], x[i], ss);
      }
      float inv_den = rsqrtf(ss);
      if (eps > 0.f) inv_den = fminf(inv_den, __fdividef(1.0f, rho_m * eps));
      const float f = inv_den * qk_mult;
      const float* sc = qk_scale + (col0 + 128 * hh - part * d);   // s_qk[h, 0..127]
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        float x[64];
        load_acc32(th + 64 * half, x);
        load_acc32(th + 64 * half + 32, x + 32);
        const int p0 = 32 * half;                                   // first rotary pair of this half
        // this half's 32 rotary pairs: vector loads issued together (pairs >= rope_half: cos 1, sin 0)
        float cs[32], sn[32];
        {
          const float* crow = cos_tab + (int64_t)t * rope_half + p0;
          const float* srow = sin_tab + (int64_t)t * rope_half + p0;
          if (rope_half == 64) {
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
              cs[i] = p0 + i < rope_half ? __ldg(crow + i) : 1.f;
              sn[i] = p0 + i < rope_half ? __ldg(srow + i) : 0.f;
            }
          }
        }
        uint4 o[8];
#pragma unroll
        for (int i = 0; i < 64; i += 8) {
          const float4 s0 = __ldg(reinterpret_cast<const float4*>(sc + 64 * half + i));
          const float4 s1 = __ldg(reinterpret_cast<const float4*>(sc + 64 * half + i + 4));
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
        out.put(col0 + 128 * hh + 64 * half, m0, o);
      }
    }
  }
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
    if (dh == 128) {
      tile128(m0, m, col0, part, tacc, rho_m, out);
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

// Output head + the log-sum-exp half of F.cross_entropy (engpt/models.py:328-333): the bf16 logits tile is
// stored as by StoreBf16, and from the same bf16-rounded values (what the loss reads under autocast) each row's
// base-2 log-sum-exp over the tile's valid columns (< vocab) is written as a (max, sum) pair to
// part[tn * rows + m].  The pairs of a row merge into its full log-sum-exp in ce_combine_kernel.
struct LseEpi {
  float2* part;
  int rows;
  int vocab;
  __device__ __forceinline__ void tile(int m0, int m, int tn, uint32_t tacc, OutStage& out) const {
    constexpr float kL2e = 1.4426950408889634f;
    const int nvalid = vocab - tn * BN;          // valid columns of this tile (>= 1)
    float mx = -INFINITY, sm = 0.f;              // base-2 running max and sum
#pragma unroll 1
    for (int oc = 0; oc < BN / 64; ++oc) {
      float v[64];
      load_acc32(tacc + 64 * oc, v);
      load_acc32(tacc + 64 * oc + 32, v + 32);
      uint4 o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j] = pack8(v + 8 * j);
        unpack8(o[j], v + 8 * j);               // the stored (rounded) logits
      }
      out.put(tn * BN + 64 * oc, m0, o);
      if (nvalid < BN) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (64 * oc + i >= nvalid) v[i] = -INFINITY;
      }
      float cm = v[0];
#pragma unroll
      for (int i = 1; i < 64; ++i) cm = fmaxf(cm, v[i]);
      if (cm == -INFINITY) continue;             // every column of this chunk is past the vocab
      const float cml = cm * kL2e;
      if (cml > mx) {
        sm *= ex2_approx(mx - cml);
        mx = cml;
      }
      const float nm = -mx;
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        s0 += ex2_approx(fmaf(v[i], kL2e, nm));
        s1 += ex2_approx(fmaf(v[i + 1], kL2e, nm));
      }
      sm += s0 + s1;
    }
    if (m < rows) part[(int64_t)tn * rows + m] = make_float2(mx, sm);
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
        int m0, tn;
        sh.coords(t, m0, tn);
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
      int m0, tn;
      sh.coords(t, m0, tn);
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

// ============================================================================ GEMM + carried residual
// branch = A[M, K] * W[d, K]^T (the out_proj / down_proj GEMM) with carried_residual_gauge
// (engpt/kernels.py:277-324) in the epilogue, so the branch never goes to HBM.  The residual needs whole
// rows (R0..R3 over all d columns before any output), so a thread-block cluster of C = d / 256 CTAs owns
// one 128-row block: CTA `rank` accumulates output columns [256 rank, 256 rank + 256) in TMEM, reduces its
// partial R0..R3 per row, and sends them to the other CTAs' shared memory (st.async, completing bytes on
// their mbarrier); every CTA then adds the C partials in rank order (identical sums on every CTA), forms
// the row scalars and writes its columns of Y' (fp32) and of the next GEMM's bf16 operand.
// Eight epilogue warps, two per TMEM lane quarter: warp half h owns accumulator columns 128 h .. 128 h + 127
// of its 32 rows, and holds that row segment of Y in registers (loaded once, with 32-byte loads issued while
// the previous tile is still being written, so the load latency overlaps work).  The branch is rounded to
// bf16 before use, as the reference's autocast GEMM output is.  Rank 0 alone reads rho and writes rho' (its
// rho reaches the other CTAs with its partial sums), so rho may be updated in place.
namespace res {

constexpr int kStagesR = 3;
constexpr int kCmax = 4;                   // d <= 1024
constexpr int kThreadsR = 320;             // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kHalfCols = BN / 2;          // accumulator columns per epilogue warp
constexpr int kYoBytes = BM * 32 * 4;      // Y' staging: 128 rows x 32 fp32 columns (128B swizzle)
constexpr int kAxBytes = BM * 32 * 2;      // operand staging: 128 rows x 32 bf16 columns (64B swizzle)

struct Layout {
  static constexpr int A = 0;
  static constexpr int B = A + kStagesR * kABytes;
  static constexpr int YO = B + kStagesR * kBBytes;            // [2 halves] Y' staging
  static constexpr int AX = YO + 2 * kYoBytes;                 // [2 halves] bf16 operand staging
  static constexpr int RX = AX + 2 * kAxBytes;                 // [2 tiles][kCmax - 1 peers][128 rows] float4
  static constexpr int RHO = RX + 2 * (kCmax - 1) * BM * 16;   // [2 tiles][128 rows] rank 0's rho
  static constexpr int XP = RHO + 2 * BM * 4;                  // [2 halves][128 rows] float4 partial sums
  static constexpr int COL = XP + 2 * BM * 16;                 // per column: alpha, beta, alpha^2, beta^2, alpha beta
  static constexpr int BAR = COL + 5 * BN * 4;
  static constexpr int kBars = 16;
  static constexpr int MISC = BAR + kBars * 8;
  static constexpr int TOTAL = MISC + 16;
  static constexpr int kDynSmem = TOTAL + 1024;
};
static_assert(Layout::kDynSmem <= 227 * 1024, "shared memory");
static_assert(Layout::YO % 1024 == 0 && Layout::AX % 1024 == 0, "swizzle alignment");

enum { R_FULL = 0, R_EMPTY = R_FULL + kStagesR, R_ACC_FULL = R_EMPTY + kStagesR, R_ACC_EMPTY = R_ACC_FULL + 2,
       R_FINAL = R_ACC_EMPTY + 2, R_RXF = R_FINAL + 1, R_END = R_RXF + 2 };
static_assert(R_END <= Layout::kBars, "barrier slots");

struct Params {
  int M, K, C, d, row_blocks;
  const float* y;
  const float* rho;
  float* rho_out;
  const float* alpha;
  float alpha_mult;
  int alpha_abs;
  float branch_eps, residual_eps, max_radius;
  int aux_mode;     // ENGPT_AUX_NONE / _BF16_Y / _BF16_H
};

// fp32 accumulator pair -> the bf16 values a bf16 GEMM output holds, back in fp32
__device__ __forceinline__ void round_bf16_pair(uint32_t a, uint32_t b, float& fa, float& fb) {
  const uint32_t pk = pack_bf16x2(__uint_as_float(a), __uint_as_float(b));
  fa = __uint_as_float(pk << 16);
  fb = __uint_as_float(pk & 0xffff0000u);
}

// 8 consecutive fp32 of row data (32-byte aligned), not kept in L1
__device__ __forceinline__ void ld8(const float* p, float* v) {
  asm volatile("ld.global.L1::no_allocate.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "l"(p));
}

// this thread's 32 Y values of chunk c (zeros past the last row)
__device__ __forceinline__ void load_y32(const float* row, bool live, float* v) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (live) {
      ld8(row + 8 * q, v + 8 * q);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[8 * q + e] = 0.f;
    }
  }
}

__global__ void __launch_bounds__(kThreadsR, 1)
    gemm_residual_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmYO,
                         const __grid_constant__ CUtensorMap tmAX, const Params p) {
  using L = Layout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sbase + L::BAR + 8 * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC + 8);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int C = p.C;
  const int rank = (int)cluster_ctarank();
  const int cluster = blockIdx.x / C;
  const int n_clusters = gridDim.x / C;
  const int kb_n = (p.K + BK - 1) / BK;
  const int my_tiles = cluster < p.row_blocks ? (p.row_blocks - 1 - cluster) / n_clusters + 1 : 0;
  const int col0 = rank * BN;                 // this CTA's 256 output columns
  // bytes the other CTAs send this one per tile: their partial sums, and rank 0's rho
  const uint32_t rx_bytes = (uint32_t)((C - 1) * BM * 16 + (rank != 0 ? BM * 4 : 0));

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesR; ++s) {
      mbar_init(bar(R_FULL + s), 1);
      mbar_init(bar(R_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(R_ACC_FULL + b), 1);
      mbar_init(bar(R_ACC_EMPTY + b), 256);
      mbar_init(bar(R_RXF + b), 1);
    }
    mbar_init(bar(R_FINAL), 1);
    *abort_flag = 0;
    fence_mbar_init();
    // the partial-sum barriers of the first two tiles are armed before any other CTA can send
    if (C > 1) {
      if (my_tiles > 0) mbar_expect_tx(bar(R_RXF + 0), rx_bytes);
      if (my_tiles > 1) mbar_expect_tx(bar(R_RXF + 1), rx_bytes);
    }
  }
  if (warp >= 2) {
    float* col = reinterpret_cast<float*>(smem + L::COL);
    for (int j = threadIdx.x - 64; j < BN; j += 256) {
      float a = p.alpha[col0 + j];
      if (p.alpha_abs) a = fabsf(a);
      a *= p.alpha_mult;
      const float be = 1.0f - a;
      col[j] = a;
      col[BN + j] = be;
      col[2 * BN + j] = a * a;
      col[3 * BN + j] = be * be;
      col[4 * BN + j] = a * be;
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync_all();      // every CTA's barriers exist (and are armed) before the first st.async
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
        const int m0 = (cluster + i * n_clusters) * BM;
        if (i + 1 < my_tiles) {   // Y rows of the next tile into L2 for the epilogue's loads
          const int m1 = m0 + n_clusters * BM;
          for (int c = 0; c < BN / 32; ++c) tma_prefetch_l2_2d(&tmY, col0 + 32 * c, m1);
        }
        for (int kb = 0; kb < kb_n; ++kb, ++it) {
          const int s = it % kStagesR;
          if (it >= kStagesR) {
            ok = mbar_wait(bar(R_EMPTY + s), ((it / kStagesR) - 1) & 1, abort_flag, 60);
            if (!ok) break;
          }
          mbar_expect_tx(bar(R_FULL + s), kABytes + kBBytes);
          tma_load_2d(sbase + L::A + s * kABytes, &tmA, kb * BK, m0, bar(R_FULL + s));
          tma_load_2d(sbase + L::B + s * kBBytes, &tmB, kb * BK, col0, bar(R_FULL + s));
          tma_load_2d(sbase + L::B + s * kBBytes + kBBytes / 2, &tmB, kb * BK, col0 + BN / 2, bar(R_FULL + s));
        }
      }
      if (!ok || *abort_flag) {
        volatile int never = 0;
        for (int j = (it - kStagesR > 0 ? it - kStagesR : 0); j < it; ++j)
          mbar_wait(bar(R_FULL + j % kStagesR), (j / kStagesR) & 1, &never, 0);
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
        ok = __all_sync(0xffffffffu, mbar_wait(bar(R_ACC_EMPTY + ab), ((i >> 1) - 1) & 1, abort_flag, 61));
        if (!ok) break;
      }
      tc_fence_after();
      const uint32_t td = tmem + BN * ab;
      for (int kb = 0; kb < kb_n; ++kb, ++it) {
        const int s = it % kStagesR;
        ok = __all_sync(0xffffffffu, mbar_wait(bar(R_FULL + s), (it / kStagesR) & 1, abort_flag, 62));
        if (!ok) break;
        tc_fence_after();
        const uint64_t da = desc_add(da0, s * kABytes);
        const uint64_t db = desc_add(db0, s * kBBytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_f16_ss_w(td, desc_add(da, kk * 32), desc_add(db, kk * 32), kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit_w(bar(R_EMPTY + s));
      }
      if (!ok) break;
      umma_commit_w(bar(R_ACC_FULL + ab));
    }
    umma_commit_w(bar(R_FINAL));
    volatile int never = 0;
    mbar_wait(bar(R_FINAL), 0, &never, 63);
  } else {
    // ------------------------------------------------------------ epilogue: thread = row, half = 128 columns
    const int wq = warp & 3;                     // TMEM lane quarter
    const int hf = (warp - 2) >> 2;              // column half
    const int r = wq * 32 + lane;
    const uint32_t t_lane = (uint32_t)(wq * 32) << 16;
    const int et = threadIdx.x - 64;             // 0..255
    const bool leader = et == 0;                 // re-arms the partial-sum barriers
    const bool hleader = (et & 127) == 0;        // issues this half's stores
    const int bar_half = 2 + hf;                 // named barrier of this half's 128 threads
    const float* col = reinterpret_cast<const float*>(smem + L::COL) + kHalfCols * hf;
    const bool aux = p.aux_mode != ENGPT_AUX_NONE;
    const int ccol = col0 + kHalfCols * hf;      // this half's first output column
    if (hleader) {
      tma_prefetch_desc(&tmYO);
      if (aux) tma_prefetch_desc(&tmAX);
    }
    uint8_t* yo_st = smem + L::YO + hf * kYoBytes;
    uint8_t* ax_st = smem + L::AX + hf * kAxBytes;
    const uint32_t yo_s = sbase + L::YO + hf * kYoBytes;
    const uint32_t ax_s = sbase + L::AX + hf * kAxBytes;
    constexpr int kChunks = kHalfCols / 32;
    bool ok = true;
    for (int i = 0; ok && i < my_tiles; ++i) {
      const int ab = i & 1;
      const int m0 = (cluster + i * n_clusters) * BM;
      const int m = m0 + r;
      const bool live = m < p.M;
      const float* yrow = p.y + (int64_t)m * p.d + ccol;
      // Y is read twice per tile (32-byte loads, one 32-column chunk ahead of its use): pass 1 from the
      // L2 copy the producer prefetched, pass 2 from L2 again
      float yv[2][32];
      load_y32(yrow, live, yv[0]);
      ok = mbar_wait(bar(R_ACC_FULL + ab), (i >> 1) & 1, abort_flag, 64);
      if (bar_red_or(1, 256, !ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem + BN * ab + kHalfCols * hf + t_lane;
      float rho_m = 1.f;
      if (rank == 0 && live) rho_m = p.rho[m];

      // pass 1: this half's part of R0..R3 (the products of the standalone residual kernel)
      float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        load_y32(yrow + 32 * ((c + 1) % kChunks), live, yv[(c + 1) & 1]);   // the last one is pass 2's first
        const float* y32 = yv[c & 1];
#pragma unroll
        for (int h16 = 0; h16 < 2; ++h16) {
          uint32_t acc[16];
          tmem_ld16(tacc + 32 * c + 16 * h16, acc);
          tmem_wait_ld16(acc);
#pragma unroll
          for (int k = 0; k < 16; k += 4) {
            const int j = 32 * c + 16 * h16 + k;
            const float4 aa = *reinterpret_cast<const float4*>(col + 2 * BN + j);
            const float4 bb = *reinterpret_cast<const float4*>(col + 3 * BN + j);
            const float4 ab4 = *reinterpret_cast<const float4*>(col + 4 * BN + j);
            const float caa[4] = {aa.x, aa.y, aa.z, aa.w}, cbb[4] = {bb.x, bb.y, bb.z, bb.w};
            const float cab[4] = {ab4.x, ab4.y, ab4.z, ab4.w};
            float b4[4];
            round_bf16_pair(acc[k], acc[k + 1], b4[0], b4[1]);
            round_bf16_pair(acc[k + 2], acc[k + 3], b4[2], b4[3]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float y = y32[16 * h16 + k + e], b = b4[e];
              const float bsq = b * b;
              r0 += bsq;
              r1 += cbb[e] * (y * y);
              r2 += caa[e] * bsq;
              r3 += (cab[e] * y) * b;
            }
          }
        }
      }
      // the CTA's partial sums: half 0 + half 1
      float4* xp = reinterpret_cast<float4*>(smem + L::XP);
      xp[hf * BM + r] = make_float4(r0, r1, r2, r3);
      bar_sync_named(1, 256);
      {
        const float4 h0 = xp[r], h1 = xp[BM + r];
        r0 = h0.x + h1.x;
        r1 = h0.y + h1.y;
        r2 = h0.z + h1.z;
        r3 = h0.w + h1.w;
      }
      // exchange within the cluster (half 0 sends; every thread receives)
      const int buf = i & 1;
      if (C > 1) {
        const uint32_t rbar_local = bar(R_RXF + buf);
        if (hf == 0) {
          for (int q = 0; q < C; ++q) {
            if (q == rank) continue;
            const int idx = rank < q ? rank : rank - 1;            // this CTA's slot at CTA q
            const uint32_t off = L::RX + ((buf * (kCmax - 1) + idx) * BM + r) * 16;
            const uint32_t rbar = mapa_shared(rbar_local, (uint32_t)q);
            st_async_v4(mapa_shared(sbase + off, (uint32_t)q), r0, r1, r2, r3, rbar);
            if (rank == 0) st_async_b32(mapa_shared(sbase + L::RHO + (buf * BM + r) * 4, (uint32_t)q), rho_m, rbar);
          }
        }
        ok = mbar_wait_cluster(rbar_local, (i >> 1) & 1, abort_flag, 66);
        if (bar_red_or(1, 256, !ok)) {
          ok = false;
          break;
        }
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int q = 0; q < C; ++q) {                          // rank order: the same sums on every CTA
          float4 v;
          if (q == rank) {
            v = make_float4(r0, r1, r2, r3);
          } else {
            const int idx = q < rank ? q : q - 1;
            v = *reinterpret_cast<const float4*>(smem + L::RX + ((buf * (kCmax - 1) + idx) * BM + r) * 16);
          }
          s0 += v.x;
          s1 += v.y;
          s2 += v.z;
          s3 += v.w;
        }
        r0 = s0;
        r1 = s1;
        r2 = s2;
        r3 = s3;
        if (rank != 0) rho_m = *reinterpret_cast<const float*>(smem + L::RHO + (buf * BM + r) * 4);
        bar_sync_named(1, 256);                                // every thread has read RX[buf] and XP
        if (leader && i + 2 < my_tiles) mbar_expect_tx(bar(R_RXF + buf), rx_bytes);
      } else {
        bar_sync_named(1, 256);                                // XP is read before the next tile writes it
      }
      const RowScalars rs = residual_row_scalars(p.branch_eps, p.residual_eps, p.max_radius, rho_m, r0, r1, r2, r3);
      const float cy = rs.coef_y * rs.inv_g, cb = rs.coef_b * rs.inv_g;

      // pass 2: Y' = (beta c_b y + alpha rho b) / g and the bf16 operand, staged and stored by TMA
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        if (c + 1 < kChunks) load_y32(yrow + 32 * (c + 1), live, yv[(c + 1) & 1]);
        const float* y32 = yv[c & 1];
        if (hleader) bulk_wait_group_read<0>();                // this half's staging buffers are free again
        bar_sync_named(bar_half, 128);
        uint8_t* yrow_st = yo_st + r * 128;
        uint8_t* arow_st = ax_st + r * 64;
        uint32_t acc[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {          // 8 columns at a time
          if ((q & 1) == 0) {
            tmem_ld16(tacc + 32 * c + 8 * q, acc);
            tmem_wait_ld16(acc);
          }
          float o[8];
#pragma unroll
          for (int k = 0; k < 8; k += 4) {
            const int j = 32 * c + 8 * q + k;
            const float4 al = *reinterpret_cast<const float4*>(col + j);
            const float4 be = *reinterpret_cast<const float4*>(col + BN + j);
            const float cal[4] = {al.x, al.y, al.z, al.w}, cbe[4] = {be.x, be.y, be.z, be.w};
            float b4[4];
            round_bf16_pair(acc[8 * (q & 1) + k], acc[8 * (q & 1) + k + 1], b4[0], b4[1]);
            round_bf16_pair(acc[8 * (q & 1) + k + 2], acc[8 * (q & 1) + k + 3], b4[2], b4[3]);
#pragma unroll
            for (int e = 0; e < 4; ++e) o[k + e] = fmaf(cbe[e] * cy, y32[8 * q + k + e], (cal[e] * cb) * b4[e]);
          }
          *reinterpret_cast<float4*>(yrow_st + (((2 * q) ^ (r & 7)) << 4)) = make_float4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<float4*>(yrow_st + (((2 * q + 1) ^ (r & 7)) << 4)) = make_float4(o[4], o[5], o[6], o[7]);
          if (aux) {
            if (p.aux_mode == ENGPT_AUX_BF16_H) {
#pragma unroll
              for (int k = 0; k < 8; ++k) o[k] *= rs.inv_rho;
            }
            *reinterpret_cast<uint4*>(arow_st + ((q ^ ((r >> 1) & 3)) << 4)) = pack8(o);
          }
        }
        fence_proxy_async_smem();
        bar_sync_named(bar_half, 128);
        if (hleader) {
          tma_store_2d(&tmYO, ccol + 32 * c, m0, yo_s);
          if (aux) tma_store_2d(&tmAX, ccol + 32 * c, m0, ax_s);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      mbar_arrive(bar(R_ACC_EMPTY + ab));
      if (rank == 0 && hf == 0 && live) p.rho_out[m] = rs.rho_new;
    }
    if (hleader) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  cluster_sync_all();      // no CTA leaves while another may still write into its shared memory
}

}  // namespace res

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
  sh.row_blocks = (M + BM - 1) / BM;
  sh.group = 64;   // measured on the 50k-column output head: 8 -> 5.5 ms, 32 -> 5.2, 64 -> 5.1
  const int64_t tiles = (int64_t)sh.row_blocks * sh.tiles_n;
  ENGPT_REQUIRE(tiles <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "gemm: too many tiles");
  sh.tiles = (int)tiles;
  const int grid = (int)std::min<int64_t>(tiles, num_sms());
  auto kern = gemm_kernel<Epi>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout::kDynSmem);
  if (e != cudaSuccess) return set_error(ENGPT_ERR_LAUNCH, "gemm: smem attribute: %s", cudaGetErrorString(e));
  kern<<<grid, kThreads, Layout::kDynSmem, st>>>(ma, mb, mc, sh, epi);
  return check_launch("gemm (tcgen05)");
}


// 2-D view [rows, cols] of an fp32 matrix with row stride ld (elements); box 32 columns x 128 rows.
static int make_map_f32(CUtensorMap* m, const void* base, int rows, int cols, int64_t ld) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ENGPT_ERR_ALIGN, "gemm_residual: tensor map encode failed (%d)", (int)r);
  return ENGPT_OK;
}

// 2-D view [rows, cols] of a bf16 matrix with row stride ld (elements); box 32 columns x 128 rows, 64B swizzle.
static int make_map_bf16_32(CUtensorMap* m, const void* base, int rows, int cols, int64_t ld) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {32, (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ENGPT_ERR_ALIGN, "gemm_residual: tensor map encode failed (%d)", (int)r);
  return ENGPT_OK;
}

// Clusters of C CTAs that can be resident at once on this device (cached per device and C).
static int max_active_clusters(int C) {
  static int cache[64][res::kCmax + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (cache[dev][C] > 0) return cache[dev][C];
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((num_sms() / C) * C);
  cfg.blockDim = dim3(res::kThreadsR);
  cfg.dynamicSmemBytes = res::Layout::kDynSmem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, res::gemm_residual_kernel, &cfg);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    set_error(ENGPT_ERR_LAUNCH, "gemm_carried_residual: cluster occupancy query: %s", cudaGetErrorString(e));
    return 0;
  }
  if (n <= 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, res::gemm_residual_kernel) == cudaSuccess)
      set_error(ENGPT_ERR_LAUNCH, "gemm_carried_residual: no cluster of %d CTAs fits (regs %d, max threads %d)", C,
                fa.numRegs, fa.maxThreadsPerBlock);
    return 0;
  }
  cache[dev][C] = n;
  return n;
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

extern "C" int engpt_qkv_projection(const void* x, int in_features, const void* w_qkv, const float* rho,
                                    const float* cos_tab, const float* sin_tab, int rope_half, const float* qk_scale,
                                    float qk_mult, float norm_eps, int B, int T, int H, int Dh, void* qkv_out,
                                    void* stream) {
  clear_error();
  ENGPT_REQUIRE(B >= 0 && T > 0 && H > 0 && (Dh == 64 || Dh == 128), ENGPT_ERR_UNSUPPORTED,
                "qkv_projection: head_dim %d (the fused tile needs 64 or 128)", Dh);
  const int d = H * Dh;
  ENGPT_REQUIRE(d % gemm::BN == 0, ENGPT_ERR_UNSUPPORTED, "qkv_projection: d=%d not a multiple of 256", d);
  ENGPT_REQUIRE(in_features > 0 && in_features % 8 == 0, ENGPT_ERR_SHAPE, "qkv_projection: in_features=%d",
                in_features);
  ENGPT_REQUIRE(rope_half >= 0 && 2 * rope_half <= Dh, ENGPT_ERR_SHAPE, "qkv_projection: rope_half=%d", rope_half);
  const int64_t M = (int64_t)B * T;
  if (M == 0) return ENGPT_OK;
  ENGPT_REQUIRE(M <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "qkv_projection: too many tokens");
  ENGPT_REQUIRE(x && w_qkv && rho && qk_scale && qkv_out && (rope_half == 0 || (cos_tab && sin_tab)), ENGPT_ERR_ARG,
                "qkv_projection: null pointer");
  ENGPT_REQUIRE(aligned(qkv_out, 16), ENGPT_ERR_ALIGN, "qkv_projection: output not 16-byte aligned");
  gemm::QkvEpi epi{rho, cos_tab, sin_tab, qk_scale, qk_mult, norm_eps, (int)M, T, d, rope_half, Dh};
  return gemm::launch(x, in_features, w_qkv, in_features, 3 * d, (int)M, 3 * d / gemm::BN, in_features, 0,
                      gemm::BN / 2, gemm::BN, qkv_out, 3 * d, 3 * d, epi, as_stream(stream));
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

extern "C" int engpt_gemm_carried_residual(const void* a, int64_t lda, const void* w, int64_t ldw, int K,
                                           const float* y, const float* rho, const float* alpha, float alpha_mult,
                                           int alpha_abs, float branch_eps, float residual_eps, float max_radius,
                                           int64_t rows, int d, float* y_out, float* rho_out, void* aux_out,
                                           int aux_mode, void* stream) {
  using namespace gemm;
  clear_error();
  ENGPT_REQUIRE(rows >= 0 && d > 0 && K > 0, ENGPT_ERR_SHAPE, "gemm_carried_residual: rows=%lld d=%d K=%d",
                (long long)rows, d, K);
  ENGPT_REQUIRE(d % BN == 0 && d / BN <= res::kCmax, ENGPT_ERR_UNSUPPORTED,
                "gemm_carried_residual: d=%d (the fused epilogue needs d = 256, 512, 768 or 1024)", d);
  ENGPT_REQUIRE(aux_mode == ENGPT_AUX_NONE || aux_mode == ENGPT_AUX_BF16_Y || aux_mode == ENGPT_AUX_BF16_H,
                ENGPT_ERR_UNSUPPORTED, "gemm_carried_residual: aux_mode %d", aux_mode);
  if (rows == 0) return ENGPT_OK;
  ENGPT_REQUIRE(rows <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "gemm_carried_residual: too many rows");
  ENGPT_REQUIRE(a && w && y && rho && alpha && y_out && rho_out && (aux_mode == ENGPT_AUX_NONE || aux_out),
                ENGPT_ERR_ARG, "gemm_carried_residual: null pointer");
  ENGPT_REQUIRE(lda >= K && ldw >= K, ENGPT_ERR_SHAPE, "gemm_carried_residual: leading dimensions");
  ENGPT_REQUIRE(aligned(a, 16) && aligned(w, 16) && (lda * 2) % 16 == 0 && (ldw * 2) % 16 == 0 && K % 8 == 0,
                ENGPT_ERR_ALIGN, "gemm_carried_residual: operands need 16-byte aligned rows (K multiple of 8)");
  ENGPT_REQUIRE(aligned(y, 32) && aligned(y_out, 16) && (aux_mode == ENGPT_AUX_NONE || aligned(aux_out, 16)),
                ENGPT_ERR_ALIGN, "gemm_carried_residual: y must be 32-byte aligned, y_out and aux_out 16-byte");
  int rc = get_encode();
  if (rc) return rc;
  const int M = (int)rows;
  const int C = d / BN;
  CUtensorMap ma, mb, my, myo, max_;
  if ((rc = make_map(&ma, a, M, K, lda, BM))) return rc;
  if ((rc = make_map(&mb, w, d, K, ldw, BN / 2))) return rc;
  if ((rc = make_map_f32(&my, y, M, d, d))) return rc;
  if ((rc = make_map_f32(&myo, y_out, M, d, d))) return rc;
  if (aux_mode != ENGPT_AUX_NONE) {
    if ((rc = make_map_bf16_32(&max_, aux_out, M, d, d))) return rc;
  } else {
    max_ = myo;                                                     // never used
  }
  auto kern = res::gemm_residual_kernel;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, res::Layout::kDynSmem);
  if (e != cudaSuccess)
    return set_error(ENGPT_ERR_LAUNCH, "gemm_carried_residual: smem attribute: %s", cudaGetErrorString(e));
  const int clusters = max_active_clusters(C);
  if (clusters <= 0) return ENGPT_ERR_LAUNCH;   // message set by max_active_clusters
  res::Params p;
  p.M = M;
  p.K = K;
  p.C = C;
  p.d = d;
  p.y = y;
  p.row_blocks = (M + BM - 1) / BM;
  p.rho = rho;
  p.rho_out = rho_out;
  p.alpha = alpha;
  p.alpha_mult = alpha_mult;
  p.alpha_abs = alpha_abs;
  p.branch_eps = branch_eps;
  p.residual_eps = residual_eps;
  p.max_radius = max_radius;
  p.aux_mode = aux_mode;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(std::min(p.row_blocks, clusters) * C);
  cfg.blockDim = dim3(res::kThreadsR);
  cfg.dynamicSmemBytes = res::Layout::kDynSmem;
  cfg.stream = as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, ma, mb, my, myo, max_, p);
  if (e != cudaSuccess) return set_error(ENGPT_ERR_LAUNCH, "gemm_carried_residual: launch: %s", cudaGetErrorString(e));
  return check_launch("gemm_carried_residual (tcgen05)");
}

namespace engpt {
namespace gemm {

// Row r: merge the (max, sum) pairs of its tiles into log-sum-exp, minus the stored bf16 logit of the target
// (ignore_index -100 rows give 0, as F.cross_entropy does).
__global__ void __launch_bounds__(256) ce_combine_kernel(const float2* __restrict__ part, int tiles, int rows,
                                                         const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                                         int64_t vocab, const int64_t* __restrict__ targets,
                                                         float* __restrict__ row_loss) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float M = -INFINITY, S = 0.f;
  for (int t = 0; t < tiles; ++t) {
    const float2 q = part[(int64_t)t * rows + r];
    const float mm = fmaxf(M, q.x);
    if (mm == -INFINITY) continue;
    S = S * ex2_approx(M - mm) + q.y * ex2_approx(q.x - mm);
    M = mm;
  }
  const int64_t t = targets[r];
  float loss;
  if (t == -100) {
    loss = 0.f;
  } else if (t < 0 || t >= vocab) {
    record_device_error(ENGPT_ERR_ARG, 3);
    loss = NAN;
  } else {
    loss = (M + log2f(S)) * 0.6931471805599453f - __bfloat162float(logits[(int64_t)r * ld + t]);
  }
  row_loss[r] = loss;
}

}  // namespace gemm
}  // namespace engpt

extern "C" int engpt_logits_cross_entropy(const void* x, const void* w_head, int64_t rows, int d, int64_t vocab,
                                          void* logits, int64_t ld, const int64_t* targets, void* partials,
                                          float* row_loss, float* loss_out, void* stream) {
  using namespace gemm;
  clear_error();
  ENGPT_REQUIRE(rows > 0 && d > 0 && vocab > 0 && ld >= vocab, ENGPT_ERR_SHAPE,
                "logits_cross_entropy: rows=%lld d=%d vocab=%lld ld=%lld", (long long)rows, d, (long long)vocab,
                (long long)ld);
  ENGPT_REQUIRE(rows <= 0x7fffffffLL && vocab <= 0x7fffffffLL, ENGPT_ERR_SHAPE, "logits_cross_entropy: too large");
  ENGPT_REQUIRE(x && w_head && logits && targets && partials && row_loss && loss_out, ENGPT_ERR_ARG,
                "logits_cross_entropy: null pointer");
  ENGPT_REQUIRE(d % 8 == 0 && ld % 8 == 0 && aligned(logits, 16) && aligned(partials, 8), ENGPT_ERR_ALIGN,
                "logits_cross_entropy: d and ld must be multiples of 8, logits 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int tiles_n = (int)((vocab + BN - 1) / BN);
  LseEpi epi{reinterpret_cast<float2*>(partials), (int)rows, (int)vocab};
  int rc = launch(x, d, w_head, d, (int)vocab, (int)rows, tiles_n, d, 0, BN / 2, BN, logits, ld, (int)vocab, epi, st);
  if (rc) return rc;
  ce_combine_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const float2*>(partials), tiles_n, (int)rows, reinterpret_cast<const __nv_bfloat16*>(logits),
      ld, vocab, targets, row_loss);
  rc = check_launch("ce_combine");
  if (rc) return rc;
  return launch_mean_loss(row_loss, targets, rows, loss_out, st);
}
