// Tensor-core matrix products of the SPARC projection variant for B200 (sm_100a): the content
// product u = x [content_real | content_imag], the readout y = h readout^T + skip * x and, in
// the backward, dh = dy readout and dx = du content^T + dp controller^T + skip * dy
// (sparc-impl/sparc/recurrence.py:39-40, layers.py:125-126 and their adjoints).
//
//   C[m, n] = sum_k A[m, k] B[n, k]  (+ skip[n] X[m, n]) (+ dp[m, 0] c0[n] + dp[m, 1] c1[n])
//
// A [rows, K] and B [N, K] are row-major bfloat16 (K-major), or stored transposed as A [K, rows]
// and B [K, N] (M/N-major: the products that contract over the tokens, the weight gradients
// x^T du and dy^T h); C is bfloat16 or float32.
// Persistent: one CTA per SM walks the 128 x 256 output tiles t = blockIdx.x, + gridDim.x, ...
// (n fastest, so the CTAs running at once share their A row panels in L2), with
// tcgen05.mma (kind::f16, bf16 inputs, float32 accumulators in tensor memory):
//   warp 0      TMA producer: 128 x 64 tiles of A and 256 x 64 tiles of B (128-byte swizzle)
//               into a 4-stage ring of shared memory (`full` mbarriers); K-major operands as
//               one box of 64 k x (128 | 256) rows, M/N-major ones as 64 x 64 boxes (64
//               contiguous rows x 64 k) side by side;
//   warp 1      allocates all 512 TMEM columns (two 256-column accumulators); one thread issues
//               four 128x256x16 MMAs per stage, tcgen05.commit's the stage's `empty` barrier,
//               and after a tile's last stage the accumulator's `tmem_full` barrier;
//   warps 2-9   epilogue: warp w reads TMEM lanes [32 (w % 4), +32) (rows) and one half of the
//               columns of the finished accumulator with tcgen05.ld (the fused skip term's
//               loads issued first, so their latency overlaps the TMEM reads), releases it
//               (`tmem_empty`) and stores,
// so a tile's epilogue overlaps the next tile's main loop. Every mbarrier wait is bounded
// (max_spin polls); a wait that runs out or's 4 into *status and its role stops, every role
// still reaches the end, where the TMEM is released. No multicast.
#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

namespace sparc {

constexpr int kGemmBM = 128, kGemmBN = 256, kGemmBK = 64;  // BK: 64 bf16 = one 128-byte swizzle row
constexpr int kGemmStages = 4;
constexpr int kGemmEpiWarps = 8;                               // two per TMEM lane quadrant
constexpr int kGemmThreads = 64 + 32 * kGemmEpiWarps;
constexpr int kGemmAccs = 2;                                   // TMEM accumulators (2 x 256 columns)
constexpr unsigned kGemmABytes = kGemmBM * kGemmBK * 2;        // 16 KB
constexpr unsigned kGemmBBytes = kGemmBN * kGemmBK * 2;        // 32 KB
constexpr unsigned kStatusGemmTimeout = 4u;

struct GemmParams {
  CUtensorMap map_a;   // A [rows, K] bf16, box {64, 128} (K-major) or [K, rows], box {64, 64} (M-major)
  CUtensorMap map_b;   // B [N, K] bf16, box {64, 256} (K-major) or [K, N], box {64, 64} (N-major)
  int a_mn, b_mn;      // operand layouts: 0 K-major, 1 M/N-major
  void* out;           // [rows, N]
  int out_f32;
  const __nv_bfloat16* x;  // [rows, N] (skip term) or null
  const float* skip;       // [N]
  const float* dp;         // [rows, 2] or null
  const float* c0;         // [N]
  const float* c1;         // [N]
  int rows, N, K;
  int mtiles, ntiles;
  int ksplit;          // K ranges per output tile (1: no split)
  int kb_per_split;    // 64-wide k blocks per range
  float* part;         // [ksplit][rows][N] float32 partial products when ksplit > 1
  unsigned max_spin;
  unsigned* status;
};

struct __align__(1024) GemmSmem {
  __nv_bfloat16 a[kGemmStages][kGemmBM * kGemmBK];  // 1024-byte aligned tiles (swizzle atoms)
  __nv_bfloat16 b[kGemmStages][kGemmBN * kGemmBK];
  unsigned long long full[kGemmStages];
  unsigned long long empty[kGemmStages];
  unsigned long long tmem_full[kGemmAccs];
  unsigned long long tmem_empty[kGemmAccs];
  unsigned tmem_base;
  // per epilogue warp: the fused terms' column vectors (skip, c0, c1) of its 128 columns
  alignas(16) float epi[kGemmEpiWarps][3][kGemmBN / 2];
};
static_assert(sizeof(GemmSmem) + 1024 <= 227 * 1024, "the product's shared memory exceeds the opt-in limit");

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle: rows of 128 bytes,
// Shared-memory matrix descriptors (PTX ISA tcgen05 matrix descriptor: start address, leading
// and stride byte offsets in 16-byte units, version 1 for sm_100, 128-byte swizzle), for the
// two canonical 128-byte-swizzle layouts the TMA boxes produce:
//   K-major: rows of 128 bytes (64 k) per M/N index, 8-row atoms 1024 bytes apart (SBO);
//   M/N-major: rows of 128 bytes (64 M/N) per k, 8-k atoms 1024 bytes apart (SBO), 64-wide
//   M/N atoms 8192 bytes apart (LBO: the next 64 x 64 box).
__device__ __forceinline__ unsigned long long smem_desc_sw128(const void* p) {
  const unsigned long long addr = smem_addr(p);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ unsigned long long smem_desc_sw128_mn(const void* p) {
  const unsigned long long addr = smem_addr(p);
  return ((addr >> 4) & 0x3FFFull) | ((8192ull >> 4) << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: float32 accumulators, bf16 A and B, N = kGemmBN,
// M = kGemmBM; bits 15 / 16: A / B M/N-major (else K-major).
constexpr unsigned kGemmIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(kGemmBN >> 3) << 17) |
                                ((unsigned)(kGemmBM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(unsigned tmem_d, unsigned long long adesc, unsigned long long bdesc,
                                          unsigned idesc, unsigned accumulate) {
  const unsigned zero = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(zero));
}

__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive columns of this thread's TMEM lane (no wait: see tmem_wait16).
__device__ __forceinline__ void tmem_ld16(unsigned taddr, unsigned (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// tcgen05.wait::ld for two 16-column loads; the registers are operands, so no use of them can be
// scheduled before the wait.
__device__ __forceinline__ void tmem_wait32(unsigned (&a)[16], unsigned (&b)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]),
                 "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                 "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15])
               :
               : "memory");
}

// The skip term's 16 bf16 of one row (raw, as two 16-byte words; zero past N or the rows).
__device__ __forceinline__ void gemm_load_x16(const GemmParams& p, int row, int n0, bool ok, uint4 (&w)[2]) {
  w[0] = w[1] = make_uint4(0u, 0u, 0u, 0u);
  if (p.x == nullptr || !ok || n0 >= p.N) return;
  const int nn = min(16, p.N - n0);
  const long long base = (long long)row * p.N + n0;
  if (nn == 16 && (base & 7) == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(p.x + base);
    w[0] = __ldg(src);
    w[1] = __ldg(src + 1);
  } else {
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(w);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < nn) h[i] = p.x[base + i];
  }
}

// Four consecutive floats of a column vector (zeros past n).
__device__ __forceinline__ float4 gemm_col4(const float* v, int n0, int n) {
  if (n0 + 3 < n && (reinterpret_cast<uintptr_t>(v + n0) & 15u) == 0) return __ldg(reinterpret_cast<const float4*>(v + n0));
  float4 r;
  r.x = n0 < n ? __ldg(v + n0) : 0.0f;
  r.y = n0 + 1 < n ? __ldg(v + n0 + 1) : 0.0f;
  r.z = n0 + 2 < n ? __ldg(v + n0 + 2) : 0.0f;
  r.w = n0 + 3 < n ? __ldg(v + n0 + 3) : 0.0f;
  return r;
}

// 16 columns of one output row: fused terms (their column vectors from this warp's staging
// area `stg`: skip at [0], c0 at [kGemmBN / 2], c1 at [kGemmBN], offset to these columns), then
// the store (vectorised when aligned).
__device__ __forceinline__ void gemm_store16(const GemmParams& p, int row, int n0, float (&v)[16], float d0, float d1,
                                             const uint4 (&xw)[2], const float* stg) {
  const int nn = min(16, p.N - n0);
  const long long base = (long long)row * p.N + n0;
  const bool vec = nn == 16 && (base & 7) == 0;
  if (p.x != nullptr) {
    float sk[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<float4*>(sk + 4 * i) = reinterpret_cast<const float4*>(stg)[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(xw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = fmaf(sk[2 * i], f.x, v[2 * i]);
      v[2 * i + 1] = fmaf(sk[2 * i + 1], f.y, v[2 * i + 1]);
    }
  }
  if (p.dp != nullptr) {
    float c0[16], c1[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      *reinterpret_cast<float4*>(c0 + 4 * i) = reinterpret_cast<const float4*>(stg + kGemmBN / 2)[i];
      *reinterpret_cast<float4*>(c1 + 4 * i) = reinterpret_cast<const float4*>(stg + kGemmBN)[i];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = fmaf(d0, c0[i], fmaf(d1, c1[i], v[i]));
  }
  if (p.out_f32) {
    float* o = static_cast<float*>(p.out) + base;
    if (nn == 16 && (base & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < nn) o[i] = v[i];
    }
  } else {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + base;
    if (vec) {
      uint4 w[2];
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(w);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      reinterpret_cast<uint4*>(o)[0] = w[0];
      reinterpret_cast<uint4*>(o)[1] = w[1];
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < nn) o[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// 16 float32 partial sums of one output row (vectorised when aligned).
__device__ __forceinline__ void gemm_store_part16(float* part, int N, int row, int n0, const float (&v)[16]) {
  const int nn = min(16, N - n0);
  float* o = part + (long long)row * N + n0;
  if (nn == 16 && (((long long)row * N + n0) & 3) == 0) {
#pragma unroll
    for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < nn) o[i] = v[i];
  }
}

// Split-K finish: out = the k ranges' partial products summed in order, then the fused terms as
// the unsplit epilogue applies them (skip, then the rank-2 term), in the output dtype.
__global__ void __launch_bounds__(256) proj_gemm_finish_kernel(const __grid_constant__ GemmParams p) {
  const long long total = (long long)p.rows * p.N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    float v = 0.0f;
    for (int sp = 0; sp < p.ksplit; ++sp) v += __ldg(p.part + sp * total + i);
    const long long row = i / p.N;
    const int n = (int)(i - row * p.N);
    if (p.x != nullptr) v = fmaf(__ldg(p.skip + n), __bfloat162float(p.x[i]), v);
    if (p.dp != nullptr) v = fmaf(__ldg(p.dp + 2 * row), __ldg(p.c0 + n), fmaf(__ldg(p.dp + 2 * row + 1), __ldg(p.c1 + n), v));
    if (p.out_f32)
      static_cast<float*>(p.out)[i] = v;
    else
      static_cast<__nv_bfloat16*>(p.out)[i] = __float2bfloat16_rn(v);
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1) proj_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) unsigned char gemm_smem_raw[];
  // the dynamic shared memory window is only 16-byte aligned: round up to the swizzle atom
  GemmSmem& S = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = (p.K + kGemmBK - 1) / kGemmBK;
  const int tiles = p.mtiles * p.ntiles;
  const int units = tiles * p.ksplit;  // work unit u: output tile u % tiles, k range u / tiles
  bool timed_out = false;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int c = 0; c < kGemmAccs; ++c) {
      mbar_init(&S.tmem_full[c], 1);
      mbar_init(&S.tmem_empty[c], kGemmEpiWarps);  // one arrive per epilogue warp
    }
    mbar_init_fence();
  }
  if (warp == 1) {  // the whole warp allocates (sync.aligned); the address lands in shared memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&S.tmem_base)),
                 "r"(kGemmAccs * kGemmBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = S.tmem_base;
  pdl_wait();  // A, B and the epilogue inputs come from the previous kernels

  if (warp == 0) {
    if (lane == 0) {
      unsigned it = 0;
      for (int u = blockIdx.x; u < units && !timed_out; u += gridDim.x) {
        const int t = u % tiles, sp = u / tiles;
        const int tm = t / p.ntiles, tn = t - tm * p.ntiles;
        const int kb0 = sp * p.kb_per_split, kb1 = min(kblocks, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = (int)(it % kGemmStages);
          const unsigned round = it / kGemmStages;
          if (round > 0 && !mbar_wait(&S.empty[s], (round - 1) & 1u, p.max_spin)) {
            timed_out = true;
            break;
          }
          mbar_arrive_expect_tx(&S.full[s], kGemmABytes + kGemmBBytes);
          if (p.a_mn) {  // 64 x 64 boxes (64 contiguous rows x 64 k), 8 KB apart
#pragma unroll
            for (int i = 0; i < kGemmBM / 64; ++i)
              tma_load_2d(S.a[s] + i * 64 * kGemmBK, &p.map_a, tm * kGemmBM + 64 * i, kb * kGemmBK, &S.full[s]);
          } else {
            tma_load_2d(S.a[s], &p.map_a, kb * kGemmBK, tm * kGemmBM, &S.full[s]);
          }
          if (p.b_mn) {
#pragma unroll
            for (int i = 0; i < kGemmBN / 64; ++i)
              tma_load_2d(S.b[s] + i * 64 * kGemmBK, &p.map_b, tn * kGemmBN + 64 * i, kb * kGemmBK, &S.full[s]);
          } else {
            tma_load_2d(S.b[s], &p.map_b, kb * kGemmBK, tn * kGemmBN, &S.full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      unsigned it = 0, lt = 0;
      for (int u = blockIdx.x; u < units && !timed_out; u += gridDim.x, ++lt) {
        const int sp = u / tiles;
        const int kb0 = sp * p.kb_per_split, kb1 = min(kblocks, kb0 + p.kb_per_split);
        const unsigned acc = lt % kGemmAccs, use = lt / kGemmAccs;
        if (use > 0 && !mbar_wait(&S.tmem_empty[acc], (use - 1) & 1u, p.max_spin)) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        const unsigned d = tmem + acc * kGemmBN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = (int)(it % kGemmStages);
          if (!mbar_wait(&S.full[s], (it / kGemmStages) & 1u, p.max_spin)) {
            timed_out = true;
            break;
          }
          tc_fence_after();
          const unsigned long long ad = p.a_mn ? smem_desc_sw128_mn(S.a[s]) : smem_desc_sw128(S.a[s]);
          const unsigned long long bd = p.b_mn ? smem_desc_sw128_mn(S.b[s]) : smem_desc_sw128(S.b[s]);
          // one MMA per 16 k: 32 bytes along a K-major row (2 address units), 16 rows of 128 bytes
          // of an M/N-major tile (128 units)
          const unsigned long long astep = p.a_mn ? 128ull : 2ull, bstep = p.b_mn ? 128ull : 2ull;
          const unsigned idesc = kGemmIdesc | ((unsigned)p.a_mn << 15) | ((unsigned)p.b_mn << 16);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k)
            umma_bf16(d, ad + astep * k, bd + bstep * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit(&S.empty[s]);
        }
        umma_commit(&S.tmem_full[acc]);  // arrives once the tile's MMAs have completed
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes [32 (w % 4), +32) = rows of the tile, columns
    // [half * 128, +128)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    unsigned lt = 0;
    float* stg = &S.epi[warp - 2][0][0];
    constexpr int kCols = kGemmBN / 2;
    for (int u = blockIdx.x; u < units && !timed_out; u += gridDim.x, ++lt) {
      const int t = u % tiles, sp = u / tiles;
      const int tm = t / p.ntiles, tn = t - tm * p.ntiles;
      const unsigned acc = lt % kGemmAccs, use = lt / kGemmAccs;
      // this warp's 128 columns of the fused terms' vectors, four per lane (loads in flight
      // during the wait; staged in the warp's own shared memory, so __syncwarp orders it)
      const bool fused = p.ksplit == 1 && (p.x != nullptr || p.dp != nullptr);
      float4 fs = make_float4(0.f, 0.f, 0.f, 0.f), f0 = fs, f1 = fs;
      if (fused) {
        const int nl = tn * kGemmBN + half * kCols + 4 * lane;
        if (p.x != nullptr) fs = gemm_col4(p.skip, nl, p.N);
        if (p.dp != nullptr) {
          f0 = gemm_col4(p.c0, nl, p.N);
          f1 = gemm_col4(p.c1, nl, p.N);
        }
      }
      if (!mbar_wait(&S.tmem_full[acc], use & 1u, p.max_spin)) {
        timed_out = true;
        break;
      }
      tc_fence_after();
      if (fused) {
        __syncwarp();  // the previous tile's reads of the staging area are complete
        reinterpret_cast<float4*>(stg)[lane] = fs;
        reinterpret_cast<float4*>(stg + kCols)[lane] = f0;
        reinterpret_cast<float4*>(stg + 2 * kCols)[lane] = f1;
        __syncwarp();
      }
      const int row = tm * kGemmBM + q * 32 + lane;
      const bool row_ok = row < p.rows;
      float d0 = 0.0f, d1 = 0.0f;
      if (p.dp != nullptr && row_ok && p.ksplit == 1) {
        d0 = p.dp[2 * (long long)row];
        d1 = p.dp[2 * (long long)row + 1];
      }
      const unsigned taddr = tmem + acc * kGemmBN + ((unsigned)(q * 32) << 16);
#pragma unroll 1
      for (int c = half * kCols; c < (half + 1) * kCols; c += 32) {
        const int n0 = tn * kGemmBN + c;
        uint4 xa[2], xb[2];  // the skip term's loads first: in flight during the TMEM reads
        gemm_load_x16(p, row, n0, row_ok && p.ksplit == 1, xa);
        gemm_load_x16(p, row, n0 + 16, row_ok && p.ksplit == 1, xb);
        unsigned ra[16], rb[16];
        __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
        tmem_ld16(taddr + (unsigned)c, ra);
        tmem_ld16(taddr + (unsigned)(c + 16), rb);
        tmem_wait32(ra, rb);
        float va[16], vb[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          va[i] = __uint_as_float(ra[i]);
          vb[i] = __uint_as_float(rb[i]);
        }
        if (p.ksplit > 1) {  // a k range's partial product: raw, the finish kernel adds the rest
          float* part = p.part + (long long)sp * p.rows * p.N;
          if (row_ok && n0 < p.N) gemm_store_part16(part, p.N, row, n0, va);
          if (row_ok && n0 + 16 < p.N) gemm_store_part16(part, p.N, row, n0 + 16, vb);
        } else {
          const int lc = c - half * kCols;  // column within this warp's staged vectors
          if (row_ok && n0 < p.N) gemm_store16(p, row, n0, va, d0, d1, xa, stg + lc);
          if (row_ok && n0 + 16 < p.N) gemm_store16(p, row, n0 + 16, vb, d0, d1, xb, stg + lc + 16);
        }
      }
      // this warp's reads of the accumulator are complete (tcgen05.wait::ld): release it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.tmem_empty[acc]);
    }
  }
  if (timed_out) atomicOr(p.status, kStatusGemmTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGemmAccs * kGemmBN)
                 : "memory");
  }
}

// ------------------------------------------------------------------ column sums (skinny products)
// The layer backward's gradients of the two controller projections (x^T dp: [w, 2] over the
// tokens, plus the bias row sum_r dp) and of the skip (sum_r dy x per column): too narrow for
// the tensor cores, one pass over x (and dy). Grid (column blocks of 256, row splits): thread
// j of a block sums its column over the split's rows (the rows' dp pairs broadcast), the
// split's partials go to the workspace, and a second kernel adds the splits in order (float64).
constexpr int kColThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kColThreads) proj_colsum_kernel(const T* __restrict__ x, const float2* __restrict__ dp,
                                                                  const T* __restrict__ dy, float* part, long long rows,
                                                                  int w, long long per_split) {
  const int j = blockIdx.x * kColThreads + threadIdx.x;
  const long long r0 = blockIdx.y * per_split, r1 = min(rows, r0 + per_split);
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, b0 = 0.0f, b1 = 0.0f;
  if (j < w) {
    long long r = r0;
    for (; r + 4 <= r1; r += 4) {
      float xv[4], dv[4];
      float2 pv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        xv[u] = to_float(__ldg(x + (r + u) * w + j));
        pv[u] = __ldg(dp + r + u);
        dv[u] = dy != nullptr ? to_float(__ldg(dy + (r + u) * w + j)) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a0 = fmaf(xv[u], pv[u].x, a0);
        a1 = fmaf(xv[u], pv[u].y, a1);
        a2 = fmaf(dv[u], xv[u], a2);
        b0 += pv[u].x;
        b1 += pv[u].y;
      }
    }
    for (; r < r1; ++r) {
      const float xv = to_float(__ldg(x + r * w + j));
      const float2 pv = __ldg(dp + r);
      a0 = fmaf(xv, pv.x, a0);
      a1 = fmaf(xv, pv.y, a1);
      if (dy != nullptr) a2 = fmaf(to_float(__ldg(dy + r * w + j)), xv, a2);
      b0 += pv.x;
      b1 += pv.y;
    }
    float* o = part + ((long long)blockIdx.y * (w + 1) + j) * 3;
    o[0] = a0;
    o[1] = a1;
    o[2] = a2;
    if (j == 0) {  // the bias row: sum_r dp over the split
      float* ob = part + ((long long)blockIdx.y * (w + 1) + w) * 3;
      ob[0] = b0;
      ob[1] = b1;
      ob[2] = 0.0f;
    }
  }
}

// Unpacks one 16-byte load into float32: eight bfloat16 or four float32 elements.
template <typename T>
struct Vec16;
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int kN = 8;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <>
struct Vec16<float> {
  static constexpr int kN = 4;
  __device__ __forceinline__ static void unpack(const uint4& r, float* f) {
    f[0] = __uint_as_float(r.x);
    f[1] = __uint_as_float(r.y);
    f[2] = __uint_as_float(r.z);
    f[3] = __uint_as_float(r.w);
  }
};

// The column sums with 16-byte loads (w a multiple of the elements per load, 16-byte aligned
// rows). A CTA is ct column threads x rl row lanes (ct = min(256, w / V), rl = 256 / ct): column
// thread c owns the V adjacent columns (blockIdx.x * ct + c) * V .. + V, row lane l takes rows
// l, l + rl, ... of the CTA's split, four at a time for float32, two for bfloat16 (eight / four
// 16-byte loads in flight per thread with dy); the row lanes' sums are then added in lane order through shared memory. Partials as
// proj_colsum_kernel's: [split][w + 1][3].
template <typename T>
__global__ void __launch_bounds__(kColThreads, 4) proj_colsum_vec_kernel(const T* __restrict__ x,
                                                                      const float2* __restrict__ dp,
                                                                      const T* __restrict__ dy, float* part,
                                                                      long long rows, int w, long long per_split,
                                                                      int ct) {
  constexpr int V = Vec16<T>::kN;
  constexpr int U = V == 8 ? 2 : 4;  // rows per step (bfloat16: fewer, for 4 CTAs per SM)
  __shared__ float red[kColThreads][3 * V + 2];
  const int rl = kColThreads / ct;
  const int c = threadIdx.x % ct, l = threadIdx.x / ct;
  const int j0 = (blockIdx.x * ct + c) * V;
  const long long r0 = blockIdx.y * per_split, r1 = min(rows, r0 + per_split);
  float a0[V], a1[V], a2[V];
#pragma unroll
  for (int v = 0; v < V; ++v) a0[v] = a1[v] = a2[v] = 0.0f;
  float b0 = 0.0f, b1 = 0.0f;
  const bool has_dy = dy != nullptr;
  const bool active = j0 < w && l < rl;
  if (active) {
    long long r = r0 + l;
    for (; r + (U - 1LL) * rl < r1; r += (long long)U * rl) {
      uint4 xr[U], dr[U];
      float2 pv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long ru = r + (long long)u * rl;
        xr[u] = __ldg(reinterpret_cast<const uint4*>(x + ru * w + j0));
        pv[u] = __ldg(dp + ru);
        dr[u] = has_dy ? __ldg(reinterpret_cast<const uint4*>(dy + ru * w + j0)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float xv[V], dv[V];
        Vec16<T>::unpack(xr[u], xv);
        Vec16<T>::unpack(dr[u], dv);
#pragma unroll
        for (int v = 0; v < V; ++v) {
          a0[v] = fmaf(xv[v], pv[u].x, a0[v]);
          a1[v] = fmaf(xv[v], pv[u].y, a1[v]);
          a2[v] = fmaf(dv[v], xv[v], a2[v]);
        }
        b0 += pv[u].x;
        b1 += pv[u].y;
      }
    }
    for (; r < r1; r += rl) {
      float xv[V], dv[V];
      Vec16<T>::unpack(__ldg(reinterpret_cast<const uint4*>(x + r * w + j0)), xv);
      Vec16<T>::unpack(has_dy ? __ldg(reinterpret_cast<const uint4*>(dy + r * w + j0)) : make_uint4(0, 0, 0, 0), dv);
      const float2 pv = __ldg(dp + r);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        a0[v] = fmaf(xv[v], pv.x, a0[v]);
        a1[v] = fmaf(xv[v], pv.y, a1[v]);
        a2[v] = fmaf(dv[v], xv[v], a2[v]);
      }
      b0 += pv.x;
      b1 += pv.y;
    }
  }
  if (rl > 1) {  // add the row lanes in order (lane 0 keeps its own sums)
    if (l > 0 && l < rl) {
      float* o = red[threadIdx.x];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        o[3 * v] = a0[v];
        o[3 * v + 1] = a1[v];
        o[3 * v + 2] = a2[v];
      }
      o[3 * V] = b0;
      o[3 * V + 1] = b1;
    }
    __syncthreads();
    if (l == 0) {
      for (int q = 1; q < rl; ++q) {
        const float* o = red[q * ct + c];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          a0[v] += o[3 * v];
          a1[v] += o[3 * v + 1];
          a2[v] += o[3 * v + 2];
        }
        b0 += o[3 * V];
        b1 += o[3 * V + 1];
      }
    }
  }
  if (l == 0 && j0 < w) {
    float* o = part + ((long long)blockIdx.y * (w + 1) + j0) * 3;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      o[3 * v] = a0[v];
      o[3 * v + 1] = a1[v];
      o[3 * v + 2] = a2[v];
    }
    if (j0 == 0) {  // the bias row: sum_r dp over the split
      float* ob = part + ((long long)blockIdx.y * (w + 1) + w) * 3;
      ob[0] = b0;
      ob[1] = b1;
      ob[2] = 0.0f;
    }
  }
}

// Adds the splits' partials per column in float64: CTA per 32 columns, warp q adds splits
// q, q + 8, ... in order, then warp 0 adds the eight warps' sums in order.
__global__ void __launch_bounds__(kColThreads) proj_colsum_finish_kernel(const float* part, int splits, int w,
                                                                         float* d_ctl, float* d_skip) {
  __shared__ double red[kColThreads / 32][32][3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x * 32 + lane;
  double s0 = 0.0, s1 = 0.0, s2 = 0.0;
  if (j <= w) {
    constexpr int kStep = kColThreads / 32;
    int k = warp;
    for (; k + 3 * kStep < splits; k += 4 * kStep) {  // four splits' loads in flight
      float v[4][3];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float* o = part + ((long long)(k + u * kStep) * (w + 1) + j) * 3;
        v[u][0] = o[0];
        v[u][1] = o[1];
        v[u][2] = o[2];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        s0 += v[u][0];
        s1 += v[u][1];
        s2 += v[u][2];
      }
    }
    for (; k < splits; k += kStep) {
      const float* o = part + ((long long)k * (w + 1) + j) * 3;
      s0 += o[0];
      s1 += o[1];
      s2 += o[2];
    }
  }
  red[warp][lane][0] = s0;
  red[warp][lane][1] = s1;
  red[warp][lane][2] = s2;
  __syncthreads();
  if (warp != 0 || j > w) return;
  s0 = s1 = s2 = 0.0;
  for (int q = 0; q < kColThreads / 32; ++q) {
    s0 += red[q][lane][0];
    s1 += red[q][lane][1];
    s2 += red[q][lane][2];
  }
  d_ctl[2 * j] = (float)s0;
  d_ctl[2 * j + 1] = (float)s1;
  if (d_skip != nullptr && j < w) d_skip[j] = (float)s2;
}

// The controller projections of the layer's forward: p[r, :] = sum_j x[r, j] c[j, :] + c[w, :]
// (x [rows, w], c [w + 1, 2] float32: the two controllers with their biases in the last row).
// One warp per row (eight rows per CTA), each lane a strided set of columns, loads of 8 bf16 /
// 4 float32 at once where the row allows, a shuffle tree in a fixed order.
template <typename T>
__global__ void __launch_bounds__(kColThreads) proj_rowdot_kernel(const T* __restrict__ x, const float2* __restrict__ c,
                                                                  float2* __restrict__ p, long long rows, int w) {
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * (kColThreads / 32) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const T* xr = x + r * w;
  float s0 = 0.0f, s1 = 0.0f;
  constexpr int V = 16 / (int)sizeof(T);  // elements per 16-byte load
  const bool vec = (w % V) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  if (vec) {
    for (int j0 = lane * V; j0 < w; j0 += 32 * V) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr + j0));
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int u = 0; u < V; ++u) {
        const float xv = to_float(e[u]);
        const float2 cv = __ldg(c + j0 + u);
        s0 = fmaf(xv, cv.x, s0);
        s1 = fmaf(xv, cv.y, s1);
      }
    }
  } else {
    for (int j = lane; j < w; j += 32) {
      const float xv = to_float(__ldg(xr + j));
      const float2 cv = __ldg(c + j);
      s0 = fmaf(xv, cv.x, s0);
      s1 = fmaf(xv, cv.y, s1);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
  }
  if (lane == 0) {
    const float2 bias = __ldg(c + w);
    p[r] = make_float2(s0 + bias.x, s1 + bias.y);
  }
}

// The controller projections with the coefficients held in registers (w a multiple of the
// elements per 16-byte load, 16-byte aligned rows): a row group of nw warps (G = 32 nw threads)
// takes R rows at a time; thread gl of the group owns the KC chunks of V adjacent columns
// (gl + k G) V, k < KC, and their coefficients, loaded once, so each row costs its own 16-byte
// loads and nothing else. The 2R partial sums of a warp are reduced by a transposing shuffle
// tree (halving the values at each of the first two levels), the group's warps are added in
// order through shared memory, one barrier per iteration (two buffers). Fixed order throughout.
constexpr int kRowR = 2;

template <typename T, int KC>
__global__ void __launch_bounds__(kColThreads) proj_rowdot_reg_kernel(const T* __restrict__ x,
                                                                      const float2* __restrict__ c,
                                                                      float* __restrict__ p, long long rows, int w,
                                                                      int nw) {
  constexpr int V = Vec16<T>::kN;
  constexpr int R = kRowR;
  static_assert(2 * R == 4, "the shuffle tree reduces four values");
  __shared__ float red[2][kColThreads / 32][2 * R];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (kColThreads / 32) / nw;
  const int grp = warp / nw, sub = warp - grp * nw;
  const int G = 32 * nw;
  const int gl = sub * 32 + lane;
  float c0[KC][V], c1[KC][V];
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    const int j = (gl + k * G) * V;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const float2 cv = j < w ? __ldg(c + j + v) : make_float2(0.0f, 0.0f);
      c0[k][v] = cv.x;
      c1[k][v] = cv.y;
    }
  }
  const float2 bias = __ldg(c + w);
  const long long per_iter = (long long)groups * R;
  const long long stride = (long long)gridDim.x * per_iter;
  // the rows' 16-byte chunks of this thread; the next iteration's are loaded into the same
  // registers as soon as the current ones are consumed, so they are in flight during the
  // reduction and the barrier
  uint4 xr[R][KC];
  auto load_rows = [&](long long base) {
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const long long r = base + grp * R + i;
#pragma unroll
      for (int k = 0; k < KC; ++k) {
        const int j = (gl + k * G) * V;
        xr[i][k] = (r < rows && j < w) ? __ldg(reinterpret_cast<const uint4*>(x + r * w + j)) : make_uint4(0, 0, 0, 0);
      }
    }
  };
  int buf = 0;
  load_rows((long long)blockIdx.x * per_iter);
  for (long long base = (long long)blockIdx.x * per_iter; base < rows; base += stride) {
    float v4[2 * R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int k = 0; k < KC; ++k) {
        float xv[V];
        Vec16<T>::unpack(xr[i][k], xv);
#pragma unroll
        for (int v = 0; v < V; ++v) {
          s0 = fmaf(xv[v], c0[k][v], s0);
          s1 = fmaf(xv[v], c1[k][v], s1);
        }
      }
      v4[2 * i] = s0;
      v4[2 * i + 1] = s1;
    }
    load_rows(base + stride);
    // lanes with bit 4 keep values {2, 3}, the others {0, 1}; then bit 3 halves again
    {
      const bool hi = (lane & 16) != 0;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = hi ? v4[i] : v4[i + 2];
        const float keep = hi ? v4[i + 2] : v4[i];
        v4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
      const bool mid = (lane & 8) != 0;
      const float send = mid ? v4[0] : v4[1];
      const float keep = mid ? v4[1] : v4[0];
      v4[0] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
#pragma unroll
      for (int o = 4; o >= 1; o >>= 1) v4[0] += __shfl_xor_sync(0xffffffffu, v4[0], o);
    }
    if ((lane & 7) == 0) red[buf][warp][lane >> 3] = v4[0];  // lane 8q holds value q
    __syncthreads();
    if (threadIdx.x < groups * 2 * R) {
      const int g = threadIdx.x / (2 * R), q = threadIdx.x - g * (2 * R);
      float t = 0.0f;
      for (int sb = 0; sb < nw; ++sb) t += red[buf][g * nw + sb][q];
      const long long r = base + g * R + (q >> 1);
      if (r < rows) p[2 * r + (q & 1)] = t + ((q & 1) ? bias.y : bias.x);
    }
    buf ^= 1;
  }
}

// Row splits for the column sums, for `cols_per_thread` columns per thread (1: the scalar
// kernel; V: the vector kernel, whose CTAs hold 256 / ct row lanes): enough CTAs for four per SM
// over the column blocks (a fixed 148 SMs, so the order of the sums does not depend on the
// device), at least 16 rows per row lane.
static void colsum_shape(int w, int cols_per_thread, int* ct, int* cblocks) {
  const int nch = (w + cols_per_thread - 1) / cols_per_thread;
  *ct = cols_per_thread == 1 ? kColThreads : std::min(kColThreads, nch);
  *cblocks = (nch + *ct - 1) / *ct;
}
static void colsum_plan(long long rows, int w, int cols_per_thread, int* splits, long long* per_split) {
  int ct, cblocks;
  colsum_shape(w, cols_per_thread, &ct, &cblocks);
  const long long rl = kColThreads / ct;
  long long s = std::max<long long>(1, std::min<long long>((rows + 16 * rl - 1) / (16 * rl), (4 * 148 + cblocks - 1) / cblocks));
  s = std::min<long long>(s, 65535);
  *per_split = (rows + s - 1) / s;
  *splits = (int)((rows + *per_split - 1) / *per_split);
}

// Split-K plan: the number of k ranges per output tile that minimises the estimated time,
// in units of one 64-deep k block of one tile on one SM (~0.38 us at the measured bf16 peak):
// waves of work units x k blocks per range, plus, when split, the partials' HBM round trip
// (write and read, 8 bytes per output element per range, at ~6.5 TB/s) and the finish launch.
// Products with at least as many tiles as SMs, or short k, stay unsplit.
static int gemm_ksplit(long long rows, int n, int k, int sms, int* kb_per_split) {
  const long long tiles = ((rows + kGemmBM - 1) / kGemmBM) * ((n + kGemmBN - 1) / kGemmBN);
  const long long kblocks = (k + kGemmBK - 1) / kGemmBK;
  int best = 1;
  long long best_kbs = kblocks;
  double best_cost = (double)((tiles + sms - 1) / sms) * (double)kblocks;
  if (tiles < sms && kblocks >= 8) {
    for (int sp = 2; sp <= 64 && sp <= kblocks / 4; ++sp) {
      const long long kbs = (kblocks + sp - 1) / sp;
      const long long eff = (kblocks + kbs - 1) / kbs;  // ranges actually needed
      const double waves = (double)((tiles * eff + sms - 1) / sms);
      const double part_us = (double)eff * (double)rows * (double)n * 8.0 / 6.5e12 * 1e6;
      const double cost = waves * (double)kbs + (part_us + 3.0) / 0.38;
      if (cost < best_cost) {
        best_cost = cost;
        best = (int)eff;
        best_kbs = kbs;
      }
    }
  }
  *kb_per_split = (int)best_kbs;
  return best;
}

static int current_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms = 148;
  }
  return sms;
}

static PFN_cuTensorMapEncodeTiled_v12000 gemm_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}

// [rows, K] bf16 row-major as a 2-D map with a {64, box_rows} box and 128-byte swizzle (K-major
// operand); mnmajor_map: [K, rows] bf16 row-major with a {64, 64} box (M/N-major operand).
static bool kmajor_map(CUtensorMap* map, const void* base, long long rows, int K, int box_rows) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = gemm_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool mnmajor_map(CUtensorMap* map, const void* base, long long K, long long rows) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = gemm_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)rows, (cuuint64_t)K};
  const cuuint64_t strides[1] = {(cuuint64_t)rows * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)kGemmBK};
  const cuuint32_t estride[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static thread_local char g_gemm_err[256];

static int gemm_fail(int code, const char* msg) {
  snprintf(g_gemm_err, sizeof(g_gemm_err), "%s", msg);
  return code;
}

}  // namespace sparc

using namespace sparc;

extern "C" {

const char* sparc_proj_gemm_last_error(void) { return g_gemm_err; }

int sparc_proj_rowdot(const SparcProjRowdotArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return gemm_fail(SPARC_ERR_ARG, "null args");
  if (!a->x || !a->c || !a->p) return gemm_fail(SPARC_ERR_ARG, "null tensor pointer");
  if (a->rows <= 0 || a->w <= 0) return gemm_fail(SPARC_ERR_SHAPE, "rows and w must be positive");
  if (a->dtype != SPARC_DTYPE_F32 && a->dtype != SPARC_DTYPE_BF16) return gemm_fail(SPARC_ERR_DTYPE, "unsupported dtype");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long blocks = (a->rows + kColThreads / 32 - 1) / (kColThreads / 32);
  if (blocks >= (1LL << 31)) return gemm_fail(SPARC_ERR_SHAPE, "too many rows");
  TimedLaunch tl(kTimeProjRowdot, s);
  // registers-held coefficients where the rows load as whole 16-byte vectors: the fewest warps
  // per row (nw) whose threads hold the row in at most 16 columns each (32 for wide bf16 rows)
  const bool bf = a->dtype == SPARC_DTYPE_BF16;
  const int V = bf ? 8 : 4;
  if (a->w % V == 0 && (reinterpret_cast<uintptr_t>(a->x) & 15u) == 0) {
    const int nch = a->w / V;
    int nw = 0, kc = 0;
    for (int kcap : {16 / V, 32 / V}) {
      for (int n = 1; n <= 8 && nw == 0; n *= 2)
        if (32 * n * kcap >= nch) nw = n;
      if (nw != 0) {
        kc = (nch + 32 * nw - 1) / (32 * nw);
        kc = kc <= 1 ? 1 : kc <= 2 ? 2 : kc <= 4 ? 4 : 8;
        break;
      }
    }
    if (nw != 0 && kc <= 4) {
      int dev = 0, sms = 148;
      if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        sms = 148;
      }
      const long long per_iter = (long long)((kColThreads / 32) / nw) * kRowR;
      const void* fn = bf ? (kc == 1   ? (const void*)proj_rowdot_reg_kernel<__nv_bfloat16, 1>
                             : kc == 2 ? (const void*)proj_rowdot_reg_kernel<__nv_bfloat16, 2>
                                       : (const void*)proj_rowdot_reg_kernel<__nv_bfloat16, 4>)
                          : (kc == 1   ? (const void*)proj_rowdot_reg_kernel<float, 1>
                             : kc == 2 ? (const void*)proj_rowdot_reg_kernel<float, 2>
                                       : (const void*)proj_rowdot_reg_kernel<float, 4>);
      int per_sm = 0;  // one full wave of persistent CTAs
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kColThreads, 0) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        per_sm = 2;
      }
      const unsigned grid =
          (unsigned)std::max<long long>(1, std::min<long long>((a->rows + per_iter - 1) / per_iter, (long long)per_sm * sms));
      float* p = static_cast<float*>(a->p);
      const float2* c = reinterpret_cast<const float2*>(a->c);
      long long rows = a->rows;
      int w = a->w;
      const void* x = a->x;
      void* args[] = {const_cast<void**>(&x), const_cast<float2**>(&c), &p, &rows, &w, &nw};
      const cudaError_t le = cudaLaunchKernel(fn, dim3(grid), dim3(kColThreads), args, 0, s);
      if (le != cudaSuccess) return gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(le));
      const cudaError_t e = cudaGetLastError();
      return e == cudaSuccess ? SPARC_OK : gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
    }
  }
  if (a->dtype == SPARC_DTYPE_BF16)
    proj_rowdot_kernel<__nv_bfloat16><<<(unsigned)blocks, kColThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(a->x), reinterpret_cast<const float2*>(a->c), reinterpret_cast<float2*>(a->p),
        a->rows, a->w);
  else
    proj_rowdot_kernel<float><<<(unsigned)blocks, kColThreads, 0, s>>>(
        static_cast<const float*>(a->x), reinterpret_cast<const float2*>(a->c), reinterpret_cast<float2*>(a->p), a->rows,
        a->w);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPARC_OK : gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

size_t sparc_proj_colsum_workspace_bytes(long long rows, int w) {
  if (rows <= 0 || w <= 0) return 0;
  int splits;
  long long per;
  size_t most = 0;
  for (int cpt : {1, 4, 8}) {  // the scalar and both vector paths
    colsum_plan(rows, w, cpt, &splits, &per);
    most = std::max(most, (size_t)splits);
  }
  splits = (int)most;
  return (size_t)splits * (size_t)(w + 1) * 3 * sizeof(float);
}

int sparc_proj_colsum(const SparcProjColsumArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return gemm_fail(SPARC_ERR_ARG, "null args");
  if (!a->x || !a->dp || !a->d_ctl || !a->workspace) return gemm_fail(SPARC_ERR_ARG, "null tensor pointer");
  if (a->rows <= 0 || a->w <= 0) return gemm_fail(SPARC_ERR_SHAPE, "rows and w must be positive");
  if (a->dtype != SPARC_DTYPE_F32 && a->dtype != SPARC_DTYPE_BF16) return gemm_fail(SPARC_ERR_DTYPE, "unsupported dtype");
  if (a->workspace_bytes < sparc_proj_colsum_workspace_bytes(a->rows, a->w))
    return gemm_fail(SPARC_ERR_WORKSPACE, "workspace too small");
  if ((a->dy != nullptr) != (a->d_skip != nullptr)) return gemm_fail(SPARC_ERR_ARG, "dy and d_skip go together");
  const int V = a->dtype == SPARC_DTYPE_BF16 ? 8 : 4;
  const bool vec = a->w % V == 0 && (reinterpret_cast<uintptr_t>(a->x) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(a->dy) & 15u) == 0;
  int splits, ct, cblocks;
  long long per;
  colsum_plan(a->rows, a->w, vec ? V : 1, &splits, &per);
  colsum_shape(a->w, vec ? V : 1, &ct, &cblocks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(cblocks, splits);
  float* part = static_cast<float*>(a->workspace);
  TimedLaunch tl(kTimeProjColsum, s);  // both launches: partial sums and the fixed-order finish
  if (vec && a->dtype == SPARC_DTYPE_BF16)
    proj_colsum_vec_kernel<__nv_bfloat16><<<grid, kColThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(a->x), reinterpret_cast<const float2*>(a->dp),
        static_cast<const __nv_bfloat16*>(a->dy), part, a->rows, a->w, per, ct);
  else if (vec)
    proj_colsum_vec_kernel<float><<<grid, kColThreads, 0, s>>>(static_cast<const float*>(a->x),
                                                               reinterpret_cast<const float2*>(a->dp),
                                                               static_cast<const float*>(a->dy), part, a->rows, a->w,
                                                               per, ct);
  else if (a->dtype == SPARC_DTYPE_BF16)
    proj_colsum_kernel<__nv_bfloat16><<<grid, kColThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(a->x), reinterpret_cast<const float2*>(a->dp),
        static_cast<const __nv_bfloat16*>(a->dy), part, a->rows, a->w, per);
  else
    proj_colsum_kernel<float><<<grid, kColThreads, 0, s>>>(static_cast<const float*>(a->x),
                                                           reinterpret_cast<const float2*>(a->dp),
                                                           static_cast<const float*>(a->dy), part, a->rows, a->w, per);
  proj_colsum_finish_kernel<<<(a->w + 1 + 31) / 32, kColThreads, 0, s>>>(part, splits, a->w, a->d_ctl, a->d_skip);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPARC_OK : gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

size_t sparc_proj_gemm_workspace_bytes(long long rows, int n, int k) {
  if (rows <= 0 || n <= 0 || k <= 0) return 0;
  int kbs = 0;
  const int sp = gemm_ksplit(rows, n, k, current_sms(), &kbs);
  return sp > 1 ? (size_t)sp * (size_t)rows * (size_t)n * sizeof(float) : 0;
}

int sparc_proj_gemm(const SparcProjGemmArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return gemm_fail(SPARC_ERR_ARG, "null args");
  if (!a->a || !a->b || !a->out || !a->status) return gemm_fail(SPARC_ERR_ARG, "null tensor pointer");
  if (a->rows <= 0 || a->n <= 0 || a->k <= 0) return gemm_fail(SPARC_ERR_SHAPE, "rows, n and k must be positive");
  if (a->a_mn < 0 || a->a_mn > 1 || a->b_mn < 0 || a->b_mn > 1) return gemm_fail(SPARC_ERR_ARG, "a_mn and b_mn are 0 or 1");
  // the contiguous dimension of each operand must be whole 16-byte rows
  if ((!a->a_mn || !a->b_mn) && a->k % 8 != 0) return gemm_fail(SPARC_ERR_SHAPE, "k must be a multiple of 8 (16-byte rows)");
  if (a->a_mn && a->rows % 8 != 0) return gemm_fail(SPARC_ERR_SHAPE, "rows must be a multiple of 8 for an M-major a");
  if (a->b_mn && a->n % 8 != 0) return gemm_fail(SPARC_ERR_SHAPE, "n must be a multiple of 8 for an N-major b");
  if ((a->x != nullptr) != (a->skip != nullptr) || (a->dp != nullptr && (!a->c0 || !a->c1)))
    return gemm_fail(SPARC_ERR_ARG, "x / skip and dp / c0 / c1 go together");
  const long long mt = (a->rows + kGemmBM - 1) / kGemmBM, nt = (a->n + kGemmBN - 1) / kGemmBN;
  if (mt * nt >= (1LL << 31)) return gemm_fail(SPARC_ERR_SHAPE, "too many output tiles");
  if (reinterpret_cast<uintptr_t>(a->a) % 16 || reinterpret_cast<uintptr_t>(a->b) % 16)
    return gemm_fail(SPARC_ERR_ARG, "a and b must be 16-byte aligned");
  GemmParams p;
  p.a_mn = a->a_mn;
  p.b_mn = a->b_mn;
  const bool ma = a->a_mn ? mnmajor_map(&p.map_a, a->a, a->k, a->rows) : kmajor_map(&p.map_a, a->a, a->rows, a->k, kGemmBM);
  const bool mb = a->b_mn ? mnmajor_map(&p.map_b, a->b, a->k, a->n) : kmajor_map(&p.map_b, a->b, a->n, a->k, kGemmBN);
  if (!ma || !mb) return gemm_fail(SPARC_ERR_ARG, "tensor map encoding failed");
  p.out = a->out;
  p.out_f32 = a->out_f32;
  p.x = static_cast<const __nv_bfloat16*>(a->x);
  p.skip = a->skip;
  p.dp = a->dp;
  p.c0 = a->c0;
  p.c1 = a->c1;
  p.rows = (int)a->rows;
  p.N = a->n;
  p.K = a->k;
  p.mtiles = (int)mt;
  p.ntiles = (int)nt;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 22);
  p.status = a->status;
  p.ksplit = 1;
  p.kb_per_split = (a->k + kGemmBK - 1) / kGemmBK;
  p.part = nullptr;
  {
    int kbs = 0;
    const int sp = gemm_ksplit(a->rows, a->n, a->k, current_sms(), &kbs);
    const size_t need = (size_t)sp * (size_t)a->rows * (size_t)a->n * sizeof(float);
    // split only into a caller workspace that holds the partials (else the unsplit product)
    if (sp > 1 && a->workspace != nullptr && a->workspace_bytes >= need &&
        reinterpret_cast<uintptr_t>(a->workspace) % 16 == 0) {
      p.ksplit = sp;
      p.kb_per_split = kbs;
      p.part = static_cast<float*>(a->workspace);
    }
  }
  const size_t smem = sizeof(GemmSmem) + 1024;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return gemm_fail(SPARC_ERR_LAUNCH, "no current CUDA device");
  }
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms = 148;
  }
  {
    // the shared-memory opt-in is a function attribute of each device's context: set it once
    // per device (one process may drive several GPUs)
    static std::mutex mu;
    static unsigned long long opted_in = 0;  // bit per device ordinal
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 64 || !((opted_in >> dev) & 1ull)) {
      const cudaError_t ae =
          cudaFuncSetAttribute((const void*)proj_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (ae != cudaSuccess) {
        cudaGetLastError();
        return gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(ae));
      }
      if (dev < 64) opted_in |= 1ull << dev;
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min<long long>(mt * nt * p.ksplit, sms), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&p};
  {
    TimedLaunch tl(kTimeProjGemm, s);
    const cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)proj_gemm_kernel, args);
    if (e != cudaSuccess) return gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
  }
  if (p.ksplit > 1) {
    TimedLaunch tl(kTimeProjGemmFinish, s);
    const long long total = (long long)p.rows * p.N;
    const unsigned blocks = (unsigned)std::min<long long>((total + 255) / 256, 8LL * sms);
    proj_gemm_finish_kernel<<<blocks, 256, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
  }
  return SPARC_OK;
}

}  // extern "C"
