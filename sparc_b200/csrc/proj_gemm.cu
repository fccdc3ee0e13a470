// Tensor-core matrix products of the SPARC projection variant for B200 (sm_100a): the content
// product u = x [content_real | content_imag], the readout y = h readout^T + skip * x and, in
// the backward, dh = dy readout and dx = du content^T + dp controller^T + skip * dy
// (sparc-impl/sparc/recurrence.py:39-40, layers.py:125-126 and their adjoints).
//
//   C[m, n] = sum_k A[m, k] B[n, k]  (+ skip[n] X[m, n]) (+ dp[m, 0] c0[n] + dp[m, 1] c1[n])
//
// A [rows, K] and B [N, K] are row-major bfloat16 (both K-major); C is bfloat16 or float32.
// Persistent: one CTA per SM walks the 128 x 256 output tiles t = blockIdx.x, + gridDim.x, ...
// (n fastest, so the CTAs running at once share their A row panels in L2), with
// tcgen05.mma (kind::f16, bf16 inputs, float32 accumulators in tensor memory):
//   warp 0      TMA producer: 128 x 64 tiles of A and 256 x 64 tiles of B (128-byte swizzle)
//               into a 4-stage ring of shared memory (`full` mbarriers);
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
  CUtensorMap map_a;   // A [rows, K] bf16, box {64, 128}, 128-byte swizzle
  CUtensorMap map_b;   // B [N, K] bf16, box {64, 256}
  void* out;           // [rows, N]
  int out_f32;
  const __nv_bfloat16* x;  // [rows, N] (skip term) or null
  const float* skip;       // [N]
  const float* dp;         // [rows, 2] or null
  const float* c0;         // [N]
  const float* c1;         // [N]
  int rows, N, K;
  int mtiles, ntiles;
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
};

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
// 8-row swizzle atoms 1024 bytes apart (stride byte offset), descriptor version 1 (sm_100).
__device__ __forceinline__ unsigned long long smem_desc_sw128(const void* p) {
  const unsigned long long addr = smem_addr(p);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: float32 accumulators, bf16 A and B, both K-major,
// N = kGemmBN, M = kGemmBM.
constexpr unsigned kGemmIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(kGemmBN >> 3) << 17) |
                                ((unsigned)(kGemmBM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(unsigned tmem_d, unsigned long long adesc, unsigned long long bdesc,
                                          unsigned accumulate) {
  const unsigned zero = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kGemmIdesc), "r"(accumulate), "r"(zero));
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
    for (int i = 0; i < nn; ++i) h[i] = p.x[base + i];
  }
}

// 16 columns of one output row: fused terms, then the store (vectorised when aligned).
__device__ __forceinline__ void gemm_store16(const GemmParams& p, int row, int n0, float (&v)[16], float d0, float d1,
                                             const uint4 (&xw)[2]) {
  const int nn = min(16, p.N - n0);
  const long long base = (long long)row * p.N + n0;
  const bool vec = nn == 16 && (base & 7) == 0;
  if (p.x != nullptr) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(xw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      if (2 * i < nn) v[2 * i] = fmaf(__ldg(p.skip + n0 + 2 * i), f.x, v[2 * i]);
      if (2 * i + 1 < nn) v[2 * i + 1] = fmaf(__ldg(p.skip + n0 + 2 * i + 1), f.y, v[2 * i + 1]);
    }
  }
  if (p.dp != nullptr) {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < nn) v[i] = fmaf(d0, __ldg(p.c0 + n0 + i), fmaf(d1, __ldg(p.c1 + n0 + i), v[i]));
  }
  if (p.out_f32) {
    float* o = static_cast<float*>(p.out) + base;
    if (nn == 16 && (base & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
      for (int i = 0; i < nn; ++i) o[i] = v[i];
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
      for (int i = 0; i < nn; ++i) o[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1) proj_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) unsigned char gemm_smem_raw[];
  // the dynamic shared memory window is only 16-byte aligned: round up to the swizzle atom
  GemmSmem& S = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = (p.K + kGemmBK - 1) / kGemmBK;
  const int tiles = p.mtiles * p.ntiles;
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
      for (int t = blockIdx.x; t < tiles && !timed_out; t += gridDim.x) {
        const int tm = t / p.ntiles, tn = t - tm * p.ntiles;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = (int)(it % kGemmStages);
          const unsigned round = it / kGemmStages;
          if (round > 0 && !mbar_wait(&S.empty[s], (round - 1) & 1u, p.max_spin)) {
            timed_out = true;
            break;
          }
          mbar_arrive_expect_tx(&S.full[s], kGemmABytes + kGemmBBytes);
          tma_load_2d(S.a[s], &p.map_a, kb * kGemmBK, tm * kGemmBM, &S.full[s]);
          tma_load_2d(S.b[s], &p.map_b, kb * kGemmBK, tn * kGemmBN, &S.full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      unsigned it = 0, lt = 0;
      for (int t = blockIdx.x; t < tiles && !timed_out; t += gridDim.x, ++lt) {
        const unsigned acc = lt % kGemmAccs, use = lt / kGemmAccs;
        if (use > 0 && !mbar_wait(&S.tmem_empty[acc], (use - 1) & 1u, p.max_spin)) {
          timed_out = true;
          break;
        }
        tc_fence_after();
        const unsigned d = tmem + acc * kGemmBN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = (int)(it % kGemmStages);
          if (!mbar_wait(&S.full[s], (it / kGemmStages) & 1u, p.max_spin)) {
            timed_out = true;
            break;
          }
          tc_fence_after();
          const unsigned long long ad = smem_desc_sw128(S.a[s]);
          const unsigned long long bd = smem_desc_sw128(S.b[s]);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k)  // 16 bf16 = 32 bytes = 2 descriptor address units
            umma_bf16(d, ad + 2ull * k, bd + 2ull * k, (kb > 0 || k > 0) ? 1u : 0u);
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
    for (int t = blockIdx.x; t < tiles && !timed_out; t += gridDim.x, ++lt) {
      const int tm = t / p.ntiles, tn = t - tm * p.ntiles;
      const unsigned acc = lt % kGemmAccs, use = lt / kGemmAccs;
      if (!mbar_wait(&S.tmem_full[acc], use & 1u, p.max_spin)) {
        timed_out = true;
        break;
      }
      tc_fence_after();
      const int row = tm * kGemmBM + q * 32 + lane;
      const bool row_ok = row < p.rows;
      float d0 = 0.0f, d1 = 0.0f;
      if (p.dp != nullptr && row_ok) {
        d0 = p.dp[2 * (long long)row];
        d1 = p.dp[2 * (long long)row + 1];
      }
      const unsigned taddr = tmem + acc * kGemmBN + ((unsigned)(q * 32) << 16);
      constexpr int kCols = kGemmBN / 2;
#pragma unroll 1
      for (int c = half * kCols; c < (half + 1) * kCols; c += 32) {
        const int n0 = tn * kGemmBN + c;
        uint4 xa[2], xb[2];  // the skip term's loads first: in flight during the TMEM reads
        gemm_load_x16(p, row, n0, row_ok, xa);
        gemm_load_x16(p, row, n0 + 16, row_ok, xb);
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
        if (row_ok && n0 < p.N) gemm_store16(p, row, n0, va, d0, d1, xa);
        if (row_ok && n0 + 16 < p.N) gemm_store16(p, row, n0 + 16, vb, d0, d1, xb);
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

// [rows, K] bf16 row-major as a 2-D map with a {64, box_rows} box and 128-byte swizzle.
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

static thread_local char g_gemm_err[256];

static int gemm_fail(int code, const char* msg) {
  snprintf(g_gemm_err, sizeof(g_gemm_err), "%s", msg);
  return code;
}

}  // namespace sparc

using namespace sparc;

extern "C" {

const char* sparc_proj_gemm_last_error(void) { return g_gemm_err; }

int sparc_proj_gemm(const SparcProjGemmArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return gemm_fail(SPARC_ERR_ARG, "null args");
  if (!a->a || !a->b || !a->out || !a->status) return gemm_fail(SPARC_ERR_ARG, "null tensor pointer");
  if (a->rows <= 0 || a->n <= 0 || a->k <= 0) return gemm_fail(SPARC_ERR_SHAPE, "rows, n and k must be positive");
  if (a->k % 8 != 0) return gemm_fail(SPARC_ERR_SHAPE, "k must be a multiple of 8 (16-byte rows)");
  if ((a->x != nullptr) != (a->skip != nullptr) || (a->dp != nullptr && (!a->c0 || !a->c1)))
    return gemm_fail(SPARC_ERR_ARG, "x / skip and dp / c0 / c1 go together");
  const long long mt = (a->rows + kGemmBM - 1) / kGemmBM, nt = (a->n + kGemmBN - 1) / kGemmBN;
  if (mt * nt >= (1LL << 31)) return gemm_fail(SPARC_ERR_SHAPE, "too many output tiles");
  if (reinterpret_cast<uintptr_t>(a->a) % 16 || reinterpret_cast<uintptr_t>(a->b) % 16)
    return gemm_fail(SPARC_ERR_ARG, "a and b must be 16-byte aligned");
  GemmParams p;
  if (!kmajor_map(&p.map_a, a->a, a->rows, a->k, kGemmBM) || !kmajor_map(&p.map_b, a->b, a->n, a->k, kGemmBN))
    return gemm_fail(SPARC_ERR_ARG, "tensor map encoding failed");
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
  cfg.gridDim = dim3((unsigned)std::min<long long>(mt * nt, sms), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&p};
  TimedLaunch tl(kTimeProjGemm, s);
  const cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)proj_gemm_kernel, args);
  return e == cudaSuccess ? SPARC_OK : gemm_fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

}  // extern "C"
