// SPARC mixer forward / backward for B200 (sm_100a).
//
// Work unit ("tile"): one batch row b and one chunk of C consecutive tokens, all M modes.
// A tile is processed by one thread-block cluster of G CTAs; CTA g owns modes
// [g*NT, g*NT + NT) with one thread per mode, so the cross-mode per-token reductions
// (controller projection in the forward, the shared-control gradient in the backward) run
// on-chip: warp transpose-reduce -> shared memory -> distributed shared memory across the
// cluster.
//
// Kernels are persistent: clusters take tiles from a ticket counter in chunk-major order
// (ticket = c*B + b forward, (chunks-1-c)*B + b backward), so a tile only ever waits on tiles
// with smaller tickets, which are held by running clusters. Chunk carries are passed by
// decoupled lookback: a tile publishes its aggregate affine map (A, B: out = A*in + B, per
// mode) and, once it knows its carry-in, its inclusive state; successors compose aggregates
// until they reach an inclusive state. The forward's inclusive states double as the saved
// chunk carries that the backward replays from.
//
// Parity targets (reference paths inside Botwwt/sparc):
//   controls  forward/control.py:129-139      write  forward/control.py:167-195
//   scan      forward/scan.py:886-1003,1277-1354  (chunk summary / prefix / replay)
//   backward  backward/scan.py:382-644 (reverse chunk kernels), backward/control.py:11-89
//             (write backward), autograd of make_controls for the controller gradient.
#include <cooperative_groups.h>

#include <algorithm>
#include <type_traits>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "sparc_b200.h"

namespace cg = cooperative_groups;

namespace sparc {

#ifndef SPARC_BF16_CHUNK
#define SPARC_BF16_CHUNK 16
#endif
// Tokens per tile (the chunk of the saved carries): 16 for bfloat16, 8 for float32 (whose
// shared-memory tiles are twice as large).
__host__ __device__ constexpr int chunk_for(int dtype) { return dtype == SPARC_DTYPE_BF16 ? SPARC_BF16_CHUNK : 8; }

struct ModeConst {
  float nu;      // e^{nu_log}
  float nl2e;    // nu * log2(e)
  float ct, st;  // cos/sin theta
  float theta;
  float gconst;  // e^{write_log_gain} / sqrt(-expm1(-2 nu))
  float stat;    // nu e^{-2nu} / -expm1(-2nu)
  float wpr, wrr;
  float d0r, d0i, d1r, d1i;  // controller directions at columns m and M+m
};

struct MixerParamPtrs {
  const float* nu_log;
  const float* theta_log;
  const float* phase_dir;   // [W+1]
  const float* radial_dir;  // [W+1]
  const float* wlg;
  const float* wpr;
  const float* wrr;
};

__device__ __forceinline__ ModeConst load_mode(const MixerParamPtrs& pp, int m, int M, bool active) {
  ModeConst mc;
  const float nu_log = active ? pp.nu_log[m] : 0.0f;
  const float theta_log = active ? pp.theta_log[m] : 0.0f;
  mc.nu = expf(nu_log);
  mc.nl2e = mc.nu * kLog2e;
  mc.theta = expf(theta_log);
  sincosf(mc.theta, &mc.st, &mc.ct);
  const float den = -expm1f(-2.0f * mc.nu);
  mc.gconst = active ? expf(pp.wlg[m]) * rsqrtf(den) : 0.0f;
  mc.stat = mc.nu * expf(-2.0f * mc.nu) / den;
  mc.wpr = active ? pp.wpr[m] : 0.0f;
  mc.wrr = active ? pp.wrr[m] : 0.0f;
  mc.d0r = active ? pp.phase_dir[m] : 0.0f;
  mc.d0i = active ? pp.phase_dir[M + m] : 0.0f;
  mc.d1r = active ? pp.radial_dir[m] : 0.0f;
  mc.d1i = active ? pp.radial_dir[M + m] : 0.0f;
  return mc;
}

struct TokenCoef {  // per-(token, mode) quantities shared by the forward and the backward
  float z, rho;
  float2 a;
  float num, gate, gain;
};

template <bool kFast>
__device__ __forceinline__ TokenCoef token_coef(const ModeConst& mc, float E, float delta,
                                                float tau0, float tau1) {
  TokenCoef k;
  k.z = mc.nu * E;
  k.rho = ex2_approx(-mc.nl2e * E);
  float s, c;
  sincos_halfpi(fmaf(-k.rho, delta, delta), &s, &c);  // (1 - rho) * delta, |.| <= pi/2
  const float rct = k.rho * mc.ct, rst = k.rho * mc.st;
  k.a = make_float2(fmaf(rct, c, -rst * s), fmaf(rst, c, rct * s));
  k.num = one_minus_exp_neg(2.0f * k.z, k.rho * k.rho);
  const float q = fmaf(tau0, mc.wpr, tau1 * mc.wrr);
  if constexpr (kFast) {
    k.gate = 1.0f + tanh_hw(0.5f * q);
  } else {
    k.gate = 2.0f * rcp_approx(1.0f + ex2_approx(-kLog2e * q));
  }
  k.gain = mc.gconst * sqrt_approx(k.num) * k.gate;
  return k;
}

// Transition a = rho e^{i(theta + (1-rho) delta)} alone (the reverse local pass needs no write).
__device__ __forceinline__ float2 token_transition(const ModeConst& mc, float E, float delta) {
  const float rho = ex2_approx(-mc.nl2e * E);
  float s, c;
  sincos_halfpi(fmaf(-rho, delta, delta), &s, &c);
  const float rct = rho * mc.ct, rst = rho * mc.st;
  return make_float2(fmaf(rct, c, -rst * s), fmaf(rst, c, rct * s));
}

// Warp transpose-reduce of N values per lane (N a power of two, N <= 32). Afterwards lane l
// holds the warp total of value l >> (5 - log2 N).
template <int N>
__device__ __forceinline__ float transpose_reduce(float (&v)[N], int lane) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "N must be a power of two <= 32");
  int n = N;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return v[0];
}

template <int N>
__host__ __device__ constexpr int log2i() { return N <= 1 ? 0 : 1 + log2i<N / 2>(); }

// Reduce N per-thread values over the whole cluster. Every CTA ends with the cluster totals
// in out[0..N) (shared memory). s_warp: [NW][N], s_cta: [N] (peers read it).
template <int N, int NT>
__device__ __forceinline__ void cluster_reduce(float (&v)[N], float (*s_warp)[N], float* s_cta,
                                               float* out, cg::cluster_group& cluster) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kShift = 5 - log2i<N>();
  const float total = transpose_reduce<N>(v, lane);
  if ((lane & ((1 << kShift) - 1)) == 0) s_warp[warp][lane >> kShift] = total;
  __syncthreads();
  if (threadIdx.x < N) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) s += s_warp[w][threadIdx.x];
    s_cta[threadIdx.x] = s;
  }
  cluster.sync();
  if (threadIdx.x < N) {
    float s = 0.0f;
    const unsigned G = cluster.num_blocks();
    for (unsigned r = 0; r < G; ++r) s += cluster.map_shared_rank(s_cta, r)[threadIdx.x];
    out[threadIdx.x] = s;
  }
  __syncthreads();
}

// Token controls from the reduced projections: eta, delta, e^eta, tanh values.
template <int C>
__device__ __forceinline__ void token_controls(const float* proj, float b0, float b1, float* s_E,
                                               float* s_delta, float* s_tau0, float* s_tau1) {
  if (threadIdx.x < C) {
    const int t = threadIdx.x;
    const float tau0 = tanh_accurate(proj[t] + b0);
    const float tau1 = tanh_accurate(proj[C + t] + b1);
    s_tau0[t] = tau0;
    s_tau1[t] = tau1;
    s_delta[t] = kHalfPi * tau0;
    s_E[t] = expf(kLn16 * tau1);
  }
  __syncthreads();
}

// Decoupled lookback with a warp-wide window. The tile publishes its aggregate (out = A*in + B)
// unless its predecessor is already inclusive. Warp 0 then polls up to 32 predecessors at once
// (lane j reads the flag of the tile j+1 steps back) and picks the nearest inclusive one; the
// aggregates in between are composed by every thread for its own mode (their loads are
// independent, so the whole window costs about two round trips instead of one per
// predecessor). pred_inclusive(j) loads the inclusive state of the tile j steps back.
// Deterministic mode waits for the immediate predecessor's inclusive state instead (a chained
// scan), so the carry's rounding does not depend on which predecessors were done first.
struct LookbackCtx {
  LaunchState* ls;
  unsigned* flags;     // [tiles * G]
  float4* agg;         // [tiles * Mp]
  unsigned epoch;
  unsigned max_spin;
  int G;
  int Mp;
  long long B;         // ticket distance to the predecessor tile
  bool deterministic;
};

__device__ __forceinline__ void publish_flag(unsigned* flag, unsigned value) {
  // every thread's payload stores precede the barrier; thread 0's release store (cumulative
  // over what the barrier ordered before it) makes them visible with the flag
  __syncthreads();
  if (threadIdx.x == 0) st_release(flag, value);
}

template <int MPT, typename InclFn>
__device__ __forceinline__ void lookback(const LookbackCtx& lc, long long ticket, int g, int steps_back_max,
                                         const float2 (&A)[MPT], const float2 (&Bv)[MPT], bool publish,
                                         unsigned pred_state, unsigned* s_win, int mp0,
                                         InclFn pred_inclusive, float2 (&carry)[MPT]) {
  const int tid = threadIdx.x;
  const unsigned ep = lc.epoch & 0x3fffffffu;
  if (lc.deterministic) {
    if (tid == 0) {
      unsigned s = wait_flag(lc.flags + (ticket - lc.B) * lc.G + g, lc.epoch, lc.max_spin, kFlagInclusive);
      if (s == 0u) atomicOr(&lc.ls->status, kStatusTimeout);
      s_win[0] = s;
    }
    __syncthreads();
    const unsigned state = s_win[0];
    __syncthreads();
    if (state == kFlagInclusive) {
      pred_inclusive(1, carry);
    } else {
#pragma unroll
      for (int q = 0; q < MPT; ++q) carry[q] = make_float2(0.0f, 0.0f);
    }
    return;
  }
  const bool pred_ready = ((pred_state >> 2) == ep) && (pred_state & 3u) == kFlagInclusive;
  if (pred_ready) {
    pred_inclusive(1, carry);
    return;
  }
  if (publish) {
#pragma unroll
    for (int q = 0; q < MPT; ++q) lc.agg[ticket * lc.Mp + mp0 + q] = make_float4(A[q].x, A[q].y, Bv[q].x, Bv[q].y);
    publish_flag(lc.flags + ticket * lc.G + g, make_flag(lc.epoch, kFlagAggregate));
  }
  float2 accA[MPT], accB[MPT];
#pragma unroll
  for (int q = 0; q < MPT; ++q) {
    accA[q] = make_float2(1.0f, 0.0f);
    accB[q] = make_float2(0.0f, 0.0f);
  }
  int base = 0;  // the window covers predecessors base+1 .. base+32
  for (unsigned spin = 0;; ++spin) {
    if (tid < 32) {
      const int j = base + tid + 1;
      unsigned st = 0u;
      if (j <= steps_back_max) {
        const unsigned v = ld_acquire(lc.flags + (ticket - (long long)j * lc.B) * lc.G + g);
        st = ((v >> 2) == ep) ? (v & 3u) : 0u;
      }
      const unsigned incl = __ballot_sync(0xffffffffu, st == kFlagInclusive);
      const unsigned notready = __ballot_sync(0xffffffffu, st == 0u && j <= steps_back_max);
      if (tid == 0) {
        const int first_incl = incl ? __ffs(incl) - 1 : 32;
        const int first_wait = notready ? __ffs(notready) - 1 : 32;
        if (first_incl < first_wait) {            // aggregates, then an inclusive: done
          s_win[0] = first_incl;
          s_win[1] = 1u;
        } else {                                  // compose what is ready; wait for the rest
          s_win[0] = first_wait;
          s_win[1] = 0u;
        }
      }
    }
    __syncthreads();
    const int n = (int)s_win[0];
    const bool done = s_win[1] != 0u;
    __syncthreads();
    // compose the n aggregates nearest first; loads are issued a batch at a time so their
    // latencies overlap instead of adding up
    constexpr int kBatch = 8 / MPT;
    for (int j0 = 0; j0 < n; j0 += kBatch) {
      float4 ag[kBatch][MPT];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (j0 + u < n) {
          const float4* ap = lc.agg + (ticket - (long long)(base + j0 + u + 1) * lc.B) * lc.Mp + mp0;
#pragma unroll
          for (int q = 0; q < MPT; ++q) ag[u][q] = __ldcg(ap + q);
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (j0 + u < n) {
#pragma unroll
          for (int q = 0; q < MPT; ++q) {
            accB[q] = cfma(accA[q], make_float2(ag[u][q].z, ag[u][q].w), accB[q]);
            accA[q] = cmul(accA[q], make_float2(ag[u][q].x, ag[u][q].y));
          }
        }
      }
    }
    base += n;
    if (done) {
      float2 h[MPT];
      pred_inclusive(base + 1, h);
#pragma unroll
      for (int q = 0; q < MPT; ++q) carry[q] = cfma(accA[q], h[q], accB[q]);
      return;
    }
    if (base >= steps_back_max || (n == 0 && spin >= lc.max_spin)) {
      // a broken chain (a tile that never published): record it and continue with zero carry
      if (tid == 0) atomicOr(&lc.ls->status, kStatusTimeout);
#pragma unroll
      for (int q = 0; q < MPT; ++q) carry[q] = accB[q];
      return;
    }
    if (n == 0 && spin > 8) __nanosleep(spin < 64 ? 32 : 256);
  }
}

// Cluster rank 0 takes the next ticket; peers read it from rank 0's shared memory after the
// next cluster barrier. Double-buffered by tile parity.
__device__ __forceinline__ void take_ticket(LaunchState* ls, unsigned* s_ticket, int parity, int g) {
  if (g == 0 && threadIdx.x == 0) s_ticket[parity] = atomicAdd(&ls->ticket, 1u);
}

#include "mixer_fwd.cuh"

#include "mixer_bwd.cuh"

struct ReduceParams {
  const double* part;
  int clusters, Mp, M, W;
  const float* theta_log;
  float* g_nu_log;
  float* g_theta_log;
  float* g_wlg;
  float* g_wpr;
  float* g_wrr;
  float* g_energy;
  float* g_phase_dir;   // [W+1]
  float* g_radial_dir;  // [W+1]
};

// grid (ceil(Mp/32), kPartModes), block (32, 8): warp w sums clusters w, w+8, ... for 32 modes
// (coalesced), then warp 0 adds the eight partial sums in a fixed order.
constexpr int kReduceWarps = 8;

__global__ void __launch_bounds__(32 * kReduceWarps) mixer_reduce_kernel(const ReduceParams r) {
  const int lane = threadIdx.x, w = threadIdx.y;
  const int m = blockIdx.x * 32 + lane;
  const int q = blockIdx.y;
  __shared__ double sm[kReduceWarps][32];
  double s = 0.0;
  if (m < r.Mp) {
    for (int k = w; k < r.clusters; k += kReduceWarps) s += r.part[((long long)k * kPartModes + q) * r.Mp + m];
  }
  sm[w][lane] = s;
  __syncthreads();
  if (w == 0 && m < r.M) {
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < kReduceWarps; ++i) t += sm[i][lane];
    switch (q) {
      case 0: r.g_nu_log[m] = (float)t; r.g_energy[m] = 0.0f; break;
      case 1: r.g_theta_log[m] = (float)(t * exp((double)r.theta_log[m])); break;
      case 2: r.g_wlg[m] = (float)t; break;
      case 3: r.g_wpr[m] = (float)t; break;
      case 4: r.g_wrr[m] = (float)t; break;
      case 5: r.g_phase_dir[m] = (float)t; break;
      case 6: r.g_phase_dir[r.M + m] = (float)t; break;
      case 7: r.g_radial_dir[m] = (float)t; break;
      default: r.g_radial_dir[r.M + m] = (float)t; break;
    }
  }
  if (blockIdx.x == 0 && q == 0 && w == 1 && lane < 2) {
    const double* pb = r.part + (long long)r.clusters * kPartModes * r.Mp;
    double t = 0.0;
    for (int k = 0; k < r.clusters; ++k) t += pb[2 * k + lane];
    (lane == 0 ? r.g_phase_dir : r.g_radial_dir)[r.W] = (float)t;
  }
}

// ------------------------------------------------------------------------------ host side
struct Plan {
  int dtype, C, chunks;
  long long tiles;
  int Gf, Mpf, clusters_fwd;  // forward: CTAs of 256 modes
  size_t fwd_smem;
  bool fvec, tma;
  int Gb, Mpb, clusters_bwd;  // backward: CTAs of 256 modes
  size_t bwd_smem;
};

static thread_local char g_err[512];
static void set_err(const char* msg) { snprintf(g_err, sizeof(g_err), "%s", msg); }

template <typename K>
static int max_clusters(K kernel, int G, int NT, size_t dyn_smem) {
  if (G > 8) cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G, 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = dyn_smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = G;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Kernel instances: forward <TIO, C, fast math, vector pairs>, backward <TIO, NT, fast math, C>.
template <typename TIO>
struct Kernels {
  static constexpr bool kFast = std::is_same<TIO, __nv_bfloat16>::value;
  static constexpr int C = kFast ? SPARC_BF16_CHUNK : 8;
  static void* fwd(bool vec) {
    return vec ? (void*)mixer_fwd_kernel<TIO, C, kFast, true> : (void*)mixer_fwd_kernel<TIO, C, kFast, false>;
  }
  static void* bwd(bool vec) {
    return vec ? (void*)mixer_bwd_kernel<TIO, C, kFast, true> : (void*)mixer_bwd_kernel<TIO, C, kFast, false>;
  }
  static size_t fwd_smem() { return sizeof(FwdSmem<TIO, C, kFast>); }
  static size_t bwd_smem() { return sizeof(BwdSmem<TIO, C>); }
};

static int make_plan(long long B, long long T, int W, int dtype, Plan* pl) {
  if (B <= 0 || T <= 0 || W <= 0) { set_err("batch, length and width must be positive"); return SPARC_ERR_SHAPE; }
  if (W % 2) { set_err("SPARC rnn_width must be even"); return SPARC_ERR_SHAPE; }
  if (dtype != SPARC_DTYPE_F32 && dtype != SPARC_DTYPE_BF16) { set_err("unsupported dtype"); return SPARC_ERR_DTYPE; }
  const int M = W / 2;
  if (M > 8 * kFwdModes) { set_err("width above 4096 is not supported"); return SPARC_ERR_SHAPE; }
  pl->dtype = dtype;
  pl->C = chunk_for(dtype);
  pl->chunks = (int)((T + pl->C - 1) / pl->C);
  pl->tiles = B * pl->chunks;
  if (pl->tiles >= (1LL << 31)) { set_err("too many tiles"); return SPARC_ERR_SHAPE; }
  pl->Gf = (M + kFwdModes - 1) / kFwdModes;
  pl->Mpf = pl->Gf * kFwdModes;
  pl->fvec = (M % 2) == 0;
  const size_t s = dtype == SPARC_DTYPE_BF16 ? 2 : 4;
  pl->tma = ((size_t)W * s) % 16 == 0 && ((size_t)M * s) % 16 == 0;
  pl->Gb = (M + kBwdModes - 1) / kBwdModes;
  pl->Mpb = pl->Gb * kBwdModes;

  int dev = 0;
  cudaGetDevice(&dev);
  struct Key { int dev, dtype, Gf, Gb, vec; int nf, nb; };
  static std::mutex mu;
  static Key cache[64];
  static int ncache = 0;
  std::lock_guard<std::mutex> lock(mu);
  int nf = -1, nb = -1;
  for (int i = 0; i < ncache; ++i) {
    const Key& k = cache[i];
    if (k.dev == dev && k.dtype == dtype && k.Gf == pl->Gf && k.Gb == pl->Gb && k.vec == (int)pl->fvec) {
      nf = k.nf;
      nb = k.nb;
    }
  }
  if (dtype == SPARC_DTYPE_BF16) {
    pl->fwd_smem = Kernels<__nv_bfloat16>::fwd_smem();
    pl->bwd_smem = Kernels<__nv_bfloat16>::bwd_smem();
  } else {
    pl->fwd_smem = Kernels<float>::fwd_smem();
    pl->bwd_smem = Kernels<float>::bwd_smem();
  }
  if (nf < 0) {
    void* fk = dtype == SPARC_DTYPE_BF16 ? Kernels<__nv_bfloat16>::fwd(pl->fvec) : Kernels<float>::fwd(pl->fvec);
    void* bk = dtype == SPARC_DTYPE_BF16 ? Kernels<__nv_bfloat16>::bwd(pl->fvec) : Kernels<float>::bwd(pl->fvec);
    nf = max_clusters(fk, pl->Gf, kFwdThreads, pl->fwd_smem);
    nb = max_clusters(bk, pl->Gb, kBwdThreads, pl->bwd_smem);
    if (nf <= 0 || nb <= 0) { set_err("cluster occupancy query failed"); return SPARC_ERR_LAUNCH; }
    if (ncache < 64) cache[ncache++] = Key{dev, dtype, pl->Gf, pl->Gb, (int)pl->fvec, nf, nb};
  }
  pl->clusters_fwd = (int)std::min<long long>(nf, pl->tiles);
  pl->clusters_bwd = (int)std::min<long long>(nb, pl->tiles);
  return SPARC_OK;
}

struct WsLayout {
  size_t flags, agg, incl, part, total;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static WsLayout ws_layout(const Plan& pl) {
  WsLayout L;
  const int G = std::max(pl.Gf, pl.Gb);
  const int Mp = std::max(pl.Mpf, pl.Mpb);
  size_t off = align256(sizeof(LaunchState));
  L.flags = off;
  off = align256(off + (size_t)pl.tiles * G * sizeof(unsigned));
  L.agg = off;
  off = align256(off + (size_t)pl.tiles * Mp * sizeof(float4));
  L.incl = off;
  off = align256(off + (size_t)pl.tiles * pl.Mpb * sizeof(float2));
  L.part = off;
  off = align256(off + ((size_t)pl.clusters_bwd * kPartModes * pl.Mpb + 2 * (size_t)pl.clusters_bwd) * sizeof(double));
  L.total = off;
  return L;
}

template <typename P>
static cudaError_t launch_cluster(void* kernel, int G, int NT, int clusters, size_t dyn, cudaStream_t s,
                                  const P& params) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G, clusters, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = G;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<P*>(&params)};
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

// Validate the forward arguments and fill the kernel parameters (scratch at `ws`).
static int forward_params(const SparcMixerFwdArgs* a, const Plan& pl, const WsLayout& L, char* ws, FwdParams* p) {
  if (!a->x || !a->y || !a->carry || !a->nu_log || !a->theta_log || !a->phase_direction ||
      !a->radial_direction || !a->write_log_gain || !a->write_phase_response || !a->write_radial_response) {
    set_err("null tensor pointer"); return SPARC_ERR_ARG;
  }
  if ((a->h0_r == nullptr) != (a->h0_i == nullptr) || (a->last_r == nullptr) != (a->last_i == nullptr)) {
    set_err("h0 / last pointers must be given in pairs"); return SPARC_ERR_ARG;
  }
  p->x = a->x;
  p->y = a->y;
  p->pp = MixerParamPtrs{a->nu_log, a->theta_log, a->phase_direction, a->radial_direction,
                         a->write_log_gain, a->write_phase_response, a->write_radial_response};
  p->h0_r = a->h0_r;
  p->h0_i = a->h0_i;
  p->last_r = a->last_r;
  p->last_i = a->last_i;
  p->carry = reinterpret_cast<float2*>(a->carry);
  p->ls = reinterpret_cast<LaunchState*>(ws);
  p->flags = reinterpret_cast<unsigned*>(ws + L.flags);
  p->agg = reinterpret_cast<float4*>(ws + L.agg);
  p->B = a->batch;
  p->T = a->length;
  p->W = a->width;
  p->M = a->width / 2;
  p->chunks = pl.chunks;
  p->tiles = pl.tiles;
  p->max_spin = a->max_spin ? a->max_spin : (1u << 20);
  p->inject_unpublished = a->inject_enable ? a->inject_tile : -1;
  p->deterministic = a->deterministic;
  p->use_tma = pl.tma && (reinterpret_cast<uintptr_t>(a->x) % 16 == 0) ? 1 : 0;
  return SPARC_OK;
}

static int launch_forward(const Plan& pl, const FwdParams& p, cudaStream_t s) {
  void* k = pl.dtype == SPARC_DTYPE_BF16 ? Kernels<__nv_bfloat16>::fwd(pl.fvec) : Kernels<float>::fwd(pl.fvec);
  const cudaError_t e = launch_cluster(k, pl.Gf, kFwdThreads, pl.clusters_fwd, pl.fwd_smem, s, p);
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  return SPARC_OK;
}

}  // namespace sparc

using namespace sparc;

extern "C" {

const char* sparc_last_error(void) { return g_err; }

long long sparc_mixer_chunk_tokens(int dtype) { return chunk_for(dtype); }

long long sparc_mixer_carry_chunks(long long length, int dtype) {
  const int C = chunk_for(dtype);
  return (length + C - 1) / C;
}

size_t sparc_mixer_workspace_bytes(long long batch, long long length, int width, int dtype) {
  Plan pl;
  if (make_plan(batch, length, width, dtype, &pl) != SPARC_OK) return 0;
  return ws_layout(pl).total;
}

int sparc_mixer_forward(const SparcMixerFwdArgs* a, void* stream) {
  if (a == nullptr) { set_err("null args"); return SPARC_ERR_ARG; }
  Plan pl;
  int rc = make_plan(a->batch, a->length, a->width, a->dtype, &pl);
  if (rc != SPARC_OK) return rc;
  const WsLayout L = ws_layout(pl);
  if (a->workspace == nullptr || a->workspace_bytes < L.total) { set_err("workspace too small"); return SPARC_ERR_WORKSPACE; }
  FwdParams p;
  rc = forward_params(a, pl, L, static_cast<char*>(a->workspace), &p);
  if (rc != SPARC_OK) return rc;
  return launch_forward(pl, p, static_cast<cudaStream_t>(stream));
}

int sparc_mixer_backward(const SparcMixerBwdArgs* a, void* stream) {
  if (a == nullptr) { set_err("null args"); return SPARC_ERR_ARG; }
  Plan pl;
  int rc = make_plan(a->batch, a->length, a->width, a->dtype, &pl);
  if (rc != SPARC_OK) return rc;
  const WsLayout L = ws_layout(pl);
  if (a->workspace == nullptr || a->workspace_bytes < L.total) { set_err("workspace too small"); return SPARC_ERR_WORKSPACE; }
  if (!a->x || !a->dy || !a->dx || !a->carry || !a->grad_nu_log || !a->grad_theta_log ||
      !a->grad_phase_direction || !a->grad_radial_direction || !a->grad_write_log_gain ||
      !a->grad_energy_response || !a->grad_write_phase_response || !a->grad_write_radial_response) {
    set_err("null tensor pointer"); return SPARC_ERR_ARG;
  }
  if ((a->h0_r == nullptr) != (a->h0_i == nullptr) || (a->grad_last_r == nullptr) != (a->grad_last_i == nullptr) ||
      (a->grad_h0_r == nullptr) != (a->grad_h0_i == nullptr)) {
    set_err("paired pointers must be given together"); return SPARC_ERR_ARG;
  }
  char* ws = static_cast<char*>(a->workspace);
  BwdParams p;
  p.x = a->x;
  p.dy = a->dy;
  p.dx = a->dx;
  p.pp = MixerParamPtrs{a->nu_log, a->theta_log, a->phase_direction, a->radial_direction,
                        a->write_log_gain, a->write_phase_response, a->write_radial_response};
  p.h0_r = a->h0_r;
  p.h0_i = a->h0_i;
  p.glast_r = a->grad_last_r;
  p.glast_i = a->grad_last_i;
  p.gh0_r = a->grad_h0_r;
  p.gh0_i = a->grad_h0_i;
  p.carry = reinterpret_cast<const float2*>(a->carry);
  p.ls = reinterpret_cast<LaunchState*>(ws);
  p.flags = reinterpret_cast<unsigned*>(ws + L.flags);
  p.agg = reinterpret_cast<float4*>(ws + L.agg);
  p.incl = reinterpret_cast<float2*>(ws + L.incl);
  p.part = reinterpret_cast<double*>(ws + L.part);
  p.B = a->batch;
  p.T = a->length;
  p.W = a->width;
  p.M = a->width / 2;
  p.chunks = pl.chunks;
  p.tiles = pl.tiles;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 20);
  p.inject_unpublished = a->inject_enable ? a->inject_tile : -1;
  p.deterministic = a->deterministic;
  p.use_tma = pl.tma && (reinterpret_cast<uintptr_t>(a->x) % 16 == 0) && (reinterpret_cast<uintptr_t>(a->dy) % 16 == 0) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* k = a->dtype == SPARC_DTYPE_BF16 ? Kernels<__nv_bfloat16>::bwd(pl.fvec) : Kernels<float>::bwd(pl.fvec);
  cudaError_t e = launch_cluster(k, pl.Gb, kBwdThreads, pl.clusters_bwd, pl.bwd_smem, s, p);
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  ReduceParams r;
  r.part = p.part;
  r.clusters = pl.clusters_bwd;
  r.Mp = pl.Mpb;
  r.M = p.M;
  r.W = p.W;
  r.theta_log = a->theta_log;
  r.g_nu_log = a->grad_nu_log;
  r.g_theta_log = a->grad_theta_log;
  r.g_wlg = a->grad_write_log_gain;
  r.g_wpr = a->grad_write_phase_response;
  r.g_wrr = a->grad_write_radial_response;
  r.g_energy = a->grad_energy_response;
  r.g_phase_dir = a->grad_phase_direction;
  r.g_radial_dir = a->grad_radial_direction;
  mixer_reduce_kernel<<<dim3((pl.Mpb + 31) / 32, kPartModes), dim3(32, kReduceWarps), 0, s>>>(r);
  e = cudaGetLastError();
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  return SPARC_OK;
}

// ------------------------------------------------------------------------------ no-alloc variant
// sparc_mixer_forward_noalloc: the same forward kernel, with its scratch (launch counters,
// lookback flags and chunk aggregates) in a fixed array that lives in the library itself, for
// callers that cannot allocate device memory. See the declaration in sparc_b200.h.
}  // extern "C"

namespace sparc {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per GPU, held until exit

// Zero-initialised when the library's module is loaded on a device. Host code must not use
// this name as a device address: noalloc_scratch() looks the address up per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* noalloc_scratch(int dev) {
  static std::mutex mu;
  static void* addr[64] = {};
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* ptr = nullptr;
    // the current device is `dev`: the lookup (and the lazy module load it may trigger) binds
    // the array of this device
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return nullptr;
    }
    addr[dev] = ptr;
  }
  return addr[dev];
}

}  // namespace sparc

extern "C" {

size_t sparc_mixer_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int sparc_mixer_forward_noalloc(const SparcMixerFwdArgs* a, void* stream) {
  if (a == nullptr) { set_err("null args"); return SPARC_ERR_ARG; }
  Plan pl;
  int rc = make_plan(a->batch, a->length, a->width, a->dtype, &pl);
  if (rc != SPARC_OK) return rc;
  const WsLayout L = ws_layout(pl);
  // the forward uses the launch state, the flags and the aggregates (everything before incl)
  const size_t need = L.incl;
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "sparc_mixer_forward_noalloc: batch %lld x length %lld x width %d needs %zu bytes of "
             "scratch, above the built-in %zu; use sparc_mixer_forward with a workspace",
             a->batch, a->length, a->width, need, kNoAllocScratchBytes);
    set_err(msg);
    return SPARC_ERR_WORKSPACE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); set_err("no current CUDA device"); return SPARC_ERR_LAUNCH; }
  char* ws = static_cast<char*>(noalloc_scratch(dev));
  if (ws == nullptr) { set_err("cudaGetSymbolAddress failed for the built-in scratch"); return SPARC_ERR_LAUNCH; }
  FwdParams p;
  rc = forward_params(a, pl, L, ws, &p);
  if (rc != SPARC_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the array keeps the previous call's contents: its flag words, laid out for another shape,
  // could alias this launch's, so they start from zero on every call (a memset, no allocation)
  const cudaError_t e = cudaMemsetAsync(ws + L.flags, 0, L.agg - L.flags, s);
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  return launch_forward(pl, p, s);
}

int sparc_read_status(const void* workspace, unsigned* status, void* stream) {
  if (workspace == nullptr || status == nullptr) { set_err("null pointer"); return SPARC_ERR_ARG; }
  const LaunchState* ls = static_cast<const LaunchState*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status, &ls->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  return SPARC_OK;
}

int sparc_clear_status(void* workspace, void* stream) {
  if (workspace == nullptr) { set_err("null pointer"); return SPARC_ERR_ARG; }
  LaunchState* ls = static_cast<LaunchState*>(workspace);
  cudaError_t e = cudaMemsetAsync(&ls->status, 0, sizeof(unsigned), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) { set_err(cudaGetErrorString(e)); return SPARC_ERR_LAUNCH; }
  return SPARC_OK;
}

}  // extern "C"
