// Real diagonal scan h_t = a_t h_{t-1} + b_t for B200 (sm_100a), forward and backward.
//
// Tile = (chunk c, batch row b, channel block). One CTA per tile, one thread per 4-byte
// column group (one float32 channel or two bfloat16 channels), so every warp load is a
// fully used 128-byte line. Persistent CTAs take tiles in chunk-major ticket order and pass
// chunk carries by decoupled lookback (see common.cuh); the forward's inclusive states are
// the saved carries the backward replays from, so the backward reads a, b and grad_out once
// and never needs the forward output.
//
// Parity targets (Botwwt/sparc): _real_forward / _real_chunk_* forward/scan.py:622-698,
// _real_backward / _real_reverse_chunk_* backward/scan.py:35-128 (grad_a = lambda_t h_{t-1},
// grad_b = lambda_t).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "sparc_b200.h"
#include "timing.cuh"

namespace sparc {

constexpr int kRealChunk = 16;
constexpr int kRealThreads = 256;

template <typename TIO, int V>
struct VecIo;
template <>
struct VecIo<float, 1> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[1]) { v[0] = __ldg(p); }
  static __device__ __forceinline__ void store(float* p, const float (&v)[1]) { *p = v[0]; }
};
template <>
struct VecIo<__nv_bfloat16, 1> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[1]) {
    v[0] = __bfloat162float(__ldg(p));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[1]) {
    *p = __float2bfloat16_rn(v[0]);
  }
};
template <>
struct VecIo<__nv_bfloat16, 2> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[2]) {
    const __nv_bfloat162 t = __ldg(reinterpret_cast<const __nv_bfloat162*>(p));
    const float2 f = __bfloat1622float2(t);
    v[0] = f.x;
    v[1] = f.y;
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[2]) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  }
};

struct RealParams {
  const void* a;
  const void* b;
  const void* g;       // backward only
  void* out;           // forward: out; backward: grad_a
  void* out2;          // backward: grad_b
  float* last;
  float* carry;        // forward inclusive states [B, chunks, D]
  LaunchState* ls;
  unsigned* flags;     // [tiles]
  float2* agg;         // [tiles, Dp]
  float* incl;         // backward inclusive [tiles, Dp]
  long long B, T, D;
  int chunks, nDB, Dp;
  long long tiles;
  unsigned max_spin;
  long long inject_unpublished;  // test hook: this forward tile never publishes (-1: none)
};

// Lookback over real affine maps out = A*in + B (one per channel). Returns the carry-in.
template <int V, typename InclFn>
__device__ __forceinline__ void real_lookback(const RealParams& p, unsigned epoch, long long ticket,
                                              long long dist, int steps_max, const float (&A)[V],
                                              const float (&Bv)[V], long long dp0, unsigned* s_state,
                                              InclFn pred_inclusive, float (&carry)[V], bool publish = true) {
  const int tid = threadIdx.x;
  long long pred = ticket - dist;
  if (tid == 0) s_state[0] = ld_acquire(p.flags + pred);
  __syncthreads();
  const unsigned st0 = s_state[0];
  const bool pred_ready = ((st0 >> 2) == (epoch & 0x3fffffffu)) && (st0 & 3u) == kFlagInclusive;
  if (!pred_ready && publish) {
#pragma unroll
    for (int v = 0; v < V; ++v) p.agg[ticket * p.Dp + dp0 + v] = make_float2(A[v], Bv[v]);
    __syncthreads();
    if (tid == 0) st_release(p.flags + ticket, make_flag(epoch, kFlagAggregate));
  }
  float accA[V], accB[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    accA[v] = 1.0f;
    accB[v] = 0.0f;
  }
  for (int j = 1;; ++j) {
    unsigned state;
    if (j == 1 && pred_ready) {
      state = kFlagInclusive;
    } else {
      if (tid == 0) {
        unsigned s = wait_flag(p.flags + pred, epoch, p.max_spin);
        if (s == 0u) atomicOr(&p.ls->status, kStatusTimeout);
        s_state[j & 1] = s;
      }
      __syncthreads();
      state = s_state[j & 1];
    }
    if (state == kFlagInclusive) {
      float h[V];
      pred_inclusive(j, h);
#pragma unroll
      for (int v = 0; v < V; ++v) carry[v] = fmaf(accA[v], h[v], accB[v]);
      return;
    }
    if (state != kFlagAggregate || j >= steps_max) {
#pragma unroll
      for (int v = 0; v < V; ++v) carry[v] = accB[v];
      return;
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const float2 ag = __ldcg(p.agg + pred * p.Dp + dp0 + v);
      accB[v] = fmaf(accA[v], ag.y, accB[v]);
      accA[v] *= ag.x;
    }
    pred -= dist;
  }
}

template <typename TIO, int V>
__global__ void __launch_bounds__(kRealThreads) real_fwd_kernel(const RealParams p) {
  constexpr int C = kRealChunk;
  __shared__ unsigned s_ticket;
  __shared__ unsigned s_state[2];
  const int tid = threadIdx.x;
  const unsigned epoch = *(volatile unsigned*)&p.ls->epoch;
  const long long B = p.B, T = p.T, D = p.D;
  const long long per_chunk = B * p.nDB;
  for (;;) {
    if (tid == 0) s_ticket = atomicAdd(&p.ls->ticket, 1u);
    __syncthreads();
    const long long ticket = s_ticket;
    __syncthreads();
    if (ticket >= p.tiles) break;
    const int c = (int)(ticket / per_chunk);
    const long long rem = ticket - (long long)c * per_chunk;
    const long long b = rem / p.nDB;
    const int db = (int)(rem - b * p.nDB);
    const long long dp0 = (long long)db * kRealThreads * V + (long long)tid * V;
    const bool active = dp0 < D;  // D % V == 0, so a vector is all in or all out
    const long long t0 = (long long)c * C;
    const int nvalid = (int)(T - t0 < C ? T - t0 : C);
    const long long base = (b * T + t0) * D + dp0;
    const TIO* pa = static_cast<const TIO*>(p.a) + base;
    const TIO* pb = static_cast<const TIO*>(p.b) + base;

    float a[C][V], bv[C][V];
    if (active && nvalid == C) {
      // full chunk: unguarded loads, all in flight together
#pragma unroll
      for (int t = 0; t < C; ++t) {
        VecIo<TIO, V>::load(pa + (long long)t * D, a[t]);
        VecIo<TIO, V>::load(pb + (long long)t * D, bv[t]);
      }
    } else {
#pragma unroll
      for (int t = 0; t < C; ++t) {
        if (active && t < nvalid) {
          VecIo<TIO, V>::load(pa + (long long)t * D, a[t]);
          VecIo<TIO, V>::load(pb + (long long)t * D, bv[t]);
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            a[t][v] = 1.0f;
            bv[t][v] = 0.0f;
          }
        }
      }
    }
    float P[V], Q[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      P[v] = 1.0f;
      Q[v] = 0.0f;
    }
#pragma unroll
    for (int t = 0; t < C; ++t) {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        Q[v] = fmaf(a[t][v], Q[v], bv[t][v]);
        P[v] *= a[t][v];
      }
    }
    float hin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) hin[v] = 0.0f;
    if (c > 0) {
      const float* carry = p.carry;
      const int chunks = p.chunks;
      real_lookback<V>(p, epoch, ticket, per_chunk, c, P, Q, dp0, s_state,
                       [&](int j, float (&h)[V]) {
#pragma unroll
                         for (int v = 0; v < V; ++v)
                           h[v] = active ? __ldcg(carry + (b * chunks + (c - j)) * D + dp0 + v) : 0.0f;
                       },
                       hin, ticket != p.inject_unpublished);
    }
    float hout[V];
#pragma unroll
    for (int v = 0; v < V; ++v) hout[v] = fmaf(P[v], hin[v], Q[v]);
    if (active) {
#pragma unroll
      for (int v = 0; v < V; ++v) p.carry[(b * p.chunks + c) * D + dp0 + v] = hout[v];
    }
    __syncthreads();  // thread 0's release store publishes what the barrier ordered before it
    if (tid == 0 && ticket != p.inject_unpublished) st_release(p.flags + ticket, make_flag(epoch, kFlagInclusive));

    TIO* po = static_cast<TIO*>(p.out) + base;
    float h[V];
#pragma unroll
    for (int v = 0; v < V; ++v) h[v] = hin[v];
#pragma unroll
    for (int t = 0; t < C; ++t) {
#pragma unroll
      for (int v = 0; v < V; ++v) h[v] = fmaf(a[t][v], h[v], bv[t][v]);
      if (active && t < nvalid) VecIo<TIO, V>::store(po + (long long)t * D, h);
    }
    if (c == p.chunks - 1 && p.last != nullptr && active) {
#pragma unroll
      for (int v = 0; v < V; ++v) p.last[b * D + dp0 + v] = hout[v];
    }
  }
  finish_launch(p.ls);
}

template <typename TIO, int V>
__global__ void __launch_bounds__(kRealThreads) real_bwd_kernel(const RealParams p) {
  constexpr int C = kRealChunk;
  __shared__ unsigned s_ticket;
  __shared__ unsigned s_state[2];
  const int tid = threadIdx.x;
  const unsigned epoch = *(volatile unsigned*)&p.ls->epoch;
  const long long B = p.B, T = p.T, D = p.D;
  const long long per_chunk = B * p.nDB;
  for (;;) {
    if (tid == 0) s_ticket = atomicAdd(&p.ls->ticket, 1u);
    __syncthreads();
    const long long ticket = s_ticket;
    __syncthreads();
    if (ticket >= p.tiles) break;
    const int c = p.chunks - 1 - (int)(ticket / per_chunk);
    const long long rem = ticket - (long long)(p.chunks - 1 - c) * per_chunk;
    const long long b = rem / p.nDB;
    const int db = (int)(rem - b * p.nDB);
    const long long dp0 = (long long)db * kRealThreads * V + (long long)tid * V;
    const bool active = dp0 < D;
    const long long t0 = (long long)c * C;
    const int nvalid = (int)(T - t0 < C ? T - t0 : C);
    const long long base = (b * T + t0) * D + dp0;
    const TIO* pa = static_cast<const TIO*>(p.a) + base;
    const TIO* pb = static_cast<const TIO*>(p.b) + base;
    const TIO* pg = static_cast<const TIO*>(p.g) + base;

    float a[C][V], h[C][V], g[C][V];
    float hin[V];
#pragma unroll
    for (int v = 0; v < V; ++v)
      hin[v] = (active && c > 0) ? p.carry[(b * p.chunks + c - 1) * D + dp0 + v] : 0.0f;
    {
      float hh[V];
#pragma unroll
      for (int v = 0; v < V; ++v) hh[v] = hin[v];
      if (active && nvalid == C) {
        // full chunk: unguarded loads, all in flight together
        float bt[C][V];
#pragma unroll
        for (int t = 0; t < C; ++t) {
          VecIo<TIO, V>::load(pa + (long long)t * D, a[t]);
          VecIo<TIO, V>::load(pb + (long long)t * D, bt[t]);
          VecIo<TIO, V>::load(pg + (long long)t * D, g[t]);
        }
#pragma unroll
        for (int t = 0; t < C; ++t) {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            hh[v] = fmaf(a[t][v], hh[v], bt[t][v]);
            h[t][v] = hh[v];
          }
        }
      } else {
#pragma unroll
        for (int t = 0; t < C; ++t) {
          float bt[V];
          if (active && t < nvalid) {
            VecIo<TIO, V>::load(pa + (long long)t * D, a[t]);
            VecIo<TIO, V>::load(pb + (long long)t * D, bt);
            VecIo<TIO, V>::load(pg + (long long)t * D, g[t]);
          } else {
#pragma unroll
            for (int v = 0; v < V; ++v) {
              a[t][v] = 1.0f;
              bt[v] = 0.0f;
              g[t][v] = 0.0f;
            }
          }
#pragma unroll
          for (int v = 0; v < V; ++v) {
            hh[v] = fmaf(a[t][v], hh[v], bt[v]);
            h[t][v] = hh[v];
          }
        }
      }
    }
    // local reverse adjoint from zero: kappa_out = P * kappa_in + Qr
    float P[V], Qr[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      P[v] = 1.0f;
      Qr[v] = 0.0f;
    }
#pragma unroll
    for (int t = C - 1; t >= 0; --t) {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        Qr[v] = (Qr[v] + g[t][v]) * a[t][v];
        P[v] *= a[t][v];
      }
    }
    float kin[V];
#pragma unroll
    for (int v = 0; v < V; ++v) kin[v] = 0.0f;
    if (c < p.chunks - 1) {
      const float* incl = p.incl;
      const int Dp = p.Dp;
      real_lookback<V>(p, epoch, ticket, per_chunk, p.chunks - 1 - c, P, Qr, dp0, s_state,
                       [&](int j, float (&hv)[V]) {
#pragma unroll
                         for (int v = 0; v < V; ++v)
                           hv[v] = active ? __ldcg(incl + (ticket - j * per_chunk) * Dp + dp0 + v) : 0.0f;
                       },
                       kin);
    }
    if (active) {
#pragma unroll
      for (int v = 0; v < V; ++v) p.incl[ticket * p.Dp + dp0 + v] = fmaf(P[v], kin[v], Qr[v]);
    }
    __syncthreads();  // thread 0's release store publishes what the barrier ordered before it
    if (tid == 0) st_release(p.flags + ticket, make_flag(epoch, kFlagInclusive));

    TIO* pga = static_cast<TIO*>(p.out) + base;
    TIO* pgb = static_cast<TIO*>(p.out2) + base;
    float lam[V];
#pragma unroll
    for (int v = 0; v < V; ++v) lam[v] = kin[v];
#pragma unroll
    for (int t = C - 1; t >= 0; --t) {
      float ga[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        lam[v] += g[t][v];
        ga[v] = lam[v] * (t > 0 ? h[t - 1][v] : hin[v]);
      }
      if (active && t < nvalid) {
        VecIo<TIO, V>::store(pga + (long long)t * D, ga);
        VecIo<TIO, V>::store(pgb + (long long)t * D, lam);
      }
#pragma unroll
      for (int v = 0; v < V; ++v) lam[v] *= a[t][v];
    }
  }
  finish_launch(p.ls);
}

struct RealPlan {
  int V, nDB, Dp, chunks;
  long long tiles;
  int grid_fwd, grid_bwd;
};

template <typename K>
static int resident_blocks(K kernel) {
  int dev = 0, sms = 0, per = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, kRealThreads, 0) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return per * sms;
}

static int real_plan(long long B, long long T, long long D, int dtype, RealPlan* pl) {
  if (B <= 0 || T <= 0 || D <= 0) return fail(SPARC_ERR_SHAPE, "batch, length and channels must be positive");
  if (dtype != SPARC_DTYPE_F32 && dtype != SPARC_DTYPE_BF16) return fail(SPARC_ERR_DTYPE, "unsupported dtype");
  pl->V = (dtype == SPARC_DTYPE_BF16 && D % 2 == 0) ? 2 : 1;
  const long long per_cta = (long long)kRealThreads * pl->V;
  pl->nDB = (int)((D + per_cta - 1) / per_cta);
  pl->Dp = (int)(pl->nDB * per_cta);
  pl->chunks = (int)((T + kRealChunk - 1) / kRealChunk);
  pl->tiles = B * pl->chunks * (long long)pl->nDB;
  if (pl->tiles >= (1LL << 31)) return fail(SPARC_ERR_SHAPE, "too many tiles");
  int gf, gb;
  if (dtype == SPARC_DTYPE_F32) {
    gf = resident_blocks(real_fwd_kernel<float, 1>);
    gb = resident_blocks(real_bwd_kernel<float, 1>);
  } else if (pl->V == 2) {
    gf = resident_blocks(real_fwd_kernel<__nv_bfloat16, 2>);
    gb = resident_blocks(real_bwd_kernel<__nv_bfloat16, 2>);
  } else {
    gf = resident_blocks(real_fwd_kernel<__nv_bfloat16, 1>);
    gb = resident_blocks(real_bwd_kernel<__nv_bfloat16, 1>);
  }
  if (gf <= 0 || gb <= 0) return fail(SPARC_ERR_LAUNCH, "occupancy query failed");
  pl->grid_fwd = (int)std::min<long long>(gf, pl->tiles);
  pl->grid_bwd = (int)std::min<long long>(gb, pl->tiles);
  return SPARC_OK;
}

struct RealWs {
  size_t flags, agg, incl, total;
};

static RealWs real_ws(const RealPlan& pl) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  RealWs L;
  size_t off = al(sizeof(LaunchState));
  L.flags = off;
  off = al(off + (size_t)pl.tiles * sizeof(unsigned));
  L.agg = off;
  off = al(off + (size_t)pl.tiles * pl.Dp * sizeof(float2));
  L.incl = off;
  off = al(off + (size_t)pl.tiles * pl.Dp * sizeof(float));
  L.total = off;
  return L;
}

}  // namespace sparc

using namespace sparc;

extern "C" {

long long sparc_real_chunk_tokens(void) { return kRealChunk; }

long long sparc_real_carry_chunks(long long length) { return (length + kRealChunk - 1) / kRealChunk; }

size_t sparc_real_workspace_bytes(long long batch, long long length, long long channels, int dtype) {
  RealPlan pl;
  if (real_plan(batch, length, channels, dtype, &pl) != SPARC_OK) return 0;
  return real_ws(pl).total;
}

int sparc_real_scan_forward(const SparcRealFwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return fail(SPARC_ERR_ARG, "null args");
  if (!a->a || !a->b || !a->out || !a->carry) return fail(SPARC_ERR_ARG, "null tensor pointer");
  RealPlan pl;
  int rc = real_plan(a->batch, a->length, a->channels, a->dtype, &pl);
  if (rc != SPARC_OK) return rc;
  const RealWs L = real_ws(pl);
  if (a->workspace == nullptr || a->workspace_bytes < L.total) return fail(SPARC_ERR_WORKSPACE, "workspace too small");
  char* ws = static_cast<char*>(a->workspace);
  RealParams p{};
  p.a = a->a;
  p.b = a->b;
  p.out = a->out;
  p.last = a->last;
  p.carry = a->carry;
  p.ls = reinterpret_cast<LaunchState*>(ws);
  p.flags = reinterpret_cast<unsigned*>(ws + L.flags);
  p.agg = reinterpret_cast<float2*>(ws + L.agg);
  p.incl = reinterpret_cast<float*>(ws + L.incl);
  p.B = a->batch;
  p.T = a->length;
  p.D = a->channels;
  p.chunks = pl.chunks;
  p.nDB = pl.nDB;
  p.Dp = pl.Dp;
  p.tiles = pl.tiles;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 20);
  p.inject_unpublished = a->inject_enable ? a->inject_tile : -1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TimedLaunch tl(kTimeRealFwd, s);
  if (a->dtype == SPARC_DTYPE_F32) real_fwd_kernel<float, 1><<<pl.grid_fwd, kRealThreads, 0, s>>>(p);
  else if (pl.V == 2) real_fwd_kernel<__nv_bfloat16, 2><<<pl.grid_fwd, kRealThreads, 0, s>>>(p);
  else real_fwd_kernel<__nv_bfloat16, 1><<<pl.grid_fwd, kRealThreads, 0, s>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPARC_OK : fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

int sparc_real_scan_backward(const SparcRealBwdArgs* a, void* stream) {
  NvtxRange nvtx(__func__);
  if (a == nullptr) return fail(SPARC_ERR_ARG, "null args");
  if (!a->a || !a->b || !a->grad_out || !a->carry || !a->grad_a || !a->grad_b)
    return fail(SPARC_ERR_ARG, "null tensor pointer");
  RealPlan pl;
  int rc = real_plan(a->batch, a->length, a->channels, a->dtype, &pl);
  if (rc != SPARC_OK) return rc;
  const RealWs L = real_ws(pl);
  if (a->workspace == nullptr || a->workspace_bytes < L.total) return fail(SPARC_ERR_WORKSPACE, "workspace too small");
  char* ws = static_cast<char*>(a->workspace);
  RealParams p{};
  p.a = a->a;
  p.b = a->b;
  p.g = a->grad_out;
  p.out = a->grad_a;
  p.out2 = a->grad_b;
  p.carry = const_cast<float*>(a->carry);
  p.ls = reinterpret_cast<LaunchState*>(ws);
  p.flags = reinterpret_cast<unsigned*>(ws + L.flags);
  p.agg = reinterpret_cast<float2*>(ws + L.agg);
  p.incl = reinterpret_cast<float*>(ws + L.incl);
  p.B = a->batch;
  p.T = a->length;
  p.D = a->channels;
  p.chunks = pl.chunks;
  p.nDB = pl.nDB;
  p.Dp = pl.Dp;
  p.tiles = pl.tiles;
  p.max_spin = a->max_spin ? a->max_spin : (1u << 20);
  p.inject_unpublished = -1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TimedLaunch tl(kTimeRealBwd, s);
  if (a->dtype == SPARC_DTYPE_F32) real_bwd_kernel<float, 1><<<pl.grid_bwd, kRealThreads, 0, s>>>(p);
  else if (pl.V == 2) real_bwd_kernel<__nv_bfloat16, 2><<<pl.grid_bwd, kRealThreads, 0, s>>>(p);
  else real_bwd_kernel<__nv_bfloat16, 1><<<pl.grid_bwd, kRealThreads, 0, s>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPARC_OK : fail(SPARC_ERR_LAUNCH, cudaGetErrorString(e));
}

}  // extern "C"
