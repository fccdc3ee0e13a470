// SPARC mixer forward kernel (included by mixer.cu, which holds the shared helpers).
//
// One thread-block cluster of G CTAs processes a tile (batch row b, chunk of C tokens, all M
// modes); CTA g owns modes [g*256, g*256+256), two adjacent modes per thread (vectorised
// bf16x2 / float2 I/O, two independent recurrences per thread). The x tile of the CTA's
// columns (C rows x (256 real + 256 imaginary) values) is brought into shared memory by TMA
// bulk copies on an mbarrier (plain loads replace the copies when the shapes are not 16-byte
// aligned). Clusters take tiles from a ticket counter, and a cluster takes its next ticket
// only when it is ready to start that tile: a ticket held but not started would stall every
// successor tile's lookback behind it. (Prefetching the next tile's copy into a second buffer
// was measured slower: the extra shared memory costs a resident CTA per SM.)
//
// Per tile: control projections of the C tokens (warp transpose-reduce, shared memory, then
// distributed shared memory across the cluster), then the recurrence. If the predecessor
// tile's carry is already published the recurrence runs in one pass; otherwise pass 1 keeps
// the transitions and writes (or write gains) in shared memory, the decoupled lookback
// resolves the carry, and pass 2 replays from shared memory.

// (included inside namespace sparc)

constexpr int kFwdThreads = 128;
constexpr int kFwdModes = 2 * kFwdThreads;  // modes per CTA

template <typename TIO, int C, bool kFast>
struct FwdSmem {
  TIO x[1][C][2][kFwdModes];                         // [buffer][token][re|im][mode]
  float2 a[C][kFwdModes];                            // slow path: transitions
  float w[C][kFwdModes * (kFast ? 1 : 2)];           // slow path: gains (bf16) or writes (fp32)
  float4 ctl[C];                                     // E, delta, tau0, tau1 per token
  float part[2][2 * C];                              // this CTA's projection partials (peers read)
  float warp_part[kFwdThreads / 32][2 * C];
  unsigned long long bar[1];
  long long ring[2];                                 // tickets, by tile parity
  unsigned win[2];
  unsigned pred;
};

struct FwdParams {
  const void* x;
  void* y;
  MixerParamPtrs pp;
  const float* h0_r;
  const float* h0_i;
  float* last_r;
  float* last_i;
  float2* carry;  // [B, chunks, M]
  LaunchState* ls;
  unsigned* flags;
  float4* agg;
  long long B, T;
  int W, M, chunks;
  long long tiles;
  unsigned max_spin;
  int deterministic;
  int use_tma;
  long long inject_unpublished;
};

template <typename TIO> struct Pair;
template <> struct Pair<float> {
  static __device__ __forceinline__ float2 load(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void store(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 load(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
  }
};

// Store the relu'd pair of states of modes (m, m+1) for one token row.
template <typename TIO, bool kVec>
__device__ __forceinline__ void store_y_pair(TIO* row, int M, int m, bool a0, bool a1, float2 h0, float2 h1) {
  if (kVec) {
    if (a1) {
      Pair<TIO>::store(row + m, fmaxf(h0.x, 0.0f), fmaxf(h1.x, 0.0f));
      Pair<TIO>::store(row + M + m, fmaxf(h0.y, 0.0f), fmaxf(h1.y, 0.0f));
      return;
    }
  }
  if (a0) {
    Io<TIO>::store(row + m, fmaxf(h0.x, 0.0f));
    Io<TIO>::store(row + M + m, fmaxf(h0.y, 0.0f));
  }
  if (a1) {
    Io<TIO>::store(row + m + 1, fmaxf(h1.x, 0.0f));
    Io<TIO>::store(row + M + m + 1, fmaxf(h1.y, 0.0f));
  }
}

// Copy (or load) the CTA's columns of x rows t0..t0+C-1 into buffer `buf`.
template <typename TIO, int C>
__device__ __forceinline__ void fetch_x_tile(const FwdParams& p, TIO (*dst)[2][kFwdModes],
                                             unsigned long long* bar, long long ticket, int g) {
  const long long b = ticket % p.B;
  const long long t0 = (long long)(ticket / p.B) * C;
  const int nvalid = (int)(p.T - t0 < C ? p.T - t0 : C);
  const int mbase = g * kFwdModes;
  const int ncols = min(kFwdModes, p.M - mbase);
  const TIO* src = static_cast<const TIO*>(p.x) + (b * p.T + t0) * p.W + mbase;
  if (p.use_tma) {
    if (threadIdx.x < 32) {  // warp 0: lane 0 sets the byte count, lane t copies row t
      const unsigned bytes = (unsigned)(ncols * sizeof(TIO));
      if (threadIdx.x == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, bytes * 2u * (unsigned)nvalid);
      }
      __syncwarp();
      for (int t = threadIdx.x; t < nvalid; t += 32) {
        bulk_copy_g2s(&dst[t][0][0], src + (long long)t * p.W, bytes, bar);
        bulk_copy_g2s(&dst[t][1][0], src + (long long)t * p.W + p.M, bytes, bar);
      }
    }
  } else {
    for (int i = threadIdx.x; i < nvalid * 2 * ncols; i += kFwdThreads) {
      const int t = i / (2 * ncols), r = i - t * 2 * ncols, half = r / ncols, mm = r - half * ncols;
      dst[t][half][mm] = src[(long long)t * p.W + half * p.M + mm];
    }
  }
}

template <typename TIO, int C, bool kFast, bool kVec>
__global__ void __launch_bounds__(kFwdThreads) mixer_fwd_kernel(const FwdParams p) {
  constexpr int NW = kFwdThreads / 32;
  cg::cluster_group cluster = cg::this_cluster();
  const int g = (int)cluster.block_rank();
  const int G = (int)cluster.num_blocks();
  const int tid = threadIdx.x;
  const int M = p.M, W = p.W;
  const int m0 = g * kFwdModes + 2 * tid;  // this thread's modes: m0, m0 + 1
  const bool act0 = m0 < M, act1 = m0 + 1 < M;
  const long long B = p.B, T = p.T;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  FwdSmem<TIO, C, kFast>& S = *reinterpret_cast<FwdSmem<TIO, C, kFast>*>(smem_raw);

  const ModeConst mc0 = load_mode(p.pp, m0, M, act0);
  const ModeConst mc1 = load_mode(p.pp, m0 + 1, M, act1);
  const float bias0 = p.pp.phase_dir[W], bias1 = p.pp.radial_dir[W];
  LookbackCtx lc{p.ls, p.flags, p.agg, *(volatile unsigned*)&p.ls->epoch, p.max_spin, G, G * kFwdModes, B,
                 p.deterministic != 0};

  // zero the x buffer once: columns past M are never copied and must read as zeros
  {
    unsigned* xs = reinterpret_cast<unsigned*>(&S.x[0][0][0][0]);
    for (int i = tid; i < (int)(sizeof(S.x) / 4); i += kFwdThreads) xs[i] = 0u;
  }
  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init_fence();
  }
  __syncthreads();
  bool timed_out = false;

  for (int it = 0;; ++it) {
    const int par = it & 1;
    if (tid == 0 && g == 0) S.ring[par] = atomicAdd(&p.ls->ticket, 1u);
    cluster.sync();  // also: every peer is done with the previous tile's shared data
    if (tid == 0 && g != 0) S.ring[par] = *cluster.map_shared_rank(&S.ring[par], 0);
    __syncthreads();
    const long long ticket = S.ring[par];
    if (ticket >= p.tiles) break;
    fetch_x_tile<TIO, C>(p, S.x[0], &S.bar[0], ticket, g);
    const int buf = par;
    const long long b = ticket % B;
    const int c = (int)(ticket / B);
    const long long t0 = (long long)c * C;
    const int nvalid = (int)(T - t0 < C ? T - t0 : C);
    if (tid == 0) S.pred = c > 0 ? ld_acquire(p.flags + (ticket - B) * G + g) : 0u;
    if (p.use_tma) {
      if (!mbar_wait(&S.bar[0], (unsigned)par, p.max_spin << 4)) timed_out = true;
    } else {
      __syncthreads();
    }
    const TIO(*xt)[2][kFwdModes] = S.x[0];

    // control projections: per-thread partials over its 4 columns, reduced over the cluster
    {
      float v[2 * C];
#pragma unroll
      for (int t = 0; t < C; ++t) {
        const float2 xr = Pair<TIO>::load(&xt[t][0][2 * tid]);
        const float2 xi = Pair<TIO>::load(&xt[t][1][2 * tid]);
        v[t] = fmaf(xr.x, mc0.d0r, fmaf(xi.x, mc0.d0i, fmaf(xr.y, mc1.d0r, xi.y * mc1.d0i)));
        v[C + t] = fmaf(xr.x, mc0.d1r, fmaf(xi.x, mc0.d1i, fmaf(xr.y, mc1.d1r, xi.y * mc1.d1i)));
      }
      constexpr int kShift = 5 - log2i<2 * C>();
      const int lane = tid & 31, warp = tid >> 5;
      const float total = transpose_reduce<2 * C>(v, lane);
      if ((lane & ((1 << kShift) - 1)) == 0) S.warp_part[warp][lane >> kShift] = total;
      __syncthreads();
      if (tid < 2 * C) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) sum += S.warp_part[w][tid];
        S.part[buf][tid] = sum;
      }
      cluster.sync();
      if (tid < C) {
        // the peers' partials are read together (their latencies overlap)
        float q0[8], q1[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if (r < G) {
            const float* peer = cluster.map_shared_rank(&S.part[buf][0], r);
            q0[r] = peer[tid];
            q1[r] = peer[C + tid];
          } else {
            q0[r] = q1[r] = 0.0f;
          }
        }
        float p0 = 0.0f, p1 = 0.0f;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          p0 += q0[r];
          p1 += q1[r];
        }
        const float tau0 = tanh_accurate(p0 + bias0);
        const float tau1 = tanh_accurate(p1 + bias1);
        S.ctl[tid] = make_float4(expf(kLn16 * tau1), kHalfPi * tau0, tau0, tau1);
      }
      __syncthreads();
    }
    // the tile body, instantiated branch-free for full chunks (so the compiler can interleave
    // independent tokens) and with guards for the ragged last chunk
    auto tile_body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr int kU = kFull ? 4 : 1;  // partial unrolling keeps the kernel's code in the i-cache
      const unsigned pst = S.pred;
      const bool pred_ready = c == 0 || (!lc.deterministic && ((pst >> 2) == (lc.epoch & 0x3fffffffu)) &&
                                         (pst & 3u) == kFlagInclusive);
      const bool publish = ticket != p.inject_unpublished;
      TIO* yrow = static_cast<TIO*>(p.y) + (b * T + t0) * W;
      float2 hout0, hout1;
      if (pred_ready) {
        float2 h0 = make_float2(0.0f, 0.0f), h1 = make_float2(0.0f, 0.0f);
        if (c > 0) {
          const float2* cp = p.carry + (b * p.chunks + (c - 1)) * M + m0;
          if (act0) h0 = __ldcg(cp);
          if (act1) h1 = __ldcg(cp + 1);
        } else if (p.h0_r != nullptr) {
          if (act0) h0 = make_float2(p.h0_r[b * M + m0], p.h0_i[b * M + m0]);
          if (act1) h1 = make_float2(p.h0_r[b * M + m0 + 1], p.h0_i[b * M + m0 + 1]);
        }
  #pragma unroll kU
        for (int t = 0; t < C; ++t) {
          if (kFull || t < nvalid) {
            const float4 k4 = S.ctl[t];
            const float2 xr = Pair<TIO>::load(&xt[t][0][2 * tid]);
            const float2 xi = Pair<TIO>::load(&xt[t][1][2 * tid]);
            const TokenCoef k0 = token_coef<kFast>(mc0, k4.x, k4.y, k4.z, k4.w);
            const TokenCoef k1 = token_coef<kFast>(mc1, k4.x, k4.y, k4.z, k4.w);
            h0 = cfma(k0.a, h0, make_float2(k0.gain * tanh_t<kFast>(xr.x), k0.gain * tanh_t<kFast>(xi.x)));
            h1 = cfma(k1.a, h1, make_float2(k1.gain * tanh_t<kFast>(xr.y), k1.gain * tanh_t<kFast>(xi.y)));
            store_y_pair<TIO, kVec>(yrow + (long long)t * W, M, m0, act0, act1, h0, h1);
          }
        }
        hout0 = h0;
        hout1 = h1;
        if (publish) {
          float2* cp = p.carry + (b * p.chunks + c) * M + m0;
          if (act0) cp[0] = hout0;
          if (act1) cp[1] = hout1;
          publish_flag(p.flags + ticket * G + g, make_flag(lc.epoch, kFlagInclusive));
        }
      } else {
        float2 P0 = make_float2(1.0f, 0.0f), Q0 = make_float2(0.0f, 0.0f);
        float2 P1 = P0, Q1 = Q0;
  #pragma unroll kU
        for (int t = 0; t < C; ++t) {
          float2 a0 = make_float2(1.0f, 0.0f), a1 = a0, b0 = make_float2(0.0f, 0.0f), b1 = b0;
          float g0 = 0.0f, g1 = 0.0f;
          if (kFull || t < nvalid) {
            const float4 k4 = S.ctl[t];
            const float2 xr = Pair<TIO>::load(&xt[t][0][2 * tid]);
            const float2 xi = Pair<TIO>::load(&xt[t][1][2 * tid]);
            const TokenCoef k0 = token_coef<kFast>(mc0, k4.x, k4.y, k4.z, k4.w);
            const TokenCoef k1 = token_coef<kFast>(mc1, k4.x, k4.y, k4.z, k4.w);
            a0 = k0.a;
            a1 = k1.a;
            g0 = k0.gain;
            g1 = k1.gain;
            b0 = make_float2(g0 * tanh_t<kFast>(xr.x), g0 * tanh_t<kFast>(xi.x));
            b1 = make_float2(g1 * tanh_t<kFast>(xr.y), g1 * tanh_t<kFast>(xi.y));
          }
          *reinterpret_cast<float4*>(&S.a[t][2 * tid]) = make_float4(a0.x, a0.y, a1.x, a1.y);
          if constexpr (kFast) {
            *reinterpret_cast<float2*>(&S.w[t][2 * tid]) = make_float2(g0, g1);
          } else {
            *reinterpret_cast<float4*>(&S.w[t][4 * tid]) = make_float4(b0.x, b0.y, b1.x, b1.y);
          }
          Q0 = cfma(a0, Q0, b0);
          P0 = cmul(a0, P0);
          Q1 = cfma(a1, Q1, b1);
          P1 = cmul(a1, P1);
        }
        const float2* carry = p.carry;
        const int chunks = p.chunks;
        float2 A[2] = {P0, P1}, Bv[2] = {Q0, Q1}, hin[2];
        lookback<2>(lc, ticket, g, c, A, Bv, publish, pst, S.win, m0,
                    [&](int j, float2 (&h)[2]) {
                      const float2* cp = carry + (b * chunks + (c - j)) * M + m0;
                      h[0] = act0 ? __ldcg(cp) : make_float2(0.0f, 0.0f);
                      h[1] = act1 ? __ldcg(cp + 1) : make_float2(0.0f, 0.0f);
                    },
                    hin);
        hout0 = cfma(P0, hin[0], Q0);
        hout1 = cfma(P1, hin[1], Q1);
        if (publish) {
          float2* cp = p.carry + (b * p.chunks + c) * M + m0;
          if (act0) cp[0] = hout0;
          if (act1) cp[1] = hout1;
          publish_flag(p.flags + ticket * G + g, make_flag(lc.epoch, kFlagInclusive));
        }
        float2 h0 = hin[0], h1 = hin[1];
  #pragma unroll kU
        for (int t = 0; t < C; ++t) {
          if (kFull || t < nvalid) {
            const float4 a4 = *reinterpret_cast<const float4*>(&S.a[t][2 * tid]);
            float2 b0, b1;
            if constexpr (kFast) {
              const float2 gg = *reinterpret_cast<const float2*>(&S.w[t][2 * tid]);
              const float2 xr = Pair<TIO>::load(&xt[t][0][2 * tid]);
              const float2 xi = Pair<TIO>::load(&xt[t][1][2 * tid]);
              b0 = make_float2(gg.x * tanh_t<kFast>(xr.x), gg.x * tanh_t<kFast>(xi.x));
              b1 = make_float2(gg.y * tanh_t<kFast>(xr.y), gg.y * tanh_t<kFast>(xi.y));
            } else {
              const float4 w4 = *reinterpret_cast<const float4*>(&S.w[t][4 * tid]);
              b0 = make_float2(w4.x, w4.y);
              b1 = make_float2(w4.z, w4.w);
            }
            h0 = cfma(make_float2(a4.x, a4.y), h0, b0);
            h1 = cfma(make_float2(a4.z, a4.w), h1, b1);
            store_y_pair<TIO, kVec>(yrow + (long long)t * W, M, m0, act0, act1, h0, h1);
          }
        }
      }
      if (c == p.chunks - 1 && p.last_r != nullptr) {
        if (act0) {
          p.last_r[b * M + m0] = hout0.x;
          p.last_i[b * M + m0] = hout0.y;
        }
        if (act1) {
          p.last_r[b * M + m0 + 1] = hout1.x;
          p.last_i[b * M + m0 + 1] = hout1.y;
        }
      }
    };
    if (nvalid == C) tile_body(std::true_type{});
    else tile_body(std::false_type{});
    __syncthreads();  // the buffer and the shared arrays are free for the next tile
  }
  if (timed_out && tid == 0) atomicOr(&p.ls->status, kStatusTimeout);
  cluster.sync();  // no CTA leaves while a peer may still read its shared memory
  finish_launch(p.ls);
}

