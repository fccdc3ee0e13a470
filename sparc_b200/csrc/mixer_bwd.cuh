// SPARC mixer backward kernels (included by mixer.cu, inside namespace sparc). Three launches
// plus the fixed-order parameter-gradient reduction:
//
//   mixer_bwd_summary_kernel  per tile: the relu-masked output gradient g_t = dy_t * [y_t > 0]
//                             (y is the forward output, so no state replay is needed here), and
//                             the chunk's reverse aggregate: with lambda_t = g_t + conj(a_{t+1})
//                             lambda_{t+1} the adjoint, the carry leaving the chunk towards
//                             earlier tokens is conj(a_t0) lambda_t0 = conj(P) k_in + q, with
//                             P = prod a_t and q the same walk from k_in = 0.
//   mixer_carry_scan_kernel   (mixer.cu) the same scan as the forward's, from the last chunk
//                             backwards: the adjoint carry leaving every chunk.
//   mixer_bwd_grad_kernel     per tile (cluster of G CTAs): pass 0 replays the states from the
//                             forward's chunk carry into shared memory and masks dy; pass B
//                             walks the true adjoint backwards with every gradient: transition
//                             (dEta, dDelta per token, dNu, dTheta per mode), write path (dx of
//                             the content, dEta, dDelta, dNu, write-gain / response gradients);
//                             the write-path dx waits in the state slots the reverse walk has
//                             consumed. dEta, dDelta are summed over all modes (warp
//                             transpose-reduce per group of tokens during the walk, then shared
//                             and distributed shared memory) into the controller gradients dp0,
//                             dp1, which finish dx and the direction gradients.
// One mode per thread, 256 threads per CTA (the tiles' shared memory then serves twice the warps
// of a two-modes-per-thread layout). Per-mode parameter gradients accumulate in float64 per
// cluster; mixer_reduce_kernel sums the clusters in a fixed order. The token controls come from
// the forward (saved per token).

// (included inside namespace sparc)

constexpr int kBwdThreads = 256;
constexpr int kBwdModes = kBwdThreads;  // one mode per thread
constexpr int kBwdWarps = kBwdThreads / 32;
constexpr int kPartModes = 9;  // nu, theta (sum of phase grads), wlg, wpr, wrr, D0r, D0i, D1r, D1i
constexpr int kGroup = 4;      // tokens per unrolled group of the reverse walk

template <typename TIO, int C>
struct RsumSmem {
  TIO dy[2][C][2][kBwdModes];
  TIO y[2][C][2][kBwdModes];
  float4 ctl[2][C];
  unsigned long long bar[2];
};

template <typename TIO, int C>
struct GradSmem {
  TIO x[C][2][kBwdModes];
  TIO dy[C][2][kBwdModes];     // masked by the relu in pass 0
  float2 h[C][kBwdModes];      // replayed states, then the write-path dx (pass B)
  float2 hin[kBwdModes];       // state entering the chunk
  float2 kin[kBwdModes];       // adjoint carry entering the chunk from the later chunks
  float4 ctl[C];               // E, delta, tau0, tau1
  float2 dp[C];                // controller gradients dp0, dp1
  float tot[2 * C];            // cluster totals of dEta / dDelta
  float part_grad[2][2 * C];   // dEta / dDelta CTA partials (peers read), by tile parity
  float warp_part[kBwdWarps][2 * C];
  unsigned long long bar;
};

struct BwdParams {
  CUtensorMap map_x;     // x, y, dy as [B*T rows][re|im][M], box {256, 2, C} (when use_tma)
  CUtensorMap map_y;
  CUtensorMap map_dy;
  const void* x;
  const void* y;
  const void* dy;
  void* dx;
  MixerParamPtrs pp;
  const float* h0_r;
  const float* h0_i;
  const float* glast_r;
  const float* glast_i;
  const float4* ctl;     // [B, T] forward token controls
  const float2* carry;   // [B, chunks, M] forward inclusive states
  const float2* kout;    // [B, chunks, M] adjoint carry leaving each chunk (scan output)
  float4* agg;           // [B, chunks, Mp] reverse aggregates (summary output)
  double* part;          // [clusters][kPartModes][Mp] then [clusters][2] bias partials
  LaunchState* ls;
  long long B, T;
  int W, M, Mp, chunks;
  long long tiles;
  unsigned max_spin;
  int use_tma;
};

// ------------------------------------------------------------------------------ reverse summary
template <typename TIO, int C, bool kFast>
__global__ void __launch_bounds__(kBwdThreads) mixer_bwd_summary_kernel(const __grid_constant__ BwdParams p) {
  const int g = blockIdx.x;
  const int tid = threadIdx.x;
  const int M = p.M, W = p.W;
  const int mbase = g * kBwdModes;
  const int m = mbase + tid;
  const bool act = m < M;
  const long long B = p.B, T = p.T;
  const long long k0 = blockIdx.y, nk = gridDim.y;
  pdl_wait();  // the first launch of the backward: dy comes from the previous kernel

  extern __shared__ __align__(128) unsigned char smem_raw[];
  RsumSmem<TIO, C>& S = *reinterpret_cast<RsumSmem<TIO, C>*>(smem_raw);

  const ModeConst mc = load_mode(p.pp, m, M, act);

  {  // columns past M are never copied: zero dy there (the walk then stays at zero)
    unsigned* z = reinterpret_cast<unsigned*>(&S.dy[0][0][0][0]);
    for (int i = tid; i < (int)(sizeof(S.dy) / 4); i += kBwdThreads) z[i] = 0u;
  }
  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init(&S.bar[1], 1);
    mbar_init_fence();
  }
  __syncthreads();

  auto issue = [&](long long i, int buf) {
    const TileRef r = tile_ref(i, B, T, C);
    const long long row0 = (r.b * T + r.t0) * W;
    const TIO* dsrc = static_cast<const TIO*>(p.dy) + row0;
    const TIO* ysrc = static_cast<const TIO*>(p.y) + row0;
    const float4* csrc = p.ctl + r.b * T + r.t0;
    if (p.use_tma) {
      if (tid == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.bar[buf], 2u * act_box_bytes<TIO, C, kBwdModes>() + 16u * (unsigned)r.nvalid);
        const int row = (int)(r.b * T + r.t0);
        tma_load_3d(&S.dy[buf][0][0][0], &p.map_dy, mbase, 0, row, &S.bar[buf]);
        tma_load_3d(&S.y[buf][0][0][0], &p.map_y, mbase, 0, row, &S.bar[buf]);
        bulk_copy_g2s(&S.ctl[buf][0], csrc, 16u * (unsigned)r.nvalid, &S.bar[buf]);
      }
    } else {
      load_act_rows<TIO, kBwdModes>(dsrc, W, M, mbase, r.nvalid, S.dy[buf], kBwdThreads);
      load_act_rows<TIO, kBwdModes>(ysrc, W, M, mbase, r.nvalid, S.y[buf], kBwdThreads);
      for (int t = tid; t < r.nvalid; t += kBwdThreads) S.ctl[buf][t] = csrc[t];
    }
  };
  if (k0 < p.tiles) issue(k0, 0);
  bool timed_out = false;

  for (long long n = 0;; ++n) {
    const long long i = k0 + n * nk;
    if (i >= p.tiles) break;
    const int buf = (int)(n & 1);
    if (i + nk < p.tiles) issue(i + nk, buf ^ 1);
    const TileRef r = tile_ref(i, B, T, C);
    if (p.use_tma) {
      if (!mbar_wait(&S.bar[buf], (unsigned)((n >> 1) & 1), p.max_spin << 4)) timed_out = true;
    } else {
      __syncthreads();
    }
    const TIO(*dyt)[2][kBwdModes] = S.dy[buf];
    const TIO(*yt)[2][kBwdModes] = S.y[buf];
    const float4* ctl = S.ctl[buf];
    auto body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr int kU = kFull ? token_unroll<C>() : 1;
      float2 q = make_float2(0.0f, 0.0f);
      float2 P = make_float2(1.0f, 0.0f);
#pragma unroll kU
      for (int t = C - 1; t >= 0; --t) {
        if (kFull || t < r.nvalid) {
          const float4 k4 = ctl[t];
          const float gr = to_float(dyt[t][0][tid]);
          const float gi = to_float(dyt[t][1][tid]);
          const float yr = to_float(yt[t][0][tid]);
          const float yi = to_float(yt[t][1][tid]);
          q.x += yr > 0.0f ? gr : 0.0f;
          q.y += yi > 0.0f ? gi : 0.0f;
          const float2 a = token_transition<kFast>(mc, k4.x, k4.y);
          q = make_float2(fmaf(a.x, q.x, a.y * q.y), fmaf(a.x, q.y, -a.y * q.x));
          P = cmul(a, P);
        }
      }
      if (act) __stcg(p.agg + (r.b * p.chunks + r.c) * (long long)p.Mp + m, make_float4(P.x, -P.y, q.x, q.y));
    };
    if (r.nvalid == C) body(std::true_type{});
    else body(std::false_type{});
    __syncthreads();
  }
  if (timed_out) atomicOr(&p.ls->status, kStatusTimeout);
}

// ------------------------------------------------------------------------------ gradients
// Gradient contributions of one (token, mode): updates the adjoint lam in place (to conj(a)
// lam) and returns the write-path dx of the content (real, imaginary); adds the token's dEta /
// dDelta contributions to ve / vd and the per-mode parameter terms to fa.
template <bool kFast>
__device__ __forceinline__ float2 grad_step(const ModeConst& mc, const float4 k4, float2& lam, float2 pv,
                                            float cx, float cy, float& ve, float& vd, float (&fa)[5]) {
  const TokenCoef k = token_coef<kFast>(mc, k4.x, k4.y, k4.z, k4.w);
  const float ar = k.a.x, ai = k.a.y;
  const float gar = fmaf(lam.x, pv.x, lam.y * pv.y);
  const float gai = fmaf(lam.y, pv.x, -lam.x * pv.y);
  const float pg = fmaf(gai, ar, -gar * ai);
  const float radial = k.z * fmaf(k.rho * k4.y, pg, -fmaf(gar, ar, gai * ai));
  const float dscan = pg - k.rho * pg;
  const float cr = tanh_t<kFast>(cx);
  const float ci = tanh_t<kFast>(cy);
  const float gg = k.gain * fmaf(lam.x, cr, lam.y * ci);
  const float gq = gg * fmaf(-0.5f, k.gate, 1.0f);
  const float dyn = k.z * k.rho * k.rho * rcp_approx(k.num);
  ve = radial + fmaf(gg, dyn, gq * mc.wrr * kInvLn16);
  vd = fmaf(gq * mc.wpr, kInvHalfPi, dscan);
  fa[0] += radial + gg * (dyn - mc.stat);
  fa[1] += pg;
  fa[2] += gg;
  fa[3] = fmaf(gq, k4.z, fa[3]);
  fa[4] = fmaf(gq, k4.w, fa[4]);
  const float2 dxc = make_float2(lam.x * k.gain * fmaf(-cr, cr, 1.0f), lam.y * k.gain * fmaf(-ci, ci, 1.0f));
  lam = make_float2(fmaf(ar, lam.x, ai * lam.y), fmaf(ar, lam.y, -ai * lam.x));
  return dxc;
}

template <typename TIO, int C, bool kFast>
__global__ void __launch_bounds__(kBwdThreads) mixer_bwd_grad_kernel(const __grid_constant__ BwdParams p) {
  static_assert(C % kGroup == 0, "the reverse walk runs in groups of kGroup tokens");
  cg::cluster_group cluster = cg::this_cluster();
  const int g = (int)cluster.block_rank();
  const int G = (int)cluster.num_blocks();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = p.M, W = p.W;
  const int mbase = g * kBwdModes;
  const int m = mbase + tid;
  const int Mp = p.Mp;
  const bool act = m < M;
  const long long B = p.B, T = p.T;
  const int chunks = p.chunks;
  const int ncols = min(kBwdModes, M - mbase);
  const long long k0 = blockIdx.y, nk = gridDim.y;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  GradSmem<TIO, C>& S = *reinterpret_cast<GradSmem<TIO, C>*>(smem_raw);

  const ModeConst mc = load_mode(p.pp, m, M, act);

  {
    unsigned* z = reinterpret_cast<unsigned*>(&S.x[0][0][0]);
    for (int i = tid; i < (int)((sizeof(S.x) + sizeof(S.dy)) / 4); i += kBwdThreads) z[i] = 0u;
  }
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    mbar_init_fence();
  }
  __syncthreads();

  double acc[kPartModes];
#pragma unroll
  for (int q = 0; q < kPartModes; ++q) acc[q] = 0.0;
  double acc_b0 = 0.0, acc_b1 = 0.0;
  bool timed_out = false;
  pdl_wait();  // the adjoint carries (scan) are complete from here on

  for (long long n = 0;; ++n) {
    const long long i = k0 + n * nk;
    if (i >= p.tiles) break;
    const int par = (int)(n & 1);
    const TileRef r = tile_ref(i, B, T, C);
    const long long b = r.b;
    const int c = r.c;
    const long long row0 = (b * T + r.t0) * W;
    {
      const TIO* xs = static_cast<const TIO*>(p.x) + row0;
      const TIO* ds = static_cast<const TIO*>(p.dy) + row0;
      const float4* cs = p.ctl + b * T + r.t0;
      const float2* hs = c > 0 ? p.carry + (b * chunks + (c - 1)) * (long long)M + mbase : nullptr;
      const float2* ks = c < chunks - 1 ? p.kout + (b * chunks + (c + 1)) * (long long)M + mbase : nullptr;
      if (p.use_tma) {
        if (tid == 0) {
          fence_proxy_async_smem();
          unsigned bytes = 2u * act_box_bytes<TIO, C, kBwdModes>() + 16u * (unsigned)r.nvalid;
          if (hs != nullptr) bytes += (unsigned)ncols * 8u;
          if (ks != nullptr) bytes += (unsigned)ncols * 8u;
          mbar_arrive_expect_tx(&S.bar, bytes);
          const int row = (int)(b * T + r.t0);
          tma_load_3d(&S.x[0][0][0], &p.map_x, mbase, 0, row, &S.bar);
          tma_load_3d(&S.dy[0][0][0], &p.map_dy, mbase, 0, row, &S.bar);
          bulk_copy_g2s(&S.ctl[0], cs, 16u * (unsigned)r.nvalid, &S.bar);
          if (hs != nullptr) bulk_copy_g2s(&S.hin[0], hs, (unsigned)ncols * 8u, &S.bar);
          if (ks != nullptr) bulk_copy_g2s(&S.kin[0], ks, (unsigned)ncols * 8u, &S.bar);
        }
        if (!mbar_wait(&S.bar, (unsigned)par, p.max_spin << 4)) timed_out = true;
      } else {
        load_act_rows<TIO, kBwdModes>(xs, W, M, mbase, r.nvalid, S.x, kBwdThreads);
        load_act_rows<TIO, kBwdModes>(ds, W, M, mbase, r.nvalid, S.dy, kBwdThreads);
        for (int t = tid; t < r.nvalid; t += kBwdThreads) S.ctl[t] = cs[t];
        for (int mm = tid; mm < ncols; mm += kBwdThreads) {
          if (hs != nullptr) S.hin[mm] = hs[mm];
          if (ks != nullptr) S.kin[mm] = ks[mm];
        }
        __syncthreads();
      }
    }
    const int nvalid = r.nvalid;

    // the tile body, instantiated branch-free for full chunks and with guards for the ragged last chunk
    auto tile_body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr int kU = kFull ? token_unroll<C>() : 1;  // partial unrolling keeps the kernel's code in the i-cache
      // pass 0: replay the states from the forward's carry; relu masks on dy
      float2 hin = make_float2(0.0f, 0.0f);
      if (c > 0) {
        if (act) hin = S.hin[tid];
      } else if (p.h0_r != nullptr && act) {
        hin = make_float2(p.h0_r[b * M + m], p.h0_i[b * M + m]);
      }
      {
        float2 h = hin;
#pragma unroll kU
        for (int t = 0; t < C; ++t) {
          if (kFull || t < nvalid) {
            const float4 k4 = S.ctl[t];
            const float xr = to_float(S.x[t][0][tid]);
            const float xi = to_float(S.x[t][1][tid]);
            const TokenCoef kc = token_coef<kFast>(mc, k4.x, k4.y, k4.z, k4.w);
            h = cfma(kc.a, h, make_float2(kc.gain * tanh_t<kFast>(xr), kc.gain * tanh_t<kFast>(xi)));
            S.h[t][tid] = h;
            const float gr = to_float(S.dy[t][0][tid]);
            const float gi = to_float(S.dy[t][1][tid]);
            S.dy[t][0][tid] = from_float<TIO>(h.x > 0.0f ? gr : 0.0f);
            S.dy[t][1][tid] = from_float<TIO>(h.y > 0.0f ? gi : 0.0f);
          }
        }
      }

      // adjoint carry entering the chunk from the later chunks
      float2 lam = make_float2(0.0f, 0.0f);
      if (c < chunks - 1) {
        if (act) lam = S.kin[tid];
      } else if (p.glast_r != nullptr && act) {
        lam = make_float2(p.glast_r[b * M + m], p.glast_i[b * M + m]);
      }

      // pass B: the true adjoint with every gradient, kGroup tokens at a time; each group's
      // dEta / dDelta are reduced over the warp at once (lane 4u+j holds value u of the group)
      float fa[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
      for (int t1 = C - 1; t1 >= 0; t1 -= kGroup) {
        float v[2 * kGroup];
#pragma unroll
        for (int u = 0; u < kGroup; ++u) {
          const int t = t1 - u;
          float ve = 0.0f, vd = 0.0f;
          if (kFull || t < nvalid) {
            const float4 k4 = S.ctl[t];
            lam.x += to_float(S.dy[t][0][tid]);
            lam.y += to_float(S.dy[t][1][tid]);
            const float2 pv = t > 0 ? S.h[t - 1][tid] : hin;
            const float cx = to_float(S.x[t][0][tid]);
            const float cy = to_float(S.x[t][1][tid]);
            // h[t] was last read as the previous state at step t+1: its slot now holds the
            // write-path dx
            S.h[t][tid] = grad_step<kFast>(mc, k4, lam, pv, cx, cy, ve, vd, fa);
          }
          v[u] = ve;
          v[kGroup + u] = vd;
        }
        constexpr int kShift = 5 - log2i<2 * kGroup>();
        const float total = transpose_reduce<2 * kGroup>(v, lane);
        if ((lane & ((1 << kShift) - 1)) == 0) {
          const int u = lane >> kShift;  // 0..2*kGroup-1: ve of tokens t1..t1-3, then vd
          const int t = t1 - (u % kGroup);
          S.warp_part[warp][(u < kGroup ? 0 : C) + t] = total;
        }
      }
      if (!act) {
#pragma unroll
        for (int q = 0; q < 5; ++q) fa[q] = 0.0f;
      }
#pragma unroll
      for (int q = 0; q < 5; ++q) acc[q] += fa[q];

      // token sums over all modes -> controller gradients
      __syncthreads();
      if (tid < 2 * C) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kBwdWarps; ++w) sum += S.warp_part[w][tid];
        S.part_grad[par][tid] = sum;
      }
      if (G > 1) cluster.sync();
      else __syncthreads();
      if (tid < 2 * C) {
        float q[8];
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) q[rr] = rr < G ? cluster.map_shared_rank(&S.part_grad[par][0], rr)[tid] : 0.0f;
        float sum = 0.0f;
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) sum += q[rr];
        S.tot[tid] = sum;
      }
      __syncthreads();
      if (tid < C) {
        const float4 k4 = S.ctl[tid];
        const float dp1 = tid < nvalid ? S.tot[tid] * kLn16 * fmaf(-k4.w, k4.w, 1.0f) : 0.0f;
        const float dp0 = tid < nvalid ? S.tot[C + tid] * kHalfPi * fmaf(-k4.z, k4.z, 1.0f) : 0.0f;
        S.dp[tid] = make_float2(dp0, dp1);
      }
      __syncthreads();
      TIO* dxrow = static_cast<TIO*>(p.dx) + row0;
      float fd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll kU
      for (int t = 0; t < C; ++t) {
        if (kFull || t < nvalid) {
          const float2 dp = S.dp[t];
          const float2 dxc = S.h[t][tid];
          const float xr = to_float(S.x[t][0][tid]);
          const float xi = to_float(S.x[t][1][tid]);
          if (act) {
            TIO* row = dxrow + (long long)t * W;
            Io<TIO>::store(row + m, fmaf(dp.x, mc.d0r, fmaf(dp.y, mc.d1r, dxc.x)));
            Io<TIO>::store(row + M + m, fmaf(dp.x, mc.d0i, fmaf(dp.y, mc.d1i, dxc.y)));
          }
          fd[0] = fmaf(xr, dp.x, fd[0]);
          fd[1] = fmaf(xi, dp.x, fd[1]);
          fd[2] = fmaf(xr, dp.y, fd[2]);
          fd[3] = fmaf(xi, dp.y, fd[3]);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[5 + q] += fd[q];
    };
    if (nvalid == C) tile_body(std::true_type{});
    else tile_body(std::false_type{});
    if (g == 0 && tid == 0) {
      float s0 = 0.0f, s1 = 0.0f;
      for (int t = 0; t < C; ++t) {
        s0 += S.dp[t].x;
        s1 += S.dp[t].y;
      }
      acc_b0 += s0;
      acc_b1 += s1;
    }
    __syncthreads();  // every shared array is free for the next tile
  }
  // per-cluster partial parameter gradients (reduced in a fixed order by mixer_reduce_kernel)
  const long long kc = blockIdx.y;
  double* part = p.part + kc * (long long)kPartModes * Mp;
#pragma unroll
  for (int q = 0; q < kPartModes; ++q) part[(long long)q * Mp + m] = act ? acc[q] : 0.0;
  if (g == 0 && tid == 0) {
    double* pb = p.part + (long long)gridDim.y * kPartModes * Mp + 2 * kc;
    pb[0] = acc_b0;
    pb[1] = acc_b1;
  }
  if (timed_out) atomicOr(&p.ls->status, kStatusTimeout);
  cluster.sync();
}
