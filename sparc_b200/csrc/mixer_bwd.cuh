// SPARC mixer backward kernel (included by mixer.cu, inside namespace sparc).
//
// Same tiling as the forward (a cluster of G CTAs per tile of C tokens x all M modes, two
// adjacent modes per thread), walked in reverse chunk order. The x and dy tiles arrive in
// shared memory by TMA bulk copies. Per tile:
//   controls    the projections are recomputed from x (cluster reduction, as in the forward);
//   pass 0      replay the states from the forward's chunk carry, keep them in shared memory and
//               zero dy where the relu was inactive;
//   carry       if the carry of the adjoint from the later chunk is already published, use it;
//               otherwise run the local reverse pass from zero (pass A), publish the aggregate
//               (conj(P), Qr) and resolve the carry by decoupled lookback;
//   pass B      the true adjoint backwards through the chunk with every gradient: transition
//               (dEta, dDelta per token, dNu, dTheta per mode), write path (dx of the content,
//               dEta, dDelta, dNu, write-gain / response gradients); the write-path dx waits in
//               the state slots the reverse walk has consumed;
//   tokens      dEta, dDelta are summed over all modes (cluster reduction), turned into the
//               controller gradients dp0, dp1, which finish dx and the direction gradients.
// Per-mode parameter gradients accumulate in float64 per cluster; mixer_reduce_kernel sums the
// clusters in a fixed order.

// (included inside namespace sparc)

constexpr int kBwdThreads = 128;
constexpr int kBwdModes = 2 * kBwdThreads;
constexpr int kPartModes = 9;  // nu, theta (sum of phase grads), wlg, wpr, wrr, D0r, D0i, D1r, D1i

template <typename TIO, int C>
struct BwdSmem {
  TIO x[C][2][kBwdModes];
  TIO dy[C][2][kBwdModes];     // masked by the relu in pass 0
  float2 h[C][kBwdModes];      // replayed states, then the write-path dx (pass B)
  float4 ctl[C];               // E, delta, tau0, tau1
  float2 dp[C];                // controller gradients dp0, dp1
  float tot[2 * C];            // cluster totals of the current reduction
  float part_ctl[2][2 * C];    // projection partials (peers read), by tile parity
  float part_grad[2][2 * C];   // dEta / dDelta partials (peers read), by tile parity
  float warp_part[kBwdThreads / 32][2 * C];
  float vt[2 * C][kBwdThreads];   // per-thread dEta / dDelta partials of pass B, by token
  unsigned long long bar;
  long long ring[2];
  unsigned win[2];
  unsigned pred;
};

struct BwdParams {
  const void* x;
  const void* dy;
  void* dx;
  MixerParamPtrs pp;
  const float* h0_r;
  const float* h0_i;
  const float* glast_r;
  const float* glast_i;
  float* gh0_r;
  float* gh0_i;
  const float2* carry;  // forward inclusive states [B, chunks, M]
  LaunchState* ls;
  unsigned* flags;
  float4* agg;
  float2* incl;         // reverse inclusive carries [tiles, Mp]
  double* part;         // [clusters][kPartModes][Mp] then [clusters][2] bias partials
  long long B, T;
  int W, M, chunks;
  long long tiles;
  unsigned max_spin;
  int deterministic;
  int use_tma;
  long long inject_unpublished;
};

// Cluster-wide sum of 2C per-thread values; every CTA gets the totals in `tot` (2C floats).
template <int C>
__device__ __forceinline__ void cluster_sum_2c(float (&v)[2 * C], float (*warp_part)[2 * C], float* part,
                                               float* tot, int G, cg::cluster_group& cluster) {
  constexpr int NW = kBwdThreads / 32;
  constexpr int kShift = 5 - log2i<2 * C>();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float total = transpose_reduce<2 * C>(v, lane);
  if ((lane & ((1 << kShift) - 1)) == 0) warp_part[warp][lane >> kShift] = total;
  __syncthreads();
  if (tid < 2 * C) {
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) sum += warp_part[w][tid];
    part[tid] = sum;
  }
  cluster.sync();
  if (tid < 2 * C) {
    float q[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) q[r] = r < G ? cluster.map_shared_rank(part, r)[tid] : 0.0f;
    float sum = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) sum += q[r];
    tot[tid] = sum;
  }
}

template <typename TIO, int C>
__device__ __forceinline__ void fetch_bwd_tile(const BwdParams& p, BwdSmem<TIO, C>& S, long long row0,
                                               int nvalid, int g) {
  const int mbase = g * kBwdModes;
  const int ncols = min(kBwdModes, p.M - mbase);
  const TIO* xs = static_cast<const TIO*>(p.x) + row0 + mbase;
  const TIO* ds = static_cast<const TIO*>(p.dy) + row0 + mbase;
  if (p.use_tma) {
    if (threadIdx.x < 32) {
      const unsigned bytes = (unsigned)(ncols * sizeof(TIO));
      if (threadIdx.x == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.bar, bytes * 4u * (unsigned)nvalid);
      }
      __syncwarp();
      for (int t = threadIdx.x; t < nvalid; t += 32) {
        const long long o = (long long)t * p.W;
        bulk_copy_g2s(&S.x[t][0][0], xs + o, bytes, &S.bar);
        bulk_copy_g2s(&S.x[t][1][0], xs + o + p.M, bytes, &S.bar);
        bulk_copy_g2s(&S.dy[t][0][0], ds + o, bytes, &S.bar);
        bulk_copy_g2s(&S.dy[t][1][0], ds + o + p.M, bytes, &S.bar);
      }
    }
  } else {
    for (int i = threadIdx.x; i < nvalid * 2 * ncols; i += kBwdThreads) {
      const int t = i / (2 * ncols), r = i - t * 2 * ncols, half = r / ncols, mm = r - half * ncols;
      const long long o = (long long)t * p.W + half * p.M + mm;
      S.x[t][half][mm] = xs[o];
      S.dy[t][half][mm] = ds[o];
    }
  }
}

template <typename TIO, int C, bool kFast, bool kVec>
__global__ void __launch_bounds__(kBwdThreads) mixer_bwd_kernel(const BwdParams p) {
  cg::cluster_group cluster = cg::this_cluster();
  const int g = (int)cluster.block_rank();
  const int G = (int)cluster.num_blocks();
  const int tid = threadIdx.x;
  const int M = p.M, W = p.W;
  const int m0 = g * kBwdModes + 2 * tid;
  const int Mp = G * kBwdModes;
  const bool act0 = m0 < M, act1 = m0 + 1 < M;
  const long long B = p.B, T = p.T;
  const int chunks = p.chunks;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  BwdSmem<TIO, C>& S = *reinterpret_cast<BwdSmem<TIO, C>*>(smem_raw);

  const ModeConst mc0 = load_mode(p.pp, m0, M, act0);
  const ModeConst mc1 = load_mode(p.pp, m0 + 1, M, act1);
  const float bias0 = p.pp.phase_dir[W], bias1 = p.pp.radial_dir[W];
  LookbackCtx lc{p.ls, p.flags, p.agg, *(volatile unsigned*)&p.ls->epoch, p.max_spin, G, Mp, B,
                 p.deterministic != 0};

  {
    unsigned* z = reinterpret_cast<unsigned*>(&S.x[0][0][0]);
    for (int i = tid; i < (int)((sizeof(S.x) + sizeof(S.dy)) / 4); i += kBwdThreads) z[i] = 0u;
  }
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    mbar_init_fence();
  }
  __syncthreads();

  double acc[2][kPartModes];
#pragma unroll
  for (int q = 0; q < kPartModes; ++q) acc[0][q] = acc[1][q] = 0.0;
  double acc_b0 = 0.0, acc_b1 = 0.0;
  bool timed_out = false;

  for (int it = 0;; ++it) {
    const int par = it & 1;
    if (tid == 0 && g == 0) S.ring[par] = atomicAdd(&p.ls->ticket, 1u);
    cluster.sync();
    if (tid == 0 && g != 0) S.ring[par] = *cluster.map_shared_rank(&S.ring[par], 0);
    __syncthreads();
    const long long ticket = S.ring[par];
    if (ticket >= p.tiles) break;
    const long long b = ticket % B;
    const int c = chunks - 1 - (int)(ticket / B);
    const long long t0 = (long long)c * C;
    const int nvalid = (int)(T - t0 < C ? T - t0 : C);
    const long long row0 = (b * T + t0) * W;
    fetch_bwd_tile<TIO, C>(p, S, row0, nvalid, g);
    if (tid == 0) S.pred = c < chunks - 1 ? ld_acquire(p.flags + (ticket - B) * G + g) : 0u;
    if (p.use_tma) {
      if (!mbar_wait(&S.bar, (unsigned)par, p.max_spin << 4)) timed_out = true;
    } else {
      __syncthreads();
    }

    // controls (recomputed from x)
    {
      float v[2 * C];
#pragma unroll
      for (int t = 0; t < C; ++t) {
        const float2 xr = Pair<TIO>::load(&S.x[t][0][2 * tid]);
        const float2 xi = Pair<TIO>::load(&S.x[t][1][2 * tid]);
        v[t] = fmaf(xr.x, mc0.d0r, fmaf(xi.x, mc0.d0i, fmaf(xr.y, mc1.d0r, xi.y * mc1.d0i)));
        v[C + t] = fmaf(xr.x, mc0.d1r, fmaf(xi.x, mc0.d1i, fmaf(xr.y, mc1.d1r, xi.y * mc1.d1i)));
      }
      cluster_sum_2c<C>(v, S.warp_part, S.part_ctl[par], S.tot, G, cluster);
      __syncthreads();
      if (tid < C) {
        const float tau0 = tanh_accurate(S.tot[tid] + bias0);
        const float tau1 = tanh_accurate(S.tot[C + tid] + bias1);
        S.ctl[tid] = make_float4(expf(kLn16 * tau1), kHalfPi * tau0, tau0, tau1);
      }
      __syncthreads();
    }

    // the tile body, instantiated branch-free for full chunks and with guards for the ragged last chunk
    auto tile_body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr int kU = kFull ? 4 : 1;  // partial unrolling keeps the kernel's code in the i-cache
      // pass 0: replay the states from the forward's carry; relu masks on dy; chunk product
      float2 hin0 = make_float2(0.0f, 0.0f), hin1 = hin0;
      if (c > 0) {
        const float2* cp = p.carry + (b * chunks + (c - 1)) * M + m0;
        if (act0) hin0 = cp[0];
        if (act1) hin1 = cp[1];
      } else if (p.h0_r != nullptr) {
        if (act0) hin0 = make_float2(p.h0_r[b * M + m0], p.h0_i[b * M + m0]);
        if (act1) hin1 = make_float2(p.h0_r[b * M + m0 + 1], p.h0_i[b * M + m0 + 1]);
      }
      float2 P0 = make_float2(1.0f, 0.0f), P1 = P0;
      {
        float2 h0 = hin0, h1 = hin1;
  #pragma unroll kU
        for (int t = 0; t < C; ++t) {
          if (kFull || t < nvalid) {
            const float4 k4 = S.ctl[t];
            const float2 xr = Pair<TIO>::load(&S.x[t][0][2 * tid]);
            const float2 xi = Pair<TIO>::load(&S.x[t][1][2 * tid]);
            const TokenCoef k0 = token_coef<kFast>(mc0, k4.x, k4.y, k4.z, k4.w);
            const TokenCoef k1 = token_coef<kFast>(mc1, k4.x, k4.y, k4.z, k4.w);
            h0 = cfma(k0.a, h0, make_float2(k0.gain * tanh_t<kFast>(xr.x), k0.gain * tanh_t<kFast>(xi.x)));
            h1 = cfma(k1.a, h1, make_float2(k1.gain * tanh_t<kFast>(xr.y), k1.gain * tanh_t<kFast>(xi.y)));
            P0 = cmul(k0.a, P0);
            P1 = cmul(k1.a, P1);
            *reinterpret_cast<float4*>(&S.h[t][2 * tid]) = make_float4(h0.x, h0.y, h1.x, h1.y);
            const float2 gr = Pair<TIO>::load(&S.dy[t][0][2 * tid]);
            const float2 gi = Pair<TIO>::load(&S.dy[t][1][2 * tid]);
            Pair<TIO>::store(&S.dy[t][0][2 * tid], h0.x > 0.0f ? gr.x : 0.0f, h1.x > 0.0f ? gr.y : 0.0f);
            Pair<TIO>::store(&S.dy[t][1][2 * tid], h0.y > 0.0f ? gi.x : 0.0f, h1.y > 0.0f ? gi.y : 0.0f);
          }
        }
      }

      // carry of the adjoint from the later chunks
      const unsigned pst = S.pred;
      const bool last_chunk = c == chunks - 1;
      const bool pred_ready = last_chunk || (!lc.deterministic && ((pst >> 2) == (lc.epoch & 0x3fffffffu)) &&
                                             (pst & 3u) == kFlagInclusive);
      const bool publish = ticket != p.inject_unpublished;
      float2 kin0 = make_float2(0.0f, 0.0f), kin1 = kin0;
      if (last_chunk) {
        if (p.glast_r != nullptr) {
          if (act0) kin0 = make_float2(p.glast_r[b * M + m0], p.glast_i[b * M + m0]);
          if (act1) kin1 = make_float2(p.glast_r[b * M + m0 + 1], p.glast_i[b * M + m0 + 1]);
        }
      } else if (pred_ready) {
        const float2* ip = p.incl + (ticket - B) * Mp + m0;
        kin0 = __ldcg(ip);
        kin1 = __ldcg(ip + 1);
      } else {
        // pass A: local reverse adjoint from zero -> aggregate (conj P, Qr)
        float2 q0 = make_float2(0.0f, 0.0f), q1 = q0;
  #pragma unroll kU
        for (int t = C - 1; t >= 0; --t) {
          if (kFull || t < nvalid) {
            const float4 k4 = S.ctl[t];
            const float2 gr = Pair<TIO>::load(&S.dy[t][0][2 * tid]);
            const float2 gi = Pair<TIO>::load(&S.dy[t][1][2 * tid]);
            q0.x += gr.x;
            q0.y += gi.x;
            q1.x += gr.y;
            q1.y += gi.y;
            const float2 a0 = token_transition(mc0, k4.x, k4.y);
            const float2 a1 = token_transition(mc1, k4.x, k4.y);
            q0 = make_float2(fmaf(a0.x, q0.x, a0.y * q0.y), fmaf(a0.x, q0.y, -a0.y * q0.x));
            q1 = make_float2(fmaf(a1.x, q1.x, a1.y * q1.y), fmaf(a1.x, q1.y, -a1.y * q1.x));
          }
        }
        const float2* incl = p.incl;
        float2 A[2] = {make_float2(P0.x, -P0.y), make_float2(P1.x, -P1.y)}, Bv[2] = {q0, q1}, kin[2];
        lookback<2>(lc, ticket, g, chunks - 1 - c, A, Bv, publish, pst, S.win, m0,
                    [&](int j, float2 (&hh)[2]) {
                      const float2* ip = incl + (ticket - (long long)j * B) * Mp + m0;
                      hh[0] = __ldcg(ip);
                      hh[1] = __ldcg(ip + 1);
                    },
                    kin);
        kin0 = kin[0];
        kin1 = kin[1];
        // publish the inclusive carry now (the fast path publishes it after pass B)
        if (publish) {
          const float2 o0 = cfma(make_float2(P0.x, -P0.y), kin0, q0);
          const float2 o1 = cfma(make_float2(P1.x, -P1.y), kin1, q1);
          *reinterpret_cast<float4*>(p.incl + ticket * Mp + m0) = make_float4(o0.x, o0.y, o1.x, o1.y);
          publish_flag(p.flags + ticket * G + g, make_flag(lc.epoch, kFlagInclusive));
        }
      }

      // pass B: the true adjoint with every gradient
      float fa[2][5];
  #pragma unroll
      for (int q = 0; q < 5; ++q) fa[0][q] = fa[1][q] = 0.0f;
      float2 lam0 = kin0, lam1 = kin1;
  #pragma unroll kU
      for (int t = C - 1; t >= 0; --t) {
        float ve = 0.0f, vd = 0.0f;
        if (kFull || t < nvalid) {
          const float4 k4 = S.ctl[t];
          const float2 gr = Pair<TIO>::load(&S.dy[t][0][2 * tid]);
          const float2 gi = Pair<TIO>::load(&S.dy[t][1][2 * tid]);
          lam0.x += gr.x;
          lam0.y += gi.x;
          lam1.x += gr.y;
          lam1.y += gi.y;
          float4 prev;
          if (t > 0) prev = *reinterpret_cast<const float4*>(&S.h[t - 1][2 * tid]);
          else prev = make_float4(hin0.x, hin0.y, hin1.x, hin1.y);
          const float2 xr = Pair<TIO>::load(&S.x[t][0][2 * tid]);
          const float2 xi = Pair<TIO>::load(&S.x[t][1][2 * tid]);
          float4 dxc;
  #pragma unroll
          for (int q = 0; q < 2; ++q) {
            const ModeConst& mc = q == 0 ? mc0 : mc1;
            float2& lam = q == 0 ? lam0 : lam1;
            const float2 pv = q == 0 ? make_float2(prev.x, prev.y) : make_float2(prev.z, prev.w);
            const float cx = q == 0 ? xr.x : xr.y, cy = q == 0 ? xi.x : xi.y;
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
            ve += radial + fmaf(gg, dyn, gq * mc.wrr * kInvLn16);
            vd += fmaf(gq * mc.wpr, kInvHalfPi, dscan);
            fa[q][0] += radial + gg * (dyn - mc.stat);
            fa[q][1] += pg;
            fa[q][2] += gg;
            fa[q][3] = fmaf(gq, k4.z, fa[q][3]);
            fa[q][4] = fmaf(gq, k4.w, fa[q][4]);
            const float dr = lam.x * k.gain * fmaf(-cr, cr, 1.0f);
            const float di = lam.y * k.gain * fmaf(-ci, ci, 1.0f);
            if (q == 0) {
              dxc.x = dr;
              dxc.y = di;
            } else {
              dxc.z = dr;
              dxc.w = di;
            }
            lam = make_float2(fmaf(ar, lam.x, ai * lam.y), fmaf(ar, lam.y, -ai * lam.x));
          }
          // h[t] was last read as `prev` at step t+1: its slot now holds the write-path dx
          *reinterpret_cast<float4*>(&S.h[t][2 * tid]) = dxc;
        }
        S.vt[t][tid] = ve;
        S.vt[C + t][tid] = vd;
      }
      if (!act0) {
        lam0 = make_float2(0.0f, 0.0f);
  #pragma unroll
        for (int q = 0; q < 5; ++q) fa[0][q] = 0.0f;
      }
      if (!act1) {
        lam1 = make_float2(0.0f, 0.0f);
  #pragma unroll
        for (int q = 0; q < 5; ++q) fa[1][q] = 0.0f;
      }
      if (pred_ready && publish) {
        // fast path: the carry toward the earlier chunk is conj(a_t0) lambda_t0 = lam now
        *reinterpret_cast<float4*>(p.incl + ticket * Mp + m0) = make_float4(lam0.x, lam0.y, lam1.x, lam1.y);
        publish_flag(p.flags + ticket * G + g, make_flag(lc.epoch, kFlagInclusive));
      }
      if (c == 0 && p.gh0_r != nullptr) {
        if (act0) {
          p.gh0_r[b * M + m0] = lam0.x;
          p.gh0_i[b * M + m0] = lam0.y;
        }
        if (act1) {
          p.gh0_r[b * M + m0 + 1] = lam1.x;
          p.gh0_i[b * M + m0 + 1] = lam1.y;
        }
      }
  #pragma unroll
      for (int q = 0; q < 5; ++q) {
        acc[0][q] += fa[0][q];
        acc[1][q] += fa[1][q];
      }

      // token sums over all modes -> controller gradients
      float v[2 * C];
#pragma unroll
      for (int i = 0; i < 2 * C; ++i) v[i] = S.vt[i][tid];
      cluster_sum_2c<C>(v, S.warp_part, S.part_grad[par], S.tot, G, cluster);
      __syncthreads();
      if (tid < C) {
        const float4 k4 = S.ctl[tid];
        const float dp1 = tid < nvalid ? S.tot[tid] * kLn16 * fmaf(-k4.w, k4.w, 1.0f) : 0.0f;
        const float dp0 = tid < nvalid ? S.tot[C + tid] * kHalfPi * fmaf(-k4.z, k4.z, 1.0f) : 0.0f;
        S.dp[tid] = make_float2(dp0, dp1);
      }
      __syncthreads();
      TIO* dxrow = static_cast<TIO*>(p.dx) + row0;
      float fd[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
  #pragma unroll kU
      for (int t = 0; t < C; ++t) {
        if (kFull || t < nvalid) {
          const float2 dp = S.dp[t];
          const float4 dxc = *reinterpret_cast<const float4*>(&S.h[t][2 * tid]);
          const float2 xr = Pair<TIO>::load(&S.x[t][0][2 * tid]);
          const float2 xi = Pair<TIO>::load(&S.x[t][1][2 * tid]);
          const float r0 = fmaf(dp.x, mc0.d0r, fmaf(dp.y, mc0.d1r, dxc.x));
          const float i0 = fmaf(dp.x, mc0.d0i, fmaf(dp.y, mc0.d1i, dxc.y));
          const float r1 = fmaf(dp.x, mc1.d0r, fmaf(dp.y, mc1.d1r, dxc.z));
          const float i1 = fmaf(dp.x, mc1.d0i, fmaf(dp.y, mc1.d1i, dxc.w));
          TIO* row = dxrow + (long long)t * W;
          if (kVec && act1) {
            Pair<TIO>::store(row + m0, r0, r1);
            Pair<TIO>::store(row + M + m0, i0, i1);
          } else {
            if (act0) {
              Io<TIO>::store(row + m0, r0);
              Io<TIO>::store(row + M + m0, i0);
            }
            if (act1) {
              Io<TIO>::store(row + m0 + 1, r1);
              Io<TIO>::store(row + M + m0 + 1, i1);
            }
          }
          fd[0][0] = fmaf(xr.x, dp.x, fd[0][0]);
          fd[0][1] = fmaf(xi.x, dp.x, fd[0][1]);
          fd[0][2] = fmaf(xr.x, dp.y, fd[0][2]);
          fd[0][3] = fmaf(xi.x, dp.y, fd[0][3]);
          fd[1][0] = fmaf(xr.y, dp.x, fd[1][0]);
          fd[1][1] = fmaf(xi.y, dp.x, fd[1][1]);
          fd[1][2] = fmaf(xr.y, dp.y, fd[1][2]);
          fd[1][3] = fmaf(xi.y, dp.y, fd[1][3]);
        }
      }
  #pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[0][5 + q] += fd[0][q];
        acc[1][5 + q] += fd[1][q];
      }
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
    __syncthreads();
  }
  // per-cluster partial parameter gradients (reduced in a fixed order by mixer_reduce_kernel)
  const long long k = blockIdx.y;
  double* part = p.part + k * (long long)kPartModes * Mp;
#pragma unroll
  for (int q = 0; q < kPartModes; ++q) {
    part[(long long)q * Mp + m0] = act0 ? acc[0][q] : 0.0;
    part[(long long)q * Mp + m0 + 1] = act1 ? acc[1][q] : 0.0;
  }
  if (g == 0 && tid == 0) {
    double* pb = p.part + (long long)gridDim.y * kPartModes * Mp + 2 * k;
    pb[0] = acc_b0;
    pb[1] = acc_b1;
  }
  if (timed_out && tid == 0) atomicOr(&p.ls->status, kStatusTimeout);
  cluster.sync();
  finish_launch(p.ls);
}
