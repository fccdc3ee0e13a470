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
//                             forward's chunk carry into shared memory; pass B
//                             walks the true adjoint backwards with every gradient: transition
//                             (dEta, dDelta per token, dNu, dTheta per mode), write path (dx of
//                             the content, dEta, dDelta, dNu, write-gain / response gradients);
//                             the write-path dx waits in the state slots the reverse walk has
//                             consumed. dEta, dDelta are summed over all modes (warp
//                             transpose-reduce per group of tokens during the walk, then shared
//                             and distributed shared memory) into the controller gradients dp0,
//                             dp1, which finish dx and the direction gradients.
//   mixer_bwd_grad_saved_kernel  the same gradients when the forward saved every token's state:
//                             no replay. Without a cluster (W <= 512) each tile is walked as two
//                             halves of C/2 tokens (the later half first, the adjoint carried
//                             between them in registers), each half's x, dy and states arriving
//                             by TMA into one of two stages, so that the next half's copies run
//                             under this half's arithmetic; in clusters, where every part costs a
//                             cross-CTA reduction, as whole tiles. The cluster's per-token sums
//                             are pushed into every CTA with asynchronous stores on an mbarrier.
// The reverse summary runs one mode per thread (256 threads per CTA); the gradient kernel two
// adjacent modes per thread with packed f32x2 arithmetic (128 threads). Per-mode parameter
// gradients accumulate per cluster; mixer_reduce_kernel sums the clusters in float64 in a fixed
// order. The token controls come from the forward (saved per token, as pairs).

// (included inside namespace sparc)

constexpr int kBwdThreads = 256;
constexpr int kBwdModes = kBwdThreads;  // one mode per thread
constexpr int kBwdWarps = kBwdThreads / 32;
constexpr int kPartModes = 11;  // nu, theta (sum of phase grads), wlg, wpr, wrr, D0r, D0i, D1r, D1i,
                                // norm weight at the real / imaginary column (blocks only)
constexpr int kGroup = 4;      // tokens per unrolled group of the reverse walk

// kY: the relu mask comes from a tile of the forward's output (or states); a block reads its
// relu bits and the projection mode has no relu, and they hold a minimal placeholder instead.
template <typename TIO, int C, bool kY>
struct RsumSmem {
  static constexpr int YB = kY ? 2 : 1, YC = kY ? C : 1;
  TIO dy[2][C][2][kBwdModes];
  TIO y[YB][YC][2][kBwdModes];    // the forward's output or states (kY)
  TokenCtl ctl[2][C];
  unsigned mask[2][C][16];        // a block's relu bits for the CTA's 256 modes
  unsigned long long bar[2];
};


struct BwdParams {
  CUtensorMap map_x;     // x, y, dy as [B*T rows][re|im][M], box {256, 2, C} (when use_tma)
  CUtensorMap map_y;
  CUtensorMap map_dy;
  CUtensorMap map_h;     // the forward's saved states, box {256, 2, S + 1} (saved-state kernel,
                         // S tokens per stage; its map_x and map_dy then have box {256, 2, S})
  const void* x;
  const void* y;
  const void* dy;
  void* dx;
  const void* states;    // [B*T, W] the forward's states [Re | Im] (dtype) (saved-state kernel)
  MixerParamPtrs pp;
  const float* h0_r;
  const float* h0_i;
  const float* glast_r;
  const float* glast_i;
  const TokenCtl* ctl;   // [B, T] forward token controls
  const float* norm_w;   // [W] RMSNorm weight of a block (kBlock kernels)
  const unsigned* mask;  // [B*T, mask_words] relu bits of a block's mixer output (kBlock)
  int mask_words;
  const float2* carry;   // [B, chunks, M] forward inclusive states
  const float2* kout;    // [B, chunks, M] adjoint carry leaving each chunk (scan output)
  float4* agg;           // [B, chunks, Mp] reverse aggregates (summary output)
  double* part;          // [clusters][kPartModes][Mp] then [clusters][2] bias partials
  float2* dp_out;        // [B*T] controller-projection gradients (dp0, dp1) (kModeProj)
  int content_linear;    // kModeProj: the content is u itself instead of tanh(u)
  LaunchState* ls;
  long long B, T;
  int W, M, Mp, chunks;
  long long tiles;
  unsigned max_spin;
  int use_tma;
};



// ------------------------------------------------------------------------------ reverse summary
template <typename TIO, int C, bool kFast, int kMode>
__global__ void __launch_bounds__(kBwdThreads) mixer_bwd_summary_kernel(const __grid_constant__ BwdParams p) {
  constexpr bool kBlock = kMode == kModeBlock, kProj = proj_like<kMode>();  // (projection / scan modes: no relu)
  constexpr bool kScan = kMode == kModeScan;
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
  constexpr bool kY = !kBlock && !kProj;
  RsumSmem<TIO, C, kY>& S = *reinterpret_cast<RsumSmem<TIO, C, kY>*>(smem_raw);

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
    const TokenCtl* csrc = p.ctl + r.b * T + r.t0;
    const unsigned* msrc = kBlock ? p.mask + (r.b * T + r.t0) * (long long)p.mask_words + (mbase >> 6) * 4 : nullptr;
    if (p.use_tma) {
      if (tid == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.bar[buf], (kBlock || kProj ? 1u : 2u) * act_box_bytes<TIO, C, kBwdModes>() +
                                               (unsigned)sizeof(TokenCtl) * (unsigned)r.nvalid +
                                               (kBlock ? 64u * (unsigned)r.nvalid : 0u));
        const int row = (int)(r.b * T + r.t0);
        tma_load_3d(&S.dy[buf][0][0][0], &p.map_dy, mbase, 0, row, &S.bar[buf]);
        if constexpr (kBlock) {
          for (int t = 0; t < r.nvalid; ++t)
            bulk_copy_g2s(&S.mask[buf][t][0], msrc + (long long)t * p.mask_words, 64u, &S.bar[buf]);
        } else if constexpr (!kProj) {
          tma_load_3d(&S.y[buf][0][0][0], &p.map_y, mbase, 0, row, &S.bar[buf]);
        }
        bulk_copy_g2s(&S.ctl[buf][0], csrc, (unsigned)sizeof(TokenCtl) * (unsigned)r.nvalid, &S.bar[buf]);
      }
    } else {
      load_act_rows<TIO, kBwdModes>(dsrc, W, M, mbase, r.nvalid, S.dy[buf], kBwdThreads);
      if constexpr (kBlock) {
        for (int j = tid; j < 16 * r.nvalid; j += kBwdThreads) S.mask[buf][j >> 4][j & 15] = msrc[(long long)(j >> 4) * p.mask_words + (j & 15)];
      } else if constexpr (!kProj) {
        load_act_rows<TIO, kBwdModes>(ysrc, W, M, mbase, r.nvalid, S.y[buf], kBwdThreads);
      }
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
    const TIO(*yt)[2][kBwdModes] = S.y[kY ? buf : 0];
    const TokenCtl* ctl = S.ctl[buf];
    auto body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr int kU = kFull ? token_unroll<C>() : 1;
      float2 q = make_float2(0.0f, 0.0f);
      float2 P = make_float2(1.0f, 0.0f);
#pragma unroll kU
      for (int t = C - 1; t >= 0; --t) {
        if (kFull || t < r.nvalid) {
          const TokenCtl& tc = ctl[t];
          const float gr = to_float(dyt[t][0][tid]);
          const float gi = to_float(dyt[t][1][tid]);
          bool on_r, on_i;
          if constexpr (kProj) {
            on_r = on_i = true;
          } else if constexpr (kBlock) {  // bit (mode % 64) / 2 of word 4 (mode / 64) + mode % 2 (+2: imaginary)
            const unsigned* mw = &S.mask[buf][t][(tid >> 6) * 4 + (tid & 1)];
            const unsigned bit = 1u << ((tid & 63) >> 1);
            on_r = (mw[0] & bit) != 0u;
            on_i = (mw[2] & bit) != 0u;
          } else {
            on_r = to_float(yt[t][0][tid]) > 0.0f;
            on_i = to_float(yt[t][1][tid]) > 0.0f;
          }
          q.x += on_r ? gr : 0.0f;
          q.y += on_i ? gi : 0.0f;
          const float2 a = token_transition<kFast, bwd_rot<kFast>(), kScan>(mc, tc.ed.x, tc.ed.z, tc.keep.x);
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
// Two adjacent modes per thread (128 threads, 256 modes per CTA): the per-mode arithmetic runs
// in packed f32x2 lanes. The replayed states and, later, the write-path dx sit in separate
// real / imaginary planes so that a thread's two modes load as one pair.
constexpr int kGradThreads = 128;
constexpr int kGradWarps = kGradThreads / 32;

template <typename TIO, int C>
struct GradSmem {
  TIO x[C][2][kBwdModes];
  TIO dy[C][2][kBwdModes];     // the output gradient as given (the relu mask applies in pass B)
  TIO h[C][2][kBwdModes];      // replayed states (real, imaginary plane), then the write-path dx
                               // (pass B). In the activation dtype: for bfloat16 that keeps the
                               // CTA within four per SM (the reference's bf16 path likewise saves
                               // its states in bf16); float32 keeps them exact
  float2 hin[kBwdModes];       // state entering the chunk, (re, im) per mode
  float2 kin[kBwdModes];       // adjoint carry entering the chunk from the later chunks
  TokenCtl ctl[C];
  float4 dp[C];                // controller gradients per token as pairs (dp0, dp0, dp1, dp1)
  float2 kap[C];               // a block's RMSNorm backward coefficient r^3/W sum(x w dn), as a pair
  float tot[3 * C];            // cluster totals of dEta / dDelta (and sum x w dxc in a block)
  float part_grad[2][3 * C];   // CTA partials (peers read), by tile parity
  float warp_part[kGradWarps][3 * C];
  unsigned long long bar;
};

__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ void st2(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }

// Gradient contributions of one token for the thread's two modes: updates the adjoint lam in
// place (to conj(a) lam) and returns the write-path dx of the content; returns the token's dEta /
// dDelta contributions in ve / vd (per lane) and adds the per-mode parameter terms to fa.
template <bool kFast, int kMode>
__device__ __forceinline__ Cx2 grad_step2(const ModeConst2& mc, const TokenCtl& tc, Cx2& lam, Cx2 pv, float2 cx,
                                          float2 cy, float2& ve, float2& vd, float2 (&fa)[5], bool lin) {
  const float2 delta = make_float2(tc.ed.z, tc.ed.w), tau0 = make_float2(tc.tau.x, tc.tau.y),
               tau1 = make_float2(tc.tau.z, tc.tau.w);
  // with a reset the transition (k.a) is zero, so every transition-gradient term below vanishes
  constexpr bool kScan = kMode == kModeScan;
  const TokenCoef2 k = token_coef2<kFast, bwd_rot<kFast>(), kScan>(mc, tc);
  const float2 gar = fma2(lam.re, pv.re, mul2(lam.im, pv.im));   // Re(lam conj(h_prev))
  const float2 gai = sub2(mul2(lam.im, pv.re), mul2(lam.re, pv.im));  // Im(lam conj(h_prev))
  const float2 pg = sub2(mul2(gai, k.a.re), mul2(gar, k.a.im));
  const float2 radial = mul2(k.z, sub2(mul2(mul2(k.rho, delta), pg), fma2(gar, k.a.re, mul2(gai, k.a.im))));
  const float2 dscan = sub2(pg, mul2(k.rho, pg));
  if constexpr (kScan) {
    // scan-level mode: the writes are inputs (unit gain), so only the transition's terms remain
    ve = radial;
    vd = dscan;
    fa[0] = add2(fa[0], radial);
    fa[1] = add2(fa[1], pg);
    const Cx2 dxc = lam;  // the writes' gradient
    lam = Cx2{fma2(k.a.re, lam.re, mul2(k.a.im, lam.im)), sub2(mul2(k.a.re, lam.im), mul2(k.a.im, lam.re))};
    return dxc;
  }
  const float2 cr = content2<kFast, kMode>(cx, lin);
  const float2 ci = content2<kFast, kMode>(cy, lin);
  const float2 gg = mul2(k.gain, fma2(lam.re, cr, mul2(lam.im, ci)));
  const float2 gq = mul2(gg, fma2(bcast2(-0.5f), k.gate, bcast2(1.0f)));
  const float2 dyn = mul2(mul2(k.z, mul2(k.rho, k.rho)), rcp_2(k.num));
  ve = add2(radial, fma2(gg, dyn, mul2(gq, mc.wrr_l)));
  vd = fma2(gq, mc.wpr_h, dscan);
  fa[0] = add2(fa[0], fma2(gg, sub2(dyn, mc.stat), radial));
  fa[1] = add2(fa[1], pg);
  fa[2] = add2(fa[2], gg);
  fa[3] = fma2(gq, tau0, fa[3]);
  fa[4] = fma2(gq, tau1, fa[4]);
  // the content's slope: 1 - tanh^2, or 1 for a linear content
  const float2 sr = lin ? bcast2(1.0f) : sub2(bcast2(1.0f), mul2(cr, cr));
  const float2 si = lin ? bcast2(1.0f) : sub2(bcast2(1.0f), mul2(ci, ci));
  const Cx2 dxc = Cx2{mul2(mul2(lam.re, k.gain), sr), mul2(mul2(lam.im, k.gain), si)};
  lam = Cx2{fma2(k.a.re, lam.re, mul2(k.a.im, lam.im)), sub2(mul2(k.a.re, lam.im), mul2(k.a.im, lam.re))};
  return dxc;
}


// In a block (kBlock) the mixer's input is n = x r w (RMSNorm) and the output gradient also
// flows straight to x (residual): dx = dy + r w dn - (r^3 / W) x sum_j(x_j w_j dn_j), with dn the
// mixer's input gradient; the weight's gradient sums x r dn per column.
template <typename TIO, int C, bool kFast, bool kVec, int kMode>
__global__ void __launch_bounds__(kGradThreads, 4) mixer_bwd_grad_kernel(const __grid_constant__ BwdParams p) {
  static_assert(C % kGroup == 0, "the reverse walk runs in groups of kGroup tokens");
  constexpr bool kBlock = kMode == kModeBlock, kProj = proj_like<kMode>(), kScan = kMode == kModeScan;
  const bool lin = kProj && p.content_linear != 0;
  cg::cluster_group cluster = cg::this_cluster();
  const int g = (int)cluster.block_rank();
  const int G = (int)cluster.num_blocks();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = p.M, W = p.W;
  const int mbase = g * kBwdModes;
  const int m0 = mbase + 2 * tid;  // this thread's modes: m0, m0 + 1
  const int Mp = p.Mp;
  const bool act0 = m0 < M, act1 = m0 + 1 < M;
  const long long B = p.B, T = p.T;
  const int chunks = p.chunks;
  const int ncols = min(kBwdModes, M - mbase);
  const long long k0 = blockIdx.y, nk = gridDim.y;
  constexpr int kVals = kBlock ? 3 * C : 2 * C;  // reduced per-token values

  extern __shared__ __align__(128) unsigned char smem_raw[];
  GradSmem<TIO, C>& S = *reinterpret_cast<GradSmem<TIO, C>*>(smem_raw);

  ModeConst2 mc = pair_modes(load_mode(p.pp, m0, M, act0), load_mode(p.pp, m0 + 1, M, act1));
  if constexpr (kBlock) load_norm_weight(mc, p.norm_w, m0, M, act0, act1);

  {
    unsigned* z = reinterpret_cast<unsigned*>(&S.x[0][0][0]);
    for (int i = tid; i < (int)((sizeof(S.x) + sizeof(S.dy)) / 4); i += kGradThreads) z[i] = 0u;
  }
  if (tid == 0) {
    mbar_init(&S.bar, 1);
    mbar_init_fence();
  }
  __syncthreads();

  // per-mode parameter-gradient sums of this cluster's tiles (float pairs; each tile adds its
  // C-token sum, the fixed-order cross-cluster reduction runs in float64)
  float2 acc[kPartModes];
#pragma unroll
  for (int q = 0; q < kPartModes; ++q) acc[q] = bcast2(0.0f);
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
      const TokenCtl* cs = p.ctl + b * T + r.t0;
      const float2* hs = c > 0 ? p.carry + (b * chunks + (c - 1)) * (long long)M + mbase : nullptr;
      const float2* ks = c < chunks - 1 ? p.kout + (b * chunks + (c + 1)) * (long long)M + mbase : nullptr;
      if (p.use_tma) {
        if (tid == 0) {
          fence_proxy_async_smem();
          unsigned bytes = 2u * act_box_bytes<TIO, C, kBwdModes>() + (unsigned)sizeof(TokenCtl) * (unsigned)r.nvalid;
          if (hs != nullptr) bytes += (unsigned)ncols * 8u;
          if (ks != nullptr) bytes += (unsigned)ncols * 8u;
          mbar_arrive_expect_tx(&S.bar, bytes);
          const int row = (int)(b * T + r.t0);
          tma_load_3d(&S.x[0][0][0], &p.map_x, mbase, 0, row, &S.bar);
          tma_load_3d(&S.dy[0][0][0], &p.map_dy, mbase, 0, row, &S.bar);
          bulk_copy_g2s(&S.ctl[0], cs, (unsigned)sizeof(TokenCtl) * (unsigned)r.nvalid, &S.bar);
          if (hs != nullptr) bulk_copy_g2s(&S.hin[0], hs, (unsigned)ncols * 8u, &S.bar);
          if (ks != nullptr) bulk_copy_g2s(&S.kin[0], ks, (unsigned)ncols * 8u, &S.bar);
        }
        if (!mbar_wait(&S.bar, (unsigned)par, p.max_spin << 4)) timed_out = true;
      } else {
        load_act_rows<TIO, kBwdModes>(xs, W, M, mbase, r.nvalid, S.x, kGradThreads);
        load_act_rows<TIO, kBwdModes>(ds, W, M, mbase, r.nvalid, S.dy, kGradThreads);
        for (int t = tid; t < r.nvalid; t += kGradThreads) S.ctl[t] = cs[t];
        for (int mm = tid; mm < ncols; mm += kGradThreads) {
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
      // the mixer's input of token t: x, or x r w in a block
      auto mixer_in = [&](int t, float2 xr, float2 xi, float2& nr, float2& ni) {
        if constexpr (kBlock) {
          const float2 rr = make_float2(S.ctl[t].keep.z, S.ctl[t].keep.w);
          nr = mul2(xr, mul2(rr, mc.wre));
          ni = mul2(xi, mul2(rr, mc.wim));
        } else {
          nr = xr;
          ni = xi;
        }
      };
      // pass 0: replay the states from the forward's carry
      float2 hin0 = make_float2(0.0f, 0.0f), hin1 = hin0;
      if (c > 0) {
        if (act0) hin0 = S.hin[2 * tid];
        if (act1) hin1 = S.hin[2 * tid + 1];
      } else if (p.h0_r != nullptr) {
        if (act0) hin0 = make_float2(p.h0_r[b * M + m0], p.h0_i[b * M + m0]);
        if (act1) hin1 = make_float2(p.h0_r[b * M + m0 + 1], p.h0_i[b * M + m0 + 1]);
      }
      const Cx2 hin = cx2(make_float2(hin0.x, hin1.x), make_float2(hin0.y, hin1.y));
      {
        Cx2 h = hin;
#pragma unroll kU
        for (int t = 0; t < C; ++t) {
          if (kFull || t < nvalid) {
            float2 nr, ni;
            mixer_in(t, Pair<TIO>::load(&S.x[t][0][2 * tid]), Pair<TIO>::load(&S.x[t][1][2 * tid]), nr, ni);
            const TokenCoef2 k = token_coef2<kFast, bwd_rot<kFast>(), kScan>(mc, S.ctl[t]);
            h = cfma2(k.a, h, cx2(mul2(k.gain, content2<kFast, kMode>(nr, lin)), mul2(k.gain, content2<kFast, kMode>(ni, lin))));
            Pair<TIO>::store(&S.h[t][0][2 * tid], h.re.x, h.re.y);
            Pair<TIO>::store(&S.h[t][1][2 * tid], h.im.x, h.im.y);
          }
        }
      }

      // adjoint carry entering the chunk from the later chunks
      float2 kin0 = make_float2(0.0f, 0.0f), kin1 = kin0;
      if (c < chunks - 1) {
        if (act0) kin0 = S.kin[2 * tid];
        if (act1) kin1 = S.kin[2 * tid + 1];
      } else if (p.glast_r != nullptr) {
        if (act0) kin0 = make_float2(p.glast_r[b * M + m0], p.glast_i[b * M + m0]);
        if (act1) kin1 = make_float2(p.glast_r[b * M + m0 + 1], p.glast_i[b * M + m0 + 1]);
      }
      Cx2 lam = cx2(make_float2(kin0.x, kin1.x), make_float2(kin0.y, kin1.y));

      // pass B: the true adjoint with every gradient, kGroup tokens at a time; each group's
      // per-token sums are reduced over the warp at once (lane 4u+j holds value u of the group)
      float2 fa[5];
#pragma unroll
      for (int q = 0; q < 5; ++q) fa[q] = bcast2(0.0f);
#pragma unroll 1
      for (int t1 = C - 1; t1 >= 0; t1 -= kGroup) {
        float v[2 * kGroup];
        float v3[kGroup];
#pragma unroll
        for (int u = 0; u < kGroup; ++u) {
          const int t = t1 - u;
          float ve = 0.0f, vd = 0.0f, vs = 0.0f;
          if (kFull || t < nvalid) {
            const TokenCtl& tc = S.ctl[t];
            // relu mask of the output gradient from this token's state (the slot still holds h_t)
            const float2 hcr = Pair<TIO>::load(&S.h[t][0][2 * tid]);
            const float2 hci = Pair<TIO>::load(&S.h[t][1][2 * tid]);
            const float2 gr = Pair<TIO>::load(&S.dy[t][0][2 * tid]);
            const float2 gi = Pair<TIO>::load(&S.dy[t][1][2 * tid]);
            if constexpr (kProj) {  // the states are the output: no relu
              lam.re = add2(lam.re, gr);
              lam.im = add2(lam.im, gi);
            } else {
              lam.re = add2(lam.re, make_float2(hcr.x > 0.0f ? gr.x : 0.0f, hcr.y > 0.0f ? gr.y : 0.0f));
              lam.im = add2(lam.im, make_float2(hci.x > 0.0f ? gi.x : 0.0f, hci.y > 0.0f ? gi.y : 0.0f));
            }
            const Cx2 pv = t > 0 ? cx2(Pair<TIO>::load(&S.h[t - 1][0][2 * tid]), Pair<TIO>::load(&S.h[t - 1][1][2 * tid]))
                                 : hin;
            const float2 xr = Pair<TIO>::load(&S.x[t][0][2 * tid]);
            const float2 xi = Pair<TIO>::load(&S.x[t][1][2 * tid]);
            float2 nr, ni;
            mixer_in(t, xr, xi, nr, ni);
            float2 ve2, vd2;
            const Cx2 dxc = grad_step2<kFast, kMode>(mc, tc, lam, pv, nr, ni, ve2, vd2, fa, lin);
            // h[t] was last read as the previous state at step t+1 and as this step's mask: its
            // slots now hold the write-path dx
            Pair<TIO>::store(&S.h[t][0][2 * tid], dxc.re.x, dxc.re.y);
            Pair<TIO>::store(&S.h[t][1][2 * tid], dxc.im.x, dxc.im.y);
            ve = (act0 ? ve2.x : 0.0f) + (act1 ? ve2.y : 0.0f);
            vd = (act0 ? vd2.x : 0.0f) + (act1 ? vd2.y : 0.0f);
            if constexpr (kBlock) {  // sum_j x_j w_j dxc_j (the norm backward's write-path part)
              const float2 sx = fma2(mul2(xr, mc.wre), dxc.re, mul2(mul2(xi, mc.wim), dxc.im));
              vs = (act0 ? sx.x : 0.0f) + (act1 ? sx.y : 0.0f);
            }
          }
          v[u] = ve;
          v[kGroup + u] = vd;
          v3[u] = vs;
        }
        {
          constexpr int kShift = 5 - log2i<2 * kGroup>();
          const float total = transpose_reduce<2 * kGroup>(v, lane);
          if ((lane & ((1 << kShift) - 1)) == 0) {
            const int u = lane >> kShift;  // 0..2*kGroup-1: ve of tokens t1..t1-3, then vd
            const int t = t1 - (u % kGroup);
            S.warp_part[warp][(u < kGroup ? 0 : C) + t] = total;
          }
        }
        if constexpr (kBlock) {
          constexpr int kShift = 5 - log2i<kGroup>();
          const float total = transpose_reduce<kGroup>(v3, lane);
          if ((lane & ((1 << kShift) - 1)) == 0) S.warp_part[warp][2 * C + t1 - (lane >> kShift)] = total;
        }
      }
#pragma unroll
      for (int q = 0; q < 5; ++q) acc[q] = add2(acc[q], fa[q]);

      // token sums over all modes -> controller gradients (and the norm's coefficient)
      __syncthreads();
      if (tid < kVals) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kGradWarps; ++w) sum += S.warp_part[w][tid];
        S.part_grad[par][tid] = sum;
      }
      if (G > 1) cluster.sync();
      else __syncthreads();
      if (tid < kVals) {
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
        const TokenCtl& tc = S.ctl[tid];
        const float tau0 = tc.tau.x, tau1 = tc.tau.z;
        // d/dp of eta = ln16 tanh(p1), delta = pi/2 tanh(p0); the scan-level mode returns the
        // gradients of (delta, eta) themselves
        const float dp1 = tid < nvalid ? (kScan ? S.tot[tid] : S.tot[tid] * kLn16 * fmaf(-tau1, tau1, 1.0f)) : 0.0f;
        const float dp0 = tid < nvalid ? (kScan ? S.tot[C + tid] : S.tot[C + tid] * kHalfPi * fmaf(-tau0, tau0, 1.0f)) : 0.0f;
        S.dp[tid] = make_float4(dp0, dp0, dp1, dp1);
        if constexpr (kProj) {  // the projections' gradient (finished by the caller's matrix products)
          if (g == 0 && tid < nvalid) p.dp_out[b * T + r.t0 + tid] = make_float2(dp0, dp1);
        }
        if constexpr (kBlock) {
          // sum_j x_j w_j dn_j = sum x w dxc + dp0 q0 + dp1 q1 (q: the projections before r)
          const float rs = tc.keep.z;
          const float sxn = fmaf(dp0, tc.proj.x, fmaf(dp1, tc.proj.y, S.tot[2 * C + tid]));
          const float kappa = tid < nvalid ? rs * rs * rs * sxn / (float)W : 0.0f;
          S.kap[tid] = make_float2(kappa, kappa);
        }
      }
      __syncthreads();
      TIO* dxrow = static_cast<TIO*>(p.dx) + row0;
      float2 fd[4] = {bcast2(0.0f), bcast2(0.0f), bcast2(0.0f), bcast2(0.0f)};
      float2 fw[2] = {bcast2(0.0f), bcast2(0.0f)};
#pragma unroll kU
      for (int t = 0; t < C; ++t) {
        if (kFull || t < nvalid) {
          const float4 dpv = S.dp[t];
          const float2 dp0 = make_float2(dpv.x, dpv.y), dp1 = make_float2(dpv.z, dpv.w);
          const float2 xr = Pair<TIO>::load(&S.x[t][0][2 * tid]);
          const float2 xi = Pair<TIO>::load(&S.x[t][1][2 * tid]);
          // the mixer's input gradient
          const float2 dnr = fma2(dp0, mc.d0r, fma2(dp1, mc.d1r, Pair<TIO>::load(&S.h[t][0][2 * tid])));
          const float2 dni = fma2(dp0, mc.d0i, fma2(dp1, mc.d1i, Pair<TIO>::load(&S.h[t][1][2 * tid])));
          float2 dre, dim, nr, ni;
          if constexpr (kBlock) {
            const float2 rr = make_float2(S.ctl[t].keep.z, S.ctl[t].keep.w);
            const float2 kap = S.kap[t];
            const float2 rwr = mul2(rr, mc.wre), rwi = mul2(rr, mc.wim);
            dre = sub2(fma2(rwr, dnr, Pair<TIO>::load(&S.dy[t][0][2 * tid])), mul2(kap, xr));
            dim = sub2(fma2(rwi, dni, Pair<TIO>::load(&S.dy[t][1][2 * tid])), mul2(kap, xi));
            nr = mul2(xr, rwr);
            ni = mul2(xi, rwi);
            fw[0] = fma2(mul2(xr, rr), dnr, fw[0]);
            fw[1] = fma2(mul2(xi, rr), dni, fw[1]);
          } else {
            dre = dnr;
            dim = dni;
            nr = xr;
            ni = xi;
          }
          TIO* row = dxrow + (long long)t * W;
          if (kVec && act1) {
            Pair<TIO>::store(row + m0, dre.x, dre.y);
            Pair<TIO>::store(row + M + m0, dim.x, dim.y);
          } else {
            if (act0) {
              Io<TIO>::store(row + m0, dre.x);
              Io<TIO>::store(row + M + m0, dim.x);
            }
            if (act1) {
              Io<TIO>::store(row + m0 + 1, dre.y);
              Io<TIO>::store(row + M + m0 + 1, dim.y);
            }
          }
          if constexpr (!kProj) {  // (projection mode: the directions' gradient is the caller's)
            fd[0] = fma2(nr, dp0, fd[0]);
            fd[1] = fma2(ni, dp0, fd[1]);
            fd[2] = fma2(nr, dp1, fd[2]);
            fd[3] = fma2(ni, dp1, fd[3]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[5 + q] = add2(acc[5 + q], fd[q]);
      if constexpr (kBlock) {
        acc[9] = add2(acc[9], fw[0]);
        acc[10] = add2(acc[10], fw[1]);
      }
    };
    if (nvalid == C) tile_body(std::true_type{});
    else tile_body(std::false_type{});
    if (g == 0 && tid == 0) {
      float s0 = 0.0f, s1 = 0.0f;
      for (int t = 0; t < C; ++t) {
        s0 += S.dp[t].x;
        s1 += S.dp[t].z;
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
  for (int q = 0; q < kPartModes; ++q) {
    part[(long long)q * Mp + m0] = act0 ? (double)acc[q].x : 0.0;
    part[(long long)q * Mp + m0 + 1] = act1 ? (double)acc[q].y : 0.0;
  }
  if (g == 0 && tid == 0) {
    double* pb = p.part + (long long)gridDim.y * kPartModes * Mp + 2 * kc;
    pb[0] = acc_b0;
    pb[1] = acc_b1;
  }
  if (timed_out) atomicOr(&p.ls->status, kStatusTimeout);
  cluster_sync_relaxed();
}


// ------------------------------------------------------------------------------ gradients from saved states
// One stage of the saved-state gradient kernel: one of kSplit parts of a tile, S = C / kSplit
// tokens of x, dy and the states, and one more state row in front (the state before the part's
// first token).
template <typename TIO, int C, int kSplit>
struct GradSavedStage {
  static constexpr int S = C / kSplit;
  TIO x[S][2][kBwdModes];
  TIO dy[S][2][kBwdModes];
  TIO h[S + 1][2][kBwdModes];  // h[0] the state before the part, h[1 + u] the state of its token u,
                               // which the reverse walk replaces with that token's write-path dx
  TokenCtl ctl[S];
};

template <typename TIO, int C, int kSplit>
struct GradSavedSmem {
  static constexpr int S = C / kSplit;
  GradSavedStage<TIO, C, kSplit> st[kSplit];
  float4 dp[S];                // controller gradients per token as pairs (dp0, dp0, dp1, dp1)
  float2 kap[S];               // a block's RMSNorm backward coefficient, as a pair
  float part_all[2][8][3 * S]; // every cluster CTA's partials of the per-token sums (pushed by the
                               // peers), by item parity
  float warp_part[kGradWarps][3 * S];
  unsigned long long bar[kSplit];
  unsigned long long red[2];   // completes when all G CTAs' partials of an item have arrived
};

// Work item w of a CTA is part kSplit - 1 - w % kSplit of its tile w / kSplit (the later part
// first); stage w % kSplit holds it. With kSplit = 2 (halves) thread 0 issues item w + 2 into
// the stage as soon as item w has finished with it, so one item's copies are always in flight
// under the other's arithmetic; with kSplit = 1 (whole tiles, one stage: the variant for
// clusters, where each part costs a cross-CTA reduction) the next tile's copies follow the
// current tile.
template <typename TIO, int C, int kSplit, bool kFast, bool kVec, int kMode>
__global__ void __launch_bounds__(kGradThreads, 4) mixer_bwd_grad_saved_kernel(const __grid_constant__ BwdParams p) {
  constexpr int S = C / kSplit;
  static_assert((kSplit == 1 || kSplit == 2) && C % kSplit == 0 && S % kGroup == 0,
                "whole tiles or halves of whole reverse-walk groups");
  constexpr bool kBlock = kMode == kModeBlock, kProj = proj_like<kMode>(), kScan = kMode == kModeScan;
  const bool lin = kProj && p.content_linear != 0;
  cg::cluster_group cluster = cg::this_cluster();
  const int g = (int)cluster.block_rank();
  const int G = (int)cluster.num_blocks();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = p.M, W = p.W;
  const int mbase = g * kBwdModes;
  const int m0 = mbase + 2 * tid;
  const int Mp = p.Mp;
  const bool act0 = m0 < M, act1 = m0 + 1 < M;
  const long long B = p.B, T = p.T;
  const int chunks = p.chunks;
  const long long k0 = blockIdx.y, nk = gridDim.y;
  constexpr int kVals = kBlock ? 3 * S : 2 * S;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  GradSavedSmem<TIO, C, kSplit>& Q = *reinterpret_cast<GradSavedSmem<TIO, C, kSplit>*>(smem_raw);

  ModeConst2 mc = pair_modes(load_mode(p.pp, m0, M, act0), load_mode(p.pp, m0 + 1, M, act1));
  if constexpr (kBlock) load_norm_weight(mc, p.norm_w, m0, M, act0, act1);

  const long long ntile = k0 < p.tiles ? (p.tiles - 1 - k0) / nk + 1 : 0;
  const long long items = kSplit * ntile;
  const unsigned red_bytes = (unsigned)(G * kVals) * 4u;  // per item: kVals floats from each CTA
  if (tid == 0) {
#pragma unroll
    for (int k = 0; k < kSplit; ++k) mbar_init(&Q.bar[k], 1);
    mbar_init(&Q.red[0], 1);
    mbar_init(&Q.red[1], 1);
    mbar_init_fence();
    if (G > 1) {  // armed for items 0 and 1 before any peer can push
      mbar_arrive_expect_tx(&Q.red[0], red_bytes);
      mbar_arrive_expect_tx(&Q.red[1], red_bytes);
    }
  }
  if (G > 1) cluster.sync();  // every CTA's barriers are initialised and armed
  else __syncthreads();

  float2 acc[kPartModes];
#pragma unroll
  for (int q = 0; q < kPartModes; ++q) acc[q] = bcast2(0.0f);
  double acc_b0 = 0.0, acc_b1 = 0.0;
  bool timed_out = false;
  auto issue = [&](long long w) {  // (thread 0)
    const TileRef r = tile_ref(k0 + (w / kSplit) * nk, B, T, C);
    const int part = kSplit - 1 - (int)(w % kSplit);
    const int nv = max(0, min(S, r.nvalid - part * S));
    GradSavedStage<TIO, C, kSplit>& st = Q.st[w % kSplit];
    unsigned long long* bar = &Q.bar[w % kSplit];
    const int row = (int)(r.b * T + r.t0 + part * S);
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, 2u * act_box_bytes<TIO, S, kBwdModes>() + act_box_bytes<TIO, S + 1, kBwdModes>() +
                                   (unsigned)sizeof(TokenCtl) * (unsigned)nv);
    tma_load_3d(&st.x[0][0][0], &p.map_x, mbase, 0, row, bar);
    tma_load_3d(&st.dy[0][0][0], &p.map_dy, mbase, 0, row, bar);
    tma_load_3d(&st.h[0][0][0], &p.map_h, mbase, 0, row - 1, bar);  // (row -1 reads zeros)
    if (nv > 0) bulk_copy_g2s(&st.ctl[0], p.ctl + r.b * T + r.t0 + part * S, (unsigned)sizeof(TokenCtl) * (unsigned)nv, bar);
  };
  // the adjoint entering a tile from the later chunks (the scan's output), or the gradient of the
  // returned last state at the last chunk
  auto tile_kin = [&](long long i) -> Cx2 {
    const TileRef r = tile_ref(i, B, T, C);
    float2 a = make_float2(0.0f, 0.0f), c = a;
    if (r.c < chunks - 1) {
      const float2* ks = p.kout + (r.b * chunks + (r.c + 1)) * (long long)M;
      if (act0) a = __ldcg(ks + m0);
      if (act1) c = __ldcg(ks + m0 + 1);
    } else if (p.glast_r != nullptr) {
      if (act0) a = make_float2(p.glast_r[r.b * M + m0], p.glast_i[r.b * M + m0]);
      if (act1) c = make_float2(p.glast_r[r.b * M + m0 + 1], p.glast_i[r.b * M + m0 + 1]);
    }
    return cx2(make_float2(a.x, c.x), make_float2(a.y, c.y));
  };
  // The first stages' copies go out before the wait: x, dy, the states and the controls come from
  // kernels before the carry scan, which have completed when this kernel starts (see pdl_wait);
  // only the adjoint carries need the wait.
  if (tid == 0) {
    for (int k = 0; k < kSplit; ++k)
      if (k < items) issue(k);
  }
  pdl_wait();  // the adjoint carries (scan) are complete from here on
  Cx2 kin_next = ntile > 0 ? tile_kin(k0) : cx2(bcast2(0.0f), bcast2(0.0f));
  Cx2 lam = kin_next;

  for (long long w = 0; w < items; ++w) {
    const long long i = k0 + (w / kSplit) * nk;
    const TileRef r = tile_ref(i, B, T, C);
    const long long b = r.b;
    const int part = kSplit - 1 - (int)(w % kSplit);
    const int tb = part * S;  // the part's first token within the chunk
    const int nv = max(0, min(S, r.nvalid - tb));
    const int par = (int)(w & 1);
    GradSavedStage<TIO, C, kSplit>& st = Q.st[w % kSplit];
    if (part == kSplit - 1) {
      lam = kin_next;  // a new tile: the adjoint from the later chunks
      if (w / kSplit + 1 < ntile) kin_next = tile_kin(i + nk);  // (in flight under this tile)
    }
    if (!mbar_wait(&Q.bar[w % kSplit], (unsigned)((w / kSplit) & 1), p.max_spin << 4)) timed_out = true;
    // the state before token 0 of the sequence: h0 (else zero), not the row in front of it
    const bool first = r.c == 0 && part == 0;
    Cx2 hfirst = cx2(bcast2(0.0f), bcast2(0.0f));
    if (first && p.h0_r != nullptr) {
      hfirst = cx2(make_float2(act0 ? p.h0_r[b * M + m0] : 0.0f, act1 ? p.h0_r[b * M + m0 + 1] : 0.0f),
                   make_float2(act0 ? p.h0_i[b * M + m0] : 0.0f, act1 ? p.h0_i[b * M + m0 + 1] : 0.0f));
    }
    const long long row0 = (b * T + r.t0 + tb) * W;

    auto body = [&](auto full_tag) {
      constexpr bool kFull = decltype(full_tag)::value;
      auto mixer_in = [&](int u, float2 xr, float2 xi, float2& nr, float2& ni) {
        if constexpr (kBlock) {
          const float2 rr = make_float2(st.ctl[u].keep.z, st.ctl[u].keep.w);
          nr = mul2(xr, mul2(rr, mc.wre));
          ni = mul2(xi, mul2(rr, mc.wim));
        } else {
          nr = xr;
          ni = xi;
        }
      };
      // pass B: the true adjoint with every gradient, kGroup tokens at a time (lane 4u+j of the
      // warp ends up with value u of the group, as in the replaying kernel)
      float2 fa[5];
#pragma unroll
      for (int q = 0; q < 5; ++q) fa[q] = bcast2(0.0f);
      // the state of the token being walked (the later neighbour's previous state, carried)
      Cx2 hc = cx2(Pair<TIO>::load(&st.h[S][0][2 * tid]), Pair<TIO>::load(&st.h[S][1][2 * tid]));
      if (!kFull && nv < S && nv > 0) hc = cx2(Pair<TIO>::load(&st.h[nv][0][2 * tid]), Pair<TIO>::load(&st.h[nv][1][2 * tid]));
#pragma unroll 1
      for (int u1 = S - 1; u1 >= 0; u1 -= kGroup) {
        float v[2 * kGroup];
        float v3[kGroup];
#pragma unroll
        for (int j = 0; j < kGroup; ++j) {
          const int u = u1 - j;
          float ve = 0.0f, vd = 0.0f, vs = 0.0f;
          if (kFull || u < nv) {
            const TokenCtl& tc = st.ctl[u];
            const float2 gr = Pair<TIO>::load(&st.dy[u][0][2 * tid]);
            const float2 gi = Pair<TIO>::load(&st.dy[u][1][2 * tid]);
            if constexpr (kProj) {
              lam.re = add2(lam.re, gr);
              lam.im = add2(lam.im, gi);
            } else {  // relu mask of the output gradient from this token's state
              lam.re = add2(lam.re, make_float2(hc.re.x > 0.0f ? gr.x : 0.0f, hc.re.y > 0.0f ? gr.y : 0.0f));
              lam.im = add2(lam.im, make_float2(hc.im.x > 0.0f ? gi.x : 0.0f, hc.im.y > 0.0f ? gi.y : 0.0f));
            }
            const Cx2 pv = (u > 0 || !first) ? cx2(Pair<TIO>::load(&st.h[u][0][2 * tid]), Pair<TIO>::load(&st.h[u][1][2 * tid]))
                                             : hfirst;
            const float2 xr = Pair<TIO>::load(&st.x[u][0][2 * tid]);
            const float2 xi = Pair<TIO>::load(&st.x[u][1][2 * tid]);
            float2 nr, ni;
            mixer_in(u, xr, xi, nr, ni);
            float2 ve2, vd2;
            const Cx2 dxc = grad_step2<kFast, kMode>(mc, tc, lam, pv, nr, ni, ve2, vd2, fa, lin);
            Pair<TIO>::store(&st.h[u + 1][0][2 * tid], dxc.re.x, dxc.re.y);  // (h[u + 1] was last read above)
            Pair<TIO>::store(&st.h[u + 1][1][2 * tid], dxc.im.x, dxc.im.y);
            hc = pv;
            ve = (act0 ? ve2.x : 0.0f) + (act1 ? ve2.y : 0.0f);
            vd = (act0 ? vd2.x : 0.0f) + (act1 ? vd2.y : 0.0f);
            if constexpr (kBlock) {
              const float2 sx = fma2(mul2(xr, mc.wre), dxc.re, mul2(mul2(xi, mc.wim), dxc.im));
              vs = (act0 ? sx.x : 0.0f) + (act1 ? sx.y : 0.0f);
            }
          }
          v[j] = ve;
          v[kGroup + j] = vd;
          v3[j] = vs;
        }
        {
          constexpr int kShift = 5 - log2i<2 * kGroup>();
          const float total = transpose_reduce<2 * kGroup>(v, lane);
          if ((lane & ((1 << kShift) - 1)) == 0) {
            const int j = lane >> kShift;
            Q.warp_part[warp][(j < kGroup ? 0 : S) + u1 - (j % kGroup)] = total;
          }
        }
        if constexpr (kBlock) {
          constexpr int kShift = 5 - log2i<kGroup>();
          const float total = transpose_reduce<kGroup>(v3, lane);
          if ((lane & ((1 << kShift) - 1)) == 0) Q.warp_part[warp][2 * S + u1 - (lane >> kShift)] = total;
        }
      }
#pragma unroll
      for (int q = 0; q < 5; ++q) acc[q] = add2(acc[q], fa[q]);

      // per-token sums over all modes: the CTA's warps, then (G > 1) the cluster's CTAs, each of
      // which pushes its partials into every CTA's part_all (asynchronous stores completing on
      // the receiver's `red` barrier: no cluster barrier in the loop)
      __syncthreads();
      if (G > 1) {
        if (tid < kVals) {
          float sum = 0.0f;
#pragma unroll
          for (int ww = 0; ww < kGradWarps; ++ww) sum += Q.warp_part[ww][tid];
          for (int rr = 0; rr < G; ++rr)
            st_async_f32(cluster_smem_addr(&Q.part_all[par][g][tid], (unsigned)rr), sum,
                         cluster_smem_addr(&Q.red[par], (unsigned)rr));
        }
        if (!mbar_wait_cluster(&Q.red[par], (unsigned)((w >> 1) & 1), p.max_spin << 4)) timed_out = true;
        // (re-armed for item w + 2: no peer can push that item before this CTA has pushed item w + 1)
        if (tid == 0 && w + 2 < items) mbar_arrive_expect_tx(&Q.red[par], red_bytes);
      }
      if (tid < S) {
        const int u = tid;
        float te = 0.0f, td = 0.0f, ts = 0.0f;
        if (G > 1) {
#pragma unroll
          for (int rr = 0; rr < 8; ++rr) {
            if (rr < G) {  // fixed rank order: the same sums in every CTA
              te += Q.part_all[par][rr][u];
              td += Q.part_all[par][rr][S + u];
              if constexpr (kBlock) ts += Q.part_all[par][rr][2 * S + u];
            }
          }
        } else {
#pragma unroll
          for (int ww = 0; ww < kGradWarps; ++ww) {
            te += Q.warp_part[ww][u];
            td += Q.warp_part[ww][S + u];
            if constexpr (kBlock) ts += Q.warp_part[ww][2 * S + u];
          }
        }
        const TokenCtl& tc = st.ctl[u];
        const bool ok = u < nv;
        const float tau0 = ok ? tc.tau.x : 0.0f, tau1 = ok ? tc.tau.z : 0.0f;
        // d/dp of eta = ln16 tanh(p1), delta = pi/2 tanh(p0); the scan-level mode returns the
        // gradients of (delta, eta) themselves
        const float dp1 = ok ? (kScan ? te : te * kLn16 * fmaf(-tau1, tau1, 1.0f)) : 0.0f;
        const float dp0 = ok ? (kScan ? td : td * kHalfPi * fmaf(-tau0, tau0, 1.0f)) : 0.0f;
        Q.dp[u] = make_float4(dp0, dp0, dp1, dp1);
        if constexpr (kProj) {
          if (g == 0 && ok) p.dp_out[b * T + r.t0 + tb + u] = make_float2(dp0, dp1);
        }
        if constexpr (kBlock) {
          const float rs = ok ? tc.keep.z : 0.0f;
          const float sxn = ok ? fmaf(dp0, tc.proj.x, fmaf(dp1, tc.proj.y, ts)) : 0.0f;
          const float kappa = rs * rs * rs * sxn / (float)W;
          Q.kap[u] = make_float2(kappa, kappa);
        }
      }
      __syncthreads();

      // pass C: dx (the write path plus the controllers' and, in a block, the norm's terms)
      TIO* dxrow = static_cast<TIO*>(p.dx) + row0;
      float2 fd[4] = {bcast2(0.0f), bcast2(0.0f), bcast2(0.0f), bcast2(0.0f)};
      float2 fw[2] = {bcast2(0.0f), bcast2(0.0f)};
#pragma unroll
      for (int u = 0; u < S; ++u) {
        if (kFull || u < nv) {
          const float4 dpv = Q.dp[u];
          const float2 dp0 = make_float2(dpv.x, dpv.y), dp1 = make_float2(dpv.z, dpv.w);
          const float2 xr = Pair<TIO>::load(&st.x[u][0][2 * tid]);
          const float2 xi = Pair<TIO>::load(&st.x[u][1][2 * tid]);
          const float2 dnr = fma2(dp0, mc.d0r, fma2(dp1, mc.d1r, Pair<TIO>::load(&st.h[u + 1][0][2 * tid])));
          const float2 dni = fma2(dp0, mc.d0i, fma2(dp1, mc.d1i, Pair<TIO>::load(&st.h[u + 1][1][2 * tid])));
          float2 dre, dim, nr, ni;
          if constexpr (kBlock) {
            const float2 rr = make_float2(st.ctl[u].keep.z, st.ctl[u].keep.w);
            const float2 kap = Q.kap[u];
            const float2 rwr = mul2(rr, mc.wre), rwi = mul2(rr, mc.wim);
            dre = sub2(fma2(rwr, dnr, Pair<TIO>::load(&st.dy[u][0][2 * tid])), mul2(kap, xr));
            dim = sub2(fma2(rwi, dni, Pair<TIO>::load(&st.dy[u][1][2 * tid])), mul2(kap, xi));
            nr = mul2(xr, rwr);
            ni = mul2(xi, rwi);
            fw[0] = fma2(mul2(xr, rr), dnr, fw[0]);
            fw[1] = fma2(mul2(xi, rr), dni, fw[1]);
          } else {
            dre = dnr;
            dim = dni;
            nr = xr;
            ni = xi;
          }
          TIO* row = dxrow + (long long)u * W;
          if (kVec && act1) {
            Pair<TIO>::store(row + m0, dre.x, dre.y);
            Pair<TIO>::store(row + M + m0, dim.x, dim.y);
          } else {
            if (act0) {
              Io<TIO>::store(row + m0, dre.x);
              Io<TIO>::store(row + M + m0, dim.x);
            }
            if (act1) {
              Io<TIO>::store(row + m0 + 1, dre.y);
              Io<TIO>::store(row + M + m0 + 1, dim.y);
            }
          }
          if constexpr (!kProj) {
            fd[0] = fma2(nr, dp0, fd[0]);
            fd[1] = fma2(ni, dp0, fd[1]);
            fd[2] = fma2(nr, dp1, fd[2]);
            fd[3] = fma2(ni, dp1, fd[3]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[5 + q] = add2(acc[5 + q], fd[q]);
      if constexpr (kBlock) {
        acc[9] = add2(acc[9], fw[0]);
        acc[10] = add2(acc[10], fw[1]);
      }
    };
    if (nv == S) body(std::true_type{});
    else body(std::false_type{});
    if (g == 0 && tid == 0) {
      float s0 = 0.0f, s1 = 0.0f;
      for (int u = 0; u < S; ++u) {
        s0 += Q.dp[u].x;
        s1 += Q.dp[u].z;
      }
      acc_b0 += s0;
      acc_b1 += s1;
    }
    __syncthreads();  // the stage, dp and kap are free
    if (tid == 0 && w + kSplit < items) issue(w + kSplit);
  }
  // per-cluster partial parameter gradients (reduced in a fixed order by mixer_reduce_kernel)
  const long long kc = blockIdx.y;
  double* part = p.part + kc * (long long)kPartModes * Mp;
#pragma unroll
  for (int q = 0; q < kPartModes; ++q) {
    part[(long long)q * Mp + m0] = act0 ? (double)acc[q].x : 0.0;
    part[(long long)q * Mp + m0 + 1] = act1 ? (double)acc[q].y : 0.0;
  }
  if (g == 0 && tid == 0) {
    double* pb = p.part + (long long)gridDim.y * kPartModes * Mp + 2 * kc;
    pb[0] = acc_b0;
    pb[1] = acc_b1;
  }
  if (timed_out) atomicOr(&p.ls->status, kStatusTimeout);
  cluster_sync_relaxed();
}
